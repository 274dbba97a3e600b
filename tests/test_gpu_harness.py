"""GPU runs of the reference-facing harness entry points and the multi-GPU
launcher on whatever GPUs are visible."""
import pytest
import torch

from oracle import rmsnorm_linear as orc

pytestmark = pytest.mark.gpu


def test_reference_correctness_script_passes():
    """python -m src.test_kimi26_kernels (a pytest driver, so run in its own
    process) prints the reference's closing sentence."""
    import os
    import subprocess
    import sys

    project = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                           "kimi26-h100-rmsnorm-swiglu-fusion_b200")
    r = subprocess.run([sys.executable, "-m", "src.test_kimi26_kernels"], cwd=project,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "All Kimi K2.6 RMSNorm fusion kernel tests passed." in r.stdout
    assert r.stdout.count("PASS: ") == 6


def test_benchmark_cli_runs(capsys):
    from src import benchmark_kimi26

    benchmark_kimi26.main(["--config", "kimi_kv_b", "--warmup", "2", "--iters", "5"])
    out = capsys.readouterr().out
    assert "fused_ms=" in out and "speedup=" in out


def test_quantized_benchmark_cli_runs(capsys):
    from src import benchmark_kimi26_quantized

    benchmark_kimi26_quantized.main(["--tokens", "256", "--warmup", "2", "--iters", "3"])
    out = capsys.readouterr().out
    assert "fused_quantized_ms=" in out


def test_token_partitioned_launcher_on_visible_gpus():
    from src.multigpu import TokenPartitionedFusedLinear

    n = torch.cuda.device_count()
    devices = [f"cuda:{i % n}" for i in range(max(2, n))]
    M, K, N = 1000, 512, 2048
    x, gamma, W = orc.make_inputs(M, K, N, seed=40)
    Wn = orc.fold_gamma(W, gamma)
    tp = TokenPartitionedFusedLinear(Wn, None, orc.EPS, devices)
    full = tp(x.to("cuda:0"), out_device="cuda:0")
    torch.cuda.synchronize()
    ref = orc.unfused_reference(x, gamma, W, None, orc.EPS).float()
    torch.testing.assert_close(full.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_int8_stack_token_partitioned_matches_reference_dequant_path():
    """Two int8 layers (q_b- and kv_b-shaped, reduced N) through the
    token-partitioned launcher on the visible GPUs, checked against the
    reference's quantization-aware forward F.linear(x * bf16(inv_rms), W_deq)."""
    from src.multigpu import TokenPartitionedFusedLinear

    n = torch.cuda.device_count()
    devices = [f"cuda:{i % n}" for i in range(max(2, n))]
    for li, (M, K, N) in enumerate([(700, 1536, 2048), (700, 512, 4096)]):
        x, gamma, W = orc.make_inputs(M, K, N, seed=60 + li)
        Wn = orc.fold_gamma(W, gamma)
        tp = TokenPartitionedFusedLinear(Wn.to("cuda:0"), None, orc.EPS, devices, int8=True)
        q, scale = orc.quantize_int8_per_output_channel(Wn)
        for wq, ws in tp.weights:  # one quantization, replicated bit for bit
            assert torch.equal(wq.cpu(), q) and torch.equal(ws.cpu(), scale)
        full = tp(x.to("cuda:0"), out_device="cuda:0")
        torch.cuda.synchronize()
        ref = orc.fused_quantized(x, q, scale, orc.EPS).float()
        torch.testing.assert_close(full.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def _nccl_column_worker(rank, world, port, q):
    import datetime
    import os

    import torch.distributed as dist

    from src.multigpu import ColumnParallelFusedLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        M, K, N = 96, 512, 16384
        x, gamma, W = orc.make_inputs(M, K, N, seed=70)
        Wn = orc.fold_gamma(W, gamma)
        col = ColumnParallelFusedLinear(Wn, None, orc.EPS, rank=rank, world=world, align=256,
                                        device=f"cuda:{rank}")
        full = col(x.to(f"cuda:{rank}"))
        torch.cuda.synchronize()
        ref = orc.unfused_reference(x, gamma, W, None, orc.EPS).float()
        q.put((rank, bool(torch.allclose(full.float().cpu(), ref, atol=2e-2, rtol=2e-2))))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_column_parallel_all_gather_over_nccl():
    """The column split with its NCCL all-gather on up to two visible GPUs
    (head-aligned 256-column slices of a kv_b-shaped weight)."""
    import socket

    import torch.multiprocessing as mp

    world = min(2, torch.cuda.device_count())
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_column_worker, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    assert all(p.exitcode == 0 for p in procs)
    assert sorted(q.get(timeout=5) for _ in range(world)) == [(r, True) for r in range(world)]
