"""GPU runs of the reference-facing harness entry points and the multi-GPU
launcher on whatever GPUs are visible."""
import pytest
import torch

from oracle import rmsnorm_linear as orc

pytestmark = pytest.mark.gpu


def test_reference_correctness_script_passes(capsys):
    from src import test_kimi26_kernels

    test_kimi26_kernels.main()
    assert "All Kimi K2.6 RMSNorm fusion kernel tests passed." in capsys.readouterr().out


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
