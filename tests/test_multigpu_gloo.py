"""Host logic of the multi-GPU launchers on CPU: shard arithmetic, and the
token-parallel and column-parallel paths as world_size-2 gloo process groups
with the oracle's fp32 math standing in for the CUDA op."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import rmsnorm_linear as orc
from src import multigpu


def _cpu_op(x, w, b, eps):
    return orc.fp32_truth(x, w, b, eps)


def _cpu_w8_op(x, w, b, eps):
    """The int8 kernel's math (inv_rms * scale * x.q^T + b) on the CPU."""
    q, scale = w
    return orc.int8_fp32_truth(x, q, scale, b, eps)


def test_shard_bounds_cover_exactly():
    for total in (0, 1, 5, 512, 4097):
        for parts in (1, 2, 3, 8):
            bounds = [multigpu.shard_bounds(total, parts, i) for i in range(parts)]
            assert bounds[0][0] == 0 and bounds[-1][1] == total
            assert all(b[1] == c[0] for b, c in zip(bounds, bounds[1:]))
            sizes = [e - s for s, e in bounds]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        multigpu.shard_bounds(10, 2, 2)


def test_column_bounds_aligned():
    b = [multigpu.column_bounds(16384, 8, r, align=256) for r in range(8)]
    assert b[0] == (0, 2048) and b[-1] == (14336, 16384)
    with pytest.raises(ValueError):
        multigpu.column_bounds(100, 2, 0)


def test_single_process_token_partition_on_cpu_devices():
    x, gamma, W = orc.make_inputs(37, 64, 24, seed=1, dtype=torch.float32)
    Wn = orc.fold_gamma(W, gamma)
    tp = multigpu.TokenPartitionedFusedLinear(Wn, None, orc.EPS, ["cpu", "cpu", "cpu"],
                                              op=_cpu_op)
    parts = tp(x)
    assert [p.shape[0] for p in parts] == [13, 12, 12]
    full = tp(x.view(1, 37, 64), out_device="cpu")
    torch.testing.assert_close(full.view(37, 24), _cpu_op(x, Wn, None, orc.EPS))


def test_single_process_int8_partition_replicates_one_quantization():
    x, gamma, W = orc.make_inputs(29, 64, 40, seed=2, dtype=torch.float32)
    Wn = orc.fold_gamma(W, gamma)
    tp = multigpu.TokenPartitionedFusedLinear(Wn, None, orc.EPS, ["cpu", "cpu"], op=_cpu_w8_op,
                                              int8=True)
    q, scale = orc.quantize_int8_per_output_channel(Wn)
    for wq, ws in tp.weights:
        assert torch.equal(wq, q) and torch.equal(ws, scale)
    full = tp(x, out_device="cpu")
    torch.testing.assert_close(full, _cpu_w8_op(x, (q, scale), None, orc.EPS))


def test_stack_runs_each_layer_on_its_own_input():
    layers, xs, want = [], [], []
    for i, (K, N) in enumerate([(64, 48), (32, 80), (64, 48)]):
        x, gamma, W = orc.make_inputs(10, K, N, seed=20 + i, dtype=torch.float32)
        Wn = orc.fold_gamma(W, gamma)
        layers.append((orc.quantize_int8_per_output_channel(Wn), None))
        xs.append(x)
        want.append(_cpu_w8_op(x, layers[-1][0], None, orc.EPS))
    outs = multigpu.fused_stack_token_parallel(xs, layers, orc.EPS, op=_cpu_w8_op)
    for o, w in zip(outs, want):
        torch.testing.assert_close(o, w)
    with pytest.raises(ValueError):
        multigpu.fused_stack_token_parallel(xs[:2], layers, orc.EPS, op=_cpu_w8_op)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, K, N = 45, 32, 48
        x, gamma, W = orc.make_inputs(M, K, N, seed=3, dtype=torch.float32)
        Wn = orc.fold_gamma(W, gamma)
        b = torch.linspace(-1, 1, N)
        s, e = multigpu.shard_bounds(M, world, rank)
        local = multigpu.fused_rmsnorm_linear_token_parallel(x[s:e], Wn, b, orc.EPS, op=_cpu_op)
        gathered = multigpu.fused_rmsnorm_linear_token_parallel(x[s:e], Wn, b, orc.EPS,
                                                                gather=True, op=_cpu_op)
        col = multigpu.ColumnParallelFusedLinear(Wn, b, orc.EPS, rank=rank, world=world,
                                                 align=8, op=_cpu_op)
        colfull = col(x.view(5, 9, K))
        want = _cpu_op(x, Wn, b, orc.EPS)
        # unequal column slices take the padded gather
        col2 = multigpu.ColumnParallelFusedLinear(Wn, b, orc.EPS, rank=rank, world=world,
                                                  align=16, op=_cpu_op)
        assert len({e2 - s2 for s2, e2 in col2.bounds}) == 2
        colfull2 = col2(x)
        # a two-layer int8 stack, each rank on its own token shard of every layer
        layers, xs, want_stack = [], [], []
        for i, (Ki, Ni) in enumerate([(K, N), (2 * K, 24)]):
            xi, gi, Wi = orc.make_inputs(M, Ki, Ni, seed=50 + i, dtype=torch.float32)
            qs = orc.quantize_int8_per_output_channel(orc.fold_gamma(Wi, gi))
            layers.append((qs, None))
            xs.append(xi[s:e])
            want_stack.append(_cpu_w8_op(xi, qs, None, orc.EPS)[s:e])
        stack = multigpu.fused_stack_token_parallel(xs, layers, orc.EPS, op=_cpu_w8_op)
        results[rank] = (
            torch.allclose(local, want[s:e], atol=1e-5),
            torch.allclose(gathered, want, atol=1e-5),
            torch.allclose(colfull.view(M, N), want, atol=1e-5)
            and torch.allclose(colfull2, want, atol=1e-5),
            all(torch.allclose(a, w) for a, w in zip(stack, want_stack)),
        )
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_gloo_world2_token_and_column_parallel():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode == 0
    assert dict(results) == {0: (True,) * 4, 1: (True,) * 4}


# ------------------------------------------------ failure detection (host side)


def _never_joined(port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # the peer never connects: init must give up
        q.put(type(e).__name__)


@pytest.mark.timeout(120)
def test_gloo_rank_that_never_joins_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_never_joined, args=(_free_port(), q))
    p.start()
    p.join(90)
    assert p.exitcode == 0
    assert q.get(timeout=5) != "joined"


def _gather_after_peer_left(rank, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=5))
    x, gamma, W = orc.make_inputs(8, 32, 16, seed=1, dtype=torch.float32)
    Wn = orc.fold_gamma(W, gamma)
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        multigpu.fused_rmsnorm_linear_token_parallel(x, Wn, None, orc.EPS, gather=True,
                                                     op=_cpu_op)
        q.put("gathered")
    except Exception as e:
        q.put(type(e).__name__)
    # os._exit skips the queue's feeder thread: flush it first, or the
    # message can be lost.
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.timeout(120)
def test_token_parallel_gather_fails_when_a_rank_left():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_after_peer_left, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) != "gathered"
