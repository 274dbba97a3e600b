"""Multi-GPU launchers for fused RMSNorm -> Linear (one box, NVLink/NVSwitch).

The reference is single-GPU.  Rows (tokens) of this op are independent --
inv_rms is per row and the GEMM is row-separable -- so large-M work is split
token-wise across GPUs with the weight replicated and NO collective on the
data path.  For weight-bound (decode) shapes the weight itself can instead be
split by output columns, with an NCCL all-gather only when a consumer needs
the full row.

Two flavours of the token split:

* ``TokenPartitionedFusedLinear`` -- one process driving several devices:
  the weight is replicated once per device, each call slices x into
  contiguous row shards, launches every shard on its own device's current
  stream (asynchronously) and either returns the per-device outputs or
  copies them into one tensor on a destination device.
* ``fused_rmsnorm_linear_token_parallel`` -- one process per GPU under
  torch.distributed: every rank runs its own shard; ``gather=True`` adds an
  all-gather (for consumers that need every row on every rank).

``fused_stack_token_parallel`` runs one rank's token shard through a whole
stack of layers (the 61 q_b + kv_b pairs of Kimi K2.6, bf16 or int8 weights),
again with no collective.

``ColumnParallelFusedLinear`` holds W[N-slice] per rank and all-gathers the
[M, N/world] outputs into [M, N] over NCCL.

The per-shard op is ``denominator_cuda.fused_rmsnorm_linear`` (or
``fused_rmsnorm_linear_w8`` for int8 weights, given as a ``(qweight,
w_scale)`` pair) by default; it can be replaced (``op=``) so the partition /
gather logic can be exercised on CPU ranks with the gloo backend.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch

FusedOp = Callable[[torch.Tensor, torch.Tensor, Optional[torch.Tensor], float], torch.Tensor]


def _default_op() -> FusedOp:
    from src.load_cuda import denominator_cuda

    return lambda x, w, b, eps: denominator_cuda.fused_rmsnorm_linear(x, w, b, float(eps))


def _default_w8_op() -> FusedOp:
    """The int8-weight fused op; `w` is a (qweight int8 [N, K], w_scale fp32 [N]) pair."""
    from src.load_cuda import denominator_cuda

    return lambda x, w, b, eps: denominator_cuda.fused_rmsnorm_linear_w8(x, w[0], w[1], b,
                                                                         float(eps))


def _out_features(w) -> int:
    return (w[0] if isinstance(w, tuple) else w).shape[0]


def shard_bounds(total: int, parts: int, index: int) -> tuple[int, int]:
    """[start, end) of contiguous shard `index` of `total` rows over `parts`;
    the first (total % parts) shards take one extra row."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError(f"bad shard {index} of {parts}")
    base, rem = divmod(total, parts)
    start = index * base + min(index, rem)
    return start, start + base + (1 if index < rem else 0)


def column_bounds(n: int, parts: int, index: int, align: int = 8) -> tuple[int, int]:
    """Column slice of rank `index` for a column split of width n, in units of
    `align` columns (16-byte rows for the fused kernel); n % align == 0."""
    if n % align:
        raise ValueError(f"N={n} is not a multiple of {align}")
    s, e = shard_bounds(n // align, parts, index)
    return s * align, e * align


class TokenPartitionedFusedLinear:
    """Fused RMSNorm -> Linear over several GPUs of one process, split by rows.

    W_new / b_new are replicated to every device in `devices` at construction;
    with ``int8=True`` W_new is quantized once per output channel (the
    reference's absmax / 127 scheme) and the (qweight, w_scale) pair is what
    gets replicated, so every device holds bit-identical int8 weights.
    ``__call__(x)`` returns a list of per-device outputs (rows in order) or,
    with ``out_device``, one [M, N] tensor gathered there.  Work on each device
    is enqueued on that device's current stream; the host does not wait.
    """

    def __init__(self, W_new: torch.Tensor, b_new: Optional[torch.Tensor], eps: float,
                 devices: Sequence[torch.device | str | int], op: Optional[FusedOp] = None,
                 int8: bool = False):
        self.devices = [torch.device(d) if not isinstance(d, int) else torch.device("cuda", d)
                        for d in devices]
        if not self.devices:
            raise ValueError("need at least one device")
        self.eps = float(eps)
        self.int8 = bool(int8)
        if self.int8:
            from src.quantized import quantize_int8_per_output_channel

            q, scale = quantize_int8_per_output_channel(W_new)
            self.weights = [(q.to(d), scale.to(d)) for d in self.devices]
        else:
            self.weights = [W_new.to(d) for d in self.devices]
        self.biases = [b_new.to(d) if b_new is not None else None for d in self.devices]
        self.op = op or (_default_w8_op() if self.int8 else _default_op())

    def shards(self, m: int) -> list[tuple[int, int]]:
        return [shard_bounds(m, len(self.devices), i) for i in range(len(self.devices))]

    def __call__(self, x: torch.Tensor, out_device=None):
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        outs = []
        for (s, e), dev, w, b in zip(self.shards(x2.shape[0]), self.devices, self.weights,
                                     self.biases):
            xs = x2[s:e]
            if xs.device != dev:
                xs = xs.to(dev, non_blocking=True)
            outs.append(self.op(xs, w, b, self.eps) if e > s else
                        torch.empty(0, _out_features(w), dtype=x.dtype, device=dev))
        if out_device is None:
            return outs
        dst = torch.device(out_device)
        full = torch.empty(x2.shape[0], _out_features(self.weights[0]), dtype=x.dtype,
                           device=dst)
        for (s, e), o in zip(self.shards(x2.shape[0]), outs):
            if e > s:
                full[s:e].copy_(o, non_blocking=True)
        return full.reshape(*lead, full.shape[-1])


def fused_rmsnorm_linear_token_parallel(x_local: torch.Tensor, W_new: torch.Tensor,
                                        b_new: Optional[torch.Tensor], eps: float, *,
                                        gather: bool = False, group=None,
                                        op: Optional[FusedOp] = None) -> torch.Tensor:
    """One rank's share of a token-partitioned fused RMSNorm -> Linear.

    x_local holds this rank's rows; W_new is the rank's replica.  With
    ``gather=False`` (the default) no communication happens.  With
    ``gather=True`` the [M_local, N] outputs of all ranks are all-gathered
    (ranks may hold different row counts) and returned as [sum M, N] in rank
    order."""
    import torch.distributed as dist

    op = op or _default_op()
    out = op(x_local, W_new, b_new, eps)
    if not gather:
        return out
    world = dist.get_world_size(group)
    counts = torch.tensor([out.shape[0]], dtype=torch.int64, device=out.device)
    all_counts = [torch.zeros_like(counts) for _ in range(world)]
    dist.all_gather(all_counts, counts, group=group)
    sizes = [int(c.item()) for c in all_counts]
    mx = max(sizes)
    padded = out.new_zeros(mx, out.shape[1])
    padded[: out.shape[0]] = out
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([b[:n] for b, n in zip(bufs, sizes)], dim=0)


def fused_stack_token_parallel(xs_local: Sequence[torch.Tensor],
                               layers: Sequence[tuple], eps: float, *,
                               op: Optional[FusedOp] = None) -> list[torch.Tensor]:
    """One rank's share of a token-partitioned stack of fused RMSNorm -> Linear
    layers, e.g. the 61 (q_b, kv_b) pairs of Kimi K2.6 flattened to 122 layers.

    ``layers[i]`` is ``(weight, bias)`` with ``weight`` either W_new [N, K]
    (bf16 / fp16) or an int8 ``(qweight, w_scale)`` pair; ``xs_local[i]`` is
    this rank's rows of layer i's input (every rank holds the same rows of
    every layer: its token shard).  Every layer's weights are replicated on
    every rank, so no collective runs; the launches go back to back on the
    current stream.  Every layer's input is given up front, so no layer
    feeds another: with the default op, consecutive int8 layers go two per
    launch (one grouped kernel, e.g. a layer's q_b with its kv_b).  Returns
    the per-layer outputs."""
    if len(xs_local) != len(layers):
        raise ValueError(f"{len(xs_local)} inputs for {len(layers)} layers")
    outs = []
    i = 0
    while i < len(layers):
        x, (w, b) = xs_local[i], layers[i]
        if (op is None and isinstance(w, tuple) and i + 1 < len(layers)
                and isinstance(layers[i + 1][0], tuple) and x.is_cuda
                and xs_local[i + 1].device == x.device and xs_local[i + 1].dtype == x.dtype):
            from src.load_cuda import denominator_cuda

            x1, (w1, b1) = xs_local[i + 1], layers[i + 1]
            outs.extend(denominator_cuda.fused_rmsnorm_linear_w8_grouped(
                x, w[0], w[1], b, x1, w1[0], w1[1], b1, float(eps)))
            i += 2
            continue
        f = op or (_default_w8_op() if isinstance(w, tuple) else _default_op())
        outs.append(f(x, w, b, eps))
        i += 1
    return outs


class ColumnParallelFusedLinear:
    """Column (N) split: this rank holds W[cols] and produces out[:, cols].

    ``__call__(x, gather=True)`` all-gathers the [M, N/world] slices of every
    rank and returns [M, N]; the gather runs over NCCL (NVLink) on GPUs.  Kimi
    kv_b's N = 64 heads x 256, so rank slices can be head-aligned by choosing
    ``align`` = one head's width.
    """

    def __init__(self, W_full: torch.Tensor, b_full: Optional[torch.Tensor], eps: float, *,
                 rank: int, world: int, group=None, align: int = 8,
                 op: Optional[FusedOp] = None, device=None):
        self.n = W_full.shape[0]
        self.rank, self.world, self.group = rank, world, group
        self.bounds = [column_bounds(self.n, world, r, align) for r in range(world)]
        s, e = self.bounds[rank]
        dev = device if device is not None else W_full.device
        self.w = W_full[s:e].contiguous().to(dev)
        self.b = b_full[s:e].contiguous().to(dev) if b_full is not None else None
        self.eps = float(eps)
        self.op = op or _default_op()

    def __call__(self, x: torch.Tensor, gather: bool = True) -> torch.Tensor:
        import torch.distributed as dist

        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        part = self.op(x2, self.w, self.b, self.eps)
        if not gather:
            return part.reshape(*lead, part.shape[-1])
        widths = [e - s for s, e in self.bounds]
        m = x2.shape[0]
        if len(set(widths)) == 1:
            # Equal (e.g. head-aligned) slices: gather straight into one
            # [world, M, w] buffer, then one layout copy to [M, world * w].
            w = widths[0]
            buf = part.new_empty(self.world * m, w)
            dist.all_gather_into_tensor(buf, part.contiguous(), group=self.group)
            full = buf.view(self.world, m, w).permute(1, 0, 2).reshape(m, self.n)
        else:
            mx = max(widths)
            padded = part.new_zeros(m, mx)
            padded[:, : part.shape[1]] = part
            bufs = [torch.empty_like(padded) for _ in range(self.world)]
            dist.all_gather(bufs, padded, group=self.group)
            full = torch.cat([b[:, :w] for b, w in zip(bufs, widths)], dim=1)
        return full.reshape(*lead, self.n)
