"""Host side of the data-parallel integer training exchange.

Mirrors crates/nsrl-train-core/src/lib.rs:344-465 (i64 weight-gradient
accumulation and the requantising apply into i8 weights) and the merge of
worker results in crates/nsrl-train/src/lib.rs:7401-7471, where the batch is
split into contiguous chunks and the per-worker i64 accumulators are summed
with checked adds in worker order.  Here a worker is a rank (one GPU per
process) and the sum is one int64 all-reduce over torch.distributed (NCCL on
GPUs).  Integer addition is associative, so the all-reduced sums equal the
ordered merge whenever no prefix of that merge overflows; the all-reduce is
used only when the sum over ranks of max |accumulator| proves that, and
otherwise the parts are gathered and merged in rank order with overflow
detection (a rejection, like the reference's `CoreRejected`).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import core

I64_MAX = 2**63 - 1


class LinearWeightGradientI64:
    """LinearWeightGradientI64 (crates/nsrl-train/src/lib.rs:13665-13750) on one device:
    accumulators [output_dim][input_dim] int64, carried residuals, sample_count."""

    def __init__(self, input_dim: int, output_dim: int, device=None):
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.input_dim, self.output_dim = input_dim, output_dim
        self.accumulators = torch.zeros((output_dim, input_dim), dtype=torch.int64, device=dev)
        self.residuals = torch.zeros((output_dim, input_dim), dtype=torch.int64, device=dev)
        self.sample_count = torch.zeros(1, dtype=torch.int64, device=dev)  # holds a u64

    def clear(self):
        self.accumulators.zero_()
        self.sample_count.zero_()


def _lib():
    L = core.lib()
    if not getattr(L, "_train_bound", False):
        vp, sz = C.c_void_p, C.c_size_t
        L.nsrl_accumulate_workspace_size.restype = sz
        L.nsrl_accumulate_workspace_size.argtypes = [sz, sz]
        L.nsrl_accumulate_linear_weight_gradient_i64.argtypes = [vp, vp, sz, sz, sz, vp, vp, vp, sz, vp, vp]
        L.nsrl_apply_linear_weight_gradient_i64_to_i8.argtypes = [vp, vp, vp, sz, vp, C.c_int32, C.c_uint8, C.c_int,
                                                                   vp, vp, vp]
        L._train_bound = True
    return L


def accumulate_linear_weight_gradient_i64_prescaled(x: torch.Tensor, scaled_grad_output: torch.Tensor,
                                                    gradient: LinearWeightGradientI64) -> bool:
    """train-core lib.rs:344-384 for every row of x [rows, input_dim] / scaled_grad_output
    [rows, output_dim] (int32).  False on an i64 overflow (the reference's CoreRejected)."""
    L = _lib()
    x = x.contiguous()
    g = scaled_grad_output.to(torch.int32).contiguous()
    rows = x.numel() // gradient.input_dim
    ws = core.workspace(L.nsrl_accumulate_workspace_size(gradient.input_dim, gradient.output_dim))
    st = core.Status()
    r = L.nsrl_accumulate_linear_weight_gradient_i64(
        core._ptr(x), core._ptr(g), rows, gradient.input_dim, gradient.output_dim, core._ptr(gradient.accumulators),
        core._ptr(gradient.sample_count), core._ptr(ws), ws.numel(), core._ptr(st.buf), core._stream())
    if r == core.NSRL_INVALID_SHAPE:
        raise ValueError(L.nsrl_last_error().decode())
    core._check(r)
    code, _ = st.fetch()
    return code == core.NSRL_OK


def apply_linear_weight_gradient_i64_to_i8(gradient: LinearWeightGradientI64, weights: torch.Tensor,
                                           learning_rate: int, learning_rate_shift: int,
                                           carry_residual: bool) -> Optional[dict]:
    """train-core lib.rs:386-465: returns the LinearWeightUpdateStats as a dict, or None
    on an arithmetic rejection.  Raises ValueError for an invalid config."""
    L = _lib()
    if weights.dtype != torch.int8 or weights.numel() != gradient.accumulators.numel():
        raise ValueError("weights must be int8 with one entry per accumulator")
    stats = torch.zeros(3, dtype=torch.int64, device=weights.device)
    st = core.Status()
    r = L.nsrl_apply_linear_weight_gradient_i64_to_i8(
        core._ptr(gradient.accumulators), core._ptr(gradient.residuals), core._ptr(weights), weights.numel(),
        core._ptr(gradient.sample_count), int(learning_rate), int(learning_rate_shift), int(bool(carry_residual)),
        core._ptr(stats), core._ptr(st.buf), core._stream())
    if r == core.NSRL_INVALID_SHAPE:
        raise ValueError(L.nsrl_last_error().decode())
    core._check(r)
    code, _ = st.fetch()
    if code != core.NSRL_OK:
        return None
    s = stats.cpu().tolist()
    return {"gradient_saturation_count": s[0], "zero_delta_count": s[1], "weight_delta_l1": s[2]}


def _abs_max(t: torch.Tensor) -> float:
    if t.numel() == 0:
        return 0.0
    mn, mx = int(t.min()), int(t.max())
    return float(max(abs(mn), abs(mx)))


def _ordered_merge(parts: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """Sum parts[0] + parts[1] + ... in order; the flag is set if a prefix overflowed."""
    out = parts[0].clone()
    ovf = torch.zeros((), dtype=torch.bool, device=parts.device)
    for w in range(1, parts.shape[0]):
        s = out + parts[w]  # wrapping int64
        ovf |= (((out ^ s) & (parts[w] ^ s)) < 0).any()
        out = s
    return out, bool(ovf)


def allreduce_weight_gradients_i64(gradients: Sequence[LinearWeightGradientI64], group=None) -> bool:
    """Sums the accumulators and sample counts of every rank into every rank
    (mini_transformer_merge_map_reduce_batch_result, lib.rs:7401-7471, with rank r
    holding worker chunk r).  Returns False, leaving the buffers unspecified, when
    the ordered merge overflows i64 (the reference rejects the batch then).  Every
    rank takes the same collective steps."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return True
    world = dist.get_world_size(group)
    flat = torch.cat([g.accumulators.reshape(-1) for g in gradients])
    counts = torch.cat([g.sample_count.reshape(-1) for g in gradients])
    bound = torch.tensor([_abs_max(flat), _abs_max(counts)], dtype=torch.float64, device=flat.device)
    dist.all_reduce(bound, op=dist.ReduceOp.SUM, group=group)
    if float(bound.max()) < 2.0**62:  # no prefix of any ordering can leave i64
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
        ok = True
    else:
        parts = [torch.empty_like(flat) for _ in range(world)]
        cparts = [torch.empty_like(counts) for _ in range(world)]
        dist.all_gather(parts, flat, group=group)
        dist.all_gather(cparts, counts, group=group)
        flat, o1 = _ordered_merge(torch.stack(parts))
        counts, o2 = _ordered_merge(torch.stack(cparts))
        ok = not (o1 or o2)
    off = 0
    for i, g in enumerate(gradients):
        n = g.accumulators.numel()
        g.accumulators.copy_(flat[off:off + n].view_as(g.accumulators))
        g.sample_count.copy_(counts[i:i + 1])
        off += n
    return ok
