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
import datetime
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


# ------------------------------------------------------- training backward --
class _TrainLayerC(C.Structure):
    _fields_ = [("attn_gamma", C.c_void_p), ("mlp_gamma", C.c_void_p), ("lin", core.LinearParamsC * 7)]


class _TrainModelC(C.Structure):
    _fields_ = [("d_model", C.c_size_t), ("heads", C.c_size_t), ("hidden_dim", C.c_size_t), ("layers", C.c_size_t),
                ("seq_len", C.c_size_t), ("embeddings", C.c_void_p), ("positions", C.c_void_p),
                ("layer", C.c_void_p), ("head", core.LinearParamsC), ("attention_kind", C.c_int32)]


LAYER_LINEARS = ("q", "k", "v", "o", "up", "gate", "down")


def _lib_bwd():
    L = _lib()
    if not getattr(L, "_bwd_bound", False):
        vp, sz = C.c_void_p, C.c_size_t
        lp = C.POINTER(core.LinearParamsC)
        L.nsrl_linear_backward_input_workspace_size.restype = sz
        L.nsrl_linear_backward_input_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_linear_backward_input.argtypes = [vp, sz, lp, vp, vp, vp, sz, vp, vp]
        L.nsrl_gated_mlp_backward_input_workspace_size.restype = sz
        L.nsrl_gated_mlp_backward_input_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_gated_mlp_backward_input.argtypes = [vp, sz, sz, sz, lp, lp, lp, vp, vp, vp, vp, vp, vp, vp, sz, vp, vp]
        L.nsrl_rms_norm_backward_rows.argtypes = [vp, sz, sz, vp, vp, C.c_uint64, vp, vp, vp, vp, vp]
        L.nsrl_attention_with_probabilities.argtypes = [vp, vp, vp, sz, sz, sz, sz, sz, vp, vp, vp, vp]
        L.nsrl_attention_backward_workspace_size.restype = sz
        L.nsrl_attention_backward_workspace_size.argtypes = [sz, sz, sz, sz]
        L.nsrl_attention_backward.argtypes = [vp, vp, vp, sz, vp, vp, sz, sz, sz, sz, vp, vp, vp, vp, sz, vp, vp]
        L.nsrl_train_arena_len.restype = sz
        L.nsrl_train_arena_len.argtypes = [vp]
        L.nsrl_train_workspace_size.restype = sz
        L.nsrl_train_workspace_size.argtypes = [vp, sz]
        L.nsrl_train_windows.argtypes = [vp, vp, vp, vp, sz, vp, vp, vp, vp, sz, vp, vp]
        L._bwd_bound = True
    return L


def _run_status(r, st):
    if r == core.NSRL_INVALID_SHAPE:
        raise ValueError(_lib().nsrl_last_error().decode())
    core._check(r)
    code, _ = st.fetch()
    return code == core.NSRL_OK


def linear_backward_input_i16_i8_i16_per_channel_checked(grad_output: torch.Tensor, lin: "core.Linear",
                                                        grad_input_scales: Optional[torch.Tensor] = None):
    """linear.rs:548-640 over the rows of grad_output [rows, output_dim]; None on a rejection."""
    L = _lib_bwd()
    g = core._i16(grad_output)
    rows = g.numel() // lin.output_dim
    dx = torch.empty((rows, lin.input_dim), dtype=torch.int16, device=g.device)
    ws = core.workspace(L.nsrl_linear_backward_input_workspace_size(rows, lin.input_dim, lin.output_dim))
    st = core.Status()
    p = lin.c()
    r = L.nsrl_linear_backward_input(core._ptr(g), rows, C.byref(p), core._ptr(grad_input_scales), core._ptr(dx),
                                     core._ptr(ws), ws.numel(), core._ptr(st.buf), core._stream())
    return dx if _run_status(r, st) else None


def gated_mlp_backward_input_i16_q15_checked(grad_output, up, gate, down, forward_up, forward_gate):
    """mlp.rs:256-357 with identity grad-input scales: (grad_up, grad_gate, grad_input, saturations) or None."""
    L = _lib_bwd()
    g = core._i16(grad_output)
    d, F = up.input_dim, up.output_dim
    rows = g.numel() // d
    dev = g.device
    gu = torch.empty((rows, F), dtype=torch.int16, device=dev)
    gg = torch.empty_like(gu)
    gi = torch.empty((rows, d), dtype=torch.int16, device=dev)
    sat = torch.zeros(1, dtype=torch.int64, device=dev)
    ws = core.workspace(L.nsrl_gated_mlp_backward_input_workspace_size(rows, d, F))
    st = core.Status()
    pu, pg, pd = up.c(), gate.c(), down.c()
    fu, fg = core._i16(forward_up), core._i16(forward_gate)  # held until the call is enqueued
    r = L.nsrl_gated_mlp_backward_input(core._ptr(g), rows, d, F, C.byref(pu), C.byref(pg), C.byref(pd),
                                        core._ptr(fu), core._ptr(fg), core._ptr(gu), core._ptr(gg), core._ptr(gi),
                                        core._ptr(sat), core._ptr(ws), ws.numel(), core._ptr(st.buf), core._stream())
    return (gu, gg, gi, int(sat.item())) if _run_status(r, st) else None


def rms_norm_backward_rows(x, gamma, grad_output, eps, gamma_grad: Optional[torch.Tensor] = None):
    """rms_norm.rs:96-170 per row: (grad_input, gamma_grad i64, saturations) or None."""
    L = _lib_bwd()
    x = core._i16(x)
    d = gamma.numel()
    rows = x.numel() // d
    gi = torch.empty((rows, d), dtype=torch.int16, device=x.device)
    gw = torch.zeros(d, dtype=torch.int64, device=x.device) if gamma_grad is None else gamma_grad
    sat = torch.zeros(1, dtype=torch.int64, device=x.device)
    st = core.Status()
    g16, go = core._i16(gamma), core._i16(grad_output)  # held until the call is enqueued
    r = L.nsrl_rms_norm_backward_rows(core._ptr(x), rows, d, core._ptr(g16), core._ptr(go), int(eps), core._ptr(gi),
                                      core._ptr(gw), core._ptr(sat), core._ptr(st.buf), core._stream())
    return (gi, gw, int(sat.item())) if _run_status(r, st) else None


def attention_with_probabilities(q, k, v, batch, seq_len, d_model, heads):
    """Causal attention on int16 q, k, v [batch*seq_len, d]: (context, P [batch, heads, S, S]) or None."""
    L = _lib_bwd()
    q, k, v = core._i16(q), core._i16(k), core._i16(v)
    ctx = torch.empty((batch * seq_len, d_model), dtype=torch.int16, device=q.device)
    P = torch.empty((batch, heads, seq_len, seq_len), dtype=torch.int16, device=q.device)
    st = core.Status()
    r = L.nsrl_attention_with_probabilities(core._ptr(q), core._ptr(k), core._ptr(v), d_model, batch, seq_len, d_model,
                                            heads, core._ptr(ctx), core._ptr(P), core._ptr(st.buf), core._stream())
    return (ctx, P) if _run_status(r, st) else None


def attention_backward(q, k, v, P, grad_context, batch, seq_len, d_model, heads):
    """nsrl-train/src/lib.rs:16623-16900: (dq, dk, dv) or None."""
    L = _lib_bwd()
    q, k, v, P, dC = (core._i16(t) for t in (q, k, v, P, grad_context))
    dq = torch.empty((batch * seq_len, d_model), dtype=torch.int16, device=q.device)
    dk = torch.empty_like(dq)
    dv = torch.empty_like(dq)
    ws = core.workspace(L.nsrl_attention_backward_workspace_size(batch, seq_len, d_model, heads))
    st = core.Status()
    r = L.nsrl_attention_backward(core._ptr(q), core._ptr(k), core._ptr(v), d_model, core._ptr(P), core._ptr(dC),
                                  batch, seq_len, d_model, heads, core._ptr(dq), core._ptr(dk), core._ptr(dv),
                                  core._ptr(ws), ws.numel(), core._ptr(st.buf), core._stream())
    return (dq, dk, dv) if _run_status(r, st) else None


class TrainModel:
    """The mini transformer (crates/nsrl-train MiniTransformerMlpModel) on one device.

    layers: list of dicts with core.Linear entries q k v o up gate down and
    optional int16 attn_gamma / mlp_gamma (RMS norm on when present)."""

    def __init__(self, embeddings, positions, layers, head, d_model, heads, hidden_dim, seq_len,
                 attention_kind: str = "softmax"):
        dev = core._dev()
        self.attention_kind = attention_kind  # "softmax" (base-2) or "linear"
        self.embeddings = embeddings.to(dev, torch.int16).contiguous()
        self.positions = None if positions is None else positions.to(dev, torch.int16).contiguous()
        self.layers = []
        for ly in layers:
            e = dict(ly)
            for g in ("attn_gamma", "mlp_gamma"):
                if e.get(g) is not None:
                    e[g] = e[g].to(dev, torch.int16).contiguous()
            self.layers.append(e)
        self.head = head
        self.d_model, self.heads, self.hidden_dim, self.seq_len = d_model, heads, hidden_dim, seq_len

    def c(self):
        arr = (_TrainLayerC * len(self.layers))()
        for i, ly in enumerate(self.layers):
            arr[i].attn_gamma = None if ly.get("attn_gamma") is None else ly["attn_gamma"].data_ptr()
            arr[i].mlp_gamma = None if ly.get("mlp_gamma") is None else ly["mlp_gamma"].data_ptr()
            for j, nm in enumerate(LAYER_LINEARS):
                arr[i].lin[j] = ly[nm].c()
        m = _TrainModelC(self.d_model, self.heads, self.hidden_dim, len(self.layers), self.seq_len,
                         self.embeddings.data_ptr(), None if self.positions is None else self.positions.data_ptr(),
                         C.cast(arr, C.c_void_p), self.head.c(), 1 if self.attention_kind == "linear" else 0)
        m._keep = arr
        return m

    def arena_layout(self):
        """(offset, length) of every gradient in the arena, the same order as the oracle's."""
        d, F, S = self.d_model, self.hidden_dim, self.seq_len
        lay = {"head": (0, 256 * d)}
        off = 256 * d
        for li in range(len(self.layers)):
            for nm, n in zip(LAYER_LINEARS + ("rms_attn", "rms_mlp"), [d * d] * 4 + [F * d] * 3 + [d, d]):
                lay[(li, nm)] = (off, n)
                off += n
        lay["emb"] = (off, 256 * d)
        off += 256 * d
        lay["pos"] = (off, S * d)
        off += S * d
        lay["total"] = off
        return lay


class TrainStepBuffers:
    """Workspace of the data-parallel step for W windows per rank over
    `nranks` ranks (nsrl_train_dp_workspace_size; it also serves
    nsrl_train_windows alone), and a gradient arena, sample counts and
    stats for the windows-only call."""

    def __init__(self, model: TrainModel, windows: int, nranks: Optional[int] = None):
        L = _lib_dp()
        m = model.c()
        dev = core._dev()
        if nranks is None:
            import torch.distributed as dist
            nranks = dist.get_world_size() if dist.is_initialized() else 1
        self.n = L.nsrl_train_arena_len(C.byref(m))
        self.arena = torch.zeros(self.n, dtype=torch.int64, device=dev)
        self.counts = torch.zeros(2 + 9 * len(model.layers), dtype=torch.int64, device=dev)
        self.stats = torch.zeros(4, dtype=torch.int64, device=dev)
        nbytes = L.nsrl_train_dp_workspace_size(C.byref(m), windows, int(nranks))
        if nbytes == 0:
            raise ValueError(L.nsrl_last_error().decode() or "invalid training-step shape")
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.status = core.Status()
        self.windows = windows

    def clear(self):
        self.arena.zero_()
        self.counts.zero_()
        self.stats.zero_()


def launch_train_windows(model: TrainModel, contexts: torch.Tensor, targets: torch.Tensor,
                         buf: TrainStepBuffers, freq_weights: Optional[torch.Tensor] = None) -> int:
    """Enqueues nsrl_train_windows on the current stream; returns the C status code."""
    L = _lib_bwd()
    m = model.c()
    return L.nsrl_train_windows(C.byref(m), core._ptr(contexts), core._ptr(targets), core._ptr(freq_weights),
                                buf.windows, core._ptr(buf.arena), core._ptr(buf.counts), core._ptr(buf.stats),
                                core._ptr(buf.ws), buf.ws.numel(), core._ptr(buf.status.buf), core._stream())


def mini_transformer_map_reduce_worker_batch(model: TrainModel, contexts: torch.Tensor, targets: torch.Tensor,
                                             freq_weights: Optional[torch.Tensor] = None):
    """nsrl-train/src/lib.rs:7051-7399 for W windows [W, seq_len] uint8 with targets [W] uint8:
    (arena i64, counts, stats dict), or None when the batch is rejected."""
    contexts = contexts.to(core._dev(), torch.uint8).contiguous()
    targets = targets.to(core._dev(), torch.uint8).contiguous()
    buf = TrainStepBuffers(model, contexts.shape[0])
    buf.status.reset()
    r = launch_train_windows(model, contexts, targets, buf, freq_weights)
    if not _run_status(r, buf.status):
        return None
    s = buf.stats.cpu().tolist()
    return buf.arena, buf.counts, {"accepted": s[0], "mlp_saturation_count": s[1], "attention_saturation_count": s[2],
                                   "residual_saturation_count": s[3]}


# --------------------------------------------------- data-parallel step --
import dataclasses


@dataclasses.dataclass(frozen=True)
class MiniTransformerTrainConfig:
    """The learning-rate fields of MiniTransformerMlpTrainConfig (nsrl-train/src/lib.rs:300-390)
    with the reference defaults (:86-91, :373-381)."""
    learning_rate: int = 1
    output_learning_rate_shift: int = 18
    mlp_learning_rate_shift: int = 16
    embedding_learning_rate_shift: int = 14
    attention_learning_rate_shift: int = 24
    attention_q_learning_rate_shift: int = 18
    attention_qk_learning_rate_shift: int = 18
    # "shift" (the residual-carrying shift apply, lib.rs:6249-6400) or
    # "integer_adam" (lib.rs:4270-4465) with IntegerAdamConfig fields
    # (learning_rate, step_shift, beta1_decay_shift, beta2_decay_shift,
    # epsilon) and a MiniTransformerAdamTrainScope (lib.rs:188-195)
    optimizer: str = "shift"
    adam: tuple = (1, 4, 3, 7, 1)
    adam_scope: str = "all"


MAX_RIGHT_SHIFT = 62
STACKED_BLOCK_EXTRA_SHIFT = 2          # nsrl-train/src/lib.rs:1541
STACKED_LOWER_LAYER_EXTRA_SHIFT = 14   # :1542
STACKED_EMBEDDING_EXTRA_SHIFT = 0      # :1543


def mini_transformer_batch_learning_rate_shift(batch_windows: int) -> Optional[int]:
    """lib.rs:13591-13605: ceil(log2(batch_windows)), None for 0."""
    if batch_windows == 0:
        return None
    shift, covered = 0, 1
    while covered < batch_windows:
        covered *= 2
        shift += 1
    return shift


def mini_transformer_batch_component_shift_config(cfg: MiniTransformerTrainConfig, batch_windows: int):
    """lib.rs:13607-13650: every component shift minus the batch shift (ValueError = InvalidConfig)."""
    b = mini_transformer_batch_learning_rate_shift(batch_windows)
    if b is None:
        raise ValueError("invalid config: zero batch windows")
    out = {}
    for f in ("output_learning_rate_shift", "mlp_learning_rate_shift", "embedding_learning_rate_shift",
              "attention_learning_rate_shift", "attention_q_learning_rate_shift", "attention_qk_learning_rate_shift"):
        v = getattr(cfg, f) - b
        if v < 0:
            raise ValueError(f"invalid config: {f} below the batch shift {b}")
        out[f] = v
    return dataclasses.replace(cfg, **out)


def mini_transformer_stacked_layer_runtime_config(cfg: MiniTransformerTrainConfig, layer_index: int,
                                                  layer_count: int):
    """lib.rs:15454-15495."""
    f4 = ("mlp_learning_rate_shift", "attention_learning_rate_shift", "attention_q_learning_rate_shift",
          "attention_qk_learning_rate_shift")
    out = {f: min(getattr(cfg, f) + STACKED_BLOCK_EXTRA_SHIFT, MAX_RIGHT_SHIFT) for f in f4}
    if layer_index + 1 < layer_count:
        out = {f: min(v + STACKED_LOWER_LAYER_EXTRA_SHIFT, MAX_RIGHT_SHIFT) for f, v in out.items()}
    return dataclasses.replace(cfg, **out)


def layer_apply_shifts(cfg: MiniTransformerTrainConfig, accepted_windows: int, layers: int) -> dict:
    """Every apply shift of one batch (lib.rs:6249-6400): output head, per layer the MLP and q/k/v/o, embeddings."""
    b = mini_transformer_batch_component_shift_config(cfg, accepted_windows)
    sh = {"head": b.output_learning_rate_shift}
    for li in range(layers):
        lc = mini_transformer_stacked_layer_runtime_config(b, li, layers) if layers > 1 else b
        for nm in ("up", "gate", "down"):
            sh[(li, nm)] = lc.mlp_learning_rate_shift
        sh[(li, "q")] = lc.attention_q_learning_rate_shift
        sh[(li, "k")] = lc.attention_qk_learning_rate_shift
        sh[(li, "v")] = lc.attention_learning_rate_shift
        sh[(li, "o")] = lc.attention_learning_rate_shift
    emb = b.embedding_learning_rate_shift
    if layers > 1:
        emb = min(emb + STACKED_EMBEDDING_EXTRA_SHIFT, MAX_RIGHT_SHIFT)
    sh["emb"] = emb
    return sh


class TrainState:
    """Carried residuals of every applied parameter (the residual arrays of
    LinearWeightGradientI64 and MiniTransformerEmbeddingGradientI64), laid
    out like the gradient arena; with adam=True also the integer-Adam state
    (MiniTransformerAdamOptimizerState, lib.rs:1001-1015)."""

    def __init__(self, model: TrainModel, adam: bool = False):
        dev = core._dev()
        self.residuals = torch.zeros(model.arena_layout()["total"], dtype=torch.int64, device=dev)
        self.adam = IntegerAdamState(_lib_dp().nsrl_train_adam_state_len(C.byref(model.c())), dev) if adam else None

    def c(self):
        a = self.adam
        return _TrainStateC(self.residuals.data_ptr(), *((a.first_moments.data_ptr(), a.second_moments.data_ptr(),
                                                          a.update_residuals.data_ptr(), a.step.data_ptr())
                                                         if a is not None else (None,) * 4))


def allreduce_flat_i64(flat: torch.Tensor, group=None) -> tuple[torch.Tensor, bool]:
    """Exact sum of an int64 vector over the ranks of `group` in rank order:
    one all-reduce when the sum over ranks of max |x| proves that no prefix of
    any ordering leaves i64, else all-gather and an ordered merge with
    overflow detection.  Returns (sum, ok)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    bound = torch.tensor([_abs_max(flat)], dtype=torch.float64, device=flat.device)
    dist.all_reduce(bound, op=dist.ReduceOp.SUM, group=group)
    if float(bound.item()) < 2.0**62:
        flat = flat.clone()
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        return flat, True
    parts = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(parts, flat, group=group)
    merged, ovf = _ordered_merge(torch.stack(parts))
    return merged, not ovf


class IntegerAdamConfigC(C.Structure):
    """IntegerAdamConfig (nsrl-train-core/src/lib.rs:279-297) with the reference defaults."""
    _fields_ = [("learning_rate", C.c_int32), ("step_shift", C.c_uint8), ("beta1_decay_shift", C.c_uint8),
                ("beta2_decay_shift", C.c_uint8), ("pad", C.c_uint8), ("epsilon", C.c_uint64)]

    def __init__(self, learning_rate=1, step_shift=4, beta1_decay_shift=3, beta2_decay_shift=7, epsilon=1):
        super().__init__(learning_rate, step_shift, beta1_decay_shift, beta2_decay_shift, 0, epsilon)


class _TrainConfigC(C.Structure):
    _fields_ = [("learning_rate", C.c_int32), ("output_learning_rate_shift", C.c_uint8),
                ("mlp_learning_rate_shift", C.c_uint8), ("embedding_learning_rate_shift", C.c_uint8),
                ("attention_learning_rate_shift", C.c_uint8), ("attention_q_learning_rate_shift", C.c_uint8),
                ("attention_qk_learning_rate_shift", C.c_uint8), ("optimizer", C.c_uint8), ("adam_scope", C.c_uint8),
                ("adam", IntegerAdamConfigC)]


class _TrainStateC(C.Structure):
    _fields_ = [("residuals", C.c_void_p), ("adam_first_moments", C.c_void_p), ("adam_second_moments", C.c_void_p),
                ("adam_update_residuals", C.c_void_p), ("adam_step", C.c_void_p)]


class _StepStatsC(C.Structure):
    _fields_ = [(f, C.c_uint64) for f in ("accepted", "mlp_saturation_count", "attention_saturation_count",
                                          "residual_saturation_count", "gradient_saturation_count",
                                          "zero_delta_count", "weight_delta_l1")]


ADAM_SCOPES = {"all": 0, "rms_norm": 1, "output": 2, "final_mlp": 3, "final_mlp_and_output": 4}


def _lib_dp():
    L = _lib_bwd()
    if not getattr(L, "_dp_bound", False):
        vp, sz = C.c_void_p, C.c_size_t
        L.nsrl_comm_unique_id.argtypes = [vp]
        L.nsrl_comm_init.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_int, vp, C.c_uint64]
        L.nsrl_comm_destroy.argtypes = [vp]
        L.nsrl_comm_abort.argtypes = [vp]
        L.nsrl_comm_nranks.argtypes = [vp]
        L.nsrl_comm_rank.argtypes = [vp]
        L.nsrl_train_adam_state_len.restype = sz
        L.nsrl_train_adam_state_len.argtypes = [vp]
        L.nsrl_train_dp_workspace_size.restype = sz
        L.nsrl_train_dp_workspace_size.argtypes = [vp, sz, C.c_int]
        L.nsrl_train_dp_step.argtypes = [vp, vp, vp, vp, sz, C.POINTER(_TrainConfigC), C.POINTER(_TrainStateC), vp,
                                         C.POINTER(_StepStatsC), vp, sz, vp, vp]
        L.nsrl_merge_worker_parts_i64.argtypes = [vp, sz, sz, sz, vp, vp, vp]
        L.nsrl_comm_selftest_wait.argtypes = [C.c_int, C.c_uint64, C.POINTER(C.c_uint64), C.POINTER(C.c_int)]
        L._dp_bound = True
    return L


class CommError(core.NsrlError):
    """The communicator timed out or reported a failed peer (it is aborted then)."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class PeerCheck:
    """A host-side check, before every step, that all ranks of the group are
    still there: each rank sets its key for the step in the group's store and
    waits (bounded) for the others'.  A rank that has left is noticed here,
    before any collective of the step is launched, so that no kernel waits on
    or writes to a peer that is gone."""

    def __init__(self, group=None, timeout_ms: int = 120_000, namespace: str = "nsrl"):
        import torch.distributed as dist
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout = datetime.timedelta(milliseconds=int(timeout_ms))
        self.store = dist.PrefixStore(f"{namespace}/peers/", dist.distributed_c10d._get_default_store())
        self.step = 0

    def wait(self):
        """Raises CommError when some rank does not arrive in time."""
        k = self.step
        self.step += 1
        self.store.set(f"{k}/{self.rank}", "1")
        try:
            self.store.wait([f"{k}/{r}" for r in range(self.world)], self.timeout)
        except Exception as e:  # the store's timeout, or its server gone with rank 0
            missing = [r for r in range(self.world) if r != self.rank and not self._has(f"{k}/{r}")]
            raise CommError(core.NSRL_COMM_ERROR, f"ranks {missing} did not arrive before step {k} "
                                                  f"({type(e).__name__})") from e
        if k >= 2:
            try:
                self.store.delete_key(f"{k - 2}/{self.rank}")
            except Exception:
                pass

    def _has(self, key):
        try:
            return self.store.check([key])
        except Exception:
            return False


class Communicator:
    """nsrl_comm: an NCCL communicator of the library over the ranks of a
    torch.distributed group (any backend: the group only carries rank 0's
    128-byte NCCL id to the other ranks).  Every wait on it is bounded by
    timeout_ms; a collective that misses the deadline aborts it (CommError)."""

    def __init__(self, group=None, timeout_ms: int = 120_000):
        import torch.distributed as dist
        L = _lib_dp()
        self.handle = None
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        uid = (C.c_uint8 * 128)()
        if self.rank == 0:
            r = L.nsrl_comm_unique_id(uid)
            if r != core.NSRL_OK:
                raise CommError(r, L.nsrl_last_error().decode())
        obj = [bytes(uid) if self.rank == 0 else None]
        src = 0 if group is None else dist.get_global_rank(group, 0)
        dist.broadcast_object_list(obj, src=src, group=group)
        uid = (C.c_uint8 * 128).from_buffer_copy(obj[0])
        h = C.c_void_p()
        r = L.nsrl_comm_init(C.byref(h), self.world, self.rank, uid, int(timeout_ms))
        if r != core.NSRL_OK:
            raise CommError(r, L.nsrl_last_error().decode())
        self.handle = h
        self.peers = PeerCheck(group, timeout_ms, namespace="nsrl/" + bytes(uid)[:8].hex())

    def check_peers(self):
        """The host-side peer check before a step; on failure the communicator
        is aborted (nothing of the step has been launched) and CommError raised."""
        try:
            self.peers.wait()
        except CommError:
            if self.handle:
                _lib_dp().nsrl_comm_abort(self.handle)
            raise

    def close(self):
        if self.handle:
            _lib_dp().nsrl_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_COMMS = {}


def default_communicator(group=None) -> Optional[Communicator]:
    """One Communicator per torch.distributed group (None for a single rank)."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return None
    key = id(group)
    if key not in _COMMS:
        _COMMS[key] = Communicator(group)
    return _COMMS[key]


def close_communicators():
    for c in _COMMS.values():
        c.close()
    _COMMS.clear()


def _config_c(cfg: "MiniTransformerTrainConfig") -> _TrainConfigC:
    return _TrainConfigC(int(cfg.learning_rate), cfg.output_learning_rate_shift, cfg.mlp_learning_rate_shift,
                         cfg.embedding_learning_rate_shift, cfg.attention_learning_rate_shift,
                         cfg.attention_q_learning_rate_shift, cfg.attention_qk_learning_rate_shift,
                         1 if cfg.optimizer == "integer_adam" else 0, ADAM_SCOPES[cfg.adam_scope],
                         IntegerAdamConfigC(*cfg.adam))


def mini_transformer_train_step(model: TrainModel, state: TrainState, contexts: torch.Tensor, targets: torch.Tensor,
                                cfg: MiniTransformerTrainConfig, buf: TrainStepBuffers, group=None,
                                freq_weights: Optional[torch.Tensor] = None,
                                comm: Optional[Communicator] = None) -> Optional[dict]:
    """One data-parallel batch through nsrl_train_dp_step: this rank's windows
    forward + backward into i64 accumulators (lib.rs:7051-7399), the exact
    int64 exchange with the other ranks (:7401-7471) and the apply of every
    parameter (:6249-6400, or integer Adam :4270-4465), with no host round
    trip in between.  Returns the batch stats, or None when the batch is
    rejected on any rank (:5371-5375; the model is unchanged then).  Raises
    CommError when the exchange times out or a peer fails."""
    L = _lib_dp()
    if comm is None:
        comm = default_communicator(group)
    if comm is not None:
        comm.check_peers()
    m = model.c()
    st = _StepStatsC()
    cc = _config_c(cfg)
    sc = state.c()
    ctx = contexts.to(core._dev(), torch.uint8).contiguous()
    tgt = targets.to(core._dev(), torch.uint8).contiguous()
    r = L.nsrl_train_dp_step(C.byref(m), core._ptr(ctx), core._ptr(tgt), core._ptr(freq_weights), ctx.shape[0],
                             C.byref(cc), C.byref(sc), comm.handle if comm else None, C.byref(st),
                             core._ptr(buf.ws), buf.ws.numel(), core._ptr(buf.status.buf), core._stream())
    if r == core.NSRL_INVALID_SHAPE:
        raise ValueError(L.nsrl_last_error().decode())
    if r in (core.NSRL_COMM_TIMEOUT, core.NSRL_COMM_ERROR):
        raise CommError(r, L.nsrl_last_error().decode())
    if r == core.NSRL_CORE_REJECTED:
        return None
    core._check(r)
    return {f: int(getattr(st, f)) for f, _ in _StepStatsC._fields_}


def accumulate_weight_gradient_i16(x: torch.Tensor, grad_output: torch.Tensor, scales: torch.Tensor,
                                   accumulators: torch.Tensor, sample_count: torch.Tensor) -> bool:
    """acc[n][k] += rhu(g[r][n], shift_n) * x[r][k] over the rows, on the tensor cores
    (nsrl-train-core/src/lib.rs:344-384 with the prescale of linear.rs:573-592);
    False when the call is rejected (a multiplier other than 1)."""
    L = _lib_bwd()
    if not getattr(L, "_acc16_bound", False):
        vp, sz = C.c_void_p, C.c_size_t
        L.nsrl_accumulate_weight_gradient_i16_workspace_size.restype = sz
        L.nsrl_accumulate_weight_gradient_i16_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_accumulate_weight_gradient_i16.argtypes = [vp, vp, sz, sz, sz, vp, vp, vp, vp, sz, vp, vp]
        L._acc16_bound = True
    x, g = core._i16(x), core._i16(grad_output)
    N, K = accumulators.shape
    rows = x.numel() // K
    ws = core.workspace(L.nsrl_accumulate_weight_gradient_i16_workspace_size(rows, K, N))
    st = core.Status()
    r = L.nsrl_accumulate_weight_gradient_i16(core._ptr(x), core._ptr(g), rows, K, N, core._ptr(scales),
                                              core._ptr(accumulators), core._ptr(sample_count), core._ptr(ws),
                                              ws.numel(), core._ptr(st.buf), core._stream())
    return _run_status(r, st)


# ------------------------------------------------------------ integer Adam --
class IntegerAdamState:
    """IntegerAdamStateWorkspace on the device: step, moments, update residuals."""

    def __init__(self, n, device=None):
        dev = device if device is not None else core._dev()
        self.step = torch.zeros(1, dtype=torch.int64, device=dev)
        self.first_moments = torch.zeros(n, dtype=torch.int64, device=dev)
        self.second_moments = torch.zeros(n, dtype=torch.int64, device=dev)  # holds u64
        self.update_residuals = torch.zeros(n, dtype=torch.int64, device=dev)


def apply_integer_adam_accumulators(accumulators: torch.Tensor, sample_count: torch.Tensor, weights: torch.Tensor,
                                    config: IntegerAdamConfigC, state: IntegerAdamState) -> Optional[dict]:
    """apply_integer_adam_accumulators_i64_to_i8 / _to_i16 (lib.rs:469-593) on device
    tensors (weights int8 or int16): the stats dict, or None on a rejection."""
    L = _lib()
    if not getattr(L, "_adam_bound", False):
        vp, sz = C.c_void_p, C.c_size_t
        for fn in (L.nsrl_apply_integer_adam_i64_to_i8, L.nsrl_apply_integer_adam_i64_to_i16):
            fn.argtypes = [vp, vp, vp, sz, C.POINTER(IntegerAdamConfigC), vp, vp, vp, vp, vp, vp, vp]
        L._adam_bound = True
    fn = L.nsrl_apply_integer_adam_i64_to_i8 if weights.dtype == torch.int8 else L.nsrl_apply_integer_adam_i64_to_i16
    stats = torch.zeros(3, dtype=torch.int64, device=weights.device)
    st = core.Status()
    r = fn(core._ptr(accumulators), core._ptr(sample_count), core._ptr(weights), weights.numel(), C.byref(config),
           core._ptr(state.first_moments), core._ptr(state.second_moments), core._ptr(state.update_residuals),
           core._ptr(state.step), core._ptr(stats), core._ptr(st.buf), core._stream())
    if r == core.NSRL_INVALID_SHAPE:
        raise ValueError(L.nsrl_last_error().decode())
    core._check(r)
    code, _ = st.fetch()
    if code != core.NSRL_OK:
        return None
    s = stats.cpu().tolist()
    return {"gradient_saturation_count": s[0], "zero_delta_count": s[1], "weight_delta_l1": s[2]}
