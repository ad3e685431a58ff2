"""numpy front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (a scalar C++ restatement of the reference's Rust
CPU kernels, see nsrl_oracle.cpp for the file:line each function follows) and
exposes it with numpy arrays.  Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py import this module; the product never does.

Every function returns None where the reference returns `None`
(shape rejection or arithmetic rejection), like the Rust `Option` API.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

_lib = None


class FixedScale(C.Structure):
    _fields_ = [("multiplier", C.c_int32), ("right_shift", C.c_uint8), ("pad", C.c_uint8 * 3)]


class LinearParams(C.Structure):
    _fields_ = [("weights", C.c_void_p), ("bias", C.c_void_p), ("scales", C.c_void_p),
                ("input_dim", C.c_size_t), ("output_dim", C.c_size_t)]


SCALE_DTYPE = np.dtype([("multiplier", "<i4"), ("right_shift", "u1"), ("pad", "u1", (3,))])


def scales(mult, shift, n=None):
    """Array of FixedScale{multiplier, right_shift}; scalars broadcast to n."""
    if n is not None:
        mult = np.full(n, mult, dtype=np.int32)
        shift = np.full(n, shift, dtype=np.uint8)
    a = np.zeros(len(mult), dtype=SCALE_DTYPE)
    a["multiplier"] = mult
    a["right_shift"] = shift
    return a


def use_native():
    """Load the -march=native build (CPU-baseline timing); call before the first lib()."""
    global _native
    _native = True


_native = False


def lib():
    global _lib
    if _lib is None:
        path = _build.build_native() if _native else _build.build()
        _lib = C.CDLL(path)
        _lib.orc_init()
        _lib.orc_rhu.restype = C.c_int64
        _lib.orc_rhu.argtypes = [C.c_int64, C.c_uint8]
        _lib.orc_requantize_i32_to_i16.restype = C.c_int16
        _lib.orc_requantize_i32_to_i16.argtypes = [C.c_int32, C.c_int32, C.c_uint8]
        _lib.orc_base2_exp_neg_q15.restype = C.c_int16
        _lib.orc_base2_exp_neg_q15.argtypes = [C.c_int32]
        _lib.orc_reciprocal_sum_q31.argtypes = [C.c_uint64, C.POINTER(C.c_uint32)]
        _lib.orc_normalize_u64.argtypes = [C.c_uint64, C.POINTER(C.c_uint8), C.POINTER(C.c_int16)]
        _lib.orc_integer_rsqrt_q30.argtypes = [C.c_uint64, C.POINTER(C.c_int64)]
        _lib.orc_gated_activation.restype = C.c_int16
        _lib.orc_gated_activation.argtypes = [C.c_int16, C.c_int16]
    return _lib


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


class Linear:
    """Mirror of LinearI16I8Params: weights [out][in] i8, optional i32 bias, per-channel scales."""

    def __init__(self, weights, scales_arr, bias=None):
        self.weights = _c(weights, np.int8)
        self.output_dim, self.input_dim = self.weights.shape
        self.scales = np.ascontiguousarray(scales_arr, dtype=SCALE_DTYPE)
        self.bias = None if bias is None else _c(bias, np.int32)

    def struct(self):
        return LinearParams(self.weights.ctypes.data, None if self.bias is None else self.bias.ctypes.data,
                            self.scales.ctypes.data, self.input_dim, self.output_dim)


def luts():
    r = np.zeros(128, np.int16)
    e = np.zeros(256, np.int16)
    c = np.zeros(128, np.uint32)
    lib().orc_luts(_p(r), _p(e), _p(c))
    return r, e, c


def rhu(v, s):
    return lib().orc_rhu(int(v), int(s))


def requantize_i32_to_i16(acc, mult, shift):
    return lib().orc_requantize_i32_to_i16(int(acc), int(mult), int(shift))


def base2_exp_neg_q15(d):
    return lib().orc_base2_exp_neg_q15(int(d))


def reciprocal_sum_q31(s):
    out = C.c_uint32()
    return None if lib().orc_reciprocal_sum_q31(int(s), C.byref(out)) else out.value


def normalize_u64(v):
    m, e = C.c_uint8(), C.c_int16()
    return None if lib().orc_normalize_u64(int(v), C.byref(m), C.byref(e)) else (m.value, e.value)


def integer_rsqrt_q30(v):
    out = C.c_int64()
    return None if lib().orc_integer_rsqrt_q30(int(v), C.byref(out)) else out.value


def gated_activation(up, gate):
    return lib().orc_gated_activation(int(up), int(gate))


def base2_softmax_i32_q15(logits):
    lg = _c(logits, np.int32)
    out = np.zeros(len(lg), np.int16)
    s = C.c_uint64()
    if lib().orc_base2_softmax_i32_q15(_p(lg), C.c_size_t(len(lg)), _p(out), C.byref(s)):
        return None
    return out, s.value


def residual_add(skip, block):
    a, b = _c(skip, np.int16), _c(block, np.int16)
    out = np.zeros_like(a)
    s = C.c_uint64()
    lib().orc_residual_add(_p(a), _p(b), _p(out), C.c_size_t(a.size), C.byref(s))
    return out, s.value


def linear(x, lin: Linear, threads=1):
    x = _c(x, np.int16)
    M = x.size // lin.input_dim
    y = np.zeros((M, lin.output_dim), np.int16)
    st = lin.struct()
    if lib().orc_linear(_p(x), C.c_size_t(M), C.byref(st), _p(y), C.c_int(threads)):
        return None
    return y


def rms_norm_rows(x, gamma, eps):
    x = _c(x, np.int16)
    g = _c(gamma, np.int16)
    d = g.size
    y = np.zeros_like(x)
    if lib().orc_rms_norm_rows(_p(x), C.c_size_t(x.size // d), C.c_size_t(d), _p(g), C.c_uint64(eps), _p(y)):
        return None
    return y


def attention_row(query, keys, values, key_dim, value_dim, mask=None):
    q = _c(query, np.int16)
    k = _c(keys, np.int16)
    v = _c(values, np.int16)
    L = k.size // key_dim
    m = None if mask is None else _c(mask, np.uint8)
    logits = np.zeros(L, np.int32)
    probs = np.zeros(L, np.int16)
    out = np.zeros(value_dim, np.int16)
    s = C.c_uint64()
    if lib().orc_attention_row(_p(q), _p(k), _p(v), C.c_size_t(key_dim), C.c_size_t(value_dim), C.c_size_t(L),
                               _p(m), _p(logits), _p(probs), _p(out), C.byref(s)):
        return None
    return out, logits, probs, s.value


def _lp_array(lins):
    arr = (LinearParams * len(lins))(*[l.struct() for l in lins])
    return arr


def self_attention(x, B, S, d, H, q, k, v, o, causal=True, threads=1):
    x = _c(x, np.int16)
    out = np.zeros((B * S, d), np.int16)
    lp = _lp_array([q, k, v, o])
    if lib().orc_self_attention(_p(x), C.c_size_t(B), C.c_size_t(S), C.c_size_t(d), C.c_size_t(H),
                                C.c_int(int(causal)), lp, _p(out), C.c_int(threads)):
        return None
    return out


def prenorm_attention_block(x, B, S, d, H, gamma, eps, q, k, v, o, causal=True, threads=1):
    x = _c(x, np.int16)
    g = _c(gamma, np.int16)
    y = np.zeros((B * S, d), np.int16)
    sat = C.c_uint64()
    lp = _lp_array([q, k, v, o])
    if lib().orc_prenorm_attention_block(_p(x), C.c_size_t(B), C.c_size_t(S), C.c_size_t(d), C.c_size_t(H),
                                         C.c_int(int(causal)), _p(g), C.c_uint64(eps), lp, _p(y),
                                         C.byref(sat), C.c_int(threads)):
        return None
    return y, sat.value


def prenorm_mlp_block(x, T, d, F, gamma, eps, up, gate, down, threads=1):
    x = _c(x, np.int16)
    g = _c(gamma, np.int16)
    y = np.zeros((T, d), np.int16)
    sat = C.c_uint64()
    lp = _lp_array([up, gate, down])
    if lib().orc_prenorm_mlp_block(_p(x), C.c_size_t(T), C.c_size_t(d), C.c_size_t(F), _p(g), C.c_uint64(eps),
                                   lp, _p(y), C.byref(sat), C.c_int(threads)):
        return None
    return y, sat.value


def decode_attention(q, kcache, vcache, lens, B, H, hd, Lmax, threads=1):
    q = _c(q, np.int16)
    kc = _c(kcache, np.int16)
    vc = _c(vcache, np.int16)
    ln = _c(lens, np.int32)
    ctx = np.zeros((B, H * hd), np.int16)
    if lib().orc_decode_attention(_p(q), _p(kc), _p(vc), _p(ln), C.c_size_t(B), C.c_size_t(H), C.c_size_t(hd),
                                  C.c_size_t(Lmax), _p(ctx), C.c_int(threads)):
        return None
    return ctx


def bench1m():
    mh, ih, oh, s = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
    if lib().orc_bench1m(C.byref(mh), C.byref(ih), C.byref(oh), C.byref(s)):
        return None
    return dict(model_hash=mh.value, input_hash=ih.value, output_hash=oh.value, saturations=s.value)


# ------------------------------------------------------ training exchange ---
def accumulate_linear_gradient_i64(x, g, acc, count):
    """train-core lib.rs:344-384 for each row; returns (acc, count) or None on overflow."""
    x = _c(x, np.int16)
    g = _c(g, np.int32)
    acc = np.array(acc, dtype=np.int64, copy=True)
    N, K = acc.shape
    rows = x.size // K
    c = C.c_uint64(count)
    if lib().orc_accumulate_linear_gradient_i64(_p(x), _p(g), C.c_size_t(rows), C.c_size_t(K), C.c_size_t(N),
                                                _p(acc), C.byref(c)):
        return None
    return acc, c.value


def apply_linear_gradient_i64_to_i8(acc, residuals, weights, count, lr, shift, carry):
    """train-core lib.rs:386-465; returns (acc, residuals, weights, count, stats) or None."""
    acc = np.array(acc, dtype=np.int64, copy=True).ravel()
    res = np.array(residuals, dtype=np.int64, copy=True).ravel()
    w = np.array(weights, dtype=np.int8, copy=True).ravel()
    c = C.c_uint64(count)
    stats = np.zeros(3, np.uint64)
    if lib().orc_apply_linear_gradient_i64_to_i8(_p(acc), _p(res), _p(w), C.c_size_t(w.size), C.byref(c),
                                                 C.c_int32(lr), C.c_uint8(shift), C.c_int(int(carry)), _p(stats)):
        return None
    return acc, res, w, c.value, [int(s) for s in stats]


def merge_i64(parts, counts):
    """nsrl-train lib.rs:7443-7471: ordered checked merge of worker accumulators."""
    parts = _c(parts, np.int64)
    counts = _c(counts, np.uint64)
    W, L = parts.shape
    out = np.zeros(L, np.int64)
    c = C.c_uint64()
    if lib().orc_merge_i64(_p(parts), C.c_size_t(W), C.c_size_t(L), _p(counts), _p(out), C.byref(c)):
        return None
    return out, c.value


# ----------------------------------------------------------- training step --
class _TrainLayer(C.Structure):
    _fields_ = [("attn_gamma", C.c_void_p), ("mlp_gamma", C.c_void_p), ("lin", LinearParams * 7)]


class _TrainModel(C.Structure):
    _fields_ = [("d", C.c_size_t), ("H", C.c_size_t), ("F", C.c_size_t), ("layers", C.c_size_t),
                ("S", C.c_size_t), ("embeddings", C.c_void_p), ("positions", C.c_void_p),
                ("layer", C.c_void_p), ("head", LinearParams), ("attention_kind", C.c_int32)]


LAYER_LINEARS = ("q", "k", "v", "o", "up", "gate", "down")


class TrainModel:
    """The mini transformer of crates/nsrl-train (embeddings, stacked blocks, byte head).

    layers: list of dicts with Linear entries q k v o up gate down and optional
    int16 attn_gamma / mlp_gamma (RMS norm enabled when present)."""

    def __init__(self, embeddings, positions, layers, head, d, H, F, S, attention_kind="softmax"):
        self.attention_kind = attention_kind  # "softmax" (base-2) or "linear"
        self.embeddings = _c(embeddings, np.int16)
        self.positions = None if positions is None else _c(positions, np.int16)
        self.layers = layers
        self.head = head
        self.d, self.H, self.F, self.S = d, H, F, S
        for ly in layers:
            for g in ("attn_gamma", "mlp_gamma"):
                if ly.get(g) is not None:
                    ly[g] = _c(ly[g], np.int16)

    def struct(self):
        arr = (_TrainLayer * len(self.layers))()
        for i, ly in enumerate(self.layers):
            arr[i].attn_gamma = None if ly.get("attn_gamma") is None else ly["attn_gamma"].ctypes.data
            arr[i].mlp_gamma = None if ly.get("mlp_gamma") is None else ly["mlp_gamma"].ctypes.data
            for j, nm in enumerate(LAYER_LINEARS):
                arr[i].lin[j] = ly[nm].struct()
        self._keep = arr
        return _TrainModel(self.d, self.H, self.F, len(self.layers), self.S, self.embeddings.ctypes.data,
                           None if self.positions is None else self.positions.ctypes.data,
                           C.cast(arr, C.c_void_p), self.head.struct(), 1 if self.attention_kind == "linear" else 0)

    def arena_layout(self):
        """Offsets of the i64 gradient arena, in the order the CUDA path uses too."""
        d, F, L, S = self.d, self.F, len(self.layers), self.S
        lay = {"head": (0, 256 * d)}
        off = 256 * d
        for li in range(L):
            for nm, n in zip(LAYER_LINEARS + ("rms_attn", "rms_mlp"), [d * d] * 4 + [F * d] * 3 + [d, d]):
                lay[(li, nm)] = (off, n)
                off += n
        lay["emb"] = (off, 256 * d)
        off += 256 * d
        lay["pos"] = (off, S * d)
        off += S * d
        lay["total"] = off
        return lay


def train_windows(model: TrainModel, contexts, targets, freq_w=None, workers=1):
    """nsrl-train/src/lib.rs:6970-7471 over W windows: returns (acc i64, counts u64, stats) or None."""
    L = lib()
    ms = model.struct()
    n = model.arena_layout()["total"]
    acc = np.zeros(n, np.int64)
    counts = np.zeros(2 + 9 * len(model.layers), np.uint64)
    stats = np.zeros(4, np.uint64)
    ctx = _c(contexts, np.uint8)
    tg = _c(targets, np.uint8)
    fw = None if freq_w is None else _c(freq_w, np.int16)
    r = L.orc_train_windows(C.byref(ms), _p(ctx), _p(tg), _p(fw), C.c_size_t(len(tg)), _p(acc), _p(counts),
                            _p(stats), C.c_int(workers))
    if r != 0:
        return None
    return acc, counts, {"accepted": int(stats[0]), "mlp_saturation_count": int(stats[1]),
                         "attention_saturation_count": int(stats[2]), "residual_saturation_count": int(stats[3])}


def train_block_forward(model: TrainModel, layer, x):
    L = lib()
    ms = model.struct()
    x = _c(x, np.int16)
    out = np.zeros_like(x)
    P = np.zeros((model.H, model.S, model.S), np.int16)
    sat = C.c_uint64()
    r = L.orc_train_block_forward(C.byref(ms), C.c_size_t(layer), _p(x), _p(out), _p(P), C.byref(sat))
    return None if r else (out, P, sat.value)


def linear_backward_input(g, lin: Linear, gin_scales=None):
    g = _c(g, np.int16)
    M = g.size // lin.output_dim
    dx = np.zeros((M, lin.input_dim), np.int16)
    s = lin.struct()
    gs = None if gin_scales is None else np.ascontiguousarray(gin_scales, dtype=SCALE_DTYPE)
    r = lib().orc_linear_backward_input(_p(g), C.c_size_t(M), C.byref(s), _p(gs), _p(dx))
    return None if r else dx


def gated_activation_backward(up, gate, g):
    gu, gg = C.c_int16(), C.c_int16()
    lib().orc_gated_activation_backward(C.c_int16(up), C.c_int16(gate), C.c_int16(g), C.byref(gu), C.byref(gg))
    return gu.value, gg.value


def gated_mlp_backward_input(grad_out, up_lin, gate_lin, down_lin, fwd_up, fwd_gate):
    """mlp.rs:256-357 with identity grad-input scales: (grad_up, grad_gate, grad_in, saturations) or None."""
    go = _c(grad_out, np.int16)
    d, F = up_lin.input_dim, up_lin.output_dim
    T = go.size // d
    arr = (LinearParams * 3)(up_lin.struct(), gate_lin.struct(), down_lin.struct())
    gu = np.zeros((T, F), np.int16)
    gg = np.zeros((T, F), np.int16)
    gi = np.zeros((T, d), np.int16)
    sat = C.c_uint64()
    fu, fg = _c(fwd_up, np.int16), _c(fwd_gate, np.int16)  # held until the call returns
    r = lib().orc_gated_mlp_backward_input(_p(go), C.c_size_t(T), C.c_size_t(d), C.c_size_t(F), arr,
                                           _p(fu), _p(fg), _p(gu), _p(gg), _p(gi), C.byref(sat))
    return None if r else (gu, gg, gi, sat.value)


def rms_norm_backward_rows(x, w, grad_out, eps, gw=None):
    x = _c(x, np.int16)
    d = len(w)
    T = x.size // d
    gi = np.zeros((T, d), np.int16)
    gw = np.zeros(d, np.int64) if gw is None else gw
    sat = C.c_uint64()
    w16, go = _c(w, np.int16), _c(grad_out, np.int16)  # held until the call returns
    r = lib().orc_rms_norm_backward_rows(_p(x), C.c_size_t(T), C.c_size_t(d), _p(w16), _p(go), C.c_uint64(eps),
                                         _p(gi), _p(gw), C.byref(sat))
    return None if r else (gi, gw, sat.value)


def attention_probabilities(q, k, B, S, d, H):
    P = np.zeros((B, H, S, S), np.int16)
    q16, k16 = _c(q, np.int16), _c(k, np.int16)  # held until the call returns
    r = lib().orc_attention_probabilities(_p(q16), _p(k16), C.c_size_t(B), C.c_size_t(S), C.c_size_t(d),
                                          C.c_size_t(H), _p(P))
    return None if r else P


def attention_backward(q, k, v, P, dC, B, S, d, H):
    dq = np.zeros((B * S, d), np.int16)
    dk = np.zeros_like(dq)
    dv = np.zeros_like(dq)
    held = [_c(a, np.int16) for a in (q, k, v, P, dC)]  # held until the call returns
    r = lib().orc_attention_backward(*[_p(a) for a in held], C.c_size_t(B), C.c_size_t(S), C.c_size_t(d),
                                     C.c_size_t(H), _p(dq), _p(dk), _p(dv))
    return None if r else (dq, dk, dv)


def apply_embedding_gradient_i64_to_i16(acc, residuals, emb, count, lr, shift, stats):
    """nsrl-train/src/lib.rs:14457-14510 in place on numpy arrays; False on a rejection."""
    return lib().orc_apply_embedding_gradient_i64_to_i16(_p(acc), _p(residuals), _p(emb), C.c_size_t(emb.size),
                                                         C.c_uint64(int(count)), C.c_int32(lr), C.c_uint8(shift),
                                                         _p(stats)) == 0


def batch_apply_shifts(cfg: dict, accepted_windows: int, layers: int):
    """Apply shifts of one batch: lib.rs:13591-13650 (batch shift), :15454-15495
    (stacked layers: +2, lower layers +14, capped at 62), :6372-6380 (embeddings)."""
    b, covered = 0, 1
    while covered < accepted_windows:
        covered *= 2
        b += 1
    c = {k: v - b for k, v in cfg.items() if k != "learning_rate"}
    if min(c.values()) < 0:
        return None
    sh = {"head": c["output_learning_rate_shift"], "emb": c["embedding_learning_rate_shift"]}
    for li in range(layers):
        m, a, aq, ak = (c["mlp_learning_rate_shift"], c["attention_learning_rate_shift"],
                        c["attention_q_learning_rate_shift"], c["attention_qk_learning_rate_shift"])
        if layers > 1:
            m, a, aq, ak = (min(v + 2, 62) for v in (m, a, aq, ak))
            if li + 1 < layers:
                m, a, aq, ak = (min(v + 14, 62) for v in (m, a, aq, ak))
        for nm in ("up", "gate", "down"):
            sh[(li, nm)] = m
        sh[(li, "q")], sh[(li, "k")], sh[(li, "v")], sh[(li, "o")] = aq, ak, a, a
    return sh


DEFAULT_TRAIN_CONFIG = {"learning_rate": 1, "output_learning_rate_shift": 18, "mlp_learning_rate_shift": 16,
                        "embedding_learning_rate_shift": 14, "attention_learning_rate_shift": 24,
                        "attention_q_learning_rate_shift": 18, "attention_qk_learning_rate_shift": 18}


def train_step(model: TrainModel, residuals, contexts, targets, cfg=None, workers=1):
    """One map-reduce batch (lib.rs:6970-7050 with `workers` chunks merged in
    order) and the apply of every parameter (lib.rs:6249-6400), in place on
    the model's numpy weights and on `residuals` (arena layout).  Returns the
    stats dict, or None when the batch is rejected."""
    cfg = cfg or DEFAULT_TRAIN_CONFIG
    r = train_windows(model, contexts, targets, workers=workers)
    if r is None:
        return None
    acc, counts, stats = r
    lay = model.arena_layout()
    sh = batch_apply_shifts(cfg, stats["accepted"], len(model.layers))
    if sh is None:
        return None
    lr = cfg["learning_rate"]
    tot = [0, 0, 0]

    def apply_i8(key, lin, count):
        o, n = lay[key]
        out = apply_linear_gradient_i64_to_i8(acc[o:o + n], residuals[o:o + n], lin.weights, count, lr, sh[key], True)
        if out is None:
            return False
        residuals[o:o + n] = out[1]
        lin.weights[...] = out[2].reshape(lin.weights.shape)
        for i in range(3):
            tot[i] += out[4][i]
        return True

    if not apply_i8("head", model.head, int(counts[0])):
        return None
    for li, ly in enumerate(model.layers):
        for j, nm in enumerate(LAYER_LINEARS):
            if not apply_i8((li, nm), ly[nm], int(counts[1 + 9 * li + j])):
                return None
    est = np.zeros(3, np.uint64)
    ce = int(counts[1 + 9 * len(model.layers)])
    for key, emb in (("emb", model.embeddings), ("pos", model.positions)):
        if emb is None:
            continue
        o, n = lay[key]
        a = np.ascontiguousarray(acc[o:o + n])
        rs = np.ascontiguousarray(residuals[o:o + n])
        flat = emb.reshape(-1)
        if not apply_embedding_gradient_i64_to_i16(a, rs, flat, ce, lr, sh["emb"], est):
            return None
        residuals[o:o + n] = rs
    for i in range(3):
        tot[i] += int(est[i])
    stats = dict(stats)
    stats.update({"gradient_saturation_count": tot[0], "zero_delta_count": tot[1], "weight_delta_l1": tot[2]})
    return stats


# --------------------------------------------------------- integer Adam --
class AdamConfig(C.Structure):
    """IntegerAdamConfig (nsrl-train-core/src/lib.rs:279-297); defaults lr 1, step 4, beta shifts 3 / 7, eps 1."""
    _fields_ = [("learning_rate", C.c_int32), ("step_shift", C.c_uint8), ("beta1_decay_shift", C.c_uint8),
                ("beta2_decay_shift", C.c_uint8), ("pad", C.c_uint8), ("epsilon", C.c_uint64)]

    def __init__(self, learning_rate=1, step_shift=4, beta1_decay_shift=3, beta2_decay_shift=7, epsilon=1):
        super().__init__(learning_rate, step_shift, beta1_decay_shift, beta2_decay_shift, 0, epsilon)


class AdamState:
    """IntegerAdamStateWorkspace: step, first / second moments, update residuals (numpy)."""

    def __init__(self, n):
        self.step = 0
        self.first = np.zeros(n, np.int64)
        self.second = np.zeros(n, np.uint64)
        self.residuals = np.zeros(n, np.int64)


def integer_adam(acc, count, weights, cfg: AdamConfig, state: AdamState):
    """apply_integer_adam_accumulators_i64_to_i8 / _to_i16 in place on `weights`
    (int8 or int16 numpy); returns the stats list, or None on a rejection."""
    a = _c(acc, np.int64)
    stats = np.zeros(3, np.uint64)
    st = C.c_uint64(state.step)
    fn = lib().orc_integer_adam_i8 if weights.dtype == np.int8 else lib().orc_integer_adam_i16
    r = fn(_p(a), C.c_uint64(int(count)), _p(weights), C.c_size_t(weights.size), C.byref(cfg), _p(state.first),
           _p(state.second), _p(state.residuals), C.byref(st), _p(stats))
    if r:
        return None
    state.step = st.value
    return [int(s) for s in stats]


ADAM_SCOPES = ("all", "rms_norm", "output", "final_mlp", "final_mlp_and_output")


def adam_state_layout(model: TrainModel):
    """mini_transformer_adam_state_ranges (nsrl-train/src/lib.rs:4165-4196):
    embeddings, positions, attention RMS, MLP RMS, then q, k, v, o, up, gate,
    down over all layers, then the output head."""
    d, F, L, S = model.d, model.F, len(model.layers), model.S
    rms = model.layers[0].get("attn_gamma") is not None
    lay, off = {}, 0
    for key, n in (("emb", 256 * d), ("pos", S * d if model.positions is not None else 0),
                   ("rms_attn", L * d if rms else 0), ("rms_mlp", L * d if rms else 0)):
        lay[key] = off
        off += n
    for nm, n in zip(LAYER_LINEARS, [d * d] * 4 + [F * d] * 3):
        lay[nm] = off
        off += L * n
    lay["output"] = off
    lay["total"] = off + 256 * d
    return lay


def adam_train_step(model: TrainModel, state: AdamState, contexts, targets, cfg: AdamConfig, scope="all",
                    workers=1):
    """One map-reduce batch and the integer-Adam batch apply
    (mini_transformer_apply_integer_adam_batch, lib.rs:4270-4465) in place on
    the model's numpy weights and `state` (one flat state in adam_state_layout
    order; its step advances once per batch, the slices' own steps are
    ignored, lib.rs:4447-4451).  Returns the stats dict, or None when the
    batch is rejected."""
    r = train_windows(model, contexts, targets, workers=workers)
    if r is None:
        return None
    acc, counts, stats = r
    lay = model.arena_layout()
    sl = adam_state_layout(model)
    L = len(model.layers)
    rms = model.layers[0].get("attn_gamma") is not None
    tot = [0, 0, 0]

    def apply(arena_key, weights, count, state_off):
        o, n = lay[arena_key]
        flat = weights.reshape(-1)
        a = np.ascontiguousarray(acc[o:o + n])
        st = np.zeros(3, np.uint64)
        stp = C.c_uint64(0)
        fn = lib().orc_integer_adam_i8 if flat.dtype == np.int8 else lib().orc_integer_adam_i16
        rr = fn(_p(a), C.c_uint64(int(count)), _p(flat), C.c_size_t(n), C.byref(cfg),
                C.c_void_p(state.first.ctypes.data + 8 * state_off),
                C.c_void_p(state.second.ctypes.data + 8 * state_off),
                C.c_void_p(state.residuals.ctypes.data + 8 * state_off), C.byref(stp), _p(st))
        if rr:
            return False
        for i in range(3):
            tot[i] += int(st[i])
        return True

    ok = True
    if scope in ("all", "output", "final_mlp_and_output"):
        ok &= apply("head", model.head.weights, counts[0], sl["output"])
    d, F = model.d, model.F
    sizes = dict(zip(LAYER_LINEARS, [d * d] * 4 + [F * d] * 3))
    for li, ly in enumerate(model.layers):
        if scope == "all":
            for j, nm in enumerate(("q", "k", "v", "o")):
                ok &= apply((li, nm), ly[nm].weights, counts[1 + 9 * li + j], sl[nm] + li * sizes[nm])
        if scope == "all" or (scope in ("final_mlp", "final_mlp_and_output") and li + 1 == L):
            for nm in ("down", "up", "gate"):
                j = LAYER_LINEARS.index(nm)
                ok &= apply((li, nm), ly[nm].weights, counts[1 + 9 * li + j], sl[nm] + li * sizes[nm])
        if scope in ("all", "rms_norm") and rms:
            ok &= apply((li, "rms_attn"), ly["attn_gamma"], counts[1 + 9 * li + 7], sl["rms_attn"] + li * d)
            ok &= apply((li, "rms_mlp"), ly["mlp_gamma"], counts[1 + 9 * li + 8], sl["rms_mlp"] + li * d)
    if scope == "all":
        ce = counts[1 + 9 * L]
        ok &= apply("emb", model.embeddings, ce, sl["emb"])
        if model.positions is not None:
            ok &= apply("pos", model.positions, ce, sl["pos"])
    if not ok:
        return None
    state.step += 1
    stats = dict(stats)
    stats.update({"gradient_saturation_count": tot[0], "zero_delta_count": tot[1], "weight_delta_l1": tot[2]})
    return stats


# ------------------------------------------------------------- generation --
def output_rows(model: TrainModel, windows, threads=1):
    """The byte-head row (logits Q8 i32, probabilities Q15 i16) of the last
    position of each window [B][S] (nsrl-train/src/lib.rs:14911-15008,
    :17455-17490); None when a window is rejected."""
    w = _c(windows, np.uint8)
    B = w.shape[0]
    logits = np.zeros((B, 256), np.int32)
    probs = np.zeros((B, 256), np.int16)
    ms = model.struct()
    if lib().orc_output_rows(C.byref(ms), _p(w), C.c_size_t(B), _p(logits), _p(probs), C.c_int(threads)):
        return None
    return logits, probs


def generate(model: TrainModel, prompt: bytes, steps: int, strategy="greedy", top_k=0, seed=0):
    """generate_mini_transformer (lib.rs:12702-12800) with greedy or seeded
    top-k sampling and no priors: (tokens, logits of the picks, probabilities
    of the picks), or None on a rejection."""
    ctx = np.zeros(len(prompt) + steps, np.uint8)
    ctx[:len(prompt)] = np.frombuffer(bytes(prompt), np.uint8)
    tok = np.zeros(steps, np.uint8)
    lg = np.zeros(steps, np.int32)
    pr = np.zeros(steps, np.int16)
    ms = model.struct()
    if lib().orc_generate(C.byref(ms), _p(ctx), C.c_size_t(len(prompt)), C.c_size_t(steps),
                          C.c_int(0 if strategy == "greedy" else 1), C.c_size_t(top_k), C.c_uint64(seed), _p(tok),
                          _p(lg), _p(pr)):
        return None
    return tok, lg, pr


def average_movement(base, values, divisor):
    """average_i8_movement / average_i16_movement (nsrl-train/src/lib.rs:14552-14583):
    sat(base + round_div(values - base, divisor)) with half-away-from-zero rounding."""
    b = base.astype(np.int64)
    m = values.astype(np.int64) - b
    half = divisor // 2
    avg = np.where(m >= 0, (m + half) // divisor, -((-m + half) // divisor))
    info = np.iinfo(values.dtype)
    return np.clip(b + avg, info.min, info.max).astype(values.dtype)


# -------------------------------------------------------- linear attention --
def linear_attention(x, B, S, d, H, q, k, v, o, causal=True):
    """linear_attention_i16_q15_checked (crates/nsrl-core/src/attention.rs:879-1041)
    per sequence of x [B*S, d]; None on a rejection."""
    x = _c(x, np.int16)
    out = np.zeros((B * S, d), np.int16)
    if lib().orc_linear_attention(_p(x), C.c_size_t(B), C.c_size_t(S), C.c_size_t(d), C.c_size_t(H),
                                  C.c_int(int(causal)), _lp_array([q, k, v, o]), _p(out)):
        return None
    return out


def linear_attention_step(x, H, q, k, v, o, state, key_sums, ttt_shift=None, delta_l1=None):
    """linear_attention_step_i16_q15_checked / _ttt_step (attention.rs:1045-1283)
    for rows x [B, d] of B streams; state [B, H*hd*hd] and key_sums [B, H*hd]
    int64 updated in place; delta_l1 [B] uint64 added to (TTT).  The output
    rows, or None on a rejection."""
    x = _c(x, np.int16)
    B, d = x.shape
    out = np.zeros((B, d), np.int16)
    dl = _c(np.zeros(B, np.uint64) if delta_l1 is None else delta_l1, np.uint64)
    if lib().orc_linear_attention_step(_p(x), C.c_size_t(B), C.c_size_t(d), C.c_size_t(H),
                                       _lp_array([q, k, v, o]), _p(state), _p(key_sums),
                                       C.c_int(0 if ttt_shift is None else 1),
                                       C.c_uint8(0 if ttt_shift is None else ttt_shift), _p(out), _p(dl)):
        return None
    if delta_l1 is not None:
        delta_l1[...] = dl
    return out


def generate_streaming(model: TrainModel, prompt: bytes, steps: int, strategy="greedy", top_k=0, seed=0,
                       ttt_shift=None):
    """generate_mini_transformer_streaming_linear_nope_with_priors (or its TTT
    variant, nsrl-train/src/lib.rs:12802-12980): (tokens, picked logits,
    picked probabilities), or None on a rejection."""
    ctx = np.zeros(len(prompt) + steps, np.uint8)
    ctx[:len(prompt)] = np.frombuffer(bytes(prompt), np.uint8)
    tok = np.zeros(steps, np.uint8)
    lg = np.zeros(steps, np.int32)
    pr = np.zeros(steps, np.int16)
    ms = model.struct()
    if lib().orc_generate_streaming(C.byref(ms), _p(ctx), C.c_size_t(len(prompt)), C.c_size_t(steps),
                                    C.c_int(0 if strategy == "greedy" else 1), C.c_size_t(top_k), C.c_uint64(seed),
                                    C.c_int(0 if ttt_shift is None else 1),
                                    C.c_uint8(0 if ttt_shift is None else ttt_shift), _p(tok), _p(lg), _p(pr)):
        return None
    return tok, lg, pr
