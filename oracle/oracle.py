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
