"""Host-side mirror of the reference's nsrl-core operator API over libnsrl_b200.

Each function keeps the reference name, argument meaning and error behaviour
(returns None where the Rust function returns `None`) and runs on CUDA
device tensors through the C ABI in include/nsrl_b200.h.  torch is used only
for device memory and the current stream.  There is no CPU fallback: without
the built library or a CUDA device every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnsrl_b200.so")

NSRL_OK, NSRL_INVALID_SHAPE, NSRL_CORE_REJECTED, NSRL_CUDA_ERROR, NSRL_COMM_TIMEOUT, NSRL_COMM_ERROR = range(6)

_lib = None


class LinearParamsC(C.Structure):
    _fields_ = [("weights", C.c_void_p), ("bias", C.c_void_p), ("scales", C.c_void_p),
                ("input_dim", C.c_size_t), ("output_dim", C.c_size_t)]


class DeviceStatusC(C.Structure):
    _fields_ = [("flags", C.c_ulonglong), ("attention_saturations", C.c_ulonglong),
                ("mlp_saturations", C.c_ulonglong), ("reserved", C.c_ulonglong * 5)]


class NsrlError(RuntimeError):
    pass


def lib():
    """Loads libnsrl_b200.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NsrlError(f"{LIB_PATH} is not built; run nsrl_b200/build.py")
        L = C.CDLL(LIB_PATH)
        vp, sz = C.c_void_p, C.c_size_t
        L.nsrl_last_error.restype = C.c_char_p
        L.nsrl_status_reset.argtypes = [vp, vp]
        L.nsrl_status_fetch.argtypes = [vp, C.POINTER(DeviceStatusC), vp]
        L.nsrl_linear_workspace_size.restype = sz
        L.nsrl_linear_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_linear_i16_i8_i16.argtypes = [vp, sz, C.POINTER(LinearParamsC), vp, vp, sz, vp, vp]
        L.nsrl_rms_norm_rows.argtypes = [vp, sz, sz, vp, C.c_uint64, vp, vp, vp]
        L.nsrl_attention_workspace_size.restype = sz
        L.nsrl_attention_workspace_size.argtypes = [sz, sz, sz, sz]
        lp = C.POINTER(LinearParamsC)
        L.nsrl_self_attention.argtypes = [vp, sz, sz, sz, sz, C.c_int, lp, lp, lp, lp, vp, vp, sz, vp, vp]
        L.nsrl_prenorm_attention_residual_block.argtypes = [vp, sz, sz, sz, sz, C.c_int, vp, C.c_uint64, lp, lp,
                                                            lp, lp, vp, vp, sz, vp, vp]
        L.nsrl_mlp_workspace_size.restype = sz
        L.nsrl_mlp_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_prenorm_gated_mlp_residual_block.argtypes = [vp, sz, sz, sz, vp, C.c_uint64, lp, lp, lp, vp, vp, sz,
                                                            vp, vp]
        L.nsrl_transformer_block_workspace_size.restype = sz
        L.nsrl_transformer_block_workspace_size.argtypes = [sz, sz, sz, sz, sz]
        L.nsrl_prenorm_transformer_block.argtypes = [vp, sz, sz, sz, sz, sz, vp, vp, C.c_uint64, lp, lp, lp, lp, lp,
                                                     lp, lp, vp, vp, sz, vp, vp]
        L.nsrl_attention_decode.argtypes = [vp, vp, vp, vp, sz, sz, sz, sz, vp, vp, vp]
        L.nsrl_transformer_block_host_workspace_size.restype = sz
        L.nsrl_transformer_block_host_workspace_size.argtypes = [sz, sz, sz, sz, sz]
        L.nsrl_prenorm_transformer_block_host.argtypes = [vp, sz, sz, sz, sz, sz, sz, vp, vp, C.c_uint64, lp, lp, lp,
                                                          lp, lp, lp, lp, vp, vp, sz, vp, vp]
        L.nsrl_profile_enable.argtypes = [C.c_int]
        L.nsrl_profile_count.restype = sz
        _lib = L
    return _lib


def _dev() -> torch.device:
    if not torch.cuda.is_available():
        raise NsrlError("nsrl_b200 needs a CUDA device")
    return torch.device("cuda", torch.cuda.current_device())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


def make_scales(multiplier, right_shift, n: Optional[int] = None, device=None) -> torch.Tensor:
    """FixedScale array as a [n, 2] int32 device tensor (multiplier, right_shift | padding)."""
    mult = torch.as_tensor(multiplier, dtype=torch.int64)
    shift = torch.as_tensor(right_shift, dtype=torch.int64)
    if n is not None:
        mult = mult.expand(n) if mult.dim() else mult.repeat(n)
        shift = shift.expand(n) if shift.dim() else shift.repeat(n)
    s = torch.stack([mult, shift & 255], dim=1).to(torch.int32)
    return s.to(device or _dev()).contiguous()


class Linear:
    """LinearI16I8Params on the device: weights [out][in] int8, optional int32 bias, FixedScale per channel."""

    def __init__(self, weights: torch.Tensor, scales: torch.Tensor, bias: Optional[torch.Tensor] = None):
        dev = _dev()
        self.weights = weights.to(dev, torch.int8).contiguous()
        self.output_dim, self.input_dim = self.weights.shape
        self.scales = scales.to(dev, torch.int32).contiguous()
        self.bias = None if bias is None else bias.to(dev, torch.int32).contiguous()

    def c(self) -> LinearParamsC:
        return LinearParamsC(self.weights.data_ptr(), None if self.bias is None else self.bias.data_ptr(),
                             self.scales.data_ptr(), self.input_dim, self.output_dim)


class Status:
    """Device status word of a call (nsrl_device_status)."""

    def __init__(self):
        self.buf = torch.zeros(8, dtype=torch.int64, device=_dev())

    def reset(self):
        _check(lib().nsrl_status_reset(_ptr(self.buf), _stream()))

    def fetch(self) -> tuple[int, DeviceStatusC]:
        h = DeviceStatusC()
        r = lib().nsrl_status_fetch(_ptr(self.buf), C.byref(h), _stream())
        if r not in (NSRL_OK, NSRL_CORE_REJECTED):
            _check(r)
        return r, h


_ws_cache: dict = {}


def workspace(nbytes: int) -> torch.Tensor:
    """A reusable device scratch buffer of at least nbytes (the caller-owned workspace)."""
    dev = _dev()
    t = _ws_cache.get(dev)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _ws_cache[dev] = t
    return t


def _check(r: int):
    if r == NSRL_OK:
        return
    msg = lib().nsrl_last_error().decode()
    if r == NSRL_CUDA_ERROR:
        raise NsrlError(msg)
    raise NsrlError(f"status {r}: {msg}")


def _run(call, status: Status):
    """Runs a C-ABI call; returns the host status or None for a reference `None`."""
    r = call()
    if r == NSRL_INVALID_SHAPE:
        return None
    _check(r)
    code, h = status.fetch()
    return None if code == NSRL_CORE_REJECTED else h


def _i16(x: torch.Tensor) -> torch.Tensor:
    if x.dtype != torch.int16 or not x.is_cuda:
        raise NsrlError("activations must be int16 CUDA tensors")
    return x.contiguous()


# ----------------------------------------------------------------- linear ---
def linear_i16_i8_i16_per_channel_checked(x: torch.Tensor, lin: Linear) -> Optional[torch.Tensor]:
    """linear.rs:115-126, one call per row of x [rows, input_dim]."""
    x = _i16(x)
    rows = x.numel() // max(lin.input_dim, 1)
    y = torch.empty((rows, lin.output_dim), dtype=torch.int16, device=x.device)
    ws = workspace(lib().nsrl_linear_workspace_size(rows, lin.input_dim, lin.output_dim))
    st = Status()
    p = lin.c()
    h = _run(lambda: lib().nsrl_linear_i16_i8_i16(_ptr(x), rows, C.byref(p), _ptr(y), _ptr(ws), ws.numel(),
                                                  _ptr(st.buf), _stream()), st)
    return None if h is None else y


# --------------------------------------------------------------- rms norm ---
def rms_norm_i16_q15_checked(x: torch.Tensor, gamma: torch.Tensor, eps: int) -> Optional[torch.Tensor]:
    """rms_norm.rs:68-89, one call per row of x [rows, dim]."""
    x = _i16(x)
    g = _i16(gamma)
    d = g.numel()
    rows = x.numel() // max(d, 1)
    y = torch.empty_like(x)
    st = Status()
    h = _run(lambda: lib().nsrl_rms_norm_rows(_ptr(x), rows, d, _ptr(g), eps, _ptr(y), _ptr(st.buf), _stream()), st)
    return None if h is None else y


# -------------------------------------------------------------- attention ---
def self_attention_i16_q15_checked(x, batch, seq_len, d_model, heads, q, k, v, o, causal=True):
    """attention.rs:727-877 over `batch` sequences of seq_len tokens: x [batch*seq_len, d_model]."""
    x = _i16(x)
    out = torch.empty((batch * seq_len, d_model), dtype=torch.int16, device=x.device)
    ws = workspace(lib().nsrl_attention_workspace_size(batch, seq_len, d_model, heads))
    st = Status()
    ps = [l.c() for l in (q, k, v, o)]
    h = _run(lambda: lib().nsrl_self_attention(_ptr(x), batch, seq_len, d_model, heads, int(causal),
                                               *[C.byref(p) for p in ps], _ptr(out), _ptr(ws), ws.numel(),
                                               _ptr(st.buf), _stream()), st)
    return None if h is None else out


def prenorm_attention_residual_block_i16_q15_checked(x, batch, seq_len, d_model, heads, rms_gamma, rms_eps, q, k, v,
                                                     o, causal=True):
    """attention.rs:1522-1583: returns (y, residual saturation count) or None."""
    x = _i16(x)
    g = _i16(rms_gamma)
    y = torch.empty((batch * seq_len, d_model), dtype=torch.int16, device=x.device)
    ws = workspace(lib().nsrl_attention_workspace_size(batch, seq_len, d_model, heads))
    st = Status()
    ps = [l.c() for l in (q, k, v, o)]
    h = _run(lambda: lib().nsrl_prenorm_attention_residual_block(
        _ptr(x), batch, seq_len, d_model, heads, int(causal), _ptr(g), rms_eps, *[C.byref(p) for p in ps], _ptr(y),
        _ptr(ws), ws.numel(), _ptr(st.buf), _stream()), st)
    return None if h is None else (y, h.attention_saturations)


# -------------------------------------------------------------------- mlp ---
def prenorm_gated_mlp_residual_block_i16_q15_checked(x, rows, d_model, hidden_dim, rms_gamma, rms_eps, up, gate,
                                                     down):
    """mlp.rs:541-594: returns (y, residual saturation count) or None."""
    x = _i16(x)
    g = _i16(rms_gamma)
    y = torch.empty((rows, d_model), dtype=torch.int16, device=x.device)
    ws = workspace(lib().nsrl_mlp_workspace_size(rows, d_model, hidden_dim))
    st = Status()
    ps = [l.c() for l in (up, gate, down)]
    h = _run(lambda: lib().nsrl_prenorm_gated_mlp_residual_block(
        _ptr(x), rows, d_model, hidden_dim, _ptr(g), rms_eps, *[C.byref(p) for p in ps], _ptr(y), _ptr(ws),
        ws.numel(), _ptr(st.buf), _stream()), st)
    return None if h is None else (y, h.mlp_saturations)


class TransformerBlock:
    """Weights of one prenorm attention + gated-MLP block (the bench-1m block shape)."""

    def __init__(self, d_model, heads, hidden_dim, q, k, v, o, up, gate, down, attn_gamma, mlp_gamma, rms_eps=1):
        self.d_model, self.heads, self.hidden_dim = d_model, heads, hidden_dim
        self.q, self.k, self.v, self.o, self.up, self.gate, self.down = q, k, v, o, up, gate, down
        self.attn_gamma = attn_gamma.to(_dev(), torch.int16).contiguous()
        self.mlp_gamma = mlp_gamma.to(_dev(), torch.int16).contiguous()
        self.rms_eps = rms_eps
        self._ps = [l.c() for l in (q, k, v, o, up, gate, down)]

    def workspace_bytes(self, batch, seq_len):
        return lib().nsrl_transformer_block_workspace_size(batch, seq_len, self.d_model, self.heads, self.hidden_dim)

    def launch(self, x, y, batch, seq_len, ws, status: Status, stream=None) -> int:
        """Enqueues the block on the stream (no synchronisation); returns the C status code."""
        return lib().nsrl_prenorm_transformer_block(
            _ptr(x), batch, seq_len, self.d_model, self.heads, self.hidden_dim, _ptr(self.attn_gamma),
            _ptr(self.mlp_gamma), self.rms_eps, *[C.byref(p) for p in self._ps], _ptr(y), _ptr(ws), ws.numel(),
            _ptr(status.buf), stream if stream is not None else _stream())

    def host_workspace_bytes(self, chunk, seq_len):
        return lib().nsrl_transformer_block_host_workspace_size(chunk, seq_len, self.d_model, self.heads,
                                                                self.hidden_dim)

    def launch_host(self, x_host, y_host, batch, seq_len, chunk, ws, status: Status, stream=None) -> int:
        """Enqueues the block over pinned host tensors x_host -> y_host in chunks of
        `chunk` sequences, copies overlapping compute; returns the C status code."""
        return lib().nsrl_prenorm_transformer_block_host(
            C.c_void_p(x_host.data_ptr()), batch, chunk, seq_len, self.d_model, self.heads, self.hidden_dim,
            _ptr(self.attn_gamma), _ptr(self.mlp_gamma), self.rms_eps, *[C.byref(p) for p in self._ps],
            C.c_void_p(y_host.data_ptr()), _ptr(ws), ws.numel(), _ptr(status.buf),
            stream if stream is not None else _stream())

    def __call__(self, x, batch, seq_len):
        """Returns (y, attention saturations, mlp saturations) or None."""
        x = _i16(x)
        y = torch.empty_like(x)
        ws = workspace(self.workspace_bytes(batch, seq_len))
        st = Status()
        h = _run(lambda: self.launch(x, y, batch, seq_len, ws, st), st)
        return None if h is None else (y, h.attention_saturations, h.mlp_saturations)


# ----------------------------------------------------------------- decode ---
def prenorm_attention_decode_block(x, heads, rms_gamma, rms_eps, q, k, v, o, k_cache, v_cache, positions):
    """One decode step of the prenorm attention block (see nsrl_prenorm_attention_decode_block):
    x [B, d]; head-major caches [B, H, Lmax, 64] (row positions[b] of every head is written);
    returns (y, saturations) or None."""
    L = lib()
    if not getattr(L, "_decode_bound", False):
        vp, sz, lp = C.c_void_p, C.c_size_t, C.POINTER(LinearParamsC)
        L.nsrl_decode_block_workspace_size.restype = sz
        L.nsrl_decode_block_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_prenorm_attention_decode_block.argtypes = [vp, sz, sz, sz, vp, C.c_uint64, lp, lp, lp, lp, vp, vp, vp,
                                                          sz, vp, vp, sz, vp, vp]
        L._decode_bound = True
    x = _i16(x)
    g = _i16(rms_gamma)
    B, d = x.shape
    y = torch.empty_like(x)
    pos = positions.to(x.device, torch.int32).contiguous()
    ws = workspace(L.nsrl_decode_block_workspace_size(B, d, heads))
    st = Status()
    ps = [l.c() for l in (q, k, v, o)]
    h = _run(lambda: L.nsrl_prenorm_attention_decode_block(
        _ptr(x), B, d, heads, _ptr(g), rms_eps, *[C.byref(p) for p in ps], _ptr(k_cache), _ptr(v_cache), _ptr(pos),
        k_cache.shape[2], _ptr(y), _ptr(ws), ws.numel(), _ptr(st.buf), _stream()), st)
    return None if h is None else (y, h.attention_saturations)

def attention_decode(q, k_cache, v_cache, lens, heads, head_dim):
    """attention.rs:671-725 for every (sequence, head): q [B, H*hd], caches [B, Lmax, H*hd], lens [B] int32."""
    q = _i16(q)
    kc, vc = _i16(k_cache), _i16(v_cache)
    B, Lmax = kc.shape[0], kc.shape[1]
    ln = lens.to(q.device, torch.int32).contiguous()
    ctx = torch.empty_like(q)
    st = Status()
    h = _run(lambda: lib().nsrl_attention_decode(_ptr(q), _ptr(kc), _ptr(vc), _ptr(ln), B, heads, head_dim, Lmax,
                                                 _ptr(ctx), _ptr(st.buf), _stream()), st)
    return None if h is None else ctx


# ------------------------------------------------------- linear attention ---
def _bind_linear_attention(L):
    if not getattr(L, "_la_bound", False):
        vp, sz, lp = C.c_void_p, C.c_size_t, C.POINTER(LinearParamsC)
        L.nsrl_linear_attention_workspace_size.restype = sz
        L.nsrl_linear_attention_workspace_size.argtypes = [sz, sz, sz]
        L.nsrl_linear_attention.argtypes = [vp, sz, sz, sz, sz, C.c_int, lp, lp, lp, lp, vp, vp, sz, vp, vp]
        L.nsrl_linear_attention_step_workspace_size.restype = sz
        L.nsrl_linear_attention_step_workspace_size.argtypes = [sz, sz]
        L.nsrl_linear_attention_step.argtypes = [vp, sz, sz, sz, lp, lp, lp, lp, vp, vp, C.c_int, vp, vp, vp, sz, vp,
                                                 vp]
        L._la_bound = True
    return L


def linear_attention_i16_q15_checked(x, batch, seq_len, d_model, heads, q, k, v, o, causal=True):
    """attention.rs:879-1041 over `batch` sequences of x [batch*seq_len, d]; None on a rejection."""
    L = _bind_linear_attention(lib())
    x = _i16(x)
    out = torch.empty((batch * seq_len, d_model), dtype=torch.int16, device=x.device)
    ws = workspace(L.nsrl_linear_attention_workspace_size(batch, seq_len, d_model))
    st = Status()
    ps = [l.c() for l in (q, k, v, o)]
    h = _run(lambda: L.nsrl_linear_attention(_ptr(x), batch, seq_len, d_model, heads, int(causal),
                                             *[C.byref(p) for p in ps], _ptr(out), _ptr(ws), ws.numel(),
                                             _ptr(st.buf), _stream()), st)
    return None if h is None else out


class LinearAttentionStreams:
    """Carried states of `batch` linear-attention streams ([batch][heads][hd][hd]
    and [batch][heads][hd] int64, zero at the start)."""

    def __init__(self, batch, d_model, heads, device=None):
        dev = device if device is not None else _dev()
        hd = d_model // heads
        self.batch, self.d_model, self.heads = batch, d_model, heads
        self.state = torch.zeros((batch, heads * hd * hd), dtype=torch.int64, device=dev)
        self.key_sums = torch.zeros((batch, heads * hd), dtype=torch.int64, device=dev)
        self.delta_l1 = torch.zeros(batch, dtype=torch.int64, device=dev)

    def step(self, x, q, k, v, o, ttt_shift=None):
        """attention.rs:1045-1283 on rows x [batch, d]; the output rows or None."""
        L = _bind_linear_attention(lib())
        x = _i16(x)
        out = torch.empty_like(x)
        ws = workspace(L.nsrl_linear_attention_step_workspace_size(self.batch, self.d_model))
        st = Status()
        ps = [l.c() for l in (q, k, v, o)]
        h = _run(lambda: L.nsrl_linear_attention_step(
            _ptr(x), self.batch, self.d_model, self.heads, *[C.byref(p) for p in ps], _ptr(self.state),
            _ptr(self.key_sums), -1 if ttt_shift is None else int(ttt_shift), _ptr(self.delta_l1), _ptr(out),
            _ptr(ws), ws.numel(), _ptr(st.buf), _stream()), st)
        return None if h is None else out
