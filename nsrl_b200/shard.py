"""Head-sharded forward of the transformer block over ranks, one GPU each.

Rank r of n owns positions [r S/n, (r+1) S/n) of every sequence for the
token-wise work (RMS norms, linears, residual adds, MLP) and heads
[r H/n, (r+1) H/n) for attention.  The Q|K|V projection stores each head's
rows straight into the exchange buffer of the head's owner (peer stores over
NVLink from the GEMM epilogue), attention stores each context row into the
buffer of the position's owner, and device-side signals order the phases
(include/nsrl_b200.h, "head-sharded forward").  The result is bit-identical
to the one-GPU block (prenorm_attention_residual_block_i16_q15_checked,
attention.rs:1522-1583, then prenorm_gated_mlp_residual_block_i16_q15_checked,
mlp.rs:541-594), which the reference computes on one CPU.

ShardGroup is one process's rank (torch.distributed carries the IPC handles
at set-up; the data path uses no collective library).  EmulatedShardGroups
runs n ranks in one process on one GPU, with every rank's exchange buffer
local and the phases issued rank by rank, so that no wait depends on a
kernel that has not been launched yet.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import core

IPC_HANDLE_BYTES = 64
MAX_RANKS = 8
FLAG_WAIT_TIMEOUT = 0x100


class ShardError(core.NsrlError):
    """A device wait of the sharded forward ran out (a rank did not signal in time);
    the group is unusable and must be recreated on every rank."""


def positions(seq_len: int, nranks: int, rank: int) -> tuple[int, int]:
    """The positions [start, end) of every sequence that `rank` owns."""
    s = seq_len // nranks
    return rank * s, (rank + 1) * s


def heads(n_heads: int, nranks: int, rank: int) -> tuple[int, int]:
    """The heads [start, end) whose attention `rank` computes."""
    h = n_heads // nranks
    return rank * h, (rank + 1) * h


def split_positions(x: torch.Tensor, batch: int, seq_len: int, nranks: int, rank: int) -> torch.Tensor:
    """Rank `rank`'s rows [batch][S/n][d] of x [batch*seq_len][d] (contiguous)."""
    a, b = positions(seq_len, nranks, rank)
    return x.view(batch, seq_len, -1)[:, a:b].contiguous().view(batch * (b - a), -1)


def join_positions(parts: Sequence[torch.Tensor], batch: int) -> torch.Tensor:
    """Inverse of split_positions over all ranks: [batch*seq_len][d]."""
    d = parts[0].shape[-1]
    return torch.cat([p.view(batch, -1, d) for p in parts], dim=1).reshape(-1, d)


def _bind():
    L = core.lib()
    if getattr(L, "_shard_bound", False):
        return L
    vp, sz, lp = C.c_void_p, C.c_size_t, C.POINTER(core.LinearParamsC)
    L.nsrl_shard_exchange_bytes.restype = sz
    L.nsrl_shard_exchange_bytes.argtypes = [sz, sz, sz, sz, sz]
    L.nsrl_shard_alloc.argtypes = [sz, C.POINTER(vp)]
    L.nsrl_shard_free.argtypes = [vp]
    L.nsrl_ipc_get_handle.argtypes = [vp, C.c_char_p]
    L.nsrl_ipc_open.argtypes = [C.c_char_p, C.POINTER(vp)]
    L.nsrl_ipc_close.argtypes = [vp]
    L.nsrl_shard_group_create.argtypes = [C.POINTER(vp), C.c_int, C.c_int, C.POINTER(vp), sz, sz, sz, sz, sz,
                                          C.c_uint64]
    L.nsrl_shard_group_destroy.argtypes = [vp]
    L.nsrl_sharded_block_workspace_size.restype = sz
    L.nsrl_sharded_block_workspace_size.argtypes = [vp, sz]
    L.nsrl_sharded_block_qkv.argtypes = [vp, vp, vp, C.c_uint64, lp, lp, lp, lp, vp, sz, vp, vp]
    L.nsrl_sharded_block_attention.argtypes = [vp, lp, vp, sz, vp, vp]
    L.nsrl_sharded_block_output.argtypes = [vp, vp, lp, vp, C.c_uint64, lp, lp, lp, sz, vp, vp, sz, vp, vp]
    L.nsrl_sharded_transformer_block.argtypes = [vp, vp, vp, vp, C.c_uint64, lp, lp, lp, lp, lp, lp, lp, sz, vp,
                                                 vp, sz, vp, vp]
    L.nsrl_shard_status_post.argtypes = [vp, vp, vp]
    L.nsrl_shard_status_combine.argtypes = [vp, vp, vp]
    L.nsrl_shard_status_allreduce.argtypes = [vp, vp, vp]
    L._shard_bound = True
    return L


class LibraryApi:
    """The exchange-buffer and group calls of the C ABI (a test may pass a fake)."""

    def exchange_bytes(self, batch, seq_len, d_model, n_heads, nranks) -> int:
        return _bind().nsrl_shard_exchange_bytes(batch, seq_len, d_model, n_heads, nranks)

    def alloc(self, nbytes: int) -> int:
        p = C.c_void_p()
        core._check(_bind().nsrl_shard_alloc(nbytes, C.byref(p)))
        return p.value

    def free(self, ptr: int):
        core._check(_bind().nsrl_shard_free(C.c_void_p(ptr)))

    def handle(self, ptr: int) -> bytes:
        buf = C.create_string_buffer(IPC_HANDLE_BYTES)
        core._check(_bind().nsrl_ipc_get_handle(C.c_void_p(ptr), buf))
        return buf.raw

    def open(self, handle: bytes) -> int:
        p = C.c_void_p()
        core._check(_bind().nsrl_ipc_open(handle, C.byref(p)))
        return p.value

    def close(self, ptr: int):
        core._check(_bind().nsrl_ipc_close(C.c_void_p(ptr)))

    def create(self, nranks, rank, buffers, nbytes, batch, seq_len, d_model, n_heads, timeout_ms) -> int:
        g = C.c_void_p()
        arr = (C.c_void_p * nranks)(*buffers)
        core._check(_bind().nsrl_shard_group_create(C.byref(g), nranks, rank, arr, nbytes, batch, seq_len, d_model,
                                                    n_heads, timeout_ms))
        return g.value

    def destroy(self, g: int):
        core._check(_bind().nsrl_shard_group_destroy(C.c_void_p(g)))

    def synchronize(self):
        torch.cuda.synchronize()


class _Rank:
    """One rank's group handle and the calls of its phases."""

    def __init__(self, g: int, nranks: int, rank: int, batch: int, seq_len: int, d_model: int, n_heads: int):
        self.g, self.nranks, self.rank = g, nranks, rank
        self.batch, self.seq_len, self.d_model, self.heads = batch, seq_len, d_model, n_heads
        self.rows = batch * seq_len // nranks

    def workspace_bytes(self, hidden_dim: int = 0) -> int:
        return _bind().nsrl_sharded_block_workspace_size(C.c_void_p(self.g), hidden_dim)

    def qkv(self, block: core.TransformerBlock, x, ws, status: core.Status, stream=None, rms=True) -> int:
        q, k, v, o = (C.byref(p) for p in block._ps[:4])
        return _bind().nsrl_sharded_block_qkv(C.c_void_p(self.g), core._ptr(x),
                                              core._ptr(block.attn_gamma) if rms else None, block.rms_eps, q, k, v,
                                              o, core._ptr(ws), ws.numel(), core._ptr(status.buf),
                                              stream if stream is not None else core._stream())

    def attention(self, block: core.TransformerBlock, ws, status: core.Status, stream=None) -> int:
        return _bind().nsrl_sharded_block_attention(C.c_void_p(self.g), C.byref(block._ps[3]), core._ptr(ws),
                                                    ws.numel(), core._ptr(status.buf),
                                                    stream if stream is not None else core._stream())

    def output(self, block: core.TransformerBlock, x, y, ws, status: core.Status, stream=None, mlp=True,
               rms=True) -> int:
        up, gate, down = ((C.byref(p) for p in block._ps[4:]) if mlp else (None, None, None))
        return _bind().nsrl_sharded_block_output(C.c_void_p(self.g), core._ptr(x), C.byref(block._ps[3]),
                                                 core._ptr(block.mlp_gamma) if rms else None, block.rms_eps, up,
                                                 gate, down, block.hidden_dim if mlp else 0, core._ptr(y),
                                                 core._ptr(ws), ws.numel(), core._ptr(status.buf),
                                                 stream if stream is not None else core._stream())

    def block(self, block: core.TransformerBlock, x, y, ws, status: core.Status, stream=None, mlp=True) -> int:
        """The three phases in one call (nsrl_sharded_transformer_block); returns the C status."""
        lin = [C.byref(p) for p in block._ps[:4]]
        up, gate, down = ((C.byref(p) for p in block._ps[4:]) if mlp else (None, None, None))
        return _bind().nsrl_sharded_transformer_block(
            C.c_void_p(self.g), core._ptr(x), core._ptr(block.attn_gamma), core._ptr(block.mlp_gamma),
            block.rms_eps, *lin, up, gate, down, block.hidden_dim if mlp else 0, core._ptr(y), core._ptr(ws),
            ws.numel(), core._ptr(status.buf), stream if stream is not None else core._stream())

    def post_status(self, status: core.Status, stream=None) -> int:
        return _bind().nsrl_shard_status_post(C.c_void_p(self.g), core._ptr(status.buf),
                                              stream if stream is not None else core._stream())

    def allreduce_status(self, status: core.Status, stream=None) -> int:
        """post_status and combine_status in one launch (ranks in separate processes)."""
        return _bind().nsrl_shard_status_allreduce(C.c_void_p(self.g), core._ptr(status.buf),
                                                   stream if stream is not None else core._stream())

    def combine_status(self, status: core.Status, stream=None) -> int:
        return _bind().nsrl_shard_status_combine(C.c_void_p(self.g), core._ptr(status.buf),
                                                 stream if stream is not None else core._stream())


def _result(status: core.Status):
    """The host status of a finished forward: None for a reference `None`;
    ShardError when a device wait ran out."""
    code, h = status.fetch()
    if h.flags & FLAG_WAIT_TIMEOUT:
        raise ShardError("a device wait of the sharded forward ran out: a rank did not signal in time")
    return None if code == core.NSRL_CORE_REJECTED else h


class ShardGroup(_Rank):
    """This process's rank of a head-sharded forward over `group` (default: the
    world), bound to one shape.  Set-up (collective over the group): allocate
    the exchange buffer, share its CUDA IPC handle, open the others', create
    the group, barrier.  close() releases it (also collective)."""

    def __init__(self, batch: int, seq_len: int, d_model: int, n_heads: int, group=None, timeout_ms: int = 10000,
                 api: Optional[LibraryApi] = None):
        import torch.distributed as dist
        self.api = api or LibraryApi()
        self.pg = group
        nranks, rank = dist.get_world_size(group), dist.get_rank(group)
        if nranks > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        nbytes = self.api.exchange_bytes(batch, seq_len, d_model, n_heads, nranks)
        if nbytes == 0:
            raise ValueError("seq_len and heads must be multiples of the number of ranks")
        self.nbytes = nbytes
        self.own = self.api.alloc(nbytes)
        handles = [None] * nranks
        dist.all_gather_object(handles, self.api.handle(self.own), group=group)
        self.opened = {}
        try:
            for r in range(nranks):
                if r != rank:
                    self.opened[r] = self.api.open(handles[r])
            buffers = [self.own if r == rank else self.opened[r] for r in range(nranks)]
            g = self.api.create(nranks, rank, buffers, nbytes, batch, seq_len, d_model, n_heads, timeout_ms)
        except Exception:
            self._release()
            raise
        super().__init__(g, nranks, rank, batch, seq_len, d_model, n_heads)
        self.buffers = buffers
        dist.barrier(group=group)  # every header is zeroed before any rank signals

    def _release(self):
        for p in self.opened.values():
            self.api.close(p)
        self.opened = {}
        if self.own:
            self.api.free(self.own)
            self.own = 0

    def close(self):
        """Collective: after every rank's last phase has finished on the device."""
        import torch.distributed as dist
        if getattr(self, "g", None):
            self.api.synchronize()
            dist.barrier(group=self.pg)
            self.api.destroy(self.g)
            self.g = None
            self._release()

    def forward(self, block: core.TransformerBlock, x_local: torch.Tensor, mlp: bool = True):
        """y for this rank's rows, with the status of the whole block: (y,
        attention saturations, mlp saturations), or None when the block is a
        reference `None` on any rank."""
        x_local = core._i16(x_local)
        y = torch.empty_like(x_local)
        ws = core.workspace(self.workspace_bytes(block.hidden_dim if mlp else 0))
        st = core.Status()
        st.reset()
        r = self.block(block, x_local, y, ws, st, mlp=mlp)
        if r == core.NSRL_INVALID_SHAPE:
            return None
        core._check(r)
        core._check(self.allreduce_status(st))
        h = _result(st)
        return None if h is None else (y, h.attention_saturations, h.mlp_saturations)


class EmulatedShardGroups:
    """n ranks of the sharded forward in one process on one GPU: each rank's
    exchange buffer is a local allocation, and every phase is issued for all
    ranks before the next phase, on one stream, so that each wait is for
    signals already issued."""

    def __init__(self, nranks: int, batch: int, seq_len: int, d_model: int, n_heads: int, timeout_ms: int = 2000):
        self.api = LibraryApi()
        self.nbytes = self.api.exchange_bytes(batch, seq_len, d_model, n_heads, nranks)
        if self.nbytes == 0:
            raise ValueError("seq_len and heads must be multiples of the number of ranks")
        self.batch, self.seq_len, self.nranks = batch, seq_len, nranks
        self.buffers, self.ranks = [], []
        try:
            for _ in range(nranks):
                self.buffers.append(self.api.alloc(self.nbytes))
            for r in range(nranks):
                g = self.api.create(nranks, r, self.buffers, self.nbytes, batch, seq_len, d_model, n_heads,
                                    timeout_ms)
                self.ranks.append(_Rank(g, nranks, r, batch, seq_len, d_model, n_heads))
        except Exception:
            self.close()
            raise

    def close(self):
        torch.cuda.synchronize()
        for r in self.ranks:
            self.api.destroy(r.g)
        for b in self.buffers:
            self.api.free(b)
        self.ranks, self.buffers = [], []

    def forward(self, block: core.TransformerBlock, x: torch.Tensor, mlp: bool = True, rms: bool = True,
                only: Optional[Sequence[int]] = None):
        """x [batch*seq_len][d] -> per-rank results [(y rows of the rank, host
        status after the combine)], or the first phase's C status code when it
        is not NSRL_OK.  `only` issues the phases of those ranks alone (the
        others never signal)."""
        x = core._i16(x)
        n = self.nranks
        live = list(range(n)) if only is None else list(only)
        xs = [split_positions(x, self.batch, self.seq_len, n, r) for r in range(n)]
        ys = [torch.empty_like(p) for p in xs]
        F = block.hidden_dim if mlp else 0
        wss = [torch.empty(max(self.ranks[r].workspace_bytes(F), 256), dtype=torch.uint8, device=x.device)
               for r in range(n)]
        sts = [core.Status() for _ in range(n)]
        for s in sts:
            s.reset()
        for r in live:
            c = self.ranks[r].qkv(block, xs[r], wss[r], sts[r], rms=rms)
            if c != core.NSRL_OK:
                return c
        for r in live:
            c = self.ranks[r].attention(block, wss[r], sts[r])
            if c != core.NSRL_OK:
                return c
        for r in live:
            c = self.ranks[r].output(block, xs[r], ys[r], wss[r], sts[r], mlp=mlp, rms=rms)
            if c != core.NSRL_OK:
                return c
        for r in live:
            core._check(self.ranks[r].post_status(sts[r]))
        for r in live:
            core._check(self.ranks[r].combine_status(sts[r]))
        out = []
        for r in live:
            code, h = sts[r].fetch()
            out.append((ys[r], code, h))
        return out
