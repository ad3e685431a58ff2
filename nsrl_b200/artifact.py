"""The mini transformer's on-disk artifact (.nsrlmt, version 5): read, write,
and turn into a device model.

Mirrors MiniTransformerMlpModel::try_to_bytes / from_bytes
(crates/nsrl-train/src/lib.rs:10066-10470) and the model hashes it records
(:9983-10040, StableHasher :19442-19519): the magic b"NSRLMT5\\n"; vocab,
d_model, heads, hidden_dim, context_seq_len as u32; the element counts of
the embeddings, positions, q, k, v, o, up, gate, down and output tensors as
u64; the embedding, q, k, v, o, MLP, output-head and model hashes as u64;
then the tensors (i16 little-endian, i8 as bytes), and the attention and
MLP RMS gammas (i16) when the artifact carries them.  Every tensor of a
stacked model holds its layers one after the other.  Loading checks the
counts, the length and every hash, as the reference does.  The version-4
format (32-wide models, which the reference upgrades on load) is rejected.

The artifact stores no scales: the forward scale tables are the build's
(crates/nsrl-train-core/src/lib.rs:51-90), named here by `profile`:
"default" (d_model and hidden linears unshifted, the byte head shifted by
8) or "calibrated" (shifts 1, 2 and 8).
"""
from __future__ import annotations

import dataclasses
import struct
from typing import Optional

import numpy as np

MAGIC = b"NSRLMT5\n"
LEGACY_MAGIC = b"NSRLMT4\n"
VOCAB = 256
PROFILES = {"default": (0, 0, 8), "calibrated": (1, 2, 8)}  # d_model, hidden, output right shifts


class ArtifactError(ValueError):
    """InvalidModel (lib.rs:10230-10470): the bytes are not a valid artifact."""


def _fnv_bytes(h: int, data: bytes) -> int:
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


class _Hasher:
    """StableHasher (lib.rs:19468-19519): FNV-1a 64; a slice is its length as a
    u64 followed by its little-endian elements."""

    def __init__(self):
        self.h = 0xCBF29CE484222325

    def usize(self, v: int):
        self.h = _fnv_bytes(self.h, struct.pack("<Q", v))

    def slice(self, a: np.ndarray):
        self.usize(a.size)
        self.h = _fnv_bytes(self.h, np.ascontiguousarray(a).astype(a.dtype.newbyteorder("<")).tobytes())


def _hash(*arrays) -> int:
    h = _Hasher()
    for a in arrays:
        h.slice(a)
    return h.h


@dataclasses.dataclass
class MiniTransformerArtifact:
    d_model: int
    heads: int
    hidden_dim: int
    seq_len: int
    embeddings: np.ndarray       # [256][d] i16
    positions: np.ndarray        # [seq_len][d] i16 (may be empty)
    q: np.ndarray                # [layers][d][d] i8
    k: np.ndarray
    v: np.ndarray
    o: np.ndarray
    up: np.ndarray               # [layers][hidden][d] i8
    gate: np.ndarray
    down: np.ndarray             # [layers][d][hidden] i8
    output: np.ndarray           # [256][d] i8
    attention_rms: Optional[np.ndarray] = None  # [layers][d] i16
    mlp_rms: Optional[np.ndarray] = None

    @property
    def layers(self) -> int:
        return self.q.shape[0]

    # ---- the hashes the artifact records (lib.rs:9983-10040)
    def embedding_hash(self):
        return _hash(self.embeddings, self.positions)

    def q_hash(self):
        return _hash(self.q)

    def k_hash(self):
        return _hash(self.k)

    def v_hash(self):
        return _hash(self.v)

    def o_hash(self):
        return _hash(self.o)

    def mlp_hash(self):
        return _hash(self.up, self.gate, self.down)

    def output_head_hash(self):
        return _hash(self.output)

    def model_hash(self):
        h = _Hasher()
        h.usize(self.seq_len)
        h.slice(self.embeddings)
        h.slice(self.positions)
        if self.attention_rms is not None:
            h.slice(self.attention_rms)
            h.slice(self.mlp_rms)
        for a in (self.q, self.k, self.v, self.o, self.up, self.gate, self.down, self.output):
            h.slice(a)
        return h.h


def to_bytes(a: MiniTransformerArtifact) -> bytes:
    """MiniTransformerMlpModel::try_to_bytes (lib.rs:10066-10216)."""
    out = [MAGIC, struct.pack("<5I", VOCAB, a.d_model, a.heads, a.hidden_dim, a.seq_len)]
    tensors = (a.embeddings, a.positions, a.q, a.k, a.v, a.o, a.up, a.gate, a.down, a.output)
    out.append(struct.pack("<10Q", *[t.size for t in tensors]))
    out.append(struct.pack("<8Q", a.embedding_hash(), a.q_hash(), a.k_hash(), a.v_hash(), a.o_hash(), a.mlp_hash(),
                           a.output_head_hash(), a.model_hash()))
    for t in tensors:
        out.append(np.ascontiguousarray(t).astype(t.dtype.newbyteorder("<")).tobytes())
    if a.attention_rms is not None:
        out.append(np.ascontiguousarray(a.attention_rms, "<i2").tobytes())
        out.append(np.ascontiguousarray(a.mlp_rms, "<i2").tobytes())
    return b"".join(out)


def serialized_model_hash(data: bytes) -> int:
    """MiniTransformerMlpModel::serialized_model_hash (lib.rs:10218-10238)."""
    hl = len(MAGIC) + 4 * 5 + 8 * 10 + 8 * 8
    if len(data) < hl:
        raise ArtifactError("artifact too short")
    if data[:8] not in (MAGIC, LEGACY_MAGIC):
        raise ArtifactError("bad magic")
    off = len(MAGIC) + 4 * 5 + 8 * 10 + 8 * 7
    return struct.unpack_from("<Q", data, off)[0]


def from_bytes(data: bytes) -> MiniTransformerArtifact:
    """MiniTransformerMlpModel::from_bytes (lib.rs:10240-10470) for version 5."""
    hl = len(MAGIC) + 4 * 5 + 8 * 10 + 8 * 8
    if len(data) < hl:
        raise ArtifactError("artifact too short")
    magic = data[:8]
    if magic == LEGACY_MAGIC:
        raise ArtifactError("version-4 artifact: load and re-save it with the reference to upgrade it")
    if magic != MAGIC:
        raise ArtifactError("bad magic")
    vocab, d, H, F, S = struct.unpack_from("<5I", data, 8)
    counts = struct.unpack_from("<10Q", data, 28)
    hashes = struct.unpack_from("<8Q", data, 108)
    off = hl
    emb_n, pos_n, q_n, k_n, v_n, o_n, up_n, gate_n, down_n, out_n = counts
    if vocab != VOCAB or d == 0 or H == 0 or F == 0 or S == 0 or d % H:
        raise ArtifactError("shape mismatch")
    L = q_n // (d * d) if q_n % (d * d) == 0 else 0
    Lm = up_n // (F * d) if up_n % (F * d) == 0 else 0
    if (emb_n != VOCAB * d or pos_n not in (0, S * d) or L == 0 or Lm != L or k_n != q_n or v_n != q_n
            or o_n != q_n or gate_n != up_n or down_n != L * d * F or out_n != VOCAB * d):
        raise ArtifactError("tensor count mismatch")
    base = off + 2 * emb_n + 2 * pos_n + q_n + k_n + v_n + o_n + up_n + gate_n + down_n + out_n
    rms_n = L * d
    if len(data) == base + 4 * rms_n:
        rms = True
    elif len(data) == base:
        rms = False
    else:
        raise ArtifactError("artifact length mismatch")

    def take(n, dt, shape):
        nonlocal off
        size = n * np.dtype(dt).itemsize
        a = np.frombuffer(data, dtype=dt, count=n, offset=off).astype(np.dtype(dt).newbyteorder("="))
        off += size
        return a.reshape(shape)

    emb = take(emb_n, "<i2", (VOCAB, d))
    pos = take(pos_n, "<i2", (pos_n // d, d) if pos_n else (0, d))
    q, k, v, o = (take(q_n, "i1", (L, d, d)) for _ in range(4))
    up = take(up_n, "i1", (L, F, d))
    gate = take(gate_n, "i1", (L, F, d))
    down = take(down_n, "i1", (L, d, F))
    out = take(out_n, "i1", (VOCAB, d))
    ar = take(rms_n, "<i2", (L, d)) if rms else None
    mr = take(rms_n, "<i2", (L, d)) if rms else None
    a = MiniTransformerArtifact(d, H, F, S, emb, pos, q, k, v, o, up, gate, down, out, ar, mr)
    if a.embedding_hash() != hashes[0]:
        raise ArtifactError("embedding hash mismatch")
    if (a.q_hash(), a.k_hash(), a.v_hash(), a.o_hash()) != hashes[1:5]:
        raise ArtifactError("attention hash mismatch")
    if a.mlp_hash() != hashes[5]:
        raise ArtifactError("mlp hash mismatch")
    if a.output_head_hash() != hashes[6]:
        raise ArtifactError("output head hash mismatch")
    if a.model_hash() != hashes[7]:
        raise ArtifactError("model hash mismatch")
    return a


def load(path: str) -> MiniTransformerArtifact:
    with open(path, "rb") as f:
        return from_bytes(f.read())


def to_train_model(a: MiniTransformerArtifact, profile: str = "default", attention_kind: str = "softmax",
                   use_positions: bool = True):
    """The device model (nsrl_b200.train.TrainModel) of an artifact, with the
    forward scales of the build profile; positions off for the position-free
    policy (NoPE) or when the artifact has none."""
    import torch

    from . import core
    from . import train as T
    sd, sf, so = PROFILES[profile]
    d, F = a.d_model, a.hidden_dim
    layers = []
    for li in range(a.layers):
        e = {}
        for nm, w, shift, n in (("q", a.q[li], sd, d), ("k", a.k[li], sd, d), ("v", a.v[li], sd, d),
                                ("o", a.o[li], sd, d), ("up", a.up[li], sf, F), ("gate", a.gate[li], sf, F),
                                ("down", a.down[li], sd, d)):
            e[nm] = core.Linear(torch.from_numpy(np.ascontiguousarray(w)), core.make_scales(1, shift, n))
        if a.attention_rms is not None:
            e["attn_gamma"] = torch.from_numpy(np.ascontiguousarray(a.attention_rms[li]))
            e["mlp_gamma"] = torch.from_numpy(np.ascontiguousarray(a.mlp_rms[li]))
        layers.append(e)
    pos = torch.from_numpy(a.positions.copy()) if use_positions and a.positions.size else None
    head = core.Linear(torch.from_numpy(np.ascontiguousarray(a.output)), core.make_scales(1, so, VOCAB))
    return T.TrainModel(torch.from_numpy(a.embeddings.copy()), pos, layers, head, d, a.heads, F, a.seq_len,
                        attention_kind=attention_kind)
