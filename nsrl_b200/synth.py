"""Seeded synthetic inputs for the NSRL integer hot path (numpy, platform-exact).

All generators draw from SplitMix64 (crates/nsrl-demo/src/bench.rs:912-925);
the i-th draw of a stream seeded with s is mix(s + (i + 1) * 0x9e3779b97f4a7c15),
which vectorises.  Tensor t of a workload uses seed ^ (t * 0x9e3779b97f4a7c15).

- Q15 activations "Gaussian sigma 4096": Irwin-Hall sum of 12 uniform 24-bit
  draws, centred and shifted right by 12 (exactly sigma 4096, support +-24576).
- i8 weights uniform in [-127, 127]: (draw >> 32) * 255 >> 32, minus 127.
- Per-channel scales FixedScale{1, s} with s = round(log2(sigma_x * 73.6 *
  sqrt(K) / 4096)) (73.6 = std of U[-127, 127]), which keeps projection
  outputs near sigma 4096 instead of saturating.
The bench-1m preset (bench.rs:38-48, :707-843) is reproduced draw for draw.
"""
from __future__ import annotations

import math

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def splitmix(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Draws start..start+n-1 of SplitMix64(seed) as uint64."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * GAMMA
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def tensor_seed(seed: int, tensor_id: int) -> int:
    return (seed ^ ((tensor_id * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF)) & 0xFFFFFFFFFFFFFFFF


def q15_gaussian(seed: int, shape, sigma_shift: int = 12) -> np.ndarray:
    """Irwin-Hall N(0, 2^(24 - sigma_shift)) in int16 (sigma 4096 by default)."""
    n = int(np.prod(shape))
    u = (splitmix(seed, 12 * n) >> np.uint64(40)).astype(np.int64).reshape(n, 12)
    s = u.sum(axis=1) - 6 * (1 << 24)
    return np.clip(s >> sigma_shift, -32768, 32767).astype(np.int16).reshape(shape)


def _to_i64(v: int) -> int:
    v &= 0xFFFFFFFFFFFFFFFF
    return v - (1 << 64) if v >> 63 else v


def q15_gaussian_torch(seed: int, shape, device, sigma_shift: int = 12, chunk: int = 1 << 22):
    """q15_gaussian computed with torch int64 ops on `device` (bit-identical:
    the same SplitMix64 draws, wrapping multiplies, logical shifts by mask)."""
    import torch
    n = int(np.prod(shape))
    out = torch.empty(n, dtype=torch.int16, device=device)
    g, m1, m2 = _to_i64(int(GAMMA)), _to_i64(int(M1)), _to_i64(int(M2))
    s0 = _to_i64(seed)

    def lsr(z, k):
        return (z >> k) & ((1 << (64 - k)) - 1)

    for c0 in range(0, n, chunk):
        cn = min(chunk, n - c0)
        z = torch.arange(12 * c0 + 1, 12 * (c0 + cn) + 1, dtype=torch.int64, device=device) * g + s0
        z = (z ^ lsr(z, 30)) * m1
        z = (z ^ lsr(z, 27)) * m2
        z = z ^ lsr(z, 31)
        u = lsr(z, 40).view(cn, 12).sum(dim=1) - 6 * (1 << 24)
        out[c0:c0 + cn] = (u >> sigma_shift).clamp_(-32768, 32767).to(torch.int16)
    return out.view(tuple(shape) if isinstance(shape, (tuple, list)) else (shape,))


def i8_uniform(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    d = splitmix(seed, n) >> np.uint64(32)
    return (((d * np.uint64(255)) >> np.uint64(32)).astype(np.int64) - 127).astype(np.int8).reshape(shape)


def shift_for(K: int, sigma_x: float = 4096.0) -> int:
    return int(round(math.log2(sigma_x * 73.6 * math.sqrt(K) / 4096.0)))


class BlockWeights:
    """One prenorm attention + gated-MLP block of synthetic weights (host numpy)."""

    def __init__(self, seed: int, d: int, hidden: int, qk_extra_shift: int = 7, gamma: int = 4096):
        self.d, self.hidden = d, hidden
        t = [tensor_seed(seed, i) for i in range(1, 8)]
        self.q = i8_uniform(t[0], (d, d))
        self.k = i8_uniform(t[1], (d, d))
        self.v = i8_uniform(t[2], (d, d))
        self.o = i8_uniform(t[3], (d, d))
        self.up = i8_uniform(t[4], (hidden, d))
        self.gate = i8_uniform(t[5], (hidden, d))
        self.down = i8_uniform(t[6], (d, hidden))
        s_d = shift_for(d)
        self.shift = dict(q=s_d + qk_extra_shift, k=s_d + qk_extra_shift, v=s_d, o=s_d, up=s_d, gate=s_d,
                          down=shift_for(hidden, 400.0))
        self.attn_gamma = np.full(d, gamma, np.int16)
        self.mlp_gamma = np.full(d, gamma, np.int16)

    def out_dim(self, name):
        return self.hidden if name in ("up", "gate") else self.d


# ------------------------------------------------------------- bench-1m ---
BENCH_1M = dict(seq_len=128, d_model=128, heads=2, hidden_dim=512, blocks=4, seed=0x4E53524C5F314D21)
BENCH_1M_SHIFTS = dict(q=10, k=10, v=7, o=5, up=9, gate=8, down=5)  # bench.rs:734-779
BENCH_1M_OUTPUT_HASH = 0xF7DD983B8CE7A156  # ENG.md:790-799


def bench1m_model():
    """Ternary weights of the bench-1m preset in generation order (bench.rs:707-735, :834-842)."""
    p = BENCH_1M
    d, F = p["d_model"], p["hidden_dim"]
    sizes = [("q", (d, d)), ("k", (d, d)), ("v", (d, d)), ("o", (d, d)), ("up", (F, d)), ("gate", (F, d)),
             ("down", (d, F))]
    per_block = sum(a * b for _, (a, b) in sizes)
    draws = splitmix(p["seed"], per_block * p["blocks"]) & np.uint64(7)
    tern = np.where(draws == 0, -1, np.where(draws == 1, 1, 0)).astype(np.int8)
    blocks, off = [], 0
    for _ in range(p["blocks"]):
        blk = {}
        for name, (a, b) in sizes:
            blk[name] = tern[off:off + a * b].reshape(a, b)
            off += a * b
        blocks.append(blk)
    return blocks


def bench1m_input():
    """bench.rs:822-832."""
    p = BENCH_1M
    S, d = p["seq_len"], p["d_model"]
    n = S * d
    noise = ((splitmix(p["seed"] ^ 0xA17E57116D5A1234, n) >> np.uint64(53)).astype(np.int64) - 512)
    idx = np.arange(n)
    token, channel = idx // d, idx % d
    x = ((token & 31) - 16) * 16 + ((channel & 15) - 8) * 8 + noise
    return x.astype(np.int16).reshape(S, d)


def fnv1a_i16(values: np.ndarray) -> int:
    """StableHasher::update_i16_slice + finish (bench.rs:928-975): length as u64 LE, then LE bytes."""
    h = 0xCBF29CE484222325
    data = int(values.size).to_bytes(8, "little") + np.ascontiguousarray(values, dtype="<i2").tobytes()
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


# ------------------------------------------------------ training workload ---
class TrainWeights:
    """Synthetic mini-transformer weights for the training step: seeded
    BlockWeights per layer, Q15 Gaussian token embeddings (sigma 4096),
    Gaussian learned positions (sigma 1024) and a uniform i8 byte head
    (output scale shift 8, the reference's fixed output scale)."""

    def __init__(self, seed: int, layers: int, d: int, hidden: int, seq_len: int):
        self.blocks = [BlockWeights(seed + 17 * (li + 1), d, hidden) for li in range(layers)]
        self.embeddings = q15_gaussian(tensor_seed(seed, 101), (256, d))
        self.positions = q15_gaussian(tensor_seed(seed, 102), (seq_len, d), sigma_shift=14)
        self.head = i8_uniform(tensor_seed(seed, 103), (256, d))
        self.head_shift = 8


def train_windows(seed: int, windows: int, seq_len: int):
    """Byte windows [windows][seq_len] and their targets, uniform over 0..255 (SplitMix64)."""
    draws = splitmix(seed, windows * (seq_len + 1)) >> np.uint64(56)
    a = draws.astype(np.uint8).reshape(windows, seq_len + 1)
    return np.ascontiguousarray(a[:, :seq_len]), np.ascontiguousarray(a[:, seq_len])
