"""Model and window builders for the training-step tests (numpy; no GPU).

reference_initial_model() restates the reference's initial mini transformer
(crates/nsrl-train/src/lib.rs:9650-9710 with :14696-14860, default build:
d_model 128, heads 2, hidden 256, identity scales from
crates/nsrl-train-core/src/lib.rs:51-90).  random_model() builds seeded
models at other sizes for the parity tests.
"""
from __future__ import annotations

import numpy as np

from oracle import oracle as O

TEXT = b"To be or not to be, that is the question. To be or not to be, that is the question. "


def _identity(dim):
    w = np.zeros((dim, dim), np.int8)
    np.fill_diagonal(w, 1)
    return w


def reference_initial_model(seq_len=4, layers=2):
    """MiniTransformerMlpModel::new_initial_with_seq_len_and_layers (lib.rs:9660-9710)."""
    d, H, F = 128, 2, 256
    tok = np.arange(256)[:, None]
    dim = np.arange(d)[None, :]
    emb = (((tok * 29 + dim * 13 + 5) % 33) - 16) * 32                      # :14696-14712
    pos_i = np.arange(seq_len)[:, None] + 1
    axis = dim + 1
    mixed = pos_i * 31 + axis * 17 + pos_i * axis * 7                       # :14899-14909
    positions = ((mixed % 17) - 8) * 128
    hid = np.arange(F)[:, None]
    up = (((hid * 7 + dim * 11 + 3) % 5) - 2).astype(np.int8)             # :14812-14824
    dm = np.arange(d)[:, None]
    hd = np.arange(F)[None, :]
    down = (((dm * 17 + hd * 5 + 1) % 5) - 2).astype(np.int8)             # :14826-14842
    cls = np.arange(256)[:, None]
    out = (((cls * 19 + dim * 23 + 7) % 7) - 3).astype(np.int8)           # :14844-14860
    sd, sf = O.scales(1, 0, d), O.scales(1, 0, F)
    ly = []
    for li in range(layers):
        final = li == layers - 1                                           # stack_i8_layers_with_active_final
        ly.append({
            "q": O.Linear(_identity(d), sd), "k": O.Linear(_identity(d), sd), "v": O.Linear(_identity(d), sd),
            "o": O.Linear(_identity(d) if final else np.zeros((d, d), np.int8), sd),
            "up": O.Linear(up, sf), "gate": O.Linear(up, sf),
            "down": O.Linear(down if final else np.zeros((d, F), np.int8), sd),
        })
    head = O.Linear(out, O.scales(1, 8, 256))
    return O.TrainModel(emb.astype(np.int16), positions.astype(np.int16), ly, head, d, H, F, seq_len)


def window_starts(token_count, seq_len, stride, max_windows):
    """mini_transformer_window_starts (lib.rs:13317-13358) with offset 0."""
    last = token_count - seq_len - 1
    available = last // stride + 1
    limit = min(max_windows, available)
    if limit >= available:
        return [i * stride for i in range(available)]
    if limit == 1:
        return [0]
    den = limit - 1
    return [((i * (available - 1) + den // 2) // den) * stride for i in range(limit)]


def windows_from_text(tokens: bytes, seq_len, starts):
    ctx = np.array([list(tokens[s:s + seq_len]) for s in starts], np.uint8)
    tgt = np.array([tokens[s + seq_len] for s in starts], np.uint8)
    return ctx, tgt


def _shift_for(K, sigma=4096):
    return max(0, int(round(np.log2(sigma * 73.6 * np.sqrt(K) / 4096))))


def random_model(d, H, F, layers, S, rms=True, positions=True, seed=0, qk_extra=7):
    """Seeded model: uniform i8 weights, shifts that keep sigma-4096 activations live."""
    rng = np.random.default_rng(seed)

    def lin(out_dim, in_dim, extra=0):
        w = rng.integers(-127, 128, (out_dim, in_dim)).astype(np.int8)
        return O.Linear(w, O.scales(1, min(62, _shift_for(in_dim) + extra), out_dim))

    ly = []
    for _ in range(layers):
        e = {"q": lin(d, d, qk_extra), "k": lin(d, d, qk_extra), "v": lin(d, d), "o": lin(d, d),
             "up": lin(F, d), "gate": lin(F, d), "down": lin(d, F)}
        if rms:
            e["attn_gamma"] = rng.integers(2048, 16384, d).astype(np.int16)
            e["mlp_gamma"] = rng.integers(2048, 16384, d).astype(np.int16)
        ly.append(e)
    emb = np.clip(rng.normal(0, 4096, (256, d)), -32768, 32767).astype(np.int16)
    pos = np.clip(rng.normal(0, 1024, (S, d)), -32768, 32767).astype(np.int16) if positions else None
    head = O.Linear(rng.integers(-127, 128, (256, d)).astype(np.int8), O.scales(1, 8, 256))
    return O.TrainModel(emb, pos, ly, head, d, H, F, S)


def random_windows(W, S, seed=0):
    rng = np.random.default_rng(seed + 1000)
    return rng.integers(0, 256, (W, S)).astype(np.uint8), rng.integers(0, 256, W).astype(np.uint8)
