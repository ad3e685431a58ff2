"""CPU restatement of the reference's integer-Adam training run -- TEST
INFRASTRUCTURE (the checker of nsrl_b200.loop, never part of the product).

run_mini_transformer_mlp_integer_adam_training_from_model_with_scope
(crates/nsrl-train/src/lib.rs:4499-4800) for base-2 softmax attention, on
the oracle's numpy model: window starts (:13291-13358), batches through
the map-reduce batch with `workers` chunks merged in order and the Adam
batch apply (oracle.adam_train_step), the candidate checked on the batch and
guard windows (:14617-14700), the optional loss-regression guard
(:13538-13581), and the evaluation counts (:17590-17660, :18539-18548).
"""
from __future__ import annotations

import copy

import numpy as np

from . import oracle as O


def _byte_window_starts(n, S, stride, off, mx):  # lib.rs:13291-13315
    out, s = [], off
    while s + S < n and (mx is None or len(out) < mx):
        out.append(s)
        s += stride
    return out


def window_starts(n, S, stride, off, mx):  # lib.rs:13317-13358
    if S == 0 or stride == 0 or off >= n or n < S + 1:
        return []
    last = n - S - 1
    if off > last:
        return []
    avail = (last - off) // stride + 1
    lim = avail if mx is None else min(mx, avail)
    if lim == 0:
        return []
    if lim >= avail:
        return _byte_window_starts(n, S, stride, off, lim)
    if lim == 1:
        return [off]
    return [off + ((i * (avail - 1) + (lim - 1) // 2) // (lim - 1)) * stride for i in range(lim)]


def _guards(n, epoch, wi, epochs):  # lib.rs:14617-14669
    out = []
    for i in (0, n // 4, n // 2, (n * 3) // 4, n - 1, max(wi - 1, 0), wi, min(wi + 1, n - 1),
              wi + 1 if wi + 1 < n else (0 if epoch + 1 < epochs else wi)):
        if i < n and i not in out:
            out.append(i)
    return out


def _loss_guard(starts, b0, b1):  # lib.rs:13538-13572
    out = []
    for s in starts[min(b0, b1):b1]:
        if s not in out:
            out.append(s)
    n = len(starts)
    pts = min(16, n)
    idx = [0] if pts == 1 else [(p * (n - 1) + (pts - 1) // 2) // (pts - 1) for p in range(pts)]
    for i in idx:
        if starts[i] not in out:
            out.append(starts[i])
    return out


def _counts(model, tok, starts):
    S = model.S
    win = np.stack([tok[s:s + S] for s in starts])
    r = O.output_rows(model, win, threads=8)
    if r is None:
        return None
    mistakes, err = 0, 0
    for i, s in enumerate(starts):
        t = int(tok[s + S])
        lg, pr = r[0][i], r[1][i].astype(np.int64)
        best = int(np.argmax(lg))
        mistakes += int(best != t)
        err += int(max(32767 - pr[t], 0) + np.maximum(np.delete(pr, t), 0).sum())
    return mistakes, err


def _copy_model(m):
    layers = []
    for ly in m.layers:
        e = {n: O.Linear(ly[n].weights.copy(), ly[n].scales.copy(), None if ly[n].bias is None else ly[n].bias.copy())
             for n in O.LAYER_LINEARS}
        for g in ("attn_gamma", "mlp_gamma"):
            if ly.get(g) is not None:
                e[g] = ly[g].copy()
        layers.append(e)
    return O.TrainModel(m.embeddings.copy(), None if m.positions is None else m.positions.copy(), layers,
                        O.Linear(m.head.weights.copy(), m.head.scales.copy()), m.d, m.H, m.F, m.S,
                        attention_kind=m.attention_kind)


def run_integer_adam_training(tokens: bytes, model: O.TrainModel, epochs=1, stride=1, window_offset=0,
                              max_windows=64, batch_windows=1, reject_loss_regression=False, adam=(1, 4, 3, 7, 1),
                              scope="all", state: O.AdamState | None = None, workers=1):
    """Returns (trace dict, model, state); the model and state are new objects."""
    tok = np.frombuffer(bytes(tokens), np.uint8)
    S = model.S
    starts = window_starts(len(tok), S, stride, window_offset, max_windows)
    cfg = O.AdamConfig(*adam)
    if state is None:
        state = O.AdamState(O.adam_state_layout(model)["total"])
    init = _counts(model, tok, starts)
    tr = {"windows": len(starts), "examined_windows": 0, "updates": 0, "accepted_batch_count": 0,
          "rejected_batch_count": 0, "initial_mistakes": init[0], "initial_probability_error_q15": init[1],
          "weight_delta_l1": 0, "mlp_saturation_count": 0, "attention_saturation_count": 0,
          "residual_saturation_count": 0}
    for epoch in range(epochs):
        b0 = 0
        while b0 < len(starts):
            b1 = min(b0 + batch_windows, len(starts))
            tr["examined_windows"] += b1 - b0
            batch = starts[b0:b1]
            ctx = np.stack([tok[s:s + S] for s in batch])
            tgt = np.array([tok[s + S] for s in batch], np.uint8)
            cand, cstate = _copy_model(model), copy.deepcopy(state)
            out = O.adam_train_step(cand, cstate, ctx, tgt, cfg, scope=scope, workers=workers)
            if out is None or out["accepted"] == 0:
                tr["rejected_batch_count"] += 1
                b0 = b1
                continue
            for k in ("mlp_saturation_count", "attention_saturation_count", "residual_saturation_count"):
                tr[k] += out[k]
            valid = _counts(cand, tok, batch) is not None and \
                _counts(cand, tok, [starts[i] for i in _guards(len(starts), epoch, b1 - 1, epochs)]) is not None
            regressed = False
            if valid and reject_loss_regression:
                g = _loss_guard(starts, b0, b1)
                before, after = _counts(model, tok, g), _counts(cand, tok, g)
                regressed = after is None or after[1] > before[1] + len(g) * 1024
            if valid and not regressed:
                model, state = cand, cstate
                tr["updates"] += out["accepted"]
                tr["accepted_batch_count"] += 1
                tr["weight_delta_l1"] += out["weight_delta_l1"]
            else:
                tr["rejected_batch_count"] += 1
            b0 = b1
    fin = _counts(model, tok, starts)
    tr["final_mistakes"], tr["final_probability_error_q15"] = fin
    tr["optimizer_step"] = state.step
    return tr, model, state
