"""The integer-Adam training loop of the mini transformer around the
data-parallel step.

Mirrors run_mini_transformer_mlp_integer_adam_training_from_model_with_scope
(crates/nsrl-train/src/lib.rs:4499-4800) for base-2 softmax attention: the
windows of a token stream (:13291-13358), epochs of batches of
`batch_windows` windows, each batch run through nsrl_train_dp_step with
integer Adam as its optimizer, the updated model checked on the batch's
windows and on guard windows (:14617-14700) and, optionally, against a loss
regression over guard windows (:13538-13581); a batch that fails is rolled
back, as the reference discards its candidate model.  The evaluation counts
(mistakes, probability error) come from the byte-head rows of every window
(:17510-17660, :18539-18548).  With several ranks, rank r runs chunk r of
every batch's windows, as worker r of the reference's map-reduce batch does
(:6970-7050); every rank keeps the same model.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch

from . import core
from . import generate as G
from . import train as T


@dataclasses.dataclass(frozen=True)
class LoopConfig:
    """The loop fields of MiniTransformerMlpTrainConfig (lib.rs:300-390,
    defaults :81-105); seq_len is the model's."""
    epochs: int = 1
    stride: int = 1
    window_offset: int = 0
    max_windows: Optional[int] = 64
    batch_windows: int = 1
    reject_loss_regression: bool = False


def byte_window_starts(token_count, seq_len, stride, window_offset, max_windows):
    """lib.rs:13291-13315."""
    out = []
    if seq_len == 0 or stride == 0:
        return out
    s = window_offset
    while s + seq_len < token_count:
        if max_windows is not None and len(out) >= max_windows:
            break
        out.append(s)
        s += stride
    return out


def window_starts(token_count, seq_len, stride, window_offset, max_windows):
    """mini_transformer_window_starts (lib.rs:13317-13358): every stride-th
    start, or `max_windows` of them spread evenly over the stream."""
    if seq_len == 0 or stride == 0 or window_offset >= token_count or token_count < seq_len + 1:
        return []
    last = token_count - seq_len - 1
    if window_offset > last:
        return []
    available = (last - window_offset) // stride + 1
    limit = available if max_windows is None else min(max_windows, available)
    if limit == 0:
        return []
    if limit >= available:
        return byte_window_starts(token_count, seq_len, stride, window_offset, limit)
    if limit == 1:
        return [window_offset]
    num, den = available - 1, limit - 1
    return [window_offset + ((i * num + den // 2) // den) * stride for i in range(limit)]


def guard_indices(n, epoch, window_index, epochs):
    """The window indices mini_transformer_validate_guard_windows checks (lib.rs:14617-14669)."""
    cand = [0, n // 4, n // 2, (n * 3) // 4, n - 1, max(window_index - 1, 0), window_index,
            min(window_index + 1, n - 1),
            window_index + 1 if window_index + 1 < n else (0 if epoch + 1 < epochs else window_index)]
    out = []
    for i in cand:
        if i < n and i not in out:
            out.append(i)
    return out


def loss_guard_starts(starts, b0, b1):
    """mini_transformer_loss_guard_starts (lib.rs:13538-13572)."""
    out = []
    if not starts:
        return out
    end = min(b1, len(starts))
    for s in starts[min(b0, end):end]:
        if s not in out:
            out.append(s)
    n = len(starts)
    points = min(16, n)
    if points == 1:
        if starts[0] not in out:
            out.append(starts[0])
        return out
    num, den = n - 1, points - 1
    for p in range(points):
        s = starts[(p * num + den // 2) // den]
        if s not in out:
            out.append(s)
    return out


def probability_error_q15(probs: np.ndarray, target: int) -> int:
    """byte_sample_probability_error_q15 (lib.rs:18539-18548) for one row."""
    p = probs.astype(np.int64)
    return int(max(32767 - p[target], 0) + np.maximum(np.delete(p, target), 0).sum())


class Evaluator:
    """Byte-head rows of windows of a token stream, in device batches."""

    def __init__(self, model: T.TrainModel, tokens: np.ndarray, chunk: int = 256):
        self.model, self.tokens, self.chunk = model, tokens, chunk
        self.S = model.seq_len

    def rows(self, starts):
        """(logits [n, 256], probs [n, 256]) host arrays, or None if any window is rejected."""
        lg, pr = [], []
        for c0 in range(0, len(starts), self.chunk):
            part = starts[c0:c0 + self.chunk]
            win = np.stack([self.tokens[s:s + self.S] for s in part])
            r = G.output_rows(self.model, torch.from_numpy(win))
            if r is None:
                return None
            lg.append(r[0].cpu().numpy())
            pr.append(r[1].cpu().numpy())
        return np.concatenate(lg), np.concatenate(pr)

    def counts(self, starts):
        """(mistakes, probability error) over the windows (lib.rs:17590-17660), or None."""
        r = self.rows(starts)
        if r is None:
            return None
        mistakes, err = 0, 0
        for i, s in enumerate(starts):
            tgt = int(self.tokens[s + self.S])
            lg = r[0][i]
            mistakes += int(int(np.argmax(lg)) != tgt)  # argmax takes the lowest index among equal logits
            err += probability_error_q15(r[1][i], tgt)
        return mistakes, err


def _snapshot(model: T.TrainModel, state: T.TrainState):
    ts = [model.head.weights, model.embeddings]
    if model.positions is not None:
        ts.append(model.positions)
    for ly in model.layers:
        ts += [ly[n].weights for n in T.LAYER_LINEARS]
        ts += [ly[g] for g in ("attn_gamma", "mlp_gamma") if ly.get(g) is not None]
    a = state.adam
    ts += [state.residuals, a.first_moments, a.second_moments, a.update_residuals, a.step]
    return [(t, t.clone()) for t in ts]


def _restore(snap):
    for t, c in snap:
        t.copy_(c)


def run_integer_adam_training(tokens: bytes, model: T.TrainModel, cfg: LoopConfig, adam=(1, 4, 3, 7, 1),
                              scope: str = "all", state: Optional[T.TrainState] = None, comm=None) -> dict:
    """The integer-Adam training run (lib.rs:4499-4800) on `model` in place;
    `state` (TrainState with adam=True) resumes a previous run.  Returns the
    trace's counters."""
    import torch.distributed as dist
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    if comm is None:
        comm = T.default_communicator()
    tok = np.frombuffer(bytes(tokens), np.uint8)
    S = model.seq_len
    if cfg.epochs == 0 or cfg.stride == 0 or cfg.batch_windows == 0:
        raise ValueError("invalid config")
    starts = window_starts(len(tok), S, cfg.stride, cfg.window_offset, cfg.max_windows)
    if not starts:
        raise ValueError("invalid config: no windows")
    if state is None:
        state = T.TrainState(model, adam=True)
    step_cfg = T.MiniTransformerTrainConfig(optimizer="integer_adam", adam=tuple(adam), adam_scope=scope)
    ev = Evaluator(model, tok)
    init = ev.counts(starts)
    if init is None:
        raise core.NsrlError("the initial model rejects a window")
    per = -(-cfg.batch_windows // world)
    buf = T.TrainStepBuffers(model, per, nranks=world)
    tr = {"windows": len(starts), "examined_windows": 0, "updates": 0, "accepted_batch_count": 0,
          "rejected_batch_count": 0, "initial_mistakes": init[0], "initial_probability_error_q15": init[1],
          "weight_delta_l1": 0, "mlp_saturation_count": 0, "attention_saturation_count": 0,
          "residual_saturation_count": 0}
    for epoch in range(cfg.epochs):
        b0 = 0
        while b0 < len(starts):
            b1 = min(b0 + cfg.batch_windows, len(starts))
            tr["examined_windows"] += b1 - b0
            batch = starts[b0:b1]
            chunk = -(-len(batch) // world)
            mine = batch[rank * chunk:(rank + 1) * chunk]
            ctx = torch.from_numpy(np.stack([tok[s:s + S] for s in mine]))
            tgt = torch.from_numpy(np.array([tok[s + S] for s in mine], np.uint8))
            snap = _snapshot(model, state)
            out = T.mini_transformer_train_step(model, state, ctx, tgt, step_cfg, buf, comm=comm)
            if out is None or out["accepted"] == 0:
                tr["rejected_batch_count"] += 1
                b0 = b1
                continue
            for k in ("mlp_saturation_count", "attention_saturation_count", "residual_saturation_count"):
                tr[k] += out[k]
            valid = ev.rows(batch) is not None
            if valid:
                g = [starts[i] for i in guard_indices(len(starts), epoch, b1 - 1, cfg.epochs)]
                valid = ev.rows(g) is not None
            regressed = False
            if valid and cfg.reject_loss_regression:
                guard = loss_guard_starts(starts, b0, b1)
                after = ev.counts(guard)                     # the candidate model
                candidate = [(t, t.clone()) for t, _ in snap]
                _restore(snap)
                before = ev.counts(guard)                    # the model before the batch
                _restore(candidate)
                if before is None:
                    raise core.NsrlError("the loss guard rejects a window of the current model")
                # mini_transformer_loss_guard_regressed: 1024 of Q15 error per guard window tolerated
                regressed = after is None or after[1] > before[1] + len(guard) * 1024
            if valid and not regressed:
                tr["updates"] += out["accepted"]
                tr["accepted_batch_count"] += 1
                tr["weight_delta_l1"] += out["weight_delta_l1"]
            else:
                _restore(snap)
                tr["rejected_batch_count"] += 1
            b0 = b1
    fin = ev.counts(starts)
    tr["final_mistakes"], tr["final_probability_error_q15"] = fin if fin else (None, None)
    tr["optimizer_step"] = int(state.adam.step.item())
    tr["state"] = state
    return tr
