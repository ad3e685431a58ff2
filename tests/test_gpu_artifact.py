"""Models loaded from .nsrlmt artifacts run on the GPU exactly as the oracle
runs them: a synthetic artifact written and read back, and (when present,
for instance through NSRL_REFERENCE_ARTIFACT) the reference's checked-in
candidate model, a two-layer linear-attention model without positions under
the calibrated scale profile."""
import os

import numpy as np
import pytest
import torch

from nsrl_b200 import artifact as A
from oracle import oracle as O

from test_artifact import REF_ARTIFACT, synthetic

pytestmark = pytest.mark.gpu


def oracle_model(a, profile, kind, use_positions):
    sd, sf, so = A.PROFILES[profile]
    layers = []
    for li in range(a.layers):
        e = {}
        for nm, shift, n in (("q", sd, a.d_model), ("k", sd, a.d_model), ("v", sd, a.d_model), ("o", sd, a.d_model),
                             ("up", sf, a.hidden_dim), ("gate", sf, a.hidden_dim), ("down", sd, a.d_model)):
            e[nm] = O.Linear(getattr(a, nm)[li].copy(), O.scales(1, shift, n))
        if a.attention_rms is not None:
            e["attn_gamma"], e["mlp_gamma"] = a.attention_rms[li].copy(), a.mlp_rms[li].copy()
        layers.append(e)
    pos = a.positions.copy() if use_positions and a.positions.size else None
    return O.TrainModel(a.embeddings.copy(), pos, layers, O.Linear(a.output.copy(), O.scales(1, so, 256)),
                        a.d_model, a.heads, a.hidden_dim, a.seq_len, attention_kind=kind)


def _rows_match(a, profile, kind, use_positions, windows):
    from nsrl_b200 import build, generate as G
    build.build()
    gm = A.to_train_model(a, profile, kind, use_positions)
    om = oracle_model(a, profile, kind, use_positions)
    ref = O.output_rows(om, windows, threads=8)
    got = G.output_rows(gm, torch.from_numpy(windows))
    assert (ref is None) == (got is None)  # a rejection (the reference's None) on both sides, or neither
    if ref is not None:
        assert np.array_equal(got[0].cpu().numpy(), ref[0]) and np.array_equal(got[1].cpu().numpy(), ref[1])
    return ref is not None


@pytest.mark.parametrize("kind,profile,pos,live_qk,accepted", [
    ("softmax", "default", True, False, False),  # random full-range q, k: the logits leave i32, rejected on both sides
    ("softmax", "calibrated", True, True, True),
    ("linear", "calibrated", False, False, True)])
def test_synthetic_artifact_runs_like_the_oracle(kind, profile, pos, live_qk, accepted):
    a = A.from_bytes(A.to_bytes(synthetic(d=64, H=4, F=128, S=16, L=2, seed=5)))
    a.output = (a.output // 8).astype(np.int8)  # a live byte softmax
    if live_qk:  # ternary q, k and small RMS gammas keep the attention logits inside i32
        r = np.random.default_rng(9)
        a.q = r.integers(-1, 2, a.q.shape).astype(np.int8)
        a.k = r.integers(-1, 2, a.k.shape).astype(np.int8)
        a.attention_rms[...] = 256
        a.mlp_rms[...] = 256
    win = np.random.default_rng(1).integers(0, 256, (8, 16)).astype(np.uint8)
    assert _rows_match(a, profile, kind, pos, win) == accepted


@pytest.mark.skipif(not os.path.exists(REF_ARTIFACT), reason="the reference's candidate artifact is not present")
def test_reference_candidate_model_runs_like_the_oracle():
    a = A.load(REF_ARTIFACT)
    win = np.random.default_rng(2).integers(32, 127, (24, a.seq_len)).astype(np.uint8)
    assert _rows_match(a, "calibrated", "linear", False, win)
