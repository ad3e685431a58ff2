"""Pins the oracle's training-step restatement to the reference's own tests.

Known-answer tests from crates/nsrl-core (linear / mlp / rms_norm backward)
and the structural claims of the reference's map-reduce tests in
crates/nsrl-train/src/lib.rs, run on the restated initial model.
"""
import numpy as np
import pytest

from oracle import oracle as O

from train_models import (TEXT, random_model, random_windows, reference_initial_model, window_starts,
                          windows_from_text)

I16MAX = 32767


def test_linear_backward_input_transposes_weight_matrix():  # linear.rs:890-922
    lin = O.Linear(np.array([[2, -1], [3, 4], [-2, 5]], np.int8), O.scales(1, 0, 3))
    dx = O.linear_backward_input(np.array([[100, -50, 25]], np.int16), lin)
    assert list(dx[0]) == [0, -175]


def test_linear_backward_input_applies_forward_and_input_scales():  # linear.rs:925-969
    lin = O.Linear(np.array([[2, 2], [2, 2]], np.int8), O.scales([1, 1], [1, 0]))
    dx = O.linear_backward_input(np.array([[100, 100]], np.int16), lin, O.scales([1, 1], [1, 0]))
    assert list(dx[0]) == [150, 300]


def test_linear_backward_input_rejects_negative_multiplier():  # linear.rs:607-612
    lin = O.Linear(np.array([[1]], np.int8), O.scales(1, 0, 1))
    assert O.linear_backward_input(np.array([[1]], np.int16), lin, O.scales(-1, 0, 1)) is None


def test_gated_activation_backward_applies_product_rule():  # mlp.rs:810-826
    assert O.gated_activation_backward(16384, 0, 16384) == (0, 4096)
    up, gate = O.gated_activation_backward(16384, 16384, 16384)
    assert up > 0 and gate > 4096


def test_gated_mlp_backward_chains_down_gate_and_input_transposes():  # mlp.rs:846-904
    up_w = np.array([[1, 0], [0, 1], [1, 1], [-1, 1]], np.int8)
    down_w = np.array([[1, 0, 1, -1], [0, 1, 1, 1]], np.int8)
    s4, s2 = O.scales(1, 0, 4), O.scales(1, 0, 2)
    up, gate, down = O.Linear(up_w, s4), O.Linear(up_w, s4), O.Linear(down_w, s2)
    x = np.array([[1000, -500]], np.int16)
    fu = O.linear(x, up)
    fg = O.linear(x, gate)
    g = np.array([[100, -50]], np.int16)
    assert list(O.linear_backward_input(g, down)[0]) == [100, -50, 50, -150]  # grad_gated
    gu, gg, gi, sat = O.gated_mlp_backward_input(g, up, gate, down, fu, fg)
    assert sat == 0
    assert gu.any() and gg.any() and gi.any()


def test_rms_norm_backward_constant_direction_cancels_cross_channel_term():  # rms_norm.rs:258-285
    gi, gw, sat = O.rms_norm_backward_rows(np.full(4, 1000), np.full(4, 16384), np.full(4, I16MAX), 0)
    assert sat == 0
    assert (np.abs(gi) <= 1).all()
    assert (gw > 32700).all()


def test_rms_norm_backward_matches_precomputed_reference():  # rms_norm.rs:287-330
    gi, gw, _ = O.rms_norm_backward_rows(np.array([300, -700, 1100, 500]), np.array([30000, 27000, 32000, 24000]),
                                         np.array([12000, -8000, 5000, 16000]), 1)
    for a, e in zip(gi[0], [13, -3, -10, 12]):
        assert abs(int(a) - e) <= 1
    for a, e in zip(gw, [5041, 7842, 0, 11202]):
        assert abs(int(a) - e) <= 1


def test_rms_norm_backward_handles_extremes():  # rms_norm.rs:332-380
    assert O.rms_norm_backward_rows(np.array([-32768, 32767]), np.full(2, I16MAX), np.array([I16MAX, -32768]), 1)


def test_attention_probabilities_rows_sum_to_one_and_are_causal():
    rng = np.random.default_rng(3)
    B, S, d, H = 2, 12, 32, 2
    q = rng.integers(-3000, 3000, (B * S, d)).astype(np.int16)
    k = rng.integers(-3000, 3000, (B * S, d)).astype(np.int16)
    P = O.attention_probabilities(q, k, B, S, d, H)
    assert (np.triu(P, 1) == 0).all()
    s = P.astype(np.int64).sum(-1)
    assert (np.abs(s - 32768) <= S).all()


def test_reference_window_starts():  # lib.rs:13317-13358 on the map-reduce test's text
    assert window_starts(len(TEXT), 4, 1, 4) == [0, 26, 53, 79]


def test_stacked_map_reduce_accumulates_lower_layers_and_embeddings():  # lib.rs:22832-22925
    m = reference_initial_model(seq_len=4, layers=2)
    ctx, tgt = windows_from_text(TEXT, 4, window_starts(len(TEXT), 4, 1, 4)[:2])
    acc, counts, stats = O.train_windows(m, ctx, tgt)
    lay = m.arena_layout()
    assert stats["accepted"] == 2
    assert counts[-1] > 0  # embedding sample count
    o, n = lay[(0, "down")]
    assert acc[o:o + n].any()
    o, n = lay[(0, "o")]
    assert acc[o:o + n].any()


def test_map_reduce_multi_worker_matches_single_worker():  # lib.rs:22927-23000
    m = random_model(32, 2, 64, 2, 8, seed=4)
    ctx, tgt = random_windows(5, 8, seed=4)
    one = O.train_windows(m, ctx, tgt, workers=1)
    three = O.train_windows(m, ctx, tgt, workers=3)
    assert one is not None and three is not None
    assert np.array_equal(one[0], three[0]) and np.array_equal(one[1], three[1]) and one[2] == three[2]


def test_sample_counts_follow_reference_rules():
    """Head and embeddings count windows, q/k/v/o and RMS count tokens, the MLP
    counts rows with a nonzero output gradient (lib.rs:13828-13831)."""
    L, S, W = 2, 6, 3
    m = random_model(32, 2, 64, L, S, seed=5)
    ctx, tgt = random_windows(W, S, seed=5)
    _, counts, _ = O.train_windows(m, ctx, tgt)
    assert counts[0] == W and counts[-1] == W
    for li in range(L):
        c = counts[1 + 9 * li:1 + 9 * li + 9]
        assert list(c[:4]) == [W * S] * 4 and list(c[7:9]) == [W * S] * 2
        assert c[4] == c[5] == c[6] and 0 < c[4] <= W * S
    top = counts[1 + 9 * (L - 1) + 4]
    assert top == W  # only the last position carries a gradient into the top block's MLP


@pytest.mark.parametrize("rms,pos", [(True, True), (False, False)])
def test_block_forward_cache_matches_prenorm_blocks(rms, pos):
    """The cached training forward equals the forward blocks (attention.rs:1495-1583, mlp.rs:519-594)."""
    S, d, H, F = 8, 32, 2, 64
    m = random_model(d, H, F, 1, S, rms=rms, positions=pos, seed=6)
    x = np.clip(np.random.default_rng(6).normal(0, 4096, (S, d)), -32768, 32767).astype(np.int16)
    out, P, _ = O.train_block_forward(m, 0, x)
    ly = m.layers[0]
    if rms:
        y1, _ = O.prenorm_attention_block(x, 1, S, d, H, ly["attn_gamma"], 1, ly["q"], ly["k"], ly["v"], ly["o"])
        y2, _ = O.prenorm_mlp_block(y1, S, d, F, ly["mlp_gamma"], 1, ly["up"], ly["gate"], ly["down"])
        assert np.array_equal(out, y2)


def test_integer_adam_zero_gradient_keeps_weights_and_advances_state():  # nsrl-train-core lib.rs:1950-1977
    w = np.array([7, -9], np.int8)
    s = O.AdamState(2)
    st = O.integer_adam(np.zeros(2, np.int64), 1, w, O.AdamConfig(), s)
    assert list(w) == [7, -9] and s.step == 1 and not s.first.any() and not s.second.any()
    assert st[1] == 2 and st[2] == 0


def test_integer_adam_constant_gradient_moves_in_descent_direction():  # lib.rs:1980-2016
    w = np.array([10, -10], np.int8)
    s = O.AdamState(2)
    for _ in range(4):
        assert O.integer_adam(np.array([1024, -1024]), 1, w, O.AdamConfig(step_shift=0), s) is not None
    assert w[0] < 10 and w[1] > -10 and s.step == 4
    assert s.first[0] > 0 and s.first[1] < 0 and (s.second > 0).all()


def test_integer_adam_carries_sub_i8_updates():  # lib.rs:2018-2057
    w = np.array([10], np.int8)
    s = O.AdamState(1)
    st = O.integer_adam(np.array([4096]), 1, w, O.AdamConfig(step_shift=4), s)
    assert list(w) == [10] and st[1] == 1 and s.residuals[0] != 0
    for _ in range(20):
        O.integer_adam(np.array([4096]), 1, w, O.AdamConfig(step_shift=4), s)
    assert w[0] < 10


def test_integer_adam_reports_gradient_and_weight_saturation():  # lib.rs:2059-2089
    w = np.array([-128], np.int8)
    s = O.AdamState(1)
    st = O.integer_adam(np.array([2**63 - 1]), 1, w, O.AdamConfig(step_shift=0), s)
    assert list(w) == [-128] and st[0] >= 2 and s.residuals[0] == 0


def test_integer_adam_i16_path_is_deterministic():  # lib.rs:2091-2120
    def run():
        w = np.array([100, -100, 0], np.int16)
        s = O.AdamState(3)
        for _ in range(12):
            O.integer_adam(np.array([500, -750, 125]), 2, w, O.AdamConfig(), s)
        return w.copy(), s.first.copy(), s.second.copy()
    a, b = run(), run()
    assert all(np.array_equal(x, y) for x, y in zip(a, b))


def test_integer_adam_rejects_invalid_config():  # lib.rs:299-309
    w = np.zeros(1, np.int8)
    assert O.integer_adam(np.zeros(1), 1, w, O.AdamConfig(beta1_decay_shift=0), O.AdamState(1)) is None
    assert O.integer_adam(np.zeros(1), 1, w, O.AdamConfig(step_shift=48), O.AdamState(1)) is None
