"""Pins the CPU oracle to the reference's own known-answer tests.

Each test restates one of the reference's inline `#[cfg(test)]` cases
(file:line given per test) against the oracle, plus the published bench-1m
output hash (ENG.md:790-799) and the LUT fixtures in tests/golden/.
"""
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
I16MIN, I16MAX = -32768, 32767
MASKED = -(2**31)


def fnv(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def test_luts_match_reference_tables():
    """The tables derived from their definitions equal rsqrt_lut_8bit.rs byte for byte."""
    g = json.load(open(os.path.join(GOLDEN, "reference_luts.json")))
    r, e, c = O.luts()
    for name, vals, fmt in (("RSQRT_LUT_8BIT", r, "<h"), ("EXP2_NEG_FRAC_LUT_8BIT", e, "<h"),
                            ("RECIP_LUT_8BIT_Q31", c, "<I")):
        data = b"".join(struct.pack(fmt, int(v)) for v in vals)
        assert len(vals) == g[name]["len"]
        assert "0x%016x" % fnv(data) == g[name]["fnv1a64"], name
        assert int(vals[0]) == g[name]["first"] and int(vals[-1]) == g[name]["last"]


def test_product_luts_match_oracle():
    """The CUDA side's generated header holds the same three tables."""
    from nsrl_b200.csrc import gen_luts
    r, e, c = O.luts()
    assert gen_luts.rsqrt_table() == [int(v) for v in r]
    assert gen_luts.exp2_table() == [int(v) for v in e]
    assert gen_luts.recip_table() == [int(v) for v in c]


def test_bench_1m_output_hash():
    """ENG.md:790-799: bench-1m output_hash 0xf7dd983b8ce7a156, 0 saturations."""
    r = O.bench1m()
    assert r is not None
    assert r["output_hash"] == 0xF7DD983B8CE7A156
    assert r["saturations"] == 0


def test_round_shift_rhu():  # numeric.rs:244-251
    assert O.rhu(3, 1) == 2
    assert O.rhu(5, 1) == 3
    assert O.rhu(-3, 1) == -1
    assert O.rhu(-5, 1) == -2
    assert O.rhu(123, 0) == 123


def test_requantize_saturates():  # numeric.rs:253-262
    assert O.requantize_i32_to_i16(100, 1000, 0) == I16MAX
    assert O.requantize_i32_to_i16(-100, 1000, 0) == I16MIN


def test_residual_add_counts():  # numeric.rs:264-279
    out, sat = O.residual_add([32000, -32000, 100], [1000, -1000, -25])
    assert list(out) == [I16MAX, I16MIN, 75]
    assert sat == 2


def test_normalize():  # lut.rs:375-395
    cases = [(1, 128, -7), (2, 128, -6), (127, 254, -1), (128, 128, 0), (255, 255, 0), (256, 128, 1),
             (2**64 - 1, 255, 56)]
    for v, m, e in cases:
        assert O.normalize_u64(v) == (m, e)
    assert O.normalize_u64(0) is None


def test_linear_identity():  # linear.rs:759-775
    w = np.eye(4, dtype=np.int8)
    lin = O.Linear(w, O.scales(1, 0, 4))
    y = O.linear(np.array([[100, -200, 300, -400]], np.int16), lin)
    assert list(y[0]) == [100, -200, 300, -400]


def test_linear_bias_and_scale():  # linear.rs:777-803
    lin = O.Linear(np.array([[2, -1], [2, -1]], np.int8), O.scales([1, 1], [0, 1]), bias=[10, 10])
    y = O.linear(np.array([[100, -50]], np.int16), lin)
    assert list(y[0]) == [260, 130]


def test_linear_rejects_accumulator_overflow():  # linear.rs:866-883
    lin = O.Linear(np.full((1, 600), 127, np.int8), O.scales(1, 0, 1), bias=[2**31 - 1])
    assert O.linear(np.full((1, 600), I16MAX, np.int16), lin) is None


def test_linear_i32_bound():  # linear.rs:1038-1054: 516 products fit, 517 do not
    assert 516 * 127 * 32767 <= 2**31 - 1 < 517 * 127 * 32767


def test_qk_dot_shift_and_softmax_kats():  # attention.rs:1830-1875
    out = O.attention_row(np.full(64, 8, np.int16), np.full(64, 8, np.int16), np.array([5], np.int16), 64, 1)
    assert out[1][0] == 512
    assert O.base2_exp_neg_q15(0) == I16MAX
    assert O.base2_exp_neg_q15(-(1 << 8)) == 16383
    assert O.base2_exp_neg_q15(-64) < I16MAX
    assert O.base2_exp_neg_q15(-64) > O.base2_exp_neg_q15(-128)
    assert O.base2_exp_neg_q15(-(15 << 8)) == 0
    assert O.reciprocal_sum_q31(1) == 1 << 31
    assert O.reciprocal_sum_q31(2) == 1 << 30
    assert O.reciprocal_sum_q31(128) == 1 << 24
    assert O.reciprocal_sum_q31(0) is None


def test_softmax_masking():  # attention.rs:1892-1910
    p, _ = O.base2_softmax_i32_q15([0, MASKED, 0])
    assert p[0] > 16000 and p[1] == 0 and p[2] > 16000 and abs(int(p[0]) - int(p[2])) <= 1
    assert O.base2_softmax_i32_q15([MASKED, MASKED]) is None


def test_attention_row_mask():  # attention.rs:2100-2130
    keys = np.full(128, 8, np.int16)
    vals = np.array([100, -100, 30000, 30000], np.int16)
    out, logits, probs, _ = O.attention_row(np.full(64, 8, np.int16), keys, vals, 64, 2, mask=[0, 1])
    assert logits[1] == MASKED and probs[1] == 0
    assert list(out) == [100, -100]
    assert O.attention_row(np.ones(64, np.int16), np.ones(64, np.int16), np.ones(2, np.int16), 64, 2,
                           mask=[1]) is None


def test_self_attention_causal_mask():  # attention.rs:2549-2581
    ident = O.Linear(np.eye(4, dtype=np.int8), O.scales(1, 0, 4))
    x = np.array([100, 0, 0, 0, 0, 1000, 0, 0], np.int16)
    y = O.self_attention(x, 1, 2, 4, 1, ident, ident, ident, ident)
    assert list(y[0]) == [100, 0, 0, 0]


def test_self_attention_rejects_non_power_of_four():  # attention.rs:2582-2625
    lin = O.Linear(np.ones((2, 2), np.int8), O.scales(1, 0, 2))
    assert O.self_attention(np.array([1, 2], np.int16), 1, 1, 2, 1, lin, lin, lin, lin, causal=False) is None
    # head_dim 32 (d 128, 4 heads) is rejected too
    lin = O.Linear(np.ones((128, 128), np.int8), O.scales(1, 10, 128))
    assert O.self_attention(np.ones(128, np.int16), 1, 1, 128, 4, lin, lin, lin, lin) is None


def test_hard_silu_gate_values():  # mlp.rs:777-806
    # gate(x) = clamp((x >> 2) + 16384, 0, 32767): 8192 / 16384 / 24575 at min / 0 / max
    assert O.gated_activation(10000, 0) == 0
    assert O.gated_activation(10000, 20000) > 0
    assert O.gated_activation(10000, -20000) < 0


def test_integer_rsqrt():  # rms_norm.rs:200-210
    one, four, sixteen = O.integer_rsqrt_q30(1), O.integer_rsqrt_q30(4), O.integer_rsqrt_q30(16)
    assert abs((1 << 30) - one) < 40000
    assert abs((1 << 29) - four) < 20000
    assert abs((1 << 28) - sixteen) < 10000
    assert O.integer_rsqrt_q30(0) is None


def test_rms_norm_kats():  # rms_norm.rs:212-256
    y = O.rms_norm_rows(np.full(4, 1000, np.int16), np.full(4, I16MAX, np.int16), 0)
    assert (y > 32700).all()
    y = O.rms_norm_rows(np.full(4, -1000, np.int16), np.full(4, I16MAX, np.int16), 0)
    assert (y < -32700).all()
    y = O.rms_norm_rows(np.zeros(4, np.int16), np.full(4, I16MAX, np.int16), 1)
    assert (y == 0).all()
    assert O.rms_norm_rows(np.zeros(4, np.int16), np.full(4, I16MAX, np.int16), 0) is None


@pytest.mark.parametrize("threads", [1, 3])
def test_oracle_batched_block_is_per_sequence(threads):
    """Batched block == the same block run one sequence at a time (the reference's caller loop)."""
    rng = np.random.default_rng(5)
    B, S, d, H = 3, 16, 64, 4
    lins = [O.Linear(rng.integers(-127, 128, (d, d)).astype(np.int8), O.scales(1, 10, d)) for _ in range(4)]
    x = np.clip(rng.normal(0, 4096, (B * S, d)), I16MIN, I16MAX).astype(np.int16)
    g = np.full(d, 16384, np.int16)
    y, sat = O.prenorm_attention_block(x, B, S, d, H, g, 1, *lins, threads=threads)
    parts = [O.prenorm_attention_block(x[b * S:(b + 1) * S], 1, S, d, H, g, 1, *lins)[0] for b in range(B)]
    assert np.array_equal(y, np.concatenate(parts))


def test_i64_gradient_average_then_update():  # crates/nsrl-train-core/src/lib.rs:1896-1927
    acc = np.zeros((2, 2), np.int64)
    x = np.array([[4096, 8192]], np.int16)
    g = np.array([[1024, 2048]], np.int32)
    acc, c = O.accumulate_linear_gradient_i64(x, g, acc, 0)
    acc, c = O.accumulate_linear_gradient_i64(x, g, acc, c)
    assert c == 2
    acc2, res, w, c2, st = O.apply_linear_gradient_i64_to_i8(acc, np.zeros(4), np.full(4, 10), c, 1, 22, False)
    assert list(w) == [9, 8, 8, 6]
    assert st == [0, 0, 9]
    assert c2 == 0 and not acc2.any()


def test_i64_gradient_carries_residuals():  # crates/nsrl-train-core/src/lib.rs:1929-1966
    acc, c = O.accumulate_linear_gradient_i64(np.array([[1]], np.int16), np.array([[1]], np.int32),
                                              np.zeros((1, 1), np.int64), 0)
    acc, res, w, c, st = O.apply_linear_gradient_i64_to_i8(acc, [0], [10], c, 1, 2, True)
    assert list(w) == [10] and st[1] == 1 and st[2] == 0 and list(res) == [1]
    acc, c = O.accumulate_linear_gradient_i64(np.array([[1]], np.int16), np.array([[1]], np.int32),
                                              acc.reshape(1, 1), c)
    acc, res, w, c, st = O.apply_linear_gradient_i64_to_i8(acc, res, w, c, 1, 2, True)
    assert list(w) == [9] and st[1] == 0 and st[2] == 1 and list(res) == [-2]


def test_ordered_merge_rejects_prefix_overflow():
    big = 2**62
    parts = np.array([[big], [big], [-big]], np.int64)
    assert O.merge_i64(parts, [1, 1, 1]) is None  # big + big overflows before the third worker
    out, c = O.merge_i64(np.array([[big], [-big], [big]], np.int64), [1, 2, 3])
    assert out[0] == big and c == 6
