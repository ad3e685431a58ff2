"""The oracle's linear attention pinned to the reference's own known-answer
tests (crates/nsrl-core/src/attention.rs:2190-2512), no GPU."""
import ctypes as C

import numpy as np

from oracle import oracle as O


def _ident(n):
    return O.Linear(np.eye(n, dtype=np.int8), O.scales(1, 0, n))


def _lin4():
    return [_ident(4)] * 4


def test_identity_single_token_round_trips():  # attention.rs:2190-2220
    x = np.array([[100, -200, 300, -400]], np.int16)
    assert np.array_equal(O.linear_attention(x, 1, 1, 4, 1, *_lin4()), x)


def test_causal_prefix_blocks_future_value():  # attention.rs:2223-2256
    x = np.array([[100, 0, 0, 0], [0, 1000, 0, 0]], np.int16)
    out = O.linear_attention(x, 1, 2, 4, 1, *_lin4())
    assert np.array_equal(out[0], x[0]) and not np.array_equal(out[1], x[0])


def test_incremental_matches_full_causal():  # attention.rs:2257-2334
    x = np.array([[100, -200, 300, -400], [250, 100, -50, 75], [-125, 225, 325, -425]], np.int16)
    full = O.linear_attention(x, 1, 3, 4, 1, *_lin4())
    st = np.zeros((1, 16), np.int64)
    ks = np.zeros((1, 4), np.int64)
    rows = [O.linear_attention_step(x[t:t + 1], 1, *_lin4(), st, ks) for t in range(3)]
    assert np.array_equal(np.concatenate(rows), full)


def test_ttt_delta_teaches_state_current_value():  # attention.rs:2335-2372
    k = np.array([100, -50], np.int16)
    v = np.array([4000, -2000], np.int16)
    S = np.zeros(4, np.int64)
    ks = (k.astype(np.int64) + 32769)
    pred = np.full(2, 999, np.int16)
    dl = C.c_uint64()
    L = O.lib()
    p = lambda a: C.c_void_p(a.ctypes.data)
    assert L.orc_linear_attention_ttt_delta(p(k), p(v), p(S), p(ks), C.c_size_t(2), C.c_uint8(0), p(pred),
                                            C.byref(dl)) == 0
    assert pred.tolist() == [0, 0] and dl.value > 0
    upd = np.zeros(2, np.int16)
    assert L.orc_linear_attention_project(p(k), p(S), p(ks), C.c_size_t(2), p(upd)) == 0
    assert np.array_equal(upd, v)


def test_ttt_step_mutates_state_before_projection():  # attention.rs:2398-2480
    x = np.array([[100, 0, 0, 0], [0, 1000, 0, 0]], np.int16)
    st_n, ks_n = np.zeros((1, 16), np.int64), np.zeros((1, 4), np.int64)
    st_t, ks_t = np.zeros((1, 16), np.int64), np.zeros((1, 4), np.int64)
    dl = np.zeros(1, np.uint64)
    normal = [O.linear_attention_step(x[t:t + 1], 1, *_lin4(), st_n, ks_n) for t in range(2)]
    ttt = [O.linear_attention_step(x[t:t + 1], 1, *_lin4(), st_t, ks_t, ttt_shift=0, delta_l1=dl) for t in range(2)]
    assert int(dl[0]) > 0
    assert not np.array_equal(st_t, st_n)
    assert not np.array_equal(ttt[1], normal[1])


def test_non_power_of_four_head_dim():  # attention.rs:2481-2512
    x = np.array([[321, -123]], np.int16)
    assert np.array_equal(O.linear_attention(x, 1, 1, 2, 1, *[_ident(2)] * 4), x)
