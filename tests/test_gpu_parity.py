"""Parity of the CUDA path (through the C ABI) with the CPU oracle: bit-exact.

Every test compares libnsrl_b200 against oracle/ on the same seeded inputs,
including the cases where the reference returns `None`.
"""
import numpy as np
import pytest

from nsrl_b200 import synth as Y
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def core():
    from nsrl_b200 import build, core as K
    build.build()
    return K


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def lin_pair(core, w, shifts, mult=None, bias=None):
    n = w.shape[0]
    shifts = np.broadcast_to(np.asarray(shifts), (n,)).astype(np.int64)
    mult = np.ones(n, np.int64) if mult is None else np.broadcast_to(np.asarray(mult), (n,)).astype(np.int64)
    o = O.Linear(w, O.scales(mult.astype(np.int32), shifts.astype(np.uint8)), bias=bias)
    g = core.Linear(dev(w), core.make_scales(torch.from_numpy(mult), torch.from_numpy(shifts)),
                    None if bias is None else dev(np.asarray(bias, np.int32)))
    return o, g


# ----------------------------------------------------------------- linear ---
@pytest.mark.parametrize("M,K,N,with_bias", [
    (256, 256, 256, False),    # one tile row, the HBM-bound sweep shape
    (300, 128, 200, True),     # M and N tails, bias (forces the prefix check)
    (129, 1024, 384, False),   # K > 516: L1-bounded prefix check, 4-stage pipeline
    (64, 4096, 128, False),    # the deepest sweep K
    (33, 40, 17, True),        # K not a multiple of 16: SIMT path
])
def test_linear_parity(core, M, K, N, with_bias):
    x = Y.q15_gaussian(11 + K, (M, K))
    w = Y.i8_uniform(12 + N, (N, K))
    shifts = (np.arange(N) % 5) + Y.shift_for(K) - 2
    mult = (np.arange(N) % 3) + 1
    bias = (np.arange(N, dtype=np.int64) * 7919 % 200001 - 100000).astype(np.int32) if with_bias else None
    o, g = lin_pair(core, w, shifts, mult, bias)
    ref = O.linear(x, o)
    got = core.linear_i16_i8_i16_per_channel_checked(dev(x), g)
    assert ref is not None and got is not None
    assert np.array_equal(host(got), ref)


def test_linear_identity_and_saturation(core):
    """linear.rs:759-803 cases on the device, plus both saturation rails."""
    o, g = lin_pair(core, np.eye(4, dtype=np.int8), 0)
    x = np.array([[100, -200, 300, -400]], np.int16)
    assert host(core.linear_i16_i8_i16_per_channel_checked(dev(x), g)).tolist() == [[100, -200, 300, -400]]
    o, g = lin_pair(core, np.array([[2, -1], [2, -1]], np.int8), [0, 1], bias=[10, 10])
    x = np.array([[100, -50]], np.int16)
    assert host(core.linear_i16_i8_i16_per_channel_checked(dev(x), g)).tolist() == [[260, 130]]
    w = np.full((2, 64), 127, np.int8)
    w[1] = -127
    o, g = lin_pair(core, w, 0)
    x = np.full((1, 64), 30000, np.int16)
    assert host(core.linear_i16_i8_i16_per_channel_checked(dev(x), g)).tolist() == [[32767, -32768]]


@pytest.mark.parametrize("N", [1, 300])  # 300 outputs: the planes path, check fused into the GEMM
def test_linear_rejects_final_overflow(core, N):
    """linear.rs:866-883: the sum leaves i32."""
    w = np.full((N, 600), 127, np.int8)
    o, g = lin_pair(core, w, 0, bias=[2**31 - 1] * N)
    x = np.full((1, 600), 32767, np.int16)
    assert O.linear(x, o) is None
    assert core.linear_i16_i8_i16_per_channel_checked(dev(x), g) is None


@pytest.mark.parametrize("N", [3, 300])  # 300 outputs: the planes path, check fused into the GEMM
def test_linear_rejects_prefix_overflow_with_fitting_total(core, N):
    """An i32 prefix overflows although the final sum fits: still `None` (checked_add per prefix)."""
    K = 1024
    w = np.where(np.arange(K) < 600, 127, -127).astype(np.int8)[None, :].repeat(N, 0)
    w[1] = 1  # a row that never overflows
    x = np.full((2, K), 32767, np.int16)
    x[1] = 1
    o, g = lin_pair(core, w, 12)
    assert O.linear(x, o) is None
    assert core.linear_i16_i8_i16_per_channel_checked(dev(x), g) is None
    ok = x[1:]
    ref = O.linear(ok, o)
    got = core.linear_i16_i8_i16_per_channel_checked(dev(ok), g)
    assert ref is not None and np.array_equal(host(got), ref)


# --------------------------------------------------------------- rms norm ---
@pytest.mark.parametrize("rows,d,eps", [(1000, 256, 1), (1001, 256, 1), (77, 512, 3), (33, 1024, 1), (37, 100, 1),
                                        (8, 4, 0), (3, 4096, 7)])
def test_rms_norm_parity(core, rows, d, eps):
    x = Y.q15_gaussian(d + rows, (rows, d))
    x[0, :] = 0
    x[-1, :] = 32767
    g = (Y.i8_uniform(5, (d,)).astype(np.int16) * 250).astype(np.int16)
    ref = O.rms_norm_rows(x, g, eps)
    got = core.rms_norm_i16_q15_checked(dev(x), dev(g), eps)
    if ref is None:
        assert got is None
    else:
        assert np.array_equal(host(got), ref)


# -------------------------------------------------------------- attention ---
def attn_weights(core, d, seed, qk_extra=7, qk_shift=None):
    bw = Y.BlockWeights(seed, d, 4 * d, qk_extra_shift=qk_extra)
    pairs = {}
    for nm in ("q", "k", "v", "o"):
        s = bw.shift[nm] if qk_shift is None or nm not in "qk" else qk_shift
        pairs[nm] = lin_pair(core, getattr(bw, nm), s)
    return pairs


@pytest.mark.parametrize("B,S,d,H,causal,qk_extra", [
    (2, 100, 128, 2, True, 7),     # head_dim 64, ragged last query tile
    (1, 256, 256, 4, True, 0),     # near one-hot softmax (no extra shift)
    (2, 64, 128, 8, True, 7),      # head_dim 16
    (1, 77, 128, 2, False, 7),     # full (non-causal) attention
    (1, 40, 16, 4, True, 2),       # head_dim 4: row-kernel path
    (1, 24, 256, 1, True, 9),      # head_dim 256: row-kernel path
    (1, 1, 64, 1, True, 7),        # one token
    (2, 48, 128, 2, True, 7),      # tensor-core path: one partial key tile
    (1, 144, 256, 4, True, 7),     # tensor-core path: ragged query and key tiles
    (2, 128, 128, 2, False, 5),    # tensor-core path, full attention
    (1, 1024, 256, 4, True, 7),    # tensor-core path at the benchmark length
    (1, 320, 64, 1, True, 0),      # tensor-core path, peaked softmax, one head
    (2, 256, 256, 16, True, 7),    # tensor-core path at head_dim 16 (the alt 16 x 16 shape)
    (1, 144, 128, 8, False, 5),    # head_dim 16, full attention, ragged tiles
    (1, 1024, 256, 16, True, 0),   # head_dim 16 at the benchmark length, peaked softmax
])
def test_self_attention_parity(core, B, S, d, H, causal, qk_extra):
    P = attn_weights(core, d, 100 + d + H, qk_extra)
    x = Y.q15_gaussian(7 + S, (B * S, d))
    ref = O.self_attention(x, B, S, d, H, *[P[n][0] for n in "qkvo"], causal=causal, threads=4)
    got = core.self_attention_i16_q15_checked(dev(x), B, S, d, H, *[P[n][1] for n in "qkvo"], causal=causal)
    assert ref is not None and got is not None
    assert np.array_equal(host(got), ref)


def test_self_attention_rejects_head_dim_32(core):
    P = attn_weights(core, 128, 3)
    x = Y.q15_gaussian(1, (16, 128))
    assert O.self_attention(x, 1, 16, 128, 4, *[P[n][0] for n in "qkvo"]) is None
    assert core.self_attention_i16_q15_checked(dev(x), 1, 16, 128, 4, *[P[n][1] for n in "qkvo"]) is None


def test_attention_rejects_logit_overflow(core):
    """(q.k) >> 3 beyond i32 (attention.rs:139) rejects the whole call."""
    d = 64
    ident = np.eye(d, dtype=np.int8)
    pair = lin_pair(core, ident, 0)
    x = np.full((4, d), 32767, np.int16)
    args_o = [pair[0]] * 4
    args_g = [pair[1]] * 4
    assert O.self_attention(x, 1, 4, d, 1, *args_o) is None
    assert core.self_attention_i16_q15_checked(dev(x), 1, 4, d, 1, *args_g) is None


@pytest.mark.parametrize("B,S,d,H", [(2, 192, 256, 4), (1, 130, 128, 8)])
def test_prenorm_attention_block_parity(core, B, S, d, H):
    P = attn_weights(core, d, 9)
    x = Y.q15_gaussian(31, (B * S, d))
    g = np.full(d, 4096, np.int16)
    ref = O.prenorm_attention_block(x, B, S, d, H, g, 1, *[P[n][0] for n in "qkvo"], threads=4)
    got = core.prenorm_attention_residual_block_i16_q15_checked(dev(x), B, S, d, H, dev(g), 1,
                                                                *[P[n][1] for n in "qkvo"])
    assert ref is not None and got is not None
    assert np.array_equal(host(got[0]), ref[0]) and got[1] == ref[1]


@pytest.mark.parametrize("T,d,F", [(256, 256, 1024), (100, 128, 512), (7, 64, 96)])
def test_prenorm_mlp_block_parity(core, T, d, F):
    bw = Y.BlockWeights(77 + F, d, F)
    P = {nm: lin_pair(core, getattr(bw, nm), bw.shift[nm]) for nm in ("up", "gate", "down")}
    x = Y.q15_gaussian(41, (T, d))
    x[3 % T] = 32767  # drive some residual saturations
    g = np.full(d, 4096, np.int16)
    ref = O.prenorm_mlp_block(x, T, d, F, g, 1, P["up"][0], P["gate"][0], P["down"][0], threads=4)
    got = core.prenorm_gated_mlp_residual_block_i16_q15_checked(dev(x), T, d, F, dev(g), 1, P["up"][1],
                                                                P["gate"][1], P["down"][1])
    assert ref is not None and got is not None
    assert np.array_equal(host(got[0]), ref[0]) and got[1] == ref[1]


def test_bench_1m_output_hash_on_gpu(core):
    """The published bench-1m output hash (ENG.md:790-799) reproduced by four GPU transformer blocks."""
    p = Y.BENCH_1M
    d, F, S, H = p["d_model"], p["hidden_dim"], p["seq_len"], p["heads"]
    g = torch.full((d,), 8192, dtype=torch.int16)
    cur = dev(Y.bench1m_input())
    sat = 0
    for blk in Y.bench1m_model():
        L = {k: lin_pair(core, blk[k], Y.BENCH_1M_SHIFTS[k])[1] for k in blk}
        tb = core.TransformerBlock(d, H, F, L["q"], L["k"], L["v"], L["o"], L["up"], L["gate"], L["down"], g, g, 1)
        out = tb(cur, 1, S)
        assert out is not None
        cur = out[0]
        sat += out[1] + out[2]
    assert Y.fnv1a_i16(host(cur)) == Y.BENCH_1M_OUTPUT_HASH
    assert sat == 0


def test_transformer_block_parity(core):
    B, S, d, H, F = 2, 256, 256, 4, 1024
    bw = Y.BlockWeights(5, d, F)
    P = {nm: lin_pair(core, getattr(bw, nm), bw.shift[nm]) for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    x = Y.q15_gaussian(3, (B * S, d))
    y1, s1 = O.prenorm_attention_block(x, B, S, d, H, bw.attn_gamma, 1, *[P[n][0] for n in "qkvo"], threads=4)
    y2, s2 = O.prenorm_mlp_block(y1, B * S, d, F, bw.mlp_gamma, 1, P["up"][0], P["gate"][0], P["down"][0], threads=4)
    tb = core.TransformerBlock(d, H, F, *[P[n][1] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                               dev(bw.attn_gamma), dev(bw.mlp_gamma), 1)
    out = tb(dev(x), B, S)
    assert out is not None
    assert np.array_equal(host(out[0]), y2) and out[1] == s1 and out[2] == s2


@pytest.mark.parametrize("B,chunk", [(5, 2), (3, 3), (4, 8), (21, 8)])
def test_transformer_block_host_buffers(core, B, chunk):
    """The host-buffer block (chunked copy / compute overlap with steps that ramp
    up and down, e.g. 2, 4, 8, 1, 4, 2 sequences for 21 in chunks of 8) equals the
    oracle, saturation counts included."""
    import torch
    S, d, H, F = 128, 128, 2, 512
    bw = Y.BlockWeights(8, d, F)
    P = {nm: lin_pair(core, getattr(bw, nm), bw.shift[nm]) for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    x = Y.q15_gaussian(4, (B * S, d))
    y1, s1 = O.prenorm_attention_block(x, B, S, d, H, bw.attn_gamma, 1, *[P[n][0] for n in "qkvo"], threads=4)
    y2, s2 = O.prenorm_mlp_block(y1, B * S, d, F, bw.mlp_gamma, 1, P["up"][0], P["gate"][0], P["down"][0], threads=4)
    tb = core.TransformerBlock(d, H, F, *[P[n][1] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                               dev(bw.attn_gamma), dev(bw.mlp_gamma), 1)
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.zeros_like(xh).pin_memory()
    ws = core.workspace(tb.host_workspace_bytes(min(chunk, B), S))
    st = core.Status()
    st.reset()
    assert tb.launch_host(xh, yh, B, S, chunk, ws, st) == 0
    code, h = st.fetch()
    assert code == 0
    assert np.array_equal(yh.numpy(), y2) and h.attention_saturations == s1 and h.mlp_saturations == s2


# ----------------------------------------------------------------- decode ---
@pytest.mark.parametrize("B,H,hd,Lmax", [(3, 2, 64, 300), (4, 4, 16, 129), (2, 1, 256, 70), (2, 3, 4, 50)])
def test_decode_attention_parity(core, B, H, hd, Lmax):
    d = H * hd
    q = Y.q15_gaussian(1, (B, d), sigma_shift=17)
    kc = Y.q15_gaussian(2, (B, Lmax, d), sigma_shift=14)
    vc = Y.q15_gaussian(3, (B, Lmax, d))
    lens = (np.arange(B) * 37 % Lmax + 1).astype(np.int32)
    lens[0] = Lmax
    ref = O.decode_attention(q, kc, vc, lens, B, H, hd, Lmax, threads=4)
    got = core.attention_decode(dev(q), dev(kc), dev(vc), dev(lens), H, hd)
    assert ref is not None and got is not None
    assert np.array_equal(host(got), ref)


def test_decode_rejects_bad_length(core):
    B, H, hd, Lmax = 2, 1, 64, 16
    q = np.ones((B, hd), np.int16)
    kc = np.ones((B, Lmax, hd), np.int16)
    lens = np.array([4, 0], np.int32)
    assert core.attention_decode(dev(q), dev(kc), dev(kc), dev(lens), H, hd) is None


@pytest.mark.parametrize("B,d,H,Lmax", [(3, 128, 2, 100), (5, 256, 4, 300), (2, 64, 1, 200)])
def test_decode_block_parity(core, B, d, H, Lmax):
    """One decode step == last causal row with cached keys/values (attention.rs:671-725, :742-877)."""
    P = attn_weights(core, d, 55 + d)
    hd = d // H
    x = Y.q15_gaussian(3, (B, d))
    gamma = np.full(d, 4096, np.int16)
    kc = Y.q15_gaussian(4, (B, Lmax, d), sigma_shift=15)
    vc = Y.q15_gaussian(5, (B, Lmax, d))
    pos = (np.arange(B) * 17 % (Lmax - 1)).astype(np.int32)
    pos[0] = Lmax - 1
    # oracle: rms -> q, k, v -> cache row pos -> attention over pos + 1 keys -> o -> residual
    xn = O.rms_norm_rows(x, gamma, 1)
    q = O.linear(xn, P["q"][0])
    k = O.linear(xn, P["k"][0])
    v = O.linear(xn, P["v"][0])
    kc_ref, vc_ref = kc.copy(), vc.copy()
    kc_ref[np.arange(B), pos] = k
    vc_ref[np.arange(B), pos] = v
    ctx = O.decode_attention(q, kc_ref, vc_ref, pos + 1, B, H, hd, Lmax, threads=4)
    att = O.linear(ctx, P["o"][0])
    y_ref, sat_ref = O.residual_add(x, att)
    # the decode block keeps its caches head-major: [B][H][Lmax][hd]
    hm = lambda c: np.ascontiguousarray(c.reshape(B, Lmax, H, hd).transpose(0, 2, 1, 3))
    kcg, vcg = dev(hm(kc)), dev(hm(vc))
    got = core.prenorm_attention_decode_block(dev(x), H, dev(gamma), 1, *[P[n][1] for n in "qkvo"], kcg, vcg,
                                              dev(pos))
    assert got is not None
    assert np.array_equal(host(got[0]), y_ref) and got[1] == sat_ref
    assert np.array_equal(host(kcg), hm(kc_ref)) and np.array_equal(host(vcg), hm(vc_ref))
