"""Linear (recurrent) attention on the GPU against the oracle, bit for bit:
the full forward (causal and not, head dims 2 to 64), the streaming step
(plain and test-time training) with carried states, the mini transformer
with the linear kind (byte-head rows, full-window generation), and the
incremental streaming generation of one-layer models
(crates/nsrl-core/src/attention.rs:879-1478, nsrl-train/src/lib.rs:12802-12980)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

from train_models import random_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def core():
    from nsrl_b200 import build, core as K
    build.build()
    return K


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def lins(core, d, seed, shift):
    rng = np.random.default_rng(seed)
    o, g = [], []
    for i in range(4):
        w = rng.integers(-127, 128, (d, d)).astype(np.int8)
        o.append(O.Linear(w, O.scales(1, shift, d)))
        g.append(core.Linear(torch.from_numpy(w), core.make_scales(1, shift, d)))
    return o, g


@pytest.mark.parametrize("B,S,d,H,causal", [(3, 40, 64, 4, True), (2, 33, 128, 2, True), (2, 17, 64, 4, False),
                                            (1, 70, 128, 8, True), (2, 9, 12, 3, True), (1, 5, 6, 3, False)])
def test_linear_attention_forward(core, B, S, d, H, causal):
    o, g = lins(core, d, d + S, 9 if d >= 64 else 6)
    x = np.random.default_rng(S).integers(-20000, 20000, (B * S, d)).astype(np.int16)
    ref = O.linear_attention(x, B, S, d, H, *o, causal=causal)
    got = core.linear_attention_i16_q15_checked(dev(x), B, S, d, H, *g, causal=causal)
    assert ref is not None and got is not None
    assert np.array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("ttt", [None, 0, 3])
def test_linear_attention_streams(core, ttt):
    B, d, H, steps = 5, 64, 4, 12
    hd = d // H
    o, g = lins(core, d, 77, 9)
    rng = np.random.default_rng(8)
    streams = core.LinearAttentionStreams(B, d, H)
    st = np.zeros((B, H * hd * hd), np.int64)
    ks = np.zeros((B, H * hd), np.int64)
    dl = np.zeros(B, np.uint64)
    for t in range(steps):
        x = rng.integers(-20000, 20000, (B, d)).astype(np.int16)
        ref = O.linear_attention_step(x, H, *o, st, ks, ttt_shift=ttt, delta_l1=dl)
        got = streams.step(dev(x), *g, ttt_shift=ttt)
        assert ref is not None and got is not None
        assert np.array_equal(got.cpu().numpy(), ref), t
    assert np.array_equal(streams.state.cpu().numpy(), st)
    assert np.array_equal(streams.key_sums.cpu().numpy(), ks)
    if ttt is not None:
        assert np.array_equal(streams.delta_l1.cpu().numpy().view(np.uint64), dl) and dl.sum() > 0


def test_streaming_steps_equal_the_full_causal_forward(core):
    """attention.rs:2257-2334 on the GPU at a larger shape."""
    B, S, d, H = 3, 24, 64, 4
    o, g = lins(core, d, 5, 9)
    x = np.random.default_rng(4).integers(-20000, 20000, (B, S, d)).astype(np.int16)
    full = core.linear_attention_i16_q15_checked(dev(x.reshape(B * S, d)), B, S, d, H, *g).cpu().numpy()
    streams = core.LinearAttentionStreams(B, d, H)
    rows = [streams.step(dev(x[:, t]), *g).cpu().numpy() for t in range(S)]
    assert np.array_equal(np.stack(rows, axis=1).reshape(B * S, d), full)


def _linear_model(layers, rms, positions, seed, H=8):
    m = random_model(128, H, 256, layers, 16, rms=rms, positions=positions, seed=seed)
    m.attention_kind = "linear"
    m.head = O.Linear(m.head.weights, O.scales(1, 14, 256))
    return m


def _gpu(m):
    from test_gpu_train_step import to_gpu
    gm = to_gpu(m)
    gm.attention_kind = m.attention_kind
    return gm


@pytest.mark.parametrize("layers,rms,pos", [(2, True, True), (1, False, False)])
def test_linear_kind_rows_and_generation(core, layers, rms, pos):
    from nsrl_b200 import generate as G
    m = _linear_model(layers, rms, pos, 30 + layers)
    gm = _gpu(m)
    win = np.random.default_rng(2).integers(0, 256, (6, 16)).astype(np.uint8)
    ref = O.output_rows(m, win)
    got = G.output_rows(gm, torch.from_numpy(win))
    assert np.array_equal(got[0].cpu().numpy(), ref[0]) and np.array_equal(got[1].cpu().numpy(), ref[1])
    prompts = [b"abc", b"the linear attention model"]
    gen = G.Generator(gm, 2, 26, 10)
    out = gen(prompts, "sample", 16, 99)
    for b, p in enumerate(prompts):
        r = O.generate(m, p, 10, "sample", 16, 99)
        assert np.array_equal(out[0][b].numpy(), r[0]), b


@pytest.mark.parametrize("ttt,strategy", [(None, "greedy"), (None, "sample"), (2, "sample")])
def test_streaming_generation(core, ttt, strategy):
    from nsrl_b200 import generate as G
    m = _linear_model(1, False, False, 44)
    gm = _gpu(m)
    prompts = [b"tyger tyger", b"burning brig", b"in the fores"][:3]
    prompts = [p[:11] for p in prompts]
    steps = 20
    gen = G.StreamingGenerator(gm, len(prompts), 11, steps)
    out = gen(prompts, strategy, 12, 5, ttt_shift=ttt)
    assert out is not None
    for b, p in enumerate(prompts):
        r = O.generate_streaming(m, p, steps, strategy, 12, 5, ttt_shift=ttt)
        assert r is not None
        assert np.array_equal(out[0][b].numpy(), r[0]), (b, out[0][b].tolist(), r[0].tolist())
        assert np.array_equal(out[1][b].numpy(), r[1]) and np.array_equal(out[2][b].numpy(), r[2])
