"""Parity at the benchmarked sizes: the CUDA path at the full shapes of the
measured workloads, compared with the oracle on sampled sequences, rows or
windows (the oracle is scalar C++, so it checks a slice while the GPU runs
the whole batch; the slice is taken from the full-size launch).

- linear sweep: M = 65,536, K = N = 4096 (the largest sweep GEMM), every
  512th row and the last row against the oracle;
- transformer block: 64 sequences x 1024 tokens, d 256, 4 x 64 heads, MLP
  1024 (the block-forward workload), four sequences against the oracle;
- decode: 4-layer d 512, 8 x 64 heads, MLP 2048, KV prefix 8192, batch 4,
  two steps (the decode workload's shapes at a smaller batch);
- training: 4 layers, d 256, 4 x 64 heads, MLP 1024, seq 512 on two
  windows, every updated weight, embedding and residual.
"""
import numpy as np
import pytest

from nsrl_b200 import synth as Y
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

LINEARS = ("q", "k", "v", "o", "up", "gate", "down")


@pytest.fixture(scope="module")
def core():
    from nsrl_b200 import build, core as K
    build.build()
    O.use_native()
    return K


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def block_linears(core, bw):
    o = {n: O.Linear(getattr(bw, n), O.scales(1, bw.shift[n], bw.out_dim(n))) for n in LINEARS}
    g = {n: core.Linear(torch.from_numpy(getattr(bw, n)), core.make_scales(1, bw.shift[n], bw.out_dim(n)))
         for n in LINEARS}
    return o, g


def q15_host(shape, seed, sigma=4096.0):
    """Gaussian int16 from a seeded torch CPU generator (cheaper than the Irwin-Hall draws at these sizes)."""
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=gen) * sigma).clamp_(-32768, 32767).to(torch.int16).numpy()


def q15_device(shape, seed):
    """Gaussian sigma 4096 int16 made on the device (the oracle reads the same values back)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=gen, device="cuda") * 4096).clamp_(-32768, 32767).to(torch.int16)


def test_linear_sweep_largest_shape(core):
    M, K = 65536, 4096
    N = K
    w = Y.i8_uniform(Y.tensor_seed(9, K), (N, K))
    o = O.Linear(w, O.scales(1, Y.shift_for(K), N))
    g = core.Linear(torch.from_numpy(w), core.make_scales(1, Y.shift_for(K), N))
    x = q15_device((M, K), 17)
    y = core.linear_i16_i8_i16_per_channel_checked(x, g)
    assert y is not None
    rows = torch.cat([torch.arange(0, M, 512), torch.tensor([M - 1])]).cuda()
    xs = x.index_select(0, rows).cpu().numpy()
    ref = O.linear(xs, o, threads=8)
    assert ref is not None
    assert np.array_equal(y.index_select(0, rows).cpu().numpy(), ref)


def test_transformer_block_full_batch(core):
    B, S, d, H, F = 64, 1024, 256, 4, 1024
    bw = Y.BlockWeights(seed=2024, d=d, hidden=F)
    ol, gl = block_linears(core, bw)
    x = q15_host((B * S, d), 99)
    blk = core.TransformerBlock(d, H, F, *[gl[n] for n in LINEARS], torch.from_numpy(bw.attn_gamma),
                                torch.from_numpy(bw.mlp_gamma), 1)
    out = blk(dev(x), B, S)
    assert out is not None
    got = out[0].cpu().numpy().reshape(B, S, d)
    for b in (0, 1, 37, 63):
        xs = x.reshape(B, S, d)[b]
        y1, _ = O.prenorm_attention_block(xs, 1, S, d, H, bw.attn_gamma, 1, *[ol[n] for n in "qkvo"])
        y2, _ = O.prenorm_mlp_block(y1, S, d, F, bw.mlp_gamma, 1, ol["up"], ol["gate"], ol["down"], threads=4)
        assert np.array_equal(got[b], y2), f"sequence {b}"


def test_decode_full_prefix(core):
    """Two decode steps of the 4-layer d512 model over an 8192-token prefix:
    every layer's output and appended cache rows against the oracle's last
    causal row over the same cache."""
    Lyr, d, H, F, B, prefix = 4, 512, 8, 2048, 4, 8192
    hd = d // H
    Lmax = prefix + 2
    layers = []
    for li in range(Lyr):
        bw = Y.BlockWeights(seed=77 + li, d=d, hidden=F)
        ol, gl = block_linears(core, bw)
        kc = q15_host((B, Lmax, d), 500 + 2 * li, sigma=512.0)  # narrower K: a live softmax
        vc = q15_host((B, Lmax, d), 501 + 2 * li)
        layers.append(dict(bw=bw, ol=ol, gl=gl, kc=kc, vc=vc))
    hm = lambda c: np.ascontiguousarray(c.reshape(B, Lmax, H, hd).transpose(0, 2, 1, 3))
    for ly in layers:
        ly["kcg"], ly["vcg"] = dev(hm(ly["kc"])), dev(hm(ly["vc"]))
    x = Y.q15_gaussian(7, (B, d))
    xg = dev(x)
    for t in range(2):
        pos = np.full(B, prefix + t, np.int32)
        pos[1] -= 3 + t  # ragged positions: rows past a sequence's length are never read
        for li, ly in enumerate(layers):
            bw, ol = ly["bw"], ly["ol"]
            xn = O.rms_norm_rows(x, bw.attn_gamma, 1)
            q, k, v = (O.linear(xn, ol[n]) for n in "qkv")
            ly["kc"][np.arange(B), pos] = k
            ly["vc"][np.arange(B), pos] = v
            ctx = O.decode_attention(q, ly["kc"], ly["vc"], pos + 1, B, H, hd, Lmax, threads=4)
            h_ref, _ = O.residual_add(x, O.linear(ctx, ol["o"]))
            y_ref, _ = O.prenorm_mlp_block(h_ref, B, d, F, bw.mlp_gamma, 1, ol["up"], ol["gate"], ol["down"])
            gl = ly["gl"]
            h = core.prenorm_attention_decode_block(xg, H, dev(bw.attn_gamma), 1, *[gl[n] for n in "qkvo"],
                                                    ly["kcg"], ly["vcg"], dev(pos))
            assert h is not None
            assert np.array_equal(h[0].cpu().numpy(), h_ref), (t, li)
            y = core.prenorm_gated_mlp_residual_block_i16_q15_checked(h[0], B, d, F, dev(bw.mlp_gamma), 1, gl["up"],
                                                                      gl["gate"], gl["down"])
            assert y is not None and np.array_equal(y[0].cpu().numpy(), y_ref), (t, li)
            x, xg = y_ref, y[0]
    for ly in layers:
        assert np.array_equal(ly["kcg"].cpu().numpy(), hm(ly["kc"]))
        assert np.array_equal(ly["vcg"].cpu().numpy(), hm(ly["vc"]))


def test_training_step_full_model(core):
    """One data-parallel step of the 4-layer d256 seq-512 model on two windows:
    stats, every i8 weight, the i16 embeddings and positions, the residuals."""
    from nsrl_b200 import train as T
    Lyr, d, H, F, S, W = 4, 256, 4, 1024, 512, 2
    tw = Y.TrainWeights(seed=4040, layers=Lyr, d=d, hidden=F, seq_len=S)
    olayers, glayers = [], []
    for bw in tw.blocks:
        ol, gl = block_linears(core, bw)
        ol = {n: O.Linear(ol[n].weights.copy(), ol[n].scales) for n in LINEARS}
        ol["attn_gamma"], ol["mlp_gamma"] = bw.attn_gamma, bw.mlp_gamma
        gl["attn_gamma"], gl["mlp_gamma"] = torch.from_numpy(bw.attn_gamma), torch.from_numpy(bw.mlp_gamma)
        olayers.append(ol)
        glayers.append(gl)
    om = O.TrainModel(tw.embeddings.copy(), tw.positions.copy(), olayers,
                      O.Linear(tw.head.copy(), O.scales(1, tw.head_shift, 256)), d, H, F, S)
    gm = T.TrainModel(torch.from_numpy(tw.embeddings), torch.from_numpy(tw.positions), glayers,
                      core.Linear(torch.from_numpy(tw.head), core.make_scales(1, tw.head_shift, 256)), d, H, F, S)
    ctx, tgt = Y.train_windows(0x7EA1, W, S)
    cfg = T.MiniTransformerTrainConfig()
    res = np.zeros(om.arena_layout()["total"], np.int64)
    ref = O.train_step(om, res, ctx, tgt, cfg={f: getattr(cfg, f) for f in O.DEFAULT_TRAIN_CONFIG}, workers=W)
    state = T.TrainState(gm)
    got = T.mini_transformer_train_step(gm, state, dev(ctx), dev(tgt), cfg, T.TrainStepBuffers(gm, W))
    assert ref is not None and got == ref
    assert np.array_equal(gm.head.weights.cpu().numpy(), om.head.weights)
    for ol, gl in zip(olayers, glayers):
        for n in LINEARS:
            assert np.array_equal(gl[n].weights.cpu().numpy(), ol[n].weights), n
    assert np.array_equal(gm.embeddings.cpu().numpy(), om.embeddings)
    assert np.array_equal(gm.positions.cpu().numpy(), om.positions)
    assert np.array_equal(state.residuals.cpu().numpy(), res)
