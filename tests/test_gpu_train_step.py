"""GPU parity of the training step: every backward primitive and the
map-reduce window step against the oracle, bit for bit."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

from train_models import (TEXT, random_model, random_windows, reference_initial_model, window_starts,
                          windows_from_text)

pytestmark = pytest.mark.gpu


def _core():
    from nsrl_b200 import core, train
    return core, train


def _lin(lin):
    core, _ = _core()
    sc = core.make_scales(lin.scales["multiplier"].astype(np.int64), lin.scales["right_shift"].astype(np.int64))
    return core.Linear(torch.from_numpy(lin.weights.copy()), sc,
                       None if lin.bias is None else torch.from_numpy(lin.bias.copy()))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def to_gpu(m):
    _, train = _core()
    layers = []
    for ly in m.layers:
        e = {nm: _lin(ly[nm]) for nm in O.LAYER_LINEARS}
        for g in ("attn_gamma", "mlp_gamma"):
            if ly.get(g) is not None:
                e[g] = torch.from_numpy(ly[g].copy())
        layers.append(e)
    return train.TrainModel(torch.from_numpy(m.embeddings.copy()),
                            None if m.positions is None else torch.from_numpy(m.positions.copy()), layers,
                            _lin(m.head), m.d, m.H, m.F, m.S)


@pytest.mark.parametrize("M,K,N,shift", [(7, 64, 48, 0), (300, 256, 256, 3), (129, 96, 1024, 0)])
def test_linear_backward_input(M, K, N, shift):
    _, train = _core()
    rng = np.random.default_rng(M + K)
    lin = O.Linear(rng.integers(-127, 128, (N, K)).astype(np.int8), O.scales(1, shift, N))
    g = rng.integers(-32768, 32768, (M, N)).astype(np.int16)
    ref = O.linear_backward_input(g, lin)
    out = train.linear_backward_input_i16_i8_i16_per_channel_checked(_dev(g), _lin(lin))
    assert np.array_equal(out.cpu().numpy(), ref)


def test_linear_backward_input_general_scales():
    """Multipliers other than 1 and per-channel grad-input scales (the SIMT form)."""
    core, train = _core()
    rng = np.random.default_rng(11)
    M, K, N = 33, 48, 32
    lin = O.Linear(rng.integers(-127, 128, (N, K)).astype(np.int8),
                   O.scales(rng.integers(1, 5, N), rng.integers(0, 4, N)))
    gin = O.scales(rng.integers(1, 3, K), rng.integers(0, 3, K))
    g = rng.integers(-32768, 32768, (M, N)).astype(np.int16)
    ref = O.linear_backward_input(g, lin, gin)
    gin_t = core.make_scales(gin["multiplier"].astype(np.int64), gin["right_shift"].astype(np.int64))
    out = train.linear_backward_input_i16_i8_i16_per_channel_checked(_dev(g), _lin(lin), gin_t)
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("T,d,F", [(5, 32, 64), (257, 128, 256)])
def test_gated_mlp_backward_input(T, d, F):
    _, train = _core()
    rng = np.random.default_rng(T)
    up = O.Linear(rng.integers(-127, 128, (F, d)).astype(np.int8), O.scales(1, 10, F))
    gate = O.Linear(rng.integers(-127, 128, (F, d)).astype(np.int8), O.scales(1, 10, F))
    down = O.Linear(rng.integers(-127, 128, (d, F)).astype(np.int8), O.scales(1, 11, d))
    fu = rng.integers(-32768, 32768, (T, F)).astype(np.int16)
    fg = rng.integers(-32768, 32768, (T, F)).astype(np.int16)
    g = rng.integers(-8000, 8000, (T, d)).astype(np.int16)
    ref = O.gated_mlp_backward_input(g, up, gate, down, fu, fg)
    out = train.gated_mlp_backward_input_i16_q15_checked(_dev(g), _lin(up), _lin(gate), _lin(down), _dev(fu), _dev(fg))
    for a, b in zip(out[:3], ref[:3]):
        assert np.array_equal(a.cpu().numpy(), b)
    assert out[3] == ref[3]


@pytest.mark.parametrize("T,d,eps", [(3, 4, 1), (513, 256, 1), (64, 128, 0)])
def test_rms_norm_backward(T, d, eps):
    _, train = _core()
    rng = np.random.default_rng(T + d)
    x = rng.integers(-32768, 32768, (T, d)).astype(np.int16)
    x[0, :] = rng.integers(-3, 4, d)  # a small row: large inverse RMS
    w = rng.integers(-32768, 32768, d).astype(np.int16)
    go = rng.integers(-32768, 32768, (T, d)).astype(np.int16)
    ref = O.rms_norm_backward_rows(x, w, go, eps)
    gi, gw, sat = train.rms_norm_backward_rows(_dev(x), _dev(w), _dev(go), eps)
    assert np.array_equal(gi.cpu().numpy(), ref[0])
    assert np.array_equal(gw.cpu().numpy(), ref[1])
    assert sat == ref[2]


# (40, 272, 128, 2): 240 query tiles of the tensor-core dL kernel, more than one per SM,
# with S past a multiple of 128 and of 64
@pytest.mark.parametrize("B,S,d,H", [(2, 33, 64, 4), (3, 64, 128, 2), (1, 200, 64, 1), (2, 48, 64, 4),
                                     (1, 520, 128, 2), (2, 4, 64, 1), (2, 256, 256, 4), (1, 528, 128, 2),
                                     (40, 272, 128, 2)])
def test_attention_probabilities_and_backward(B, S, d, H):
    _, train = _core()
    rng = np.random.default_rng(B * S)
    q = rng.integers(-6000, 6000, (B * S, d)).astype(np.int16)
    k = rng.integers(-6000, 6000, (B * S, d)).astype(np.int16)
    v = rng.integers(-32768, 32768, (B * S, d)).astype(np.int16)
    dC = rng.integers(-32768, 32768, (B * S, d)).astype(np.int16)
    P = O.attention_probabilities(q, k, B, S, d, H)
    ctx_g, P_g = train.attention_with_probabilities(_dev(q), _dev(k), _dev(v), B, S, d, H)
    assert np.array_equal(P_g.cpu().numpy(), P)
    ref = O.attention_backward(q, k, v, P, dC, B, S, d, H)
    out = train.attention_backward(_dev(q), _dev(k), _dev(v), P_g, _dev(dC), B, S, d, H)
    for a, b in zip(out, ref):
        assert np.array_equal(a.cpu().numpy(), b)


def _check_step(m, ctx, tgt):
    _, train = _core()
    ref = O.train_windows(m, ctx, tgt)
    assert ref is not None
    out = train.mini_transformer_map_reduce_worker_batch(to_gpu(m), torch.from_numpy(ctx), torch.from_numpy(tgt))
    assert out is not None
    arena, counts, stats = out
    a = arena.cpu().numpy()
    lay = m.arena_layout()
    for key, span in lay.items():
        if key == "total":
            continue
        o, n = span
        assert np.array_equal(a[o:o + n], ref[0][o:o + n]), key
    assert np.array_equal(counts.cpu().numpy().astype(np.uint64), ref[1])
    assert stats == ref[2]


def test_train_step_reference_initial_model():
    """The reference's stacked map-reduce test case (lib.rs:22832-22925) on the GPU."""
    m = reference_initial_model(seq_len=4, layers=2)
    ctx, tgt = windows_from_text(TEXT, 4, window_starts(len(TEXT), 4, 1, 4))
    _check_step(m, ctx, tgt)


@pytest.mark.parametrize("d,H,F,L,S,W,rms,pos", [
    (64, 4, 128, 2, 16, 3, True, True),
    (64, 1, 128, 1, 24, 2, False, False),
    (128, 2, 256, 2, 40, 2, True, False),
    (128, 2, 256, 2, 144, 2, True, True),   # head_dim 64, S % 16 == 0: the tensor-core backward, a ragged key tile
    (128, 2, 256, 1, 272, 2, False, True),  # three 128-query tiles: P cached as planes, dQ on the tensor cores
])
def test_train_step_random_models(d, H, F, L, S, W, rms, pos):
    m = random_model(d, H, F, L, S, rms=rms, positions=pos, seed=d + S)
    ctx, tgt = random_windows(W, S, seed=d + S)
    _check_step(m, ctx, tgt)


def _weights_equal(m, gm):
    assert np.array_equal(gm.head.weights.cpu().numpy(), m.head.weights)
    for ly, gly in zip(m.layers, gm.layers):
        for nm in O.LAYER_LINEARS:
            assert np.array_equal(gly[nm].weights.cpu().numpy(), ly[nm].weights), nm
    assert np.array_equal(gm.embeddings.cpu().numpy(), m.embeddings)
    if m.positions is not None:
        assert np.array_equal(gm.positions.cpu().numpy(), m.positions)


@pytest.mark.parametrize("L,rms", [(2, True), (1, False)])
def test_data_parallel_step_updates_weights_bit_exact(L, rms):
    """Two batches of the full step (windows, exchange, apply) against the oracle:
    every updated i8 weight, i16 embedding and carried residual."""
    _, train = _core()
    d, H, F, S, W = 64, 4, 128, 16, 4
    m = random_model(d, H, F, L, S, rms=rms, positions=True, seed=21 + L)
    gm = to_gpu(m)
    res = np.zeros(m.arena_layout()["total"], np.int64)
    state = train.TrainState(gm)
    buf = train.TrainStepBuffers(gm, W)
    cfg = train.MiniTransformerTrainConfig(output_learning_rate_shift=10, mlp_learning_rate_shift=12,
                                           embedding_learning_rate_shift=8, attention_learning_rate_shift=14,
                                           attention_q_learning_rate_shift=12, attention_qk_learning_rate_shift=12)
    ocfg = {f: getattr(cfg, f) for f in O.DEFAULT_TRAIN_CONFIG}
    for step in range(2):
        ctx, tgt = random_windows(W, S, seed=30 + step)
        ref = O.train_step(m, res, ctx, tgt, cfg=ocfg)
        out = train.mini_transformer_train_step(gm, state, torch.from_numpy(ctx).cuda(), torch.from_numpy(tgt).cuda(),
                                                cfg, buf)
        assert ref is not None and out is not None
        assert out == ref
        _weights_equal(m, gm)
        assert np.array_equal(state.residuals.cpu().numpy(), res)


def test_sharded_windows_sum_to_the_whole_batch():
    """Rank chunks run separately and merged in order equal the one-GPU batch
    (the reference's multi-worker == single-worker pin, lib.rs:22927-23000)."""
    _, train = _core()
    m = random_model(64, 4, 128, 2, 16, seed=40)
    gm = to_gpu(m)
    ctx, tgt = random_windows(6, 16, seed=41)
    whole = train.mini_transformer_map_reduce_worker_batch(gm, torch.from_numpy(ctx), torch.from_numpy(tgt))
    parts = [train.mini_transformer_map_reduce_worker_batch(gm, torch.from_numpy(ctx[i:i + 3]),
                                                            torch.from_numpy(tgt[i:i + 3])) for i in (0, 3)]
    merged, ovf = train._ordered_merge(torch.stack([p[0] for p in parts]))
    assert not ovf
    assert torch.equal(merged, whole[0])
    assert torch.equal(parts[0][1] + parts[1][1], whole[1])


@pytest.mark.parametrize("rows,K,N,shift", [(300, 64, 48, 0), (1000, 256, 1024, 2), (4133, 200, 72, 0),
                                          (777, 100, 37, 1)])
def test_weight_gradient_tensor_cores(rows, K, N, shift):
    """The tcgen05 weight-gradient product against an exact int64 matmul of the prescaled grads."""
    core, train = _core()
    rng = np.random.default_rng(rows + K)
    x = rng.integers(-32768, 32768, (rows, K)).astype(np.int16)
    g = rng.integers(-32768, 32768, (rows, N)).astype(np.int16)
    acc0 = rng.integers(-2**40, 2**40, (N, K)).astype(np.int64)
    gp = g.astype(np.int64)
    if shift:
        gp = (gp + (1 << (shift - 1))) >> shift  # rhu with multiplier 1
    ref = acc0 + gp.T @ x.astype(np.int64)
    acc = torch.from_numpy(acc0.copy()).cuda()
    cnt = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert train.accumulate_weight_gradient_i16(_dev(x), _dev(g), core.make_scales(1, shift, N), acc, cnt)
    assert np.array_equal(acc.cpu().numpy(), ref)
    assert int(cnt.item()) == rows


def test_weight_gradient_tensor_cores_extreme_values():
    """Byte-plane extremes over a 32768-row work item (the s32 limit of the
    accumulators): 304 output tiles make one item per tile, so each item sums
    all 32768 rows.  -32513 gives |gh xl + gl xh| = 65280 and -1 x 255 gives
    gl xl = 65025 per row, the largest mid and low sums."""
    core, train = _core()
    rows, K, N = 32768, 2048, 2432
    for gv, xv in ((-32768, -32768), (-32513, -32513), (-1, 255), (32767, 32767), (32767, -32768)):
        x = torch.full((rows, K), xv, dtype=torch.int16, device="cuda")
        g = torch.full((rows, N), gv, dtype=torch.int16, device="cuda")
        acc = torch.zeros((N, K), dtype=torch.int64, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int64, device="cuda")
        assert train.accumulate_weight_gradient_i16(x, g, core.make_scales(1, 0, N), acc, cnt)
        assert bool((acc == rows * gv * xv).all()), (gv, xv)
        del x, g, acc


@pytest.mark.parametrize("wdtype,count", [(np.int8, 3), (np.int16, 7), (np.int8, 1)])
def test_integer_adam_matches_oracle(wdtype, count):
    """Five steps of integer Adam over random and extreme accumulators, moments,
    residuals, weights and stats, against the oracle."""
    _, train = _core()
    rng = np.random.default_rng(count)
    n = 3000
    info = np.iinfo(wdtype)
    w = rng.integers(info.min, info.max + 1, n).astype(wdtype)
    cfg_o = O.AdamConfig(learning_rate=3, step_shift=2, beta1_decay_shift=3, beta2_decay_shift=7, epsilon=1)
    cfg_g = train.IntegerAdamConfigC(learning_rate=3, step_shift=2, beta1_decay_shift=3, beta2_decay_shift=7,
                                     epsilon=1)
    so = O.AdamState(n)
    sg = train.IntegerAdamState(n)
    wg = torch.from_numpy(w.copy()).cuda()
    cnt = torch.tensor([count], dtype=torch.int64, device="cuda")
    for step in range(5):
        acc = rng.integers(-2**40, 2**40, n).astype(np.int64)
        acc[:4] = [2**62, -2**62, 0, 2**33]  # the first two saturate the moment gradient
        ref = O.integer_adam(acc, count, w, cfg_o, so)
        got = train.apply_integer_adam_accumulators(torch.from_numpy(acc).cuda(), cnt, wg, cfg_g, sg)
        assert ref is not None and got is not None
        assert [got["gradient_saturation_count"], got["zero_delta_count"], got["weight_delta_l1"]] == ref
        assert np.array_equal(wg.cpu().numpy(), w)
        assert np.array_equal(sg.first_moments.cpu().numpy(), so.first)
        assert np.array_equal(sg.second_moments.cpu().numpy().view(np.uint64), so.second)
        assert np.array_equal(sg.update_residuals.cpu().numpy(), so.residuals)
        assert int(sg.step.item()) == so.step == step + 1
