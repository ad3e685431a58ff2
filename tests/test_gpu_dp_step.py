"""The data-parallel step behind the C ABI (nsrl_train_dp_step) on one GPU:
the integer-Adam optimizer in every train scope, a rejected batch, an
invalid learning-rate config, and the ordered worker merge it falls back
to, each against the oracle bit for bit."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

from train_models import random_model, random_windows

pytestmark = pytest.mark.gpu


def _train():
    from nsrl_b200 import build, train
    build.build()
    return train


def _gpu_model(m):
    from test_gpu_train_step import to_gpu
    return to_gpu(m)


def _check_model(m, gm):
    assert np.array_equal(gm.head.weights.cpu().numpy(), m.head.weights)
    for ly, gly in zip(m.layers, gm.layers):
        for nm in O.LAYER_LINEARS:
            assert np.array_equal(gly[nm].weights.cpu().numpy(), ly[nm].weights), nm
        for g in ("attn_gamma", "mlp_gamma"):
            if ly.get(g) is not None:
                assert np.array_equal(gly[g].cpu().numpy(), ly[g]), g
    assert np.array_equal(gm.embeddings.cpu().numpy(), m.embeddings)
    if m.positions is not None:
        assert np.array_equal(gm.positions.cpu().numpy(), m.positions)


@pytest.mark.parametrize("scope", ["all", "rms_norm", "output", "final_mlp", "final_mlp_and_output"])
def test_integer_adam_step_every_scope(scope):
    """Three batches with integer Adam as the optimizer (lib.rs:4270-4465):
    weights, RMS gammas, embeddings, the moments, the update residuals and
    the step, against the oracle's map-reduce batch and Adam batch apply."""
    T = _train()
    d, H, F, L, S, W = 64, 4, 128, 2, 16, 4
    m = random_model(d, H, F, L, S, rms=True, positions=True, seed=51)
    gm = _gpu_model(m)
    acfg = (1, 4, 3, 7, 1)
    ocfg = O.AdamConfig(*acfg)
    ostate = O.AdamState(O.adam_state_layout(m)["total"])
    state = T.TrainState(gm, adam=True)
    assert state.adam.first_moments.numel() == ostate.first.size
    cfg = T.MiniTransformerTrainConfig(optimizer="integer_adam", adam=acfg, adam_scope=scope)
    buf = T.TrainStepBuffers(gm, W)
    for step in range(3):
        ctx, tgt = random_windows(W, S, seed=60 + step)
        ref = O.adam_train_step(m, ostate, ctx, tgt, ocfg, scope=scope)
        got = T.mini_transformer_train_step(gm, state, torch.from_numpy(ctx).cuda(), torch.from_numpy(tgt).cuda(),
                                            cfg, buf)
        assert ref is not None and got == ref, (step, got, ref)
        _check_model(m, gm)
        assert np.array_equal(state.adam.first_moments.cpu().numpy(), ostate.first)
        assert np.array_equal(state.adam.second_moments.cpu().numpy().view(np.uint64), ostate.second)
        assert np.array_equal(state.adam.update_residuals.cpu().numpy(), ostate.residuals)
        assert int(state.adam.step.item()) == ostate.step == step + 1


def test_rejected_batch_leaves_the_model_unchanged():
    """A forward multiplier other than 1 is a rejection of the training step
    (the reference's scale tables all have multiplier 1): the whole batch is
    rejected and nothing is applied (lib.rs:5371-5375)."""
    T = _train()
    from nsrl_b200 import core
    d, H, F, L, S, W = 64, 4, 128, 1, 16, 2
    m = random_model(d, H, F, L, S, seed=5)
    gm = _gpu_model(m)
    gm.layers[0]["up"] = core.Linear(gm.layers[0]["up"].weights, core.make_scales(2, 10, F))
    before = [gm.head.weights.clone()] + [gm.layers[0][n].weights.clone() for n in O.LAYER_LINEARS]
    emb = gm.embeddings.clone()
    state = T.TrainState(gm)
    ctx, tgt = random_windows(W, S, seed=3)
    out = T.mini_transformer_train_step(gm, state, torch.from_numpy(ctx).cuda(), torch.from_numpy(tgt).cuda(),
                                        T.MiniTransformerTrainConfig(), T.TrainStepBuffers(gm, W))
    assert out is None
    after = [gm.head.weights] + [gm.layers[0][n].weights for n in O.LAYER_LINEARS]
    assert all(torch.equal(a, b) for a, b in zip(before, after))
    assert torch.equal(emb, gm.embeddings) and int(state.residuals.abs().sum()) == 0


def test_shift_below_the_batch_shift_is_an_invalid_config():
    """mini_transformer_batch_component_shift_config (lib.rs:13607-13650):
    8 windows make a batch shift of 3, above an output shift of 2."""
    T = _train()
    d, H, F, L, S, W = 64, 4, 128, 1, 16, 8
    m = random_model(d, H, F, L, S, seed=8)
    gm = _gpu_model(m)
    ctx, tgt = random_windows(W, S, seed=4)
    cfg = T.MiniTransformerTrainConfig(output_learning_rate_shift=2)
    with pytest.raises(ValueError, match="batch shift"):
        T.mini_transformer_train_step(gm, T.TrainState(gm), torch.from_numpy(ctx).cuda(),
                                      torch.from_numpy(tgt).cuda(), cfg, T.TrainStepBuffers(gm, W))


@pytest.mark.parametrize("case", ["random", "overflow", "large_ok"])
def test_ordered_worker_merge(case):
    """nsrl_merge_worker_parts_i64 against the oracle's merge (lib.rs:7443-7471):
    checked adds in worker order, including an overflow that only a prefix sees."""
    T = _train()
    from nsrl_b200 import core
    L = T._lib_dp()
    rng = np.random.default_rng(7)
    workers, n = 4, 100_003
    if case == "random":
        parts = rng.integers(-2**50, 2**50, size=(workers, n), dtype=np.int64)
    elif case == "overflow":  # 2^62 + 2^62 leaves i64 at the second worker; the total would come back
        parts = np.zeros((workers, n), np.int64)
        parts[:, 77] = [2**62, 2**62, -2**62, -2**62]
    else:  # the all-reduce bound fails, no prefix overflows
        parts = np.zeros((workers, n), np.int64)
        parts[:, 5] = [2**62, -2**62, 2**62, -2**62]
    counts = rng.integers(0, 1000, size=(workers, 9), dtype=np.uint64)
    ref = O.merge_i64(parts, counts.sum(axis=1))
    both = torch.from_numpy(np.concatenate([parts, counts.astype(np.int64)], axis=1)).cuda()
    out = torch.empty(n + 9, dtype=torch.int64, device="cuda")
    st = core.Status()
    st.reset()
    r = L.nsrl_merge_worker_parts_i64(core._ptr(both), workers, n, n + 9, core._ptr(out), core._ptr(st.buf),
                                      core._stream())
    assert r == core.NSRL_OK
    code, _ = st.fetch()
    if ref is None:
        assert code == core.NSRL_CORE_REJECTED
        return
    assert code == core.NSRL_OK
    got = out.cpu().numpy()
    assert np.array_equal(got[:n], ref[0])
    assert np.array_equal(got[n:].view(np.uint64), counts.sum(axis=0))


@pytest.mark.parametrize("dtype,divisor", [(np.int8, 1), (np.int8, 3), (np.int8, 8), (np.int16, 5), (np.int16, 2)])
def test_average_batch_movement(dtype, divisor):
    """average_mini_transformer_batch_movement's per-tensor rule (lib.rs:14552-14583)
    against the oracle, saturation at both rails included."""
    T = _train()
    import ctypes as C
    from nsrl_b200 import core
    L = T._lib_dp()
    info = np.iinfo(dtype)
    rng = np.random.default_rng(divisor)
    n = 70_001
    base = rng.integers(info.min, info.max + 1, n).astype(dtype)
    vals = rng.integers(info.min, info.max + 1, n).astype(dtype)
    base[:4] = [info.max, info.min, info.max, 0]
    vals[:4] = [info.min, info.max, info.max, info.min]
    ref = O.average_movement(base, vals, divisor)
    fn = L.nsrl_average_movement_i8 if dtype == np.int8 else L.nsrl_average_movement_i16
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_uint64, C.c_void_p]
    b, v = torch.from_numpy(base).cuda(), torch.from_numpy(vals).cuda()
    assert fn(core._ptr(b), core._ptr(v), n, divisor, core._stream()) == core.NSRL_OK
    assert np.array_equal(v.cpu().numpy(), ref)
    assert fn(core._ptr(b), core._ptr(v), n, 0, core._stream()) == core.NSRL_INVALID_SHAPE


def test_apply_divider_matches_integer_division():
    """The apply's divider (a 32-bit multiply-shift below 2^32, a double
    reciprocal of the count with one exact integer correction below 2^52,
    integer division above) against Python's exact round-half-away-from-zero
    division, at the edges: halves, the 2^32 and 2^52 boundaries, i64
    extremes, counts on both sides of 2^32 and 2^52."""
    import ctypes as C
    from nsrl_b200 import core
    T = _train()
    L = T._lib_dp()
    L.nsrl_selftest_round_div.argtypes = [C.c_void_p, C.c_size_t, C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p]
    rng = np.random.default_rng(11)
    edge = [0, 1, -1, 2, -2, 3, -3, (1 << 52) - 1, 1 << 52, (1 << 52) + 1, -(1 << 52), (1 << 62), -(1 << 62),
            (1 << 63) - 1, -(1 << 63) + 1, -(1 << 63)]

    def ref(n, d):
        half = d // 2
        m = abs(n)
        if n == -(1 << 63) or m > (1 << 63) - 1 - half:
            return None
        q = (m + half) // d
        return q if n >= 0 else -q

    # dens on both sides of 2^32 (the 32-bit multiply-shift path) and 2^52 (the double path)
    for den in (1, 2, 3, 7, 255, 256, 1000, 65537, (1 << 31) - 1, (1 << 32) - 1, 1 << 32, (1 << 32) + 1,
                (1 << 52) - 1, 1 << 52, (1 << 60) + 7):
        nums = list(edge)
        nums += [k * den + den // 2 + o for k in (0, 1, 5, 12345) for o in (-1, 0, 1) if abs(k * den) < (1 << 62)]
        nums += [(1 << 32) - 1 - den // 2 + o for o in (-1, 0, 1)] + [-((1 << 32) - 1 - den // 2) + o for o in (-1, 0, 1)]
        nums += list(rng.integers(-(1 << 32), 1 << 32, 2000))
        nums += list(rng.integers(-(1 << 53), 1 << 53, 2000))
        nums += list(rng.integers(-(1 << 62), 1 << 62, 2000))
        a = np.array(nums, dtype=np.int64)
        num = torch.from_numpy(a).cuda()
        out = torch.empty_like(num)
        ok = torch.empty(len(nums), dtype=torch.uint8, device="cuda")
        assert L.nsrl_selftest_round_div(core._ptr(num), len(nums), den, core._ptr(out), core._ptr(ok),
                                         core._stream()) == core.NSRL_OK
        got, good = out.cpu().numpy(), ok.cpu().numpy()
        for i, n in enumerate(nums):
            r = ref(int(n), den)
            assert (r is None) == (good[i] == 0), (n, den)
            if r is not None:
                assert int(got[i]) == r, (n, den, int(got[i]), r)


def _sgd_values(rng, n, big):
    """Gradient sums and residuals on both sides of the fast path's limits
    (|sum| <= 2^30, residual an i32), up to 2^40 when big."""
    edge = [0, 1, -1, (1 << 30) - 1, 1 << 30, (1 << 30) + 1, -(1 << 30), -(1 << 30) - 1]
    raw = rng.integers(-(1 << 24), 1 << 24, n)
    raw[: len(edge)] = edge
    raw[::11] = 0
    if big:
        raw[1::5] = rng.integers(-(1 << 40), 1 << 40, len(raw[1::5]))
    res = rng.integers(-(1 << 12), 1 << 12, n)
    res[::3] = 0
    if big:
        res[2::7] = rng.integers(-(1 << 40), 1 << 40, len(res[2::7]))
        res[3::13] = [(1 << 31) - 1, 1 << 31, -(1 << 31), -(1 << 31) - 1] * (len(res[3::13]) // 4) + \
            [1 << 31] * (len(res[3::13]) % 4)
    return raw.astype(np.int64), res.astype(np.int64)


@pytest.mark.parametrize("i8", [True, False])
@pytest.mark.parametrize("count,lr,shift", [(1, 1, 0), (3, 1, 7), (256, 3, 12), (255, 1, 30), (7, 5, 31),
                                            ((1 << 32) - 1, 1, 3), ((1 << 32) + 5, 1 << 20, 9), (9, 1, 45)])
@pytest.mark.parametrize("big", [False, True])
def test_sgd_apply_rule_matches_oracle(i8, count, lr, shift, big):
    """The element rule of the data-parallel apply's SGD segments (its 32-bit
    fast path and the checked 64-bit path) against the oracle's i8 apply with
    the residual carried and its i16 embedding apply: residuals, weights and
    the three statistics."""
    import ctypes as C
    from nsrl_b200 import core
    T = _train()
    L = T._lib_dp()
    L.nsrl_selftest_sgd_apply.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_size_t, C.c_ulonglong,
                                          C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    n = 20000
    rng = np.random.default_rng(count % 1000 + 31 * shift + 7 * lr + (5 if big else 0) + (1 if i8 else 0))
    raw, res = _sgd_values(rng, n, big)
    w = rng.integers(-128, 128, n).astype(np.int8) if i8 else rng.integers(-32768, 32768, n).astype(np.int16)
    if i8:
        ref = O.apply_linear_gradient_i64_to_i8(raw, res, w, count, lr, shift, True)
        assert ref is not None
        ref_res, ref_w, ref_stats = ref[1], ref[2], ref[4]
    else:
        ref_res, ref_w, st = res.copy(), w.copy(), np.zeros(3, np.uint64)
        assert O.apply_embedding_gradient_i64_to_i16(raw.copy(), ref_res, ref_w, count, lr, shift, st)
        ref_stats = [int(x) for x in st]
    g_raw, g_res, g_w = (torch.from_numpy(a.copy()).cuda() for a in (raw, res, w))
    stats = torch.zeros(3, dtype=torch.int64, device="cuda")
    bad = torch.zeros(1, dtype=torch.uint8, device="cuda")
    assert L.nsrl_selftest_sgd_apply(core._ptr(g_raw), core._ptr(g_res), core._ptr(g_w), int(i8), n, count, lr, shift,
                                     core._ptr(stats), core._ptr(bad), core._stream()) == core.NSRL_OK
    assert int(bad.item()) == 0
    assert np.array_equal(g_res.cpu().numpy(), ref_res)
    assert np.array_equal(g_w.cpu().numpy(), ref_w)
    assert [int(x) for x in stats.cpu().numpy()] == ref_stats


@pytest.mark.parametrize("i8", [True, False])
@pytest.mark.parametrize("case", ["sum_min", "product", "residual_add"])
def test_sgd_apply_rule_flags_overflow(i8, case):
    """One element whose checked arithmetic fails among ordinary ones: the
    oracle rejects the apply and the element rule reports it."""
    import ctypes as C
    from nsrl_b200 import core
    T = _train()
    L = T._lib_dp()
    L.nsrl_selftest_sgd_apply.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_size_t, C.c_ulonglong,
                                          C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    n = 1000
    rng = np.random.default_rng(3)
    raw, res = _sgd_values(rng, n, False)
    lr = 1
    if case == "sum_min":
        raw[500] = -(1 << 63)
    elif case == "product":
        raw[500], lr = (1 << 62) - 5, 4
    else:
        raw[500], res[500] = (1 << 62), (1 << 62)
    w = rng.integers(-100, 100, n).astype(np.int8) if i8 else rng.integers(-1000, 1000, n).astype(np.int16)
    if i8:
        assert O.apply_linear_gradient_i64_to_i8(raw, res, w, 1, lr, 5, True) is None
    else:
        assert not O.apply_embedding_gradient_i64_to_i16(raw.copy(), res.copy(), w.copy(), 1, lr, 5,
                                                         np.zeros(3, np.uint64))
    g_raw, g_res, g_w = (torch.from_numpy(a.copy()).cuda() for a in (raw, res, w))
    stats = torch.zeros(3, dtype=torch.int64, device="cuda")
    bad = torch.zeros(1, dtype=torch.uint8, device="cuda")
    assert L.nsrl_selftest_sgd_apply(core._ptr(g_raw), core._ptr(g_res), core._ptr(g_w), int(i8), n, 1, lr, 5,
                                     core._ptr(stats), core._ptr(bad), core._stream()) == core.NSRL_OK
    assert int(bad.item()) == 1
