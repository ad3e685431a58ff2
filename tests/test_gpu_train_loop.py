"""The integer-Adam training loop (nsrl_b200.loop) on the GPU against the
oracle's restatement of the reference's run (lib.rs:4499-4800), over several
batches: the trace counters, every weight and the optimizer state; resuming
from a saved state equals the uninterrupted run (lib.rs:20770-20810); the
loss-regression guard rejects the same batches."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import train_loop as OL

from train_models import random_model

pytestmark = pytest.mark.gpu

TEXT = (b"The road of excess leads to the palace of wisdom. Tyger Tyger, burning bright, in the forests of the "
        b"night; what immortal hand or eye could frame thy fearful symmetry? Shall I compare thee to a summer's day?")


def _model(seed=3, rms=True):
    m = random_model(64, 4, 128, 2, 16, rms=rms, positions=True, seed=seed)
    m.head = O.Linear(m.head.weights, O.scales(1, 14, 256))
    return m


def _gpu(m):
    from test_gpu_train_step import to_gpu
    return to_gpu(m)


def _same_model(om, gm):
    from test_gpu_dp_step import _check_model
    _check_model(om, gm)


def _trace(tr):
    return {k: v for k, v in tr.items() if k != "state"}


@pytest.mark.parametrize("scope,adam", [("all", (1, 1, 3, 7, 1)), ("final_mlp_and_output", (2, 0, 2, 5, 3))])
def test_training_loop_matches_the_oracle(scope, adam):
    from nsrl_b200 import loop as Lp
    m = _model()
    gm = _gpu(m)
    kw = dict(epochs=2, stride=3, max_windows=24, batch_windows=8)
    ref, om, ost = OL.run_integer_adam_training(TEXT, m, adam=adam, scope=scope, **kw)
    got = Lp.run_integer_adam_training(TEXT, gm, Lp.LoopConfig(**kw), adam=adam, scope=scope)
    assert _trace(got) == ref
    assert ref["accepted_batch_count"] == 6
    _same_model(om, gm)
    st = got["state"].adam
    assert np.array_equal(st.first_moments.cpu().numpy(), ost.first)
    assert np.array_equal(st.second_moments.cpu().numpy().view(np.uint64), ost.second)
    assert np.array_equal(st.update_residuals.cpu().numpy(), ost.residuals)


def test_resume_matches_uninterrupted_training():
    """Two epochs at once == one epoch, the model and optimizer state saved to
    the host, then a second epoch from them (lib.rs:20770-20810)."""
    from nsrl_b200 import loop as Lp
    from nsrl_b200 import train as T
    cfg1 = Lp.LoopConfig(epochs=1, stride=3, max_windows=24, batch_windows=8)
    cfg2 = Lp.LoopConfig(epochs=2, stride=3, max_windows=24, batch_windows=8)
    adam = (1, 1, 3, 7, 1)
    m = _model(seed=9)
    whole = _gpu(m)
    t2 = Lp.run_integer_adam_training(TEXT, whole, cfg2, adam=adam)
    part = _gpu(m)
    t1 = Lp.run_integer_adam_training(TEXT, part, cfg1, adam=adam)
    saved = {k: getattr(t1["state"].adam, k).cpu() for k in ("first_moments", "second_moments", "update_residuals",
                                                               "step")}
    resumed = T.TrainState(part, adam=True)
    for k, v in saved.items():
        getattr(resumed.adam, k).copy_(v)
    t3 = Lp.run_integer_adam_training(TEXT, part, cfg1, adam=adam, state=resumed)
    assert t3["optimizer_step"] == t2["optimizer_step"] == 6
    for a, b in [(whole.head.weights, part.head.weights), (whole.embeddings, part.embeddings),
                 (whole.positions, part.positions)]:
        assert torch.equal(a, b)
    for la, lb in zip(whole.layers, part.layers):
        for n in T.LAYER_LINEARS:
            assert torch.equal(la[n].weights, lb[n].weights), n
        assert torch.equal(la["attn_gamma"], lb["attn_gamma"]) and torch.equal(la["mlp_gamma"], lb["mlp_gamma"])
    for k in saved:
        assert torch.equal(getattr(t2["state"].adam, k), getattr(t3["state"].adam, k)), k


def test_loss_regression_guard_rejects_like_the_oracle():
    """A large Adam step size makes some batches raise the guard windows' loss:
    the same batches are rejected and rolled back as in the oracle."""
    from nsrl_b200 import loop as Lp
    m = _model(seed=21)
    gm = _gpu(m)
    kw = dict(epochs=2, stride=2, max_windows=32, batch_windows=4, reject_loss_regression=True)
    adam = (64, 0, 1, 2, 1)
    ref, om, _ = OL.run_integer_adam_training(TEXT, m, adam=adam, **kw)
    got = Lp.run_integer_adam_training(TEXT, gm, Lp.LoopConfig(**kw), adam=adam)
    assert _trace(got) == ref
    _same_model(om, gm)
