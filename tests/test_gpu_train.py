"""GPU parity of the training-exchange kernels (accumulate, apply) with the oracle."""
import numpy as np
import pytest

from nsrl_b200 import synth as Y
from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def T():
    from nsrl_b200 import build, train
    build.build()
    return train


@pytest.mark.parametrize("rows,K,N", [(37, 100, 70), (256, 256, 1024), (1, 4, 2)])
def test_accumulate_matches_oracle(T, rows, K, N):
    x = Y.q15_gaussian(K + rows, (rows, K))
    g = (Y.q15_gaussian(N, (rows, N)).astype(np.int32) * 1021)
    g[0, : N // 2] = 0  # zero terms are skipped by the reference
    acc0 = Y.q15_gaussian(7, (N, K)).astype(np.int64) * 12345
    ref = O.accumulate_linear_gradient_i64(x, g, acc0, 5)
    grad = T.LinearWeightGradientI64(K, N)
    grad.accumulators.copy_(torch.from_numpy(acc0))
    grad.sample_count.fill_(5)
    assert T.accumulate_linear_weight_gradient_i64_prescaled(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                                                             grad)
    assert np.array_equal(grad.accumulators.cpu().numpy(), ref[0])
    assert int(grad.sample_count.item()) == ref[1]


def test_accumulate_rejects_i64_overflow(T):
    grad = T.LinearWeightGradientI64(2, 1)
    grad.accumulators.fill_(2**63 - 10)
    x = torch.tensor([[1, 1]], dtype=torch.int16).cuda()
    g = torch.tensor([[100]], dtype=torch.int32).cuda()
    assert O.accumulate_linear_gradient_i64(x.cpu().numpy(), g.cpu().numpy(),
                                            grad.accumulators.cpu().numpy(), 0) is None
    assert not T.accumulate_linear_weight_gradient_i64_prescaled(x, g, grad)


@pytest.mark.parametrize("carry,shift,lr", [(False, 22, 1), (True, 12, 3), (True, 0, 1), (True, 30, 7)])
def test_apply_matches_oracle(T, carry, shift, lr):
    n = 5000
    rng = np.random.default_rng(shift)
    acc = rng.integers(-2**40, 2**40, n).astype(np.int64)
    acc[::7] = 0
    res = rng.integers(-2**20, 2**20, n).astype(np.int64)
    w = rng.integers(-128, 128, n).astype(np.int8)
    ref = O.apply_linear_gradient_i64_to_i8(acc, res, w, 9, lr, shift, carry)
    grad = T.LinearWeightGradientI64(n, 1)
    grad.accumulators.copy_(torch.from_numpy(acc).view(1, n))
    grad.residuals.copy_(torch.from_numpy(res).view(1, n))
    grad.sample_count.fill_(9)
    wt = torch.from_numpy(w).cuda()
    st = T.apply_linear_weight_gradient_i64_to_i8(grad, wt, lr, shift, carry)
    assert st is not None
    assert np.array_equal(wt.cpu().numpy(), ref[2])
    assert np.array_equal(grad.residuals.cpu().numpy().ravel(), ref[1])
    assert not grad.accumulators.any() and int(grad.sample_count.item()) == 0
    assert [st["gradient_saturation_count"], st["zero_delta_count"], st["weight_delta_l1"]] == ref[4]


def test_apply_kats_on_gpu(T):
    """crates/nsrl-train-core/src/lib.rs:1896-1966 through the device path."""
    grad = T.LinearWeightGradientI64(2, 2)
    x = torch.tensor([[4096, 8192]], dtype=torch.int16).cuda()
    g = torch.tensor([[1024, 2048]], dtype=torch.int32).cuda()
    assert T.accumulate_linear_weight_gradient_i64_prescaled(x, g, grad)
    assert T.accumulate_linear_weight_gradient_i64_prescaled(x, g, grad)
    w = torch.full((4,), 10, dtype=torch.int8).cuda()
    st = T.apply_linear_weight_gradient_i64_to_i8(grad, w, 1, 22, False)
    assert w.cpu().tolist() == [9, 8, 8, 6]
    assert st == {"gradient_saturation_count": 0, "zero_delta_count": 0, "weight_delta_l1": 9}
    grad = T.LinearWeightGradientI64(1, 1)
    one16 = torch.tensor([[1]], dtype=torch.int16).cuda()
    one32 = torch.tensor([[1]], dtype=torch.int32).cuda()
    w = torch.tensor([10], dtype=torch.int8).cuda()
    T.accumulate_linear_weight_gradient_i64_prescaled(one16, one32, grad)
    st = T.apply_linear_weight_gradient_i64_to_i8(grad, w, 1, 2, True)
    assert w.item() == 10 and st["zero_delta_count"] == 1 and grad.residuals.item() == 1
    T.accumulate_linear_weight_gradient_i64_prescaled(one16, one32, grad)
    st = T.apply_linear_weight_gradient_i64_to_i8(grad, w, 1, 2, True)
    assert w.item() == 9 and st["weight_delta_l1"] == 1 and grad.residuals.item() == -2
    # nothing accumulated: a no-op
    st = T.apply_linear_weight_gradient_i64_to_i8(grad, w, 1, 2, True)
    assert w.item() == 9 and st["weight_delta_l1"] == 0
