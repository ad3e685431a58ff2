"""Host logic of the training loop (no GPU): window starts, guard windows,
loss-guard windows and the regression rule against the reference's own unit
tests (crates/nsrl-train/src/lib.rs:23613-23786), and the product's helpers
against the oracle's restatement."""
import pytest

from nsrl_b200 import loop as Lp
from oracle import train_loop as OL


def test_byte_window_starts_remain_sequential():  # lib.rs:23613-23617
    assert Lp.byte_window_starts(1000, 4, 10, 0, 5) == [0, 10, 20, 30, 40]


def test_window_starts_spread_capped_runs():  # lib.rs:23619-23623
    assert Lp.window_starts(1000, 4, 10, 0, 5) == [0, 250, 500, 740, 990]


def test_window_starts_keep_full_runs_sequential():  # lib.rs:23625-23630
    assert Lp.window_starts(1000, 4, 10, 0, None) == Lp.byte_window_starts(1000, 4, 10, 0, None)


def test_loss_guard_starts_mix_batch_and_global_points():  # lib.rs:23757-23769
    starts = [i * 10 for i in range(32)]
    g = Lp.loss_guard_starts(starts, 5, 7)
    assert g[:2] == [50, 60] and 0 in g and 310 in g and len(g) == 17


@pytest.mark.parametrize("n,S,stride,off,mx", [(1000, 4, 10, 0, 5), (1000, 4, 10, 0, None), (50, 16, 3, 2, 24),
                                                (17, 16, 1, 0, 8), (16, 16, 1, 0, 8), (300, 7, 2, 11, 1),
                                                (300, 7, 2, 11, 0)])
def test_window_starts_match_the_oracle(n, S, stride, off, mx):
    assert Lp.window_starts(n, S, stride, off, mx) == OL.window_starts(n, S, stride, off, mx)


@pytest.mark.parametrize("n,epoch,wi,epochs", [(24, 0, 7, 2), (24, 1, 23, 2), (24, 0, 23, 2), (1, 0, 0, 1),
                                               (5, 0, 4, 1)])
def test_guard_indices_match_the_oracle(n, epoch, wi, epochs):
    assert Lp.guard_indices(n, epoch, wi, epochs) == OL._guards(n, epoch, wi, epochs)
