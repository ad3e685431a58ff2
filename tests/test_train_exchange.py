"""The int64 gradient exchange between data-parallel ranks, on CPU with gloo.

Each of two ranks holds its own i64 accumulators (one contiguous chunk of
the batch each, as the reference's map-reduce workers do); after
allreduce_weight_gradients_i64 every rank must hold the reference's ordered,
checked merge (crates/nsrl-train/src/lib.rs:7443-7471) of both parts, or
report a rejection exactly when that merge overflows i64.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _parts(case, rank):
    rng = np.random.default_rng(10 + rank)
    if case == "random":
        a = rng.integers(-2**40, 2**40, size=(3, 5), dtype=np.int64)
        b = rng.integers(-2**40, 2**40, size=(4,), dtype=np.int64).reshape(1, 4)
        return [a, b], [rank + 2, 5 * rank + 1]
    if case == "overflow":  # 2^62 + 2^62 leaves i64 in the first merge step
        return [np.full((1, 2), 2**62, np.int64)], [1]
    if case == "large_ok":  # the bound fails but no prefix overflows: the exact path
        return [np.array([[2**62 if rank == 0 else -2**62, 7]], np.int64)], [3]
    raise ValueError(case)


def _worker(rank, world, port, case, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import torch.distributed as dist
    from nsrl_b200 import train as T
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    parts, counts = _parts(case, rank)
    grads = []
    for p, c in zip(parts, counts):
        g = T.LinearWeightGradientI64(p.shape[1], p.shape[0], device=torch.device("cpu"))
        g.accumulators.copy_(torch.from_numpy(p))
        g.sample_count.fill_(c)
        grads.append(g)
    ok = T.allreduce_weight_gradients_i64(grads)
    res = {"ok": ok, "acc": [g.accumulators.numpy().copy() for g in grads],
           "count": [int(g.sample_count.item()) for g in grads]}
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("case", ["random", "overflow", "large_ok"])
def test_allreduce_matches_ordered_merge(tmp_path, case):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), case, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    results = [np.load(tmp_path / f"r{r}.npy", allow_pickle=True).item() for r in range(world)]
    nbuf = len(results[0]["acc"])
    for i in range(nbuf):
        parts = np.stack([_parts(case, r)[0][i].ravel() for r in range(world)])
        counts = [_parts(case, r)[1][i] for r in range(world)]
        ref = O.merge_i64(parts, counts)
        for res in results:
            if ref is None:
                assert not res["ok"]
            else:
                assert res["ok"]
                assert np.array_equal(res["acc"][i].ravel(), ref[0]) and res["count"][i] == ref[1]


def _flat_worker(rank, world, port, case, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import torch.distributed as dist
    from nsrl_b200 import train as T
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    parts, _ = _parts(case, rank)
    flat = torch.from_numpy(np.concatenate([p.ravel() for p in parts]))
    out, ok = T.allreduce_flat_i64(flat)
    np.save(os.path.join(out_dir, f"f{rank}.npy"), np.array({"ok": ok, "out": out.numpy().copy()}, dtype=object),
            allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("case", ["random", "overflow", "large_ok"])
def test_flat_arena_allreduce_matches_ordered_merge(tmp_path, case):
    """The training step's single-vector exchange (arena + counts + stats)."""
    world = 2
    mp.start_processes(_flat_worker, args=(world, _free_port(), case, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    parts = np.stack([np.concatenate([p.ravel() for p in _parts(case, r)[0]]) for r in range(world)])
    ref = O.merge_i64(parts, [0] * world)
    for r in range(world):
        res = np.load(tmp_path / f"f{r}.npy", allow_pickle=True).item()
        if ref is None:
            assert not res["ok"]
        else:
            assert res["ok"] and np.array_equal(res["out"], ref[0])


def test_apply_shift_rules_match_oracle():
    """Batch and stacked-layer learning-rate shifts (lib.rs:13591-13650, :15454-15495)."""
    from nsrl_b200 import train as T
    cfg = T.MiniTransformerTrainConfig()
    for layers in (1, 2, 4):
        for windows in (1, 2, 3, 64, 256, 1000):
            a = T.layer_apply_shifts(cfg, windows, layers)
            b = O.batch_apply_shifts(O.DEFAULT_TRAIN_CONFIG, windows, layers)
            assert a == b, (layers, windows)
    assert T.mini_transformer_batch_learning_rate_shift(0) is None
    with pytest.raises(ValueError):
        T.mini_transformer_batch_component_shift_config(T.MiniTransformerTrainConfig(output_learning_rate_shift=1), 8)
