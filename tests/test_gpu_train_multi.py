"""The data-parallel training step on two GPUs (NCCL): each rank runs its
contiguous chunk of the batch's windows; after the exact int64 exchange and
the apply, every rank's weights equal the oracle's one-worker batch
(the reference's multi-worker == single-worker pin, nsrl-train/src/lib.rs:22927-23000).
Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O

from train_models import random_model, random_windows

pytestmark = pytest.mark.gpu

D, H, F, L, S, W, STEPS = 64, 4, 128, 2, 16, 8, 2
SHIFTS = dict(output_learning_rate_shift=10, mlp_learning_rate_shift=12, embedding_learning_rate_shift=8,
              attention_learning_rate_shift=14, attention_q_learning_rate_shift=12,
              attention_qk_learning_rate_shift=12)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from nsrl_b200 import train as T
    from test_gpu_train_step import to_gpu
    m = random_model(D, H, F, L, S, seed=77)
    gm = to_gpu(m)
    state = T.TrainState(gm)
    per = W // world
    buf = T.TrainStepBuffers(gm, per)
    cfg = T.MiniTransformerTrainConfig(**SHIFTS)
    stats = []
    for step in range(STEPS):
        ctx, tgt = random_windows(W, S, seed=90 + step)
        lo, hi = rank * per, (rank + 1) * per
        r = T.mini_transformer_train_step(gm, state, torch.from_numpy(ctx[lo:hi]).cuda(),
                                          torch.from_numpy(tgt[lo:hi]).cuda(), cfg, buf)
        stats.append(r)
    res = {"stats": stats, "head": gm.head.weights.cpu().numpy(),
           "layers": [{nm: ly[nm].weights.cpu().numpy() for nm in O.LAYER_LINEARS} for ly in gm.layers],
           "emb": gm.embeddings.cpu().numpy(), "pos": gm.positions.cpu().numpy(),
           "res": state.residuals.cpu().numpy()}
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_training_step_matches_one_worker(tmp_path):
    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    m = random_model(D, H, F, L, S, seed=77)
    res = np.zeros(m.arena_layout()["total"], np.int64)
    ocfg = dict(O.DEFAULT_TRAIN_CONFIG, **SHIFTS)
    ref_stats = []
    for step in range(STEPS):
        ctx, tgt = random_windows(W, S, seed=90 + step)
        ref_stats.append(O.train_step(m, res, ctx, tgt, cfg=ocfg))
    for r in range(world):
        out = np.load(tmp_path / f"rank{r}.npy", allow_pickle=True).item()
        assert out["stats"] == ref_stats
        assert np.array_equal(out["head"], m.head.weights)
        for ly, oly in zip(out["layers"], m.layers):
            for nm in O.LAYER_LINEARS:
                assert np.array_equal(ly[nm], oly[nm].weights), nm
        assert np.array_equal(out["emb"], m.embeddings) and np.array_equal(out["pos"], m.positions)
        assert np.array_equal(out["res"], res)


def _leaving_rank(rank, world, port, out_dir):
    """Two data-parallel steps, then rank 1 leaves between steps (none of its
    work in flight: the step call returns only when its GPU work is done).
    Rank 0 learns of it on the host, in the peer check before its third step,
    so nothing of that step is launched; the communicator is aborted and the
    GPU stays usable.  NVLS is off (a rank leaving while bound to an NVLink
    multicast object is to be avoided)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from nsrl_b200 import core, train as T
    from test_gpu_train_step import to_gpu
    m = random_model(D, H, F, L, S, seed=77)
    gm = to_gpu(m)
    state = T.TrainState(gm)
    per = W // world
    buf = T.TrainStepBuffers(gm, per, nranks=world)
    cfg = T.MiniTransformerTrainConfig(**SHIFTS)
    comm = T.Communicator(timeout_ms=4000)
    out = []
    for step in range(3):
        if rank == 1 and step == 2:
            T._lib_dp().nsrl_comm_abort(comm.handle)  # leaves as a failed rank would: no finalize handshake
            comm.close()
            break
        ctx, tgt = random_windows(W, S, seed=90 + step)
        lo, hi = rank * per, (rank + 1) * per
        try:
            r = T.mini_transformer_train_step(gm, state, torch.from_numpy(ctx[lo:hi]).cuda(),
                                              torch.from_numpy(tgt[lo:hi]).cuda(), cfg, buf, comm=comm)
            out.append("ok" if r is not None else "rejected")
        except T.CommError as e:
            out.append(f"comm-error-{e.code}")
            break
    if rank == 0:
        comm.close()  # aborted already: frees it
        lin = core.Linear(torch.eye(64, dtype=torch.int8), core.make_scales(1, 0, 64))
        x = torch.arange(64 * 64, dtype=torch.int16).reshape(64, 64).cuda()
        y = core.linear_i16_i8_i16_per_channel_checked(x, lin)
        out.append("gpu-ok" if y is not None and torch.equal(y, x) else "gpu-bad")
    np.save(os.path.join(out_dir, f"leave{rank}.npy"), np.array(out, dtype=object), allow_pickle=True)
    if rank == 0:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_rank_leaving_between_steps(tmp_path):
    mp.start_processes(_leaving_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = list(np.load(tmp_path / "leave0.npy", allow_pickle=True))
    r1 = list(np.load(tmp_path / "leave1.npy", allow_pickle=True))
    assert r1 == ["ok", "ok"]
    assert r0 == ["ok", "ok", "comm-error-5", "gpu-ok"]
