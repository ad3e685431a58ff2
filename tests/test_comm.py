"""Failure handling of the data-parallel communicator, without a GPU.

- The bounded wait that every collective of nsrl_train_dp_step goes
  through, run by nsrl_comm_selftest_wait against a fake clock and fake
  completion / error reports: it returns once the work completes, gives up
  at the deadline with NSRL_COMM_TIMEOUT, and stops at a peer's error with
  NSRL_COMM_ERROR, aborting the communicator in both failure cases.
- The bootstrap of Communicator over two gloo ranks: rank 0's NCCL id
  reaches rank 1 intact, and a rank that never joins makes the other fail
  within the group's timeout instead of hanging.
"""
import ctypes as C
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp


def _lib():
    from nsrl_b200 import build, train
    build.build()
    return train._lib_dp()


@pytest.mark.parametrize("scenario,timeout_ms,code,aborted", [(0, 50, 0, 0), (1, 50, 4, 1), (2, 50, 5, 1)])
def test_bounded_comm_wait(scenario, timeout_ms, code, aborted):
    L = _lib()
    polls, ab = C.c_uint64(), C.c_int()
    r = L.nsrl_comm_selftest_wait(scenario, timeout_ms, C.byref(polls), C.byref(ab))
    assert r == code and ab.value == aborted
    if scenario == 0:
        assert polls.value == 3
    elif scenario == 1:
        assert polls.value == timeout_ms + 2  # 1 ms of fake clock per poll: the first poll past the deadline
        assert b"aborted" in L.nsrl_last_error()
    else:
        assert polls.value == 3 and b"peer" in L.nsrl_last_error()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _boot(rank, world, port, out_dir, absent):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from nsrl_b200 import core, train as T
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == absent:
        return  # this rank leaves without joining the communicator
    seen = {}
    L = T._lib_dp()
    orig = L.nsrl_comm_init

    def record(handle, nranks, r, uid, timeout):
        seen["id"] = bytes(uid)
        seen["args"] = (nranks, r, timeout)
        return orig(handle, nranks, r, uid, timeout)

    L.nsrl_comm_init = record
    t0 = time.time()
    try:
        T.Communicator(timeout_ms=3000)
        outcome = "joined"
    except T.CommError as e:  # no CUDA device here: the join itself fails, loudly
        outcome = f"comm-error-{e.code}"
    except RuntimeError as e:  # the group's own timeout: a rank never arrived
        outcome = f"group-error: {type(e).__name__}"
    res = {"outcome": outcome, "id": seen.get("id"), "args": seen.get("args"), "elapsed": time.time() - t0,
           "code_cuda": core.NSRL_CUDA_ERROR}
    np.save(os.path.join(out_dir, f"boot{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)


def test_communicator_bootstrap_over_gloo(tmp_path):
    mp.start_processes(_boot, args=(2, _free_port(), str(tmp_path), -1), nprocs=2, join=True, start_method="spawn")
    r0 = np.load(tmp_path / "boot0.npy", allow_pickle=True).item()
    r1 = np.load(tmp_path / "boot1.npy", allow_pickle=True).item()
    assert r0["id"] is not None and r0["id"] == r1["id"]  # rank 0's NCCL id, intact on rank 1
    assert r0["args"] == (2, 0, 3000) and r1["args"] == (2, 1, 3000)
    for r in (r0, r1):
        assert r["outcome"] == f"comm-error-{r['code_cuda']}"  # no CUDA device in this container


def test_communicator_bootstrap_with_an_absent_rank(tmp_path):
    mp.start_processes(_boot, args=(2, _free_port(), str(tmp_path), 1), nprocs=2, join=True, start_method="spawn")
    r0 = np.load(tmp_path / "boot0.npy", allow_pickle=True).item()
    assert r0["outcome"].startswith("group-error")
    assert r0["id"] is None and r0["elapsed"] < 60


def _peers(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from nsrl_b200 import train as T
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    pc = T.PeerCheck(timeout_ms=2000, namespace="test")
    outcome = []
    for step in range(3):
        if rank == 1 and step == 2:
            break  # rank 1 leaves between steps
        t0 = time.time()
        try:
            pc.wait()
            outcome.append(("ok", time.time() - t0))
        except T.CommError as e:
            outcome.append((f"comm-error-{e.code}: {e}", time.time() - t0))
            break
    np.save(os.path.join(out_dir, f"peers{rank}.npy"), np.array(outcome, dtype=object), allow_pickle=True)
    if rank == 0:
        time.sleep(0.5)  # keep the store (served by rank 0) up until rank 1 has saved


def test_peer_check_notices_a_rank_that_left(tmp_path):
    """Both ranks pass two steps; rank 1 then leaves and rank 0's check for the
    third step fails with NSRL_COMM_ERROR after its 2 s limit, before anything
    of that step would be launched."""
    mp.start_processes(_peers, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0 = list(np.load(tmp_path / "peers0.npy", allow_pickle=True))
    r1 = list(np.load(tmp_path / "peers1.npy", allow_pickle=True))
    assert [o[0] for o in r1] == ["ok", "ok"]
    assert [o[0] for o in r0[:2]] == ["ok", "ok"]
    assert r0[2][0].startswith("comm-error-5") and "[1]" in r0[2][0]
    assert 1.5 < r0[2][1] < 30
