"""The head-sharded forward on real GPUs, one process per rank: exchange
buffers shared by CUDA IPC, the q|k|v and context rows crossing NVLink as
peer stores from the kernels' epilogues, device-side signals between the
phases.  Two blocks in a row (the second reuses the exchange buffers and the
epochs) must equal the oracle's blocks bit for bit on every rank, with the
whole blocks' saturation counts.  Skipped with fewer GPUs than ranks."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from nsrl_b200 import synth as Y
from oracle import oracle as O

pytestmark = pytest.mark.gpu

B, S, D, F = 2, 256, 512, 1024
H = D // 64


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights():
    return [Y.BlockWeights(400 + i, D, F) for i in range(2)]


def _rank(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from nsrl_b200 import core, shard
    blocks = []
    for bw in _weights():
        L = {nm: core.Linear(torch.from_numpy(getattr(bw, nm)).cuda(), core.make_scales(1, bw.shift[nm],
                                                                                           bw.out_dim(nm)))
             for nm in ("q", "k", "v", "o", "up", "gate", "down")}
        blocks.append(core.TransformerBlock(D, H, F, *[L[n] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                                            torch.from_numpy(bw.attn_gamma).cuda(),
                                            torch.from_numpy(bw.mlp_gamma).cuda(), 1))
    x = Y.q15_gaussian(17, (B * S, D))
    x[7] = 32767
    cur = shard.split_positions(torch.from_numpy(x).cuda(), B, S, world, rank)
    g = shard.ShardGroup(B, S, D, H, timeout_ms=20000)
    out = []
    try:
        for tb in blocks:
            r = g.forward(tb, cur)
            if r is None:
                out.append(None)
                break
            cur = r[0]
            out.append((r[1], r[2]))
    finally:
        g.close()
    res = {"y": cur.cpu().numpy(), "sat": out}
    np.save(os.path.join(out_dir, f"shard{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_blocks_across_gpus(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    cur = Y.q15_gaussian(17, (B * S, D))
    cur[7] = 32767
    sats = []
    for bw in _weights():
        L = {nm: O.Linear(getattr(bw, nm), O.scales(1, bw.shift[nm], bw.out_dim(nm)))
             for nm in ("q", "k", "v", "o", "up", "gate", "down")}
        y1, s1 = O.prenorm_attention_block(cur, B, S, D, H, bw.attn_gamma, 1, L["q"], L["k"], L["v"], L["o"],
                                           threads=8)
        cur, s2 = O.prenorm_mlp_block(y1, B * S, D, F, bw.mlp_gamma, 1, L["up"], L["gate"], L["down"], threads=8)
        sats.append((s1, s2))
    sl = S // world
    for r in range(world):
        got = np.load(tmp_path / f"shard{r}.npy", allow_pickle=True).item()
        assert got["sat"] == sats
        want = cur.reshape(B, S, D)[:, r * sl:(r + 1) * sl].reshape(-1, D)
        assert np.array_equal(got["y"], want)
