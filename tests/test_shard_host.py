"""Host side of the head-sharded forward, without a GPU.

- The exchange-buffer layout: a restatement of its regions against
  nsrl_shard_exchange_bytes, and the shapes that do not split.
- ShardGroup's set-up over two gloo ranks with a fake library: every rank
  gets the others' IPC handles intact, opens them, and hands the group its
  own buffer at its own index and the opened ones at theirs; close() undoes
  all of it.
- The split itself over two gloo ranks on the oracle: positions owned by
  rank for the token-wise work, heads owned by rank for attention, the q|k|v
  and context rows exchanged between them.  The joined rows equal the
  oracle's unsplit transformer block, which shows the split reorders work
  without changing a value.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _al(v):
    return (v + 255) // 256 * 256


def _layout_bytes(B, S, d, H, n):
    if n < 1 or n > 8 or S % n or H % n or d % H:
        return 0
    sl, dl = S // n, d // n
    off = 4096
    for size in (B * S * 2 * dl, B * S * 2 * dl, B * dl * S, B * dl * S, B * sl * d, B * sl * d, 8 * B * sl):
        off = _al(off + size)
    if n > 1 and sl % 16 == 0:  # one staging slot per destination rank: q|k hi, lo and v hi, lo
        off += n * (2 * _al(B * S * 2 * dl) + 2 * _al(B * dl * S))
    return off


@pytest.mark.parametrize("B,S,d,H,n", [(1, 128, 256, 4, 2), (3, 96, 128, 2, 2), (2, 1024, 512, 8, 8),
                                       (1, 48, 192, 3, 3), (64, 1024, 256, 4, 4), (1, 100, 256, 4, 3),
                                       (1, 128, 256, 4, 8), (1, 128, 256, 4, 0), (1, 144, 576, 9, 9)])
def test_exchange_layout(B, S, d, H, n):
    from nsrl_b200 import build, shard
    build.build()
    assert shard.LibraryApi().exchange_bytes(B, S, d, H, n) == _layout_bytes(B, S, d, H, n)


def test_positions_and_heads():
    from nsrl_b200 import shard
    assert [shard.positions(1024, 4, r) for r in range(4)] == [(0, 256), (256, 512), (512, 768), (768, 1024)]
    assert [shard.heads(8, 2, r) for r in range(2)] == [(0, 4), (4, 8)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class FakeApi:
    """Stands in for the exchange-buffer calls: pointers and handles derived
    from the rank, every call recorded."""

    def __init__(self, rank):
        self.rank, self.calls = rank, []

    def exchange_bytes(self, *shape):
        self.calls.append(("bytes", shape))
        return 1 << 20

    def alloc(self, nbytes):
        self.calls.append(("alloc", nbytes))
        return 0x1000_0000 * (self.rank + 1)

    def free(self, ptr):
        self.calls.append(("free", ptr))

    def handle(self, ptr):
        return bytes([self.rank + 1]) * 32 + ptr.to_bytes(32, "little")

    def open(self, h):
        self.calls.append(("open", h))
        return 0x7000_0000 + h[0]

    def close(self, ptr):
        self.calls.append(("close", ptr))

    def create(self, nranks, rank, buffers, nbytes, *rest):
        self.calls.append(("create", nranks, rank, list(buffers), nbytes, rest))
        return 0xABC0 + rank

    def destroy(self, g):
        self.calls.append(("destroy", g))

    def synchronize(self):
        self.calls.append(("sync",))


def _setup(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from nsrl_b200 import shard
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    api = FakeApi(rank)
    g = shard.ShardGroup(2, 256, 256, 4, timeout_ms=1234, api=api)
    res = {"g": g.g, "nranks": g.nranks, "rank": g.rank, "rows": g.rows}
    g.close()
    res["calls"] = api.calls
    np.save(os.path.join(out_dir, f"setup{rank}.npy"), np.array(res, dtype=object), allow_pickle=True)
    dist.destroy_process_group()


def test_group_setup_over_gloo(tmp_path):
    mp.start_processes(_setup, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for rank in (0, 1):
        r = np.load(tmp_path / f"setup{rank}.npy", allow_pickle=True).item()
        other = 1 - rank
        own, peer = 0x1000_0000 * (rank + 1), 0x7000_0000 + other + 1
        assert (r["g"], r["nranks"], r["rank"], r["rows"]) == (0xABC0 + rank, 2, rank, 2 * 256 // 2)
        calls = r["calls"]
        assert calls[0] == ("bytes", (2, 256, 256, 4, 2))
        opened = [c for c in calls if c[0] == "open"]
        assert opened == [("open", bytes([other + 1]) * 32 + (0x1000_0000 * (other + 1)).to_bytes(32, "little"))]
        create = [c for c in calls if c[0] == "create"][0]
        bufs = [own, peer] if rank == 0 else [peer, own]
        assert create[1:5] == (2, rank, bufs, 1 << 20) and create[5] == (2, 256, 256, 4, 1234)
        tail = [c for c in calls if c[0] in ("sync", "destroy", "close", "free")]
        assert tail == [("sync",), ("destroy", 0xABC0 + rank), ("close", peer), ("free", own)]


def _flow(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    from nsrl_b200 import synth as Y
    from oracle import oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    B, S, d, H, F = 2, 32, 128, 2, 256
    hd, n = d // H, world
    sl, hl = S // n, H // n
    bw = Y.BlockWeights(21, d, F)
    L = {nm: O.Linear(getattr(bw, nm), O.scales(1, bw.shift[nm], bw.out_dim(nm)))
         for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    x = Y.q15_gaussian(5, (B * S, d))
    x[3] = 32767
    xl = x.reshape(B, S, d)[:, rank * sl:(rank + 1) * sl].reshape(-1, d)

    def gather(a):  # int16 rows, carried as int32 (gloo has no int16 all-gather)
        parts = [torch.zeros(a.shape, dtype=torch.int32) for _ in range(n)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)))
        return [p.numpy().astype(np.int16) for p in parts]

    # token-wise: norm and Q|K|V of this rank's positions
    nrm = O.rms_norm_rows(xl, bw.attn_gamma, 1)
    qkv = np.concatenate([O.linear(nrm, L[nm]) for nm in "qkv"], axis=1)  # [B*sl][3d]
    # exchange: every rank's positions, then this rank's heads
    full = np.concatenate([p.reshape(B, sl, 3 * d) for p in gather(qkv)], axis=1)  # [B][S][3d]
    ctx = np.zeros((B, S, hl * hd), np.int16)
    for b in range(B):
        for j in range(hl):
            c0 = (rank * hl + j) * hd
            for t in range(S):
                r = O.attention_row(full[b, t, c0:c0 + hd], full[b, :t + 1, d + c0:d + c0 + hd],
                                    full[b, :t + 1, 2 * d + c0:2 * d + c0 + hd], hd, hd)
                ctx[b, t, j * hd:(j + 1) * hd] = r[0]
    # exchange back: this rank's positions, every rank's heads
    parts = gather(ctx)
    mine = np.concatenate([p[:, rank * sl:(rank + 1) * sl] for p in parts], axis=2).reshape(-1, d)
    h, s1 = O.residual_add(xl, O.linear(mine, L["o"]))
    y, s2 = O.prenorm_mlp_block(h, B * sl, d, F, bw.mlp_gamma, 1, L["up"], L["gate"], L["down"])
    ys = gather(y)
    t = torch.tensor([s1, s2], dtype=torch.int64)
    dist.all_reduce(t)
    if rank == 0:
        got = np.concatenate([p.reshape(B, sl, d) for p in ys], axis=1).reshape(-1, d)
        y1, r1 = O.prenorm_attention_block(x, B, S, d, H, bw.attn_gamma, 1, L["q"], L["k"], L["v"], L["o"])
        ref, r2 = O.prenorm_mlp_block(y1, B * S, d, F, bw.mlp_gamma, 1, L["up"], L["gate"], L["down"])
        res = {"equal": bool(np.array_equal(got, ref)), "sat": t.tolist(), "ref_sat": [r1, r2]}
        np.save(os.path.join(out_dir, "flow.npy"), np.array(res, dtype=object), allow_pickle=True)
    dist.destroy_process_group()


def test_split_reproduces_the_block_over_gloo(tmp_path):
    mp.start_processes(_flow, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r = np.load(tmp_path / "flow.npy", allow_pickle=True).item()
    assert r["equal"]
    assert r["sat"] == r["ref_sat"] and r["sat"][0] > 0
