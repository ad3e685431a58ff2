"""The head-sharded forward (nsrl_sharded_* through the C ABI) with n ranks
emulated on one GPU: every rank's exchange buffer is a local allocation and
each phase runs for all ranks before the next.  The joined rows equal the
one-GPU block and the oracle bit for bit, each rank's combined status equals
the whole block's, a rejection on one rank's heads rejects every rank, and a
rank that never signals ends the others' waits with a timeout status."""
import numpy as np
import pytest

from nsrl_b200 import synth as Y
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def mods():
    from nsrl_b200 import build, core, shard
    build.build()
    return core, shard


def _block(core, d, F, seed, qk_extra=7):
    from test_gpu_parity import lin_pair
    bw = Y.BlockWeights(seed, d, F, qk_extra_shift=qk_extra)
    P = {nm: lin_pair(core, getattr(bw, nm), bw.shift[nm]) for nm in ("q", "k", "v", "o", "up", "gate", "down")}
    tb = core.TransformerBlock(d, d // 64, F, *[P[n][1] for n in ("q", "k", "v", "o", "up", "gate", "down")],
                               torch.from_numpy(bw.attn_gamma).cuda(), torch.from_numpy(bw.mlp_gamma).cuda(), 1)
    return bw, P, tb


@pytest.mark.parametrize("n,B,S,d,F,mlp", [
    (2, 2, 256, 256, 1024, True),   # the benchmark block's widths, two ranks
    (4, 1, 512, 256, 1024, True),   # one head per rank
    (2, 3, 96, 128, 512, False),    # attention block alone, ragged query tiles per rank
    (3, 1, 48, 192, 256, True),     # d_model not a multiple of 128: SIMT Q|K|V projection
    (4, 1, 128, 1024, 512, True),   # d_model > 516: the exact prefix check reads the summed context L1
    (8, 1, 256, 512, 512, True),    # eight ranks, one head each
    (2, 2, 48, 128, 256, True),     # 24 positions per rank: peer stores from the epilogue, no staging
])
def test_sharded_block_matches_one_gpu_and_oracle(mods, n, B, S, d, F, mlp):
    core, shard = mods
    H = d // 64
    bw, P, tb = _block(core, d, F, 300 + n + d)
    x = Y.q15_gaussian(11 + S, (B * S, d))
    x[5] = 32767  # some residual saturations
    y1, s1 = O.prenorm_attention_block(x, B, S, d, H, bw.attn_gamma, 1, *[P[k][0] for k in "qkvo"], threads=8)
    ref, s2 = (O.prenorm_mlp_block(y1, B * S, d, F, bw.mlp_gamma, 1, P["up"][0], P["gate"][0], P["down"][0],
                                   threads=8) if mlp else (y1, 0))
    grp = shard.EmulatedShardGroups(n, B, S, d, H)
    try:
        out = grp.forward(tb, torch.from_numpy(x).cuda(), mlp=mlp)
    finally:
        grp.close()
    assert isinstance(out, list) and len(out) == n
    got = shard.join_positions([o[0] for o in out], B).cpu().numpy()
    assert np.array_equal(got, ref)
    for y, code, h in out:
        assert code == core.NSRL_OK and h.flags == 0
        assert h.attention_saturations == s1 and h.mlp_saturations == s2
    if mlp and n == 2:
        one = tb(torch.from_numpy(x).cuda(), B, S)
        assert one is not None and np.array_equal(one[0].cpu().numpy(), got)


def test_rejection_on_one_rank_reaches_every_rank(mods):
    """Logits of the last head leave i32 (attention.rs:139): only the rank that
    owns that head sees it, and after the status combine every rank holds the
    rejection, as the one-GPU block (a `None`) does."""
    core, shard = mods
    from test_gpu_parity import lin_pair
    B, S, d, H, F = 1, 64, 128, 2, 256
    bw, P, _ = _block(core, d, F, 9)
    wq = bw.q.copy()
    wk = bw.k.copy()
    wq[:] = 0  # head 0: zero queries, logits 0
    wk[64:] = 0
    wq[64:, :64] = np.eye(64, dtype=np.int8) * 127
    wk[64:, :64] = np.eye(64, dtype=np.int8) * 127
    Pq, Pk = lin_pair(core, wq, 0), lin_pair(core, wk, 0)
    x = np.full((B * S, d), 32767, np.int16)
    g = np.full(d, 32767, np.int16)
    assert O.prenorm_attention_block(x, B, S, d, H, g, 1, Pq[0], Pk[0], P["v"][0], P["o"][0]) is None
    tb = core.TransformerBlock(d, H, F, Pq[1], Pk[1], P["v"][1], P["o"][1], P["up"][1], P["gate"][1],
                               P["down"][1], torch.from_numpy(g).cuda(), torch.from_numpy(g).cuda(), 1)
    grp = shard.EmulatedShardGroups(2, B, S, d, H)
    try:
        out = grp.forward(tb, torch.from_numpy(x).cuda(), mlp=False)
    finally:
        grp.close()
    for _, code, h in out:
        assert code == core.NSRL_CORE_REJECTED and h.flags & 0x2


def test_rank_that_never_signals_times_out(mods):
    """Only rank 0 of two runs its phases: its waits for rank 1 give up after
    the group's timeout with the WAIT_TIMEOUT flag, the call returns, and the
    GPU stays usable."""
    core, shard = mods
    B, S, d, H, F = 1, 64, 128, 2, 256
    _, _, tb = _block(core, d, F, 4)
    x = torch.from_numpy(Y.q15_gaussian(2, (B * S, d))).cuda()
    grp = shard.EmulatedShardGroups(2, B, S, d, H, timeout_ms=100)
    try:
        out = grp.forward(tb, x, only=[0])
    finally:
        grp.close()
    (_, code, h), = out
    assert code == core.NSRL_CORE_REJECTED and h.flags & shard.FLAG_WAIT_TIMEOUT
    assert tb(x, B, S) is not None


def test_shape_rules(mods):
    core, shard = mods
    api = shard.LibraryApi()
    assert api.exchange_bytes(1, 100, 256, 4, 3) == 0       # seq_len not a multiple of the ranks
    assert api.exchange_bytes(1, 128, 256, 4, 8) == 0       # fewer heads than ranks
    assert api.exchange_bytes(1, 128, 256, 4, 9) == 0       # more than eight ranks
    with pytest.raises(core.NsrlError, match="head_dim 64"):
        shard.EmulatedShardGroups(2, 1, 64, 128, 8)         # head_dim 16
