"""Byte generation on the GPU against the oracle's generate_mini_transformer
(nsrl-train/src/lib.rs:12702-12800), token for token: greedy and seeded top-k
sampling, prompts shorter and longer than the window, with and without RMS
norm and learned positions; and the byte-head rows of single windows."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

from train_models import random_model

pytestmark = pytest.mark.gpu


def _live_head(m, shift):
    """A head scale that keeps the byte logits unsaturated (a live softmax)."""
    m.head = O.Linear(m.head.weights, O.scales(1, shift, 256))
    return m


def _gpu(m):
    from test_gpu_train_step import to_gpu
    return to_gpu(m)


@pytest.mark.parametrize("rms,pos,heads", [(True, True, 1), (False, True, 4), (True, False, 1)])
def test_output_rows_match_the_oracle(rms, pos, heads):
    from nsrl_b200 import generate as G
    d, F, L, S, B = 64, 128, 2, 32, 5
    m = _live_head(random_model(d, heads, F, L, S, rms=rms, positions=pos, seed=70 + heads), 14)
    win = np.random.default_rng(5).integers(0, 256, (B, S)).astype(np.uint8)
    ref = O.output_rows(m, win, threads=4)
    got = G.output_rows(_gpu(m), torch.from_numpy(win))
    assert ref is not None and got is not None
    assert np.array_equal(got[0].cpu().numpy(), ref[0]) and np.array_equal(got[1].cpu().numpy(), ref[1])
    assert len(np.unique(ref[0])) > 16  # the logits are live, not one saturated value


@pytest.mark.parametrize("strategy,top_k,seed", [("greedy", 0, 0), ("sample", 0, 11), ("sample", 8, 12345)])
def test_generation_token_for_token(strategy, top_k, seed):
    from nsrl_b200 import generate as G
    d, H, F, L, S, steps = 64, 1, 128, 2, 16, 24
    m = _live_head(random_model(d, H, F, L, S, rms=True, positions=True, seed=90), 14)
    prompts = [b"to be or not to be", b"x", b"the question is whether", b"0123456789abcdefghij"]
    gen = G.Generator(_gpu(m), len(prompts), max(len(p) for p in prompts), steps)
    got = gen(prompts, strategy, top_k, seed)
    assert got is not None
    for b, p in enumerate(prompts):
        ref = O.generate(m, p, steps, strategy, top_k, seed)
        assert ref is not None
        assert np.array_equal(got[0][b].numpy(), ref[0]), (b, got[0][b].tolist(), ref[0].tolist())
        assert np.array_equal(got[1][b].numpy(), ref[1]) and np.array_equal(got[2][b].numpy(), ref[2])


def test_generation_on_the_training_model_shape():
    """The 4-layer d256 seq-512 model of the training workload: a prompt longer
    than the window and a short one, 4 sampled bytes each."""
    from nsrl_b200 import generate as G
    from nsrl_b200 import synth as Y
    tw = Y.TrainWeights(seed=4040, layers=4, d=256, hidden=1024, seq_len=512)
    layers = []
    for bw in tw.blocks:
        e = {n: O.Linear(getattr(bw, n), O.scales(1, bw.shift[n], bw.out_dim(n))) for n in O.LAYER_LINEARS}
        e["attn_gamma"], e["mlp_gamma"] = bw.attn_gamma, bw.mlp_gamma
        layers.append(e)
    m = O.TrainModel(tw.embeddings, tw.positions, layers, O.Linear(tw.head, O.scales(1, 15, 256)), 256, 4, 1024, 512)
    rng = np.random.default_rng(3)
    prompts = [bytes(rng.integers(32, 127, n).astype(np.uint8)) for n in (600, 3)]
    steps = 4
    gen = G.Generator(_gpu(m), len(prompts), 600, steps)
    got = gen(prompts, "sample", 40, 7)
    assert got is not None
    for b, p in enumerate(prompts):
        ref = O.generate(m, p, steps, "sample", 40, 7)
        assert np.array_equal(got[0][b].numpy(), ref[0]), b
