"""The .nsrlmt model artifact (nsrl_b200.artifact) without a GPU: round
trips, the checks of MiniTransformerMlpModel::from_bytes (lib.rs:10240-10470),
and the reference's checked-in candidate model (its recorded hashes and a
byte-identical re-serialisation), when the reference checkout is present."""
import os

import numpy as np
import pytest

from nsrl_b200 import artifact as A

REF_ARTIFACT = os.environ.get(
    "NSRL_REFERENCE_ARTIFACT",
    "/root/reference/data/experiments/integer-transformer-proof-v1/candidate-default/candidate.nsrlmt")
CANDIDATE_MODEL_HASH = 0x6FFD37DE48A3121B  # candidate.eval.json / manifest of that experiment


def synthetic(d=32, H=2, F=64, S=8, L=2, rms=True, positions=True, seed=0):
    r = np.random.default_rng(seed)
    i8 = lambda *s: r.integers(-127, 128, s).astype(np.int8)
    i16 = lambda *s: r.integers(-32768, 32768, s).astype(np.int16)
    return A.MiniTransformerArtifact(d, H, F, S, i16(256, d), i16(S, d) if positions else np.zeros((0, d), np.int16),
                                     i8(L, d, d), i8(L, d, d), i8(L, d, d), i8(L, d, d), i8(L, F, d), i8(L, F, d),
                                     i8(L, d, F), i8(256, d), i16(L, d) if rms else None, i16(L, d) if rms else None)


@pytest.mark.parametrize("rms,positions,L", [(True, True, 2), (False, True, 1), (True, False, 3)])
def test_round_trip(rms, positions, L):
    a = synthetic(rms=rms, positions=positions, L=L, seed=L)
    b = A.to_bytes(a)
    c = A.from_bytes(b)
    assert A.to_bytes(c) == b
    assert c.layers == L and (c.attention_rms is not None) == rms and c.model_hash() == a.model_hash()
    assert A.serialized_model_hash(b) == a.model_hash()
    for f in ("embeddings", "positions", "q", "k", "v", "o", "up", "gate", "down", "output"):
        assert np.array_equal(getattr(a, f), getattr(c, f)), f


def test_rejections():
    b = bytearray(A.to_bytes(synthetic()))
    with pytest.raises(A.ArtifactError, match="bad magic"):
        A.from_bytes(b"XSRLMT5\n" + bytes(b[8:]))
    with pytest.raises(A.ArtifactError, match="version-4"):
        A.from_bytes(A.LEGACY_MAGIC + bytes(b[8:]))
    with pytest.raises(A.ArtifactError, match="length"):
        A.from_bytes(bytes(b[:-1]))
    with pytest.raises(A.ArtifactError, match="too short"):
        A.from_bytes(bytes(b[:100]))
    flipped = bytearray(b)
    flipped[len(b) - 5 * 2 * 32 - 10] ^= 1  # a byte of the last layer's MLP gamma... or the head
    with pytest.raises(A.ArtifactError, match="hash"):
        A.from_bytes(bytes(flipped))
    q_at = 8 + 20 + 80 + 64 + 2 * 256 * 32 + 2 * 8 * 32
    bad_q = bytearray(b)
    bad_q[q_at] ^= 0x40
    with pytest.raises(A.ArtifactError, match="attention hash"):
        A.from_bytes(bytes(bad_q))


@pytest.mark.skipif(not os.path.exists(REF_ARTIFACT), reason="the reference checkout is not present")
def test_reference_candidate_artifact():
    data = open(REF_ARTIFACT, "rb").read()
    a = A.from_bytes(data)  # every recorded hash checked
    assert (a.d_model, a.heads, a.hidden_dim, a.seq_len, a.layers) == (128, 8, 256, 64, 2)
    assert a.attention_rms is not None
    assert a.model_hash() == A.serialized_model_hash(data) == CANDIDATE_MODEL_HASH
    assert A.to_bytes(a) == data
