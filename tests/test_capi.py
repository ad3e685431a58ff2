"""CPU-side checks of the C ABI: the library builds, loads without a GPU and
exports every entry point include/nsrl_b200.h declares; host-side shape
validation answers like the reference's `None` without touching a device."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nsrl_b200.h")


@pytest.fixture(scope="module")
def lib():
    from nsrl_b200 import build
    path = build.build()
    return C.CDLL(path)


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(nsrl_[a-z0-9_]+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared()
    for n in ("nsrl_linear_i16_i8_i16", "nsrl_rms_norm_rows", "nsrl_self_attention",
              "nsrl_prenorm_attention_residual_block", "nsrl_prenorm_gated_mlp_residual_block",
              "nsrl_prenorm_transformer_block", "nsrl_attention_decode", "nsrl_status_fetch",
              "nsrl_linear_backward_input", "nsrl_gated_mlp_backward_input", "nsrl_rms_norm_backward_rows",
              "nsrl_attention_with_probabilities", "nsrl_attention_backward", "nsrl_train_windows",
              "nsrl_accumulate_weight_gradient_i16", "nsrl_apply_embedding_gradient_i64_to_i16",
              "nsrl_prenorm_transformer_block_host"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_workspace_sizes_are_consistent(lib):
    lib.nsrl_linear_workspace_size.restype = C.c_size_t
    lib.nsrl_linear_workspace_size.argtypes = [C.c_size_t] * 3
    lib.nsrl_transformer_block_workspace_size.restype = C.c_size_t
    lib.nsrl_transformer_block_workspace_size.argtypes = [C.c_size_t] * 5
    lib.nsrl_attention_workspace_size.restype = C.c_size_t
    lib.nsrl_attention_workspace_size.argtypes = [C.c_size_t] * 4
    # planes (2 bytes / element) + 8 bytes of row L1, each 256-byte aligned
    assert lib.nsrl_linear_workspace_size(4096, 1024, 1024) == 2 * 4096 * 1024 + 4096 * 8
    T, d, H, F = 64 * 1024, 256, 4, 1024
    a = lib.nsrl_attention_workspace_size(64, 1024, d, H)
    # + transposed V planes (2 bytes / element) for the tensor-core attention (head_dim 64)
    # + its weight scratch: 128-row query tiles x 64-key-padded rows of int16 per (sequence, head)
    S, B = 1024, 64
    assert a == T * d * 2 + T * 8 + T * 3 * d * 2 + T * d * 2 + T * 8 + T * d * 2 + B * H * S * S * 2
    assert lib.nsrl_transformer_block_workspace_size(64, 1024, d, H, F) >= a + T * d * 2


class LinearParamsC(C.Structure):
    _fields_ = [("weights", C.c_void_p), ("bias", C.c_void_p), ("scales", C.c_void_p),
                ("input_dim", C.c_size_t), ("output_dim", C.c_size_t)]


def test_shape_validation_matches_reference_none(lib):
    """Shape errors are caught on the host (NSRL_INVALID_SHAPE = 1) before any launch."""
    f = lib.nsrl_self_attention
    lp = C.POINTER(LinearParamsC)
    f.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, lp, lp, lp, lp, C.c_void_p,
                  C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
    dummy = C.c_void_p(16)
    good = LinearParamsC(16, None, 16, 128, 128)
    # head_dim 32 (128 / 4) is not a power of four: attention.rs:1599-1602
    r = f(dummy, 1, 8, 128, 4, 1, C.byref(good), C.byref(good), C.byref(good), C.byref(good), dummy, dummy, 1 << 30,
          dummy, None)
    assert r == 1
    # seq_len 0: attention.rs:1591-1593
    r = f(dummy, 1, 0, 128, 2, 1, C.byref(good), C.byref(good), C.byref(good), C.byref(good), dummy, dummy, 1 << 30,
          dummy, None)
    assert r == 1
    # q with the wrong output dim
    bad = LinearParamsC(16, None, 16, 128, 64)
    r = f(dummy, 1, 8, 128, 2, 1, C.byref(bad), C.byref(good), C.byref(good), C.byref(good), dummy, dummy, 1 << 30,
          dummy, None)
    assert r == 1
    lib.nsrl_last_error.restype = C.c_char_p
    assert b"invalid shape" in lib.nsrl_last_error()


def test_training_step_shape_rules(lib):
    """nsrl_train_windows validates the model on the host (no launch): head_dim a
    power of four and 16 or 64, RMS gammas in every layer or none, [256][d] head."""
    from nsrl_b200.core import LinearParamsC as LP
    from nsrl_b200.train import _TrainLayerC, _TrainModelC
    lib.nsrl_train_workspace_size.restype = C.c_size_t
    lib.nsrl_train_workspace_size.argtypes = [C.c_void_p, C.c_size_t]
    lib.nsrl_train_arena_len.restype = C.c_size_t
    lib.nsrl_train_arena_len.argtypes = [C.c_void_p]

    def model(d, H, F, L, S, gammas=(True, True)):
        arr = (_TrainLayerC * L)()
        for i in range(L):
            arr[i].attn_gamma = 16 if gammas[0] else None
            arr[i].mlp_gamma = 16 if gammas[1] else None
            dims = [(d, d)] * 4 + [(d, F), (d, F), (F, d)]
            for j, (inp, out) in enumerate(dims):
                arr[i].lin[j] = LP(16, None, 16, inp, out)
        m = _TrainModelC(d, H, F, L, S, 16, 16, C.cast(arr, C.c_void_p), LP(16, None, 16, d, 256))
        m._keep = arr
        return m

    good = model(256, 4, 1024, 4, 512)
    assert lib.nsrl_train_workspace_size(C.byref(good), 256) > 0
    # arena: head, per layer 4 d^2 + 3 d F + 2 d, embeddings, positions
    assert lib.nsrl_train_arena_len(C.byref(good)) == 256 * 256 + 4 * (4 * 65536 + 3 * 262144 + 512) + 65536 + 512 * 256
    for bad in (model(128, 4, 256, 2, 8),            # head_dim 32: not a power of four
                model(256, 1, 1024, 2, 8),           # head_dim 256: not taken by the training step
                model(64, 4, 128, 2, 8, (True, False))):  # RMS gammas: both or neither
        assert lib.nsrl_train_workspace_size(C.byref(bad), 4) == 0


def test_integer_adam_config_rules(lib):
    """IntegerAdamConfig::is_valid (nsrl-train-core/src/lib.rs:299-309) is checked on the host."""
    from nsrl_b200.train import IntegerAdamConfigC
    f = lib.nsrl_apply_integer_adam_i64_to_i8
    f.argtypes = [C.c_void_p] * 4 + [C.POINTER(IntegerAdamConfigC)] + [C.c_void_p] * 7
    f.argtypes[3] = C.c_size_t
    p = C.c_void_p(16)
    for bad in (IntegerAdamConfigC(learning_rate=0), IntegerAdamConfigC(beta1_decay_shift=0),
                IntegerAdamConfigC(beta2_decay_shift=63), IntegerAdamConfigC(step_shift=48),
                IntegerAdamConfigC(epsilon=0)):
        assert f(p, p, p, 4, C.byref(bad), p, p, p, p, p, p, None) == 1
