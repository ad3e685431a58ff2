"""The allocation-free linear (nsrl_linear_i16_i8_i16_noalloc) against the
workspace linear (nsrl_linear_i16_i8_i16).

Some callers of this library cannot allocate device memory: shims that keep
nsrl-core's workspace-free signature, and host paths where cudaMalloc /
cudaFree are not allowed because they can synchronise the device or exceed a
budget owned by another allocator.  The no-alloc entry point serves them from
a static device scratch array.  This test calls it through the C ABI twice in
a row, with different shapes, and requires the output to match the workspace
entry point bit for bit (integer path: tolerance 0), and both to match the
oracle.  It also checks that a
shape beyond the scratch is rejected.  It runs last (file name) and passes
both alone and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _call_noalloc(core, x, lin):
    L = core.lib()
    f = L.nsrl_linear_i16_i8_i16_noalloc
    f.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(core.LinearParamsC), C.c_void_p, C.c_void_p, C.c_void_p]
    rows = x.numel() // lin.input_dim
    y = torch.full((rows, lin.output_dim), -7, dtype=torch.int16, device=x.device)
    st = core.Status()
    p = lin.c()
    r = f(C.c_void_p(x.data_ptr()), rows, C.byref(p), C.c_void_p(y.data_ptr()), C.c_void_p(st.buf.data_ptr()),
          C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return r, y, st


def test_noalloc_linear_matches_workspace_linear_on_two_calls():
    from nsrl_b200 import build, core, synth as Y
    build.build()
    torch.cuda.set_device(0)
    cases = [(512, 1024, 384, True), (1000, 256, 256, False)]  # prefix check on / off
    for M, K, N, with_bias in cases:
        x_np = Y.q15_gaussian(3 + M, (M, K))
        w_np = Y.i8_uniform(4 + N, (N, K))
        x = torch.from_numpy(x_np).cuda()
        bias = torch.arange(N, dtype=torch.int32) * 37 - 5000 if with_bias else None
        lin = core.Linear(torch.from_numpy(w_np), core.make_scales(1, Y.shift_for(K), N), bias)
        ref = core.linear_i16_i8_i16_per_channel_checked(x, lin)
        assert ref is not None
        r, y, st = _call_noalloc(core, x, lin)
        assert r == core.NSRL_OK, core.lib().nsrl_last_error()
        code, _ = st.fetch()
        assert code == core.NSRL_OK
        assert torch.equal(y, ref)
        oref = O.linear(x_np, O.Linear(w_np, O.scales(1, Y.shift_for(K), N),
                                       None if bias is None else bias.numpy()))
        assert oref is not None and np.array_equal(y.cpu().numpy(), oref)


def test_noalloc_linear_rejects_shapes_beyond_its_scratch():
    from nsrl_b200 import build, core
    build.build()
    L = core.lib()
    L.nsrl_linear_noalloc_scratch_bytes.restype = C.c_size_t
    cap = L.nsrl_linear_noalloc_scratch_bytes()
    K = 1024
    rows = cap // (2 * K) + 1  # needs more than the static scratch
    lin = core.Linear(torch.ones((16, K), dtype=torch.int8), core.make_scales(1, 10, 16))
    x = torch.zeros((rows, K), dtype=torch.int16, device="cuda")
    r, _, _ = _call_noalloc(core, x, lin)
    assert r == core.NSRL_INVALID_SHAPE
    assert b"static scratch" in L.nsrl_last_error()
