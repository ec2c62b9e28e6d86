"""The allocation-free C entry point of the LM-head cross-entropy forward.

``pb_lmhead_ce_forward_noalloc`` is for callers that may not allocate device memory
while they run (their device heap is owned by another runtime's pool, or their
memory budget is fixed at start-up, or cudaMalloc's synchronisation is not
acceptable in their loop).  It keeps its partial sums in a static device array.
This test calls it through its exported C symbol (ctypes) and checks it against the
regular extension op on two calls in a row, so stale scratch contents from the first
call cannot leak into the second.  It lives in its own file, collected last.
"""

import ctypes

import pytest
import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.cross_entropy import lmhead_ce_forward

pytestmark = pytest.mark.gpu


def _lib():
    lib = ctypes.CDLL(_native.module().__file__)
    f = lib.pb_lmhead_ce_forward_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.pb_noalloc_last_error.restype = ctypes.c_char_p
    lib.pb_noalloc_scratch_floats.restype = ctypes.c_long
    lib.pb_noalloc_status.restype = ctypes.c_int
    lib.pb_noalloc_status.argtypes = [ctypes.c_int]
    return lib, f


def _call(f, x, w, tgt, z, loss, lse):
    t, d = x.shape
    v = w.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return f(x.data_ptr(), w.data_ptr(), tgt.data_ptr(), t, d, v, -100, z, loss.data_ptr(), lse.data_ptr(), stream)


@pytest.mark.parametrize("shape,z", [((2048, 768, 32000), 0.0), ((1000, 256, 1000), 1e-3)])
def test_noalloc_matches_extension_op(shape, z):
    lib, f = _lib()
    t, d, v = shape
    for call in range(2):
        torch.manual_seed(call)
        x = (torch.randn(t, d, device="cuda") * 0.5).to(torch.bfloat16)
        w = (torch.randn(v, d, device="cuda") * 0.05).to(torch.bfloat16)
        tgt = torch.randint(0, v, (t,), device="cuda")
        tgt[:: 3 + call] = -100
        loss = torch.full((), float("nan"), device="cuda")
        lse = torch.full((t,), float("nan"), device="cuda")
        rc = _call(f, x, w, tgt, z, loss, lse)
        assert rc == 0, lib.pb_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert lib.pb_noalloc_status(1) == 0
        ref_loss, ref_lse = lmhead_ce_forward(x, w, tgt, -100, z)
        torch.cuda.synchronize()
        torch.testing.assert_close(lse, ref_lse, atol=1e-4, rtol=1e-5)
        torch.testing.assert_close(loss, ref_loss, atol=1e-2, rtol=1e-5)


def test_noalloc_rejects_sizes_beyond_scratch():
    lib, f = _lib()
    cap = lib.pb_noalloc_scratch_floats()
    x = torch.zeros(8, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(256, 64, device="cuda", dtype=torch.bfloat16)
    tgt = torch.zeros(8, device="cuda", dtype=torch.long)
    loss = torch.zeros((), device="cuda")
    lse = torch.zeros(8, device="cuda")
    too_many_rows = cap // 3 + 1  # (2 * ceil(256 / 256) + 1) * T > cap; checked before any memory is touched
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(x.data_ptr(), w.data_ptr(), tgt.data_ptr(), too_many_rows, 64, 256, -100, 0.0, loss.data_ptr(),
           lse.data_ptr(), stream)
    assert rc == 2
    assert "scratch" in lib.pb_noalloc_last_error().decode()


@pytest.mark.parametrize("case", ["d_not_multiple_of_8", "x_misaligned"])
def test_noalloc_rejects_bad_arguments_and_leaves_outputs(case):
    """Return code 3 for a row width that is not a whole number of 16-byte pieces and
    for an x pointer that is not 16-byte aligned; the outputs keep their contents."""
    lib, f = _lib()
    d = 60 if case == "d_not_multiple_of_8" else 64
    buf = torch.zeros(8 * d + 8, device="cuda", dtype=torch.bfloat16)
    x_ptr = buf.data_ptr() + (2 if case == "x_misaligned" else 0)
    w = torch.zeros(256, d, device="cuda", dtype=torch.bfloat16)
    tgt = torch.zeros(8, device="cuda", dtype=torch.long)
    loss = torch.full((), 123.0, device="cuda")
    lse = torch.full((8,), -7.0, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(x_ptr, w.data_ptr(), tgt.data_ptr(), 8, d, 256, -100, 0.0, loss.data_ptr(), lse.data_ptr(), stream)
    assert rc == 3, lib.pb_noalloc_last_error().decode()
    assert lib.pb_noalloc_last_error().decode()
    torch.cuda.synchronize()
    assert float(loss) == 123.0
    assert torch.equal(lse, torch.full((8,), -7.0, device="cuda"))
