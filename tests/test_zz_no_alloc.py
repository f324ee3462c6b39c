"""The allocation-free column-sum entry point, called through its exported C
symbol, against the regular entry point (dlvk::colsum via the PyTorch
binding).

Callers that cannot allocate device memory at call time (strict memory
budgets, plugins inside a runtime that owns device memory, latency-critical
threads) use `dlvk_colsum_noalloc`; this test checks it computes the same
sums, twice in a row on the shared static scratch array, and that it
allocates nothing through PyTorch.  The file name sorts last so that a run
that stops at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, BAD_ARG, TOO_LARGE = 0, 1, 2
MAX_COLS = (1 << 20) // 64


def _lib():
    from dlvk_b200 import _ext

    mod = _ext.C()
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.dlvk_colsum_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_void_p]
    msg = lib.dlvk_noalloc_error_string
    msg.restype = ctypes.c_char_p
    msg.argtypes = [ctypes.c_int]
    return mod, fn, msg


def _call(fn, x, out, scale, accumulate):
    code = 0 if x.dtype == torch.float32 else 1
    stream = torch.cuda.current_stream().cuda_stream
    return fn(x.data_ptr(), code, x.shape[0], x.shape[1], scale, out.data_ptr(), int(accumulate), stream)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(8192, 4096), (300, 1000), (70000, 129)])
def test_noalloc_colsum_matches_regular_entry_point(dtype, rows, cols):
    mod, fn, msg = _lib()
    torch.manual_seed(rows + cols)
    out = torch.zeros(cols, device="cuda")
    xs = [torch.randn(rows, cols, device="cuda").to(dtype) for _ in range(2)]
    # two calls in a row: the second reuses the scratch the first left behind
    for x in xs:
        torch.cuda.synchronize()
        # cumulative count of PyTorch device allocations: must not move
        before = torch.cuda.memory_stats()["allocation.all.allocated"]
        rc = _call(fn, x, out, 0.5, accumulate=False)
        assert rc == OK, msg(rc)
        torch.cuda.synchronize()
        assert torch.cuda.memory_stats()["allocation.all.allocated"] == before
        ref = mod.colsum(x, 0.5)
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-4)
        # and against an independent fp64 sum, which shares no code with either
        exact = (x.double().sum(0) * 0.5).float()
        torch.testing.assert_close(out, exact, rtol=1e-5, atol=1e-3)
    # accumulate mode against the regular entry point's accumulate mode
    acc0 = torch.randn(cols, device="cuda")
    acc_ref = acc0.clone()
    acc = acc0.clone()
    assert _call(fn, xs[0], acc, 1.0, accumulate=True) == OK
    mod.colsum(xs[0], 1.0, out=acc_ref, accumulate=True)
    torch.testing.assert_close(acc, acc_ref, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(acc, (acc0.double() + xs[0].double().sum(0)).float(), rtol=1e-5, atol=2e-3)


def test_noalloc_colsum_rejects_too_many_columns():
    mod, fn, msg = _lib()
    x = torch.zeros(4, MAX_COLS + 1, device="cuda")
    out = torch.zeros(MAX_COLS + 1, device="cuda")
    rc = _call(fn, x, out, 1.0, False)
    assert rc == TOO_LARGE
    assert b"16384" in msg(rc)
    assert fn(None, 0, 4, 4, 1.0, None, 0, None) == BAD_ARG
