"""The allocation-free column-sum entry point, called through its C symbol.

``msb_colsum_noalloc`` serves callers that cannot allocate device memory
when they run the operation (a runtime that fixes all device memory at
start-up, code living under another framework's allocator, or a caller
that only has a C ABI and device pointers it already owns).  Its scratch is
a fixed array inside the library.  This test calls it twice in a row (the
array keeps the previous call's contents) and compares each result with the
library's regular column-sum path.  It lives in its own file, collected
last, so a run that stops at the first failure has run every other test.
"""

import ctypes

import pytest
import torch

from minispeed_b200.ops import _ext

pytestmark = pytest.mark.gpu

DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _symbol():
    lib = ctypes.CDLL(_ext.get().__file__)
    fn = lib.msb_colsum_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_longlong,
                   ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    return fn


def _regular(a2d: torch.Tensor, out: torch.Tensor, accumulate: bool) -> None:
    C = _ext.get()
    part = torch.empty(256 * a2d.shape[1], dtype=torch.float32, device=a2d.device)
    nb = C.colsum_partial(a2d, part, 256)
    C.colsum_finish(part, nb, out, accumulate)


def _tol(dtype):
    return {torch.float32: (1e-5, 1e-4), torch.float16: (2e-3, 2e-2),
            torch.bfloat16: (1.6e-2, 1e-1)}[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_noalloc_colsum_matches_regular_path_twice(dtype):
    fn = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    shapes = [(4096, 768), (1000, 3072 + 8)]        # two different calls back to back
    for M, N in shapes:
        torch.manual_seed(M + N)
        buf = torch.randn(M, N + 8, device="cuda").to(dtype)
        a = buf[:, :N]                               # padded row stride
        init = torch.randn(N, device="cuda").to(dtype)
        for accumulate in (0, 1):
            got = init.clone()
            rc = fn(a.data_ptr(), DTYPE[dtype], M, N, a.stride(0), got.data_ptr(), accumulate,
                    stream)
            assert rc == 0
            want = init.clone()
            _regular(a, want, bool(accumulate))
            torch.cuda.synchronize()
            rtol, atol = _tol(dtype)
            torch.testing.assert_close(got.float(), want.float(), rtol=rtol, atol=atol)
            ref = a.float().sum(0) + (init.float() if accumulate else 0)
            torch.testing.assert_close(got.float(), ref, rtol=rtol, atol=atol * 4)


def test_noalloc_colsum_rejects_too_wide_input():
    fn = _symbol()
    a = torch.zeros(2, 8, device="cuda")
    out = torch.zeros(8, device="cuda")
    # N beyond the scratch capacity is refused before any launch
    rc = fn(a.data_ptr(), 0, 1, (1 << 20) + 1, (1 << 20) + 1, out.data_ptr(), 0,
            torch.cuda.current_stream().cuda_stream)
    assert rc == -2
    rc = fn(a.data_ptr(), 0, 2, 8, 4, out.data_ptr(), 0, None)   # ld < N
    assert rc == -1
