"""The allocation-free loss entry point, called through its exported C symbol.

``pan2_mse_sums_noalloc`` serves callers that cannot allocate device memory (runtimes or allocators
that forbid hidden device allocations, or a C/C++ host that has no caching allocator to borrow
from): its scratch is a fixed device array inside the library.  This test calls it through ctypes twice in a
row and compares each result with the allocating ``mse_fwd`` binding.  It lives in its own file,
collected last, so a failure here never hides the results of the other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from pan2_b200.ops._ext import ext
    import pan2_b200._C as C
    ext()
    lib = ctypes.CDLL(C.__file__)
    fn = lib.pan2_mse_sums_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.pan2_noalloc_last_error
    err.restype = ctypes.c_char_p
    return fn, err


def test_noalloc_mse_matches_allocating_path_twice():
    from pan2_b200.ops._ext import ext
    fn, err = _lib()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream()
    for trial in range(2):
        rows, cols = 4096 + 512 * trial, 192
        pred = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
        tgt = torch.randn(rows, cols, device="cuda").to(torch.bfloat16)
        out = torch.full((2,), -1.0, device="cuda")
        rc = fn(pred.data_ptr(), tgt.data_ptr(), rows * cols, out.data_ptr(), stream.cuda_stream)
        assert rc == 0, err().decode()
        ref = ext().mse_fwd(pred, tgt, rows)
        torch.cuda.synchronize()
        assert out[1].item() == rows * cols
        assert abs(out[0].item() - ref[0].item()) <= 1e-4 * abs(ref[0].item()), (trial, out, ref)


@pytest.mark.parametrize("n", [0, 8, 2048 * 3 + 8, 16384 * 2048])
def test_noalloc_mse_edge_sizes(n):
    """Empty input, one partial tile, a ragged last tile and the largest size the scratch holds."""
    from pan2_b200.ops._ext import ext
    fn, err = _lib()
    torch.manual_seed(n % 97)
    pred = torch.randn(max(n, 8), device="cuda").to(torch.bfloat16)
    tgt = torch.randn(max(n, 8), device="cuda").to(torch.bfloat16)
    out = torch.full((2,), -1.0, device="cuda")
    rc = fn(pred.data_ptr(), tgt.data_ptr(), n, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, err().decode()
    torch.cuda.synchronize()
    if n == 0:
        assert out.tolist() == [0.0, 0.0]
        return
    ref = ext().mse_fwd(pred[:n].view(n // 8, 8), tgt[:n].view(n // 8, 8), n // 8)
    torch.cuda.synchronize()
    assert out[1].item() == n
    assert abs(out[0].item() - ref[0].item()) <= 1e-4 * abs(ref[0].item()), (n, out, ref)


def test_noalloc_mse_rejects_sizes_above_the_limit():
    fn, err = _lib()
    x = torch.zeros(8, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(2, device="cuda")
    rc = fn(x.data_ptr(), x.data_ptr(), 16384 * 2048 + 8, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert b"scratch limit" in err()
