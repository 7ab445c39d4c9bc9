"""The allocation-free small-M GEMM entry point, called through its exported
C symbol the way a caller that cannot allocate device memory would call it
(for example a host framework that owns every allocation, or a real-time path
that may not enter the allocator): its output must match the regular entry
point's, which uses caller-allocated scratch, on two calls in a row (the
second call reuses the library's static scratch left by the first)."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = -8


def _lib():
    from sglang_legolink_b200 import ops
    from sglang_legolink_b200.ops import _ext

    ops._cuda()  # loads the extension (and torch's CUDA libraries it links against)
    lib = ctypes.CDLL(_ext.so_path("legolink_cuda"))
    fn = lib.ll_gemm_bf16_small_m_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    msg = lib.ll_gemm_small_m_noalloc_error_string
    msg.restype = ctypes.c_char_p
    msg.argtypes = [ctypes.c_int]
    return fn, msg


def _call(fn, a, w, bias, out, err):
    return fn(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
              bias.data_ptr() if bias is not None else None, a.shape[0], w.shape[0], a.shape[1], err.data_ptr(),
              torch.cuda.current_stream().cuda_stream)


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-6)).item()


@pytest.mark.parametrize("M,N,K", [(1, 4608, 3584), (16, 3584, 18944), (5, 1000, 512)])
def test_no_alloc_matches_regular_entry_point_twice(M, N, K):
    from sglang_legolink_b200 import ops

    fn, msg = _lib()
    torch.manual_seed(11)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call in range(2):
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
        bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
        got = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        rc = _call(fn, a, w, bias, got, err)
        assert rc == 0, msg(rc).decode()
        exp = torch.empty_like(got)
        ops._small_m(ops._cuda(), ops.workspace("cuda"), a, w, bias, exp)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert _rel(got, exp) < 1e-2, call
        assert _rel(got, a.float() @ w.float().t() + bias.float()) < 1e-2, call


def test_warm_call_takes_no_device_memory():
    """After the one-time set-up call on a device, a call leaves the
    device's free memory unchanged (cudaMemGetInfo before and after)."""
    fn, msg = _lib()
    M, N, K = 16, 3584, 18944
    torch.manual_seed(3)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call(fn, a, w, None, out, err) == 0  # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        rc = _call(fn, a, w, None, out, err)
        assert rc == 0, msg(rc).decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert int(err.item()) == 0


def test_no_alloc_rejects_problems_beyond_its_scratch():
    fn, msg = _lib()
    M, N, K = 128, 3584, 18944  # split-K partials far above the static scratch
    a = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), 7.0, device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _call(fn, a, w, None, out, err)
    assert rc == TOO_LARGE
    assert b"static scratch" in msg(rc)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
