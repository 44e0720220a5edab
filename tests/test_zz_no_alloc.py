"""qb_gemm_fp8_noalloc, called through its exported C symbol.

The C entry point serves callers that cannot allocate device memory (a
server that gives all of the GPU to its own pool, a C program without a
caching allocator): its scratch lives in a fixed device array inside the
library. Here its output is checked against the PyTorch-facing GEMM entry
point on two calls in a row with different shapes, so a second call that
saw stale scratch from the first would fail. This file is named to be
collected last.
"""

import ctypes
import glob
import os

import pytest
import torch

from quail_b200 import ops
from quail_b200.ops.quant import dequantize_act, dequantize_weight

pytestmark = pytest.mark.gpu

QB_NOALLOC_MAX_SCALES = ((4 << 20) - 256) // 4


def _lib():
    import quail_b200
    here = os.path.dirname(quail_b200.__file__)
    path = sorted(glob.glob(os.path.join(here, "_C*.so")))[0]
    lib = ctypes.CDLL(path)
    fn = lib.qb_gemm_fp8_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    return fn


def _call(fn, a8, sa_rows, b8, sb, out, status=True):
    M, K = a8.shape
    N = b8.shape[0]
    st = ctypes.c_int(-7)
    rc = fn(a8.data_ptr(), a8.stride(0), sa_rows.data_ptr(), b8.data_ptr(), b8.stride(0), sb.data_ptr(),
            out.data_ptr(), out.stride(0), M, N, K, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
            ctypes.byref(st) if status else None)
    return rc, st.value


def _case(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a8, sa = ops.quantize_act(torch.randn(M, K, device="cuda", generator=g))
    b8, sb = ops.quantize_weight(torch.randn(N, K, device="cuda", generator=g) * 0.02)
    return a8, sa, b8, sb


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_noalloc_gemm_matches_the_torch_entry_point_on_two_calls():
    fn = _lib()
    for M, N, K, seed in ((300, 512, 1024, 0), (1000, 2560, 2560, 1)):
        a8, sa, b8, sb = _case(M, N, K, seed)
        want = ops.gemm(a8, b8, sa=sa, sb=sb)
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc, st = _call(fn, a8, sa.t().contiguous(), b8, sb, out)
        assert rc == 0 and st == 0, (rc, st)
        assert _rel(out, want) < 5e-3
        # and directly against the fp32 product of the dequantized operands
        a32 = dequantize_act(a8, sa)
        b32 = dequantize_weight(b8, sb)
        assert _rel(out, a32 @ b32.t()) < 1e-2


def test_noalloc_gemm_with_no_rows_reports_its_status():
    fn = _lib()
    a8, sa, b8, sb = _case(128, 256, 256, 2)
    sa_rows = sa.t().contiguous()
    out = torch.empty(128, 256, device="cuda", dtype=torch.bfloat16)
    st = ctypes.c_int(-7)
    # M = 0 with valid pointers: nothing runs, and the status word asked for is still written
    rc = fn(a8.data_ptr(), a8.stride(0), sa_rows.data_ptr(), b8.data_ptr(), b8.stride(0), sb.data_ptr(),
            out.data_ptr(), out.stride(0), 0, 256, 256, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
            ctypes.byref(st))
    assert rc == 0 and st.value == 0


def test_noalloc_gemm_rejects_a_call_beyond_its_scratch():
    fn = _lib()
    K = 1024
    M = QB_NOALLOC_MAX_SCALES // (K // 128) + 1
    a8 = torch.empty(M, K, device="cuda", dtype=torch.float8_e4m3fn)
    sa = torch.empty(M, K // 128, device="cuda")
    b8 = torch.empty(256, K, device="cuda", dtype=torch.float8_e4m3fn)
    sb = torch.empty(2, K // 128, device="cuda")
    out = torch.empty(M, 256, device="cuda", dtype=torch.bfloat16)
    rc, _ = _call(fn, a8, sa, b8, sb, out)
    assert rc == -2
