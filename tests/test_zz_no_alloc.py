"""The allocation-free SSD forward (C symbol ``ahb_ssd_fwd_noalloc``).

Some callers of this library cannot allocate device memory while they run --
for example code executing under another framework's CUDA-graph capture, or a
serving engine that reserves all HBM up front.  For them the library exports
one ``extern "C"`` entry point whose scratch is a fixed device array.  This test
calls it through ctypes, twice in a row with different inputs (the scratch keeps
the previous call's contents), and compares each result with the regular,
allocating SSD forward.  It lives in its own file, collected last.
"""
import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
dev = "cuda"


def _fn():
    import atomic_ai_hybrid_b200._ahb_cuda as mod
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.ahb_ssd_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _inputs(B, L, H, seed):
    g_ = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(B, L, H, 64, generator=g_, device=dev).to(torch.bfloat16)
    dt = F.softplus(torch.randn(B, L, H, 64, generator=g_, device=dev) - 2).clamp(1e-2, 1.0).to(torch.bfloat16)
    A = -torch.exp(torch.rand(H, generator=g_, device=dev) * math.log(16.0))
    Bm = (torch.randn(B, L, 128, generator=g_, device=dev) / math.sqrt(128)).to(torch.bfloat16)
    Cm = (torch.randn(B, L, 128, generator=g_, device=dev) / math.sqrt(128)).to(torch.bfloat16)
    return x, dt, A, Bm, Cm


def _call(fn, x, dt, A, Bm, Cm, y):
    B, L, H, _ = x.shape
    return fn(x.data_ptr(), dt.data_ptr(), A.data_ptr(), Bm.data_ptr(), Cm.data_ptr(), B, L, H, y.data_ptr(),
              torch.cuda.current_stream().cuda_stream)


# the largest problem the fixed scratch holds: B * H * (L / 64) = 1 * 2 * 407 = 814 chunk-heads
MAX_CASE = (1, 407 * 64, 2)


def test_noalloc_ssd_forward_matches_allocating_entry_point():
    """Same kernels as the allocating forward, only another scratch base: the outputs must
    agree bit for bit, on two calls in a row and on the largest accepted problem (whose
    decay sums sit at the end of the fixed array)."""
    from atomic_ai_hybrid_b200.ops._ext import ext
    fn = _fn()
    for seed, (B, L, H) in enumerate([(2, 256, 4), (1, 384, 3), MAX_CASE]):
        x, dt, A, Bm, Cm = _inputs(B, L, H, seed)
        ref = ext().ssd_fwd(x, dt, A, Bm, Cm)
        y = torch.full_like(x, float("nan"))
        rc = _call(fn, x, dt, A, Bm, Cm, y)
        torch.cuda.synchronize()
        assert rc == 0
        assert torch.equal(y, ref), (B, L, H)


def test_noalloc_rejects_oversized_problem():
    fn = _fn()
    # one chunk-head beyond the fixed scratch (1 * 5 * 163 = 815 > 814), and a far larger one:
    # both rejected before any launch
    for B, L, H in [(1, 163 * 64, 5), (64, 8192, 64)]:
        x, dt, A, Bm, Cm = _inputs(1, 64, 1, 0)
        y = torch.empty_like(x)
        rc = fn(x.data_ptr(), dt.data_ptr(), A.data_ptr(), Bm.data_ptr(), Cm.data_ptr(), B, L, H, y.data_ptr(),
                torch.cuda.current_stream().cuda_stream)
        assert rc == -2
