"""The allocation-free weight-gradient entry point, called through its exported C symbol.

``maloq_weight_grad_noalloc`` serves callers that cannot allocate device memory while they
launch work (they hand the library fixed buffers made up front); it keeps its split-K
partials in a fixed device array instead of a fresh workspace.  This file is collected
last so that a run stopping at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    from maloq_b200.ops import _ext, kernels

    kernels.lib()  # build/load the library
    so = ctypes.CDLL(_ext.load().__file__)
    fn = so.maloq_weight_grad_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p]
    err = so.maloq_noalloc_last_error
    err.restype = ctypes.c_char_p
    return fn, err


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (64, 256, 128), (100, 128, 136), (1500, 512, 256),
                                   (5000, 128, 136), (43000, 1152, 1280)])
def test_noalloc_matches_fp32_torch_twice(cuda_device, M, N, K):
    """Two calls in a row against an fp32 PyTorch product of the same bf16 inputs, and against
    the allocating entry point.  M = 1 and 64 take the single-slice path (no scratch), larger M
    the split-K path through the shared array; NaN-filled outputs catch unwritten elements."""
    from maloq_b200.ops import kernels

    fn, err = _entry()
    torch.manual_seed(3)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        gy = torch.randn(M, N, device=cuda_device).bfloat16()
        x = torch.randn(M, K, device=cuda_device).bfloat16()
        out = torch.full((N, K), float("nan"), device=cuda_device)
        rc = fn(gy.data_ptr(), x.data_ptr(), out.data_ptr(), M, N, K, stream)
        assert rc == 0, err()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all(), call
        ref = gy.float().T @ x.float()
        scale = ref.abs().max().item()
        assert (out - ref).abs().max().item() / scale < 1e-4, call
        alloc = kernels.gemm_tn_weight_grad(gy, x)
        assert (out - alloc).abs().max().item() / scale < 1e-4, call
    assert kernels.error_status() == 0


def test_noalloc_rejects_oversize(cuda_device):
    fn, err = _entry()
    dummy = torch.empty(8, device=cuda_device)
    rc = fn(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 1024, 4096, 4096,
            torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and b"too large" in err()
