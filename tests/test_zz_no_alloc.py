"""The allocation-free W4A16 GEMV entry point (qg_gemv_w4a16_noalloc), on a B200.

Who it is for: callers that cannot allocate device memory where they call the
GEMV -- a process whose device-memory budget is already claimed, or a
latency-critical decode path where an allocation is not acceptable.  It takes
its split-K scratch from a fixed array inside the library instead of a
caller-provided workspace.

The test calls it through the C ABI, twice in a row, and checks each output
against the existing entry point (qg_gemv_w4a16 with its own workspace)
within the tolerance the other GEMV tests use; then a sequence of calls of
different shapes, bf16 and fp32 out, each against the workspace entry point
bit for bit; and that a shape whose scratch would exceed the built-in maximum
is rejected.  This file is
collected last, so a failure here comes after every other test has run; it
passes on its own in a fresh process as well as after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu
RTOL = 1e-2   # same bar as tests/test_gpu_w4a16.py


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _bf16_bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("M", [1, 8, 12, 16])   # CUDA cores; warp MMAs (two, three B fragments); tcgen05
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, oracle, qglib, M):
    N, K = 28672, 8192                       # configs[3]
    X, W, S, Z = pb.gen_w4a16(M, N, K, seed=21 + M)
    ref = pb.gemv_w4a16(X, W, S, Z, out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        y = torch.full_like(ref, float("nan"))
        rc = qglib.qg_gemv_w4a16_noalloc(_ptr(X), _ptr(W), _ptr(S), _ptr(Z), _ptr(y), pb.QG_OUT_BF16,
                                         M, N, K, stream)
        assert rc == 0, pb._lib.last_error()
        torch.cuda.synchronize()
        assert oracle.max_rel_err(_bf16_bits(y), _bf16_bits(ref), 0) < RTOL


@pytest.mark.parametrize("out_type", [pb.QG_OUT_BF16, pb.QG_OUT_F32])
def test_noalloc_after_calls_of_other_shapes(cuda_device, qglib, out_type):
    """Each call starts from what the previous call, of another shape, left in the shared
    scratch: partial sums where this call keeps its tickets.  A sequence of shapes
    (all three GEMV kernels, 1 to 24 rows, so also two row chunks) must still give exactly
    the output of the workspace entry point with a fresh zeroed workspace."""
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for M, N, K in [(16, 28672, 8192), (1, 4096, 2048), (8, 28672, 8192), (24, 4096, 4096), (2, 28672, 8192),
                    (12, 28672, 8192), (28, 4096, 2048), (16, 28672, 8192)]:
        X, W, S, Z = pb.gen_w4a16(M, N, K, seed=100 + M + N)
        ref = pb.gemv_w4a16(X, W, S, Z, out_type=out_type)
        y = torch.full_like(ref, float("nan"))
        rc = qglib.qg_gemv_w4a16_noalloc(_ptr(X), _ptr(W), _ptr(S), _ptr(Z), _ptr(y), out_type, M, N, K, stream)
        assert rc == 0, pb._lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16 if out_type == pb.QG_OUT_BF16 else torch.int32),
                           ref.view(torch.int16 if out_type == pb.QG_OUT_BF16 else torch.int32)), (M, N, K)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device, qglib):
    X, W, S, Z = pb.gen_w4a16(1, 512, 128, seed=1)
    y = torch.empty((1, 512), dtype=torch.bfloat16, device=cuda_device)
    # 16 rows x 2^20 columns needs far more than the built-in scratch
    rc = qglib.qg_gemv_w4a16_noalloc(_ptr(X), _ptr(W), _ptr(S), _ptr(Z), _ptr(y), pb.QG_OUT_BF16,
                                     16, 1 << 20, 8192, None)
    assert rc == pb._lib.QG_ERR_ARG
    assert "maximum" in pb._lib.last_error()
