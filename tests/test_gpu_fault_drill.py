"""The bounded-wait failure path, run for real on a B200 without a GPU fault.

qg_fault_drill_i8 runs one small INT8 GEMM whose producers stop issuing before
one K block, so the MMA issuer's wait for that block can never complete; every
wait is limited to 1 ms.  The wait must give up: the kernel records where,
lets its copies and MMAs in flight land, frees its TMEM and returns, the host
reads QG_ERR_DEVICE_TIMEOUT with every CTA counted as drained, and the next
ordinary GEMM in the same process is bit-exact against the oracle.  (The
reference's kernels have no bounded waits; a lost producer there is a hang
the runner's timeout ends, pantheon.py:4018.)
"""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def test_expired_wait_ends_the_kernel_and_the_next_gemm_is_exact(cuda_device, oracle, qglib):
    import torch
    import pantheon_b200 as pb
    M, N, K = 128, 512, 1024                 # 2 CTAs (128x256 tiles), 8 K blocks of 128
    A, B, sa, sb = oracle.int8_operands(M, N, K, seed=5)
    dev = cuda_device
    tA, tB = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
    tsa, tsb = torch.from_numpy(sa).to(dev), torch.from_numpy(sb).to(dev)
    out = torch.zeros((M, N), dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0          # nothing pending from earlier tests

    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    t0 = time.perf_counter()
    rc = qglib.qg_fault_drill_i8(_ptr(tA), _ptr(tB), _ptr(tsa), _ptr(tsb), _ptr(out), M, N, K,
                                 C.c_uint64(1_000_000), 2, stream)
    assert rc == 0
    torch.cuda.synchronize()                 # the kernel returned: no hang, no fault
    assert time.perf_counter() - t0 < 10.0

    site, waits, drained = C.c_uint32(), C.c_uint32(), C.c_uint32()
    st = qglib.qg_device_status_detail(0, C.byref(site), C.byref(waits), C.byref(drained))
    assert st == pb._lib.QG_ERR_DEVICE_TIMEOUT
    assert site.value >> 16 == 1             # kernel id 1: the INT8 GEMM
    assert waits.value >= 1
    assert drained.value == 2                # both CTAs drained and freed their TMEM
    assert pb.device_status(0) == 0          # the detail call cleared the status

    # the process and the device stay usable: an ordinary GEMM is bit-exact
    good = pb.gemm_i8(tA, tB, tsa, tsb, out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0
    got = good.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle.gemm_i8(A, B, sa, sb, out_type=0)
    assert int((got != ref).sum()) == 0


def test_drill_rejects_bad_arguments(cuda_device, qglib):
    import torch
    dev = cuda_device
    a = torch.zeros((256, 256), dtype=torch.int8, device=dev)
    s = torch.ones((256,), dtype=torch.float32, device=dev)
    o = torch.zeros((256, 256), dtype=torch.bfloat16, device=dev)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    # M >= 256 would take the pair kernel, which has no drill; the limit must stay in range
    assert qglib.qg_fault_drill_i8(_ptr(a), _ptr(a), _ptr(s), _ptr(s), _ptr(o), 256, 256, 256,
                                   C.c_uint64(1_000_000), 1, stream) == -1
    assert qglib.qg_fault_drill_i8(_ptr(a), _ptr(a), _ptr(s), _ptr(s), _ptr(o), 128, 256, 256,
                                   C.c_uint64(10), 1, stream) == -1
    assert qglib.qg_fault_drill_i8(_ptr(a), _ptr(a), _ptr(s), _ptr(s), _ptr(o), 128, 256, 256,
                                   C.c_uint64(1_000_000), 7, stream) == -1
