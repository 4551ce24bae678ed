"""NVFP4 tcgen05 GEMM (kind::mxf4nvf4, ue4m3 scales per 16): parity with the CPU oracle.

M=N=K=16384; values N(0,1) quantised to e2m1 with an ue4m3 scale
per 16 along K and a per-tensor fp32 scale; fp32 accumulation; bf16 output;
tolerance 1e-2 relative (|y - ref| <= 1e-2 * max(|ref|, rms(ref))).  The device
quantiser must reproduce the oracle's codes, scales (in the atom layout) and
per-tensor scales bit for bit.
"""
import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu
RTOL = 1e-2


def _np(t):
    return t.detach().cpu().numpy()


def test_quantiser_matches_oracle(cuda_device, oracle):
    M, N, K = 130, 300, 512
    A, sfa, B, sfb, g = pb.gen_nvfp4(M, N, K, seed=4, tid0=8)
    rA, rSFA, rGA, rB, rSFB, rGB = oracle.nvfp4_operands(M, N, K, seed=4, copy=1)
    gh = _np(g)
    assert gh[0] == rGA and gh[1] == rGB
    np.testing.assert_array_equal(_np(A), rA)
    np.testing.assert_array_equal(_np(B), rB)
    np.testing.assert_array_equal(_np(sfa), oracle.sf_to_atoms(rSFA))
    np.testing.assert_array_equal(_np(sfb), oracle.sf_to_atoms(rSFB))


SHAPES = [(128, 256, 256), (256, 512, 1024), (130, 200, 512), (1, 17, 256), (1000, 1000, 2048), (384, 128, 4096)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemm_nvfp4_matches_oracle(cuda_device, oracle, shape):
    M, N, K = shape
    A, SFA, GA, B, SFB, GB = oracle.nvfp4_operands(M, N, K, seed=M + 5 * N + K)
    d = [torch.from_numpy(x).to(cuda_device) for x in (A, oracle.sf_to_atoms(SFA), B, oracle.sf_to_atoms(SFB))]
    y32 = pb.gemm_nvfp4(d[0], d[1], d[2], d[3], float(GA), float(GB), out_type=pb.QG_OUT_F32)
    ybf = pb.gemm_nvfp4(d[0], d[1], d[2], d[3], float(GA), float(GB), out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0
    ref32 = oracle.gemm_nvfp4(A, SFA, GA, B, SFB, GB, out_type=1)
    assert oracle.max_rel_err(_np(y32), ref32, 1) < 1e-5
    refbf = oracle.gemm_nvfp4(A, SFA, GA, B, SFB, GB, out_type=0)
    assert oracle.max_rel_err(_np(ybf.view(torch.int16)).view(np.uint16), refbf, 0) < RTOL


def test_full_size_config4_sampled_rows(cuda_device, oracle):
    """configs[4] at full size (16384^3): 6 sampled rows against the oracle, then self-reproduction."""
    M = N = K = 16384
    with pb.Workload(pb.QG_FMT_NVFP4, M, N, K, seed=4) as w:
        w.fill(4)
        w.golden()
        A = _np(w.tensor(0, 0)).reshape(M, K // 2)
        B = _np(w.tensor(0, 2)).reshape(N, K // 2)
        sfa_atoms = _np(w.tensor(0, 1))
        sfb_atoms = _np(w.tensor(0, 3))
        g = _np(w.tensor(0, 4, torch.float32))
        Y = _np(w.tensor(0, w.SLOT_OUT, torch.int16)).view(np.uint16).reshape(M, N)
        rows = np.array([0, 127, 8191, 16383] + list(np.random.default_rng(4).integers(0, M, 2)), dtype=np.int32)
        # plain-layout scales of the sampled rows of A and all of B, recovered from the atoms
        def plain(atoms, R):
            a = atoms.reshape((R + 127) // 128, K // 64, 512)
            r = np.arange(R)
            out = np.empty((R, K // 16), dtype=np.uint8)
            for j in range(K // 16):
                out[:, j] = a[r // 128, j // 4, (r % 32) * 16 + ((r // 32) % 4) * 4 + j % 4]
            return out
        SFA = plain(sfa_atoms, M)
        SFB = plain(sfb_atoms, N)
        ref = oracle.gemm_nvfp4(A, SFA, g[0], B, SFB, g[1], out_type=0, rows=rows)
        assert oracle.max_rel_err(Y[rows].copy(), ref, 0) < RTOL
        w.run(2)
        assert w.verify() == 0
        assert pb.device_status(0) == 0
