"""ctypes binding of the CPU oracle (oracle/libqg_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker or the timed CPU baseline; never
by pantheon_b200/.  Parity of the workload's NUMERICS with the reference is
unpinned (the reference has no such arithmetic, see qg_oracle.h); the oracle's
conversions and integer GEMM are pinned against numpy/torch in tests.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libqg_oracle.so"
REF_DIR = HERE / "_ref"

_lib = None
_P = C.c_void_p


def build(quiet: bool = True) -> None:
    """Build the oracle (and, when the reference tree is present, oracle/_ref)."""
    proc = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stdout}\n{proc.stderr}")
    if not quiet:
        print(proc.stdout)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        sig = {
            "qgo_splitmix64": (C.c_uint64, [C.c_uint64]),
            "qgo_hash64": (C.c_uint64, [C.c_uint64, C.c_uint32, C.c_uint64]),
            "qgo_normal_from_hash": (C.c_float, [C.c_uint64]),
            "qgo_logf": (C.c_float, [C.c_float]),
            "qgo_gen_i8": (None, [_P, C.c_uint64, C.c_uint64, C.c_uint32]),
            "qgo_gen_uniform_f32": (None, [_P, C.c_uint64, C.c_float, C.c_float, C.c_uint64, C.c_uint32]),
            "qgo_gen_normal_f32": (None, [_P, C.c_uint64, C.c_uint64, C.c_uint32]),
            "qgo_f32_to_bf16": (C.c_uint16, [C.c_float]),
            "qgo_bf16_to_f32": (C.c_float, [C.c_uint16]),
            "qgo_f32_to_f16": (C.c_uint16, [C.c_float]),
            "qgo_f16_to_f32": (C.c_float, [C.c_uint16]),
            "qgo_f32_to_e4m3": (C.c_uint8, [C.c_float]),
            "qgo_e4m3_to_f32": (C.c_float, [C.c_uint8]),
            "qgo_f32_to_e2m1": (C.c_uint8, [C.c_float]),
            "qgo_e2m1_to_f32": (C.c_float, [C.c_uint8]),
            "qgo_cksum_weight": (C.c_uint32, [C.c_uint32, C.c_uint32]),
            "qgo_gemm_i8": (None, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int, _P, _P, _P]),
            "qgo_quant_fp8_rows": (None, [_P, C.c_int, C.c_int, _P, _P]),
            "qgo_quant_fp8_blocks": (None, [_P, C.c_int, C.c_int, _P, _P]),
            "qgo_gemm_fp8_b128": (None, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int, _P]),
            "qgo_gemm_dense": (None, [C.c_int, _P, _P, C.c_float, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int, _P]),
            "qgo_gen_dense": (None, [C.c_int, _P, C.c_uint64, C.c_uint64, C.c_uint32]),
            "qgo_f32_to_tf32_bits": (C.c_uint32, [C.c_float]),
            "qgo_dense_value": (C.c_float, [C.c_uint64]),
            "qgo_nvfp4_global_scale": (C.c_float, [_P, C.c_uint64]),
            "qgo_quant_nvfp4": (None, [_P, C.c_int, C.c_int, C.c_float, _P, _P]),
            "qgo_gemm_nvfp4": (None, [_P, _P, C.c_float, _P, _P, C.c_float, C.c_int, C.c_int, C.c_int, _P,
                                      C.c_int, C.c_int, _P]),
            "qgo_gemv_w4a16": (None, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int, _P]),
            "qgo_gen_w4a16": (None, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_uint32]),
            "qgo_count_mismatch_u32": (C.c_uint64, [_P, _P, C.c_uint64]),
            "qgo_max_rel_err": (C.c_double, [_P, _P, C.c_uint64, C.c_int]),
            "qgo_threads": (C.c_int, []),
            "qgo_set_threads": (None, [C.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags.c_contiguous
    return C.c_void_p(a.ctypes.data)


# ---------------------------------------------------------------- generator
def gen_i8(n: int, seed: int, tensor_id: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int8)
    lib().qgo_gen_i8(_p(out), n, seed, tensor_id)
    return out


def gen_uniform_f32(n: int, lo: float, hi: float, seed: int, tensor_id: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().qgo_gen_uniform_f32(_p(out), n, lo, hi, seed, tensor_id)
    return out


def gen_normal_f32(n: int, seed: int, tensor_id: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().qgo_gen_normal_f32(_p(out), n, seed, tensor_id)
    return out


def int8_operands(M: int, N: int, K: int, seed: int, copy: int = 0):
    """The INT8 workload's operands of copy `copy` (tensor ids 8*copy + 0..3)."""
    b = 8 * copy
    A = gen_i8(M * K, seed, b + 0).reshape(M, K)
    B = gen_i8(N * K, seed, b + 1).reshape(N, K)
    sa = gen_uniform_f32(M, 0.001, 0.01, seed, b + 2)
    sb = gen_uniform_f32(N, 0.001, 0.01, seed, b + 3)
    return A, B, sa, sb


# ---------------------------------------------------------------- GEMMs
def gemm_i8(A, B, sa, sb, out_type: int = 0, rows=None, want_acc: bool = False, want_cksum: bool = False):
    """Oracle INT8 GEMM. out_type 0 = bf16 (returned as uint16 bits), 1 = f32, 2 = s32."""
    A = np.ascontiguousarray(A, dtype=np.int8)
    B = np.ascontiguousarray(B, dtype=np.int8)
    M, K = A.shape
    N = B.shape[0]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    nr = M if r is None else len(r)
    dt = {0: np.uint16, 1: np.float32, 2: np.int32}[out_type]
    C_ = np.empty((nr, N), dtype=dt)
    acc = np.empty((nr, N), dtype=np.int32) if want_acc else None
    ck = np.empty(nr, dtype=np.uint32) if want_cksum else None
    sa = None if sa is None else np.ascontiguousarray(sa, dtype=np.float32)
    sb = None if sb is None else np.ascontiguousarray(sb, dtype=np.float32)
    lib().qgo_gemm_i8(_p(A), _p(B), _p(sa), _p(sb), M, N, K, _p(r), nr, out_type, _p(C_), _p(acc), _p(ck))
    res = [C_]
    if want_acc:
        res.append(acc)
    if want_cksum:
        res.append(ck)
    return res[0] if len(res) == 1 else tuple(res)


def fp8_operands(M: int, N: int, K: int, seed: int, copy: int = 0):
    """The FP8 block-128 workload's operands of copy `copy`: A e4m3 [M,K] with sa [M,K/128]
    (values: tensor id 8*copy+0), B e4m3 [N,K] with sb [ceil(N/128),K/128] (tensor id 8*copy+2)."""
    b = 8 * copy
    xa = gen_normal_f32(M * K, seed, b + 0)
    xb = gen_normal_f32(N * K, seed, b + 2)
    A = np.empty((M, K), dtype=np.uint8)
    B = np.empty((N, K), dtype=np.uint8)
    sa = np.empty((M, K // 128), dtype=np.float32)
    sb = np.empty(((N + 127) // 128, K // 128), dtype=np.float32)
    lib().qgo_quant_fp8_rows(_p(xa), M, K, _p(A), _p(sa))
    lib().qgo_quant_fp8_blocks(_p(xb), N, K, _p(B), _p(sb))
    return A, B, sa, sb


def gemm_fp8(A, B, sa, sb, out_type: int = 0, rows=None):
    """Oracle FP8 block-128 GEMM (bf16 bits for out_type 0, f32 for 1)."""
    A = np.ascontiguousarray(A, dtype=np.uint8)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    sa = np.ascontiguousarray(sa, dtype=np.float32)
    sb = np.ascontiguousarray(sb, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    nr = M if r is None else len(r)
    C_ = np.empty((nr, N), dtype=np.uint16 if out_type == 0 else np.float32)
    lib().qgo_gemm_fp8_b128(_p(A), _p(B), _p(sa), _p(sb), M, N, K, _p(r), nr, out_type, _p(C_))
    return C_


# Dense (tensor-furnace) formats: workload format id -> (GEMM kind, storage dtype).
FMT_BF16, FMT_FP16, FMT_TF32, FMT_E4M3, FMT_FP32 = 4, 5, 6, 7, 8
KIND_BF16, KIND_E4M3, KIND_F16, KIND_TF32, KIND_F32 = 1, 2, 3, 4, 5
DENSE_FORMATS = {FMT_BF16: (KIND_BF16, np.uint16), FMT_FP16: (KIND_F16, np.uint16),
                 FMT_TF32: (KIND_TF32, np.uint32), FMT_E4M3: (KIND_E4M3, np.uint8), FMT_FP32: (KIND_F32, np.uint32)}
_KIND_DTYPE = {KIND_BF16: np.uint16, KIND_F16: np.uint16, KIND_TF32: np.uint32, KIND_E4M3: np.uint8,
               KIND_F32: np.uint32}
_OUT_DTYPE = {0: np.uint16, 1: np.float32, 3: np.uint16}


def gen_dense(fmt: int, n: int, seed: int, tensor_id: int):
    """The dense workload's operand stream: format `fmt` bit patterns (uint16 / uint32 / uint8)."""
    out = np.empty(n, dtype=DENSE_FORMATS[fmt][1])
    lib().qgo_gen_dense(fmt, _p(out), n, seed, tensor_id)
    return out


def dense_operands(fmt: int, M: int, N: int, K: int, seed: int, copy: int = 0):
    """A [M,K] and B [N,K] of copy `copy` of a dense workload (tensor ids 8*copy, 8*copy+1)."""
    b = 8 * copy
    return gen_dense(fmt, M * K, seed, b).reshape(M, K), gen_dense(fmt, N * K, seed, b + 1).reshape(N, K)


def gemm_dense(kind: int, A, B, alpha: float = 1.0, out_type: int = 0, rows=None):
    """Oracle tensor-furnace GEMM C = alpha * A B^T: kind 1 = bf16, 3 = fp16 (A, B as uint16
    bits), 4 = tf32 and 5 = fp32 (uint32 fp32 words), 2 = e4m3 (uint8); out_type 0 = bf16 bits,
    1 = f32, 3 = fp16 bits."""
    dt = _KIND_DTYPE[kind]
    A = np.ascontiguousarray(A, dtype=dt)
    B = np.ascontiguousarray(B, dtype=dt)
    M, K = A.shape
    N = B.shape[0]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    nr = M if r is None else len(r)
    C_ = np.empty((nr, N), dtype=_OUT_DTYPE[out_type])
    lib().qgo_gemm_dense(kind, _p(A), _p(B), float(alpha), M, N, K, _p(r), nr, out_type, _p(C_))
    return C_


def nvfp4_operands(M: int, N: int, K: int, seed: int, copy: int = 0):
    """The NVFP4 workload's operands of copy `copy`: A, B packed e2m1 [R, K/2] (low nibble =
    even k), scales ue4m3 in the PLAIN layout [R, K/16], per-tensor scales GA, GB
    (values: tensor ids 8*copy+0 and 8*copy+2)."""
    b = 8 * copy
    out = []
    for R, tid in ((M, b + 0), (N, b + 2)):
        x = gen_normal_f32(R * K, seed, tid)
        g = lib().qgo_nvfp4_global_scale(_p(x), x.size)
        q = np.empty((R, K // 2), dtype=np.uint8)
        sf = np.empty((R, K // 16), dtype=np.uint8)
        lib().qgo_quant_nvfp4(_p(x), R, K, g, _p(q), _p(sf))
        out.append((q, sf, np.float32(g)))
    (A, SFA, GA), (B, SFB, GB) = out
    return A, SFA, GA, B, SFB, GB


def sf_to_atoms(sf: np.ndarray) -> np.ndarray:
    """Plain scales [R, K/16] -> the tcgen05 atom layout (512-byte atom per 128 rows x 64 K;
    row r's 4 scales at (r%32)*16 + ((r/32)%4)*4), atoms ordered [row block][K/64]."""
    R, nb = sf.shape
    rb = (R + 127) // 128
    kc = nb // 4
    out = np.zeros((rb, kc, 512), dtype=np.uint8)
    r = np.arange(R)
    for j in range(nb):
        out[r // 128, j // 4, (r % 32) * 16 + ((r // 32) % 4) * 4 + (j % 4)] = sf[:, j]
    return out.reshape(-1)


def gemm_nvfp4(A, SFA, GA, B, SFB, GB, out_type: int = 0, rows=None):
    """Oracle NVFP4 GEMM (plain-layout scales). bf16 bits for out_type 0, f32 for 1."""
    A = np.ascontiguousarray(A, dtype=np.uint8)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    SFA = np.ascontiguousarray(SFA, dtype=np.uint8)
    SFB = np.ascontiguousarray(SFB, dtype=np.uint8)
    M, K = A.shape[0], A.shape[1] * 2
    N = B.shape[0]
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    nr = M if r is None else len(r)
    C_ = np.empty((nr, N), dtype=np.uint16 if out_type == 0 else np.float32)
    lib().qgo_gemm_nvfp4(_p(A), _p(SFA), float(GA), _p(B), _p(SFB), float(GB), M, N, K, _p(r), nr, out_type, _p(C_))
    return C_


def nvfp4_dequant(Q: np.ndarray, SF: np.ndarray, G: float) -> np.ndarray:
    """float64 values q * sf * G of packed codes and plain scales (independent numpy decode)."""
    grid = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    lo = Q & 0xF
    hi = Q >> 4
    codes = np.stack([lo, hi], axis=-1).reshape(Q.shape[0], -1)
    vals = grid[codes & 7] * np.where(codes & 8, -1.0, 1.0)
    sf = e4m3_to_f32(SF).astype(np.float64)
    return vals * np.repeat(sf, 16, axis=1) * float(G)


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    import torch
    return torch.from_numpy(np.ascontiguousarray(q, dtype=np.uint8)).view(torch.float8_e4m3fn).float().numpy()


def w4a16_operands(M: int, N: int, K: int, seed: int, copy: int = 0):
    """The W4A16 workload's operands of copy `copy` (tensor ids 8*copy + 0..3):
    X bf16 bits [M,K], W uint32 [K/8,N], S and Z fp16 bits [K/128,N]."""
    X = np.empty((M, K), dtype=np.uint16)
    W = np.empty((K // 8, N), dtype=np.uint32)
    S = np.empty((K // 128, N), dtype=np.uint16)
    Z = np.empty((K // 128, N), dtype=np.uint16)
    lib().qgo_gen_w4a16(_p(X), _p(W), _p(S), _p(Z), M, N, K, seed, 8 * copy)
    return X, W, S, Z


def gemv_w4a16(X, W, S, Z, out_type: int = 0, cols=None):
    """Oracle W4A16 GEMV; returns [M, ncols] (bf16 bits for out_type 0, f32 for 1)."""
    X = np.ascontiguousarray(X, dtype=np.uint16)
    W = np.ascontiguousarray(W, dtype=np.uint32)
    S = np.ascontiguousarray(S, dtype=np.uint16)
    Z = np.ascontiguousarray(Z, dtype=np.uint16)
    M, K = X.shape
    N = W.shape[1]
    c = None if cols is None else np.ascontiguousarray(cols, dtype=np.int32)
    nc = N if c is None else len(c)
    Y = np.empty((M, nc), dtype=np.uint16 if out_type == 0 else np.float32)
    lib().qgo_gemv_w4a16(_p(X), _p(W), _p(S), _p(Z), M, N, K, _p(c), nc, out_type, _p(Y))
    return Y


def gemv_w4a16_numpy(X, W, S, Z) -> np.ndarray:
    """Independent float64 numpy evaluation of the W4A16 GEMV (for pinning the oracle)."""
    x = bf16_bits_to_f32(X).astype(np.float64)
    K = x.shape[1]
    N = W.shape[1]
    shifts = (4 * np.arange(8, dtype=np.uint32))[None, :, None]
    u = ((W[:, None, :] >> shifts) & np.uint32(0xF)).reshape(K, N).astype(np.float64)
    s = np.repeat(S.view(np.float16).astype(np.float64), 128, axis=0)
    z = np.repeat(Z.view(np.float16).astype(np.float64), 128, axis=0)
    w = (u - 8.0 - z) * s
    return x @ w


# ---------------------------------------------------------------- conversions
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    f = lib().qgo_f32_to_bf16
    return np.array([f(float(v)) for v in np.asarray(x, dtype=np.float32).ravel()], dtype=np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def max_rel_err(y: np.ndarray, r: np.ndarray, kind: int) -> float:
    y = np.ascontiguousarray(y)
    r = np.ascontiguousarray(r)
    return lib().qgo_max_rel_err(_p(y), _p(r), y.size, kind)


def threads() -> int:
    return lib().qgo_threads()


def set_threads(n: int) -> None:
    """OpenMP threads for the oracle from now on (overrides OMP_NUM_THREADS)."""
    lib().qgo_set_threads(int(n))


def host_threads() -> int:
    """Cores this process may run on."""
    import os
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
