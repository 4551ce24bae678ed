"""Python entry points over the C ABI (torch tensors in, device pointers out).

These mirror, one for one, the pieces of the reference workload harness
(kernels/common/ai_workload_template.h:85-94 init, :157-177 kernel, :343-349
verify, :351-380 main) that include/pantheon_qgemm.h replaces.  Every call goes
to the sm_100a kernels in libpantheon_qgemm.so; there is no other path.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import (QG_GEMV_ACTIVATIONS_CONST, QG_GEMV_WEIGHTS_CONST, QG_FMT_INT8, QG_FMT_BF16, QG_FMT_FP16, QG_FMT_TF32, QG_FMT_E4M3, QG_FMT_FP32, QG_OUT_BF16, QG_OUT_F16,
                   QG_OUT_F32, QG_OUT_S32, QGCfg, QGMismatch, QGError, check,
                   last_error, load_library)

_OUT_DTYPES = {QG_OUT_BF16: torch.bfloat16, QG_OUT_F32: torch.float32, QG_OUT_S32: torch.int32,
               QG_OUT_F16: torch.float16}


class _DeviceBytes:
    """A raw device allocation of the library seen as a uint8 array (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream(device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("pantheon_b200 kernels take CUDA tensors only (no CPU fallback)")
        if t is not None and not t.is_contiguous():
            raise ValueError("pantheon_b200 kernels take contiguous tensors")


def gemm_i8(A: torch.Tensor, B: torch.Tensor, sa: torch.Tensor | None, sb: torch.Tensor | None,
            out_type: int = QG_OUT_BF16, row_checksums: bool = False, out: torch.Tensor | None = None):
    """C = out(f32(A @ B^T) * sa[:, None] * sb[None, :]) on the tcgen05 INT8 path.

    A int8 [M,K], B int8 [N,K] (K contiguous, K % 16 == 0); sa fp32 [M]; sb fp32 [N].
    Returns C (and the uint32 per-row checksums of the INT32 accumulators when
    row_checksums=True).  Asynchronous on the current stream.
    """
    _require_cuda(A, B, sa, sb)
    if A.dtype != torch.int8 or B.dtype != torch.int8:
        raise ValueError("A and B must be int8")
    M, K = A.shape
    N, K2 = B.shape
    if K != K2:
        raise ValueError(f"K mismatch {K} vs {K2}")
    if out is None:
        out = torch.empty((M, N), dtype=_OUT_DTYPES[out_type], device=A.device)
    ck = torch.empty((M,), dtype=torch.int32, device=A.device) if row_checksums else None
    lib = load_library()
    check("qg_gemm_i8", lib.qg_gemm_i8(_ptr(A), _ptr(B), _ptr(sa), _ptr(sb), _ptr(out), out_type, _ptr(ck),
                                       M, N, K, _stream(A.device)))
    return (out, ck) if row_checksums else out


def gemm_fp8_b128(A: torch.Tensor, B: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor,
                  out_type: int = QG_OUT_BF16, out: torch.Tensor | None = None) -> torch.Tensor:
    """C = sum_kb (A_kb @ B_kb^T) * sa[:, kb] * sb[n/128, kb] on the tcgen05 FP8 path.

    A, B e4m3 bytes (uint8 or float8_e4m3fn) [M,K] / [N,K]; sa fp32 [M,K/128];
    sb fp32 [ceil(N/128),K/128].  Asynchronous on the current stream.
    """
    _require_cuda(A, B, sa, sb)
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=_OUT_DTYPES[out_type], device=A.device)
    check("qg_gemm_fp8_b128", load_library().qg_gemm_fp8_b128(_ptr(A), _ptr(B), _ptr(sa), _ptr(sb), _ptr(out),
                                                               out_type, M, N, K, _stream(A.device)))
    return out


def _gemm_dense(entry: str, A: torch.Tensor, B: torch.Tensor, alpha: float, out_type: int,
                out: torch.Tensor | None) -> torch.Tensor:
    _require_cuda(A, B)
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=_OUT_DTYPES[out_type], device=A.device)
    check(entry, getattr(load_library(), entry)(_ptr(A), _ptr(B), float(alpha), _ptr(out), out_type, M, N, K,
                                                _stream(A.device)))
    return out


def gemm_bf16(A: torch.Tensor, B: torch.Tensor, alpha: float = 1.0, out_type: int = QG_OUT_BF16,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * A @ B^T (fp32 accumulate) on the tcgen05 bf16 path: A bf16 [M,K], B bf16 [N,K]."""
    return _gemm_dense("qg_gemm_bf16", A, B, alpha, out_type, out)


def gemm_f16(A: torch.Tensor, B: torch.Tensor, alpha: float = 1.0, out_type: int = QG_OUT_F16,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * A @ B^T (fp32 accumulate) on the tcgen05 fp16 path: A fp16 [M,K], B fp16 [N,K]."""
    return _gemm_dense("qg_gemm_f16", A, B, alpha, out_type, out)


def gemm_tf32(A: torch.Tensor, B: torch.Tensor, alpha: float = 1.0, out_type: int = QG_OUT_F32,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * A @ B^T (fp32 accumulate) on the tcgen05 tf32 path: A, B fp32 [M,K] / [N,K]
    holding tf32 values (low 13 mantissa bits zero)."""
    return _gemm_dense("qg_gemm_tf32", A, B, alpha, out_type, out)


def gemm_f32(A: torch.Tensor, B: torch.Tensor, alpha: float = 1.0, out_type: int = QG_OUT_F32,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * A @ B^T with fp32 operands and fp32 FMAs on the CUDA cores: A, B fp32 [M,K] / [N,K]."""
    return _gemm_dense("qg_gemm_f32", A, B, alpha, out_type, out)


def gemm_e4m3(A: torch.Tensor, B: torch.Tensor, alpha: float = 1.0, out_type: int = QG_OUT_BF16,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """C = alpha * A @ B^T (fp32 accumulate) on the tcgen05 e4m3 path: A, B e4m3 bytes [M,K] / [N,K]."""
    return _gemm_dense("qg_gemm_e4m3", A, B, alpha, out_type, out)


_DENSE_DTYPES = {QG_FMT_BF16: torch.bfloat16, QG_FMT_FP16: torch.float16, QG_FMT_TF32: torch.float32,
                 QG_FMT_E4M3: torch.uint8, QG_FMT_FP32: torch.float32}


def gen_dense(fmt: int, rows: int, cols: int, seed: int, tensor_id: int, device="cuda") -> torch.Tensor:
    """A dense workload operand [rows, cols] from the generator stream (seed, tensor_id)."""
    out = torch.empty((rows, cols), dtype=_DENSE_DTYPES[fmt], device=device)
    check("qg_gen_dense", load_library().qg_gen_dense(fmt, _ptr(out), rows * cols, seed, tensor_id,
                                                       _stream(out.device)))
    return out


def gen_fp8(M: int, N: int, K: int, seed: int, tid0: int = 0, device="cuda"):
    """The FP8 workload's generated operands (A, B as uint8 e4m3 bytes; sa, sb fp32)."""
    A = torch.empty((M, K), dtype=torch.uint8, device=device)
    B = torch.empty((N, K), dtype=torch.uint8, device=device)
    sa = torch.empty((M, K // 128), dtype=torch.float32, device=device)
    sb = torch.empty(((N + 127) // 128, K // 128), dtype=torch.float32, device=device)
    check("qg_gen_fp8", load_library().qg_gen_fp8(_ptr(A), _ptr(sa), _ptr(B), _ptr(sb), M, N, K, seed, tid0,
                                                   _stream(A.device)))
    return A, B, sa, sb


def nvfp4_sf_bytes(rows: int, K: int) -> int:
    b = C.c_uint64()
    check("qg_nvfp4_sf_bytes", load_library().qg_nvfp4_sf_bytes(rows, K, C.byref(b)))
    return b.value


def gemm_nvfp4(A: torch.Tensor, sfa: torch.Tensor, B: torch.Tensor, sfb: torch.Tensor, ga: float, gb: float,
               out_type: int = QG_OUT_BF16, out: torch.Tensor | None = None) -> torch.Tensor:
    """C = ga*gb * (A .* sfa) @ (B .* sfb)^T on the tcgen05 NVFP4 path.

    A [M, K/2], B [N, K/2] uint8 (two e2m1 codes per byte, low nibble = even k);
    sfa, sfb uint8 ue4m3 scales in the atom layout (see include/pantheon_qgemm.h).
    """
    _require_cuda(A, sfa, B, sfb)
    M, K2 = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=_OUT_DTYPES[out_type], device=A.device)
    check("qg_gemm_nvfp4", load_library().qg_gemm_nvfp4(_ptr(A), _ptr(sfa), _ptr(B), _ptr(sfb), ga, gb, _ptr(out),
                                                         out_type, M, N, 2 * K2, _stream(A.device)))
    return out


def gen_nvfp4(M: int, N: int, K: int, seed: int, tid0: int = 0, device="cuda"):
    """The NVFP4 workload's generated operands: (A, sfa, B, sfb, gscales[2]) on the device."""
    A = torch.empty((M, K // 2), dtype=torch.uint8, device=device)
    B = torch.empty((N, K // 2), dtype=torch.uint8, device=device)
    sfa = torch.empty((nvfp4_sf_bytes(M, K),), dtype=torch.uint8, device=device)
    sfb = torch.empty((nvfp4_sf_bytes(N, K),), dtype=torch.uint8, device=device)
    g = torch.empty((2,), dtype=torch.float32, device=device)
    work = torch.empty((2,), dtype=torch.int32, device=device)
    check("qg_gen_nvfp4", load_library().qg_gen_nvfp4(_ptr(A), _ptr(sfa), _ptr(B), _ptr(sfb), _ptr(g), _ptr(work),
                                                       M, N, K, seed, tid0, _stream(A.device)))
    return A, sfa, B, sfb, g


def gemv_w4a16_workspace_bytes(M: int, N: int, K: int) -> int:
    b = C.c_uint64()
    check("qg_gemv_w4a16_workspace_bytes", load_library().qg_gemv_w4a16_workspace_bytes(M, N, K, C.byref(b)))
    return b.value


def gemv_w4a16(X: torch.Tensor, W: torch.Tensor, S: torch.Tensor, Z: torch.Tensor, out_type: int = QG_OUT_BF16,
               workspace: torch.Tensor | None = None, out: torch.Tensor | None = None,
               weights_const: bool = False, activations_const: bool = False) -> torch.Tensor:
    """Y = X @ dequant(W) on the W4A16 path (1 row CUDA cores, 2-12 warp MMAs, 13-16 tcgen05).

    X bf16 [M,K]; W int32/uint32 [K/8,N] packed int4 (nibble j = k offset j);
    S, Z fp16 [K/128,N]; returns Y [M,N] (bf16 or fp32).  `workspace` (uint8,
    zero-filled, qg_gemv_w4a16_workspace_bytes) is allocated when not given.
    `weights_const`: the kernel before this call on the stream does not write
    W, S or Z (QG_GEMV_WEIGHTS_CONST), so the first weight loads may start
    before it finishes; `activations_const`: it does not write X
    (QG_GEMV_ACTIVATIONS_CONST), so the activations may be quantised before.
    """
    _require_cuda(X, W, S, Z)
    M, K = X.shape
    N = W.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=_OUT_DTYPES[out_type], device=X.device)
    need = gemv_w4a16_workspace_bytes(M, N, K)
    if workspace is None:
        workspace = torch.zeros((need,), dtype=torch.uint8, device=X.device)
    flags = (QG_GEMV_WEIGHTS_CONST if weights_const else 0) | (QG_GEMV_ACTIVATIONS_CONST if activations_const else 0)
    check("qg_gemv_w4a16_ex", load_library().qg_gemv_w4a16_ex(_ptr(X), _ptr(W), _ptr(S), _ptr(Z), _ptr(out), out_type,
                                                               M, N, K, _ptr(workspace), workspace.numel(), flags,
                                                               _stream(X.device)))
    return out


def gen_w4a16(M: int, N: int, K: int, seed: int, tid0: int = 0, device="cuda"):
    """The W4A16 workload's generated operands (X bf16, W int32, S fp16, Z fp16) on the device."""
    X = torch.empty((M, K), dtype=torch.bfloat16, device=device)
    W = torch.empty((K // 8, N), dtype=torch.int32, device=device)
    S = torch.empty((K // 128, N), dtype=torch.float16, device=device)
    Z = torch.empty((K // 128, N), dtype=torch.float16, device=device)
    check("qg_gen_w4a16", load_library().qg_gen_w4a16(_ptr(X), _ptr(W), _ptr(S), _ptr(Z), M, N, K, seed, tid0,
                                                       _stream(X.device)))
    return X, W, S, Z


def gen_i8(n: int, seed: int, tensor_id: int, device="cuda") -> torch.Tensor:
    """Counter-based uniform int8 in [-127, 127] (same bits as the CPU oracle)."""
    out = torch.empty(((n + 15) // 16) * 16, dtype=torch.int8, device=device)
    check("qg_gen_i8", load_library().qg_gen_i8(_ptr(out), n, seed, tensor_id, _stream(out.device)))
    return out[:n]


def gen_uniform_f32(n: int, lo: float, hi: float, seed: int, tensor_id: int, device="cuda") -> torch.Tensor:
    out = torch.empty((n,), dtype=torch.float32, device=device)
    check("qg_gen_uniform_f32",
          load_library().qg_gen_uniform_f32(_ptr(out), n, lo, hi, seed, tensor_id, _stream(out.device)))
    return out


def gen_normal_f32(n: int, seed: int, tensor_id: int, device="cuda") -> torch.Tensor:
    out = torch.empty((n,), dtype=torch.float32, device=device)
    check("qg_gen_normal_f32", load_library().qg_gen_normal_f32(_ptr(out), n, seed, tensor_id, _stream(out.device)))
    return out


def verify_words(actual: torch.Tensor, expected: torch.Tensor, log_cap: int = 16):
    """Device word compare: returns (mismatching words, [(index, expected, actual), ...])."""
    _require_cuda(actual, expected)
    nwords = actual.numel() * actual.element_size() // 4
    counters = torch.zeros((2,), dtype=torch.int64, device=actual.device)
    log = torch.zeros((max(log_cap, 1), 2), dtype=torch.int64, device=actual.device)
    check("qg_verify_words", load_library().qg_verify_words(_ptr(actual), _ptr(expected), nwords, _ptr(counters),
                                                            _ptr(log), log_cap, _stream(actual.device)))
    c = counters.cpu().tolist()
    entries = []
    for idx, packed in log[: min(c[1], log_cap)].cpu().tolist():
        entries.append((idx, packed & 0xFFFFFFFF, (packed >> 32) & 0xFFFFFFFF))
    return c[0], entries


def device_status(device: int = 0) -> int:
    """QG_OK, or QG_ERR_DEVICE_TIMEOUT if a kernel's bounded wait expired (clears it)."""
    return load_library().qg_device_status(device)


class Workload:
    """One workload instance (the qg_ctx of the C ABI): operands, outputs, golden."""

    SLOT_OUT, SLOT_GOLDEN, SLOT_CKSUM = 5, 6, 7

    def __init__(self, fmt: int = QG_FMT_INT8, m: int = 0, n: int = 0, k: int = 0, copies: int = 1,
                 seed: int = 1, out_type: int = QG_OUT_BF16, device: int = 0):
        self.lib = load_library()
        self.device = device
        self.cfg = QGCfg(fmt, m, n, k, out_type, copies, seed)
        h = C.c_void_p()
        code = self.lib.qg_create(C.byref(h), device, C.byref(self.cfg))
        if code != 0:
            raise QGError("qg_create", code, last_error(None))
        self.ctx = h

    def _check(self, where, code):
        return check(where, code, self.ctx)

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.qg_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def ops_per_launch(self) -> float:
        return self.lib.qg_ops_per_launch(self.ctx)

    @property
    def bytes_per_launch(self) -> float:
        return self.lib.qg_bytes_per_launch(self.ctx)

    def fill(self, seed: int):
        self._check("qg_fill", self.lib.qg_fill(self.ctx, seed))

    def golden(self):
        self._check("qg_golden", self.lib.qg_golden(self.ctx))

    def run(self, iters: int = 1, stream=None):
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream(self.device)
        self._check("qg_run", self.lib.qg_run(self.ctx, iters, s))

    def run_graph(self, iters: int = 1, stream=None):
        """run(), as one CUDA graph per (iters, first copy), captured on first use and replayed."""
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream(self.device)
        self._check("qg_run_graph", self.lib.qg_run_graph(self.ctx, iters, s))

    def run_copy(self, copy: int, stream=None):
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream(self.device)
        self._check("qg_run_copy", self.lib.qg_run_copy(self.ctx, copy, s))

    def synchronize(self):
        self._check("qg_synchronize", self.lib.qg_synchronize(self.ctx))

    def verify(self) -> int:
        mm = C.c_uint64()
        self._check("qg_verify", self.lib.qg_verify(self.ctx, C.byref(mm)))
        return mm.value

    def verify_detail(self):
        """(differing words of the last qg_verify's final compare, differences the per-launch
        checks found, launches that ran with a check) -- the parts of the last verify()."""
        w, d, n = C.c_uint64(), C.c_uint64(), C.c_uint64()
        self._check("qg_verify_detail", self.lib.qg_verify_detail(self.ctx, C.byref(w), C.byref(d), C.byref(n)))
        return w.value, d.value, n.value

    def golden_digest(self, copy: int = 0) -> int:
        """64-bit digest of copy `copy`'s golden result (qg_golden_digest): equal on every
        healthy GPU that ran the same workload with the same seed."""
        d = C.c_uint64()
        self._check("qg_golden_digest", self.lib.qg_golden_digest(self.ctx, copy, C.byref(d)))
        return d.value

    def flip_operand_bit(self, copy: int, slot: int, byte: int, bit: int, stream=None):
        """Flip one bit of an operand of copy `copy` on `stream` (a second flip restores it)."""
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream(self.device)
        self._check("qg_flip_operand_bit", self.lib.qg_flip_operand_bit(self.ctx, copy, slot, byte, bit, s))

    def mismatch_log(self, cap: int = 16):
        arr = (QGMismatch * cap)()
        n = self.lib.qg_mismatch_log(self.ctx, arr, cap)
        if n < 0:
            self._check("qg_mismatch_log", n)
        return [(arr[i].index, arr[i].expected, arr[i].actual) for i in range(n)]

    def inject(self):
        self._check("qg_inject", self.lib.qg_inject(self.ctx))

    def tensor_ptr(self, copy: int, slot: int):
        p = C.c_void_p()
        b = C.c_uint64()
        self._check("qg_tensor", self.lib.qg_tensor(self.ctx, copy, slot, C.byref(p), C.byref(b)))
        return p.value, b.value

    def n_operands(self) -> int:
        """Operand slots of this format (the tensors qg_upload copies): 2 for the dense
        formats, 4 for INT8 / FP8 / W4A16, 5 for NVFP4."""
        n = 0
        p = C.c_void_p()
        b = C.c_uint64()
        while n < 5 and self.lib.qg_tensor(self.ctx, 0, n, C.byref(p), C.byref(b)) == 0 and b.value > 0:
            n += 1
        return n

    def tensor(self, copy: int, slot: int, dtype=torch.uint8) -> torch.Tensor:
        """Copy a device tensor of the context to a new CUDA tensor (raw bytes viewed as dtype)."""
        ptr, nbytes = self.tensor_ptr(copy, slot)
        torch.cuda.synchronize(self.device)
        view = torch.as_tensor(_DeviceBytes(ptr, nbytes), device=f"cuda:{self.device}")
        return view.clone().view(dtype)

    def upload(self, copy: int, host_tensors, stream=None):
        """Copy host operands (one per operand slot, in slot order) into copy `copy`."""
        if len(host_tensors) != self.n_operands():
            raise ValueError(f"upload: {len(host_tensors)} host tensors for {self.n_operands()} operand slots")
        arr = (C.c_void_p * len(host_tensors))(*[t.data_ptr() for t in host_tensors])
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream(self.device)
        self._check("qg_upload", self.lib.qg_upload(self.ctx, copy, arr, s))

    def download(self, copy: int, host_out, stream=None):
        s = C.c_void_p(stream.cuda_stream) if stream is not None else _stream(self.device)
        self._check("qg_download", self.lib.qg_download(self.ctx, copy, C.c_void_p(host_out.data_ptr()), s))
