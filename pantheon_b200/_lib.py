"""ctypes binding of include/pantheon_qgemm.h (libpantheon_qgemm.so)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libpantheon_qgemm.so"
BIN_PATH = PKG / "lib" / "quantized_gemm"
DECODE_BIN_PATH = PKG / "lib" / "llm_decode"
MMA_BIN_PATH = PKG / "lib" / "mma_virus"
HEADER = PKG.parent / "include" / "pantheon_qgemm.h"

QG_OK = 0
QG_ERR_ARG = -1
QG_ERR_CUDA = -2
QG_ERR_UNSUPPORTED = -3
QG_ERR_DEVICE_TIMEOUT = 1

QG_FMT_INT8, QG_FMT_FP8, QG_FMT_NVFP4, QG_FMT_W4A16 = 0, 1, 2, 3
QG_FMT_BF16, QG_FMT_FP16, QG_FMT_TF32, QG_FMT_E4M3, QG_FMT_FP32 = 4, 5, 6, 7, 8
QG_OUT_BF16, QG_OUT_F32, QG_OUT_S32, QG_OUT_F16 = 0, 1, 2, 3
QG_GEMV_WEIGHTS_CONST = 1
QG_GEMV_ACTIVATIONS_CONST = 2


class QGError(RuntimeError):
    """A C-ABI call returned an error code."""

    def __init__(self, where: str, code: int, message: str):
        super().__init__(f"{where} failed ({code}): {message}")
        self.code = code


class QGCfg(C.Structure):
    _fields_ = [("format", C.c_int32), ("m", C.c_int32), ("n", C.c_int32), ("k", C.c_int32),
                ("out_type", C.c_int32), ("copies", C.c_int32), ("seed", C.c_uint64)]


class QGMismatch(C.Structure):
    _fields_ = [("index", C.c_uint64), ("expected", C.c_uint32), ("actual", C.c_uint32)]


_V = C.c_void_p
_SIGNATURES = {
    "qg_create": (C.c_int, [C.POINTER(_V), C.c_int, C.POINTER(QGCfg)]),
    "qg_required_bytes": (C.c_int, [C.POINTER(QGCfg), C.POINTER(C.c_uint64)]),
    "qg_fill": (C.c_int, [_V, C.c_uint64]),
    "qg_golden": (C.c_int, [_V]),
    "qg_run": (C.c_int, [_V, C.c_int, _V]),
    "qg_run_graph": (C.c_int, [_V, C.c_int, _V]),
    "qg_verify": (C.c_int, [_V, C.POINTER(C.c_uint64)]),
    "qg_verify_detail": (C.c_int, [_V, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "qg_golden_digest": (C.c_int, [_V, C.c_int, C.POINTER(C.c_uint64)]),
    "qg_flip_operand_bit": (C.c_int, [_V, C.c_int, C.c_int, C.c_uint64, C.c_int, _V]),
    "qg_mismatch_log": (C.c_int, [_V, C.POINTER(QGMismatch), C.c_int]),
    "qg_inject": (C.c_int, [_V]),
    "qg_ops_per_launch": (C.c_double, [_V]),
    "qg_bytes_per_launch": (C.c_double, [_V]),
    "qg_upload": (C.c_int, [_V, C.c_int, C.POINTER(_V), _V]),
    "qg_download": (C.c_int, [_V, C.c_int, _V, _V]),
    "qg_run_copy": (C.c_int, [_V, C.c_int, _V]),
    "qg_tensor": (C.c_int, [_V, C.c_int, C.c_int, C.POINTER(_V), C.POINTER(C.c_uint64)]),
    "qg_synchronize": (C.c_int, [_V]),
    "qg_mem_info": (C.c_int, [C.c_int, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "qg_abi_version": (C.c_int, []),
    "qg_last_error": (C.c_int, [_V, C.c_char_p, C.c_size_t]),
    "qg_destroy": (None, [_V]),
    "qg_gemm_i8": (C.c_int, [_V, _V, _V, _V, _V, C.c_int, _V, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gemm_fp8_b128": (C.c_int, [_V, _V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gemm_bf16": (C.c_int, [_V, _V, C.c_float, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gemm_e4m3": (C.c_int, [_V, _V, C.c_float, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gemm_f16": (C.c_int, [_V, _V, C.c_float, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gemm_tf32": (C.c_int, [_V, _V, C.c_float, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gemm_f32": (C.c_int, [_V, _V, C.c_float, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gen_dense": (C.c_int, [C.c_int, _V, C.c_uint64, C.c_uint64, C.c_uint32, _V]),
    "qg_pci_bus_id": (C.c_int, [C.c_int, C.c_char_p, C.c_int]),
    "qg_device_check": (C.c_int, [C.c_int]),
    "qg_gen_fp8": (C.c_int, [_V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_uint32, _V]),
    "qg_gemm_nvfp4": (C.c_int, [_V, _V, _V, _V, C.c_float, C.c_float, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_nvfp4_sf_bytes": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_uint64)]),
    "qg_gen_nvfp4": (C.c_int, [_V, _V, _V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_uint32, _V]),
    "qg_gemv_w4a16_workspace_bytes": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_uint64)]),
    "qg_gemv_w4a16": (C.c_int, [_V, _V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V, C.c_uint64, _V]),
    "qg_gemv_w4a16_ex": (C.c_int, [_V, _V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V, C.c_uint64, C.c_uint,
                                   _V]),
    "qg_gemv_w4a16_noalloc": (C.c_int, [_V, _V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    "qg_gen_w4a16": (C.c_int, [_V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_uint32, _V]),
    "qg_device_status": (C.c_int, [C.c_int]),
    "qg_device_status_detail": (C.c_int, [C.c_int, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                          C.POINTER(C.c_uint32)]),
    "qg_fault_drill_i8": (C.c_int, [_V, _V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int, _V]),
    "qg_verify_words": (C.c_int, [_V, _V, C.c_uint64, _V, _V, C.c_int, _V]),
    "qg_gen_i8": (C.c_int, [_V, C.c_uint64, C.c_uint64, C.c_uint32, _V]),
    "qg_gen_uniform_f32": (C.c_int, [_V, C.c_uint64, C.c_float, C.c_float, C.c_uint64, C.c_uint32, _V]),
    "qg_gen_normal_f32": (C.c_int, [_V, C.c_uint64, C.c_uint64, C.c_uint32, _V]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"QG_API\s+(?:int|void|double)\s+(qg_\w+)\s*\(", text)))


def load_library(path: Path | None = None) -> C.CDLL:
    """Load the in-tree C-ABI library; raise if it was not built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: build it with `python -m pantheon_b200.build` "
                                "(the sm_100a kernels have no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def last_error(ctx=None) -> str:
    buf = C.create_string_buffer(512)
    load_library().qg_last_error(ctx, buf, len(buf))
    return buf.value.decode(errors="replace")


def check(where: str, code: int, ctx=None) -> int:
    if code != QG_OK:
        raise QGError(where, code, last_error(ctx))
    return code
