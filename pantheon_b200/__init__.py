"""pantheon_b200 -- B200-native quantized-GEMM stress workload (sm_100a).

Python side of the C ABI in include/pantheon_qgemm.h.  The workload itself is
the `quantized_gemm` binary (pantheon_b200/lib/quantized_gemm) that Pantheon's
runner launches once per GPU, with its `llm_decode` and `mma_virus` siblings;
this module is the same library seen from Python, for the tests and the
benchmark.

There is no CPU fallback: importing works anywhere, but every compute call
needs the in-tree library (built by `python -m pantheon_b200.build`) and a
B200; otherwise it raises.
"""
from __future__ import annotations

from ._lib import (  # noqa: F401
    LIB_PATH,
    BIN_PATH,
    DECODE_BIN_PATH,
    MMA_BIN_PATH,
    QG_FMT_INT8,
    QG_FMT_FP8,
    QG_FMT_NVFP4,
    QG_FMT_W4A16,
    QG_FMT_BF16,
    QG_FMT_FP16,
    QG_FMT_TF32,
    QG_FMT_E4M3,
    QG_FMT_FP32,
    QG_OUT_BF16,
    QG_OUT_F32,
    QG_OUT_S32,
    QG_OUT_F16,
    QG_GEMV_WEIGHTS_CONST,
    QG_GEMV_ACTIVATIONS_CONST,
    QGError,
    load_library,
)
from .ops import (  # noqa: F401
    Workload,
    device_status,
    gemm_fp8_b128,
    gemm_bf16,
    gemm_f16,
    gemm_tf32,
    gemm_f32,
    gemm_e4m3,
    gemm_i8,
    gemm_nvfp4,
    gen_dense,
    gen_nvfp4,
    nvfp4_sf_bytes,
    gen_fp8,
    gemv_w4a16,
    gemv_w4a16_workspace_bytes,
    gen_i8,
    gen_w4a16,
    gen_normal_f32,
    gen_uniform_f32,
    verify_words,
)

__all__ = [
    "LIB_PATH", "BIN_PATH", "DECODE_BIN_PATH", "MMA_BIN_PATH", "QGError", "load_library", "Workload",
    "device_status", "gemm_i8", "gemm_fp8_b128", "gemm_bf16", "gemm_f16", "gemm_tf32", "gemm_f32", "gemm_e4m3", "gen_dense",
    "gen_fp8", "gemm_nvfp4", "gen_nvfp4", "nvfp4_sf_bytes", "gemv_w4a16", "gemv_w4a16_workspace_bytes",
    "gen_w4a16", "gen_i8", "gen_uniform_f32", "gen_normal_f32", "verify_words",
    "QG_FMT_INT8", "QG_FMT_FP8", "QG_FMT_NVFP4", "QG_FMT_W4A16",
    "QG_FMT_BF16", "QG_FMT_FP16", "QG_FMT_TF32", "QG_FMT_E4M3", "QG_FMT_FP32",
    "QG_OUT_BF16", "QG_OUT_F32", "QG_OUT_S32", "QG_OUT_F16", "QG_GEMV_WEIGHTS_CONST", "QG_GEMV_ACTIVATIONS_CONST",
]
