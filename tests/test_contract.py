"""The drop-in boundary, checked without a GPU.

* The C-ABI library loads on a machine without a driver and exports every
  function include/pantheon_qgemm.h declares.
* The quantized_gemm binary keeps the reference's argv contract
  (ai_workload_template.h:352: fewer than 3 arguments -> exit 1) and, with no
  usable GPU, fails loudly: a reason on stderr, a non-zero exit, and no
  Throughput line (common.h:444-465) -- never a silent CPU fallback.
* The output parser restated from the runner reads the reference's own MOCK
  binary (built from its sources into oracle/_ref) the way the runner does,
  so the GPU tests can hold our binary to the same reader.
"""
import subprocess

import pytest

from tests.contract_parse import parse_kernel_output


def _gpu_visible() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_library_exports_every_header_symbol(qglib):
    from pantheon_b200 import _lib
    declared = _lib.header_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(qglib, s)]
    assert missing == [], f"declared in include/pantheon_qgemm.h but not exported: {missing}"
    assert qglib.qg_abi_version() == 1


def _binaries():
    from pantheon_b200 import BIN_PATH, DECODE_BIN_PATH, MMA_BIN_PATH
    return [(BIN_PATH, "quantized_gemm"), (DECODE_BIN_PATH, "llm_decode"), (MMA_BIN_PATH, "mma_virus")]


def test_binaries_need_three_arguments(qglib):
    """ai_workload_template.h:352-353, llm_decode.cpp:60 and mma_virus.cpp:182: argc < 4 exits 1."""
    for path, _ in _binaries():
        for args in ([], ["0"], ["0", "1"]):
            proc = subprocess.run([str(path), *args], capture_output=True, text=True, timeout=60)
            assert proc.returncode == 1
            assert "Throughput:" not in proc.stdout


@pytest.mark.skipif(_gpu_visible(), reason="checks the no-GPU failure path")
def test_binaries_without_gpu_fail_loudly(qglib):
    for path, name in _binaries():
        proc = subprocess.run([str(path), "0", "1", "5", "--verify"], capture_output=True, text=True, timeout=60)
        assert proc.returncode != 0
        assert "[PANTHEON ERROR]" in proc.stderr
        assert "Throughput:" not in proc.stdout
        assert "Verification: PASS" not in proc.stdout
        status = parse_kernel_output(proc.stdout, proc.stderr, proc.returncode, name)[2]
        assert status == "FAIL"


@pytest.mark.skipif(_gpu_visible(), reason="checks the no-GPU failure path")
def test_python_entry_points_have_no_cpu_fallback(qglib):
    import ctypes as C
    import pantheon_b200 as pb
    h = C.c_void_p()
    cfg = pb._lib.QGCfg(pb.QG_FMT_INT8, 128, 256, 128, 0, 1, 0)
    rc = qglib.qg_create(C.byref(h), 0, C.byref(cfg))
    assert rc == pb._lib.QG_ERR_CUDA
    with pytest.raises(pb.QGError):
        pb.Workload(pb.QG_FMT_INT8, 128, 256, 128)


def test_library_rejects_bad_shapes_before_touching_a_device(qglib):
    import ctypes as C
    import pantheon_b200 as pb
    rc = qglib.qg_gemm_i8(None, None, None, None, None, 0, None, 128, 128, 128, None)
    assert rc == pb._lib.QG_ERR_ARG
    cfg = pb._lib.QGCfg(pb.QG_FMT_INT8, 128, 128, 100, 0, 1, 0)   # K % 16 != 0
    b = C.c_uint64()
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == pb._lib.QG_ERR_ARG
    cfg = pb._lib.QGCfg(pb.QG_FMT_INT8, 8192, 8192, 8192, 0, 1, 0)
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == 0
    # A, B, sa, sb, C and golden (bf16), row checksums and golden checksums, and the
    # per-launch check's fingerprints (one uint32 per row and 256-column tile)
    assert b.value == (8192 * 8192 * 2 + 8 * 8192 + 2 * 8192 * 8192 * 2 + 2 * 4 * 8192 + 4 * 8192 * 32 + 4096)


@pytest.mark.parametrize("gemm_type, why", [("int4", "Unknown --gemm_type"), ("fp64", "Unknown --gemm_type")])
def test_mma_virus_rejects_gemm_types_it_cannot_run(qglib, gemm_type, why):
    """vendor_gemm.h:525-529: an unknown --gemm_type is an error (exit 1), checked before any device call."""
    from pantheon_b200 import MMA_BIN_PATH
    proc = subprocess.run([str(MMA_BIN_PATH), "0", "1", "5", "--gemm_type", gemm_type], capture_output=True, text=True,
                          timeout=60)
    assert proc.returncode == 1
    assert why in proc.stderr
    assert "Throughput:" not in proc.stdout


def test_device_check_without_a_gpu(qglib):
    """qg_device_check reports a missing device as a CUDA error (the binaries then FAIL with the
    reason on stderr); only a GPU that is present but not sm_100 gives QG_ERR_UNSUPPORTED (SKIP)."""
    import torch
    import pantheon_b200 as pb
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert qglib.qg_device_check(0) == pb._lib.QG_ERR_CUDA
    assert pb._lib.last_error()


def test_gemv_rejects_unknown_flags(qglib):
    """qg_gemv_w4a16_ex checks its flags before touching the device."""
    import pantheon_b200 as pb
    fake = 1 << 20   # aligned, never dereferenced: the call returns before any device access
    known = pb.QG_GEMV_WEIGHTS_CONST | pb.QG_GEMV_ACTIVATIONS_CONST
    assert qglib.qg_gemv_w4a16_ex(fake, fake, fake, fake, fake, pb.QG_OUT_BF16, 1, 128, 128, fake, 1 << 20,
                                  known << 1, None) == pb._lib.QG_ERR_ARG
    assert "unknown flags" in pb._lib.last_error()


def test_mma_virus_rejects_small_gemm_dims(qglib):
    """vendor_gemm.h:530-533: --gemm_m/n/k below 16 is an error."""
    from pantheon_b200 import MMA_BIN_PATH
    proc = subprocess.run([str(MMA_BIN_PATH), "0", "1", "5", "--gemm_m", "8"], capture_output=True, text=True,
                          timeout=60)
    assert proc.returncode == 1 and "at least 16" in proc.stderr


def test_dense_formats_size_and_validate(qglib):
    import ctypes as C
    import pantheon_b200 as pb
    b = C.c_uint64()
    # A, B (bf16) and C, golden (bf16) at the 8192^3 default, plus the per-launch
    # check's fingerprints (one uint32 per row and 256-column tile)
    cfg = pb._lib.QGCfg(pb.QG_FMT_BF16, 0, 0, 0, pb.QG_OUT_BF16, 1, 0)
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == 0
    assert b.value == 4 * 8192 * 8192 * 2 + 4 * 8192 * 32 + 4096
    cfg = pb._lib.QGCfg(pb.QG_FMT_TF32, 256, 256, 256, pb.QG_OUT_F32, 2, 0)
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == 0
    assert b.value == 2 * (2 * 256 * 256 * 4 + 2 * 256 * 256 * 4 + 4 * 256) + 4096
    # the fp32 CUDA-core GEMM has no per-launch check
    cfg = pb._lib.QGCfg(pb.QG_FMT_FP32, 256, 256, 256, pb.QG_OUT_F32, 1, 0)
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == 0
    assert b.value == 2 * 256 * 256 * 4 + 2 * 256 * 256 * 4 + 4096
    cfg = pb._lib.QGCfg(pb.QG_FMT_FP16, 256, 256, 100, pb.QG_OUT_F16, 1, 0)   # 200-byte rows
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == pb._lib.QG_ERR_ARG
    cfg = pb._lib.QGCfg(pb.QG_FMT_E4M3, 256, 256, 256, pb.QG_OUT_S32, 1, 0)   # no integer output
    assert qglib.qg_required_bytes(C.byref(cfg), C.byref(b)) == pb._lib.QG_ERR_ARG
    for entry in ("qg_gemm_bf16", "qg_gemm_f16", "qg_gemm_tf32", "qg_gemm_e4m3"):
        assert getattr(qglib, entry)(None, None, 1.0, None, 0, 128, 128, 128, None) == pb._lib.QG_ERR_ARG


def test_runner_parser_on_reference_mock_binary():
    from pathlib import Path
    ref = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "quantized_gemm_mock"
    if not ref.exists():
        pytest.skip("reference MOCK binary not built (oracle/Makefile needs the reference tree)")
    clean = subprocess.run([str(ref), "0", "1", "5", "--verify"], capture_output=True, text=True, timeout=120)
    t, unit, status, err, kept = parse_kernel_output(clean.stdout, clean.stderr, clean.returncode, "quantized_gemm")
    assert status == "PASS" and unit == "ai-ops/s" and t > 0
    bad = subprocess.run([str(ref), "0", "1", "5", "--verify", "--inject_error"], capture_output=True, text=True,
                         timeout=120)
    assert bad.returncode == 1
    assert parse_kernel_output(bad.stdout, bad.stderr, bad.returncode, "quantized_gemm")[2] == "FAIL"


def test_parser_rules():
    assert parse_kernel_output("Throughput:\t12.5   TOPS\n", "", 0, "quantized_gemm")[:3] == (12.5, "TOPS", "PASS")
    assert parse_kernel_output("Throughput: 1 TOPS\nVerification: FAIL (3 mismatches)\n", "", 0)[2] == "FAIL"
    assert parse_kernel_output("Throughput: 1 TOPS\n[SDC FAULT][X] bad\n", "", 0)[2] == "FAIL"
    assert parse_kernel_output("Throughput: nan TOPS\n", "", 0)[2] == "FAIL"
    assert parse_kernel_output("Throughput: 0.0 TOPS\n", "", 0, "quantized_gemm")[2] == "FAIL"
    assert parse_kernel_output("Skipping: no B200\n", "", 0, "quantized_gemm")[2] == "SKIP"
    assert parse_kernel_output("Throughput: 5 TOPS\n", "boom", 1)[2] == "FAIL"
