"""The end-to-end path of every workload format through the C ABI: host operands
uploaded into a context filled with OTHER operands (qg_upload), one launch
(qg_run_copy), the result read back (qg_download) -- bitwise equal to the golden
output of a context that generated those operands itself."""
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu

CASES = [
    (pb.QG_FMT_INT8, 256, 512, 256, pb.QG_OUT_BF16, 4),
    (pb.QG_FMT_FP8, 256, 384, 512, pb.QG_OUT_BF16, 4),
    (pb.QG_FMT_NVFP4, 256, 256, 512, pb.QG_OUT_BF16, 5),
    (pb.QG_FMT_W4A16, 4, 1024, 1024, pb.QG_OUT_BF16, 4),
    (pb.QG_FMT_BF16, 256, 256, 256, pb.QG_OUT_BF16, 2),
    (pb.QG_FMT_FP16, 128, 256, 256, pb.QG_OUT_F16, 2),
    (pb.QG_FMT_TF32, 256, 128, 256, pb.QG_OUT_F32, 2),
    (pb.QG_FMT_E4M3, 256, 256, 512, pb.QG_OUT_BF16, 2),
]


@pytest.mark.parametrize("fmt, m, n, k, out_type, nops", CASES,
                         ids=["int8", "fp8", "nvfp4", "w4a16", "bf16", "fp16", "tf32", "e4m3"])
def test_upload_run_download_matches_golden(cuda_device, fmt, m, n, k, out_type, nops):
    with pb.Workload(fmt, m, n, k, seed=7, out_type=out_type) as src, \
         pb.Workload(fmt, m, n, k, seed=8, out_type=out_type) as dst:
        src.fill(7)
        src.golden()
        dst.fill(8)
        assert src.n_operands() == dst.n_operands() == nops
        host_ops = [src.tensor(0, s).cpu().pin_memory() for s in range(nops)]
        golden = src.tensor(0, src.SLOT_GOLDEN).cpu()
        _, out_bytes = dst.tensor_ptr(0, dst.SLOT_OUT)
        host_out = torch.empty((out_bytes,), dtype=torch.uint8).pin_memory()
        stream = torch.cuda.current_stream()
        dst.upload(0, host_ops, stream)
        dst.run_copy(0, stream)
        dst.download(0, host_out, stream)
        torch.cuda.synchronize()
        assert torch.equal(host_out, golden)
        with pytest.raises(ValueError):
            dst.upload(0, host_ops[:-1], stream)
