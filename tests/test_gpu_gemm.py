"""The quantized GEMM on the 5th-generation tensor cores (csrc/gemm.cu:
tcgen05.mma kind::f16 into tensor memory, weights dequantized into shared
memory), which serves vbs_cu_matvec above 8 sequences: prompt chunks and
large decode batches. Every sequence's output against the reference's
double-accumulated host math (vbs_host_linear_tile), for Q4_K, Q6_K and
Q8_0, ragged row tiles (rows not a multiple of 128) and ragged token tiles
(batches not a multiple of 512, the tokens of one CTA, and batches over
two such tiles), with and without accumulation.

Tolerance: the tensor cores take fp16 operands, so each weight and each
activation carries one fp16 rounding (2^-11 relative); 2e-3 of
(|want| + rms(want)) per element, the bar the batched prefill holds."""
import numpy as np
import pytest

from test_gpu_kernels import dev, rel_ok

pytestmark = pytest.mark.gpu

TOL_GEMM = 2e-3


@pytest.fixture(scope="module")
def torch(gpu):
    import torch as T
    return T


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("rows,cols,B", [(512, 4096, 128), (300, 1024, 200), (128, 256, 17), (1000, 4096, 9), (256, 2048, 300), (128, 1024, 600)])
def test_gemm_matches_host_math(vbs, orc, torch, t, rows, cols, B, clean_errors):
    rb = orc.row_bytes(t, cols)
    w = torch.empty(rows * rb + 256, dtype=torch.uint8, device="cuda")
    vbs.synth(t, w.data_ptr(), rows, cols, 901 + rows + B, orc.synth_scale(0.02))
    x = np.random.default_rng(rows * 7 + B).standard_normal((B, cols)).astype(np.float32)
    y = torch.full((B, rows), float("nan"), dtype=torch.float32, device="cuda")
    xd = dev(torch, x)
    vbs.matvec(t, w.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, batch=B)
    torch.cuda.synchronize()
    wh = w.cpu().numpy()[: rows * rb]
    yh = y.cpu().numpy()
    for b in sorted({0, 1, B // 2, B - 1}):
        assert rel_ok(yh[b], orc.linear_tile(wh, t, x[b], rows, cols), TOL_GEMM), b


def test_gemm_accumulate(vbs, orc, torch, clean_errors):
    t, rows, cols, B = 12, 256, 4096, 40
    rb = orc.row_bytes(t, cols)
    w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    vbs.synth(t, w.data_ptr(), rows, cols, 5, orc.synth_scale(0.02))
    x = np.random.default_rng(2).standard_normal((B, cols)).astype(np.float32)
    base = np.random.default_rng(3).standard_normal((B, rows)).astype(np.float32)
    y = dev(torch, base)
    vbs.matvec(t, w.data_ptr(), dev(torch, x).data_ptr(), y.data_ptr(), rows, cols, batch=B, flags=vbs.MV_ACCUMULATE)
    torch.cuda.synchronize()
    wh, yh = w.cpu().numpy(), y.cpu().numpy()
    for b in (0, B - 1):
        want = base[b] + orc.linear_tile(wh, t, x[b], rows, cols)
        assert rel_ok(yh[b], want, TOL_GEMM)
