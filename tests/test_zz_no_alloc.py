"""vbs_cu_attention_static, the entry point with a fixed per-device scratch
and no device allocation, against vbs_cu_attention on the same inputs.

Two consecutive calls each: the second shows that the first left the
scratch's merge counters at zero. The file name sorts last so the check
also runs after every other GPU test in one session; it passes alone too.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_gpu(gpu):
    import torch
    return torch


def _tol_ok(got, want):
    return bool(np.all(np.abs(got - want) <= 1e-4 + 1e-3 * np.abs(want)))   # the attention tolerance of test_gpu_kernels


# (4096, 32, 32, 8, 128): two splits would need 2.2 MB, so the static entry
# point drops to one; (16, 64, 64, 8, 128): one split, whose result needs no
# scratch at all, although the partials of even that split would not fit.
@pytest.mark.parametrize("ctx,batch,nqh,nkh,hd", [(4096, 1, 32, 8, 128), (512, 16, 32, 8, 128), (777, 2, 16, 2, 64),
                                                  (4096, 32, 32, 8, 128), (16, 64, 64, 8, 128)])
def test_static_scratch_matches_allocating_entry_point(vbs, torch_gpu, ctx, batch, nqh, nkh, hd, clean_errors):
    torch = torch_gpu
    g = torch.Generator(device="cuda").manual_seed(ctx * 7 + batch)
    kc = torch.randn((batch, ctx, nkh * hd), generator=g, device="cuda").half()
    vc = torch.randn((batch, ctx, nkh * hd), generator=g, device="cuda").half()
    q = torch.randn((batch, nqh * hd), generator=g, device="cuda")
    ref = torch.empty((batch, nqh * hd), dtype=torch.float32, device="cuda")
    scale = float(np.float32(1) / np.sqrt(np.float32(hd)))
    args = (ctx, 0, ctx, nqh, nkh, hd, scale)
    vbs.attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ref.data_ptr(), *args, batch=batch,
                  kv_batch_stride=ctx * nkh * hd)
    torch.cuda.synchronize()
    want = ref.cpu().numpy()
    for _ in range(2):
        out = torch.full((batch, nqh * hd), float("nan"), dtype=torch.float32, device="cuda")
        vbs.attention_static(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), *args, batch=batch,
                             kv_batch_stride=ctx * nkh * hd)
        torch.cuda.synchronize()
        assert _tol_ok(out.cpu().numpy(), want)
