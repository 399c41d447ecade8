"""Kernel parity on a B200 through the C ABI (vbs_cu_*): dequantization and
weight synthesis bit-exact against the oracle, the TMA/MMA matvec and the
split-KV attention within 1e-3 relative of the reference's
double-accumulated host math at the BASELINE shapes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3   # north star: matvec/attention outputs within 1e-3 relative fp32 error


def rel_ok(got, want, tol=TOL):
    """Per element |got - want| <= tol * (|want| + rms(want)): relative to
    the element, with the outputs' RMS as the floor for elements near zero
    (a 4096-term dot product's rounding is set by the row's scale, not by
    how close its sum lands to zero)."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    rms = np.sqrt(np.mean(want * want))
    return bool(np.all(np.abs(got - want) <= tol * (np.abs(want) + rms)))


@pytest.fixture(scope="module")
def torch(gpu):
    import torch as T
    return T


def dev(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


@pytest.mark.parametrize("t", [2, 3, 8, 12, 14, 1])
def test_dequant_golden_bit_exact(vbs, torch, golden, t, clean_errors):
    blob, want = golden[f"dq_in_{t}"], golden[f"dq_out_{t}"]
    d = dev(torch, blob)
    out = torch.empty(want.size, dtype=torch.float32, device="cuda")
    vbs.dequant(t, d.data_ptr(), out.data_ptr(), want.size)
    torch.cuda.synchronize()
    assert (out.cpu().numpy().view(np.uint32) == want.view(np.uint32)).all()


@pytest.mark.parametrize("t", [0, 1, 8, 12, 14])
def test_synth_bytes_match_oracle(vbs, orc, torch, t, clean_errors):
    rows, cols, seed = 37, 2048, 12345 + t
    sc = orc.synth_scale(0.02)
    want = orc.synth_tensor(t, seed, rows, cols, sc, row0=5, col0=512, full_cols=4096)
    d = torch.empty(want.size, dtype=torch.uint8, device="cuda")
    vbs.synth(t, d.data_ptr(), rows, cols, seed, sc, row0=5, col0=512, full_cols=4096)
    torch.cuda.synchronize()
    assert (d.cpu().numpy() == want).all()


@pytest.mark.parametrize("t,rows,cols", [(12, 14336, 4096), (14, 4096, 14336)])
def test_dequant_8b_tensor_bit_exact(vbs, orc, torch, t, rows, cols, clean_errors):
    rb = orc.row_bytes(t, cols)
    w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    vbs.synth(t, w.data_ptr(), rows, cols, 7, orc.synth_scale(0.02))
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    vbs.dequant(t, w.data_ptr(), out.data_ptr(), rows * cols)
    torch.cuda.synchronize()
    want = orc.dequant(t, w.cpu().numpy())
    assert (out.cpu().numpy().view(np.uint32) == want.view(np.uint32)).all()


SWEEP = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


@pytest.mark.parametrize("t", [12, 14])
@pytest.mark.parametrize("rows,cols", SWEEP)
def test_matvec_sweep_b1(vbs, orc, torch, t, rows, cols, clean_errors):
    rb = orc.row_bytes(t, cols)
    w = torch.empty(rows * rb + 256, dtype=torch.uint8, device="cuda")
    vbs.synth(t, w.data_ptr(), rows, cols, 1000 + rows + cols, orc.synth_scale(0.02))
    x = np.random.default_rng(rows ^ cols).standard_normal(cols).astype(np.float32)
    xd = dev(torch, x)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    vbs.matvec(t, w.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    want = orc.linear_tile(w[:rows * rb].cpu().numpy(), t, x, rows, cols)
    assert rel_ok(y.cpu().numpy(), want)


@pytest.mark.parametrize("t", [12, 14, 8])
def test_matvec_batch8(vbs, orc, torch, t, clean_errors):
    rows, cols, B = 4096, 4096, 8
    rb = orc.row_bytes(t, cols)
    w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    vbs.synth(t, w.data_ptr(), rows, cols, 55, orc.synth_scale(0.02))
    x = np.random.default_rng(3).standard_normal((B, cols)).astype(np.float32)
    y = torch.empty((B, rows), dtype=torch.float32, device="cuda")
    xd = dev(torch, x)
    vbs.matvec(t, w.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, batch=B)
    torch.cuda.synchronize()
    wh = w.cpu().numpy()
    for b in (0, 3, 7):
        assert rel_ok(y[b].cpu().numpy(), orc.linear_tile(wh, t, x[b], rows, cols))


@pytest.mark.parametrize("t,rows,cols,B", [(12, 14336, 4096, 8), (14, 4096, 14336, 8), (12, 4096, 14336, 3),
                                           (14, 301, 3328, 5), (12, 19, 512, 2), (14, 1000, 7936, 8),
                                           (12, 33, 4352, 7)])
def test_matvec_batched_tensor_cores(vbs, orc, torch, t, rows, cols, B, clean_errors):
    """The batched kernel (mvb.cu): every batch row against the oracle, for
    ragged batches (sequences beyond B padded), partial 16-row tiles, Q6_K
    rows that are only 2-byte aligned, and rows split into column chunks
    (wider than 4096, summed in chunk order)."""
    rb = orc.row_bytes(t, cols)
    w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    vbs.synth(t, w.data_ptr(), rows, cols, 77 + rows + cols + B, orc.synth_scale(0.02))
    x = np.random.default_rng(rows + B).standard_normal((B, cols)).astype(np.float32)
    y = torch.full((B, rows), float("nan"), dtype=torch.float32, device="cuda")
    xd = dev(torch, x)
    vbs.matvec(t, w.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, batch=B)
    torch.cuda.synchronize()
    wh = w.cpu().numpy()
    yh = y.cpu().numpy()
    for b in range(B):
        assert rel_ok(yh[b], orc.linear_tile(wh, t, x[b], rows, cols)), b


def test_matvec_batched_accumulate(vbs, orc, torch, clean_errors):
    """VBS_CU_MV_ACCUMULATE on the batched path, one chunk and several."""
    for rows, cols in ((64, 4096), (64, 8192)):
        t, B = 12, 4
        rb = orc.row_bytes(t, cols)
        w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
        vbs.synth(t, w.data_ptr(), rows, cols, 9, orc.synth_scale(0.02))
        x = np.random.default_rng(1).standard_normal((B, cols)).astype(np.float32)
        y0 = np.random.default_rng(2).standard_normal((B, rows)).astype(np.float32)
        y = dev(torch, y0.copy())
        vbs.matvec(t, w.data_ptr(), dev(torch, x).data_ptr(), y.data_ptr(), rows, cols, batch=B, flags=vbs.MV_ACCUMULATE)
        torch.cuda.synchronize()
        wh = w.cpu().numpy()
        for b in range(B):
            assert rel_ok(y[b].cpu().numpy(), y0[b] + orc.linear_tile(wh, t, x[b], rows, cols)), (rows, cols, b)


@pytest.mark.parametrize("t,rows,cols", [(8, 1, 32), (8, 17, 96), (8, 100, 4128), (14, 3, 256), (14, 33, 768),
                                         (14, 250, 1792), (12, 1, 256), (12, 19, 512), (12, 301, 3328),
                                         (0, 7, 688), (1, 9, 200), (2, 13, 64), (3, 13, 64)])
def test_matvec_ragged_shapes(vbs, orc, torch, t, rows, cols, clean_errors):
    """Row counts that do not fill a 16-row tile, chunks that do not fill a
    stage, Q6_K / Q8_0 rows that are only 2-byte aligned (head/tail copies)."""
    if t in (2, 3):
        from golden.make_golden import finite_blocks
        wh = finite_blocks(t, rows * cols // 32, np.random.default_rng(rows))
    else:
        wh = orc.synth_tensor(t, 3 * rows + cols, rows, cols, orc.synth_scale(0.05))
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    y = torch.full((rows,), 7.0, dtype=torch.float32, device="cuda")
    want = orc.linear_tile(wh, t, x, rows, cols)
    wd, xd = dev(torch, wh), dev(torch, x)      # keep the device copies alive across the launches
    for flags in (0, vbs.MV_PORTABLE):
        vbs.matvec(t, wd.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, flags=flags)
        torch.cuda.synchronize()
        assert rel_ok(y.cpu().numpy(), want), flags
    # accumulate
    vbs.matvec(t, wd.data_ptr(), xd.data_ptr(), y.data_ptr(), rows, cols, flags=vbs.MV_ACCUMULATE)
    torch.cuda.synchronize()
    assert rel_ok(y.cpu().numpy(), 2 * want)


@pytest.mark.parametrize("t", [12, 14])
def test_ffn_gate_up_fused(vbs, orc, torch, t, clean_errors):
    rows, cols = 14336, 4096
    rb = orc.row_bytes(t, cols)
    wg = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    wu = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
    vbs.synth(t, wg.data_ptr(), rows, cols, 1, orc.synth_scale(0.02))
    vbs.synth(t, wu.data_ptr(), rows, cols, 2, orc.synth_scale(0.02))
    x = np.random.default_rng(4).standard_normal(cols).astype(np.float32)
    nw = (1.0 + 0.1 * np.random.default_rng(5).standard_normal(cols)).astype(np.float32)
    h = torch.empty(rows, dtype=torch.float32, device="cuda")
    xd, nwd = dev(torch, x), dev(torch, nw)
    vbs.ffn_gate_up(t, wg.data_ptr(), wu.data_ptr(), xd.data_ptr(), nwd.data_ptr(), 1e-5, h.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    L = orc.lib()
    xn = np.empty(cols, np.float32)
    L.orc_rms_norm(orc.ptr(x), orc.ptr(nw), orc.ptr(xn), cols, 1e-5)
    g = orc.linear_tile(wg.cpu().numpy(), t, xn, rows, cols)
    u = orc.linear_tile(wu.cpu().numpy(), t, xn, rows, cols)
    want = np.empty(rows, np.float32)
    L.orc_silu_mul(orc.ptr(g), orc.ptr(u), orc.ptr(want), rows)
    assert rel_ok(h.cpu().numpy(), want, 2e-3)


@pytest.mark.parametrize("ctx,batch", [(512, 1), (4096, 1), (32768, 1), (4096, 16), (512, 16)])
def test_attention_sweep(vbs, orc, torch, ctx, batch, clean_errors):
    """32 query / 8 KV heads, head_dim 128, fp16 cache
    ~N(0,1), RoPE theta 5e5 already applied to q (a rotation keeps q normal)."""
    nqh, nkh, hd = 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(ctx + batch)
    kc = torch.randn((batch, ctx, nkh * hd), generator=g, device="cuda").half()
    vc = torch.randn((batch, ctx, nkh * hd), generator=g, device="cuda").half()
    q = torch.randn((batch, nqh * hd), generator=g, device="cuda")
    out = torch.empty((batch, nqh * hd), dtype=torch.float32, device="cuda")
    scale = float(np.float32(1) / np.sqrt(np.float32(hd)))
    vbs.attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), ctx, 0, ctx, nqh, nkh, hd, scale,
                  batch=batch, kv_batch_stride=ctx * nkh * hd)
    torch.cuda.synchronize()
    for b in sorted({0, batch - 1}):
        want = orc.attention(q[b].cpu().numpy(), kc[b].cpu().numpy().view(np.uint16).reshape(-1),
                             vc[b].cpu().numpy().view(np.uint16).reshape(-1), ctx, 0, ctx, nqh, nkh, hd, scale)
        got = out[b].cpu().numpy()
        assert np.all(np.abs(got - want) <= 1e-4 + 1e-3 * np.abs(want))


def test_attention_partial_context(vbs, orc, torch, clean_errors):
    """seq_len shorter than the cache, a later layer, GQA group 4."""
    nqh, nkh, hd, mc, layer, seq = 16, 4, 64, 300, 2, 211
    g = torch.Generator(device="cuda").manual_seed(1)
    kc = torch.randn(((layer + 1) * mc * nkh * hd,), generator=g, device="cuda").half()
    vc = torch.randn(((layer + 1) * mc * nkh * hd,), generator=g, device="cuda").half()
    q = torch.randn((nqh * hd,), generator=g, device="cuda")
    out = torch.empty((nqh * hd,), dtype=torch.float32, device="cuda")
    vbs.attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), seq, layer, mc, nqh, nkh, hd, 0.125)
    torch.cuda.synchronize()
    want = orc.attention(q.cpu().numpy(), kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16), seq,
                         layer, mc, nqh, nkh, hd, 0.125)
    assert np.all(np.abs(out.cpu().numpy() - want) <= 1e-4 + 1e-3 * np.abs(want))


@pytest.mark.parametrize("nqh,nkh,hd,seq,mc", [(8, 1, 256, 300, 301), (64, 8, 128, 1000, 1024), (16, 2, 32, 777, 800),
                                               (4, 4, 64, 50, 64), (8, 8, 128, 1, 16), (32, 8, 128, 17, 40)])
def test_attention_shapes(vbs, orc, torch, nqh, nkh, hd, seq, mc, clean_errors):
    """Head dims 32/64/128 (tensor-core kernel) and 256 (SIMT kernel), GQA
    groups 1, 4 and 8, single-position and ragged contexts."""
    g = torch.Generator(device="cuda").manual_seed(nqh * hd + seq)
    layer = 1
    kc = torch.randn(((layer + 1) * mc * nkh * hd,), generator=g, device="cuda").half()
    vc = torch.randn(((layer + 1) * mc * nkh * hd,), generator=g, device="cuda").half()
    q = torch.randn((nqh * hd,), generator=g, device="cuda")
    out = torch.empty((nqh * hd,), dtype=torch.float32, device="cuda")
    scale = float(np.float32(1) / np.sqrt(np.float32(hd)))
    vbs.attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), seq, layer, mc, nqh, nkh, hd, scale)
    torch.cuda.synchronize()
    want = orc.attention(q.cpu().numpy(), kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16), seq,
                         layer, mc, nqh, nkh, hd, scale)
    assert np.all(np.abs(out.cpu().numpy() - want) <= 1e-4 + 1e-3 * np.abs(want))


def test_attention_peaked_scores(vbs, orc, torch, clean_errors):
    """Large-magnitude q (scores spanning hundreds of log2 units) exercises
    the running-maximum rescale."""
    nqh, nkh, hd, seq = 32, 8, 128, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    kc = torch.randn((seq * nkh * hd,), generator=g, device="cuda").half()
    vc = torch.randn((seq * nkh * hd,), generator=g, device="cuda").half()
    q = 12.0 * torch.randn((nqh * hd,), generator=g, device="cuda")
    out = torch.empty((nqh * hd,), dtype=torch.float32, device="cuda")
    vbs.attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), seq, 0, seq, nqh, nkh, hd, 0.0883883)
    torch.cuda.synchronize()
    want = orc.attention(q.cpu().numpy(), kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16), seq, 0,
                         seq, nqh, nkh, hd, 0.0883883)
    assert np.all(np.abs(out.cpu().numpy() - want) <= 1e-4 + 1e-3 * np.abs(want))


def test_kernel_launch_counter_moves(vbs, torch, clean_errors):
    before = vbs.kernel_launches()
    x = torch.zeros(256, device="cuda")
    w = torch.zeros(144, dtype=torch.uint8, device="cuda")
    y = torch.empty(1, device="cuda")
    vbs.matvec(12, w.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 256)
    torch.cuda.synchronize()
    assert vbs.kernel_launches() == before + 1


def test_lns8_matvec_and_dequant(vbs, orc, torch, clean_errors):
    """The reference's LNS8 type (value = 2^q * scale; linear tiles only,
    src/vbs_host_math.h:111-121, :250-255): bit-exact dequant and the
    portable matvec against the oracle's host math."""
    rng = np.random.default_rng(40)
    rows, cols = 37, 512
    q = rng.integers(0, 128, (rows * cols // 32, 32), dtype=np.uint8)
    s = (rng.random(rows * cols // 32, dtype=np.float32) * np.float32(2.0 ** -122)).astype(np.float32)
    w = np.ascontiguousarray(np.concatenate([q, s.view(np.uint8).reshape(-1, 4)], axis=1).reshape(-1))
    x = rng.standard_normal(cols).astype(np.float32)
    wd = torch.from_numpy(w).cuda()
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    vbs.dequant(vbs.LNS8, wd.data_ptr(), out.data_ptr(), rows * cols)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    vbs.matvec(vbs.LNS8, wd.data_ptr(), torch.from_numpy(x).cuda().data_ptr(), y.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    assert (out.cpu().numpy().view(np.uint32) == orc.dequant(orc.LNS8, w).view(np.uint32)).all()
    want = orc.linear_tile(w, orc.LNS8, x, rows, cols)
    assert np.abs(y.cpu().numpy() - want).max() <= 1e-3 * np.abs(want).max()

