"""The ops table on a B200, test for test the reference's backend self-test
(src/vbs_backend_test.c:456-963) driven through g_vbs_cuda_backend exactly
as the bridge and the slice executor call it. Expected values are the
reference's own outputs (tests/golden/golden.npz) or the oracle
restatement pinned to them."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


class Harness:
    def __init__(self, vbs, ops):
        self.vbs, self.ops = vbs, ops
        self.dev = ops.get_device(0)
        self.bufs = []

    def alloc(self, nbytes, shared=False):
        b = self.ops.alloc_buffer(self.dev, nbytes, shared)
        assert b, self.vbs.last_error()
        self.bufs.append(b)
        return b

    def put(self, arr):
        arr = np.ascontiguousarray(arr)
        b = self.alloc(arr.nbytes)
        assert self.ops.copy_to_device(b, arr.ctypes.data, arr.nbytes)
        return b

    def get(self, b, n, dtype=np.float32):
        out = np.empty(n, dtype=dtype)
        assert self.ops.copy_to_host(out.ctypes.data, b, out.nbytes), self.vbs.last_error()
        return out

    def prim(self, kind, args, ptype=None):
        err = C.create_string_buffer(256)
        if ptype is None:
            pipe = self.ops.compile_primitive_pipeline(self.dev, kind, err, 256)
        else:
            pipe = self.ops.compile_embed_pipeline(self.dev, ptype, err, 256)
        assert pipe, err.value
        keep, arr = [], (self.vbs.Arg * len(args))()
        for i, a in enumerate(args):
            if isinstance(a, C.POINTER(self.vbs.Buffer)):
                arr[i] = self.vbs.Arg(self.vbs.ARG_BUFFER, a.contents.internal_handle, 0)
            else:
                v = C.c_float(a) if isinstance(a, float) else C.c_uint32(a)
                keep.append(v)
                arr[i] = self.vbs.Arg(self.vbs.ARG_SCALAR, C.cast(C.pointer(v), C.c_void_p), 4)
        ok = self.ops.dispatch_primitive(self.dev, pipe, arr, len(args), 1, 256)
        self.ops.synchronize_device(self.dev)
        return ok

    def free(self):
        for b in self.bufs:
            self.ops.free_buffer(b)
        self.bufs = []


@pytest.fixture()
def H(vbs, gpu, clean_errors):
    h = Harness(vbs, gpu)
    yield h
    h.free()


def close(got, want, tol_abs, tol_rel):
    return np.all(np.abs(got - want) <= tol_abs + tol_rel * np.abs(want))


def test_device_fields(H):
    d = H.dev.contents
    assert d.type == 1 and d.max_working_set_bytes > 100 << 30 and d.max_buffer_bytes > 0
    assert b"B200" in d.name


def test_copy_roundtrip_1mib(H):
    src = (np.arange(1 << 20, dtype=np.uint64) * 2654435761 >> 24).astype(np.uint8)
    b = H.put(src)
    assert (H.get(b, src.size, np.uint8) == src).all()


def test_shared_buffer_has_pinned_host_ptr(H):
    b = H.alloc(4096, shared=True)
    assert b.contents.host_ptr


def test_add_n1000(H):
    rng = np.random.default_rng(1)
    a, b = rng.uniform(-1, 1, 1000).astype(np.float32), rng.uniform(-1, 1, 1000).astype(np.float32)
    ba, bb, bo = H.put(a), H.put(b), H.alloc(4000)
    assert H.prim(H.vbs.OP_ELEMENTWISE, [ba, bb, bo, 1000])
    assert (H.get(bo, 1000) == a + b).all()


def test_silu_mul_n777(H, golden):
    bg, bu, bo = H.put(golden["silu_g"]), H.put(golden["silu_u"]), H.alloc(777 * 4)
    assert H.prim(H.vbs.OP_ACTIVATION, [bg, bu, bo, 777])
    assert close(H.get(bo, 777), golden["silu_out"], 1e-5, 1e-5)


def test_rms_norm_dim384(H, golden):
    bi, bw, bo = H.put(golden["rms_x"]), H.put(golden["rms_w"]), H.alloc(384 * 4)
    assert H.prim(H.vbs.OP_NORMALIZE, [bi, bw, bo, 384, 1e-5])
    assert close(H.get(bo, 384), golden["rms_y"], 1e-5, 1e-5)


@pytest.mark.parametrize("theta", [10000, 500000])
def test_rope_two_thetas(H, golden, theta):
    bx = H.put(golden[f"rope_in_{theta}"])
    assert H.prim(H.vbs.OP_ROTARY, [bx, 7, 64, 4, float(theta)])
    assert close(H.get(bx, 256), golden[f"rope_out_{theta}"], 1e-5, 1e-5)


@pytest.mark.parametrize("t", [0, 1, 2, 3, 8, 12, 14])
def test_embed_all_types_exact(H, orc, t):
    dim, vocab, tok = 256, 8, 3
    if t in (2, 3):
        from golden.make_golden import finite_blocks
        w = finite_blocks(t, vocab * dim // 32, np.random.default_rng(t))
    else:
        w = orc.synth_tensor(t, 40 + t, vocab, dim, orc.synth_scale(0.5))
    want = orc.dequant(t, w[tok * orc.row_bytes(t, dim):(tok + 1) * orc.row_bytes(t, dim)])
    bw, bo = H.put(w), H.alloc(dim * 4)
    assert H.prim(H.vbs.OP_EMBEDDING, [bw, tok, bo, dim], ptype=t)
    assert (H.get(bo, dim).view(np.uint32) == want.view(np.uint32)).all()


@pytest.mark.parametrize("tag", ["small", "l3"])
def test_kv_store_and_attention(H, orc, golden, tag):
    nqh, nkh, hd, seq, layer, mc = map(int, golden[f"attn_{tag}_dims"])
    kvd = nkh * hd
    # KV store through the CACHE primitive is bit-exact with the reference's
    rng = np.random.default_rng(5)
    k, v = rng.standard_normal(kvd).astype(np.float32), rng.standard_normal(kvd).astype(np.float32)
    kc0 = np.zeros((layer + 1) * mc * kvd, np.uint16)
    bkc, bvc = H.put(kc0), H.put(kc0)
    assert H.prim(H.vbs.OP_CACHE, [H.put(k), H.put(v), bkc, bvc, 2, layer, mc, kvd])
    want_k, want_v = kc0.copy(), kc0.copy()
    orc.lib().orc_cache_store(orc.ptr(k), orc.ptr(v), orc.ptr(want_k), orc.ptr(want_v), 2, layer, mc, kvd)
    assert (H.get(bkc, kc0.size, np.uint16) == want_k).all() and (H.get(bvc, kc0.size, np.uint16) == want_v).all()
    # attention over the golden cache
    bq, bo = H.put(golden[f"attn_{tag}_q"]), H.alloc(nqh * hd * 4)
    bk2, bv2 = H.put(golden[f"attn_{tag}_kc"]), H.put(golden[f"attn_{tag}_vc"])
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    assert H.prim(H.vbs.OP_ATTENTION, [bq, bk2, bv2, bo, seq, layer, mc, nqh, nkh, hd, scale])
    # tolerance of the reference self-test (src/vbs_backend_test.c:786)
    assert close(H.get(bo, nqh * hd), golden[f"attn_{tag}_out"], 1e-4, 1e-4)


def _linear(H, pipe, w, x, rows, cols, staged, col_off=0, row_off=0, accumulate=False, y0=None):
    bx = H.put(x)
    by = H.put(y0 if y0 is not None else np.zeros(rows + row_off, np.float32))
    if staged:
        stage = H.alloc(w.nbytes, shared=True)
        C.memmove(stage.contents.host_ptr, w.ctypes.data, w.nbytes)
        priv = H.alloc(w.nbytes)
        ok = H.ops.dispatch_linear_tile(H.dev, pipe, priv, stage, w.nbytes, bx, by, cols, rows, col_off, row_off,
                                        accumulate)
    else:
        bw = H.put(w)
        ok = H.ops.dispatch_linear_tile(H.dev, pipe, bw, None, 0, bx, by, cols, rows, col_off, row_off, accumulate)
    H.ops.synchronize_device(H.dev)
    assert ok, H.vbs.last_error()
    return H.get(by, rows + row_off)


@pytest.mark.parametrize("staged", [False, True])
@pytest.mark.parametrize("t", [0, 1, 2, 3, 8, 12, 14])
def test_linear_tile_both_conventions(H, golden, t, staged):
    err = C.create_string_buffer(256)
    pipe = H.ops.compile_linear_pipeline(H.dev, t, err, 256)
    assert pipe, err.value
    w, x, want = golden[f"lin_w_{t}"], golden[f"lin_x_{t}"], golden[f"lin_y_{t}"]
    got = _linear(H, pipe, w, x, 24, 512, staged)
    # 1e-3 relative to the row scale (fp32 kernels vs the reference's double sums)
    assert np.all(np.abs(got - want) <= 1e-3 * (np.abs(want) + np.abs(want).max() * 1e-2) + 1e-6)


@pytest.mark.parametrize("t", [0, 12])
def test_linear_offsets_accumulate(H, orc, t):
    rows, cols, half = 4, 512, 256
    rng = np.random.default_rng(9)
    full = orc.synth_tensor(t, 77, rows, cols, orc.synth_scale(0.1))
    x = rng.standard_normal(cols).astype(np.float32)
    want = orc.linear_tile(full, t, x, rows, cols)
    err = C.create_string_buffer(256)
    pipe = H.ops.compile_linear_pipeline(H.dev, t, err, 256)
    rb = orc.row_bytes(t, cols)
    y = np.zeros(rows, np.float32)
    for tile in range(2):
        cb = orc.row_bytes(t, half)
        tw = np.concatenate([full[r * rb + tile * cb:r * rb + (tile + 1) * cb] for r in range(rows)])
        y = _linear(H, pipe, tw, x, rows, half, True, col_off=tile * half, accumulate=(tile == 1), y0=y)
    assert np.all(np.abs(y - want) <= 1e-4 + 1e-3 * np.abs(want))


def test_refusals_are_loud(H):
    err = C.create_string_buffer(256)
    assert not H.ops.compile_linear_pipeline(H.dev, 15, err, 256)   # Q8_K
    assert b"refusal" in err.value
    assert not H.ops.compile_embed_pipeline(H.dev, 40, err, 256)    # LNS8
    assert not H.ops.compile_primitive_pipeline(H.dev, H.vbs.OP_STATE_SPACE, err, 256)


def test_dropped_dispatch_error_fails_next_readback(H, vbs):
    bo = H.alloc(64)
    # NORMALIZE with the wrong argument count: the bridge would drop the
    # False; the latched error must make the next copy_to_host fail.
    assert not H.prim(vbs.OP_NORMALIZE, [bo, bo, 4])
    out = np.empty(16, np.float32)
    assert not H.ops.copy_to_host(out.ctypes.data, bo, 64)
    assert "bad arguments" in vbs.last_error()
    vbs.clear_error()
    assert H.ops.copy_to_host(out.ctypes.data, bo, 64)
