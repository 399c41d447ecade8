"""The oracle restatement pinned to the reference's outputs (fixtures made
by tests/golden/make_golden.py from the reference compiled unmodified)."""
import ctypes as C
import hashlib

import numpy as np
import pytest


@pytest.mark.parametrize("t", [2, 3, 8, 12, 14, 1])
def test_dequant_bit_exact(orc, golden, t):
    blob, want = golden[f"dq_in_{t}"], golden[f"dq_out_{t}"]
    got = orc.dequant(t, blob)
    assert got.view(np.uint32).tolist() == want.view(np.uint32).tolist()


def test_half_conversions(orc, golden):
    L = orc.lib()
    allh = np.array([L.orc_f16_to_f32(h) for h in range(65536)], dtype=np.float32)
    assert hashlib.sha256(allh.view(np.uint32).tobytes()).digest() == golden["f16_to_f32_sha"].tobytes()
    got = np.array([L.orc_f32_to_f16(float(v)) for v in golden["f32_to_f16_in"]], dtype=np.uint16)
    assert (got == golden["f32_to_f16_out"]).all()


def test_host_math_ops(orc, golden):
    L = orc.lib()
    y = np.empty(384, np.float32)
    L.orc_rms_norm(orc.ptr(golden["rms_x"]), orc.ptr(golden["rms_w"]), orc.ptr(y), 384, 1e-5)
    assert (y == golden["rms_y"]).all()
    for th in (10000, 500000):
        v = golden[f"rope_in_{th}"].copy()
        L.orc_rope(orc.ptr(v), 7, 64, 4, float(th))
        assert (v == golden[f"rope_out_{th}"]).all()
    o = np.empty(777, np.float32)
    L.orc_silu_mul(orc.ptr(golden["silu_g"]), orc.ptr(golden["silu_u"]), orc.ptr(o), 777)
    assert (o == golden["silu_out"]).all()


@pytest.mark.parametrize("tag", ["small", "l3"])
def test_attention(orc, golden, tag):
    nqh, nkh, hd, seq, layer, mc = map(int, golden[f"attn_{tag}_dims"])
    out = orc.attention(golden[f"attn_{tag}_q"], golden[f"attn_{tag}_kc"], golden[f"attn_{tag}_vc"], seq, layer, mc,
                        nqh, nkh, hd, float(np.float32(1.0) / np.sqrt(np.float32(hd))))
    assert (out == golden[f"attn_{tag}_out"]).all()


@pytest.mark.parametrize("t", [0, 1, 2, 3, 8, 12, 14])
def test_linear_tile(orc, golden, t):
    y = orc.linear_tile(golden[f"lin_w_{t}"], t, golden[f"lin_x_{t}"], 24, 512)
    assert (y == golden[f"lin_y_{t}"]).all()


def test_hot_kernels(orc, golden):
    L = orc.lib()
    y = np.empty(20, np.float32)
    L.orc_cpu_matvec_q8_0(orc.ptr(golden["hot_w"]), 20, 256, orc.ptr(golden["hot_xq"]), orc.ptr(golden["hot_qd"]),
                          orc.ptr(y))
    assert (y == golden["hot_y"]).all()
    L.orc_cpu_matvec_f32(orc.ptr(golden["hotf_w"]), 20, 688, orc.ptr(golden["hotf_x"]), orc.ptr(y))
    assert (y == golden["hotf_y"]).all()


def test_tiny_greedy_tokens(orc, tiny_gguf, tiny_golden):
    """vbs_cpu semantics (mode 0) reproduce the reference CLI's 64 greedy
    tokens and its final logits bit for bit."""
    hm = orc.load_gguf_host(tiny_gguf)
    st = orc.OrcState(hm, 128, 0)
    toks = st.generate(tiny_golden["prompt"], 64)
    assert toks == tiny_golden["generated"]
    # final logits: after feeding the 63rd generated token
    st2 = orc.OrcState(hm, 128, 0)
    for t in tiny_golden["prompt"]:
        st2.step(t, logits=False)
    lg = None
    for t in tiny_golden["generated"][:-1]:
        lg = st2.step(t)
    want = np.array(tiny_golden["final_logits"], dtype=np.float32)
    np.testing.assert_array_equal(lg, want)
