"""The decode program on a B200 through the C ABI.

* Tiny model, strict mode: the 64 greedy tokens of the reference's CPU
  path (vbs-cpu, golden fixture) exactly.
* Tiny model, fast mode: logits step by step against the oracle with the
  engine's semantics (exact dequant, double sums, fp16 KV cache), the path
  the reference's GPU backends implement; teacher-forced so one near-tie
  cannot end the comparison.
* An 8B-width model (two Llama-3-8B layers, Q4_K/Q6_K, vocab cut to 4096)
  against the same oracle; two Llama-3-70B layers and a 6144-wide model,
  wider than one stage, through the step kernel.
* Graph replay, plain launches and PDL give identical bits; the on-device
  greedy loop equals the host-driven one.
"""
import numpy as np
import pytest

import models

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_dev(gpu, vbs, tiny_gguf):
    return vbs.upload_gguf(tiny_gguf)


def test_tiny_strict_greedy_matches_reference(vbs, tiny_dev, tiny_golden, clean_errors):
    dec = vbs.Decoder(tiny_dev, 128, vbs.DEC_STRICT)
    toks = dec.generate(tiny_golden["prompt"], 64)
    assert toks == tiny_golden["generated"]
    dec.close()


def test_tiny_strict_final_logits(vbs, tiny_dev, tiny_golden, clean_errors):
    dec = vbs.Decoder(tiny_dev, 128, vbs.DEC_STRICT)
    lg = dec.forward(list(tiny_golden["prompt"]) + list(tiny_golden["generated"][:-1]))
    want = np.array(tiny_golden["final_logits"], np.float32)
    # only expf/powf/sinf/cosf differ (CUDA's vs glibc's, <= 2 ulp)
    assert np.abs(lg - want).max() <= 1e-5 * np.abs(want).max()
    dec.close()


def _teacher_forced(dec, state, tokens, tol):
    worst = 0.0
    for t in tokens:
        got = dec.forward([t])
        want = state.step(t)
        err = np.abs(got - want).max() / np.abs(want).max()
        worst = max(worst, err)
        assert err <= tol, f"step {t}: rel err {err}"
    return worst


def test_tiny_fast_vs_engine_oracle(vbs, orc, tiny_dev, tiny_gguf, tiny_golden, clean_errors):
    hm = orc.load_gguf_host(tiny_gguf)
    st = orc.OrcState(hm, 128, 1)
    dec = vbs.Decoder(tiny_dev, 128)
    toks = list(tiny_golden["prompt"]) + list(tiny_golden["generated"][:24])
    _teacher_forced(dec, st, toks, 1e-3)
    dec.close()


@pytest.fixture(scope="module")
def l8b_2layer(gpu, vbs):
    cfg = dict(models.L8B, n_layers=2, vocab=4096)
    return cfg, vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)


def _host_model(orc, cfg, dm):
    return models.host_model_from_device(cfg, dm)


@pytest.mark.parametrize("path", ["persistent", "per_op"])
def test_8b_width_vs_engine_oracle(vbs, orc, l8b_2layer, path, clean_errors):
    """Both fast paths: the one-launch persistent step kernel (default) and
    the per-op kernels (VBS_CU_DEC_NO_PERSIST)."""
    cfg, dm = l8b_2layer
    st = orc.OrcState(_host_model(orc, cfg, dm), 64, 1)
    dec = vbs.Decoder(dm, 64, 0 if path == "persistent" else vbs.DEC_NO_PERSIST)
    assert dec.kernels_per_step == (1 if path == "persistent" else 13)
    _teacher_forced(dec, st, [17, 2044, 5, 4000], 2e-3)
    dec.close()


@pytest.mark.parametrize("base", [0, 8])
def test_graph_pdl_plain_identical(vbs, l8b_2layer, base, clean_errors):
    """Graph replay and direct launches give identical bits, for the
    persistent step (base 0) and the per-op kernels (base NO_PERSIST)."""
    _, dm = l8b_2layer
    toks = [1, 2, 3, 4, 5, 6]
    outs = []
    for flags in (0, vbs.DEC_NO_PDL, vbs.DEC_NO_GRAPH, vbs.DEC_NO_GRAPH | vbs.DEC_NO_PDL):
        dec = vbs.Decoder(dm, 32, flags | base)
        outs.append(dec.forward(toks))
        dec.close()
    for o in outs[1:]:
        assert (o.view(np.uint32) == outs[0].view(np.uint32)).all()


def test_persistent_matches_per_op_long_context(vbs, l8b_2layer, clean_errors):
    """300 positions: the persistent kernel's attention runs on several
    splits per KV head, the new row lands in different stages and warps.
    Logits at every 50th step agree with the per-op kernels within 1e-3."""
    _, dm = l8b_2layer
    toks = models.splitmix_ints(5, 300, 4096)
    a, b = vbs.Decoder(dm, 512), vbs.Decoder(dm, 512, vbs.DEC_NO_PERSIST)
    for i in range(0, 300, 50):
        la, lb = a.forward(toks[i:i + 50]), b.forward(toks[i:i + 50])
        assert np.abs(la - lb).max() <= 1e-3 * np.abs(lb).max(), i
    a.close()
    b.close()


def test_tp_instance_on_one_gpu_identical(vbs, l8b_2layer, clean_errors):
    """The step kernel's tensor-parallel instance (DEC_WORDS: exchange words
    over a local area, no grid barrier after o_proj and down, logits
    gathered as words) gives the plain instance's bits at every step. The
    word tags come from a counter that reset() leaves alone, so the second
    pass over the same positions must not accept the first pass's words."""
    _, dm = l8b_2layer
    toks = models.splitmix_ints(9, 120, 4096)
    a, b = vbs.Decoder(dm, 256, vbs.DEC_WORDS), vbs.Decoder(dm, 256)
    assert a.kernels_per_step == 1 and a.tp_mode == "single"
    for rep in range(2):
        for i in range(0, 120, 40):
            la, lb = a.forward(toks[i:i + 40]), b.forward(toks[i:i + 40])
            assert (la.view(np.uint32) == lb.view(np.uint32)).all(), (rep, i)
        a.reset()
        b.reset()
    assert a.generate([11, 12, 13], 24) == b.generate([11, 12, 13], 24)
    a.close()
    b.close()


# Models wider than one stage's 4096-column chunk: the step kernel streams
# their rows as chunks in consecutive stages (sums accumulated, written
# whole), splits the down projection into up to 7 chunk planes and runs the
# norm prologue in passes. 70B width (8 query heads per KV head), and 6144
# (6 per KV head), whose second row chunk and second prologue pass are
# half-full.
WIDE = {
    "70b": dict(models.L70B, n_layers=2, vocab=4096),
    "w6144": dict(n_layers=2, dim=6144, n_heads=48, n_kv_heads=8, ffn=16384, vocab=4096, eps=1e-5, theta=500000.0),
}


@pytest.fixture(scope="module", params=sorted(WIDE))
def wide_2layer(request, gpu, vbs):
    cfg = WIDE[request.param]
    return cfg, vbs.synth_llama(models.shape_of(cfg), models.L70B_TYPES, seed=71)


def test_wide_model_vs_engine_oracle(vbs, orc, wide_2layer, clean_errors):
    """The persistent step kernel on a model above 4096 columns against
    the oracle, then against the per-op kernels over 200 positions
    (attention over several splits, 8 and 6 query heads per KV head)."""
    cfg, dm = wide_2layer
    st = orc.OrcState(_host_model(orc, cfg, dm), 256, 1)
    dec = vbs.Decoder(dm, 256)
    assert dec.kernels_per_step == 1
    _teacher_forced(dec, st, [17, 2044, 5], 2e-3)
    ref = vbs.Decoder(dm, 256, vbs.DEC_NO_PERSIST)
    ref.forward([17, 2044, 5])
    toks = models.splitmix_ints(23, 200, 4096)
    for i in range(0, 200, 50):
        la, lb = dec.forward(toks[i:i + 50]), ref.forward(toks[i:i + 50])
        assert np.abs(la - lb).max() <= 1e-3 * np.abs(lb).max(), i
    dec.close()
    ref.close()


HD64 = dict(n_layers=2, dim=1024, n_heads=16, n_kv_heads=4, ffn=2816, vocab=2048, eps=1e-5, theta=10000.0)


@pytest.mark.parametrize("wt", ["kquant", "q8_0"])
def test_head_dim_64_vs_engine_oracle(vbs, orc, gpu, wt, clean_errors):
    """head_dim 64 and Q8_0 weights through the persistent step kernel."""
    types = dict(models.L8B_TYPES) if wt == "kquant" else {k: orc.Q8_0 for k in models.L8B_TYPES}
    dm = vbs.synth_llama(models.shape_of(HD64), types, seed=31)
    st = orc.OrcState(_host_model(orc, HD64, dm), 64, 1)
    dec = vbs.Decoder(dm, 64)
    assert dec.kernels_per_step == 1
    _teacher_forced(dec, st, [5, 1000, 77, 2047, 3, 3], 2e-3)
    dec.close()


def test_device_greedy_loop_equals_host_loop(vbs, l8b_2layer, clean_errors):
    _, dm = l8b_2layer
    dec = vbs.Decoder(dm, 64)
    dev_toks = dec.generate([11, 12, 13], 20)
    dec2 = vbs.Decoder(dm, 64)
    lg = dec2.forward([11, 12, 13])
    host_toks = []
    for i in range(20):
        t = int(np.argmax(lg))
        host_toks.append(t)
        if i + 1 < 20:
            lg = dec2.forward([t])
    assert dev_toks == host_toks
    dec.close()
    dec2.close()


def test_device_greedy_loop_large_vocab(vbs, gpu, clean_errors):
    """A vocabulary of 40000 rows spreads the on-device argmax over several
    CTAs (slice maxima merged by the last CTA); the tokens must still be the
    host's first-maximum argmax of the returned logits."""
    cfg = dict(models.L8B, n_layers=1, vocab=40000)
    dm = vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=7)
    dec = vbs.Decoder(dm, 32)
    dev_toks = dec.generate([3, 1, 4], 12)
    dec2 = vbs.Decoder(dm, 32)
    lg = dec2.forward([3, 1, 4])
    host_toks = []
    for i in range(12):
        host_toks.append(int(np.argmax(lg)))
        if i + 1 < 12:
            lg = dec2.forward([host_toks[-1]])
    assert dev_toks == host_toks
    dec.close()
    dec2.close()


def test_context_capacity_is_enforced(vbs, tiny_dev, clean_errors):
    dec = vbs.Decoder(tiny_dev, 8)
    dec.forward([1] * 8, logits=False)
    with pytest.raises(vbs.VbsError):
        dec.forward([1])
    vbs.clear_error()
    dec.reset()
    assert dec.forward([1, 2]).shape == (512,)
    dec.close()


def test_out_of_range_token_rejected(vbs, tiny_dev, clean_errors):
    dec = vbs.Decoder(tiny_dev, 8)
    with pytest.raises(vbs.VbsError):
        dec.forward([512])
    dec.close()
