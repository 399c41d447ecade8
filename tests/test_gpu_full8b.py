"""The benchmarked model itself, at full size.

bench.py times the Llama-3-8B shape (32 layers, dim 4096, 32/8 heads, FFN
14336, vocab 128256; Q4_K attention and gate/up, Q6_K down, output and
embedding; seed 2024) after a 4096-token prompt. The other decoder tests cut
that model (two layers, a small vocabulary); these run the full instance:

* its first two steps through the persistent step kernel against the
  oracle with the engine's semantics (exact dequant, double sums, fp16 KV;
  src/vbs_host_math.h:170-267), over the whole 128256-row Q6_K output
  projection;
* after the bench's 4096-token prompt (batched prefill), 8 teacher-forced
  steps past position 4096 through the persistent step kernel against the
  per-op kernels (a separate code path: separate matvec, attention with its
  own split count, separate cache layout), then 8 greedy tokens of each.
"""
import numpy as np
import pytest

import models

pytestmark = pytest.mark.gpu

CTX = 4096


@pytest.fixture(scope="module")
def l8b(gpu, vbs):
    dm = vbs.synth_llama(models.shape_of(models.L8B), models.L8B_TYPES, seed=2024)
    yield dm
    del dm


def _rel(got, want):
    return float(np.abs(got - want).max() / np.abs(want).max())


def test_full_8b_first_steps_vs_engine_oracle(vbs, orc, l8b, clean_errors):
    dec = vbs.Decoder(l8b, 8)
    assert dec.kernels_per_step == 1
    st = orc.OrcState(models.host_model_from_device(models.L8B, l8b), 8, 1)
    for t in (128000, 9906):
        got, want = dec.forward([t]), st.step(t)
        assert _rel(got, want) <= 2e-3, t
        assert int(np.argmax(got)) == int(np.argmax(want)) or \
            np.sort(want)[-1] - np.sort(want)[-2] <= 4e-3 * np.abs(want).max()
    dec.close()


def test_full_8b_persistent_vs_per_op_past_4096(vbs, l8b, clean_errors):
    prompt = models.splitmix_ints(4096, CTX, models.L8B["vocab"])   # the bench's prompt
    a = vbs.Decoder(l8b, CTX + 24)
    b = vbs.Decoder(l8b, CTX + 24, vbs.DEC_NO_PERSIST)
    assert a.kernels_per_step == 1 and b.kernels_per_step > 1
    a.prefill(prompt)
    b.prefill(prompt)
    assert a.position == b.position == CTX
    forced = models.splitmix_ints(77, 8, models.L8B["vocab"])
    for i, t in enumerate(forced):
        la, lb = a.forward([t]), b.forward([t])
        assert _rel(la, lb) <= 1e-3, (i, _rel(la, lb))
    # greedy: the step kernel's tokens, then the per-op kernels fed the same
    # tokens must pick each of them (unless the per-op logits hold a near-tie
    # within the tolerance, which would make the pick arbitrary)
    toks = a.generate([forced[-1]], 8)
    lb = b.forward([forced[-1]])
    for i, t in enumerate(toks):
        best = int(np.argmax(lb))
        gap = float(lb[best] - lb[t])
        assert best == t or gap <= 2e-3 * np.abs(lb).max(), (i, best, t, gap)
        if i + 1 < len(toks):
            lb = b.forward([t])
    a.close()
    b.close()
