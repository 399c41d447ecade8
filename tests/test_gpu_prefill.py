"""Batched prompt pass (vbs_cu_decoder_prefill) on a B200. The reference
feeds a prompt one token at a time (src/main.c:901-904); the prefill runs
up to 512 tokens per pass over the weights (the tcgen05 GEMM) and must leave the same KV cache
behind, to the kernels' rounding:

* against the oracle fed one token at a time: the logits of the prompt's
  last token and of teacher-forced steps after it (which attend to every
  prefilled row), for both cache layouts (persistent and per-op decoders);
* against the same decoder fed token by token, over 556 positions that
  cross a 512-token chunk boundary (and end on a short chunk through the
  batched matvec), and in two prefill calls;
* refused, with the reason, where it does not apply.
"""
import numpy as np
import pytest

import models

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def l8b_2layer(gpu, vbs):
    cfg = dict(models.L8B, n_layers=2, vocab=4096)
    return cfg, vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)


def _host_model(orc, cfg, dm):
    host = {}
    for name, t in dm.tensors.items():
        arr = t.cpu().numpy()
        if name.endswith("norm"):
            host[name] = (orc.F32, 1, cfg["dim"], arr)
        else:
            base = name.split(".")[-1]
            rows, cols, *_ = models.vbs.shard_spec(name, dm.shape, 0, 1)
            host[name] = (dm.types[base], rows, cols, arr[:rows * orc.row_bytes(dm.types[base], cols)])
    return orc.HostModel(cfg, host)


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("path", ["persistent", "per_op"])
def test_prefill_vs_engine_oracle(vbs, orc, l8b_2layer, path, clean_errors):
    """21 prompt tokens: 20 through the prefill (chunks of 8, 8, 4), the
    last through a step; then three teacher-forced steps."""
    cfg, dm = l8b_2layer
    st = orc.OrcState(_host_model(orc, cfg, dm), 64, 1)
    dec = vbs.Decoder(dm, 64, 0 if path == "persistent" else vbs.DEC_NO_PERSIST)
    prompt = models.splitmix_ints(21, 21, 4096)
    for t in prompt[:-1]:
        st.step(t, logits=False)
    dec.prefill(prompt[:-1])
    assert dec.position == 20
    for t in prompt[-1:] + [7, 300, 4095]:
        got, want = dec.forward([t]), st.step(t)
        assert _rel(got, want) <= 2e-3, t
    dec.close()


def test_prefill_matches_token_by_token(vbs, l8b_2layer, clean_errors):
    _, dm = l8b_2layer
    toks = models.splitmix_ints(6, 556, 4096)
    a, b, c = vbs.Decoder(dm, 1024), vbs.Decoder(dm, 1024), vbs.Decoder(dm, 1024)
    lb = b.forward(toks)
    assert _rel(a.forward_prompt(toks), lb) <= 2e-3
    c.prefill(toks[:37])               # two calls: positions carry over
    c.prefill(toks[37:-1])             # chunks of 512 and 6
    assert c.position == 555
    assert _rel(c.forward(toks[-1:]), lb) <= 2e-3
    for t in (1, 2, 3):
        want = b.forward([t])
        assert _rel(a.forward([t]), want) <= 2e-3
        assert _rel(c.forward([t]), want) <= 2e-3
    for d in (a, b, c):
        d.close()


def test_prefill_refusals(vbs, l8b_2layer, tiny_gguf, clean_errors):
    _, dm = l8b_2layer
    dec = vbs.Decoder(dm, 16)
    with pytest.raises(vbs.VbsError, match="capacity"):
        dec.prefill(list(range(17)))
    vbs.clear_error()
    with pytest.raises(vbs.VbsError, match="vocab"):
        dec.prefill([1, 4096])
    vbs.clear_error()
    assert dec.position == 0           # nothing was stored
    dec.close()
    strict = vbs.Decoder(vbs.upload_gguf(tiny_gguf), 16, vbs.DEC_STRICT)
    with pytest.raises(vbs.VbsError, match="strict"):
        strict.prefill([1, 2])
    strict.close()
