"""Slice streaming (VBS_CU_DEC_STREAM): the layers' matrices stay in pinned
host memory and every step copies each layer into one of two device slots
while the previous layer's kernels run, as the reference's slice executor
stages tiles through double-buffered windows (src/vbs_slice_executor.c:8-107)
for models above device memory. The kernels are the per-op decode kernels,
so the logits must be bit-identical to the same model resident on the device
(VBS_CU_DEC_NO_PERSIST), step by step, through the batched prefill, and
after a reset."""
import numpy as np
import pytest

import models

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair(gpu, vbs):
    cfg = dict(models.L8B, n_layers=3, vocab=4096)
    dm = vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)
    return dm, vbs.streamed_model(dm)


def _same(a, b):
    return bool((a.view(np.uint32) == b.view(np.uint32)).all())


def test_streamed_steps_bit_identical(vbs, pair, clean_errors):
    dm, hm = pair
    ref = vbs.Decoder(dm, 64, vbs.DEC_NO_PERSIST)
    dec = vbs.Decoder(hm, 64, vbs.DEC_STREAM)
    toks = models.splitmix_ints(3, 12, 4096)
    for t in toks:
        assert _same(dec.forward([t]), ref.forward([t]))
    dec.reset()
    ref.reset()
    assert dec.generate([5, 6, 7], 10) == ref.generate([5, 6, 7], 10)
    dec.close()
    ref.close()


def test_streamed_prefill_bit_identical(vbs, pair, clean_errors):
    dm, hm = pair
    prompt = models.splitmix_ints(4, 37, 4096)
    ref = vbs.Decoder(dm, 64, vbs.DEC_NO_PERSIST)
    dec = vbs.Decoder(hm, 64, vbs.DEC_STREAM)
    assert _same(dec.forward_prompt(prompt), ref.forward_prompt(prompt))
    assert _same(dec.forward([9]), ref.forward([9]))
    dec.close()
    ref.close()


def test_stream_refusals(vbs, pair, clean_errors):
    _, hm = pair
    with pytest.raises(vbs.VbsError, match="slice streaming"):
        vbs.Decoder(hm, 16, vbs.DEC_STREAM | vbs.DEC_STRICT)
    vbs.clear_error()
