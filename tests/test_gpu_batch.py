"""Batched decode (vbs_cu_batch_decoder): B sequences in lockstep on a B200.

The reference decodes one sequence per engine (src/vbs_engine.c:240-327).
The batch decoder steps B sequences together, each with its own KV cache,
through the per-op kernels with B rows: the batched tensor-core matvec for
8 sequences, the tcgen05 GEMM for 12. Every sequence's logits must match a
one-sequence per-op decoder fed the same tokens at every step.

Tolerance 2e-3 of max |logit|: the batched paths take x (and the GEMM the
weights) in fp16, the one-sequence decoder a two-level int8 x, on two
Llama-3-8B-width layers.
"""
import numpy as np
import pytest

import models

pytestmark = pytest.mark.gpu

STEPS = 6


@pytest.fixture(scope="module")
def l8b_2layer(gpu, vbs):
    cfg = dict(models.L8B, n_layers=2, vocab=4096)
    return cfg, vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)


def _rel(got, want):
    return float(np.abs(got - want).max() / np.abs(want).max())


@pytest.mark.parametrize("batch", [8, 12], ids=["batched-matvec", "gemm"])
def test_batch_matches_one_sequence_decoders(vbs, l8b_2layer, batch, clean_errors):
    _, dm = l8b_2layer
    toks = [models.splitmix_ints(500 + b, STEPS, 4096) for b in range(batch)]
    bd = vbs.BatchDecoder(dm, 64, batch)
    refs = [vbs.Decoder(dm, 64, vbs.DEC_NO_PERSIST) for _ in range(batch)]
    for t in range(STEPS):
        got, nxt = bd.step([toks[b][t] for b in range(batch)])
        assert bd.position == t + 1
        for b in range(batch):
            want = refs[b].forward([toks[b][t]])
            assert _rel(got[b], want) <= 2e-3, (t, b)
            assert nxt[b] == int(np.argmax(got[b]))   # first maximum
    for d in refs:
        d.close()
    bd.close()


def test_batch_greedy_feedback_and_enqueue(vbs, l8b_2layer, clean_errors):
    """step(None) feeds the previous argmaxes; enqueued steps do the same."""
    _, dm = l8b_2layer
    first = [3, 99, 4000, 17]
    a, b = vbs.BatchDecoder(dm, 32, 4), vbs.BatchDecoder(dm, 32, 4)
    _, nxt = a.step(first, logits=False)
    for _ in range(3):
        _, nxt = a.step(None, logits=False)
    b.step(first, logits=False)
    b.enqueue_steps(2)
    lg_b, nxt_b = b.step(None)
    assert (a.position, b.position) == (4, 4)
    assert nxt_b == nxt
    # the same tokens fed by hand continue identically
    c = vbs.BatchDecoder(dm, 32, 4)
    seq = [first]
    for _ in range(4):   # the same four steps
        _, n = c.step(seq[-1], logits=False)
        seq.append(n)
    assert seq[-1] == nxt
    for d in (a, b, c):
        d.close()


def test_batch_refusals(vbs, l8b_2layer, clean_errors):
    _, dm = l8b_2layer
    for bad in (0, 65):
        with pytest.raises(vbs.VbsError):
            vbs.BatchDecoder(dm, 16, bad)
        vbs.clear_error()
    d = vbs.BatchDecoder(dm, 2, 2)
    d.step([1, 2], logits=False)
    d.step(None, logits=False)
    with pytest.raises(vbs.VbsError, match="KV capacity"):
        d.step(None, logits=False)
    vbs.clear_error()
    with pytest.raises(vbs.VbsError):
        d.step([1, 4096])   # token out of the vocabulary
    vbs.clear_error()
    d.close()
