"""Device-driven generation through the ops table's launch_persistent_kernel
hook (include/vbs_backend.h:94-98 of the reference, NULL in all of its
backends), steered by the engine's control block vbs_gpu_control_t
(include/vbs_engine.h:31-40).

The engine's own loop (src/vbs_engine.c:240-327) feeds the prompt, takes the
argmax of each step's logits on the host, stores the token, stops on EOS or
max_tokens and feeds the token back. Here the same decisions run on the
device; the tests compare them with vbs_cu_decoder_generate (the device
greedy loop already pinned against the host loop) and with the reference
loop's stop rules.
"""
import ctypes as C

import numpy as np
import pytest

import models

pytestmark = pytest.mark.gpu

PROMPT = [11, 12, 13, 14, 15]


@pytest.fixture(scope="module")
def l8b_2layer(gpu, vbs):
    cfg = dict(models.L8B, n_layers=2, vocab=4096)
    return cfg, vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)


class Run:
    """Buffers of one generation run, allocated through the ops table as the
    engine allocates them (src/vbs_engine.c:255-266)."""

    def __init__(self, vbs, ops, max_tokens, vocab, first_token, eos=None, logits=True):
        self.vbs, self.ops = vbs, ops
        self.dev = ops.get_device(0)
        self.max_tokens, self.vocab = max_tokens, vocab
        self.gen = ops.alloc_buffer(self.dev, max_tokens * 4, False)
        self.lg = ops.alloc_buffer(self.dev, vocab * 4, False) if logits else None
        self.ctl = ops.alloc_buffer(self.dev, C.sizeof(vbs.GpuControl), False)
        c = vbs.GpuControl(state=vbs.PGAE_GENERATE, current_token=first_token, position=0, max_tokens=max_tokens,
                           vocab_size=vocab, eos_token_id=vbs.PGAE_EOS_NONE if eos is None else eos,
                           generated_tokens_dev=self.gen.contents.internal_handle,
                           logits_dev=self.lg.contents.internal_handle if logits else 0)
        assert ops.copy_to_device(self.ctl, C.byref(c), C.sizeof(c))

    def launch(self, dec) -> bool:
        return bool(self.ops.launch_persistent_kernel(self.dev, C.c_void_p(dec.h), self.ctl))

    def control(self):
        c = self.vbs.GpuControl()
        assert self.ops.copy_to_host(C.byref(c), self.ctl, C.sizeof(c))
        return c

    def tokens(self, n):
        out = np.zeros(self.max_tokens, np.uint32)
        assert self.ops.copy_to_host(out.ctypes.data, self.gen, self.max_tokens * 4)
        return [int(t) for t in out[:n]]

    def logits(self):
        out = np.zeros(self.vocab, np.float32)
        assert self.ops.copy_to_host(out.ctypes.data, self.lg, self.vocab * 4)
        return out

    def close(self):
        for b in (self.gen, self.lg, self.ctl):
            if b:
                self.ops.free_buffer(b)


@pytest.mark.parametrize("flags", [0, 8], ids=["persistent", "per_op"])
def test_hook_greedy_matches_device_generate(vbs, gpu, l8b_2layer, flags, clean_errors):
    _, dm = l8b_2layer
    ref = vbs.Decoder(dm, 64, flags)
    want = ref.generate(PROMPT, 24)
    ref.close()
    dec = vbs.Decoder(dm, 64, flags)
    dec.forward(PROMPT[:-1], logits=False)   # the context; the hook feeds the prompt's last token
    run = Run(vbs, gpu, 24, 4096, PROMPT[-1])
    assert run.launch(dec), vbs.last_error()
    c = run.control()
    assert (c.state, c.position) == (vbs.PGAE_EXIT, 24)
    assert run.tokens(24) == want
    assert c.current_token == want[-1]
    # the last step's logits, whose argmax is the last token
    lg = run.logits()
    assert int(np.argmax(lg)) == want[-1]
    # the decoder continues from where the run left it: position = prompt + 23 fed tokens
    assert dec.position == len(PROMPT) + 23
    nxt = dec.forward([want[-1]])
    chk = vbs.Decoder(dm, 64, flags)
    exp = chk.forward(PROMPT + want)
    assert (nxt.view(np.uint32) == exp.view(np.uint32)).all()
    run.close()
    dec.close()
    chk.close()


def test_hook_stops_on_eos(vbs, gpu, l8b_2layer, clean_errors):
    _, dm = l8b_2layer
    ref = vbs.Decoder(dm, 64)
    want = ref.generate(PROMPT, 24)
    ref.close()
    k = next(i for i in range(3, 24) if want[i] not in want[:i])   # the first time this token appears
    dec = vbs.Decoder(dm, 64)
    dec.forward(PROMPT[:-1], logits=False)
    run = Run(vbs, gpu, 24, 4096, PROMPT[-1], eos=want[k])
    assert run.launch(dec), vbs.last_error()
    c = run.control()
    # the EOS token is not stored (src/vbs_engine.c:298); k tokens were
    assert (c.state, c.position) == (vbs.PGAE_EXIT, k)
    assert run.tokens(k) == want[:k]
    # the EOS step ran (its token came from it), the queued steps after it did not
    assert dec.position == len(PROMPT) + k
    assert dec.generate([want[k]], 3) == vbs.Decoder(dm, 64).generate(PROMPT + want[:k + 1], 3)
    run.close()
    dec.close()


def test_hook_refusals(vbs, gpu, l8b_2layer, clean_errors):
    _, dm = l8b_2layer
    dec = vbs.Decoder(dm, 16)
    dec.forward(PROMPT[:-1], logits=False)
    # more steps than the KV cache holds
    run = Run(vbs, gpu, 16, 4096, PROMPT[-1], logits=False)
    assert not run.launch(dec)
    assert "KV capacity" in vbs.last_error()
    vbs.clear_error()
    run.close()
    # a control block that is not in a generation state
    run = Run(vbs, gpu, 4, 4096, PROMPT[-1], logits=False)
    c = run.control()
    c.state = vbs.PGAE_IDLE
    assert gpu.copy_to_device(run.ctl, C.byref(c), C.sizeof(c))
    assert not run.launch(dec)
    vbs.clear_error()
    # and a vocabulary that is not the decoder's
    c.state, c.vocab_size = vbs.PGAE_GENERATE, 512
    assert gpu.copy_to_device(run.ctl, C.byref(c), C.sizeof(c))
    assert not run.launch(dec)
    vbs.clear_error()
    # the decoder was left untouched
    assert dec.position == len(PROMPT) - 1
    run.close()
    dec.close()
