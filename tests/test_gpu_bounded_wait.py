"""Bounded waits of the persistent step kernel run out without hanging.

Every wait in the step kernel (mbarriers, grid barriers, tensor-parallel
exchange words, attention head counters) gives up after a limit of global
time, records DERR_TIMEOUT_* in the device error word and unwinds every CTA.
These tests make a wait run out on purpose, without a fault: on one GPU, CTA
0 withholds its arrival at one grid barrier (vbs_cu_decoder_set_wait_test);
on two GPUs, rank 1 stops launching steps between two steps (no kernel of
it in flight) while rank 0 keeps going. Each checks that the call returns
the timeout error within the shortened limit and that the GPU context stays
usable: the same decoder, and a fresh one, then give bit-identical logits.
"""
import os
import queue
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

import models

pytestmark = pytest.mark.gpu

TOKENS = [17, 2044, 5]


@pytest.fixture(scope="module")
def l8b_2layer(gpu, vbs):
    cfg = dict(models.L8B, n_layers=2, vocab=4096)
    return cfg, vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)


# op index 5 * layer + {0 QKV, 1 ATTN, 2 O, 3 GU, 4 DOWN}; 10 is the output
# projection of the two-layer model. The plain instance takes a grid barrier
# before each of these; the tensor-parallel instance (DEC_WORDS) before ATTN.
@pytest.mark.parametrize("flags,drop_op", [(0, 2), (0, 7), (0, 10), (32, 6)], ids=["O", "O-layer1", "OUT", "words-ATTN"])
def test_wait_runs_out_and_context_survives(vbs, l8b_2layer, flags, drop_op, clean_errors):
    _, dm = l8b_2layer
    ref = vbs.Decoder(dm, 32)
    want = ref.forward(TOKENS)
    ref.close()
    dec = vbs.Decoder(dm, 32, flags)
    dec.set_wait_test(20_000_000, drop_op)   # 20 ms
    t0 = time.perf_counter()
    with pytest.raises(vbs.VbsError, match="bounded wait expired"):
        dec.forward(TOKENS[:1])
    assert time.perf_counter() - t0 < 1.0   # the 20 ms limit, not the default 2 s
    vbs.clear_error()
    # the same decoder, back at the default limit and position 0
    dec.set_wait_test(2_000_000_000)
    dec.reset()
    got = dec.forward(TOKENS)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    dec.close()
    fresh = vbs.Decoder(dm, 32)
    assert (fresh.forward(TOKENS).view(np.uint32) == want.view(np.uint32)).all()
    fresh.close()


def test_wait_test_needs_the_step_kernel(vbs, l8b_2layer, clean_errors):
    _, dm = l8b_2layer
    dec = vbs.Decoder(dm, 16, vbs.DEC_NO_PERSIST)
    with pytest.raises(vbs.VbsError, match="persistent"):
        dec.set_wait_test(20_000_000, 2)
    vbs.clear_error()
    dec.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    """Rank 1 runs two steps and stops launching; rank 0 runs a third step,
    whose exchange waits for rank 1's words and must run out."""
    import ctypes as C
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "tests")]
    import torch
    import torch.distributed as dist
    import vbs_b200 as vbs
    import models as mdl
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    dec = None
    try:
        assert vbs.ops().init(), vbs.last_error()
        idb = (C.c_uint8 * 128)()
        if rank == 0:
            vbs.check(vbs.lib().vbs_cu_tp_unique_id(idb), "tp unique id")
        obj = [bytes(idb)]
        dist.broadcast_object_list(obj, src=0)
        idb = (C.c_uint8 * 128).from_buffer_copy(obj[0])
        vbs.check(vbs.lib().vbs_cu_tp_init(rank, world, idb), "tp init")
        cfg = dict(mdl.L8B, n_layers=2, vocab=4096)
        model = vbs.synth_llama(mdl.shape_of(cfg), mdl.L8B_TYPES, seed=99, tp_rank=rank, tp_world=world)
        dec = vbs.Decoder(model, 64)
        dec.set_wait_test(50_000_000)   # 50 ms
        dec.forward(TOKENS[:2])          # both ranks, in step
        dist.barrier()                   # no kernel of either rank in flight from here
        result = ("ok", None)
        if rank == 0:
            t0 = time.perf_counter()
            try:
                dec.forward(TOKENS[2:3])
                result = ("error", "rank 0's step returned without its peer")
            except vbs.VbsError as e:
                dt = time.perf_counter() - t0
                result = ("ok", (str(e), dt)) if "bounded wait expired" in str(e) and dt < 2.0 else ("error", f"{e} after {dt:.3f} s")
            vbs.clear_error()
            q.put(result)
        dist.barrier()                   # rank 1 keeps its region alive until rank 0 is done
    except Exception as e:
        q.put(("error", f"rank {rank}: {e!r}"))
    finally:
        if dec is not None:
            dec.close()
        vbs.lib().vbs_cu_tp_finalize()
        dist.destroy_process_group()


def test_peer_that_stops_launching_times_out(vbs, gpu):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        status, info = q.get(timeout=300)
    except queue.Empty:
        status, info = "error", "no result within 300 s"
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert status == "ok", info
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
