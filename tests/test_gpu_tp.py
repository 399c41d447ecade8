"""Tensor parallelism on real GPUs, one process per GPU. Each rank builds
its Megatron shard of the same seeded two-layer 8B-width model
(`synth_llama(tp_rank, tp_world)`), the ranks join one NCCL communicator
(unique id broadcast over gloo), and the TP decoder's logits (o_proj/down
partials summed across ranks, output rows all-gathered) are compared step by
step with a single-GPU decoder on the unsharded model. Both ways of summing
are covered: peer memory (the default: the matvec epilogue stores into every
rank's slots over NVLink, the next kernel waits for the flags) and NCCL's
all-reduce (VBS_CU_DEC_TP_NCCL, the reference collective). Skipped with fewer
GPUs than ranks: two ranks never share one GPU."""
import os
import queue
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import models

pytestmark = pytest.mark.gpu

TOKENS = [17, 2044, 5, 4000, 9, 9, 123]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q, flags):
    import sys
    import datetime
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "tests")]
    import ctypes as C
    import torch
    import torch.distributed as dist
    import vbs_b200 as vbs
    import models as mdl
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
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
        dec = vbs.Decoder(model, 64, flags)
        out = [dec.forward([t]).copy() for t in TOKENS]
        dec.reset()
        toks = dec.generate([11, 12, 13], 8)
        if rank == 0:
            q.put(("ok", out, toks, (dec.kernels_per_step, dec.tp_mode)))
        dist.barrier()
    except Exception as e:  # reported to the parent; the other ranks fail their next collective
        q.put(("error", f"rank {rank}: {e!r}", None, None))
    finally:
        if dec is not None:
            dec.close()   # the graph holding NCCL calls goes before the communicator
        vbs.lib().vbs_cu_tp_finalize()
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["persistent", "peer-memory", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decoder_matches_single_gpu(vbs, gpu, world, mode):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if world > 2 and mode == "nccl":
        pytest.skip("the NCCL check runs at 2 ranks")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    # persistent: the one-launch step kernel with its exchanges over peer
    # memory; peer-memory / nccl: the per-op kernels with either sum
    flags = {"persistent": 0, "peer-memory": vbs.DEC_NO_PERSIST, "nccl": vbs.DEC_NO_PERSIST | vbs.DEC_TP_NCCL}[mode]
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, flags)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        status, out, toks, kps = q.get(timeout=600)
    except queue.Empty:
        status, out = "error", "no result within 600 s"
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert status == "ok", out
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    cfg = dict(models.L8B, n_layers=2, vocab=4096)
    ref_model = vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=99)
    ref = vbs.Decoder(ref_model, 64)
    for i, t in enumerate(TOKENS):
        want = ref.forward([t])
        err = np.abs(out[i] - want).max() / np.abs(want).max()
        assert err <= 2e-3, f"step {i}: rel err {err}"
    ref.close()
    ref2 = vbs.Decoder(ref_model, 64)
    assert toks == ref2.generate([11, 12, 13], 8)
    ref2.close()
    kernels, tp_mode = kps
    assert tp_mode == ("peer-memory" if mode == "persistent" else mode)
    assert (kernels == 1) == (mode == "persistent")   # one launch per step, or the per-op kernels
