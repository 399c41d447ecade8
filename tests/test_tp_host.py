"""Host-side tensor-parallel logic on CPU with gloo, world_size 2 and 4: each rank
takes its Megatron shard (q/k/v/gate/up/output by rows, o/down by columns,
shard_spec) of seeded tensors, computes its partial with the oracle, and the
all-reduced / gathered result equals the unsharded computation."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "oracle"), str(root / "tests")]
    import torch
    import torch.distributed as dist
    import vbs_b200 as vbs
    import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape = vbs.LlamaShape(1, 512, 8, 4, 1024, 1024)
        sc = orc.synth_scale(0.02)
        x = np.random.default_rng(0).standard_normal(1024).astype(np.float32)
        # column-sharded down projection: partial sums, all-reduced
        rows, cols, r0, c0, fc = vbs.shard_spec("blk.0.ffn_down", shape, rank, world)
        w = orc.synth_tensor(orc.Q4_K, vbs.tensor_seed(1, "blk.0.ffn_down"), rows, cols, sc, r0, c0, fc)
        part = torch.from_numpy(orc.linear_tile(w, orc.Q4_K, x[c0:c0 + cols], rows, cols))
        dist.all_reduce(part)
        # row-sharded output projection: slices, all-gathered
        rows2, cols2, r02, _, _ = vbs.shard_spec("output", shape, rank, world)
        w2 = orc.synth_tensor(orc.Q6_K, vbs.tensor_seed(1, "output"), rows2, cols2, sc, r02, 0, cols2)
        xo = x[:512]
        sl = torch.from_numpy(orc.linear_tile(w2, orc.Q6_K, xo, rows2, cols2))
        parts = [torch.empty_like(sl) for _ in range(world)]
        dist.all_gather(parts, sl)
        if rank == 0:
            wf = orc.synth_tensor(orc.Q4_K, vbs.tensor_seed(1, "blk.0.ffn_down"), 512, 1024, sc)
            full = orc.linear_tile(wf, orc.Q4_K, x, 512, 1024)
            wf2 = orc.synth_tensor(orc.Q6_K, vbs.tensor_seed(1, "output"), 1024, 512, sc)
            full2 = orc.linear_tile(wf2, orc.Q6_K, xo, 1024, 512)
            q.put((float(np.abs(part.numpy() - full).max()), float(np.abs(full).max()),
                   bool((torch.cat(parts).numpy() == full2).all())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_shards_match_full_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    err, scale, gathered_exact = q.get(timeout=10)
    assert err <= 1e-5 * max(scale, 1.0)
    assert gathered_exact


def test_shard_spec_covers_tensor():
    import vbs_b200 as vbs
    shape = vbs.LlamaShape(32, 4096, 32, 8, 14336, 128256)
    for world in (2, 4, 8):
        for name in ("blk.0.attn_q", "blk.0.attn_k", "blk.0.attn_output", "blk.0.ffn_down", "output"):
            specs = [vbs.shard_spec(name, shape, r, world) for r in range(world)]
            full_rows, full_cols, _, _, _ = vbs.shard_spec(name, shape, 0, 1)
            if name.endswith(("attn_output", "ffn_down")):
                assert sum(s[1] for s in specs) == full_cols and all(s[0] == full_rows for s in specs)
                assert all(s[1] % 256 == 0 for s in specs)
            else:
                assert sum(s[0] for s in specs) == full_rows


def test_output_rows_split_evenly_in_rank_order():
    """The decoder gathers the logits in rank order and requires rank r to
    own rows r * vocab .. (r + 1) * vocab - 1 with vocab = vocab_full / world:
    the shards and the model description the package builds satisfy it."""
    import vbs_b200 as vbs
    shape = vbs.LlamaShape(32, 4096, 32, 8, 14336, 128256)
    for world in (2, 4, 8):
        specs = [vbs.shard_spec("output", shape, r, world) for r in range(world)]
        assert all(s[0] == shape.vocab // world for s in specs)
        assert [s[2] for s in specs] == [r * (shape.vocab // world) for r in range(world)]
