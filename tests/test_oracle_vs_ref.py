"""Randomised cross-checks of the restatement against the reference built
from its own sources (oracle/_ref). Skipped where the reference was not
compiled (the GPU box carries it only if it was built before the copy)."""
import ctypes as C

import numpy as np
import pytest

from oracle import REF_LIB

pytestmark = pytest.mark.skipif(not REF_LIB.exists(), reason="reference not compiled into oracle/_ref")


@pytest.mark.parametrize("t", [2, 3, 8, 12, 14])
def test_random_blocks(orc, t):
    R = orc.ref()
    rng = np.random.default_rng(t)
    e, b = orc.BLOCK[t]
    for _ in range(200):
        blk = rng.integers(0, 256, b, dtype=np.uint8)
        want = np.empty(e, np.float32)
        R.ref_dequant_block(t, orc.ptr(blk), orc.ptr(want))
        got = orc.dequant(t, blk)
        fin = np.isfinite(want)
        assert (got[fin].view(np.uint32) == want[fin].view(np.uint32)).all()
        assert (np.isnan(got) == np.isnan(want)).all()


def test_f32_to_f16_random_bits(orc):
    R, L = orc.ref(), orc.lib()
    rng = np.random.default_rng(3)
    for bits in rng.integers(0, 2**32, 20000, dtype=np.uint64):
        v = float(np.array([bits], np.uint32).view(np.float32)[0])
        assert L.orc_f32_to_f16(v) == R.ref_f32_to_f16(v)


@pytest.mark.parametrize("t", [0, 8, 12, 14])
def test_linear_tile_offsets_accumulate(orc, t):
    R = orc.ref()
    rows, cols = 9, 512
    w = orc.synth_tensor(t, 11, rows, cols, orc.synth_scale(0.05))
    x = np.random.default_rng(1).standard_normal(cols + 64).astype(np.float32)
    for acc in (0, 1):
        y1 = np.arange(rows + 5, dtype=np.float32)
        y2 = y1.copy()
        assert R.ref_linear_tile(orc.ptr(w), t, orc.ptr(x), orc.ptr(y1), cols, rows, 64, 5, acc) == 0
        assert orc.lib().orc_linear_tile(orc.ptr(w), t, orc.ptr(x), orc.ptr(y2), cols, rows, 64, 5, acc) == 0
        assert (y1 == y2).all()


def _lns8_blocks(rng, nblocks, qmax=128):
    """LNS8 blocks: 32 log2 values in [0, qmax), then an f32 scale."""
    q = rng.integers(0, qmax, (nblocks, 32), dtype=np.uint8)
    s = (rng.random(nblocks, dtype=np.float32) * np.float32(2.0 ** -120)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([q, s.view(np.uint8).reshape(nblocks, 4)], axis=1).reshape(-1))


def test_lns8_dequant_formula(orc):
    """value = 2^q * scale (src/vbs_host_math.h:111-121), q >= 128 -> inf."""
    rng = np.random.default_rng(40)
    blk = _lns8_blocks(rng, 64, qmax=256)
    got = orc.dequant(orc.LNS8, blk)
    q = blk.reshape(64, 36)[:, :32].astype(np.int32)
    s = blk.reshape(64, 36)[:, 32:].copy().view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        # float32 throughout: the exact power 2^q (inf from 128 on, as exp2f), times the scale
        want = (np.ldexp(np.ones(q.shape, np.float32), q) * s).astype(np.float32).reshape(-1)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()


def test_lns8_linear_tile_matches_reference(orc):
    R = orc.ref()
    rng = np.random.default_rng(41)
    rows, cols = 7, 256
    w = _lns8_blocks(rng, rows * cols // 32)
    x = rng.standard_normal(cols).astype(np.float32)
    y1, y2 = np.zeros(rows, np.float32), np.zeros(rows, np.float32)
    assert R.ref_linear_tile(orc.ptr(w), orc.LNS8, orc.ptr(x), orc.ptr(y1), cols, rows, 0, 0, 0) == 0
    assert orc.lib().orc_linear_tile(orc.ptr(w), orc.LNS8, orc.ptr(x), orc.ptr(y2), cols, rows, 0, 0, 0) == 0
    assert (y1 == y2).all()
