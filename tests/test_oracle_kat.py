"""The oracle restatement against the reference's own known-answer dequant
blocks (src/main.c:433-519, `verum-slice --dequant`): a zero block cannot
catch a layout error, so each block puts nonzero scales at the type's real
offsets and checks exact decoded values."""
import struct

import numpy as np


def h(orc, v):
    return orc.lib().orc_f32_to_f16(v)


def put16(blk, off, v):
    blk[off:off + 2] = np.frombuffer(struct.pack("<H", v), dtype=np.uint8)


def test_q4_0_known_block(orc):
    blk = np.zeros(18, np.uint8)
    put16(blk, 0, h(orc, 0.5))
    for i in range(16):
        blk[2 + i] = i | ((15 - i) << 4)
    y = orc.dequant(orc.Q4_0, blk)
    assert y.size == 32 and y[0] == 0.5 * (0 - 8) and y[16] == 0.5 * (15 - 8)


def test_q8_0_known_block(orc):
    blk = np.zeros(34, np.uint8)
    put16(blk, 0, h(orc, 0.125))
    for i in range(32):
        blk[2 + i] = (i * 7 - 80) & 0xFF   # the reference's (int8_t) wrap
    y = orc.dequant(orc.Q8_0, blk)
    assert y[0] == 0.125 * -80 and y[31] == 0.125 * ((31 * 7 - 80) - 256)


def test_q4_k_scale_min_first_layout(orc):
    # d=2, dmin=1 at offset 0; sub-block scales (2,1),(3,0); qs[0]=0x21
    blk = np.zeros(144, np.uint8)
    put16(blk, 0, h(orc, 2.0))
    put16(blk, 2, h(orc, 1.0))
    blk[4], blk[8], blk[5], blk[9] = 2, 1, 3, 0
    blk[16] = 0x21
    y = orc.dequant(orc.Q4_K, blk)
    assert y[0] == 3.0 and y[32] == 12.0


def test_q6_k_known_block(orc):
    blk = np.zeros(210, np.uint8)
    blk[192], blk[194], blk[0], blk[32] = 3, 1, 0x21, 0x05
    put16(blk, 208, h(orc, 2.0))
    y = orc.dequant(orc.Q6_K, blk)
    assert y[0] == -186.0 and y[32] == -54.0


def test_half_round_trip_normals(orc):
    L = orc.lib()
    for v in (1.0, -2.5, 65504.0, 6.1035156e-05, 0.333251953125):
        assert L.orc_f16_to_f32(L.orc_f32_to_f16(v)) == np.float32(v)
