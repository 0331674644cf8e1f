"""The oracle's MXFP4 matvec (mxfp4_fma_matvec_with_group_size,
experts/slots.rs:1239-1287) against the reference's golden."""

import numpy as np
import pytest


def test_mxfp4_reference_golden(oracle):
    """tests/metal.rs:328-380: rows 0x22 (1.0, 1.0) and 0x95 (3.0, -0.5) over
    x = 1..32, E8M0 127 -> [528, 632]."""
    packed = np.array([0x22] * 16 + [0x95] * 16, np.uint8)
    y = oracle.mxfp4_matvec(packed, np.arange(1, 33, dtype=np.float32), np.array([127, 127], np.uint8), 2, 32, 32)
    assert abs(y[0] - 528.0) < 1e-4 and abs(y[1] - 632.0) < 1e-4


def test_mxfp4_e2m1_table_and_scales(oracle):
    """Each nibble value once (low nibble = even column) at scales 2^0, 2^3
    and the e = 0 pattern 2^-127."""
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    vals = mags + [-m for m in mags]
    packed = np.array([n | ((n + 1) % 16) << 4 for n in range(0, 16, 2)] * 4, np.uint8).reshape(1, 32)
    nib = [n for b in packed[0][:16] for n in (b & 15, b >> 4)]
    for e, s in ((127, 1.0), (130, 8.0), (0, 2.0 ** -127)):
        x = np.zeros(32, np.float32)
        x[:32] = 1.0
        y = oracle.mxfp4_matvec(packed.reshape(-1), x, np.array([e], np.uint8), 1, 32, 32)
        assert y[0] == np.float32(sum(vals[n] for n in nib) * s)


def test_mxfp4_non_finite_scale_bails(oracle):
    with pytest.raises(Exception):
        oracle.mxfp4_matvec(np.zeros(16, np.uint8), np.ones(32, np.float32), np.array([255], np.uint8), 1, 32, 32)
