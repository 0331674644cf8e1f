"""The oracle's newer restatements against independent numpy formulations on
random inputs (CPU): topk_vocab (shaders.metal:1796-1831) as a stable sort
by (value desc, id asc) over the allowed ids with non-finite values as -inf,
and the MXFP4 matvec (experts/slots.rs:1239-1287) as a float64 dequantise-
and-dot."""

import numpy as np
import pytest


def _topk_numpy(logits, k, allowed=None):
    v = np.where(np.isfinite(logits), logits, -np.inf).astype(np.float64)
    ids = np.arange(v.size)
    if allowed is not None:
        bits = (allowed[ids >> 5] >> (ids & 31)) & 1
        ids = ids[bits == 1]
    order = ids[np.lexsort((ids, -v[ids]))]
    n = min(k, v.size)
    out_i = np.zeros(n, np.uint32)
    out_v = np.full(n, -np.inf, np.float32)
    m = min(n, order.size)
    out_i[:m] = order[:m]
    out_v[:m] = v[order[:m]]
    return out_i, out_v


@pytest.mark.parametrize("seed", range(12))
def test_topk_vocab_matches_stable_sort(oracle, seed):
    rng = np.random.default_rng(seed)
    V = int(rng.integers(5, 600))
    k = int(rng.integers(1, 40))
    lg = np.round(rng.standard_normal(V) * 3).astype(np.float32)  # ties
    lg[rng.random(V) < 0.05] = np.nan
    lg[rng.random(V) < 0.05] = np.inf
    lg[rng.random(V) < 0.05] = -np.inf
    mask = None
    if seed % 2:
        mask = rng.integers(0, 2**32, (V + 31) // 32, dtype=np.uint64).astype(np.uint32)
        if seed % 4 == 3:
            mask &= np.uint32(0x01010101)  # few allowed ids: slots past them are (0, -inf)
    ids, vals = oracle.topk_vocab(lg, k, mask)
    rid, rval = _topk_numpy(lg, k, mask)
    assert ids.tolist() == rid.tolist()
    assert np.array_equal(vals, rval)


@pytest.mark.parametrize("seed", range(6))
def test_mxfp4_matches_float64(oracle, seed):
    rng = np.random.default_rng(100 + seed)
    rows, cols = int(rng.integers(1, 40)), 32 * int(rng.integers(1, 9))
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(100, 150, (rows, cols // 32), dtype=np.uint8)
    scales[rng.random(scales.shape) < 0.1] = 0
    x = rng.standard_normal(cols).astype(np.float32)
    mags = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float64)
    nib = np.stack([packed & 15, packed >> 4], axis=-1).reshape(rows, cols)
    w = mags[nib & 7] * np.where(nib & 8, -1.0, 1.0)
    s = np.where(scales == 0, 2.0 ** -127, 2.0 ** (scales.astype(np.float64) - 127))
    ref = (w * np.repeat(s, 32, axis=1)) @ x.astype(np.float64)
    y = oracle.mxfp4_matvec(packed.reshape(-1), x, scales.reshape(-1), rows, cols, 32)
    scale = np.maximum(np.abs(ref), np.sqrt(np.mean(ref ** 2)) + 1e-300)
    assert np.max(np.abs(y - ref) / scale) < 1e-5
