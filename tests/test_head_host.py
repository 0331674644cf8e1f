"""The oracle's topk_vocab (shaders.metal:1796-1831) on hand-checked rows:
value descending, the lower id first among equal values, non-finite logits
as -inf, disallowed ids skipped, passes past the allowed ids (0, -inf)."""

import numpy as np


def test_topk_vocab_order_ties_and_non_finite(oracle):
    lg = np.array([1.0, 3.0, np.nan, 3.0, -np.inf, 2.0, 0.5], np.float32)
    ids, vals = oracle.topk_vocab(lg, 5)
    assert ids.tolist() == [1, 3, 5, 0, 6]
    assert vals.tolist() == [3.0, 3.0, 2.0, 1.0, 0.5]
    ids, vals = oracle.topk_vocab(lg, 7)
    assert ids.tolist()[5:] == [2, 4] and np.all(np.isneginf(vals[5:]))  # NaN and -inf count as -inf, by id


def test_topk_vocab_mask_and_exhaustion(oracle):
    lg = np.array([1.0, 3.0, np.nan, 3.0, -np.inf, 2.0, 0.5], np.float32)
    mask = np.array([0b1011010], np.uint32)  # ids 1, 3, 4, 6
    ids, vals = oracle.topk_vocab(lg, 6, mask)
    assert ids.tolist() == [1, 3, 6, 4, 0, 0]
    assert vals[:3].tolist() == [3.0, 3.0, 0.5] and np.all(np.isneginf(vals[3:]))


def test_topk_vocab_clamps_to_vocab(oracle):
    ids, vals = oracle.topk_vocab(np.array([0.25, -1.0], np.float32), 10)
    assert ids.tolist() == [0, 1] and vals.tolist() == [0.25, -1.0]


def test_head_topk_projection(oracle):
    """Logits are the dense bf16 row dots of the LM head."""
    rng = np.random.default_rng(3)
    w = oracle.f32_to_bf16_bits((rng.standard_normal((50, 64)) * 0.1).astype(np.float32)).reshape(50, 64)
    x = rng.standard_normal((2, 64)).astype(np.float32)
    ids, vals, logits = oracle.head_topk(w, x, 5)
    ref = oracle.bf16_bits_to_f32(w).reshape(50, 64).astype(np.float64) @ x.T.astype(np.float64)
    assert np.max(np.abs(logits - ref.T)) < 1e-5
    assert ids[0].tolist() == np.argsort(-ref[:, 0], kind="stable")[:5].tolist()
