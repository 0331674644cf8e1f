"""Vocab head (LM head + topk_vocab) through the C-ABI against the CPU oracle.

  pbmoe_head_topk   logits = W . x (dense_mmap_fma_matvec_bf16,
                    shaders.metal:1059-1075) and topk_vocab
                    (shaders.metal:1796-1831) as run by
                    MetalResidentTopKBuilder (metal/mod.rs:2661-2800)
  pbmoe_head_merge  candidate lists of vocabulary shards -> the full top-k

Logits agree with the oracle's within 1e-5 for bf16 activations and 1e-4 for
f32 activations, which the kernel carries as bf16 hi + lo halves (~16
significant bits); both are max relative errors against max(|r|, rms(r)).
The selection is bit-exact: ids and values equal the
oracle's topk_vocab run on the kernel's own logits, and the oracle's own
logits give the same ids wherever neighbouring candidates are separated by
more than the logit tolerance.
"""

import numpy as np
import pytest

from parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import torch

    from pb_b200 import capi

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = capi.Context(0)
    c.head_reserve(32, 151936, 256)
    yield c
    c.close()


def _weight(V, H, seed):
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", seed)
    return synth.normal_bf16((V, H), 0.02, g, "cuda")


def _u16(t):
    from pb_b200.synth import bf16_bits

    return bf16_bits(t).cpu().numpy().view(np.uint16)


def _run(ctx, w, x, k, allowed=None, id_base=0):
    import torch

    T, V = x.shape[0], w.shape[0]
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    vals = torch.empty(T, k, dtype=torch.float32, device="cuda")
    keys = torch.empty(T, k, dtype=torch.int32, device="cuda")
    logits = torch.empty(T, V, dtype=torch.float32, device="cuda")
    ctx.head_topk(w, x, ids, vals, id_base=id_base, allowed=allowed, keys=keys, logits=logits)
    torch.cuda.synchronize()
    assert ctx.device_status() == 0
    return (ids.cpu().numpy().view(np.uint32), vals.cpu().numpy(), keys.cpu().numpy().view(np.uint32),
            logits.cpu().numpy())


def _check(oracle, w, x, k, got, allowed_np=None, tol=1e-5):
    ids, vals, _, logits = got
    T, V = logits.shape
    n = min(k, V)
    ref_ids, ref_vals, ref_logits = oracle.head_topk(_u16(w), x.float().cpu().numpy(), k, allowed_np)
    assert_close(logits, ref_logits, tol=tol, what="head logits")
    rms = float(np.sqrt(np.mean(ref_logits.astype(np.float64) ** 2)))
    for t in range(T):
        # selection: bit-exact on the kernel's own logits
        sid, sval = oracle.topk_vocab(logits[t], k, allowed_np)
        assert np.array_equal(ids[t, :n], sid), f"token {t}: ids differ from topk_vocab on the same logits"
        assert np.array_equal(vals[t, :n], sval)
        assert np.all(ids[t, n:] == 0) and np.all(np.isneginf(vals[t, n:]))
        # against the oracle's own logits: equal unless two candidates are closer than the tolerance
        for r in range(n):
            if ids[t, r] != ref_ids[t, r]:
                a, b = ref_logits[t, ids[t, r]], ref_logits[t, ref_ids[t, r]]
                assert abs(a - b) <= 4 * tol * max(rms, 1e-30), f"token {t} rank {r}: {ids[t, r]} vs {ref_ids[t, r]}"


@pytest.mark.parametrize("V,H,T,k", [(3000, 512, 1, 10), (3000, 512, 5, 64), (20000, 1024, 8, 40),
                                     (20000, 512, 13, 1), (17000, 512, 32, 100), (40, 512, 3, 64)])
def test_head_small(ctx, oracle, V, H, T, k):
    from pb_b200 import synth

    w = _weight(V, H, V + T)
    x = synth.normal_bf16((T, H), 1.0, synth.gen("cuda", 7 * T + k), "cuda")
    _check(oracle, w, x, k, _run(ctx, w, x, k))


def test_head_f32_input(ctx, oracle):
    import torch

    w = _weight(5000, 512, 3)
    x = torch.randn(9, 512, generator=torch.Generator("cuda").manual_seed(4), device="cuda")
    _check(oracle, w, x, 20, _run(ctx, w, x, 20), tol=1e-4)


def test_head_ties_lower_id_first(ctx, oracle):
    """Duplicated weight rows give equal logits: the lower token id ranks first."""
    from pb_b200 import synth

    w = _weight(4096, 512, 11)
    w[2048:] = w[:2048]
    x = synth.normal_bf16((4, 512), 1.0, synth.gen("cuda", 12), "cuda")
    got = _run(ctx, w, x, 32)
    _check(oracle, w, x, 32, got)
    ids, _, _, logits = got
    for t in range(4):
        assert np.array_equal(logits[t, :2048], logits[t, 2048:])
        # each pair (i, i + 2048) is adjacent with i first
        assert np.array_equal(ids[t, 0::2] + 2048, ids[t, 1::2])


def test_head_allowed_mask(ctx, oracle):
    import torch

    from pb_b200 import synth

    V, k = 9000, 50
    w = _weight(V, 512, 21)
    x = synth.normal_bf16((6, 512), 1.0, synth.gen("cuda", 22), "cuda")
    rng = np.random.default_rng(5)
    mask = rng.integers(0, 2**32, (V + 31) // 32, dtype=np.uint64).astype(np.uint32)
    got = _run(ctx, w, x, k, allowed=torch.tensor(mask.view(np.int32), device="cuda"))
    _check(oracle, w, x, k, got, allowed_np=mask)
    for t in range(6):
        for i in got[0][t]:
            assert (mask[i >> 5] >> (i & 31)) & 1


def test_head_fewer_allowed_than_k(ctx, oracle):
    """Three allowed tokens and k 10: the rest of the slots are (0, -inf)."""
    import torch

    from pb_b200 import synth

    V = 5000
    w = _weight(V, 512, 31)
    x = synth.normal_bf16((2, 512), 1.0, synth.gen("cuda", 32), "cuda")
    mask = np.zeros((V + 31) // 32, np.uint32)
    for i in (17, 2500, 4999):
        mask[i >> 5] |= np.uint32(1 << (i & 31))
    ids, vals, keys, logits = _run(ctx, w, x, 10, allowed=torch.tensor(mask.view(np.int32), device="cuda"))
    for t in range(2):
        sid, sval = oracle.topk_vocab(logits[t], 10, mask)
        assert np.array_equal(ids[t], sid) and np.array_equal(vals[t], sval)
        assert sorted(ids[t, :3].tolist()) == [17, 2500, 4999]
        assert np.all(ids[t, 3:] == 0) and np.all(np.isneginf(vals[t, 3:])) and np.all(keys[t, 3:] == 0)


def test_head_non_finite_logits(ctx, oracle):
    """An infinite activation makes every logit non-finite: they all count as
    -inf, so the lowest ids are chosen, with value -inf."""
    import torch

    w = _weight(2000, 512, 41)
    x = torch.zeros(1, 512, device="cuda")
    x[0, 5] = float("inf")
    ids, vals, _, logits = _run(ctx, w, x, 8)
    sid, sval = oracle.topk_vocab(logits[0], 8)
    assert np.array_equal(ids[0], sid) and np.array_equal(vals[0], sval)
    ref_ids, ref_vals, _ = oracle.head_topk(_u16(w), x.cpu().numpy(), 8)
    assert np.array_equal(ids[0], ref_ids[0]) and np.all(np.isneginf(vals[0]))


def test_head_vocab_shards_merge(ctx, oracle):
    """Three vocabulary shards (id_base offsets) merged with pbmoe_head_merge
    equal the single full-vocabulary call, ids and values."""
    import torch

    from pb_b200 import synth

    V, H, T, k = 24000, 512, 7, 64
    w = _weight(V, H, 51)
    x = synth.normal_bf16((T, H), 1.0, synth.gen("cuda", 52), "cuda")
    full = _run(ctx, w, x, k)
    bounds = [0, 9000, 16000, V]
    keys, ids, vals = [], [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        i, v, kk, _ = _run(ctx, w[a:b].contiguous(), x, k, id_base=a)
        keys.append(kk), ids.append(i), vals.append(v)
    dev = lambda arrs, dt: torch.tensor(np.stack(arrs).view(dt), device="cuda")
    out_ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    out_vals = torch.empty(T, k, dtype=torch.float32, device="cuda")
    ctx.head_merge(dev(keys, np.int32), dev(ids, np.int32), dev(vals, np.float32), out_ids, out_vals)
    torch.cuda.synchronize()
    assert np.array_equal(out_ids.cpu().numpy().view(np.uint32), full[0])
    assert np.array_equal(out_vals.cpu().numpy(), full[1])


def test_head_config4_shape(ctx, oracle):
    """Vocabulary 151936 x hidden 2048 (config 4), two tokens checked
    against the oracle; 32 tokens run for the selection against the
    kernel's own logits."""
    from pb_b200 import synth

    V, H = 151936, 2048
    w = _weight(V, H, 61)
    x = synth.normal_bf16((32, H), 1.0, synth.gen("cuda", 62), "cuda")
    got = _run(ctx, w, x, 64)
    _check(oracle, w, x[:2], 64, tuple(a[:2] for a in got))
    for t in range(2, 32, 7):
        sid, sval = oracle.topk_vocab(got[3][t], 64)
        assert np.array_equal(got[0][t], sid) and np.array_equal(got[1][t], sval)


def test_head_rejects(ctx):
    import torch

    from pb_b200 import capi

    w = _weight(1000, 512, 71)
    ids = torch.empty(33, 4, dtype=torch.int32, device="cuda")
    vals = torch.empty(33, 4, device="cuda")
    with pytest.raises(capi.PbmoeError, match="unsupported"):
        ctx.head_topk(w, torch.zeros(33, 512, device="cuda"), ids, vals)  # > 32 tokens
    w2 = _weight(1000, 320, 72)
    with pytest.raises(capi.PbmoeError, match="unsupported"):
        ctx.head_topk(w2, torch.zeros(2, 320, device="cuda"), ids[:2], vals[:2])  # hidden not a multiple of 512
    other = capi.Context(0)
    try:
        with pytest.raises(capi.PbmoeError, match="reserve"):
            other.head_topk(w, torch.zeros(2, 512, device="cuda"), ids[:2], vals[:2])
    finally:
        other.close()
