"""pbmoe_mla_decode (MLA absorbed decode attention) against the CPU oracle.

The oracle restates mla_absorbed_attention (weights/store.rs:1179-1327) with
bf16 W_UK / W_UV and is pinned to the reference's closed-form MLA test
(tests/metal.rs:1872-2028) in test_oracle_kats.py. Shapes are config 3's:
16 heads, nope 128, rope 64, latent 512, v 128, scale 1/sqrt(192); caches
bf16 ~N(0,1), W_UK / W_UV ~N(0, 0.02), queries ~N(0,1).
"""

import numpy as np
import pytest

from parity import assert_close

pytestmark = pytest.mark.gpu

H, NOPE, ROPE, LAT, V = 16, 128, 64, 512, 128


@pytest.fixture(scope="module")
def ctx():
    import torch

    from pb_b200 import capi

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = capi.Context(0)
    c.mla_reserve(capi.mla_config(), 32)
    yield c
    c.close()


def _bits(t):
    from pb_b200.synth import bf16_bits

    return bf16_bits(t).cpu().numpy().view(np.uint16)


def _make(seed, lens, q_scale=1.0, device="cuda"):
    import torch

    from pb_b200 import synth

    g = synth.gen(device, seed)
    q = synth.normal_bf16((len(lens), H, NOPE + ROPE), q_scale, g, device)
    ckv = [synth.normal_bf16((L, LAT), 1.0, g, device) for L in lens]
    kr = [synth.normal_bf16((L, ROPE), 1.0, g, device) for L in lens]
    wuk = synth.normal_bf16((H, NOPE, LAT), 0.02, g, device)
    wuv = synth.normal_bf16((H, V, LAT), 0.02, g, device)
    return q, ckv, kr, wuk, wuv


def _oracle(oracle, q, ckv, kr, wuk, wuv):
    """The oracle per sequence, sequences on parallel threads (each call is
    independent and releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    bk, bv = _bits(wuk), _bits(wuv)
    one = lambda b: oracle.mla_absorbed_attention(q[b].float().cpu().numpy(), ckv[b].float().cpu().numpy(),
                                                  kr[b].float().cpu().numpy(), bk, bv, H, NOPE, ROPE, LAT, V)
    with ThreadPoolExecutor(max_workers=8) as pool:
        outs = list(pool.map(one, range(len(ckv))))
    return np.stack(outs).reshape(len(ckv), H, V)


def _run(ctx, q, ckv, kr, wuk, wuv, out_dtype=None, q_dtype=None):
    import torch

    from pb_b200 import capi

    qq = q if q_dtype is None else q.to(q_dtype)
    out = torch.empty(len(ckv), H, V, device="cuda", dtype=out_dtype or torch.float32)
    ctx.mla_decode(capi.mla_config(), qq, ckv, kr, wuk, wuv, out)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("lens", [[1], [7], [64], [65], [200], [1000], [3, 130, 64]])
def test_mla_small(ctx, oracle, lens):
    q, ckv, kr, wuk, wuv = _make(11 + sum(lens), lens)
    ref = _oracle(oracle, q, ckv, kr, wuk, wuv)
    got = _run(ctx, q, ckv, kr, wuk, wuv)
    assert_close(got, ref, what=f"mla lens={lens}")


def test_mla_f32_query_bf16_out(ctx, oracle):
    import torch

    lens = [300, 77]
    q, ckv, kr, wuk, wuv = _make(5, lens)
    ref = _oracle(oracle, q, ckv, kr, wuk, wuv)
    got = _run(ctx, q, ckv, kr, wuk, wuv, out_dtype=torch.bfloat16, q_dtype=torch.float32)
    assert_close(got, ref, what="mla f32 query / bf16 out")


def test_mla_peaked_scores(ctx, oracle):
    # large queries make the softmax nearly one-hot: exercises the running maximum
    lens = [513]
    q, ckv, kr, wuk, wuv = _make(8, lens, q_scale=40.0)
    ref = _oracle(oracle, q, ckv, kr, wuk, wuv)
    got = _run(ctx, q, ckv, kr, wuk, wuv)
    assert_close(got, ref, what="mla peaked")


@pytest.mark.parametrize("L,batch", [(4096, 1), (4096, 8), (32768, 1), (32768, 8)])
def test_mla_config3(ctx, oracle, L, batch):
    """Every config-3 case, including the benchmarked (32768, 8)."""
    lens = [L] * batch
    q, ckv, kr, wuk, wuv = _make(3 + L + batch, lens)
    ref = _oracle(oracle, q, ckv, kr, wuk, wuv)
    got = _run(ctx, q, ckv, kr, wuk, wuv)
    assert_close(got, ref, what=f"mla config3 L={L} batch={batch}")


def test_mla_rejects(ctx):
    import torch

    from pb_b200 import capi

    q, ckv, kr, wuk, wuv = _make(1, [10])
    out = torch.empty(1, H, V, device="cuda")
    with pytest.raises(capi.PbmoeError) as e:
        ctx.mla_decode(capi.mla_config(heads=8), q, ckv, kr, wuk, wuv, out)
    assert e.value.code == capi.PBMOE_ERR_UNSUPPORTED
    empty = [torch.empty(0, LAT, device="cuda", dtype=torch.bfloat16)]
    with pytest.raises(capi.PbmoeError) as e:
        ctx.mla_decode(capi.mla_config(), q, empty, [torch.empty(0, ROPE, device="cuda", dtype=torch.bfloat16)], wuk,
                       wuv, out)
    assert e.value.code == capi.PBMOE_ERR_INVALID_ARGUMENT
