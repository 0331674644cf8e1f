"""pbmoe_q4_matvec against the CPU oracle (math.rs:861-911 with bf16
scale/bias, the production arithmetic of experts/slots.rs:629-670)."""

import json
import os

import numpy as np
import pytest

from parity import assert_close

pytestmark = pytest.mark.gpu

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


@pytest.fixture(scope="module")
def ctx():
    import torch

    from pb_b200 import capi

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = capi.Context(0)
    yield c
    c.close()


def _run(ctx, packed, s16, b16, rows, cols, group, x, out_dtype, batch=1):
    import torch

    y = torch.empty(batch, rows, device="cuda", dtype=out_dtype)
    ctx.q4_matvec(packed, s16, b16, rows, cols, group, x, y, batch=batch)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def _oracle(oracle, packed, s16, b16, rows, cols, group, x):
    from pb_b200.synth import bf16_bits

    p = packed.cpu().numpy().reshape(-1)
    sb = bf16_bits(s16).cpu().numpy().view(np.uint16).reshape(-1)
    bb = bf16_bits(b16).cpu().numpy().view(np.uint16).reshape(-1)
    xs = x.float().cpu().numpy()
    return np.stack([oracle.q4_fma_matvec_bf16(p, xs[i], sb, bb, rows, cols, group) for i in range(xs.shape[0])])


@pytest.mark.parametrize("x_dtype", ["bf16", "f32"])
@pytest.mark.parametrize("out_dtype", ["bf16", "f32"])
def test_config0_matvec(ctx, oracle, x_dtype, out_dtype):
    """Config 0: W [4096 x 2048], group 64, x ~ N(0,1) bf16, y bf16 (fp32 accumulate)."""
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", 1234)
    packed, s, b = synth.q4_matrix(4096, 2048, 64, g, "cuda")
    x = synth.normal_bf16((1, 2048), 1.0, g, "cuda")
    xd = x if x_dtype == "bf16" else x.float()
    od = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    y = _run(ctx, packed, s, b, 4096, 2048, 64, xd, od)
    ref = _oracle(oracle, packed, s, b, 4096, 2048, 64, x)
    assert_close(y, ref, what="config0")


@pytest.mark.parametrize("rows,cols,group,batch", [
    (512, 2048, 64, 3), (2048, 512, 64, 1), (2048, 512, 64, 8), (300, 1024, 32, 5), (77, 4096, 128, 2),
    (5, 5, 3, 2), (3, 7, 4, 1), (64, 96, 16, 3), (33, 100, 64, 4), (1, 8, 8, 1), (129, 256, 64, 9),
])
def test_odd_shapes(ctx, oracle, rows, cols, group, batch):
    """Odd geometry (cols not multiple of 32, group 3/4/16, ragged rows) takes
    the per-element kernel; aligned shapes take the fast path."""
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", rows * 1000 + cols)
    packed, s, b = synth.q4_matrix(rows, cols, group, g, "cuda")
    x = synth.normal_bf16((batch, cols), 1.0, g, "cuda").float()
    y = _run(ctx, packed, s, b, rows, cols, group, x, torch.float32, batch=batch)
    ref = _oracle(oracle, packed, s, b, rows, cols, group, x)
    assert_close(y, ref, what=f"{rows}x{cols} g{group} b{batch}")


def test_reference_kats_on_gpu(ctx):
    """The reference's own Q4 matvec goldens, run through the CUDA path."""
    import torch

    from oracle.pb_oracle import f32_to_bf16_bits

    def dev(a, dt):
        return torch.tensor(np.asarray(a), dtype=dt, device="cuda")

    k = KATS["q4_matvec_closed_form"]
    s = f32_to_bf16_bits(k["scales"]).view(np.int16)
    bb = f32_to_bf16_bits(k["biases"]).view(np.int16)
    x = dev(np.asarray(k["input"], np.float32), torch.float32)[None]
    y = _run(ctx, dev(k["packed"], torch.uint8), dev(s, torch.int16), dev(bb, torch.int16), 1, 4, 64, x,
             torch.float32)
    assert abs(y[0, 0] - k["expected"][0]) < k["abs_tol"]

    k = KATS["q4_bf16_u32_word"]
    packed = np.frombuffer(np.uint32(k["packed_word_le"]).tobytes(), np.uint8)
    x = dev(np.asarray(k["input"], np.float32), torch.float32)[None]
    y = _run(ctx, dev(packed, torch.uint8), dev(np.array([k["scale_bf16"]], np.uint16).view(np.int16), torch.int16),
             dev(np.array([k["bias_bf16"]], np.uint16).view(np.int16), torch.int16), 1, 8, 8, x, torch.float32)
    assert abs(y[0, 0] - k["expected"][0]) <= k["abs_tol"]


def test_zero_rows_and_invalid_group(ctx):
    import torch

    from pb_b200 import capi

    z = torch.zeros(16, dtype=torch.uint8, device="cuda")
    s = torch.zeros(4, dtype=torch.int16, device="cuda")
    x = torch.zeros(1, 32, device="cuda")
    y = torch.zeros(1, 4, device="cuda")
    ctx.q4_matvec(z, s, s, 0, 32, 32, x, y)  # empty is a no-op
    with pytest.raises(capi.PbmoeError) as e:
        ctx.q4_matvec(z, s, s, 1, 32, 0, x, y)
    assert e.value.code == capi.PBMOE_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("batch", [1, 8])
@pytest.mark.parametrize("x_dtype", ["bf16", "f32"])
def test_matvec_batch_matches_single_calls(ctx, oracle, batch, x_dtype):
    """pbmoe_q4_matvec_batch (resident_mmap_matvec_batch, runtime/mod.rs:1184):
    20 projections of different row counts on one input, run as launches of
    up to 16 matrices, equal pbmoe_q4_matvec on each matrix bit for bit (same
    kernel, same arithmetic), and the oracle within 1e-2."""
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", 700 + batch)
    rows = [4096, 1536, 576, 3072, 2048, 64, 128, 1024, 512, 2048, 96, 4096, 1536, 256, 32, 2048, 1024, 576, 3072, 64]
    cols, group = 2048, 64
    mats = [synth.q4_matrix(r, cols, group, g, "cuda") for r in rows]
    dt = torch.bfloat16 if x_dtype == "bf16" else torch.float32
    x = synth.normal_bf16((batch, cols), 1.0, g, "cuda").to(dt)
    ys = [torch.empty(batch, r, device="cuda", dtype=torch.float32) for r in rows]
    ctx.q4_matvec_batch([(p, s, b, r, cols, group) for (p, s, b), r in zip(mats, rows)], x, ys)
    torch.cuda.synchronize()
    for i, ((p, s, b), r) in enumerate(zip(mats, rows)):
        ref = torch.empty(batch, r, device="cuda", dtype=torch.float32)
        ctx.q4_matvec(p, s, b, r, cols, group, x, ref, batch=batch)
        torch.cuda.synchronize()
        assert torch.equal(ys[i], ref), f"matrix {i} ({r} rows) differs from pbmoe_q4_matvec"
    for i in (0, 5, 19):
        p, s, b = mats[i]
        assert_close(ys[i].cpu().numpy(), _oracle(oracle, p, s, b, rows[i], cols, group, x), what=f"batch matrix {i}")


def test_matvec_batch_refuses_mixed_columns(ctx):
    import torch

    from pb_b200 import capi, synth

    g = synth.gen("cuda", 710)
    a = synth.q4_matrix(64, 2048, 64, g, "cuda")
    b = synth.q4_matrix(64, 1024, 64, g, "cuda")
    x = synth.normal_bf16((1, 2048), 1.0, g, "cuda")
    ys = [torch.empty(1, 64, device="cuda") for _ in range(2)]
    with pytest.raises(capi.PbmoeError, match="cols"):
        ctx.q4_matvec_batch([(*a, 64, 2048, 64), (*b, 64, 1024, 64)], x, ys)
