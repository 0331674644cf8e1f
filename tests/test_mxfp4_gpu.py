"""pbmoe_mxfp4_matvec against the oracle's mxfp4_fma_matvec_with_group_size
(experts/slots.rs:1239-1287): the reference golden (tests/metal.rs:328-380),
expert shapes with E8M0 scales around 2^0 (and the e = 0 subnormal), bf16 and
f32 activations, batches 1-11, and the e = 255 status."""

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
    yield c
    c.close()


def _matrix(rows, cols, seed, lo=118, hi=136):
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(lo, hi, (rows, cols // 32), dtype=np.uint8)
    return packed, scales


def _run(ctx, packed, scales, x, y_dtype=None):
    import torch

    rows, cols = packed.shape[0], packed.shape[1] * 2
    p = torch.tensor(packed, device="cuda")
    s = torch.tensor(scales, device="cuda")
    y = torch.empty(x.shape[0], rows, device="cuda", dtype=y_dtype or torch.float32)
    ctx.mxfp4_matvec(p, s, rows, cols, x, y)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_mxfp4_golden(ctx):
    import torch

    packed = np.array([[0x22] * 16, [0x95] * 16], np.uint8)
    x = torch.arange(1, 33, dtype=torch.float32, device="cuda").reshape(1, 32)
    y = _run(ctx, packed, np.array([[127], [127]], np.uint8), x)
    assert abs(y[0, 0] - 528.0) < 1e-4 and abs(y[0, 1] - 632.0) < 1e-4
    assert ctx.device_status() == 0


@pytest.mark.parametrize("rows,cols,batch,xdt", [(512, 2048, 1, "bf16"), (2048, 512, 1, "f32"),
                                                 (4096, 2048, 2, "bf16"), (513, 2048, 3, "f32"),
                                                 (1000, 1024, 8, "bf16"), (96, 4096, 11, "f32")])
def test_mxfp4_parity(ctx, oracle, rows, cols, batch, xdt):
    import torch

    packed, scales = _matrix(rows, cols, rows + cols + batch)
    g = torch.Generator("cuda").manual_seed(batch)
    x = torch.randn(batch, cols, generator=g, device="cuda").to(torch.bfloat16 if xdt == "bf16" else torch.float32)
    y = _run(ctx, packed, scales, x)
    xn = x.float().cpu().numpy()
    ref = np.stack([oracle.mxfp4_matvec(packed.reshape(-1), xn[t], scales.reshape(-1), rows, cols, 32)
                    for t in range(batch)])
    assert_close(y, ref, tol=1e-5, what="mxfp4 matvec")
    assert ctx.device_status() == 0


def test_mxfp4_subnormal_scale_and_bf16_out(ctx, oracle):
    import torch

    packed, scales = _matrix(64, 256, 7)
    scales[::3] = 0  # 2^-127
    scales[1::3] = 140
    x = (torch.randn(2, 256, device="cuda") * 1e30).float()
    y = _run(ctx, packed, scales, x)
    xn = x.cpu().numpy()
    ref = np.stack([oracle.mxfp4_matvec(packed.reshape(-1), xn[t], scales.reshape(-1), 64, 256, 32) for t in range(2)])
    assert_close(y, ref, tol=1e-5, what="mxfp4 with e = 0 scales")
    yb = _run(ctx, packed, scales, x, y_dtype=torch.bfloat16)
    assert_close(yb, ref, tol=8e-3, what="mxfp4 bf16 output")


def test_mxfp4_scale_255_latches(ctx):
    import torch

    from pb_b200 import capi

    packed, scales = _matrix(32, 64, 9)
    scales[5, 1] = 255
    ctx.device_status(clear=True)
    _run(ctx, packed, scales, torch.ones(1, 64, device="cuda"))
    assert ctx.device_status(clear=True) & capi.PBMOE_DEV_ERR_MXFP4_SCALE


def test_mxfp4_rejects(ctx):
    import torch

    from pb_b200 import capi

    p = torch.zeros(4, 24, dtype=torch.uint8, device="cuda")
    s = torch.zeros(4, 2, dtype=torch.uint8, device="cuda")
    y = torch.empty(1, 4, device="cuda")
    with pytest.raises(capi.PbmoeError, match="unsupported"):
        ctx.mxfp4_matvec(p, s, 4, 48, torch.zeros(1, 48, device="cuda"), y)  # cols not a multiple of 32
