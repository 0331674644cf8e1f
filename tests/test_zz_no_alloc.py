"""pbmoe_moe_layer_static: the MoE layer for callers that cannot allocate.

Hosts whose device memory belongs to their own arena, code running under
CUDA graph capture, and loops that must not risk an allocation's implicit
synchronisation cannot call cudaMalloc, so they cannot use pbmoe_reserve (or
even pbmoe_init). This entry point takes no context and keeps its scratch in a
fixed device array inside the library. These tests call it through the C ABI
and check it against the regular entry point, pbmoe_moe_layer, on two calls in
a row (the second call reuses the array the first one left behind), and check
that an oversized call is refused with a message instead of running.

The file is named to be collected last so that a run stopping at the first
failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest

from parity import assert_close

pytestmark = pytest.mark.gpu


def _call_static(cfg, weights, x, out, tokens, residual=None, norm_w=None, next_normed=None, status=None):
    import torch

    from pb_b200 import capi

    lib = capi.load()
    err = ctypes.create_string_buffer(512)
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    rc = lib.pbmoe_moe_layer_static(
        ctypes.byref(cfg), ctypes.byref(weights), p(x), capi._dtype_code(x), p(residual), p(out),
        capi._dtype_code(out), tokens, p(norm_w), p(next_normed), p(status), err, len(err),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, err.value.decode()


def test_static_entry_point_matches_pbmoe_moe_layer():
    import torch

    from pb_b200 import capi, synth

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    w = synth.MoeLayerWeights("cuda", seed=31, hidden=512, num_experts=64, intermediate=256, group=64)
    cfg = capi.moe_config(w.layout, w.num_experts, 6)
    ctx = capi.Context(0)
    ctx.reserve(8, cfg)
    g = synth.gen("cuda", 32)
    norm_w = torch.rand(w.hidden, device="cuda", generator=g) + 0.5
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for tokens in (3, 8):  # two calls in a row, different sizes
        x = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
        res = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
        ref_out, ref_nn = torch.empty_like(x), torch.empty_like(x)
        ctx.moe_layer(cfg, w.c_weights(), x, ref_out, tokens, residual=res, next_norm_weight=norm_w,
                      next_normed=ref_nn)
        out, nn = torch.empty_like(x), torch.empty_like(x)
        rc, msg = _call_static(cfg, w.c_weights(), x, out, tokens, residual=res, norm_w=norm_w, next_normed=nn,
                               status=status)
        assert rc == capi.PBMOE_OK, msg
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_close(out.float().cpu().numpy(), ref_out.float().cpu().numpy(), what=f"static out T={tokens}")
        assert_close(nn.float().cpu().numpy(), ref_nn.float().cpu().numpy(), what=f"static norm T={tokens}")
    ctx.close()


def test_static_entry_point_config1_shape_twice():
    """Config-1 geometry (hidden 2048, 512 experts top-10, I=512, G=64), one
    token then eight, against pbmoe_moe_layer; no status pointer given."""
    import torch

    from pb_b200 import capi, synth

    w = synth.MoeLayerWeights("cuda", seed=41)
    cfg = capi.moe_config(w.layout, w.num_experts, 10)
    ctx = capi.Context(0)
    ctx.reserve(8, cfg)
    g = synth.gen("cuda", 42)
    for tokens in (1, 8):
        x = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
        ref = torch.empty_like(x)
        ctx.moe_layer(cfg, w.c_weights(), x, ref, tokens)
        out = torch.empty_like(x)
        rc, msg = _call_static(cfg, w.c_weights(), x, out, tokens)
        assert rc == capi.PBMOE_OK, msg
        torch.cuda.synchronize()
        assert_close(out.float().cpu().numpy(), ref.float().cpu().numpy(), what=f"config1 static T={tokens}")
    ctx.close()


def test_static_entry_point_rejects_oversize_call():
    import torch

    from pb_b200 import capi, synth

    w = synth.MoeLayerWeights("cuda", seed=51, hidden=512, num_experts=64, intermediate=256, group=64)
    cfg = capi.moe_config(w.layout, w.num_experts, 6)
    tokens = 512
    x = torch.zeros(tokens, w.hidden, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(x)
    rc, msg = _call_static(cfg, w.c_weights(), x, out, tokens)
    assert rc == capi.PBMOE_ERR_UNSUPPORTED
    assert "scratch" in msg and str(4 << 20) in msg
