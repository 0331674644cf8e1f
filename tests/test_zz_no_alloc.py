"""pbmoe_moe_layer_static: the MoE layer for callers that cannot allocate.

Hosts whose device memory belongs to their own arena, code running under
CUDA graph capture, and loops that must not risk an allocation's implicit
synchronisation cannot call cudaMalloc, so they cannot use pbmoe_reserve (or
even pbmoe_init). This entry point takes no context and keeps its scratch in a
fixed device array inside the library. These tests call it through the C ABI:

* up to 8 tokens it launches exactly the kernels pbmoe_moe_layer launches on
  the same inputs, so its outputs must be bit-identical to the regular entry
  point's, on two calls in a row (the second call reuses the array the first
  one left behind);
* 9 to 29 tokens run as one launch of the gathered expert pipe (as
  pbmoe_moe_layer runs them), checked against the CPU oracle;
* at config-1 shapes 29 tokens fit the fixed array and 30 are refused with a
  message instead of running.

The file is named to be collected last so that a run stopping at the first
failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest

from parity import assert_close

pytestmark = pytest.mark.gpu

# Largest config-1 batch (hidden 2048, 512 experts top-10, I 512, group 64)
# whose workspace fits PBMOE_STATIC_SCRATCH_BYTES with the 256-byte status word.
CONFIG1_MAX_TOKENS = 29


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


def _host_u16(t):
    from pb_b200.synth import bf16_bits

    return bf16_bits(t).cpu().numpy().view(np.uint16)


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
        assert torch.equal(out, ref_out), f"static out differs from pbmoe_moe_layer at T={tokens}"
        assert torch.equal(nn, ref_nn), f"static next-layer norm differs from pbmoe_moe_layer at T={tokens}"
    ctx.close()


def test_static_entry_point_config1_shape_twice():
    """Config-1 geometry (hidden 2048, 512 experts top-10, I=512, G=64), one
    token then eight, bit-identical to pbmoe_moe_layer; no status pointer
    given (device-side errors would then be dropped)."""
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
        assert torch.equal(out, ref), f"config-1 static output differs from pbmoe_moe_layer at T={tokens}"
    ctx.close()


@pytest.fixture(scope="module")
def config1_weights():
    from pb_b200 import synth

    return synth.MoeLayerWeights("cuda", seed=43)


@pytest.mark.parametrize("tokens", [24, CONFIG1_MAX_TOKENS])
def test_static_unchunked_batch_against_oracle(oracle, config1_weights, tokens):
    """More than 8 tokens run as one launch here (the regular entry point
    chunks them), so this path is checked against the CPU oracle: outputs of
    every token within 1e-2, the status word clear."""
    import torch

    from pb_b200 import capi, synth

    w = config1_weights
    cfg = capi.moe_config(w.layout, w.num_experts, 10)
    g = synth.gen("cuda", 44 + tokens)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
    res = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
    out = torch.empty_like(x)
    rc, msg = _call_static(cfg, w.c_weights(), x, out, tokens, residual=res, status=status)
    assert rc == capi.PBMOE_OK, msg
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    offs = np.array(list(w.layout.component_offsets), np.uint64)
    ref_out, _, _, _ = oracle.moe_layer(
        x.float().cpu().numpy(), _host_u16(w.router), w.experts.cpu().numpy(), offs, int(w.layout.expert_bytes),
        w.num_experts, 10, w.intermediate, w.group, shared_slot=w.shared.cpu().numpy(),
        shared_gate_bits=_host_u16(w.shared_gate), residual=res.float().cpu().numpy(), threads=8)
    assert_close(out.float().cpu().numpy(), ref_out, what=f"static T={tokens} vs oracle")


def test_static_capacity_at_config1_shapes(config1_weights):
    """29 config-1 tokens fit the fixed array (the previous test ran them);
    30 are refused with PBMOE_ERR_UNSUPPORTED and a message, and nothing runs."""
    import torch

    from pb_b200 import capi

    w = config1_weights
    cfg = capi.moe_config(w.layout, w.num_experts, 10)
    lib = capi.load()
    need = lambda t: 256 + lib.pbmoe_moe_workspace_bytes(t, ctypes.byref(cfg))
    assert need(CONFIG1_MAX_TOKENS) <= 4 << 20 < need(CONFIG1_MAX_TOKENS + 1)
    tokens = CONFIG1_MAX_TOKENS + 1
    x = torch.zeros(tokens, w.hidden, device="cuda", dtype=torch.bfloat16)
    out = torch.full_like(x, 7.0)
    rc, msg = _call_static(cfg, w.c_weights(), x, out, tokens)
    assert rc == capi.PBMOE_ERR_UNSUPPORTED
    assert "scratch" in msg and str(4 << 20) in msg
    torch.cuda.synchronize()
    assert bool((out == 7.0).all()), "a refused call must not write its output"


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
