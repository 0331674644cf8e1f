"""The MoE layer's two model-family variants against the CPU oracle:

* sigmoid/noaux routing (routing_sigmoid_noaux_top_k, math.rs:788-819: the
  GLM / DeepSeek router that selects on sigmoid(logit) + correction bias and
  weights by the raw sigmoid), as pbmoe_route_sigmoid_noaux on given logits
  and inside pbmoe_moe_layer through pbmoe_moe_weights.router_correction_bias;
* FIXED_MXFP4 expert slots (E2M1 nibbles + E8M0 scale per 32 columns, no
  biases; QwenMoeQ4ExpertLayout::fixed_mxfp4, model_family.rs:846-952), run
  by the MXFP4 expert kernels behind the same router, plan and combine.

Route ids are compared bit for bit, float outputs within 1e-2 relative.
"""

import ctypes

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


def _host_u16(t):
    from pb_b200.synth import bf16_bits

    return bf16_bits(t).cpu().numpy().view(np.uint16)


def test_route_sigmoid_noaux_golden(ctx, oracle):
    """math.rs:1521-1531: logits [0, 2, -2], bias [1, -1, 0], K=2 select
    experts 0 and 2 (biased scores 1.5, 0.88, 0.12) with raw weights 0.5 and
    1/(1+e^2), renormalised over the two selected."""
    import torch

    logits = torch.tensor([[0.0, 2.0, -2.0]], device="cuda")
    bias = torch.tensor([1.0, -1.0, 0.0], device="cuda")
    ids = torch.empty(1, 2, dtype=torch.int32, device="cuda")
    w = torch.empty(1, 2, device="cuda")
    ctx.route_sigmoid_noaux(logits, bias, 1, 3, 2, ids, w)
    torch.cuda.synchronize()
    got = sorted(zip(ids[0].tolist(), w[0].tolist()))
    assert [e for e, _ in got] == [0, 2]
    raw = np.array([0.5, 1.0 / (1.0 + np.exp(2.0))], np.float32)
    want = raw / raw.sum()
    assert abs(got[0][1] - want[0]) < 1e-6 and abs(got[1][1] - want[1]) < 1e-6
    oid, ow = oracle.routing_sigmoid_noaux_top_k(np.array([0.0, 2.0, -2.0], np.float32),
                                                 np.array([1.0, -1.0, 0.0], np.float32), 2)
    assert ids[0].tolist() == oid.tolist(), "slot order differs from routing_top_k_iter"
    assert abs(ow[0] - 0.5) < 1e-6 and abs(ow[1] - raw[1]) < 1e-6


@pytest.mark.parametrize("tokens,experts,top_k,norm", [(64, 256, 8, 0), (33, 512, 10, 1), (8, 160, 6, 0)])
def test_route_sigmoid_noaux_vs_oracle(ctx, oracle, tokens, experts, top_k, norm):
    """Random logits and biases, ties included (logits rounded to a coarse grid
    so several experts share a biased score): ids bit-exact in slot order,
    weights after the config's normalisation within 1e-5."""
    import torch

    rng = np.random.default_rng(tokens * 7 + experts)
    lg = (np.round(rng.normal(0, 2, (tokens, experts)) * 8) / 8).astype(np.float32)
    bias = (np.round(rng.normal(0, 0.5, experts) * 16) / 16).astype(np.float32)
    logits = torch.from_numpy(lg).cuda()
    b = torch.from_numpy(bias).cuda()
    ids = torch.empty(tokens, top_k, dtype=torch.int32, device="cuda")
    w = torch.empty(tokens, top_k, device="cuda")
    ctx.route_sigmoid_noaux(logits, b, tokens, experts, top_k, ids, w, normalization=norm, scale=2.5)
    torch.cuda.synchronize()
    gid = ids.cpu().numpy().view(np.uint32)
    gw = w.cpu().numpy()
    for t in range(tokens):
        oid, ow = oracle.routing_sigmoid_noaux_top_k(lg[t], bias, top_k)
        assert gid[t].tolist() == oid.tolist(), f"token {t}: ids differ"
        assert_close(gw[t], oracle.renormalize_routes(ow, 2.5, norm), tol=1e-5, what=f"token {t} weights")


def _layer(ctx, w, x, tokens, top_k, residual=None, bias=None):
    import torch

    from pb_b200 import capi

    cfg = capi.moe_config(w.layout, w.num_experts, top_k)
    ctx.reserve(max(tokens, 1), cfg)
    out = torch.empty(tokens, w.hidden, device="cuda", dtype=x.dtype)
    logits = torch.empty(tokens, w.num_experts, device="cuda")
    ids = torch.empty(tokens, top_k, device="cuda", dtype=torch.int32)
    rw = torch.empty(tokens, top_k, device="cuda")
    dbg = capi.MoeDebug(logits.data_ptr(), ids.data_ptr(), rw.data_ptr(), None, None, None)
    cw = w.c_weights()
    if bias is not None:
        cw.router_correction_bias = bias.data_ptr()
    ctx.moe_layer(cfg, cw, x, out, tokens, residual=residual, debug=dbg)
    torch.cuda.synchronize()
    return out, logits, ids, rw, ctx.device_status()


def _oracle(oracle, w, x, top_k, residual=None, bias=None):
    offs = np.array(list(w.layout.component_offsets), np.uint64)
    return oracle.moe_layer(
        x.float().cpu().numpy(), _host_u16(w.router), w.experts.cpu().numpy(), offs, int(w.layout.expert_bytes),
        w.num_experts, top_k, w.intermediate, w.group,
        shared_slot=None if w.shared is None else w.shared.cpu().numpy(),
        shared_gate_bits=None if w.shared_gate is None else _host_u16(w.shared_gate),
        residual=None if residual is None else residual.float().cpu().numpy(), threads=8,
        correction_bias=None if bias is None else bias.cpu().numpy(), mxfp4=w.mxfp4)


def _compare(r, ref, what):
    out, logits, ids, rw, status = r
    ref_out, ref_ids, ref_w, ref_logits = ref
    assert status == 0, f"{what}: device status {status:#x}"
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), ref_logits.view(np.uint32)), f"{what}: logits"
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_ids), f"{what}: routed experts differ"
    assert_close(rw.cpu().numpy(), ref_w, what=f"{what} route weights")
    assert_close(out.float().cpu().numpy(), ref_out, what=f"{what} output")


@pytest.mark.parametrize("tokens", [1, 5, 8, 19])
def test_moe_layer_sigmoid_noaux(ctx, oracle, tokens):
    """Config-1 geometry with a router correction bias: the selection runs on
    sigmoid + bias inside the router kernel (19 tokens: three 8-token chunks)."""
    import torch

    from pb_b200 import synth

    w = synth.MoeLayerWeights("cuda", seed=61)
    g = synth.gen("cuda", 62 + tokens)
    bias = (torch.randn(w.num_experts, device="cuda", generator=g) * 0.05).contiguous()
    x = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
    res = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
    r = _layer(ctx, w, x, tokens, 10, residual=res, bias=bias)
    _compare(r, _oracle(oracle, w, x, 10, residual=res, bias=bias), f"sigmoid/noaux T={tokens}")


@pytest.fixture(scope="module")
def mx_small():
    from pb_b200 import synth

    return synth.MoeLayerWeights("cuda", seed=71, hidden=512, num_experts=64, intermediate=256, mxfp4=True)


@pytest.fixture(scope="module")
def mx_config1():
    from pb_b200 import synth

    return synth.MoeLayerWeights("cuda", seed=72, mxfp4=True)


@pytest.mark.parametrize("tokens", [1, 3, 8])
def test_mxfp4_moe_layer_small(ctx, oracle, mx_small, tokens):
    from pb_b200 import synth

    g = synth.gen("cuda", 73 + tokens)
    x = synth.normal_bf16((tokens, mx_small.hidden), 1.0, g, "cuda")
    r = _layer(ctx, mx_small, x, tokens, 6)
    _compare(r, _oracle(oracle, mx_small, x, 6), f"mxfp4 small T={tokens}")


@pytest.mark.parametrize("tokens", [1, 8, 12])
def test_mxfp4_moe_layer_config1_shape(ctx, oracle, mx_config1, tokens):
    """hidden 2048, 512 experts top-10, intermediate 512, shared expert with a
    gate, MXFP4 slots (fixed_mxfp4(2048, 512, 32)); 12 tokens run as two chunks."""
    from pb_b200 import synth

    g = synth.gen("cuda", 80 + tokens)
    x = synth.normal_bf16((tokens, mx_config1.hidden), 1.0, g, "cuda")
    res = synth.normal_bf16((tokens, mx_config1.hidden), 1.0, g, "cuda")
    r = _layer(ctx, mx_config1, x, tokens, 10, residual=res)
    _compare(r, _oracle(oracle, mx_config1, x, 10, residual=res), f"mxfp4 config-1 T={tokens}")


def test_mxfp4_moe_layer_f32_input_and_sigmoid(ctx, oracle):
    """f32 activations in and out, sigmoid/noaux routing over MXFP4 experts."""
    import torch

    from pb_b200 import synth

    w = synth.MoeLayerWeights("cuda", seed=91, hidden=1024, num_experts=128, intermediate=384, mxfp4=True)
    g = synth.gen("cuda", 92)
    bias = (torch.randn(w.num_experts, device="cuda", generator=g) * 0.05).contiguous()
    x = torch.randn(4, w.hidden, device="cuda", generator=g)
    r = _layer(ctx, w, x, 4, 8, bias=bias)
    _compare(r, _oracle(oracle, w, x, 8, bias=bias), "mxfp4 f32 sigmoid")


def test_mxfp4_non_finite_scale_sets_status(ctx, mx_small):
    """An E8M0 byte of 255 (not a finite scale: the reference's bail) in the
    shared expert, which every token runs, latches PBMOE_DEV_ERR_MXFP4_SCALE."""
    import torch

    from pb_b200 import capi, synth

    w = mx_small
    bad = w.shared.clone()
    bad[int(w.layout.component_offsets[7]) + 5] = 255  # a down-projection scale byte
    cw = w.c_weights()
    cw.shared_expert = bad.data_ptr()
    cfg = capi.moe_config(w.layout, w.num_experts, 6)
    ctx.reserve(2, cfg)
    x = synth.normal_bf16((2, w.hidden), 1.0, synth.gen("cuda", 95), "cuda")
    out = torch.empty_like(x)
    ctx.moe_layer(cfg, cw, x, out, 2)
    torch.cuda.synchronize()
    assert ctx.device_status() & capi.PBMOE_DEV_ERR_MXFP4_SCALE


def test_mxfp4_static_entry_matches_layer(ctx, mx_small):
    """pbmoe_moe_layer_static on MXFP4 slots launches the same kernels."""
    import torch

    from pb_b200 import capi, synth

    w = mx_small
    cfg = capi.moe_config(w.layout, w.num_experts, 6)
    ctx.reserve(8, cfg)
    x = synth.normal_bf16((5, w.hidden), 1.0, synth.gen("cuda", 96), "cuda")
    ref = torch.empty_like(x)
    ctx.moe_layer(cfg, w.c_weights(), x, ref, 5)
    out = torch.empty_like(x)
    lib = capi.load()
    err = ctypes.create_string_buffer(512)
    rc = lib.pbmoe_moe_layer_static(ctypes.byref(cfg), ctypes.byref(w.c_weights()), ctypes.c_void_p(x.data_ptr()),
                                    capi._dtype_code(x), None, ctypes.c_void_p(out.data_ptr()), capi._dtype_code(out),
                                    5, None, None, None, err, len(err),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == capi.PBMOE_OK, err.value.decode()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
