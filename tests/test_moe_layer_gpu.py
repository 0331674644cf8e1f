"""pbmoe_moe_layer and pbmoe_route_topk against the CPU oracle.

Routing is integer work: route ids must match bit-exactly. The router kernel
computes every logit as the reference's sequential fp32 fma chain over the
columns (dense_mmap_fma_matvec_bf16, shaders.metal:1059-1075, restated by the
oracle), so the logits themselves are compared bit for bit, and with them the
route ids of every token; the selection function is also checked on
identical logits. Each check reports how many tokens are near-ties (a K-th /
(K+1)-th logit gap inside a summation-order rounding bound): those are the
tokens any other summation order could route differently, and they are
asserted like all the others.
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
    yield c
    c.close()


def _host_u16(t):
    from pb_b200.synth import bf16_bits

    return bf16_bits(t).cpu().numpy().view(np.uint16)


def _run_layer(ctx, w, x, tokens, top_k, residual=None, norm_w=None, out_dtype=None, routed_scale=1.0,
               normalization=0, input_norm=None):
    import torch

    from pb_b200 import capi

    cfg = capi.moe_config(w.layout, w.num_experts, top_k, normalization=normalization, routed_scale=routed_scale)
    ctx.reserve(max(tokens, 1), cfg)
    od = out_dtype or x.dtype
    out = torch.empty(tokens, w.hidden, device="cuda", dtype=od)
    nn = torch.empty_like(out) if norm_w is not None else None
    logits = torch.empty(tokens, w.num_experts, device="cuda")
    ids = torch.empty(tokens, top_k, device="cuda", dtype=torch.int32)
    rw = torch.empty(tokens, top_k, device="cuda")
    sl = torch.empty(tokens, device="cuda")
    xn = torch.empty(tokens, w.hidden, device="cuda", dtype=torch.bfloat16)
    dbg = capi.MoeDebug(logits.data_ptr(), ids.data_ptr(), rw.data_ptr(), sl.data_ptr(), None, xn.data_ptr())
    cw = w.c_weights()
    if input_norm is not None:
        cw.input_norm_weight = input_norm.data_ptr()
    ctx.moe_layer(cfg, cw, x, out, tokens, residual=residual, next_norm_weight=norm_w, next_normed=nn,
                  debug=dbg)
    torch.cuda.synchronize()
    status = ctx.device_status()
    return dict(out=out, nn=nn, logits=logits, ids=ids, rw=rw, sl=sl, xn=xn, status=status)


def _oracle_layer(oracle, w, x_np, top_k, residual=None, routed_scale=1.0):
    offs = np.array(list(w.layout.component_offsets), np.uint64)
    return oracle.moe_layer(
        x_np, _host_u16(w.router), w.experts.cpu().numpy(), offs, int(w.layout.expert_bytes),
        w.num_experts, top_k, w.intermediate, w.group,
        shared_slot=None if w.shared is None else w.shared.cpu().numpy(),
        shared_gate_bits=None if w.shared_gate is None else _host_u16(w.shared_gate),
        residual=residual, routed_scale=routed_scale, threads=8)


def near_ties(logits_ref, k, hidden, x):
    """Tokens whose routing a different summation order could flip: the gap
    between the K-th and (K+1)-th largest logit is inside a generous bound on
    two dot products' rounding difference (reported, not excused)."""
    srt = -np.sort(-logits_ref, axis=1)
    gap = srt[:, k - 1] - srt[:, k]
    bound = 64 * np.finfo(np.float32).eps * np.sqrt(hidden) * (np.abs(x).max(axis=1) * 0.1 + 1)
    return int(np.sum(gap <= bound))


def check_routing(oracle, r, ref_logits, ref_ids, ref_w, top_k, hidden, x_np, what=""):
    """Router logits and every token's route ids bit-exact; weights within tolerance."""
    lg = r["logits"].cpu().numpy()
    assert np.array_equal(lg.view(np.uint32), ref_logits.view(np.uint32)), \
        f"{what}: router logits differ from the sequential fma chain ({np.sum(lg != ref_logits)} entries)"
    gids = r["ids"].cpu().numpy().view(np.uint32)
    for t in range(lg.shape[0]):
        oid, _ = oracle.routing_softmax_top_k(lg[t], top_k)
        assert gids[t].tolist() == oid.tolist(), f"{what} token {t}: selection differs on identical logits"
    assert np.array_equal(gids, ref_ids), f"{what}: routed experts differ from the oracle"
    assert_close(r["rw"].cpu().numpy(), ref_w, what=f"{what} route weights")
    ties = near_ties(ref_logits, top_k, hidden, x_np)
    print(f"{what}: {lg.shape[0]} tokens routed bit-exactly, {ties} of them near-ties")
    return ties


def _check_layer(ctx, oracle, w, tokens, top_k, seed, residual=False, norm=False, out_dtype=None):
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", seed)
    x = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda")
    res = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda") if residual else None
    norm_w = torch.rand(w.hidden, device="cuda", generator=g) + 0.5 if norm else None
    r = _run_layer(ctx, w, x, tokens, top_k, residual=res, norm_w=norm_w, out_dtype=out_dtype)
    assert r["status"] == 0
    x_np = x.float().cpu().numpy()
    ref_out, ref_ids, ref_w, ref_logits = _oracle_layer(oracle, w, x_np, top_k,
                                                        residual=None if res is None else res.float().cpu().numpy())
    check_routing(oracle, r, ref_logits, ref_ids, ref_w, top_k, w.hidden, x_np, what=f"T={tokens}")
    assert_close(r["out"].float().cpu().numpy(), ref_out, what="layer output")
    if norm:
        ref_nn = np.stack([oracle.rms_norm(ref_out[t], norm_w.cpu().numpy()) for t in range(tokens)])
        assert_close(r["nn"].float().cpu().numpy(), ref_nn, what="next-layer norm")
    return r


@pytest.fixture(scope="module")
def small_layer():
    from pb_b200 import synth

    return synth.MoeLayerWeights("cuda", seed=11, hidden=512, num_experts=64, intermediate=256, group=64)


@pytest.mark.parametrize("tokens", [1, 3, 8, 33])
def test_small_layer(ctx, oracle, small_layer, tokens):
    _check_layer(ctx, oracle, small_layer, tokens, top_k=6, seed=100 + tokens, residual=True, norm=True)


def test_small_layer_f32_activations(ctx, oracle, small_layer):
    import torch

    _check_layer(ctx, oracle, small_layer, 4, top_k=4, seed=7, out_dtype=torch.float32)


def test_no_shared_expert(ctx, oracle):
    from pb_b200 import synth

    w = synth.MoeLayerWeights("cuda", seed=5, hidden=256, num_experts=32, intermediate=128, group=32, shared=False)
    _check_layer(ctx, oracle, w, 5, top_k=4, seed=9)


def test_shared_expert_without_gate(ctx, oracle):
    from pb_b200 import synth

    w = synth.MoeLayerWeights("cuda", seed=6, hidden=256, num_experts=16, intermediate=96, group=32,
                              shared_gate=False)
    _check_layer(ctx, oracle, w, 2, top_k=2, seed=3)


@pytest.mark.parametrize("tokens,x_f32", [(3, True), (12, False), (9, True)])
def test_tensor_core_path_i256(ctx, oracle, tokens, x_f32):
    """Hidden 2048 / group 64 selects the tensor-core expert kernels; this
    covers intermediate 256, f32 activations (hi/lo rows) and bf16 passes of
    up to 16 tokens."""
    import torch

    from pb_b200 import synth

    w = synth.MoeLayerWeights("cuda", seed=21, hidden=2048, num_experts=48, intermediate=256, group=64)
    if x_f32:
        g = synth.gen("cuda", 5)
        x = synth.normal_bf16((tokens, w.hidden), 1.0, g, "cuda").float() * 1.37
        r = _run_layer(ctx, w, x, tokens, 8, out_dtype=torch.float32)
        assert r["status"] == 0
        x_np = x.cpu().numpy()
        ref_out, ref_ids, ref_w, ref_logits = _oracle_layer(oracle, w, x_np, 8)
        check_routing(oracle, r, ref_logits, ref_ids, ref_w, 8, w.hidden, x_np, what="f32 x")
        assert_close(r["out"].cpu().numpy(), ref_out, what="f32 layer output")
    else:
        _check_layer(ctx, oracle, w, tokens, top_k=8, seed=13)


@pytest.fixture(scope="module")
def config1_layer():
    from pb_b200 import synth

    return synth.MoeLayerWeights("cuda", seed=2024)


@pytest.mark.parametrize("tokens", [1, 8, 9, 20, 32, 33, 40])
def test_config1_layer(ctx, oracle, config1_layer, tokens):
    """Config 1: hidden 2048, 512 experts top-10, I=512, group 64, shared expert;
    every token's route ids bit-exact, every output within 1e-2. 9 to 32
    tokens run as one launch of the gathered expert pipe (groups of at most 8
    routes; up to 12 tokens the expert kernels build the group plan by
    ranking, above by block scans), 33 and 40 as a 32-token launch and a
    1- or 8-token one."""
    _check_layer(ctx, oracle, config1_layer, tokens, top_k=10, seed=77 + tokens)


def _check_layer_x(ctx, oracle, w, x, top_k):
    r = _run_layer(ctx, w, x, x.shape[0], top_k)
    assert r["status"] == 0
    x_np = x.float().cpu().numpy()
    ref_out, ref_ids, ref_w, ref_logits = _oracle_layer(oracle, w, x_np, top_k)
    check_routing(oracle, r, ref_logits, ref_ids, ref_w, top_k, w.hidden, x_np, what=f"T={x.shape[0]}")
    assert_close(r["out"].float().cpu().numpy(), ref_out, what="layer output")
    return r


def test_config1_repeated_tokens_split_groups(ctx, oracle, config1_layer):
    """32 tokens, 27 of them the same row: those route to the same 10
    experts, whose 27+ routes each (and the shared expert's 32) the plan
    splits into groups of at most 8 for the gathered expert pipe."""
    from pb_b200 import synth

    g = synth.gen("cuda", 4242)
    x = synth.normal_bf16((32, config1_layer.hidden), 1.0, g, "cuda")
    x[6:] = x[5]
    ids = _check_layer_x(ctx, oracle, config1_layer, x, 10)["ids"].cpu().numpy()
    assert (ids[6:] == ids[5]).all()


def test_config1_all_distinct_experts(ctx, oracle, config1_layer):
    """32 tokens whose top-10 experts are all different (a router of unit
    rows: logit e of a token is its column e, set high on 10 columns per
    token): 320 single-route groups + 4 shared-expert groups, so some CTAs of
    the down kernel walk three groups and reuse an activation buffer."""
    import copy

    import torch

    from pb_b200 import synth

    w = copy.copy(config1_layer)
    w.router = torch.zeros_like(config1_layer.router)
    w.router[torch.arange(w.num_experts), torch.arange(w.num_experts)] = 1.0
    g = synth.gen("cuda", 777)
    x = synth.normal_bf16((32, w.hidden), 1.0, g, "cuda")
    for t in range(32):
        x[t, 10 * t:10 * t + 10] = 8.0 + 0.25 * torch.arange(10, device="cuda")
    ids = _check_layer_x(ctx, oracle, w, x, 10)["ids"].cpu().numpy()
    assert len(set(ids.ravel().tolist())) == 320


@pytest.mark.parametrize("tokens", [1, 8, 32])
def test_config1_fused_input_norm(ctx, oracle, config1_layer, tokens):
    """The layer normalising its own input (input_norm_weight): x is the f32
    residual sum h, the router kernel writes bf16(RMSNorm(h) * w), and the
    layer output is h + MoE(that). The normalised rows are within 1e-2 of the
    oracle's rms_norm (its sum of squares runs in another order); routing and
    the layer are then checked bit-exactly / within 1e-2 on the GPU's own
    normalised rows, and the whole layer against the oracle chain from h."""
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", 300 + tokens)
    h = torch.randn(tokens, config1_layer.hidden, device="cuda", generator=g) * 3.0
    wn = (1.0 + 0.1 * torch.randn(config1_layer.hidden, device="cuda", generator=g)).float()
    r = _run_layer(ctx, config1_layer, h, tokens, 10, residual=h, input_norm=wn)
    assert r["status"] == 0
    h_np, wn_np = h.cpu().numpy(), wn.cpu().numpy()
    ref_n = np.stack([oracle.rms_norm(h_np[t], wn_np) for t in range(tokens)])
    xn = r["xn"].float().cpu().numpy()
    assert_close(xn, ref_n, what="normalised input")
    # teacher-forced on the GPU's normalised rows: routing bit-exact
    ref_out, ref_ids, ref_w, ref_logits = _oracle_layer(oracle, config1_layer, xn, 10, residual=h_np)
    check_routing(oracle, r, ref_logits, ref_ids, ref_w, 10, config1_layer.hidden, xn, what=f"fused norm T={tokens}")
    assert_close(r["out"].cpu().numpy(), ref_out, what="fused-norm layer output")


# ---------------------------------------------------------------- routing only
def _route(ctx, logits_np, k, normalization=0, scale=1.0):
    import torch

    T, E = logits_np.shape
    lg = torch.tensor(logits_np, device="cuda")
    ids = torch.empty(T, k, device="cuda", dtype=torch.int32)
    w = torch.empty(T, k, device="cuda")
    ctx.route_topk(lg, T, E, k, ids, w, normalization=normalization, scale=scale)
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint32), w.cpu().numpy(), ctx.device_status()


def _oracle_route(oracle, logits_np, k, scale=1.0):
    ids, ws = [], []
    for row in logits_np:
        i, p = oracle.routing_softmax_top_k(row, k)
        ids.append(i)
        ws.append(oracle.renormalize_routes(p, scale))
    return np.stack(ids), np.stack(ws)


def test_route_reference_slot_order(ctx, oracle):
    """math.rs:1257-1279: slot order [5, 1, 8, 3]."""
    ids, w, st = _route(ctx, np.array([[0.1, 2.0, -1.0, 3.0, 0.5, 2.5, -0.2, 1.5, 4.0]], np.float32), 4)
    assert ids[0].tolist() == [5, 1, 8, 3]
    assert st == 0
    assert np.max(np.abs(w[0] - np.array([0.12925005, 0.07839412, 0.57925856, 0.2130973]))) <= 1e-6


def test_route_huge_negative(ctx):
    """math.rs:1292-1305."""
    ids, w, st = _route(ctx, np.array([[-2.0e30, -3.0e30, -4.0e30]], np.float32), 2)
    assert ids[0].tolist() == [0, 1]
    assert abs(float(w[0].sum()) - 1.0) < 1e-6 and st == 0


@pytest.mark.parametrize("E,k", [(512, 10), (64, 8), (33, 32), (128, 1), (1000, 7)])
def test_route_random_bit_exact(ctx, oracle, E, k):
    rng = np.random.default_rng(E * 31 + k)
    lg = rng.standard_normal((64, E)).astype(np.float32)
    ids, w, st = _route(ctx, lg, k)
    rid, rw = _oracle_route(oracle, lg, k)
    assert st == 0
    assert np.array_equal(ids, rid)
    assert_close(w, rw, tol=1e-5, what="weights")


def test_route_ties_and_specials(ctx, oracle):
    """Ties (earlier expert wins, first minimum slot replaced), -inf and NaN
    scores, signed zeros."""
    rows = [
        np.zeros(40, np.float32),
        np.array([1.0, 1.0, 1.0, 2.0, 2.0, 0.5, 2.0, 1.0] * 5, np.float32),
        np.concatenate([np.full(20, -np.inf, np.float32), np.arange(20, dtype=np.float32)]),
        np.where(np.arange(40) % 3 == 0, np.nan, np.arange(40, dtype=np.float32)).astype(np.float32),
        np.array([-0.0, 0.0] * 20, np.float32),
        np.round(np.random.default_rng(3).standard_normal(40) * 2).astype(np.float32),
    ]
    lg = np.stack(rows)
    ids, w, st = _route(ctx, lg, 6)
    rid, rw = _oracle_route(oracle, lg, 6)
    assert np.array_equal(ids, rid)
    assert_close(w, rw, tol=1e-5, what="weights")
    assert st == 0


@pytest.mark.parametrize("k", [1, 2, 10, 16, 32])
def test_route_selection_paths(ctx, oracle, k):
    """Rows that take the parallel selection (distinct scores, at most 64
    insertions) and rows that fall back to the replay (ties among inserted
    scores, ascending scores with one insertion per expert), all bit-exact."""
    rng = np.random.default_rng(500 + k)
    E = 512
    rows = [rng.standard_normal(E) for _ in range(6)]
    rows.append(np.sort(rng.standard_normal(E)))  # every expert inserted
    rows.append(np.sort(rng.standard_normal(E))[::-1])  # only the first k inserted
    rows.append(np.round(rng.standard_normal(E) * 4))  # ties
    r = rng.standard_normal(E)
    r[::7] = np.nan
    r[3::11] = -np.inf
    rows.append(r)  # NaN and -inf are never inserted
    bf = rng.standard_normal(E).astype(np.float32).view(np.uint32) & 0xFFFF0000
    rows.append(bf.view(np.float32))  # bf16-valued scores
    rows.append(np.linspace(-1.0, 1.0, E) + rng.standard_normal(E) * 0.05)  # drifting upwards
    lg = np.stack(rows).astype(np.float32)
    ids, w, st = _route(ctx, lg, k)
    rid, rw = _oracle_route(oracle, lg, k)
    assert np.array_equal(ids, rid)
    assert_close(w, rw, tol=1e-5, what="weights")
    assert st == 0


def test_route_all_neg_inf_latches_error(ctx):
    """All -inf logits: the reference bails on the selected-probability sum;
    the kernel latches PBMOE_DEV_ERR_ROUTE_WEIGHTS."""
    from pb_b200 import capi

    _, _, st = _route(ctx, np.full((1, 16), -np.inf, np.float32), 4)
    assert st & capi.PBMOE_DEV_ERR_ROUTE_WEIGHTS


def test_route_routed_scale_and_floor(ctx, oracle):
    rng = np.random.default_rng(12)
    lg = rng.standard_normal((8, 96)).astype(np.float32)
    ids, w, st = _route(ctx, lg, 8, scale=2.5)
    rid, rw = _oracle_route(oracle, lg, 8, scale=2.5)
    assert np.array_equal(ids, rid) and st == 0
    assert_close(w, rw, tol=1e-5, what="scaled weights")
    ids, w, st = _route(ctx, lg, 8, normalization=1)
    ref = []
    for row in lg:
        _, p = oracle.routing_softmax_top_k(row, 8)
        ref.append(oracle.renormalize_routes(p, 1.0, policy=1))
    assert_close(w, np.stack(ref), tol=1e-5, what="floor weights")


def test_moe_layer_rejects_bad_calls(ctx, small_layer):
    import torch

    from pb_b200 import capi

    cfg = capi.moe_config(small_layer.layout, small_layer.num_experts, 6)
    ctx.reserve(2, cfg)
    x = torch.zeros(4, small_layer.hidden, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(x)
    with pytest.raises(capi.PbmoeError) as e:  # more tokens than reserved
        ctx.moe_layer(cfg, small_layer.c_weights(), x, out, 4)
    assert e.value.code == capi.PBMOE_ERR_NO_WORKSPACE
    bad = capi.moe_config(small_layer.layout, small_layer.num_experts, 40)
    with pytest.raises(capi.PbmoeError) as e:
        ctx.moe_layer(bad, small_layer.c_weights(), x, out, 1)
    assert e.value.code == capi.PBMOE_ERR_UNSUPPORTED


@pytest.mark.parametrize("tokens,out_f32,pinned", [(1, False, True), (8, True, True), (12, False, True),
                                                   (8, False, False)])
def test_moe_layer_host_rows(ctx, config1_layer, tokens, out_f32, pinned):
    """pbmoe_moe_layer_host (host x / residual / out) equals pbmoe_moe_layer on
    device rows, bit for bit: with page-locked buffers the residual and the
    output are used in place, with pageable ones everything is copied."""
    import torch

    from pb_b200 import capi, synth

    w = config1_layer
    cfg = capi.moe_config(w.layout, w.num_experts, 10)
    ctx.reserve(32, cfg)
    dt = torch.float32 if out_f32 else torch.bfloat16
    x = synth.normal_bf16((tokens, w.hidden), 1.0, synth.gen("cuda", 90 + tokens), "cuda")
    res = synth.normal_bf16((tokens, w.hidden), 1.0, synth.gen("cuda", 91), "cuda").to(dt)
    ref = torch.empty(tokens, w.hidden, device="cuda", dtype=dt)
    ctx.moe_layer(cfg, w.c_weights(), x, ref, tokens, residual=res)
    pin = (lambda t: t.pin_memory()) if pinned else (lambda t: t)
    hx, hres = pin(x.cpu()), pin(res.cpu())
    hout = pin(torch.full((tokens, w.hidden), float("nan"), dtype=dt))
    s = torch.cuda.current_stream()
    ctx.moe_layer_host(cfg, w.c_weights(), hx, hout, tokens, residual=hres, stream=s)
    s.synchronize()
    assert ctx.device_status() == 0
    assert torch.equal(hout, ref.cpu())


def test_sync_bounded_wait(ctx, small_layer):
    """pbmoe_sync returns once the stream is idle (the CMD3 submission's wait)."""
    import torch

    from pb_b200 import capi, synth

    cfg = capi.moe_config(small_layer.layout, small_layer.num_experts, 6)
    ctx.reserve(4, cfg)
    x = synth.normal_bf16((4, small_layer.hidden), 1.0, synth.gen("cuda", 5), "cuda")
    out = torch.empty_like(x)
    for _ in range(20):
        ctx.moe_layer(cfg, small_layer.c_weights(), x, out, 4)
    ctx.sync(timeout_ms=10000)
    assert torch.cuda.current_stream().query()
    ctx.sync(timeout_ms=0)  # idle: polling succeeds
