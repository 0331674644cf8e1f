"""Decode-step glue and a whole config-4-shaped step against the CPU oracle.

  pbmoe_rms_norm         rms_norm_reduced (shaders.metal:1176-1213) / the
                         reference's rms_norm_with_weight_and_epsilon_in_place
                         (math.rs:151-167), with the fused residual add
  pbmoe_mla_rope_append  apply_rotary_interleaved_to_split_half (math.rs:
                         822-846) on the query and key rope parts, bit-exact,
                         and the cache rows of KvCache::record_mla_kv
  DecodeStep             two layers of MLA attention + MoE and the vocab head,
                         chained from the oracle's functions in the same order
                         (runtime/mod.rs:1432-2024, 2779-2940); hidden state
                         within 2e-2 after two layers
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


def _f32_of_bf16(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("x_dtype,out_dtype", [("f32", "f32"), ("bf16", "bf16"), ("f32", "bf16")])
def test_rms_norm_rows(ctx, oracle, x_dtype, out_dtype):
    import torch

    dt = {"f32": torch.float32, "bf16": torch.bfloat16}
    g = torch.Generator("cuda").manual_seed(3)
    x = torch.randn(5, 700, generator=g, device="cuda").to(dt[x_dtype])
    res = torch.randn(5, 700, generator=g, device="cuda").to(dt[x_dtype])
    w = (1 + 0.1 * torch.randn(700, generator=g, device="cuda")).float()
    out = torch.empty(5, 700, device="cuda", dtype=dt[out_dtype])
    s = torch.empty(5, 700, device="cuda", dtype=torch.float32)
    ctx.rms_norm(x, w, out, eps=1e-6, residual=res, sum_out=s)
    torch.cuda.synchronize()
    xs = x.float().cpu().numpy() + res.float().cpu().numpy()
    ref = np.stack([oracle.rms_norm(r, w.cpu().numpy(), 1e-6) for r in xs])
    assert np.array_equal(s.cpu().numpy(), xs.astype(np.float32))
    assert_close(out.float().cpu().numpy(), ref, tol=1e-5 if out_dtype == "f32" else 8e-3, what="rms norm")


def test_rms_norm_strided_in_place(ctx, oracle):
    """The kv_a case: the first 512 of 576 columns normed in place."""
    import torch

    g = torch.Generator("cuda").manual_seed(4)
    kv = torch.randn(3, 576, generator=g, device="cuda")
    w = (1 + 0.1 * torch.randn(512, generator=g, device="cuda")).float()
    before = kv.cpu().numpy()
    ctx.rms_norm(kv, w, kv, width=512)
    torch.cuda.synchronize()
    after = kv.cpu().numpy()
    assert np.array_equal(after[:, 512:], before[:, 512:])
    ref = np.stack([oracle.rms_norm(r[:512], w.cpu().numpy(), 1e-6) for r in before])
    assert_close(after[:, :512], ref, tol=1e-5, what="strided rms norm")


def test_mla_rope_append_bit_exact(ctx, oracle):
    import torch

    from pb_b200 import capi, synth

    cfg = capi.mla_config()
    B, ctxlen = 3, 40
    ctx.rope_reserve(ctxlen, 64, 10000.0)
    g = torch.Generator("cuda").manual_seed(5)
    q = torch.randn(B, 16, 192, generator=g, device="cuda")
    kv = torch.randn(B, 576, generator=g, device="cuda")
    pos = [0, 17, 39]
    ckv = [synth.normal_bf16((ctxlen, 512), 1.0, synth.gen("cuda", 10 + b), "cuda") for b in range(B)]
    kr = [synth.normal_bf16((ctxlen, 64), 1.0, synth.gen("cuda", 20 + b), "cuda") for b in range(B)]
    ptr = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")
    q0, kv0 = q.cpu().numpy(), kv.cpu().numpy()
    ctx.mla_rope_append(cfg, q, kv, torch.tensor(pos, dtype=torch.int32, device="cuda"), ptr(ckv), ptr(kr), ctxlen)
    torch.cuda.synchronize()
    assert ctx.device_status() == 0
    qg = q.cpu().numpy()
    for b in range(B):
        for h in range(16):
            ref = oracle.rope_interleaved_to_split_half(q0[b, h, 128:], pos[b], 64, 10000.0)
            assert np.array_equal(qg[b, h, 128:], ref)
            assert np.array_equal(qg[b, h, :128], q0[b, h, :128])
        kref = oracle.rope_interleaved_to_split_half(kv0[b, 512:], pos[b], 64, 10000.0)
        assert np.array_equal(_f32_of_bf16(kr[b][pos[b]]), oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(kref)))
        assert np.array_equal(_f32_of_bf16(ckv[b][pos[b]]),
                              oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(kv0[b, :512])))


def test_mla_rope_append_bad_position(ctx):
    import torch

    from pb_b200 import capi, synth

    cfg = capi.mla_config()
    ctx.rope_reserve(16, 64, 10000.0)
    ckv = synth.normal_bf16((16, 512), 1.0, synth.gen("cuda", 1), "cuda")
    kr = synth.normal_bf16((16, 64), 1.0, synth.gen("cuda", 2), "cuda")
    before = ckv.clone()
    q = torch.zeros(1, 16, 192, device="cuda")
    kv = torch.ones(1, 576, device="cuda")
    ptr = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device="cuda")
    ctx.device_status(clear=True)
    ctx.mla_rope_append(cfg, q, kv, torch.tensor([16], dtype=torch.int32, device="cuda"), ptr(ckv), ptr(kr), 16)
    torch.cuda.synchronize()
    assert ctx.device_status(clear=True) & capi.PBMOE_DEV_ERR_POSITION
    assert torch.equal(ckv, before)


def _oracle_step(oracle, model, caches_np, x, positions):
    """The same step on the CPU from the oracle's functions."""
    from pb_b200 import synth

    cfg = model.cfg
    u16 = lambda t: synth.bf16_bits(t).cpu().numpy().view(np.uint16)
    bf = lambda a: oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(np.asarray(a, np.float32)))
    q4 = lambda P, v: oracle.q4_fma_matvec_bf16(P.packed.cpu().numpy(), v, u16(P.scales).reshape(-1),
                                                u16(P.biases).reshape(-1), P.rows, P.cols, P.group)
    B = x.shape[0]
    x = x.copy()
    xn = np.stack([oracle.rms_norm(x[b], model.layers[0].input_norm.cpu().numpy(), cfg.eps) for b in range(B)])
    for i, L in enumerate(model.layers):
        n_rows, h_rows = [], []
        for b in range(B):
            qa = oracle.rms_norm(q4(L.q_a, xn[b]), L.q_a_norm.cpu().numpy(), cfg.eps)
            kv = q4(L.kv_a, xn[b])
            kv[:cfg.latent] = oracle.rms_norm(kv[:cfg.latent], L.kv_a_norm.cpu().numpy(), cfg.eps)
            q = q4(L.q_b, qa).reshape(cfg.heads, cfg.nope + cfg.rope)
            for h in range(cfg.heads):
                q[h, cfg.nope:] = oracle.rope_interleaved_to_split_half(q[h, cfg.nope:], positions[b], cfg.rope,
                                                                        cfg.theta)
            krot = oracle.rope_interleaved_to_split_half(kv[cfg.latent:], positions[b], cfg.rope, cfg.theta)
            lat, rot = caches_np[0][i][b], caches_np[1][i][b]
            lat[positions[b]] = bf(kv[:cfg.latent])
            rot[positions[b]] = bf(krot)
            n = positions[b] + 1
            attn = oracle.mla_absorbed_attention(q.reshape(-1), lat[:n], rot[:n], u16(L.w_uk), u16(L.w_uv),
                                                 cfg.heads, cfg.nope, cfg.rope, cfg.latent, cfg.v_dim)
            o = q4(L.o_proj, attn)
            h_row = x[b] + o
            h_rows.append(h_row)
            n_rows.append(bf(oracle.rms_norm(h_row, L.post_norm.cpu().numpy(), cfg.eps)))
        m = L.moe
        offs = np.array(list(m.layout.component_offsets), np.uint64)
        out, ids, _, _ = oracle.moe_layer(np.stack(n_rows), u16(m.router), m.experts.cpu().numpy(), offs,
                                          int(m.layout.expert_bytes), cfg.experts, cfg.top_k, cfg.inter, cfg.group,
                                          shared_slot=m.shared.cpu().numpy(), shared_gate_bits=u16(m.shared_gate),
                                          residual=np.stack(h_rows))
        x = out
        nxt = model.layers[i + 1].input_norm if i + 1 < len(model.layers) else model.final_norm
        xn = np.stack([oracle.rms_norm(x[b], nxt.cpu().numpy(), cfg.eps) for b in range(B)])
    return x, xn


def test_decode_step_two_layers(ctx, oracle):
    import torch

    from pb_b200 import decode

    cfg = decode.StepConfig(hidden=512, layers=2, q_lora=512, experts=64, top_k=6, inter=256, vocab=3000,
                            context=40, candidates=16)
    model = decode.Model(cfg, seed=3)
    B, positions = 3, [4, 21, 39]
    caches = decode.Caches(cfg, B, seed=3)
    caches_np = ([[t.float().cpu().numpy() for t in l] for l in caches.c_kv],
                 [[t.float().cpu().numpy() for t in l] for l in caches.k_rope])
    step = decode.DecodeStep(ctx, model, caches, B, positions)
    x0 = torch.randn(B, cfg.hidden, generator=torch.Generator("cuda").manual_seed(9), device="cuda")
    step.set_input(x0)
    step.launch()
    torch.cuda.synchronize()
    assert ctx.device_status() == 0
    rx, rxn = _oracle_step(oracle, model, caches_np, x0.cpu().numpy(), positions)
    assert_close(step.x.cpu().numpy(), rx, tol=2e-2, what="hidden after two layers")
    assert_close(step.xn.cpu().numpy(), rxn, tol=2e-2, what="final-normed hidden")
    # the head ran on the kernel's final-normed hidden: its selection is the oracle's on those inputs
    from pb_b200 import synth

    ids = step.ids.cpu().numpy().view(np.uint32)
    rid, _, _ = oracle.head_topk(synth.bf16_bits(model.head).cpu().numpy().view(np.uint16),
                                 step.xn.cpu().numpy(), cfg.candidates)
    overlap = np.mean([len(set(ids[b]) & set(rid[b])) / cfg.candidates for b in range(B)])
    assert overlap >= 0.9, f"head candidates overlap {overlap:.2f}"
