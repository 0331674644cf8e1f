"""Prefill path (config 2) through the C-ABI against the CPU oracle:

  pbmoe_q4_gemm            dense X . W^T (q4_mmap_fma_matvec_batch_bf16_scale_bias,
                           shaders.metal:973-1057, one matrix)
  pbmoe_prefill_group_plan slots in ascending expert order
                           (scheduler/mod.rs:720-765) + qwen_layer_major_group_plan
                           (metal/mod.rs:3197-3233): bit-exact
  pbmoe_q4_gemm_grouped    per-slot X_group . W_e^T with the gather fused
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
    c.prefill_reserve(20480, 2048)
    yield c
    c.close()


def _u16(t):
    from pb_b200.synth import bf16_bits

    return bf16_bits(t).cpu().numpy().view(np.uint16).reshape(-1)


def _gemm(ctx, packed, s, b, n, k, x, out_dtype):
    import torch

    y = torch.empty(x.shape[0], n, device="cuda", dtype=out_dtype)
    ctx.q4_gemm(packed, s, b, n, k, 64, x, y)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


@pytest.mark.parametrize("m,n,k", [
    (1, 128, 512), (5, 200, 512), (130, 257, 1024), (128, 128, 2048), (300, 512, 512), (17, 1000, 1536),
    (520, 384, 3072), (129, 5, 512),
])
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_dense_gemm_shapes(ctx, oracle, m, n, k, out):
    """Ragged token counts (tiles of 128 tokens), weight rows not a multiple
    of 128, K from one to eight 512-wide runs of groups."""
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", m * 7919 + n * 31 + k)
    packed, s, b = synth.q4_matrix(n, k, 64, g, "cuda")
    x = synth.normal_bf16((m, k), 1.0, g, "cuda")
    y = _gemm(ctx, packed, s, b, n, k, x, torch.bfloat16 if out == "bf16" else torch.float32)
    ref = oracle.q4_gemm(x.float().cpu().numpy(), packed.cpu().numpy(), _u16(s), _u16(b), n, k, 64, threads=8)
    assert_close(y, ref, what=f"gemm {m}x{n}x{k}")


def test_dense_gemm_f16_input(ctx, oracle):
    """fp16 activations go straight to the tensor cores (no workspace)."""
    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", 77)
    packed, s, b = synth.q4_matrix(384, 512, 64, g, "cuda")
    x = synth.normal_bf16((70, 512), 1.0, g, "cuda")
    y = _gemm(ctx, packed, s, b, 384, 512, x.half(), torch.float32)
    ref = oracle.q4_gemm(x.float().cpu().numpy(), packed.cpu().numpy(), _u16(s), _u16(b), 384, 512, 64, threads=8)
    assert_close(y, ref, what="f16 input")


def test_dense_gemm_needs_workspace():
    import torch

    from pb_b200 import capi, synth

    c = capi.Context(0)
    try:
        g = synth.gen("cuda", 8)
        packed, s, b = synth.q4_matrix(128, 512, 64, g, "cuda")
        x = synth.normal_bf16((4, 512), 1.0, g, "cuda")
        y = torch.empty(4, 128, device="cuda", dtype=torch.float32)
        with pytest.raises(capi.PbmoeError) as e:
            c.q4_gemm(packed, s, b, 128, 512, 64, x, y)
        assert e.value.code == capi.PBMOE_ERR_NO_WORKSPACE
        c.prefill_reserve(4, 512)
        c.q4_gemm(packed, s, b, 128, 512, 64, x, y)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
    finally:
        c.close()


def test_dense_gemm_config2(ctx, oracle):
    """Config 2 dense: X bf16 [2048 x 2048], W Q4 [5120 x 2048], y bf16;
    every one of the 2048 x 5120 outputs against the oracle."""
    import os

    import torch

    from pb_b200 import synth

    g = synth.gen("cuda", 2002)
    packed, s, b = synth.q4_matrix(5120, 2048, 64, g, "cuda")
    x = synth.normal_bf16((2048, 2048), 1.0, g, "cuda")
    y = _gemm(ctx, packed, s, b, 5120, 2048, x, torch.bfloat16)
    xs = x.float().cpu().numpy()
    ref = oracle.q4_gemm(xs, packed.cpu().numpy(), _u16(s), _u16(b), 5120, 2048, 64, threads=os.cpu_count() or 8)
    assert_close(y, ref, what="config2 dense")


def test_dense_gemm_rejects(ctx):
    import torch

    from pb_b200 import capi, synth

    g = synth.gen("cuda", 5)
    packed, s, b = synth.q4_matrix(64, 96, 32, g, "cuda")
    x = synth.normal_bf16((4, 96), 1.0, g, "cuda")
    y = torch.empty(4, 64, device="cuda", dtype=torch.float32)
    with pytest.raises(capi.PbmoeError) as e:
        ctx.q4_gemm(packed, s, b, 64, 96, 32, x, y)
    assert e.value.code == capi.PBMOE_ERR_UNSUPPORTED
    packed, s, b = synth.q4_matrix(64, 512, 64, g, "cuda")
    with pytest.raises(capi.PbmoeError) as e:
        ctx.q4_gemm(packed, s, b, 64, 512, 64, torch.zeros(4, 512, device="cuda"), y)  # f32 x
    assert e.value.code == capi.PBMOE_ERR_UNSUPPORTED
    packed, s, b = synth.q4_matrix(64, 576, 64, g, "cuda")
    with pytest.raises(capi.PbmoeError) as e:  # K not a multiple of 512
        ctx.q4_gemm(packed, s, b, 64, 576, 64, synth.normal_bf16((4, 576), 1.0, g, "cuda"), y)
    assert e.value.code == capi.PBMOE_ERR_UNSUPPORTED


def test_dense_gemm_f16_range_latches(ctx):
    """fp16 operands: an activation of magnitude >= 65536 has no fp16 value,
    so the GEMM latches PBMOE_DEV_ERR_F16_RANGE; 65280 (the largest bf16
    below it) converts exactly and does not."""
    import torch

    from pb_b200 import capi, synth

    g = synth.gen("cuda", 6)
    packed, s, b = synth.q4_matrix(128, 512, 64, g, "cuda")
    x = synth.normal_bf16((3, 512), 1.0, g, "cuda")
    y = torch.empty(3, 128, device="cuda", dtype=torch.float32)
    ctx.device_status(clear=True)
    x[1, 5] = 65280.0
    ctx.q4_gemm(packed, s, b, 128, 512, 64, x, y)
    assert ctx.device_status(clear=True) == 0
    x[2, 70] = -70000.0
    ctx.q4_gemm(packed, s, b, 128, 512, 64, x, y)
    assert ctx.device_status(clear=True) & capi.PBMOE_DEV_ERR_F16_RANGE


# ---------------------------------------------------------------- group plan
def _plan(ctx, route_ids, rows, k, E):
    import torch

    n = rows * k
    dev = dict(device="cuda", dtype=torch.int32)
    out = dict(slot_experts=torch.full((E,), -1, **dev), unique=torch.zeros(1, **dev),
               route_slots=torch.full((n,), -1, **dev), source_rows=torch.full((n,), -1, **dev),
               output_indices=torch.full((n,), -1, **dev), groups=torch.full((E, 2), -1, **dev))
    ctx.prefill_group_plan(route_ids, rows, k, E, out["slot_experts"], out["unique"], out["source_rows"],
                           out["output_indices"], out["groups"], route_slots=out["route_slots"])
    torch.cuda.synchronize()
    return {key: v.cpu().numpy().astype(np.int64) for key, v in out.items()}


def _host_slots(ids, E):
    """ScheduledLayerMajorExperts: slot = rank of the expert among the selected, ascending."""
    uniq = np.unique(ids)
    slot_of = np.full(E, -1, np.int64)
    slot_of[uniq] = np.arange(uniq.size)
    return uniq, slot_of[ids.reshape(-1)]


def test_plan_reference_golden(ctx):
    """tests/metal.rs:536-547: route slots [1,0,0,1], 2 unique, K=2 ->
    source_rows [0,1,0,1], output_indices [2,0,1,3], groups [(0,2),(2,2)]
    (slot 0 = the smaller expert id)."""
    import torch

    ids = torch.tensor([[9, 4], [4, 9]], device="cuda", dtype=torch.int32)
    p = _plan(ctx, ids, 2, 2, 16)
    assert p["unique"][0] == 2
    assert list(p["slot_experts"][:2]) == [4, 9]
    assert list(p["route_slots"]) == [1, 0, 0, 1]
    assert list(p["source_rows"]) == [0, 1, 0, 1]
    assert list(p["output_indices"]) == [2, 0, 1, 3]
    assert p["groups"][:2].tolist() == [[0, 2], [2, 2]]


@pytest.mark.parametrize("rows,k,E", [(1, 1, 1), (1, 10, 512), (7, 3, 20), (2048, 10, 512), (4354, 8, 256),
                                      (300, 6, 1024), (1000, 1, 64)])
def test_plan_matches_oracle(ctx, oracle, rows, k, E):
    from pb_b200 import synth

    ids = synth.random_routes(rows, E, k, synth.gen("cuda", rows + 13 * k + E), "cuda")
    p = _plan(ctx, ids, rows, k, E)
    ids_np = ids.cpu().numpy()
    uniq, slots = _host_slots(ids_np, E)
    src, idx, groups = oracle.layer_major_group_plan(slots.astype(np.uint32), uniq.size, k)
    u = int(p["unique"][0])
    assert u == uniq.size
    assert np.array_equal(p["slot_experts"][:u], uniq)
    assert np.array_equal(p["route_slots"], slots)
    assert np.array_equal(p["source_rows"], src.astype(np.int64))
    assert np.array_equal(p["output_indices"], idx.astype(np.int64))
    assert np.array_equal(p["groups"][:u], groups.astype(np.int64))


def test_plan_skewed_routes(ctx, oracle):
    """Every token on the same few experts (one group holds most routes)."""
    import torch

    rows, k, E = 3000, 4, 64
    ids = torch.arange(k, device="cuda", dtype=torch.int32).repeat(rows, 1).contiguous()
    ids[::97, 0] = 63
    p = _plan(ctx, ids, rows, k, E)
    uniq, slots = _host_slots(ids.cpu().numpy(), E)
    src, idx, groups = oracle.layer_major_group_plan(slots.astype(np.uint32), uniq.size, k)
    assert np.array_equal(p["source_rows"], src.astype(np.int64))
    assert np.array_equal(p["output_indices"], idx.astype(np.int64))
    assert np.array_equal(p["groups"][: uniq.size], groups.astype(np.int64))


def test_plan_bad_expert_latches(ctx):
    import torch

    from pb_b200 import capi

    ctx.device_status(clear=True)
    ids = torch.tensor([[1, 2], [3, 40]], device="cuda", dtype=torch.int32)
    p = _plan(ctx, ids, 2, 2, 16)
    assert p["unique"][0] == 0
    assert ctx.device_status(clear=True) & capi.PBMOE_DEV_ERR_EXPERT_ID
    with pytest.raises(capi.PbmoeError) as e:
        _plan(ctx, ids, 0, 2, 16)
    assert e.value.code == capi.PBMOE_ERR_INVALID_ARGUMENT


# ---------------------------------------------------------------- grouped gemm
def _grouped_case(ctx, oracle, tokens, E, k, H, I, projection, seed, check_slots=None, out_dtype=None):
    import torch

    from pb_b200 import capi, synth

    out_dtype = out_dtype or torch.bfloat16
    g = synth.gen("cuda", seed)
    layout = capi.fixed_q4_layout(H, I, 64)
    table = synth.expert_table(E, layout, g, "cuda")
    x = synth.normal_bf16((tokens, H if projection != "down" else I), 1.0, g, "cuda")
    ids = synth.random_routes(tokens, E, k, g, "cuda")
    p = _plan(ctx, ids, tokens, k, E)
    dev = {key: torch.from_numpy(v.astype(np.int32)).cuda() for key, v in p.items()}
    mat = capi.expert_matrix(table, layout, E, projection)
    routes = tokens * k
    y = torch.full((routes, mat.rows), float("nan"), device="cuda", dtype=out_dtype)
    ctx.q4_gemm_grouped(mat, dev["slot_experts"], dev["unique"], dev["groups"], dev["source_rows"], routes, E, x, y)
    torch.cuda.synchronize()
    assert ctx.device_status(clear=True) == 0
    yh = y.float().cpu().numpy()
    xs = x.float().cpu().numpy()
    u = int(p["unique"][0])
    slots = range(u) if check_slots is None else check_slots
    host_table = table.cpu().numpy()

    def ref_slot(s):  # the oracle for one slot's rows (slots on parallel threads)
        e = int(p["slot_experts"][s])
        start, cnt = p["groups"][s]
        blob = host_table[e]
        pk = np.ascontiguousarray(blob[mat.packed_offset: mat.packed_offset + mat.rows * mat.cols // 2])
        nb = mat.rows * (mat.cols // 64) * 2
        sc = np.ascontiguousarray(blob[mat.scales_offset: mat.scales_offset + nb]).view(np.uint16)
        bi = np.ascontiguousarray(blob[mat.biases_offset: mat.biases_offset + nb]).view(np.uint16)
        return s, e, start, cnt, oracle.q4_gemm(np.ascontiguousarray(xs[p["source_rows"][start: start + cnt]]), pk,
                                                sc, bi, mat.rows, mat.cols, 64, threads=1)

    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=16) as pool:
        for s, e, start, cnt, ref in pool.map(ref_slot, slots):
            assert_close(yh[start: start + cnt], ref, what=f"slot {s} expert {e}")
    return yh, p


@pytest.mark.parametrize("projection", ["gate", "up", "down"])
def test_grouped_small(ctx, oracle, projection):
    _grouped_case(ctx, oracle, tokens=37, E=16, k=3, H=1024, I=512, projection=projection, seed=11)


def test_grouped_big_group(ctx, oracle):
    """A slot with more than one 64-route tile (few experts, many tokens)."""
    _grouped_case(ctx, oracle, tokens=300, E=4, k=2, H=512, I=512, projection="up", seed=12)


def test_grouped_f32_out(ctx, oracle):
    import torch

    _grouped_case(ctx, oracle, tokens=50, E=8, k=2, H=512, I=512, projection="gate", seed=13,
                  out_dtype=torch.float32)


def test_grouped_bad_source_row_latches(ctx):
    """A source row outside x latches PBMOE_DEV_ERR_EXPERT_ID (the row is not read)."""
    import torch

    from pb_b200 import capi, synth

    g = synth.gen("cuda", 15)
    layout = capi.fixed_q4_layout(512, 512, 64)
    table = synth.expert_table(2, layout, g, "cuda")
    x = synth.normal_bf16((4, 512), 1.0, g, "cuda")
    i32 = dict(device="cuda", dtype=torch.int32)
    slot_experts = torch.tensor([1], **i32)
    unique = torch.tensor([1], **i32)
    groups = torch.tensor([[0, 3]], **i32)
    source_rows = torch.tensor([0, 9, 2], **i32)
    y = torch.empty(3, 512, device="cuda", dtype=torch.float32)
    ctx.device_status(clear=True)
    ctx.q4_gemm_grouped(capi.expert_matrix(table, layout, 2, "gate"), slot_experts, unique, groups, source_rows, 3,
                        1, x, y)
    torch.cuda.synchronize()
    assert ctx.device_status(clear=True) & capi.PBMOE_DEV_ERR_EXPERT_ID


@pytest.mark.parametrize("projection", ["gate", "up", "down"])
def test_grouped_config2(ctx, oracle, projection):
    """Config 2 grouped: 2048 tokens, random top-10 over 512 experts; the gate,
    up ([512 x 2048]) and down ([2048 x 512]) projections, every slot's rows
    (all 20,480 routes) against the oracle."""
    yh, p = _grouped_case(ctx, oracle, tokens=2048, E=512, k=10, H=2048, I=512, projection=projection, seed=14)
    assert np.all(np.isfinite(yh))
