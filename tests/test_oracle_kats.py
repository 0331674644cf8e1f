"""Pins the C++ oracle to the reference's own known-answer tests.

Each case in tests/golden/reference_kats.json was transcribed from a Rust unit
test of the reference (file:line in the case's "source"); the assertions here
use the tolerance that test uses.
"""

import json
import math
import os

import numpy as np
import pytest

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def f32(a):
    return np.asarray(a, np.float32)


def test_q4_matvec_closed_form(oracle):
    k = KATS["q4_matvec_closed_form"]
    out = oracle.q4_fma_matvec(k["packed"], k["input"], k["scales"], k["biases"], k["rows"], k["cols"], k["group_size"])
    assert abs(out[0] - k["expected"][0]) < k["abs_tol"]


def _nib(packed, row, col, cols):
    byte = packed[row * ((cols + 1) // 2) + col // 2]
    return (byte & 0x0F) if col % 2 == 0 else (byte >> 4)


def test_q4_matvec_variable_groups(oracle):
    k = KATS["q4_matvec_variable_groups"]
    rows, cols, g = k["rows"], k["cols"], k["group_size"]
    out = oracle.q4_fma_matvec(k["packed"], k["input"], k["scales"], k["biases"], rows, cols, g)
    gpr = -(-cols // g)
    x, s, b = f32(k["input"]), f32(k["scales"]), f32(k["biases"])
    for r in range(rows):
        exp = np.float32(0)
        for c in range(cols):
            idx = r * gpr + c // g
            q = np.float32(_nib(k["packed"], r, c, cols))
            # q.mul_add(s*x, b*x): exact product then one rounding
            exp = np.float32(exp + np.float32(np.float64(q) * np.float64(s[idx] * x[c]) + np.float64(b[idx] * x[c])))
        assert abs(out[r] - exp) < k["abs_tol"]


def test_q4_matvec_explicit_dequant(oracle):
    k = KATS["q4_matvec_explicit_dequant"]
    rows, cols, g = k["rows"], k["cols"], k["group_size"]
    out = oracle.q4_fma_matvec(k["packed"], k["input"], k["scales"], k["biases"], rows, cols, g)
    gpr = -(-cols // g)
    x, s, b = f32(k["input"]), f32(k["scales"]), f32(k["biases"])
    for r in range(rows):
        exp = np.float32(0)
        for c in range(cols):
            idx = r * gpr + c // g
            q = np.float32(_nib(k["packed"], r, c, cols))
            exp = np.float32(exp + np.float32(np.float32(q * s[idx] + b[idx]) * x[c]))
        assert abs(out[r] - exp) <= k["abs_tol"]


def test_q4_dequantize_rows_golden(oracle):
    k = KATS["q4_dequantize_rows"]
    out = oracle.q4_dequantize_rows(k["packed"], k["scales"], k["biases"], k["rows"], k["cols"], k["group_size"])
    assert out.tolist() == k["expected"]


def test_q4_unpacked_nibbles(oracle):
    k = KATS["q4_dequantize_rows"]
    nib = oracle.q4_unpack_nibbles(k["packed"], 2, 5)
    assert nib.tolist() == [[0, 1, 2, 3, 4], [5, 6, 7, 8, 9]]


def test_q4_bf16_u32_word(oracle):
    k = KATS["q4_bf16_u32_word"]
    packed = np.frombuffer(np.uint32(k["packed_word_le"]).tobytes(), np.uint8)
    out = oracle.q4_fma_matvec_bf16(packed, k["input"], [k["scale_bf16"]], [k["bias_bf16"]], 1, 8, 8)
    assert abs(out[0] - k["expected"][0]) <= k["abs_tol"]
    # The test-only reference_q4_matvec form (no FMA) agrees as well.
    out2 = oracle.reference_q4_matvec(packed, k["input"], [k["scale_bf16"]], [k["bias_bf16"]], 1, 8, 8)
    assert abs(out2[0] - k["expected"][0]) <= k["abs_tol"]


def _bf(a):
    from oracle.pb_oracle import f32_to_bf16_bits

    return f32_to_bf16_bits(f32(a))


def test_expert_pack_mlp(oracle):
    k = KATS["expert_pack_mlp"]
    H, I, G = k["hidden"], k["intermediate"], k["group_size"]
    gate = oracle.q4_fma_matvec_bf16(k["gate_packed"], k["input"], _bf(k["gate_scales"]), _bf(k["gate_biases"]), I, H, G)
    up = oracle.q4_fma_matvec_bf16(k["up_packed"], k["input"], _bf(k["up_scales"]), _bf(k["up_biases"]), I, H, G)
    assert gate.tolist() == k["expected_gate"]
    assert up.tolist() == k["expected_up"]
    # Whole-expert slot with one group per row (G >= cols): build it with the
    # generic nine-offset layout and run the SwiGLU expert.
    parts = [
        np.asarray(k["gate_packed"], np.uint8), _bf(k["gate_scales"]), _bf(k["gate_biases"]),
        np.asarray(k["up_packed"], np.uint8), _bf(k["up_scales"]), _bf(k["up_biases"]),
        np.asarray(k["down_packed"], np.uint8), _bf(k["down_scales"]), _bf(k["down_biases"]),
    ]
    offs, blob, off = [], b"", 0
    for p in parts:
        offs.append(off)
        raw = p.tobytes()
        blob += raw
        off += len(raw)
    out = oracle.expert_swiglu(np.frombuffer(blob, np.uint8), np.asarray(offs, np.uint64), H, I, G, k["input"])
    silu = lambda v: v / (1.0 + math.exp(-v))
    inter = [silu(gate[i]) * up[i] for i in range(I)]
    for i in range(H):
        assert abs(out[i] - 15.0 * inter[i]) <= k["abs_tol"]


def test_routing_slot_order(oracle):
    k = KATS["routing_slot_order"]
    ids, _ = oracle.routing_top_k(k["scores"], k["k"])
    assert ids.tolist() == k["expected_ids"]
    ids, _ = oracle.routing_softmax_top_k(k["scores"], k["k"])
    assert ids.tolist() == k["expected_ids"]


def test_routing_huge_negative(oracle):
    k = KATS["routing_huge_negative"]
    ids, w = oracle.routing_softmax_top_k(k["scores"], k["k"])
    assert ids.tolist() == k["expected_ids"]
    assert np.all(np.isfinite(w))
    assert abs(float(w.sum()) - 1.0) < k["sum_tol"]


def test_routing_sorted_set(oracle):
    k = KATS["routing_sorted_top_k_set"]
    ids, vals = oracle.routing_top_k(k["scores"], k["k"])
    order = sorted(range(len(ids)), key=lambda i: (-vals[i], ids[i]))
    assert [int(ids[i]) for i in order] == k["expected_sorted_ids"]


def test_routing_weights_softmax_then_topk(oracle):
    k = KATS["routing_weights_softmax_then_topk"]
    ids, probs = oracle.routing_softmax_top_k(k["scores"], k["k"])
    w = oracle.renormalize_routes(probs, 1.0)
    sel = f32([k["scores"][i] for i in ids])
    pb = oracle.softmax_in_place(sel)  # pb's weights: softmax over the selected scores
    assert np.max(np.abs(w - pb)) <= k["abs_tol"]


def test_routing_cmd3_weights(oracle):
    k = KATS["routing_cmd3_weights"]
    ids, probs = oracle.routing_softmax_top_k(k["scores"], k["k"])
    assert ids.tolist() == k["expected_ids"]
    w = oracle.renormalize_routes(probs, 1.0)
    assert np.max(np.abs(w - f32(k["expected_weights"]))) <= k["abs_tol"]


def test_renormalize_routes(oracle):
    k = KATS["renormalize_routes"]
    w = oracle.renormalize_routes(k["scores"], k["routed_expert_scale"])
    assert np.max(np.abs(w - f32(k["expected"]))) < k["abs_tol"]
    from oracle.pb_oracle import OracleError

    with pytest.raises(OracleError):
        oracle.renormalize_routes([0.0, 0.0], 1.0)  # non-positive sum
    with pytest.raises(OracleError):
        oracle.renormalize_routes([0.5, -0.1], 1.0)  # negative probability
    with pytest.raises(OracleError):
        oracle.renormalize_routes([0.5], 0.0)  # scale must be positive


def test_sigmoid_noaux(oracle):
    k = KATS["sigmoid_noaux_routing"]
    ids, w = oracle.routing_sigmoid_noaux_top_k(k["logits"], k["bias"], k["k"])
    order = np.argsort(ids)
    assert ids[order].tolist() == k["expected_sorted_ids"]
    assert np.max(np.abs(w[order] - f32(k["expected_sorted_weights"]))) < k["abs_tol"]


def test_cmd3_identity_combine(oracle):
    k = KATS["cmd3_identity_combine"]
    slot = np.zeros(k["slot_bytes"], np.uint8)
    offs = k["component_offsets"]
    one = np.uint16(k["one_bf16"]).tobytes()
    for wi, si in ((0, 1), (3, 4), (6, 7)):
        w_off, s_off = offs[wi], offs[si]
        slot[w_off:w_off + 2] = k["identity_weight_bytes"]
        slot[s_off:s_off + 2] = np.frombuffer(one, np.uint8)
        slot[s_off + 2:s_off + 4] = np.frombuffer(one, np.uint8)
    H, I, G = k["hidden"], k["intermediate"], k["group_size"]
    ids, probs = oracle.routing_softmax_top_k(k["router_scores"], k["k"])
    w = oracle.renormalize_routes(probs, 1.0)
    y = np.stack([oracle.expert_swiglu(slot, np.asarray(offs, np.uint64), H, I, G, k["normed"]) for _ in ids])
    hidden = oracle.combine(y[None], w[None], residual=f32(k["residual"])[None], shared=f32(k["shared_output"])[None],
                            shared_weight=f32([1.0]))
    assert np.max(np.abs(hidden[0] - f32(k["expected_hidden"]))) <= k["abs_tol"]
    nxt = oracle.rms_norm(hidden[0], k["next_norm_weights"])
    assert np.max(np.abs(nxt - f32(k["expected_next_normed"]))) <= k["abs_tol"]


def test_layer_major_group_plan(oracle):
    k = KATS["layer_major_group_plan"]
    src, idx, groups = oracle.layer_major_group_plan(k["route_slots"], k["unique"], k["active"])
    assert src.tolist() == k["expected_source_rows"]
    assert idx.tolist() == k["expected_output_indices"]
    assert groups.tolist() == k["expected_groups"]
    from oracle.pb_oracle import OracleError

    for slots, unique, active in k["errors"]:
        with pytest.raises(OracleError):
            oracle.layer_major_group_plan(slots, unique, active)


def _mla_q4_projection(rows, cols, nibble):
    packed = np.zeros((rows, (cols + 1) // 2), np.uint8)
    for r in range(rows):
        v = nibble(r) & 0x0F
        packed[r, :] = v | (v << 4)
    scales = np.full(rows, 0x3F80, np.uint16)
    biases = np.zeros(rows, np.uint16)
    return packed.reshape(-1), scales, biases, cols


def test_mla_closed_form(oracle):
    k = KATS["mla_closed_form"]
    H, L, N, R, V, S = k["heads"], k["latent"], k["nope"], k["rope"], k["v"], k["sequence"]
    eq = _mla_q4_projection(H * L, N, lambda r: r % 3 + 1)
    uo = _mla_q4_projection(H * V, L, lambda r: r % 5 + 1)
    qn = np.concatenate([np.full(N, v, np.float32) for v in k["query_nope_per_head"]])
    qr = f32(k["query_rope"])
    query = np.concatenate([np.concatenate([qn[h * N:(h + 1) * N], qr[h * R:(h + 1) * R]]) for h in range(H)])
    lat = np.array([[(d + 1) / L if p == 0 else (L - d) / L for d in range(L)] for p in range(S)], np.float32)
    rot = f32(k["record_rotary"])
    out = oracle.mla_absorbed_attention_q4(query, lat, rot, eq, uo, H, N, R, L, V)
    scale = np.float32(1.0) / np.sqrt(np.float32(N + R))
    expected = []
    for h in range(H):
        qsum = float(qn[h * N:(h + 1) * N].sum())
        absorbed = [((h * L + d) % 3 + 1) * qsum for d in range(L)]
        scores = []
        for p in range(S):
            ls = sum(a * b for a, b in zip(absorbed, lat[p]))
            rs = sum(a * b for a, b in zip(qr[h * R:(h + 1) * R], rot[p * R:(p + 1) * R]))
            scores.append((ls + rs) * scale)
        m = max(scores)
        den = sum(math.exp(s - m) for s in scores)
        probs = [math.exp(s - m) / den for s in scores]
        ctx = [sum(probs[p] * lat[p][d] for p in range(S)) for d in range(L)]
        cs = sum(ctx)
        expected.extend(((h * V + r) % 5 + 1) * cs for r in range(V))
    assert np.max(np.abs(out - f32(expected))) < k["abs_tol"]


def test_mla_bf16_matches_q4_form_on_identity_weights(oracle):
    """The dense-bf16 FusedKvB arm and the Q4 multilinear arm agree when their
    weights describe the same matrices (here: the closed-form case's weights)."""
    k = KATS["mla_closed_form"]
    H, L, N, R, V, S = k["heads"], k["latent"], k["nope"], k["rope"], k["v"], k["sequence"]
    rng = np.random.default_rng(7)
    query = rng.standard_normal(H * (N + R)).astype(np.float32)
    lat = rng.standard_normal((S, L)).astype(np.float32)
    rot = rng.standard_normal(S * R).astype(np.float32)
    # embed_q rows (h*L + c) x nope cols == w_uk[h, d, c]; unembed rows (h*V+d) x L == w_uv[h, d, :]
    eq = _mla_q4_projection(H * L, N, lambda r: r % 3 + 1)
    uo = _mla_q4_projection(H * V, L, lambda r: r % 5 + 1)
    w_uk = np.zeros((H, N, L), np.float32)
    for h in range(H):
        for c in range(L):
            w_uk[h, :, c] = ((h * L + c) % 3 + 1)
    w_uv = np.zeros((H, V, L), np.float32)
    for h in range(H):
        for d in range(V):
            w_uv[h, d, :] = ((h * V + d) % 5 + 1)
    a = oracle.mla_absorbed_attention_q4(query, lat, rot, eq, uo, H, N, R, L, V)
    b = oracle.mla_absorbed_attention(query, lat, rot, _bf(w_uk), _bf(w_uv), H, N, R, L, V)
    assert np.max(np.abs(a - b) / np.maximum(np.abs(a), 1.0)) < 1e-4


def test_rope(oracle):
    k = KATS["rope_interleaved_to_split_half"]
    out = oracle.rope_interleaved_to_split_half(k["values"], k["position"], k["rotary_dim"], k["theta"])
    assert out.tolist() == k["expected"]
    from oracle.pb_oracle import OracleError

    with pytest.raises(OracleError):
        oracle.rope_interleaved_to_split_half([1.0, 2.0, 3.0], 0, 3, 1e4)


def test_bf16_rne(oracle):
    from oracle.pb_oracle import f32_to_bf16_bits

    for value, bits in KATS["bf16_round_nearest_even"]["cases"]:
        assert oracle.lib().oracle_f32_to_bf16(value) == bits
        assert int(f32_to_bf16_bits([value])[0]) == bits


def test_fixed_q4_layout_matches_slot_size(oracle):
    offs, nbytes = oracle.fixed_q4_layout(2048, 512, 64)
    assert nbytes == 1_769_472
    assert offs.tolist() == [0, 524288, 557056, 589824, 1114112, 1146880, 1179648, 1703936, 1736704]
    from oracle.pb_oracle import OracleError

    with pytest.raises(OracleError):
        oracle.fixed_q4_layout(2048, 500, 64)
