"""ctypes binding of the CPU oracle (oracle/pb_oracle.cpp).

Test infrastructure only: tests/, ``__graft_entry__.smoke()`` and the CPU
baseline legs of bench.py load this module, as the checker or as the timed CPU
baseline. The product library (pb_b200, libpbmoe.so) never imports it.

Every wrapper takes and returns numpy arrays; shapes follow the C signatures in
pb_oracle.cpp, which cite the reference function each one restates.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libpb_oracle.so")

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def _declare(L):
    L.oracle_f32_to_bf16.restype = C.c_uint16
    L.oracle_f32_to_bf16.argtypes = [C.c_float]
    L.oracle_bf16_to_f32.restype = C.c_float
    L.oracle_bf16_to_f32.argtypes = [C.c_uint16]
    L.oracle_q4_fma_matvec.argtypes = [_u8p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _f32p]
    L.oracle_q4_fma_matvec_bf16.argtypes = [_u8p, _f32p, _u16p, _u16p, _sz, _sz, _sz, _f32p, C.c_int]
    L.oracle_reference_q4_matvec.argtypes = [_u8p, _f32p, _u16p, _u16p, _sz, _sz, _sz, _f32p]
    L.oracle_q4_dequantize_rows.argtypes = [_u8p, _f32p, _f32p, _sz, _sz, _sz, _f32p]
    L.oracle_q4_unpack_nibbles.argtypes = [_u8p, _sz, _sz, _u8p]
    L.oracle_softmax_in_place.restype = None
    L.oracle_softmax_in_place.argtypes = [_f32p, _sz]
    L.oracle_routing_top_k.restype = _sz
    L.oracle_routing_top_k.argtypes = [_f32p, _sz, _sz, _u32p, _f32p]
    L.oracle_routing_softmax_top_k.restype = _sz
    L.oracle_routing_softmax_top_k.argtypes = [_f32p, _sz, _sz, _u32p, _f32p]
    L.oracle_routing_sigmoid_noaux_top_k.restype = _sz
    L.oracle_routing_sigmoid_noaux_top_k.argtypes = [_f32p, _f32p, _sz, _sz, _u32p, _f32p]
    L.oracle_renormalize_routes.argtypes = [_f32p, _sz, C.c_int, C.c_float, _f32p]
    L.oracle_layer_major_group_plan.argtypes = [_u32p, _sz, _sz, _sz, _u32p, _u32p, _u32p]
    L.oracle_rms_norm.restype = None
    L.oracle_rms_norm.argtypes = [_f32p, _sz, C.c_void_p, C.c_float]
    L.oracle_rope_interleaved_to_split_half.argtypes = [_f32p, _sz, _sz, _sz, C.c_double]
    L.oracle_rope_tables.argtypes = [_sz, _sz, C.c_double, _f32p, _f32p]
    L.oracle_dense_bf16_matvec.argtypes = [_u16p, _f32p, _sz, _sz, _f32p]
    L.oracle_fixed_q4_layout.argtypes = [_sz, _sz, _sz, _u64p, _u64p]
    L.oracle_expert_swiglu.argtypes = [_u8p, _u64p, _sz, _sz, _sz, _f32p, _f32p]
    L.oracle_combine.argtypes = [C.c_void_p, _f32p, _f32p, C.c_void_p, C.c_void_p, _sz, _sz, _sz, _f32p]
    L.oracle_moe_layer.argtypes = [
        _f32p, C.c_void_p, _sz, _sz, _sz, _sz, _sz, _sz, C.c_float, _u16p, C.c_void_p,
        _u8p, _u64p, _sz, C.c_void_p, _f32p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
    ]
    L.oracle_mla_absorbed_attention.argtypes = [
        _f32p, _f32p, _f32p, _sz, _u16p, _u16p, _sz, _sz, _sz, _sz, _sz, _f32p,
    ]
    L.oracle_mla_absorbed_attention_q4.argtypes = [
        _f32p, _f32p, _f32p, _sz, _u8p, _u16p, _u16p, _sz, _u8p, _u16p, _u16p, _sz,
        _sz, _sz, _sz, _sz, _sz, _f32p,
    ]
    L.oracle_q4_gemm.argtypes = [_f32p, _sz, _u8p, _u16p, _u16p, _sz, _sz, _sz, _f32p, C.c_int]
    L.oracle_mxfp4_matvec.argtypes = [_u8p, _f32p, _u8p, _sz, _sz, _sz, _f32p]
    L.oracle_topk_vocab.restype = _sz
    L.oracle_topk_vocab.argtypes = [_f32p, _sz, _sz, C.c_void_p, _u32p, _f32p]


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class OracleError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise OracleError(f"{what} rejected its arguments (status {rc})")


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(a) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (experts/slots.rs:1165-1169), vectorised."""
    a = _c(a, np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    return (((bits + 0x7FFF + lsb) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = _c(b, np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- Q4
def q4_fma_matvec(packed, x, scales, biases, rows, cols, group):
    out = np.zeros(rows, np.float32)
    _check(lib().oracle_q4_fma_matvec(_c(packed, np.uint8), _c(x, np.float32), _c(scales, np.float32),
                                      _c(biases, np.float32), rows, cols, group, out), "q4_fma_matvec")
    return out


def q4_fma_matvec_bf16(packed, x, scale_bits, bias_bits, rows, cols, group, threads=1):
    out = np.zeros(rows, np.float32)
    _check(lib().oracle_q4_fma_matvec_bf16(_c(packed, np.uint8), _c(x, np.float32), _c(scale_bits, np.uint16),
                                           _c(bias_bits, np.uint16), rows, cols, group, out, threads),
           "q4_fma_matvec_bf16")
    return out


def reference_q4_matvec(packed, x, scale_bits, bias_bits, rows, cols, group):
    out = np.zeros(rows, np.float32)
    _check(lib().oracle_reference_q4_matvec(_c(packed, np.uint8), _c(x, np.float32), _c(scale_bits, np.uint16),
                                            _c(bias_bits, np.uint16), rows, cols, group, out),
           "reference_q4_matvec")
    return out


def q4_dequantize_rows(packed, scales, biases, rows, cols, group):
    out = np.zeros(rows * cols, np.float32)
    _check(lib().oracle_q4_dequantize_rows(_c(packed, np.uint8), _c(scales, np.float32), _c(biases, np.float32),
                                           rows, cols, group, out), "q4_dequantize_rows")
    return out


def q4_unpack_nibbles(packed, rows, cols):
    out = np.zeros(rows * cols, np.uint8)
    lib().oracle_q4_unpack_nibbles(_c(packed, np.uint8), rows, cols, out)
    return out.reshape(rows, cols)


def q4_gemm(x, packed, scale_bits, bias_bits, n, k, group, threads=1):
    x = _c(x, np.float32)
    m = x.shape[0]
    out = np.zeros((m, n), np.float32)
    _check(lib().oracle_q4_gemm(x, m, _c(packed, np.uint8), _c(scale_bits, np.uint16), _c(bias_bits, np.uint16),
                                n, k, group, out, threads), "q4_gemm")
    return out


# ---------------------------------------------------------------- routing
def softmax_in_place(v):
    v = _c(v, np.float32).copy()
    lib().oracle_softmax_in_place(v, v.size)
    return v


def routing_top_k(scores, k):
    s = _c(scores, np.float32)
    ids = np.zeros(max(k, 1), np.uint32)
    vals = np.zeros(max(k, 1), np.float32)
    n = lib().oracle_routing_top_k(s, s.size, k, ids, vals)
    return ids[:n], vals[:n]


def routing_softmax_top_k(scores, k):
    s = _c(scores, np.float32)
    ids = np.zeros(max(k, 1), np.uint32)
    w = np.zeros(max(k, 1), np.float32)
    n = lib().oracle_routing_softmax_top_k(s, s.size, k, ids, w)
    return ids[:n], w[:n]


def routing_sigmoid_noaux_top_k(logits, bias, k):
    s = _c(logits, np.float32)
    ids = np.zeros(max(k, 1), np.uint32)
    w = np.zeros(max(k, 1), np.float32)
    n = lib().oracle_routing_sigmoid_noaux_top_k(s, _c(bias, np.float32), s.size, k, ids, w)
    return ids[:n], w[:n]


def renormalize_routes(scores, routed_scale=1.0, policy=0):
    s = _c(scores, np.float32)
    out = np.zeros(s.size, np.float32)
    _check(lib().oracle_renormalize_routes(s, s.size, policy, routed_scale, out), "renormalize_routes")
    return out


def layer_major_group_plan(route_slots, unique, active):
    rs = _c(route_slots, np.uint32)
    n = rs.size
    src = np.zeros(max(n, 1), np.uint32)
    idx = np.zeros(max(n, 1), np.uint32)
    groups = np.zeros(max(2 * unique, 2), np.uint32)
    _check(lib().oracle_layer_major_group_plan(rs if n else np.zeros(1, np.uint32), n, unique, active, src, idx,
                                               groups), "layer_major_group_plan")
    return src[:n], idx[:n], groups[: 2 * unique].reshape(unique, 2)


# ---------------------------------------------------------------- norms / rope
def rms_norm(values, weight=None, eps=1e-6):
    v = _c(values, np.float32).copy()
    w = None if weight is None else _c(weight, np.float32)
    lib().oracle_rms_norm(v, v.size, _ptr(w), eps)
    return v


def rope_interleaved_to_split_half(values, position, rotary_dim, theta):
    v = _c(values, np.float32).copy()
    _check(lib().oracle_rope_interleaved_to_split_half(v, v.size, position, rotary_dim, theta), "rope")
    return v


def rope_tables(position, rotary_dim, theta):
    c = np.zeros(rotary_dim // 2, np.float32)
    s = np.zeros(rotary_dim // 2, np.float32)
    _check(lib().oracle_rope_tables(position, rotary_dim, theta, c, s), "rope_tables")
    return c, s


# ---------------------------------------------------------------- experts / MoE
def dense_bf16_matvec(weight_bits, x, rows, cols):
    out = np.zeros(rows, np.float32)
    lib().oracle_dense_bf16_matvec(_c(weight_bits, np.uint16), _c(x, np.float32), rows, cols, out)
    return out


def fixed_q4_layout(hidden, inter, group):
    offs = np.zeros(9, np.uint64)
    nbytes = np.zeros(1, np.uint64)
    _check(lib().oracle_fixed_q4_layout(hidden, inter, group, offs, nbytes), "fixed_q4_layout")
    return offs, int(nbytes[0])


def expert_swiglu(slot, offsets, hidden, inter, group, x):
    out = np.zeros(hidden, np.float32)
    _check(lib().oracle_expert_swiglu(_c(slot, np.uint8), _c(offsets, np.uint64), hidden, inter, group,
                                      _c(x, np.float32), out), "expert_swiglu")
    return out


def combine(expert_out, weights, residual=None, shared=None, shared_weight=None):
    eo = _c(expert_out, np.float32)
    tokens, top_k, hidden = eo.shape
    w = _c(weights, np.float32)
    r = None if residual is None else _c(residual, np.float32)
    sh = None if shared is None else _c(shared, np.float32)
    sw = None if shared_weight is None else _c(shared_weight, np.float32)
    out = np.zeros((tokens, hidden), np.float32)
    lib().oracle_combine(_ptr(r), eo, w, _ptr(sh), _ptr(sw), tokens, top_k, hidden, out)
    return out


def moe_layer(x, router_bits, expert_table, offsets, slot_stride, num_experts, top_k, inter, group,
              shared_slot=None, shared_gate_bits=None, residual=None, routed_scale=1.0, threads=1,
              correction_bias=None, mxfp4=False):
    """Full MoE FFN decode layer per token. Returns (out, ids, weights, logits).
    correction_bias (f32 [E]) routes by sigmoid/noaux; mxfp4 reads MXFP4 expert slots."""
    cb = None if correction_bias is None else _c(correction_bias, np.float32)
    x = _c(x, np.float32)
    tokens, hidden = x.shape
    out = np.zeros((tokens, hidden), np.float32)
    ids = np.zeros((tokens, top_k), np.uint32)
    w = np.zeros((tokens, top_k), np.float32)
    logits = np.zeros((tokens, num_experts), np.float32)
    r = None if residual is None else _c(residual, np.float32)
    sg = None if shared_gate_bits is None else _c(shared_gate_bits, np.uint16)
    ss = None if shared_slot is None else _c(shared_slot, np.uint8)
    _check(lib().oracle_moe_layer(x, _ptr(r), tokens, hidden, num_experts, top_k, inter, group, routed_scale,
                                  _c(router_bits, np.uint16), _ptr(sg), _c(expert_table, np.uint8),
                                  _c(offsets, np.uint64), slot_stride, _ptr(ss), out, _ptr(ids), _ptr(w),
                                  _ptr(logits), threads, _ptr(cb), 1 if mxfp4 else 0), "moe_layer")
    return out, ids, w, logits


# ---------------------------------------------------------------- MLA
def mla_absorbed_attention(query, latents, rotary, w_uk_bits, w_uv_bits, heads, nope, rope, latent, v_dim):
    q = _c(query, np.float32)
    lat = _c(latents, np.float32)
    rot = _c(rotary, np.float32)
    seq = lat.size // latent
    out = np.zeros(heads * v_dim, np.float32)
    _check(lib().oracle_mla_absorbed_attention(q, lat, rot, seq, _c(w_uk_bits, np.uint16), _c(w_uv_bits, np.uint16),
                                               heads, nope, rope, latent, v_dim, out), "mla_absorbed_attention")
    return out


def mla_absorbed_attention_q4(query, latents, rotary, eq, uo, heads, nope, rope, latent, v_dim):
    """eq/uo: (packed u8, scale bits u16, bias bits u16, group) for embed_q / unembed_out."""
    q = _c(query, np.float32)
    lat = _c(latents, np.float32)
    rot = _c(rotary, np.float32)
    seq = lat.size // latent
    out = np.zeros(heads * v_dim, np.float32)
    _check(lib().oracle_mla_absorbed_attention_q4(
        q, lat, rot, seq, _c(eq[0], np.uint8), _c(eq[1], np.uint16), _c(eq[2], np.uint16), eq[3],
        _c(uo[0], np.uint8), _c(uo[1], np.uint16), _c(uo[2], np.uint16), uo[3], heads, nope, rope, latent,
        v_dim, out), "mla_absorbed_attention_q4")
    return out


# ---------------------------------------------------------------- vocab head
def topk_vocab(logits, top_k, allowed=None):
    """topk_vocab on one token's logits: (ids, values) of min(top_k, vocab) passes."""
    lg = _c(logits, np.float32)
    n = min(int(top_k), lg.size)
    ids = np.zeros(max(n, 1), np.uint32)
    vals = np.zeros(max(n, 1), np.float32)
    al = None if allowed is None else _c(allowed, np.uint32)
    lib().oracle_topk_vocab(lg, lg.size, int(top_k), None if al is None else al.ctypes.data, ids, vals)
    return ids[:n], vals[:n]


def head_topk(weight_bits, x, top_k, allowed=None):
    """LM-head candidates per token: dense bf16 projection (fma in column
    order) then topk_vocab. Returns (ids [T, n], values [T, n], logits [T, V])."""
    w = _c(weight_bits, np.uint16)
    V, H = w.shape
    xs = np.atleast_2d(np.asarray(x, np.float32))
    logits = np.stack([dense_bf16_matvec(w, row, V, H) for row in xs])
    res = [topk_vocab(row, top_k, allowed) for row in logits]
    return np.stack([r[0] for r in res]), np.stack([r[1] for r in res]), logits


# ---------------------------------------------------------------- MXFP4
def mxfp4_matvec(packed, x, scales, rows, cols, group=32):
    """y = W x for MXFP4 W (E2M1 nibbles, E8M0 scale bytes per group)."""
    out = np.zeros(rows, np.float32)
    _check(lib().oracle_mxfp4_matvec(_c(packed, np.uint8), _c(x, np.float32), _c(scales, np.uint8), rows, cols,
                                     group, out), "mxfp4_matvec")
    return out
