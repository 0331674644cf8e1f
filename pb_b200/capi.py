"""ctypes binding of include/pbmoe_cuda.h (libpbmoe.so).

This is plumbing for tests and the benchmark: it passes device pointers (from
torch tensors) straight to the C ABI, so every call here exercises exactly the
entry point a Rust host would bind. There is no fallback: if the library is
missing or the device is absent, loading raises.
"""

from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libpbmoe.so")

PBMOE_OK = 0
PBMOE_ERR_INVALID_ARGUMENT = -1
PBMOE_ERR_UNSUPPORTED = -2
PBMOE_ERR_CUDA = -3
PBMOE_ERR_TIMEOUT = -4
PBMOE_ERR_PEER = -5
PBMOE_ERR_NO_WORKSPACE = -6
PBMOE_ERR_DEVICE_STATUS = -7

PBMOE_DEV_ERR_ROUTE_WEIGHTS = 0x1
PBMOE_DEV_ERR_EXPERT_ID = 0x2
PBMOE_DEV_ERR_PEER_TIMEOUT = 0x4
PBMOE_DEV_ERR_PIPE_TIMEOUT = 0x8
PBMOE_DEV_ERR_F16_RANGE = 0x10
PBMOE_DEV_ERR_POSITION = 0x20
PBMOE_DEV_ERR_MXFP4_SCALE = 0x40

PBMOE_F32 = 0
PBMOE_BF16 = 1
PBMOE_F16 = 2

ROUTE_RENORMALIZE_SELECTED = 0
ROUTE_DEEPSEEK_RENORMALIZE_WITH_FLOOR = 1

# Every symbol the header declares (checked by tests/test_capi_symbols.py).
EXPORTED = [
    "pbmoe_init", "pbmoe_destroy", "pbmoe_last_error", "pbmoe_abi_version", "pbmoe_reserve",
    "pbmoe_moe_workspace_bytes", "pbmoe_device_status", "pbmoe_fixed_q4_layout", "pbmoe_q4_matvec",
    "pbmoe_route_topk", "pbmoe_moe_layer", "pbmoe_moe_layer_static", "pbmoe_mla_reserve", "pbmoe_mla_decode",
    "pbmoe_prefill_reserve", "pbmoe_q4_gemm", "pbmoe_prefill_group_plan", "pbmoe_q4_gemm_grouped",
    "pbmoe_ep_expert_range", "pbmoe_ep_reserve", "pbmoe_ep_ipc_handle", "pbmoe_ep_open_peers", "pbmoe_ep_set_peers",
    "pbmoe_ep_buffer", "pbmoe_ep_moe_layer", "pbmoe_head_reserve", "pbmoe_head_topk", "pbmoe_head_merge",
    "pbmoe_rms_norm", "pbmoe_rope_reserve", "pbmoe_mla_rope_append", "pbmoe_mla_append_decode", "pbmoe_expert_layer_read",
    "pbmoe_expert_layer_load", "pbmoe_mxfp4_matvec", "pbmoe_moe_layer_host", "pbmoe_sync",
    "pbmoe_fixed_mxfp4_layout", "pbmoe_q4_matvec_fused", "pbmoe_q4_matvec_batch", "pbmoe_route_sigmoid_noaux",
]

EP_HANDLE_BYTES = 64


class Q4Tensor(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("rows", C.c_uint32), ("cols", C.c_uint32), ("group_size", C.c_uint32)]


class ExpertLayout(C.Structure):
    _fields_ = [("component_offsets", C.c_uint64 * 9), ("expert_bytes", C.c_uint64),
                ("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("group_size", C.c_uint32),
                ("encoding", C.c_uint32)]


PBMOE_EXPERT_AFFINE_Q4 = 0
PBMOE_EXPERT_MXFP4 = 1


class MoeConfig(C.Structure):
    _fields_ = [("layout", ExpertLayout), ("num_experts", C.c_uint32), ("top_k", C.c_uint32),
                ("normalization", C.c_uint32), ("routed_scaling_factor", C.c_float), ("norm_epsilon", C.c_float)]


class MoeWeights(C.Structure):
    _fields_ = [("router_weight", C.c_void_p), ("experts", C.c_void_p), ("shared_expert", C.c_void_p),
                ("shared_expert_gate", C.c_void_p), ("input_norm_weight", C.c_void_p),
                ("router_correction_bias", C.c_void_p)]


class MoeDebug(C.Structure):
    _fields_ = [("router_logits", C.c_void_p), ("route_ids", C.c_void_p), ("route_weights", C.c_void_p),
                ("shared_logit", C.c_void_p), ("phase_events", C.c_void_p), ("normed_input", C.c_void_p)]


class MlaConfig(C.Structure):
    _fields_ = [("heads", C.c_uint32), ("nope_dim", C.c_uint32), ("rope_dim", C.c_uint32),
                ("latent_dim", C.c_uint32), ("v_dim", C.c_uint32), ("softmax_scale", C.c_float)]


class MlaArgs(C.Structure):
    _fields_ = [("batch", C.c_uint32), ("seq_lens", C.c_void_p), ("query", C.c_void_p), ("query_dtype", C.c_int),
                ("c_kv", C.c_void_p), ("k_rope", C.c_void_p), ("w_uk", C.c_void_p), ("w_uv", C.c_void_p),
                ("out", C.c_void_p), ("out_dtype", C.c_int)]


class Q4ExpertMatrix(C.Structure):
    _fields_ = [("experts", C.c_void_p), ("expert_bytes", C.c_uint64), ("packed_offset", C.c_uint64),
                ("scales_offset", C.c_uint64), ("biases_offset", C.c_uint64), ("num_experts", C.c_uint32),
                ("rows", C.c_uint32), ("cols", C.c_uint32), ("group_size", C.c_uint32)]


class EpShard(C.Structure):
    _fields_ = [("expert_begin", C.c_uint32), ("expert_count", C.c_uint32), ("timeout_us", C.c_uint32)]


class Head(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("vocab", C.c_uint32), ("hidden", C.c_uint32), ("id_base", C.c_uint32)]


class Mxfp4Tensor(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("rows", C.c_uint32), ("cols", C.c_uint32),
                ("group_size", C.c_uint32)]


class NormArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("x_dtype", C.c_int), ("residual", C.c_void_p), ("sum_out", C.c_void_p),
                ("sum_dtype", C.c_int), ("weight", C.c_void_p), ("epsilon", C.c_float), ("out", C.c_void_p),
                ("out_dtype", C.c_int), ("rows", C.c_uint32), ("width", C.c_uint32), ("x_stride", C.c_uint32),
                ("residual_stride", C.c_uint32), ("sum_stride", C.c_uint32), ("out_stride", C.c_uint32)]


class Q4FusedArgs(C.Structure):
    _fields_ = [("w", C.POINTER(Q4Tensor) * 2), ("y", C.c_void_p * 2), ("x", C.c_void_p), ("x_dtype", C.c_int),
                ("y_dtype", C.c_int), ("batch", C.c_uint32), ("input_norm_weight", C.c_void_p),
                ("epsilon", C.c_float), ("residual", C.c_void_p)]


class PbmoeError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"pbmoe status {code}: {message}")
        self.code = code


_lib = None


def load():
    """Load libpbmoe.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m pb_b200.build`")
        L = C.CDLL(LIB_PATH)
        vp, u32, i32 = C.c_void_p, C.c_uint32, C.c_int
        L.pbmoe_init.argtypes = [i32, C.POINTER(vp)]
        L.pbmoe_destroy.argtypes = [vp]
        L.pbmoe_last_error.restype = C.c_char_p
        L.pbmoe_last_error.argtypes = [vp]
        L.pbmoe_abi_version.restype = i32
        L.pbmoe_reserve.argtypes = [vp, u32, C.POINTER(MoeConfig)]
        L.pbmoe_moe_workspace_bytes.restype = C.c_size_t
        L.pbmoe_moe_workspace_bytes.argtypes = [u32, C.POINTER(MoeConfig)]
        L.pbmoe_device_status.argtypes = [vp, vp, C.POINTER(u32), i32]
        L.pbmoe_fixed_q4_layout.argtypes = [u32, u32, u32, C.POINTER(ExpertLayout)]
        L.pbmoe_fixed_mxfp4_layout.argtypes = [u32, u32, u32, C.POINTER(ExpertLayout)]
        L.pbmoe_q4_matvec.argtypes = [vp, C.POINTER(Q4Tensor), vp, i32, vp, i32, u32, vp]
        L.pbmoe_route_topk.argtypes = [vp, vp, u32, u32, u32, u32, C.c_float, vp, vp, vp]
        L.pbmoe_moe_layer.argtypes = [vp, C.POINTER(MoeConfig), C.POINTER(MoeWeights), vp, i32, vp, vp, i32, u32,
                                      vp, vp, C.POINTER(MoeDebug), vp]
        L.pbmoe_mla_reserve.argtypes = [vp, C.POINTER(MlaConfig), u32]
        L.pbmoe_mla_decode.argtypes = [vp, C.POINTER(MlaConfig), C.POINTER(MlaArgs), vp]
        L.pbmoe_moe_layer_static.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), vp, i32, vp, vp, i32,
                                             u32, vp, vp, vp, C.c_char_p, C.c_size_t, vp]
        L.pbmoe_prefill_reserve.argtypes = [vp, u32, u32]
        L.pbmoe_q4_gemm.argtypes = [vp, C.POINTER(Q4Tensor), vp, i32, vp, i32, u32, vp]
        L.pbmoe_prefill_group_plan.argtypes = [vp, vp, u32, u32, u32, vp, vp, vp, vp, vp, vp, vp]
        L.pbmoe_q4_gemm_grouped.argtypes = [vp, C.POINTER(Q4ExpertMatrix), vp, vp, vp, vp, u32, u32, vp, i32, u32,
                                            vp, i32, vp]
        L.pbmoe_ep_expert_range.argtypes = [u32, u32, u32, C.POINTER(u32), C.POINTER(u32)]
        L.pbmoe_ep_reserve.argtypes = [vp, u32, u32, u32, u32]
        L.pbmoe_ep_ipc_handle.argtypes = [vp, vp]
        L.pbmoe_ep_open_peers.argtypes = [vp, vp]
        L.pbmoe_ep_set_peers.argtypes = [vp, vp]
        L.pbmoe_ep_buffer.restype = vp
        L.pbmoe_ep_buffer.argtypes = [vp]
        L.pbmoe_ep_moe_layer.argtypes = [vp, C.POINTER(MoeConfig), C.POINTER(MoeWeights), C.POINTER(EpShard), vp, i32,
                                         vp, vp, i32, u32, vp, vp, C.POINTER(MoeDebug), vp]
        L.pbmoe_head_reserve.argtypes = [vp, u32, u32, u32]
        L.pbmoe_head_topk.argtypes = [vp, C.POINTER(Head), vp, i32, u32, u32, vp, vp, vp, vp, vp, vp]
        L.pbmoe_head_merge.argtypes = [vp, vp, vp, vp, u32, u32, u32, vp, vp, vp]
        L.pbmoe_rms_norm.argtypes = [vp, C.POINTER(NormArgs), vp]
        L.pbmoe_rope_reserve.argtypes = [vp, u32, u32, C.c_double]
        L.pbmoe_mla_rope_append.argtypes = [vp, C.POINTER(MlaConfig), u32, vp, vp, vp, C.c_float, vp, vp, vp, u32,
                                             vp]
        L.pbmoe_mla_append_decode.argtypes = [vp, C.POINTER(MlaConfig), C.POINTER(MlaArgs), vp, vp, C.c_float, vp,
                                               vp, vp, u32, vp]
        L.pbmoe_q4_matvec_fused.argtypes = [vp, C.POINTER(Q4FusedArgs), vp]
        L.pbmoe_q4_matvec_batch.argtypes = [vp, C.POINTER(Q4Tensor), u32, vp, C.c_int, C.POINTER(vp), C.c_int, u32,
                                            vp]
        L.pbmoe_route_sigmoid_noaux.argtypes = [vp, vp, vp, u32, u32, u32, u32, C.c_float, vp, vp, vp]
        L.pbmoe_sync.argtypes = [vp, vp, u32]
        L.pbmoe_moe_layer_host.argtypes = [vp, C.POINTER(MoeConfig), C.POINTER(MoeWeights), vp, i32, vp, vp, i32,
                                           u32, vp]
        L.pbmoe_mxfp4_matvec.argtypes = [vp, C.POINTER(Mxfp4Tensor), vp, i32, vp, i32, u32, vp]
        L.pbmoe_expert_layer_read.argtypes = [C.c_char_p, u32, C.POINTER(ExpertLayout), u32, u32, vp, C.c_size_t,
                                              C.c_char_p, C.c_size_t]
        L.pbmoe_expert_layer_load.argtypes = [vp, C.c_char_p, u32, C.POINTER(ExpertLayout), u32, u32, vp,
                                              C.c_size_t, vp]
        _lib = L
    return _lib


def fixed_mxfp4_layout(hidden, intermediate, group=32):
    """The fixed MXFP4 expert slot layout (nibbles + E8M0 per projection, no biases)."""
    lay = ExpertLayout()
    rc = load().pbmoe_fixed_mxfp4_layout(hidden, intermediate, group, C.byref(lay))
    if rc != PBMOE_OK:
        raise PbmoeError(rc, "invalid fixed-MXFP4 layout")
    return lay


def fixed_q4_layout(hidden, intermediate, group):
    lay = ExpertLayout()
    rc = load().pbmoe_fixed_q4_layout(hidden, intermediate, group, C.byref(lay))
    if rc != PBMOE_OK:
        raise PbmoeError(rc, "invalid fixed-Q4 layout")
    return lay


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _same_dtype(out, *others):
    """residual / next_normed travel in the output's dtype (the C-ABI cannot see it)."""
    for t in others:
        if t is not None and t.dtype != out.dtype:
            raise TypeError(f"expected {out.dtype} like the output, got {t.dtype}")


def _dtype_code(t):
    import torch

    if t.dtype == torch.float32:
        return PBMOE_F32
    if t.dtype == torch.bfloat16:
        return PBMOE_BF16
    if t.dtype == torch.float16:
        return PBMOE_F16
    raise TypeError(f"unsupported activation dtype {t.dtype}")


class Context:
    """One pbmoe_ctx on one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = load()
        self.device = device
        h = C.c_void_p()
        rc = self.lib.pbmoe_init(device, C.byref(h))
        if rc != PBMOE_OK:
            raise PbmoeError(rc, f"pbmoe_init({device}) failed")
        self.h = h

    def close(self):
        if self.h:
            self.lib.pbmoe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self) -> str:
        return self.lib.pbmoe_last_error(self.h).decode()

    def check(self, rc):
        if rc != PBMOE_OK:
            raise PbmoeError(rc, self.last_error())

    def stream_ptr(self, stream=None):
        import torch

        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return C.c_void_p(s.cuda_stream)

    # -------------------------------------------------------------- entry points
    def q4_matvec(self, packed, scales, biases, rows, cols, group, x, y, batch=1, stream=None):
        t = Q4Tensor(packed.data_ptr(), scales.data_ptr(), biases.data_ptr(), rows, cols, group)
        self.check(self.lib.pbmoe_q4_matvec(self.h, C.byref(t), _ptr(x), _dtype_code(x), _ptr(y), _dtype_code(y),
                                            batch, self.stream_ptr(stream)))

    def route_topk(self, logits, tokens, num_experts, top_k, ids, weights, normalization=0, scale=1.0, stream=None):
        self.check(self.lib.pbmoe_route_topk(self.h, _ptr(logits), tokens, num_experts, top_k, normalization, scale,
                                             _ptr(ids), _ptr(weights), self.stream_ptr(stream)))

    def route_sigmoid_noaux(self, logits, bias, tokens, num_experts, top_k, ids, weights, normalization=0,
                            scale=1.0, stream=None):
        self.check(self.lib.pbmoe_route_sigmoid_noaux(self.h, _ptr(logits), _ptr(bias), tokens, num_experts, top_k,
                                                      normalization, scale, _ptr(ids), _ptr(weights),
                                                      self.stream_ptr(stream)))

    def reserve(self, max_tokens, config: MoeConfig):
        self.check(self.lib.pbmoe_reserve(self.h, max_tokens, C.byref(config)))

    def moe_layer(self, config, weights: MoeWeights, x, out, tokens, residual=None, next_norm_weight=None,
                  next_normed=None, debug: MoeDebug | None = None, stream=None):
        _same_dtype(out, residual, next_normed)
        self.check(self.lib.pbmoe_moe_layer(
            self.h, C.byref(config), C.byref(weights), _ptr(x), _dtype_code(x), _ptr(residual), _ptr(out),
            _dtype_code(out), tokens, _ptr(next_norm_weight), _ptr(next_normed),
            C.byref(debug) if debug is not None else None, self.stream_ptr(stream)))

    def sync(self, stream=None, timeout_ms=10000):
        """Bounded wait for `stream`; PbmoeError (PBMOE_ERR_TIMEOUT) if it is still busy."""
        self.check(self.lib.pbmoe_sync(self.h, self.stream_ptr(stream), timeout_ms))

    def moe_layer_host(self, config, weights: MoeWeights, x, out, tokens, residual=None, stream=None):
        """The layer on host tensors (pinned for asynchronous copies): x [tokens, H] bf16/f32,
        out (and residual) [tokens, H] in the output dtype; ordered on `stream`."""
        _same_dtype(out, residual)
        self.check(self.lib.pbmoe_moe_layer_host(self.h, C.byref(config), C.byref(weights), _ptr(x), _dtype_code(x),
                                                 _ptr(residual), _ptr(out), _dtype_code(out), tokens,
                                                 self.stream_ptr(stream)))

    def mla_reserve(self, config: MlaConfig, max_batch: int):
        self.check(self.lib.pbmoe_mla_reserve(self.h, C.byref(config), max_batch))

    def mla_decode(self, config: MlaConfig, query, c_kv, k_rope, w_uk, w_uv, out, stream=None):
        """query [B, heads, nope+rope]; c_kv / k_rope: lists of B device tensors."""
        b = len(c_kv)
        lens = (C.c_uint32 * b)(*[int(t.shape[0]) for t in c_kv])
        ckv = (C.c_void_p * b)(*[t.data_ptr() for t in c_kv])
        kr = (C.c_void_p * b)(*[t.data_ptr() for t in k_rope])
        args = MlaArgs(b, C.cast(lens, C.c_void_p), query.data_ptr(), _dtype_code(query), C.cast(ckv, C.c_void_p),
                       C.cast(kr, C.c_void_p), w_uk.data_ptr(), w_uv.data_ptr(), out.data_ptr(), _dtype_code(out))
        self.check(self.lib.pbmoe_mla_decode(self.h, C.byref(config), C.byref(args), self.stream_ptr(stream)))

    def head_reserve(self, max_tokens, vocab, max_top_k):
        self.check(self.lib.pbmoe_head_reserve(self.h, max_tokens, vocab, max_top_k))

    def head_topk(self, weight, x, ids, values, id_base=0, allowed=None, keys=None, logits=None, stream=None):
        """weight bf16 [vocab, hidden]; x [tokens, hidden] bf16/f32; ids/values [tokens, top_k]."""
        head = Head(weight.data_ptr(), int(weight.shape[0]), int(weight.shape[1]), id_base)
        self.check(self.lib.pbmoe_head_topk(self.h, C.byref(head), _ptr(x), _dtype_code(x), int(x.shape[0]),
                                            int(ids.shape[1]), _ptr(allowed), _ptr(ids), _ptr(values), _ptr(keys),
                                            _ptr(logits), self.stream_ptr(stream)))

    def head_merge(self, keys, ids, values, out_ids, out_values, stream=None):
        """keys/ids/values [lists, tokens, top_k] (shards in id order) -> out [tokens, top_k]."""
        lists, tokens, top_k = (int(d) for d in keys.shape)
        self.check(self.lib.pbmoe_head_merge(self.h, _ptr(keys), _ptr(ids), _ptr(values), lists, tokens, top_k,
                                             _ptr(out_ids), _ptr(out_values), self.stream_ptr(stream)))

    def rms_norm(self, x, weight, out, eps=1e-6, residual=None, sum_out=None, width=None, stream=None):
        """Rows of x (2-D, f32/bf16; `width` leading columns of each row, default all):
        s = x (+ residual); sum_out <- s; out = rms_norm(s) * weight."""
        rows = int(x.shape[0])
        w = int(width if width is not None else x.shape[1])
        st = lambda t: int(t.stride(0)) if t is not None else 0
        a = NormArgs(x.data_ptr(), _dtype_code(x), None if residual is None else residual.data_ptr(),
                     None if sum_out is None else sum_out.data_ptr(),
                     _dtype_code(sum_out) if sum_out is not None else 0,
                     None if weight is None else weight.data_ptr(), eps, out.data_ptr(), _dtype_code(out), rows, w,
                     st(x), st(residual), st(sum_out), st(out))
        self.check(self.lib.pbmoe_rms_norm(self.h, C.byref(a), self.stream_ptr(stream)))

    def expert_layer_load(self, root, layer, layout: ExpertLayout, expert_begin, expert_count, dst, stream=None):
        """FIXED_Q4_EXPERT_LAYER_V1 slots into the device tensor dst (>= count x expert_bytes bytes)."""
        self.check(self.lib.pbmoe_expert_layer_load(self.h, str(root).encode(), layer, C.byref(layout), expert_begin,
                                                    expert_count, _ptr(dst), dst.numel() * dst.element_size(),
                                                    self.stream_ptr(stream)))

    def mxfp4_matvec(self, packed, scales, rows, cols, x, y, group=32, stream=None):
        """y [batch, rows] = W x for MXFP4 W: packed uint8 [rows, cols/2], scales uint8 [rows, cols/group]."""
        t = Mxfp4Tensor(packed.data_ptr(), scales.data_ptr(), rows, cols, group)
        self.check(self.lib.pbmoe_mxfp4_matvec(self.h, C.byref(t), _ptr(x), _dtype_code(x), _ptr(y), _dtype_code(y),
                                               int(x.shape[0]), self.stream_ptr(stream)))

    def rope_reserve(self, max_positions, rope_dim, theta=10000.0):
        self.check(self.lib.pbmoe_rope_reserve(self.h, max_positions, rope_dim, theta))

    def mla_append_decode(self, config, query, kv, positions, c_kv_ptrs, k_rope_ptrs, cache_len, c_kv, k_rope, w_uk,
                          w_uv, out, latent_norm=None, eps=1e-6, stream=None):
        """mla_rope_append followed by mla_decode in one call (pbmoe_mla_append_decode): query f32 [B, heads,
        nope+rope] rotated in place; kv, positions, c_kv_ptrs, k_rope_ptrs, cache_len, latent_norm as for
        mla_rope_append; c_kv / k_rope lists of B device tensors (the attended rows) as for mla_decode."""
        b = len(c_kv)
        lens = (C.c_uint32 * b)(*[int(t.shape[0]) for t in c_kv])
        ckv = (C.c_void_p * b)(*[t.data_ptr() for t in c_kv])
        kr = (C.c_void_p * b)(*[t.data_ptr() for t in k_rope])
        args = MlaArgs(b, C.cast(lens, C.c_void_p), query.data_ptr(), _dtype_code(query), C.cast(ckv, C.c_void_p),
                       C.cast(kr, C.c_void_p), w_uk.data_ptr(), w_uv.data_ptr(), out.data_ptr(), _dtype_code(out))
        self.check(self.lib.pbmoe_mla_append_decode(self.h, C.byref(config), C.byref(args), _ptr(kv), _ptr(latent_norm),
                                                    eps, _ptr(positions), _ptr(c_kv_ptrs), _ptr(k_rope_ptrs),
                                                    cache_len, self.stream_ptr(stream)))

    def mla_rope_append(self, config, query, kv, positions, c_kv_ptrs, k_rope_ptrs, cache_len, latent_norm=None,
                        eps=1e-6, stream=None):
        """query f32 [B, heads, nope+rope] (in place); kv f32 [B, latent+rope] (latent part normed here when
        latent_norm, f32 [latent], is given); positions int32 [B] device; c_kv_ptrs / k_rope_ptrs int64 [B]
        device tensors of cache addresses."""
        self.check(self.lib.pbmoe_mla_rope_append(self.h, C.byref(config), int(query.shape[0]), _ptr(query), _ptr(kv),
                                                  _ptr(latent_norm), eps, _ptr(positions), _ptr(c_kv_ptrs),
                                                  _ptr(k_rope_ptrs), cache_len, self.stream_ptr(stream)))

    def q4_fused(self, mats, x, ys, norm=None, eps=1e-6, residual=None, stream=None):
        """One launch of pbmoe_q4_matvec_fused: mats = [(packed, scales, biases, rows, cols, group)] (one or two
        on the same x), ys the outputs [batch, rows_i]; norm (f32 [cols]) normalises x first; residual is
        added to the single output."""
        ts = [Q4Tensor(p.data_ptr(), s.data_ptr(), b.data_ptr(), r, c, g) for (p, s, b, r, c, g) in mats]
        a = Q4FusedArgs()
        a.w[0] = C.pointer(ts[0])
        a.w[1] = C.pointer(ts[1]) if len(ts) > 1 else C.POINTER(Q4Tensor)()
        a.y[0] = ys[0].data_ptr()
        a.y[1] = ys[1].data_ptr() if len(ys) > 1 else None
        a.x, a.x_dtype, a.y_dtype, a.batch = x.data_ptr(), _dtype_code(x), _dtype_code(ys[0]), int(x.shape[0])
        a.input_norm_weight = None if norm is None else norm.data_ptr()
        a.epsilon = eps
        a.residual = None if residual is None else residual.data_ptr()
        self.check(self.lib.pbmoe_q4_matvec_fused(self.h, C.byref(a), self.stream_ptr(stream)))

    def q4_matvec_batch(self, mats, x, ys, stream=None):
        """pbmoe_q4_matvec_batch: mats = [(packed, scales, biases, rows, cols, group)] on the same x, ys the
        outputs [batch, rows_i] (one dtype)."""
        n = len(mats)
        ts = (Q4Tensor * n)(*[Q4Tensor(p.data_ptr(), s.data_ptr(), b.data_ptr(), r, c, g) for (p, s, b, r, c, g) in mats])
        yp = (C.c_void_p * n)(*[y.data_ptr() for y in ys])
        self.check(self.lib.pbmoe_q4_matvec_batch(self.h, ts, n, x.data_ptr(), _dtype_code(x), yp,
                                                  _dtype_code(ys[0]), int(x.shape[0]), self.stream_ptr(stream)))

    def prefill_reserve(self, max_rows, max_cols):
        self.check(self.lib.pbmoe_prefill_reserve(self.h, max_rows, max_cols))

    def q4_gemm(self, packed, scales, biases, rows, cols, group, x, y, stream=None):
        """y [m, rows] = x [m, cols] . W^T for a dense Q4 weight (x bf16 needs prefill_reserve)."""
        t = Q4Tensor(packed.data_ptr(), scales.data_ptr(), biases.data_ptr(), rows, cols, group)
        self.check(self.lib.pbmoe_q4_gemm(self.h, C.byref(t), _ptr(x), _dtype_code(x), _ptr(y), _dtype_code(y),
                                          int(x.shape[0]), self.stream_ptr(stream)))

    def prefill_group_plan(self, route_ids, rows, top_k, num_experts, slot_experts, unique_count, source_rows,
                           output_indices, groups, route_slots=None, stream=None):
        self.check(self.lib.pbmoe_prefill_group_plan(
            self.h, _ptr(route_ids), rows, top_k, num_experts, _ptr(slot_experts), _ptr(unique_count),
            _ptr(route_slots), _ptr(source_rows), _ptr(output_indices), _ptr(groups), self.stream_ptr(stream)))

    def q4_gemm_grouped(self, matrix: Q4ExpertMatrix, slot_experts, unique_count, groups, source_rows, routes,
                        max_unique, x, y, stream=None):
        self.check(self.lib.pbmoe_q4_gemm_grouped(
            self.h, C.byref(matrix), _ptr(slot_experts), _ptr(unique_count), _ptr(groups), _ptr(source_rows),
            routes, max_unique, _ptr(x), _dtype_code(x), int(x.shape[0]), _ptr(y), _dtype_code(y),
            self.stream_ptr(stream)))

    # ---------------------------------------------------------- expert parallelism
    def ep_reserve(self, rank, world, max_tokens, hidden):
        self.check(self.lib.pbmoe_ep_reserve(self.h, rank, world, max_tokens, hidden))

    def ep_ipc_handle(self) -> bytes:
        buf = (C.c_char * EP_HANDLE_BYTES)()
        self.check(self.lib.pbmoe_ep_ipc_handle(self.h, C.cast(buf, C.c_void_p)))
        return bytes(buf)

    def ep_open_peers(self, handles):
        blob = b"".join(handles)
        buf = (C.c_char * len(blob)).from_buffer_copy(blob)
        self.check(self.lib.pbmoe_ep_open_peers(self.h, C.cast(buf, C.c_void_p)))

    def ep_buffer(self) -> int:
        return self.lib.pbmoe_ep_buffer(self.h) or 0

    def ep_set_peers(self, pointers):
        arr = (C.c_void_p * len(pointers))(*pointers)
        self.check(self.lib.pbmoe_ep_set_peers(self.h, C.cast(arr, C.c_void_p)))

    def ep_moe_layer(self, config, weights: MoeWeights, shard: EpShard, x, out, tokens, residual=None,
                     next_norm_weight=None, next_normed=None, debug: MoeDebug | None = None, stream=None):
        _same_dtype(out, residual, next_normed)
        self.check(self.lib.pbmoe_ep_moe_layer(
            self.h, C.byref(config), C.byref(weights), C.byref(shard), _ptr(x), _dtype_code(x), _ptr(residual),
            _ptr(out), _dtype_code(out), tokens, _ptr(next_norm_weight), _ptr(next_normed),
            C.byref(debug) if debug is not None else None, self.stream_ptr(stream)))

    def device_status(self, clear=True, stream=None) -> int:
        v = C.c_uint32()
        self.check(self.lib.pbmoe_device_status(self.h, self.stream_ptr(stream), C.byref(v), 1 if clear else 0))
        return v.value


def mla_config(heads=16, nope=128, rope=64, latent=512, v_dim=128, scale=0.0) -> MlaConfig:
    return MlaConfig(heads, nope, rope, latent, v_dim, scale)


def expert_matrix(experts, layout: ExpertLayout, num_experts, projection) -> Q4ExpertMatrix:
    """One projection ("gate", "up" or "down") of an expert table laid out by `layout`."""
    i = {"gate": 0, "up": 3, "down": 6}[projection]
    rows, cols = ((layout.intermediate, layout.hidden) if projection != "down"
                  else (layout.hidden, layout.intermediate))
    off = layout.component_offsets
    return Q4ExpertMatrix(experts.data_ptr(), layout.expert_bytes, off[i], off[i + 1], off[i + 2], num_experts,
                          rows, cols, layout.group_size)


def moe_config(layout: ExpertLayout, num_experts, top_k, normalization=0, routed_scale=1.0, eps=1e-6) -> MoeConfig:
    return MoeConfig(layout, num_experts, top_k, normalization, routed_scale, eps)


def expert_layer_read(root, layer, layout: ExpertLayout, expert_begin, expert_count):
    """Slots of experts [begin, begin + count) of a FIXED_Q4_EXPERT_LAYER_V1 store, as host bytes
    (numpy uint8 [count, expert_bytes]); PbmoeError on invalid metadata."""
    import numpy as np

    out = np.zeros((expert_count, layout.expert_bytes), np.uint8)
    err = C.create_string_buffer(512)
    rc = load().pbmoe_expert_layer_read(str(root).encode(), layer, C.byref(layout), expert_begin, expert_count,
                                        out.ctypes.data_as(C.c_void_p), out.nbytes, err, 512)
    if rc != PBMOE_OK:
        raise PbmoeError(rc, err.value.decode())
    return out


def ep_expert_range(num_experts, rank, world):
    """(begin, count) of the experts rank `rank` of `world` owns (host-only)."""
    b, n = C.c_uint32(), C.c_uint32()
    rc = load().pbmoe_ep_expert_range(num_experts, rank, world, C.byref(b), C.byref(n))
    if rc != PBMOE_OK:
        raise PbmoeError(rc, f"invalid expert partition E={num_experts} rank={rank} world={world}")
    return b.value, n.value
