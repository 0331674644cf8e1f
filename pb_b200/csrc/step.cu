// step.cu — the per-layer glue of a decode step around the MLA attention and
// MoE kernels (config 4):
//
//   rms_norm_rows_kernel   s = x (+ residual), out = s * rsqrt(mean(s^2) + eps) * w
//                          per row: rms_norm_reduced (shaders.metal:1176-1213), run on
//                          q_a and the latent part of kv_a by the MLA input
//                          projection chain (metal/qwen_execution.rs:405-437), and
//                          the residual add + post-attention norm ahead of the router
//                          (CMD2, metal/mod.rs:2864-3012)
//   mla_rope_append_kernel RoPE on every head's rope part of the query and on the
//                          key's rope part (apply_rotary_interleaved_to_split_half,
//                          math.rs:822-846, as called at runtime/mod.rs:2896-2913),
//                          then the latent and rotated key rows written into the
//                          sequence's cache at its position (KvCache::record_mla_kv,
//                          state/kv_cache.rs:414-450)
//
// The cos/sin table is built on the host in f64 exactly as the reference
// builds its angles (runtime/mod.rs:2825-2836), so the rotation, done with
// unfused f32 multiplies and adds as in the reference, is bit-exact. Both
// kernels use programmatic dependent launch (griddepcontrol.wait first).

#include "common.cuh"
#include "kernels.h"
#include "rope.cuh"

namespace pbmoe {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float ld_any(const void* p, pbmoe_dtype t, size_t i) {
    return t == PBMOE_BF16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]) : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_any(void* p, pbmoe_dtype t, size_t i, float v) {
    if (t == PBMOE_BF16)
        static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
    else
        static_cast<float*>(p)[i] = v;
}

__global__ void __launch_bounds__(kNormThreads) rms_norm_rows_kernel(NormArgs a) {
    __shared__ float red[kNormThreads / 32];
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t r = blockIdx.x;
    const size_t xo = static_cast<size_t>(r) * a.x_stride, ro = static_cast<size_t>(r) * a.residual_stride;
    const size_t so = static_cast<size_t>(r) * a.sum_stride, oo = static_cast<size_t>(r) * a.out_stride;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < a.width; i += blockDim.x) {
        float s = ld_any(a.x, a.x_dtype, xo + i);
        if (a.residual) s += ld_any(a.residual, a.x_dtype, ro + i);
        if (a.sum_out) st_any(a.sum_out, a.sum_dtype, so + i, s);
        ss += s * s;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(a.width) + a.epsilon);
    for (uint32_t i = threadIdx.x; i < a.width; i += blockDim.x) {
        // the sum as written (its own rounding when stored in bf16), else recomputed
        float s;
        if (a.sum_out) {
            s = ld_any(a.sum_out, a.sum_dtype, so + i);
        } else {
            s = ld_any(a.x, a.x_dtype, xo + i);
            if (a.residual) s += ld_any(a.residual, a.x_dtype, ro + i);
        }
        st_any(a.out, a.out_dtype, oo + i, s * scale * (a.weight ? a.weight[i] : 1.0f));
    }
}

cudaError_t rms_norm_launch(const NormArgs& a, cudaStream_t s) {
    if (a.rows == 0) return cudaSuccess;
    return launch_pdl_kernel(rms_norm_rows_kernel, dim3(a.rows), dim3(kNormThreads), 0, s, a);
}

constexpr int kRopeThreads = 256;
constexpr uint32_t kRopeMaxPairs = 2048;  // heads x rope/2 rotated per token

// The query pairs of every head rotated in place (all of a thread's pairs
// read before any is written), then the key and latent rows appended
// (rope_append_kv, rope.cuh).
constexpr uint32_t kRopeMaxLatent = kRopeMaxLatentPerThread * kRopeThreads;
__global__ void __launch_bounds__(kRopeThreads) mla_rope_append_kernel(RopeAppendArgs a) {
    __shared__ float red[kRopeThreads / 32];
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t b = blockIdx.x;
    uint32_t pos;
    if (!rope_token_position(a, b, pos)) return;
    const uint32_t half = a.rope / 2, qk = a.nope + a.rope;
    const float2* cs = a.table + static_cast<size_t>(pos) * half;
    float* q = a.query + static_cast<size_t>(b) * a.heads * qk;
    constexpr int kPer = kRopeMaxPairs / kRopeThreads;
    float va[kPer], vb[kPer];
    float2 tq[kPer];
    const uint32_t pairs = a.heads * half;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t i = threadIdx.x + j * kRopeThreads;
        if (i < pairs) {
            const uint32_t h = i / half, p = i - h * half;
            va[j] = q[h * qk + a.nope + 2 * p];
            vb[j] = q[h * qk + a.nope + 2 * p + 1];
            tq[j] = cs[p];  // (cos, sin)
        }
    }
    __syncthreads();  // every query pair read before the split halves are written
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t i = threadIdx.x + j * kRopeThreads;
        if (i < pairs) {
            const uint32_t h = i / half, p = i - h * half;
            q[h * qk + a.nope + p] = __fsub_rn(__fmul_rn(va[j], tq[j].x), __fmul_rn(vb[j], tq[j].y));
            q[h * qk + a.nope + half + p] = __fadd_rn(__fmul_rn(vb[j], tq[j].x), __fmul_rn(va[j], tq[j].y));
        }
    }
    rope_append_kv(a, b, pos, red);
}

bool rope_append_supported(uint32_t heads, uint32_t rope) {
    return rope > 0 && rope % 2 == 0 && heads > 0 && heads * (rope / 2) <= kRopeMaxPairs && rope / 2 <= kRopeThreads;
}

cudaError_t mla_rope_append_launch(const RopeAppendArgs& a, cudaStream_t s) {
    if (a.batch == 0) return cudaSuccess;
    if (!rope_append_supported(a.heads, a.rope) || a.latent > kRopeMaxLatent) return cudaErrorInvalidValue;
    return launch_pdl_kernel(mla_rope_append_kernel, dim3(a.batch), dim3(kRopeThreads), 0, s, a);
}

}  // namespace pbmoe
