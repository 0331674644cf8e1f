// rope.cuh — per-token pieces of the MLA RoPE + KV-cache append
// (apply_rotary_interleaved_to_split_half, math.rs:822-846, as called at
// runtime/mod.rs:2896-2913; KvCache::record_mla_kv, state/kv_cache.rs:414-450),
// shared by the standalone append kernel (step.cu) and the absorb kernel that
// does the append on the way (mla.cu). The rotation uses unfused f32
// multiplies and adds from the f64-built cos/sin table, as the reference.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace pbmoe {

constexpr uint32_t kRopeMaxLatentPerThread = 4;  // latent values a thread holds (latent <= 4 x blockDim.x)

// The token's position, or false (and PBMOE_DEV_ERR_POSITION latched by
// thread 0) when it lies past the cache or the RoPE table.
__device__ __forceinline__ bool rope_token_position(const RopeAppendArgs& a, uint32_t b, uint32_t& pos) {
    pos = a.positions[b];
    if (pos >= a.max_positions || pos >= a.cache_len) {
        if (threadIdx.x == 0 && a.status) atomicOr(a.status, PBMOE_DEV_ERR_POSITION);
        return false;
    }
    return true;
}

// The key's rope part rotated and written as the bf16 cache row of token b at
// `pos`, then the latent row (normalised here with a.latent_norm_w: the
// formula of rms_norm_rows_kernel, the sum of squares in the order of a
// strided loop). Run by the whole CTA (blockDim.x threads, rope/2 <=
// blockDim.x, latent <= 4 blockDim.x); `red` is shared scratch of
// blockDim.x / 32 floats. Every load of a thread is issued before any use.
__device__ __forceinline__ void rope_append_kv(const RopeAppendArgs& a, uint32_t b, uint32_t pos, float* red) {
    const uint32_t half = a.rope / 2, nthr = blockDim.x;
    const float2* cs = a.table + static_cast<size_t>(pos) * half;
    const float* kv = a.kv + static_cast<size_t>(b) * (a.latent + a.rope);
    const bool key_lane = threadIdx.x < half;
    float k0 = 0.f, k1 = 0.f;
    float2 tk = make_float2(0.f, 0.f);
    if (key_lane) {
        k0 = kv[a.latent + 2 * threadIdx.x];
        k1 = kv[a.latent + 2 * threadIdx.x + 1];
        tk = cs[threadIdx.x];
    }
    float lv[kRopeMaxLatentPerThread], nw[kRopeMaxLatentPerThread];
#pragma unroll
    for (uint32_t j = 0; j < kRopeMaxLatentPerThread; ++j) {
        const uint32_t i = threadIdx.x + j * nthr;
        lv[j] = i < a.latent ? kv[i] : 0.f;
        nw[j] = (i < a.latent && a.latent_norm_w) ? a.latent_norm_w[i] : 1.0f;
    }
    if (key_lane) {
        uint16_t* krow = a.k_rope[b] + static_cast<size_t>(pos) * a.rope;
        krow[threadIdx.x] = f32_to_bf16_bits(__fsub_rn(__fmul_rn(k0, tk.x), __fmul_rn(k1, tk.y)));
        krow[half + threadIdx.x] = f32_to_bf16_bits(__fadd_rn(__fmul_rn(k1, tk.x), __fmul_rn(k0, tk.y)));
    }
    float scale = 1.0f;
    if (a.latent_norm_w) {
        float ss = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < kRopeMaxLatentPerThread; ++j) ss += lv[j] * lv[j];
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
        for (uint32_t w = 0; w < nthr / 32; ++w) tot += red[w];
        scale = 1.0f / sqrtf(tot / static_cast<float>(a.latent) + a.eps);
    }
    uint16_t* crow = a.c_kv[b] + static_cast<size_t>(pos) * a.latent;
#pragma unroll
    for (uint32_t j = 0; j < kRopeMaxLatentPerThread; ++j) {
        const uint32_t i = threadIdx.x + j * nthr;
        if (i < a.latent) crow[i] = f32_to_bf16_bits(a.latent_norm_w ? lv[j] * scale * nw[j] : lv[j]);
    }
}

}  // namespace pbmoe
