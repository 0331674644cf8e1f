// common.cuh — shared device helpers for the sm_100a FlashMoE kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pbmoe_cuda.h"

namespace pbmoe {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// bf16 bits -> f32 (experts/mod.rs:917-934: bits << 16).
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
    return __uint_as_float(bits16 << 16);
}

// f32 -> bf16 bits, round to nearest even (experts/slots.rs:1165-1169). NaN
// inputs keep the reference's wrapping-add behaviour.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
    uint32_t bits = __float_as_uint(v);
    uint32_t lsb = (bits >> 16) & 1u;
    return static_cast<uint16_t>((bits + 0x7fffu + lsb) >> 16);
}

template <typename T>
__device__ __forceinline__ float load_act(const T* p, size_t i);
template <>
__device__ __forceinline__ float load_act<float>(const float* p, size_t i) {
    return p[i];
}
template <>
__device__ __forceinline__ float load_act<uint16_t>(const uint16_t* p, size_t i) {
    return bf16_bits_to_f32(p[i]);
}

template <typename T>
__device__ __forceinline__ void store_act(T* p, size_t i, float v);
template <>
__device__ __forceinline__ void store_act<float>(float* p, size_t i, float v) {
    p[i] = v;
}
template <>
__device__ __forceinline__ void store_act<uint16_t>(uint16_t* p, size_t i, float v) {
    p[i] = f32_to_bf16_bits(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Sum over aligned groups of `width` lanes (width a power of two <= 32).
template <int WIDTH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// L2 policy for bytes a decode step reads once (weights, KV cache rows):
// evict first. The step streams far more than L2 holds, and with the normal
// policy those bytes push out what its kernels keep re-reading (activations,
// workspace, the kernels' own instructions).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Streaming 128-bit load of weight bytes that are read once per launch:
// bypass L1 allocation, evict first from L2.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(l2_evict_first()));
    return r;
}

// The same for 8 bytes.
__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p), "l"(l2_evict_first()));
    return r;
}

__device__ __forceinline__ uint32_t ld_nc_u32(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

// ---------------------------------------------------------------------------
// Q4 chunk arithmetic.
//
// A chunk is 16 bytes of packed nibbles = 32 consecutive columns c0..c0+31 of
// one row, all inside one quantisation group (the fast path requires
// group_size % 32 == 0). Within u32 word i of the chunk, nibble k is column
// c0 + 8i + k (little-endian, low nibble first).
//
// The per-group sum  sum_c (q_c*s + b) * x_c  is evaluated as
//     s * sum_c q_c x_c + b * sum_c x_c
// with sum_c x_c precomputed once per activation vector. q_c * x_c is formed
// without an int->float conversion: placing the nibble at mantissa bit p of
// 1.0f gives the exact float 1 + q*2^(p-23), so
//     sum_c q_c x_c = 2^(23-p) * (sum_c (1 + q_c 2^(p-23)) x_c - sum_c x_c).
// Shifting the word by 12, 4, -4 and -12 bits puts the even nibbles of each
// pair at p = 12 and the odd nibbles at p = 16: one shift per two nibbles,
// one LOP3 and one FFMA per nibble. The relative error of the recovered
// products is about 2^-(p+1) (<= 1.2e-4), far inside the 1e-2 parity bound.
// ---------------------------------------------------------------------------
struct ChunkF {
    float f[32];  // f[2m] even column, f[2m+1] odd column, m = 0..15 in column order
};

__device__ __forceinline__ void decode_chunk(const uint4 w, ChunkF& c) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t s0 = words[i] << 12;  // n0 -> bit 12, n1 -> bit 16
        const uint32_t s1 = words[i] << 4;   // n2 -> 12, n3 -> 16
        const uint32_t s2 = words[i] >> 4;   // n4 -> 12, n5 -> 16
        const uint32_t s3 = words[i] >> 12;  // n6 -> 12, n7 -> 16
        const uint32_t s[4] = {s0, s1, s2, s3};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            c.f[8 * i + 2 * m] = __uint_as_float((s[m] & 0x0000F000u) | 0x3F800000u);
            c.f[8 * i + 2 * m + 1] = __uint_as_float((s[m] & 0x000F0000u) | 0x3F800000u);
        }
    }
}

// Shared-memory activation chunks are stored swizzled: logical float4 k of
// chunk j sits at physical float4 (k ^ (j & 7)) of the chunk's 128 bytes, so
// eight lanes reading float4 k of eight consecutive chunks hit distinct banks.
__host__ __device__ __forceinline__ uint32_t xs_index(uint32_t chunk, uint32_t col_in_chunk) {
    return (chunk << 5) + ((((col_in_chunk >> 2) ^ (chunk & 7u)) << 2) | (col_in_chunk & 3u));
}

// Dot of a decoded chunk with its 32 activations (the chunk's swizzled 128
// bytes in shared memory, `swz` = chunk & 7) whose even/odd sums are xse/xso.
// Returns sum_c q_c x_c.
__device__ __forceinline__ float chunk_qdot(const ChunkF& c, const float* __restrict__ x, uint32_t swz,
                                            float xse, float xso) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float ae = 0.f, ao = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float4 v = x4[j ^ swz];
        ae = fmaf(c.f[4 * j + 0], v.x, ae);
        ao = fmaf(c.f[4 * j + 1], v.y, ao);
        ae = fmaf(c.f[4 * j + 2], v.z, ae);
        ao = fmaf(c.f[4 * j + 3], v.w, ao);
    }
    return 2048.0f * (ae - xse) + 128.0f * (ao - xso);
}

// Device status word helpers.
__device__ __forceinline__ void latch_status(uint32_t* status, uint32_t bits) {
    if (status) atomicOr(status, bits);
}

// Programmatic dependent launch: wait for the preceding kernel's memory, and
// allow the next kernel in the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" :::);
}

// Host: launch `fn` with programmatic stream serialization, so it may start
// while its predecessor in the stream finishes; the kernel must call
// pdl_wait() before reading anything an earlier kernel wrote.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_kernel(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, static_cast<KArgs>(args)...);
}

}  // namespace pbmoe
