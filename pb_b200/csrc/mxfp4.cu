// mxfp4.cu — MXFP4 (E2M1 values, E8M0 scale per 32 columns) matvec for
// decode: y[t][r] = sum_c e2m1(W[r][c]) * 2^(S[r][c/32] - 127) * x[t][c], the
// GLM-5.2 expert format (FIXED_MXFP4_EXPERT_LAYER_V1). Reference:
// mxfp4_fma_matvec_e8m0 (shaders.metal:200-298) and its CPU restatement
// mxfp4_fma_matvec_with_group_size (experts/slots.rs:1239-1287).
//
// HBM-bound: 4.25 bits per weight. A lane owns whole 32-column groups: one
// 16-byte load of 32 nibbles plus one scale byte per group; a warp works on
// R rows at once (2 for 1-2 tokens, 1 for wider batches, whose per-token
// accumulators take the registers) so each lane has several loads in flight.
//
// Decode: two nibbles at a time are placed into the exponent/mantissa fields
// of an fp16 pair (bits (n & 7) << 9 and sign (n & 8) << 12): the fp16 value
// is e2m1(n) * 2^-14 exactly (e = 0 lands in the fp16 subnormals), converted
// to f32 exactly. Products with x accumulate per group; the group sum is then
// scaled by 2^14 and by the E8M0 scale, both powers of two, so each term
// rounds as the reference's weight * scale * x does and only the summation
// order differs. E8M0 255 (not finite, where the reference bails) latches
// PBMOE_DEV_ERR_MXFP4_SCALE.

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace pbmoe {

constexpr int kMxWarps = 8;

// nibbles n0 (bits 0-3) and n1 (bits 16-19) of `v` -> two floats e2m1 * 2^-14
__device__ __forceinline__ float2 e2m1_pair(uint32_t v) {
    const uint32_t h = ((v & 0x00070007u) << 9) | ((v & 0x00080008u) << 12);
    __half2 hh;
    memcpy(&hh, &h, 4);
    return __half22float2(hh);
}

__device__ __forceinline__ float e8m0_scale(uint32_t e) {
    return __uint_as_float(e == 0 ? 0x00400000u : (e << 23));
}

template <typename XT, typename YT, int NT, int kMxRows>
__global__ void __launch_bounds__(kMxWarps * 32)
mxfp4_matvec_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales, uint32_t rows,
                    uint32_t cols, const XT* __restrict__ x, YT* __restrict__ y, uint32_t batch,
                    uint32_t* status) {
    // x [NT][cols] with 4 floats of padding after every 32 columns: lane l
    // reads group l, so unpadded rows would put every lane's 16-byte reads
    // in the same banks
    extern __shared__ float xs[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t groups = cols / 32;
    const uint32_t pcols = groups * 36;
    const uint32_t r0 = (blockIdx.x * kMxWarps + warp) * kMxRows;
    for (uint32_t t0 = 0; t0 < batch; t0 += NT) {
        const int nt = static_cast<int>(min(batch - t0, static_cast<uint32_t>(NT)));
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < NT * cols; i += blockDim.x) {
            const uint32_t t = i / cols, c = i - t * cols;
            xs[t * pcols + c + (c >> 5) * 4] =
                static_cast<int>(t) < nt ? load_act<XT>(x, static_cast<size_t>(t0 + t) * cols + c) : 0.f;
        }
        __syncthreads();
        float acc[kMxRows][NT];
#pragma unroll
        for (int r = 0; r < kMxRows; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        for (uint32_t g = lane; g < groups; g += 32) {
            uint4 w[kMxRows];
            uint32_t sb[kMxRows];
#pragma unroll
            for (int r = 0; r < kMxRows; ++r) {
                const uint32_t row = min(r0 + r, rows - 1);  // rows past the end read the last row, dropped
                w[r] = ld_stream_u4(packed + static_cast<size_t>(row) * (cols / 2) + static_cast<size_t>(g) * 16);
                sb[r] = scales[static_cast<size_t>(row) * groups + g];
            }
#pragma unroll
            for (int r = 0; r < kMxRows; ++r) {
                if (sb[r] == 255u && r0 + r < rows && status) atomicOr(status, PBMOE_DEV_ERR_MXFP4_SCALE);
                const uint32_t words[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
                float part[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) part[t] = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    // bytes b0..b3 of the word = columns 8q + 2j (low nibble), 8q + 2j + 1 (high)
                    const uint32_t v = words[q];
                    const float2 lo02 = e2m1_pair(__byte_perm(v, 0, 0x4140));         // cols 0, 2
                    const float2 hi02 = e2m1_pair(__byte_perm(v, 0, 0x4140) >> 4);    // cols 1, 3
                    const float2 lo46 = e2m1_pair(__byte_perm(v, 0, 0x4342));         // cols 4, 6
                    const float2 hi46 = e2m1_pair(__byte_perm(v, 0, 0x4342) >> 4);    // cols 5, 7
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        const float* xr = xs + t * pcols + g * 36 + q * 8;
                        const float4 xa = *reinterpret_cast<const float4*>(xr);
                        const float4 xb = *reinterpret_cast<const float4*>(xr + 4);
                        float s = part[t];
                        s = fmaf(lo02.x, xa.x, s);
                        s = fmaf(hi02.x, xa.y, s);
                        s = fmaf(lo02.y, xa.z, s);
                        s = fmaf(hi02.y, xa.w, s);
                        s = fmaf(lo46.x, xb.x, s);
                        s = fmaf(hi46.x, xb.y, s);
                        s = fmaf(lo46.y, xb.z, s);
                        s = fmaf(hi46.y, xb.w, s);
                        part[t] = s;
                    }
                }
                const float scale = e8m0_scale(sb[r]);
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[r][t] += (part[t] * 16384.0f) * scale;
            }
        }
#pragma unroll
        for (int r = 0; r < kMxRows; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(acc[r][t]);
                if (lane == 0 && r0 + r < rows && t < nt)
                    store_act<YT>(y, static_cast<size_t>(t0 + t) * rows + r0 + r, v);
            }
    }
}

bool mxfp4_supported(uint32_t rows, uint32_t cols, uint32_t group, uint32_t batch) {
    return rows > 0 && cols > 0 && group == 32 && cols % 32 == 0 && batch > 0 &&
           static_cast<size_t>(cols / 32) * 36 * 8 * sizeof(float) <= 200 * 1024;
}

template <typename XT, typename YT, int NT>
static cudaError_t mxfp4_t(const Mxfp4Args& a, cudaStream_t s) {
    constexpr int kMxRows = NT <= 2 ? 2 : 1;
    auto fn = mxfp4_matvec_kernel<XT, YT, NT, kMxRows>;
    const size_t smem = static_cast<size_t>(NT) * (a.cols / 32) * 36 * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const uint32_t per_cta = kMxWarps * kMxRows;
    fn<<<(a.rows + per_cta - 1) / per_cta, kMxWarps * 32, smem, s>>>(
        a.packed, a.scales, a.rows, a.cols, static_cast<const XT*>(a.x), static_cast<YT*>(a.y), a.batch, a.status);
    return cudaGetLastError();
}

template <typename XT, typename YT>
static cudaError_t mxfp4_b(const Mxfp4Args& a, cudaStream_t s) {
    if (a.batch == 1) return mxfp4_t<XT, YT, 1>(a, s);
    if (a.batch == 2) return mxfp4_t<XT, YT, 2>(a, s);
    if (a.batch <= 4) return mxfp4_t<XT, YT, 4>(a, s);
    return mxfp4_t<XT, YT, 8>(a, s);
}

cudaError_t mxfp4_matvec_launch(const Mxfp4Args& a, cudaStream_t s) {
    if (!mxfp4_supported(a.rows, a.cols, a.group, a.batch)) return cudaErrorInvalidValue;
    if (a.x_dtype == PBMOE_BF16)
        return a.y_dtype == PBMOE_BF16 ? mxfp4_b<uint16_t, uint16_t>(a, s) : mxfp4_b<uint16_t, float>(a, s);
    return a.y_dtype == PBMOE_BF16 ? mxfp4_b<float, uint16_t>(a, s) : mxfp4_b<float, float>(a, s);
}

}  // namespace pbmoe
