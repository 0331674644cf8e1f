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
// Decode and per-group arithmetic: mxfp4.cuh. E8M0 255 (not finite, where
// the reference bails) latches PBMOE_DEV_ERR_MXFP4_SCALE.

#include "kernels.h"
#include "mxfp4.cuh"

namespace pbmoe {

constexpr int kMxWarps = 8;

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
                float part[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) part[t] = 0.f;
                mx_group_dot<NT>(w[r], xs + g * 36, pcols, part);
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
