// q4_matvec.cu — decode Q4 matvec y[b] = W x[b] (pbmoe_q4_matvec).
//
// Replaces q4_fma_matvec_bf16_scale_bias (shaders.metal:164-199), which gives
// each Apple SIMD group one row and stages x in an 8192-float threadgroup
// cache. Here each warp owns kRows rows per lane group; every lane streams
// 16-byte chunks of packed nibbles with ld.global.nc.L1::no_allocate (all of a
// warp's chunk loads are issued before its arithmetic), x is staged once per
// CTA in shared memory (swizzled, with per-chunk sums), and the row sums are
// finished with warp shuffles. Shapes outside the fast path (cols % 32 != 0,
// non power-of-two groups, unaligned rows) run a per-element kernel with the
// reference's own per-element arithmetic.

#include "kernels.h"
#include "q4_rows.cuh"

namespace pbmoe {

constexpr int kMvThreads = 128;
constexpr int kMvRows = 4;  // rows per lane group per pass

template <typename XT, typename YT, int LPR, int CPL, int NT>
__global__ void __launch_bounds__(kMvThreads)
q4_matvec_fast_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                      const uint16_t* __restrict__ biases, Q4Geom g, const XT* __restrict__ x,
                      YT* __restrict__ y, uint32_t batch) {
    extern __shared__ __align__(16) float smem[];
    constexpr int kGroups = 32 / LPR;
    constexpr int kRowsPerCta = kMvRows * kGroups * (kMvThreads / 32);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane / LPR;
    float* xs = smem;
    float* xe = xs + NT * g.cols;
    float* xo = xe + NT * g.chunks;
    const uint32_t r0 = blockIdx.x * kRowsPerCta + (warp * kGroups + sub) * kMvRows;
    const uint8_t* pk[kMvRows];
    const uint16_t* ps[kMvRows];
    const uint16_t* pb[kMvRows];
#pragma unroll
    for (int r = 0; r < kMvRows; ++r) {
        const uint32_t row = r0 + r;
        pk[r] = row < g.rows ? packed + static_cast<size_t>(row) * (g.cols / 2) : nullptr;
        ps[r] = scales + static_cast<size_t>(row) * g.gpr;
        pb[r] = biases + static_cast<size_t>(row) * g.gpr;
    }
    for (uint32_t b0 = 0; b0 < batch; b0 += NT) {
        const int nt = static_cast<int>(min(batch - b0, static_cast<uint32_t>(NT)));
        __syncthreads();
        stage_x_fast<XT>(x + static_cast<size_t>(b0) * g.cols, g.cols, nullptr, nt, g.cols, xs, xe, xo);
        __syncthreads();
        float acc[kMvRows][NT];
        q4_rows_partial<LPR, kMvRows, CPL, NT>(pk, ps, pb, g, xs, xe, xo, nt, acc);
#pragma unroll
        for (int r = 0; r < kMvRows; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float s = group_sum<LPR>(acc[r][t]);
                if ((lane & (LPR - 1)) == 0 && t < nt && r0 + r < g.rows)
                    store_act<YT>(y, static_cast<size_t>(b0 + t) * g.rows + r0 + r, s);
            }
        }
    }
}

template <typename XT, typename YT>
__global__ void __launch_bounds__(kMvThreads)
q4_matvec_generic_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                         const uint16_t* __restrict__ biases, uint32_t rows, uint32_t cols, uint32_t group,
                         const XT* __restrict__ x, YT* __restrict__ y, uint32_t batch) {
    extern __shared__ __align__(16) float smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t gpr = (cols + group - 1) / group;
    const uint32_t row = blockIdx.x * (kMvThreads / 32) + warp;
    for (uint32_t b = 0; b < batch; ++b) {
        __syncthreads();
        stage_x_generic<XT>(x + static_cast<size_t>(b) * cols, cols, nullptr, 1, cols, smem);
        __syncthreads();
        if (row < rows) {
            const float p = q4_row_partial_generic(packed + static_cast<size_t>(row) * ((cols + 1) / 2),
                                                   scales + static_cast<size_t>(row) * gpr,
                                                   biases + static_cast<size_t>(row) * gpr, cols, group, smem, lane,
                                                   32);
            const float s = warp_sum(p);
            if (lane == 0) store_act<YT>(y, static_cast<size_t>(b) * rows + row, s);
        }
    }
}

template <typename XT, typename YT, int LPR, int CPL, int NT>
static cudaError_t launch_fast(const Q4MatvecArgs& a, const Q4Geom& g, cudaStream_t s) {
    constexpr int kGroups = 32 / LPR;
    constexpr int kRowsPerCta = kMvRows * kGroups * (kMvThreads / 32);
    const size_t smem = static_cast<size_t>(NT) * (g.cols + 2ull * g.chunks) * sizeof(float);
    auto fn = q4_matvec_fast_kernel<XT, YT, LPR, CPL, NT>;
    cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const dim3 grid((g.rows + kRowsPerCta - 1) / kRowsPerCta);
    fn<<<grid, kMvThreads, smem, s>>>(a.packed, a.scales, a.biases, g, static_cast<const XT*>(a.x),
                                      static_cast<YT*>(a.y), a.batch);
    return cudaGetLastError();
}

template <typename XT, typename YT>
static cudaError_t q4_matvec_launch_t(const Q4MatvecArgs& a, cudaStream_t s) {
    constexpr size_t kSmemLimit = 200 * 1024;
    if (q4_fast_ok(a.cols, a.group, a.packed)) {
        Q4Geom g{a.rows, a.cols, (a.cols + a.group - 1) / a.group, a.cols / 32, ilog2_u32(a.group / 32)};
        const size_t per_tok = (g.cols + 2ull * g.chunks) * sizeof(float);
        const bool multi = a.batch > 1 && 4 * per_tok <= kSmemLimit;
        if (per_tok <= kSmemLimit) {
            if (g.chunks >= 32) {
                return multi ? launch_fast<XT, YT, 32, 2, 4>(a, g, s) : launch_fast<XT, YT, 32, 2, 1>(a, g, s);
            } else if (g.chunks >= 16) {
                return multi ? launch_fast<XT, YT, 16, 1, 4>(a, g, s) : launch_fast<XT, YT, 16, 1, 1>(a, g, s);
            } else if (g.chunks >= 8) {
                return multi ? launch_fast<XT, YT, 8, 1, 4>(a, g, s) : launch_fast<XT, YT, 8, 1, 1>(a, g, s);
            }
        }
    }
    const size_t smem = static_cast<size_t>(a.cols) * sizeof(float);
    if (smem > kSmemLimit) return cudaErrorNotSupported;
    auto fn = q4_matvec_generic_kernel<XT, YT>;
    cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const dim3 grid((a.rows + (kMvThreads / 32) - 1) / (kMvThreads / 32));
    fn<<<grid, kMvThreads, smem, s>>>(a.packed, a.scales, a.biases, a.rows, a.cols, a.group,
                                      static_cast<const XT*>(a.x), static_cast<YT*>(a.y), a.batch);
    return cudaGetLastError();
}

cudaError_t q4_matvec_launch(const Q4MatvecArgs& a, cudaStream_t s) {
    if (a.x_dtype == PBMOE_BF16)
        return a.y_dtype == PBMOE_BF16 ? q4_matvec_launch_t<uint16_t, uint16_t>(a, s)
                                       : q4_matvec_launch_t<uint16_t, float>(a, s);
    return a.y_dtype == PBMOE_BF16 ? q4_matvec_launch_t<float, uint16_t>(a, s) : q4_matvec_launch_t<float, float>(a, s);
}

}  // namespace pbmoe
