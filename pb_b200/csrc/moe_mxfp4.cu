// moe_mxfp4.cu — expert kernels of the MoE decode layer for
// FIXED_MXFP4_EXPERT_LAYER_V1 slots (QwenMoeQ4ExpertLayout::fixed_mxfp4,
// model_family.rs:846-952: per projection the E2M1 nibbles [rows x cols/2],
// then one E8M0 byte per 32 columns, no biases). The reference runs these
// experts through mxfp4_fma_matvec_with_group_size (experts/slots.rs:
// 1239-1287) and the Metal mxfp4_fma_matvec_e8m0 (shaders.metal:200-298);
// SwiGLU is silu(g) * u (shaders.metal:1699-1708).
//
// They replace kernels 2 and 3 of the Q4 layer (router, plan and combine are
// shared): the router kernel's plan lists, per expert group, the grouped
// positions of its routes; gate/up rows write f32 SwiGLU activations to
// ws.h[route], down rows write ws.y[route].
//
// Both are HBM-bound CUDA-core matvecs over 4.25-bit weights: a lane owns
// 32-column groups (16 weight bytes + 1 scale byte), decodes nibbles through
// the fp16 exponent field (mxfp4.cuh) and multiplies against activations
// staged once per CTA in shared memory (padded 36 floats per group so that
// lanes reading consecutive groups hit different banks).

#include "kernels.h"
#include "mxfp4.cuh"

namespace pbmoe {

namespace {

constexpr int kMxUpThreads = 128;
constexpr int kMxUpRows = 2;  // intermediate indices per warp: gate + up = 4 weight rows
constexpr int kMxUpRowsPerCta = kMxUpRows * (kMxUpThreads / 32);
constexpr int kMxDownThreads = 128;
constexpr int kMxDownRows = 4;  // hidden rows per lane group

// x rows of `nt` grouped positions into xs[NT][pcols] (zeros past nt)
template <typename XT, int NT>
__device__ __forceinline__ void mx_stage(const XT* __restrict__ x, uint32_t cols, const uint32_t* rows_of, int nt,
                                         float* xs) {
    const uint32_t pcols = mx_padded_cols(cols);
    for (uint32_t i = threadIdx.x; i < NT * cols; i += blockDim.x) {
        const uint32_t t = i / cols, c = i - t * cols;
        xs[t * pcols + c + (c >> 5) * 4] =
            static_cast<int>(t) < nt ? load_act<XT>(x, static_cast<size_t>(rows_of[t]) * cols + c) : 0.f;
    }
}

template <typename XT, int NT>
__global__ void __launch_bounds__(kMxUpThreads)
moe_mx_up_kernel(const XT* __restrict__ x, uint32_t E, const uint8_t* __restrict__ experts,
                 const uint8_t* __restrict__ shared_slot, MoeLayoutDev L, MoeWs ws) {
    extern __shared__ __align__(16) float xs[];
    const uint32_t g = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_wait();
    if (g >= *ws.num_groups) return;
    const uint32_t e = ws.group_expert[g];
    const uint32_t start = ws.group_start[g], n = ws.group_count[g];
    const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * L.expert_bytes;
    const uint32_t H = L.hidden, I = L.inter, groups = H >> 5, pcols = mx_padded_cols(H);
    const uint32_t i0 = blockIdx.x * kMxUpRowsPerCta + warp * kMxUpRows;
    // rows 0..kMxUpRows-1 gate, then up; rows past I read row I-1 and are dropped
    const uint8_t* wp[2 * kMxUpRows];
    const uint8_t* sp[2 * kMxUpRows];
#pragma unroll
    for (int r = 0; r < kMxUpRows; ++r) {
        const uint32_t i = min(i0 + r, I - 1);
        wp[r] = slot + L.off[0] + static_cast<size_t>(i) * (H / 2);
        sp[r] = slot + L.off[1] + static_cast<size_t>(i) * groups;
        wp[kMxUpRows + r] = slot + L.off[3] + static_cast<size_t>(i) * (H / 2);
        sp[kMxUpRows + r] = slot + L.off[4] + static_cast<size_t>(i) * groups;
    }
    for (uint32_t p0 = 0; p0 < n; p0 += NT) {
        const int nt = static_cast<int>(min(n - p0, static_cast<uint32_t>(NT)));
        __syncthreads();
        mx_stage<XT, NT>(x, H, ws.group_tokens + start + p0, nt, xs);
        __syncthreads();
        float acc[2 * kMxUpRows][NT];
#pragma unroll
        for (int r = 0; r < 2 * kMxUpRows; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
#pragma unroll 2
        for (uint32_t c = lane; c < groups; c += 32) {
            uint4 w[2 * kMxUpRows];
            uint32_t sb[2 * kMxUpRows];
#pragma unroll
            for (int r = 0; r < 2 * kMxUpRows; ++r) {
                w[r] = ld_stream_u4(wp[r] + static_cast<size_t>(c) * 16);
                sb[r] = sp[r][c];
            }
#pragma unroll
            for (int r = 0; r < 2 * kMxUpRows; ++r) {
                if (sb[r] == 255u) atomicOr(ws.status, PBMOE_DEV_ERR_MXFP4_SCALE);
                float part[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) part[t] = 0.f;
                mx_group_dot<NT>(w[r], xs + c * 36, pcols, part);
                const float scale = e8m0_scale(sb[r]);
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[r][t] += (part[t] * 16384.0f) * scale;
            }
        }
#pragma unroll
        for (int r = 0; r < kMxUpRows; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float gs = warp_sum(acc[r][t]);
                const float us = warp_sum(acc[kMxUpRows + r][t]);
                if (lane == 0 && t < nt && i0 + r < I) {
                    const uint32_t route = ws.group_routes[start + p0 + t];
                    ws.h[static_cast<size_t>(route) * I + i0 + r] = gs / (1.0f + expf(-gs)) * us;
                }
            }
        }
    }
    pdl_launch_dependents();
}

// LPR lanes per hidden row (I/32 groups spread over them), 32/LPR rows per
// warp pass times kMxDownRows
template <int LPR, int NT>
__global__ void __launch_bounds__(kMxDownThreads)
moe_mx_down_kernel(uint32_t E, const uint8_t* __restrict__ experts, const uint8_t* __restrict__ shared_slot,
                   MoeLayoutDev L, MoeWs ws) {
    extern __shared__ __align__(16) float xs[];
    constexpr int kLaneGroups = 32 / LPR;
    constexpr int kRowsPerCta = kMxDownRows * kLaneGroups * (kMxDownThreads / 32);
    const uint32_t g = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane / LPR, sl = lane & (LPR - 1);
    const uint32_t H = L.hidden, I = L.inter, groups = I >> 5, pcols = mx_padded_cols(I);
    // the plan was written by the router kernel, which finished before the
    // gate/up kernel started
    const uint32_t ng = *ws.num_groups;
    if (g >= ng) {
        pdl_wait();
        return;
    }
    const uint32_t e = ws.group_expert[g];
    const uint32_t start = ws.group_start[g], n = ws.group_count[g];
    const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * L.expert_bytes;
    const uint32_t r0 = blockIdx.x * kRowsPerCta + (warp * kLaneGroups + sub) * kMxDownRows;
    const uint8_t* wp[kMxDownRows];
    const uint8_t* sp[kMxDownRows];
#pragma unroll
    for (int r = 0; r < kMxDownRows; ++r) {
        const uint32_t row = min(r0 + r, H - 1);
        wp[r] = slot + L.off[6] + static_cast<size_t>(row) * (I / 2);
        sp[r] = slot + L.off[7] + static_cast<size_t>(row) * groups;
    }
    pdl_wait();
    for (uint32_t p0 = 0; p0 < n; p0 += NT) {
        const int nt = static_cast<int>(min(n - p0, static_cast<uint32_t>(NT)));
        __syncthreads();
        mx_stage<float, NT>(ws.h, I, ws.group_routes + start + p0, nt, xs);
        __syncthreads();
        float acc[kMxDownRows][NT];
#pragma unroll
        for (int r = 0; r < kMxDownRows; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        for (uint32_t c = sl; c < groups; c += LPR) {
            uint4 w[kMxDownRows];
            uint32_t sb[kMxDownRows];
#pragma unroll
            for (int r = 0; r < kMxDownRows; ++r) {
                w[r] = ld_stream_u4(wp[r] + static_cast<size_t>(c) * 16);
                sb[r] = sp[r][c];
            }
#pragma unroll
            for (int r = 0; r < kMxDownRows; ++r) {
                if (sb[r] == 255u) atomicOr(ws.status, PBMOE_DEV_ERR_MXFP4_SCALE);
                float part[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) part[t] = 0.f;
                mx_group_dot<NT>(w[r], xs + c * 36, pcols, part);
                const float scale = e8m0_scale(sb[r]);
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[r][t] += (part[t] * 16384.0f) * scale;
            }
        }
#pragma unroll
        for (int r = 0; r < kMxDownRows; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float s = group_sum<LPR>(acc[r][t]);
                if (sl == 0 && t < nt && r0 + r < H) {
                    const uint32_t route = ws.group_routes[start + p0 + t];
                    ws.y[static_cast<size_t>(route) * H + r0 + r] = s;
                }
            }
        }
    }
    pdl_launch_dependents();
}

template <typename F>
cudaError_t mx_smem(F* fn, size_t bytes) {
    return cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bytes));
}

template <typename XT>
cudaError_t mx_up(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    const XT* x = static_cast<const XT*>(a.x);
    void* args[] = {(void*)&x, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    const dim3 grid((L.inter + kMxUpRowsPerCta - 1) / kMxUpRowsPerCta, gmax);
    cudaError_t err;
    if (a.tokens == 1) {
        const size_t smem = size_t(mx_padded_cols(L.hidden)) * sizeof(float);
        if ((err = mx_smem(moe_mx_up_kernel<XT, 1>, smem)) != cudaSuccess) return err;
        return moe_launch_pdl(reinterpret_cast<const void*>(moe_mx_up_kernel<XT, 1>), grid, dim3(kMxUpThreads), smem,
                              s, args, pdl);
    }
    const size_t smem = 4 * size_t(mx_padded_cols(L.hidden)) * sizeof(float);
    if ((err = mx_smem(moe_mx_up_kernel<XT, 4>, smem)) != cudaSuccess) return err;
    return moe_launch_pdl(reinterpret_cast<const void*>(moe_mx_up_kernel<XT, 4>), grid, dim3(kMxUpThreads), smem, s,
                          args, pdl);
}

template <int LPR>
cudaError_t mx_down(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    void* args[] = {(void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    constexpr uint32_t rows_per_cta = kMxDownRows * (32 / LPR) * (kMxDownThreads / 32);
    const dim3 grid((L.hidden + rows_per_cta - 1) / rows_per_cta, gmax);
    cudaError_t err;
    if (a.tokens == 1) {
        const size_t smem = size_t(mx_padded_cols(L.inter)) * sizeof(float);
        if ((err = mx_smem(moe_mx_down_kernel<LPR, 1>, smem)) != cudaSuccess) return err;
        return moe_launch_pdl(reinterpret_cast<const void*>(moe_mx_down_kernel<LPR, 1>), grid, dim3(kMxDownThreads),
                              smem, s, args, pdl);
    }
    const size_t smem = 4 * size_t(mx_padded_cols(L.inter)) * sizeof(float);
    if ((err = mx_smem(moe_mx_down_kernel<LPR, 4>, smem)) != cudaSuccess) return err;
    return moe_launch_pdl(reinterpret_cast<const void*>(moe_mx_down_kernel<LPR, 4>), grid, dim3(kMxDownThreads),
                          smem, s, args, pdl);
}

}  // namespace

cudaError_t moe_up_mxfp4_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    return a.x_dtype == PBMOE_BF16 ? mx_up<uint16_t>(a, gmax, s, pdl) : mx_up<float>(a, gmax, s, pdl);
}

cudaError_t moe_down_mxfp4_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    const uint32_t groups = a.layout.inter / 32;  // lanes per row: no more than the row's groups
    return groups >= 32 ? mx_down<32>(a, gmax, s, pdl)
           : groups >= 16 ? mx_down<16>(a, gmax, s, pdl)
           : groups >= 8  ? mx_down<8>(a, gmax, s, pdl)
                          : mx_down<4>(a, gmax, s, pdl);
}

}  // namespace pbmoe
