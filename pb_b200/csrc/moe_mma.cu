// moe_mma.cu — tensor-core (mma.sync) versions of the MoE expert kernels for
// group-64 Q4 experts (the reference's fixed-Q4 layout, GROUP_SIZE = 64,
// types.rs:35). Same contract as moe_expert_up_kernel / moe_expert_down_kernel
// in moe_decode.cu; see q4_mma.cuh for the arithmetic.
//
//   moe_expert_up_mma_kernel   CTA = 8 warps = one tile of 8 intermediate
//       rows (gate and up) x 8 K-slices of the hidden dimension; the slices
//       are summed in shared memory and SwiGLU is applied (silu(g) * u, as
//       silu_product, shaders.metal:1699-1708).
//   moe_expert_down_mma_kernel CTA = 8 warps, each one tile of 8 down rows
//       over the whole intermediate dimension; the f32 SwiGLU activations are
//       split into bf16 hi + lo rows so the product keeps ~16 mantissa bits.

#include "kernels.h"
#include "q4_mma.cuh"

namespace pbmoe {

constexpr int kMmaThreads = 256;

__host__ __device__ inline size_t up_mma_smem(uint32_t H, bool rows16) {
    return act_tile_bytes(H, rows16 ? 16 : 8) + size_t(8) * 2 * 16 * 8 * 4;
}

__host__ __device__ inline size_t down_mma_smem(uint32_t I) { return act_tile_bytes(I, 16); }

// Variant of stage_act_mma for tiles with only 8 token rows (bf16 input,
// tokens <= 8): same layout, rows 8..15 absent.
template <typename XT>
__device__ void stage_act_rows8(const XT* __restrict__ x, size_t x_stride, const uint32_t* rows_idx, int ntok,
                                uint32_t K, const ActTile& tile) {
    const uint32_t slots = K / 8;
    for (uint32_t i = threadIdx.x; i < 8 * slots; i += blockDim.x)
        if (i / slots >= static_cast<uint32_t>(ntok)) tile.act[(i / slots) * tile.stride + (i % slots)] = make_uint4(0, 0, 0, 0);
    for (uint32_t i = threadIdx.x; i < 8 * tile.groups; i += blockDim.x)
        if (i / tile.groups >= static_cast<uint32_t>(ntok)) tile.gsum[i] = 0.f;
    const uint32_t total = static_cast<uint32_t>(ntok) * slots;
    constexpr int kBatch = 4;
    for (uint32_t base = 0; base < total; base += kBatch * blockDim.x) {
        uint4 v[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const uint32_t idx = base + i * blockDim.x + threadIdx.x;
            if (idx < total) {
                const uint32_t t = idx / slots, w = idx - t * slots;
                const size_t src = rows_idx ? rows_idx[t] : static_cast<size_t>(t);
                v[i] = *reinterpret_cast<const uint4*>(x + src * x_stride + static_cast<size_t>(w) * 8);
            }
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const uint32_t idx = base + i * blockDim.x + threadIdx.x;
            float sum = 0.f;
            uint32_t t = 0, w = 0;
            const bool ok = idx < total;
            if (ok) {
                t = idx / slots;
                w = idx - t * slots;
                const uint4 r = v[i];
                tile.act[t * tile.stride + w] = make_uint4(pack_pairs_lo(r.x, r.z), pack_pairs_hi(r.x, r.z),
                                                                  pack_pairs_lo(r.y, r.w), pack_pairs_hi(r.y, r.w));
                const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) sum += __uint_as_float(rr[q] << 16) + __uint_as_float(rr[q] & 0xffff0000u);
            }
            sum += __shfl_xor_sync(kFull, sum, 1);
            sum += __shfl_xor_sync(kFull, sum, 2);
            sum += __shfl_xor_sync(kFull, sum, 4);
            if (ok && (w & 7u) == 0) tile.gsum[t * tile.groups + (w >> 3)] = sum;
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------- up
// XT: activation type (bf16 bits or f32). kTok16: bf16 with up to 16 tokens
// per pass (rows g+8 carry tokens 8..15). f32 activations use the hi/lo rows
// (8 tokens per pass).
template <typename XT, bool kTok16>
__global__ void __launch_bounds__(kMmaThreads, 2)
moe_expert_up_mma_kernel(const XT* __restrict__ x, uint32_t E, const uint8_t* __restrict__ experts,
                         const uint8_t* __restrict__ shared_slot, MoeLayoutDev L, MoeWs ws) {
    constexpr bool kLo = sizeof(XT) == 4;
    constexpr bool kRows16 = kLo || kTok16;
    constexpr int kPass = kTok16 ? 16 : 8;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t H = L.hidden, I = L.inter;
    const uint32_t rows = kRows16 ? 16 : 8;
    const ActTile tile = act_tile_at(smem_raw, H, rows);
    float* red = reinterpret_cast<float*>(smem_raw + act_tile_bytes(H, rows));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;

    pdl_wait();
    const uint32_t gi = blockIdx.y;
    if (gi >= *ws.num_groups) return;
    const uint32_t e = ws.group_expert[gi];
    const uint32_t start = ws.group_start[gi], n = ws.group_count[gi];
    const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * L.expert_bytes;
    const uint32_t gpr = H / kMmaGroup;
    const uint32_t gps = gpr / 8;  // groups per warp slice, a multiple of 4
    const uint32_t i0 = blockIdx.x * 8;
    const uint8_t* gate_row = slot + L.off[0] + static_cast<size_t>(i0 + g) * (H / 2);
    const uint8_t* up_row = slot + L.off[3] + static_cast<size_t>(i0 + g) * (H / 2);
    const uint16_t* gs = reinterpret_cast<const uint16_t*>(slot + L.off[1]) + static_cast<size_t>(i0 + 2 * t) * gpr;
    const uint16_t* gb = reinterpret_cast<const uint16_t*>(slot + L.off[2]) + static_cast<size_t>(i0 + 2 * t) * gpr;
    const uint16_t* us = reinterpret_cast<const uint16_t*>(slot + L.off[4]) + static_cast<size_t>(i0 + 2 * t) * gpr;
    const uint16_t* ub = reinterpret_cast<const uint16_t*>(slot + L.off[5]) + static_cast<size_t>(i0 + 2 * t) * gpr;
    const uint32_t grp0 = warp * gps;

    Q4MmaFrag4 fg, fu;
    fg.load(gate_row, gs, gb, gpr, grp0, t);  // weights in flight while x is staged
    fu.load(up_row, us, ub, gpr, grp0, t);
    for (uint32_t p0 = 0; p0 < n; p0 += kPass) {
        const int nt = static_cast<int>(min(n - p0, static_cast<uint32_t>(kPass)));
        __syncthreads();
        if (kRows16)
            stage_act_mma<XT, 1>(x, H, ws.group_tokens + start + p0, nt, H, tile);
        else
            stage_act_rows8<XT>(x, H, ws.group_tokens + start + p0, nt, H, tile);
        float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
        for (uint32_t b = 0; b < gps; b += 4) {
            if (b > 0) {
                fg.load(gate_row, gs, gb, gpr, grp0 + b, t);
                fu.load(up_row, us, ub, gpr, grp0 + b, t);
            }
            fg.compute<kLo, kTok16>(tile, grp0 + b, g, t, ag);
            fu.compute<kLo, kTok16>(tile, grp0 + b, g, t, au);
        }
        // red[warp][matrix][token][row]
        float* rw = red + warp * (2 * 16 * 8);
        rw[(0 * 16 + g) * 8 + 2 * t] = ag[0];
        rw[(0 * 16 + g) * 8 + 2 * t + 1] = ag[1];
        rw[(1 * 16 + g) * 8 + 2 * t] = au[0];
        rw[(1 * 16 + g) * 8 + 2 * t + 1] = au[1];
        if (kTok16) {
            rw[(0 * 16 + g + 8) * 8 + 2 * t] = ag[2];
            rw[(0 * 16 + g + 8) * 8 + 2 * t + 1] = ag[3];
            rw[(1 * 16 + g + 8) * 8 + 2 * t] = au[2];
            rw[(1 * 16 + g + 8) * 8 + 2 * t + 1] = au[3];
        }
        __syncthreads();
        if (threadIdx.x < 16 * 8) {
            const uint32_t tok = threadIdx.x >> 3, r = threadIdx.x & 7;
            if (tok < static_cast<uint32_t>(nt)) {
                float gsum = 0.f, usum = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    gsum += red[w * (2 * 16 * 8) + (0 * 16 + tok) * 8 + r];
                    usum += red[w * (2 * 16 * 8) + (1 * 16 + tok) * 8 + r];
                }
                const uint32_t route = ws.group_routes[start + p0 + tok];
                ws.h[static_cast<size_t>(route) * I + i0 + r] = gsum / (1.0f + expf(-gsum)) * usum;
            }
        }
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------- down
__global__ void __launch_bounds__(kMmaThreads, 2)
moe_expert_down_mma_kernel(uint32_t E, const uint8_t* __restrict__ experts, const uint8_t* __restrict__ shared_slot,
                           MoeLayoutDev L, MoeWs ws) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const uint32_t H = L.hidden, I = L.inter;
    const ActTile tile = act_tile_at(smem_raw, I, 16);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    // The group plan comes from the router kernel, which completed before the
    // up kernel began; the down weights do not depend on the up kernel, so
    // they are requested before waiting for it.
    const uint32_t gi = blockIdx.y;
    const uint32_t ng = *ws.num_groups;
    if (gi >= ng) {
        pdl_wait();
        return;
    }
    const uint32_t e = ws.group_expert[gi];
    const uint32_t start = ws.group_start[gi], n = ws.group_count[gi];
    const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * L.expert_bytes;
    const uint32_t gpr = I / kMmaGroup;
    const uint32_t r0 = blockIdx.x * 64 + warp * 8;
    const uint8_t* drow = slot + L.off[6] + static_cast<size_t>(r0 + g) * (I / 2);
    const uint16_t* ds = reinterpret_cast<const uint16_t*>(slot + L.off[7]) + static_cast<size_t>(r0 + 2 * t) * gpr;
    const uint16_t* db = reinterpret_cast<const uint16_t*>(slot + L.off[8]) + static_cast<size_t>(r0 + 2 * t) * gpr;
    Q4MmaFrag4 f0, f1;
    f0.load(drow, ds, db, gpr, 0, t);
    if (gpr > 4) f1.load(drow, ds, db, gpr, 4, t);
    pdl_wait();
    for (uint32_t p0 = 0; p0 < n; p0 += 8) {
        const int nt = static_cast<int>(min(n - p0, 8u));
        __syncthreads();
        stage_act_mma<float, 1>(ws.h, I, ws.group_routes + start + p0, nt, I, tile);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        f0.compute<true, false>(tile, 0, g, t, acc);
        if (gpr > 4) f1.compute<true, false>(tile, 4, g, t, acc);
        if (g < nt) {
            const uint32_t route = ws.group_routes[start + p0 + g];
            float* yr = ws.y + static_cast<size_t>(route) * H + r0 + 2 * t;
            *reinterpret_cast<float2*>(yr) = make_float2(acc[0], acc[1]);
        }
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------- launch
static cudaError_t launch_k(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args,
                            bool pdl) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

bool moe_mma_supported(const MoeLayoutDev& L) {
    // group 64; hidden a multiple of 8*4*64 (eight K-slices of 4-group
    // blocks in the up kernel); intermediate 256 or 512 (one or two 4-group
    // blocks held in registers by the down kernel)
    return !L.mxfp4 && L.group == kMmaGroup && L.hidden % 2048 == 0 && (L.inter == 256 || L.inter == 512) &&
           L.off[0] % 16 == 0 && L.off[3] % 16 == 0 && L.off[6] % 16 == 0 && L.off[1] % 8 == 0 && L.off[2] % 8 == 0 &&
           L.off[4] % 8 == 0 && L.off[5] % 8 == 0 && L.off[7] % 8 == 0 && L.off[8] % 8 == 0 && L.expert_bytes % 16 == 0;
}

cudaError_t moe_up_mma_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    dim3 grid(L.inter / 8, gmax);
    if (a.x_dtype == PBMOE_BF16) {
        const uint16_t* x = static_cast<const uint16_t*>(a.x);
        void* args[] = {(void*)&x, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
        if (a.tokens <= 8)
            return launch_k(reinterpret_cast<const void*>(moe_expert_up_mma_kernel<uint16_t, false>), grid,
                            dim3(kMmaThreads), up_mma_smem(L.hidden, false), s, args, pdl);
        return launch_k(reinterpret_cast<const void*>(moe_expert_up_mma_kernel<uint16_t, true>), grid,
                        dim3(kMmaThreads), up_mma_smem(L.hidden, true), s, args, pdl);
    }
    const float* x = static_cast<const float*>(a.x);
    void* args[] = {(void*)&x, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    return launch_k(reinterpret_cast<const void*>(moe_expert_up_mma_kernel<float, false>), grid, dim3(kMmaThreads),
                    up_mma_smem(L.hidden, true), s, args, pdl);
}

cudaError_t moe_down_mma_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    void* args[] = {(void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    return launch_k(reinterpret_cast<const void*>(moe_expert_down_mma_kernel), dim3(L.hidden / 64, gmax),
                    dim3(kMmaThreads), down_mma_smem(L.inter), s, args, pdl);
}

}  // namespace pbmoe
