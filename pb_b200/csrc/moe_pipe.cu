// moe_pipe.cu — persistent, asynchronously pipelined MoE expert kernels for
// decode batches of at most 8 tokens (group-64 Q4 experts).
//
// Each CTA (8 warps) walks a strided list of work items. The bytes of each
// item are moved into one of several shared-memory stages by 16-byte
// cp.async copies that every thread of the CTA issues a share of, and each
// thread's completion is counted on the stage's mbarrier; after the item's
// compute the CTA synchronises once, refills the stage it just released with
// the item `stages` ahead, and runs the item's epilogue. Several items' bytes
// are therefore always in flight per SM while the tensor cores (mma.sync,
// q4_mma.cuh) consume the current one. Rows land in padded shared rows so
// fragment loads are bank-conflict free.
//
//   moe_up_pipe_kernel    item = (group, 8 intermediate rows): gate and up
//       rows + their scales/biases; the batch's tokens stay resident in shared
//       memory for the whole kernel. 8 warps = 8 K-slices, summed in shared
//       memory; SwiGLU (silu(g)*u, shaders.metal:1699-1708) is written as bf16
//       hi/lo pair slots + per-8 partial sums (MoeWs::h_perm), the down
//       kernel's input layout, by one warp per routed token of the group.
//   moe_down_pipe_kernel  item = (group, 64 down rows): rows, scales, and the
//       group's routes' h_perm rows; warp w owns rows 8w..8w+7. Weights of the
//       first stages are requested before the programmatic-dependent-launch
//       wait (they do not depend on the up kernel).
//
// Every mbarrier wait is bounded (kPipeWaitNs); on expiry the kernel latches
// PBMOE_DEV_ERR_PIPE_TIMEOUT, waits for its own copies, and returns.

#include "kernels.h"
#include "pipe.cuh"
#include "q4_mma.cuh"

namespace pbmoe {

// Stage counts: bf16 activations run two CTAs per SM (3 stages each, 16 warps
// per SM); f32 activations keep a 16-row token tile and run one CTA per SM.
constexpr int kUpStagesBf16 = 3;
constexpr int kUpStagesF32 = 5;
constexpr int kDownStages = 2;
template <typename XT>
struct UpCfg {
    static constexpr int kStages = sizeof(XT) == 4 ? kUpStagesF32 : kUpStagesBf16;
    static constexpr int kCtasPerSm = sizeof(XT) == 4 ? 1 : 2;
};

static int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

// The layer-major group plan (written by the router kernel) copied into
// shared memory once per CTA, so that per-item lookups are shared-memory
// loads instead of dependent L2 round trips. `cap_g` groups and `cap_r`
// grouped positions fit (host-checked: T*K + 1 and T*K + T).
struct PlanSmem {
    uint32_t* expert;  // [cap_g]
    uint32_t* start;   // [cap_g]
    uint32_t* count;   // [cap_g]
    uint32_t* token;   // [cap_r]
    uint32_t* route;   // [cap_r]
};

__host__ __device__ inline size_t plan_smem_bytes(uint32_t cap_g, uint32_t cap_r) {
    return (size_t(3) * cap_g + size_t(2) * cap_r) * 4;
}

__device__ inline PlanSmem plan_at(void* base, uint32_t cap_g, uint32_t cap_r) {
    uint32_t* p = reinterpret_cast<uint32_t*>(base);
    return {p, p + cap_g, p + 2 * cap_g, p + 3 * cap_g, p + 3 * cap_g + cap_r};
}

// All threads: copy the plan (ng groups, positions 0..npos) through L2.
__device__ inline void load_plan(const MoeWs& ws, uint32_t ng, uint32_t npos, const PlanSmem& pl) {
    for (uint32_t i = threadIdx.x; i < ng; i += blockDim.x) {
        pl.expert[i] = __ldcg(ws.group_expert + i);
        pl.start[i] = __ldcg(ws.group_start + i);
        pl.count[i] = __ldcg(ws.group_count + i);
    }
    for (uint32_t i = threadIdx.x; i < npos; i += blockDim.x) {
        pl.token[i] = __ldcg(ws.group_tokens + i);
        pl.route[i] = __ldcg(ws.group_routes + i);
    }
}

// ---------------------------------------------------------------- layouts
struct UpStage {
    uint32_t rs;     // padded row stride (bytes) = H/2 + 32
    uint32_t gate, up, gs, gb, us, ub;
    uint32_t bytes;  // stage size, multiple of 128
};

__host__ __device__ inline UpStage up_stage(uint32_t H) {
    UpStage L;
    L.rs = H / 2 + 32;
    const uint32_t sb = 8 * (H / 32);  // 8 rows of H/64 bf16
    L.gate = 0;
    L.up = 8 * L.rs;
    L.gs = 16 * L.rs;
    L.gb = L.gs + sb;
    L.us = L.gb + sb;
    L.ub = L.us + sb;
    L.bytes = (L.ub + sb + 127) / 128 * 128;
    return L;
}

__host__ __device__ inline size_t up_pipe_smem(uint32_t H, bool lo, uint32_t cap_g, uint32_t cap_r) {
    const UpStage L = up_stage(H);
    const int stages = lo ? kUpStagesF32 : kUpStagesBf16;
    // stages, token tile, 2 x 8 warps x 128 partial sums, flags, mbarriers, plan
    return size_t(stages) * L.bytes + act_tile_bytes(H, lo ? 16 : 8) + 2 * 8 * 128 * 4 + 16 + stages * 8 +
           plan_smem_bytes(cap_g, cap_r);
}

struct DownStage {
    uint32_t rs;  // padded row stride = I/2 + 32
    uint32_t w, s, b, act, part;
    uint32_t part_stride;  // padded stride of the per-route partial-sum rows
    uint32_t bytes;
};

__host__ __device__ inline DownStage down_stage(uint32_t I) {
    DownStage L;
    L.rs = I / 2 + 32;
    const uint32_t sb = 64 * (I / 32);  // 64 rows of I/64 bf16
    L.w = 0;
    L.s = 64 * L.rs;
    L.b = L.s + sb;
    L.act = (L.b + sb + 127) / 128 * 128;
    L.part = L.act + static_cast<uint32_t>(act_tile_bytes(I, 16));
    L.part = (L.part + 15) / 16 * 16;
    L.part_stride = (I / 8) * 4 + 32;
    L.bytes = (L.part + 8 * L.part_stride + 127) / 128 * 128;
    return L;
}

__host__ __device__ inline size_t down_pipe_smem(uint32_t I, uint32_t cap_g, uint32_t cap_r) {
    return size_t(kDownStages) * down_stage(I).bytes + 16 + kDownStages * 8 + plan_smem_bytes(cap_g, cap_r);
}

// Warp roles: warps 0..7 compute; warp 8 ("producer") only issues copies.
// A thread's cp.async may stall at issue until the SM's request queue has
// room, so the producer spends most of its time blocked there, keeping the
// queue full, while no compute warp ever waits behind a copy it issued.
// Handshakes: stage s is full when its mbarrier has the producer's 32 lane
// arrivals (cp.async completion); compute warps release it with
// bar.arrive EMPTY(s), on which the producer bar.syncs before refilling. An
// arrival is made only for items whose stage the producer refills, so the
// two sides always match.
constexpr uint32_t kPipeH = 2048, kPipeI = 512;
constexpr int kWarps = 8;
constexpr int kPipeThreads = (kWarps + 1) * 32;
constexpr int kComputeThreads = kWarps * 32;
constexpr int kBarCompute = 1;                                        // compute warps only
__device__ __forceinline__ int bar_empty(int s) { return 2 + s; }  // ids 2..6

// ---------------------------------------------------------------- up
template <typename XT, uint32_t H, uint32_t I>
__global__ void __launch_bounds__(kPipeThreads, UpCfg<XT>::kCtasPerSm)
moe_up_pipe_kernel(const XT* __restrict__ x, uint32_t T, uint32_t E, const uint8_t* __restrict__ experts,
                   const uint8_t* __restrict__ shared_slot, MoeLayoutDev Ld, MoeWs ws, uint32_t cap_g,
                   uint32_t cap_r) {
    constexpr bool kLo = sizeof(XT) == 4;
    constexpr int kUpStages = UpCfg<XT>::kStages;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const UpStage SL = up_stage(H);
    unsigned char* stages = smem_raw;
    const ActTile tile = act_tile_at(stages + kUpStages * SL.bytes, H, kLo ? 16 : 8);
    // partial sums: [2 buffers][8 warps][gate 64 | up 64], entry tok*8 + row
    float* red = reinterpret_cast<float*>(stages + kUpStages * SL.bytes + act_tile_bytes(H, kLo ? 16 : 8));
    uint32_t* flags = reinterpret_cast<uint32_t*>(red + 2 * kWarps * 128);  // [0] error
    uint64_t* bar = reinterpret_cast<uint64_t*>(flags + 4);
    const PlanSmem pl = plan_at(bar + kUpStages, cap_g, cap_r);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    constexpr uint32_t tiles = I / 8;
    constexpr uint32_t gpr = H / kMmaGroup;
    constexpr uint32_t gps = gpr / kWarps;  // groups per warp K-slice (multiple of 4)
    const size_t hps = hperm_stride(I);

    pdl_wait();
    const uint32_t ng = min(__ldcg(ws.num_groups), cap_g);
    const uint32_t total = ng * tiles;
    // a contiguous run of items per CTA: consecutive tiles of one expert
    const uint32_t k0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * total / gridDim.x);
    const uint32_t k1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * total / gridDim.x);
    if (k0 >= k1) return;
    const uint32_t my_items = k1 - k0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kUpStages; ++s) mbar_init(&bar[s], 32);  // the producer's lanes
        flags[0] = 0;
        fence_mbar_init();
    }
    load_plan(ws, ng, cap_r, pl);
    __syncthreads();

    if (warp == kWarps) {
        // producer: 16-byte copies of the 8 gate rows, the 8 up rows and the
        // four 8-row scale/bias blocks of item k into stage s, then each
        // lane's completion arrival. The 8 rows of a matrix are contiguous in
        // the slot; warp iteration i copies bytes 512i..512i+511 of them, so
        // every copy address is a per-lane base plus a constant.
        constexpr uint32_t kRowBytes = H / 2;
        constexpr uint32_t kIters = 8 * kRowBytes / 512;
        constexpr uint32_t kScaleBlock = 8 * (H / 32);  // one 8-row block of H/64 bf16 per row
        static_assert(kRowBytes % 512 == 0 && kScaleBlock == 512, "row and block shapes");
        auto issue = [&](uint32_t k, int s) {
            const uint32_t gi = k / tiles, i0 = (k % tiles) * 8;
            const uint32_t e = pl.expert[gi];
            const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * Ld.expert_bytes;
            unsigned char* st = stages + s * SL.bytes + lane * 16;
            const uint8_t* gsrc = slot + Ld.off[0] + static_cast<size_t>(i0) * kRowBytes + lane * 16;
            const uint8_t* usrc = slot + Ld.off[3] + static_cast<size_t>(i0) * kRowBytes + lane * 16;
#pragma unroll
            for (uint32_t i = 0; i < kIters; ++i) {
                const uint32_t d = (i * 512) / kRowBytes * SL.rs + (i * 512) % kRowBytes;
                cp_async16(st + SL.gate + d, gsrc + i * 512);
                cp_async16(st + SL.up + d, usrc + i * 512);
            }
            const size_t so = static_cast<size_t>(i0) * (H / 32) + lane * 16;
            cp_async16(st + SL.gs, slot + Ld.off[1] + so);
            cp_async16(st + SL.gb, slot + Ld.off[2] + so);
            cp_async16(st + SL.us, slot + Ld.off[4] + so);
            cp_async16(st + SL.ub, slot + Ld.off[5] + so);
            cp_async_arrive(&bar[s]);
        };
        for (int j = 0; j < kUpStages && static_cast<uint32_t>(j) < my_items; ++j) issue(k0 + j, j);
        for (uint32_t j = 0; j + kUpStages < my_items; ++j) {
            const int s = static_cast<int>(j % kUpStages);
            named_sync(bar_empty(s), kPipeThreads);  // every compute warp has released item j's stage
            if (*reinterpret_cast<volatile uint32_t*>(&flags[0])) break;
            issue(k0 + j + kUpStages, s);
        }
        cp_async_wait_all();  // no copy of this CTA outlives it
        return;
    }

    // compute warps: the batch's tokens stay resident for the whole kernel
    if constexpr (kLo)
        stage_act_mma<XT>(x, H, nullptr, static_cast<int>(T), H, tile, kBarCompute, kComputeThreads);
    else
        stage_act_rows8_tok<XT>(x, H, static_cast<int>(T), H, tile, kBarCompute, kComputeThreads);
    // Every CTA of this grid is resident, so the down kernel may be scheduled
    // now: its CTAs take SMs as these exit and prefetch weights while the
    // rest of this grid finishes (it waits for all of it before reading h_perm).
    pdl_launch_dependents();

    const uint32_t grp0 = warp * gps;
    for (uint32_t j = 0; j < my_items; ++j) {
        const int s = static_cast<int>(j % kUpStages);
        const int p = static_cast<int>(j & 1u);
        const uint32_t k = k0 + j;
        const bool ok = mbar_wait_bounded(&bar[s], (j / kUpStages) & 1u, kPipeWaitNs);
        float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
            const unsigned char* st = stages + s * SL.bytes;
            const uint16_t* gs = reinterpret_cast<const uint16_t*>(st + SL.gs) + (2 * t) * gpr;
            const uint16_t* gb = reinterpret_cast<const uint16_t*>(st + SL.gb) + (2 * t) * gpr;
            const uint16_t* us = reinterpret_cast<const uint16_t*>(st + SL.us) + (2 * t) * gpr;
            const uint16_t* ub = reinterpret_cast<const uint16_t*>(st + SL.ub) + (2 * t) * gpr;
            for (uint32_t b = 0; b < gps; b += 4) {
                Q4MmaFrag4 fg, fu;
                fg.load_smem(st + SL.gate + g * SL.rs, gs, gb, gpr, grp0 + b, t);
                fu.load_smem(st + SL.up + g * SL.rs, us, ub, gpr, grp0 + b, t);
                q4_mma_pair<kLo>(fg, fu, tile, grp0 + b, g, t, ag, au);
            }
        } else if (lane == 0) {
            atomicOr(&flags[0], 1u);
        }
        if (j + kUpStages < my_items) named_arrive(bar_empty(s), kPipeThreads);  // stage s released
        float* rw = red + (p * kWarps + warp) * 128;
        *reinterpret_cast<float2*>(rw + g * 8 + 2 * t) = make_float2(ag[0], ag[1]);
        *reinterpret_cast<float2*>(rw + 64 + g * 8 + 2 * t) = make_float2(au[0], au[1]);
        // red[p] complete and the error flag visible. Item j+2 overwrites
        // red[p] only after the next such barrier, which every warp reaches
        // after this item's epilogue.
        named_sync(kBarCompute, kComputeThreads);
        if (*reinterpret_cast<volatile uint32_t*>(&flags[0])) {
            if (threadIdx.x == 0) latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
            break;
        }

        // epilogue: the group's q-th route (token) of this tile is finished by
        // warp (q + j) mod 8, so the work rotates over the warps
        const uint32_t gi = k / tiles, ti = k % tiles;
        const uint32_t n = pl.count[gi];
        const uint32_t q = (static_cast<uint32_t>(warp) + kWarps - (j & (kWarps - 1))) & (kWarps - 1);
        if (q < n) {
            const uint32_t pos = pl.start[gi] + q;
            const uint32_t tok = pl.token[pos];
            const float* rb = red + p * kWarps * 128;
            // lane: row = lane/4 sums the partials of K-slices 2(lane%4), 2(lane%4)+1
            const int row = lane >> 2, sl = lane & 3;
            const float* r0 = rb + (2 * sl) * 128 + tok * 8 + row;
            float gsum = r0[0] + r0[128];
            float usum = r0[64] + r0[128 + 64];
            gsum += __shfl_xor_sync(kFull, gsum, 1);
            gsum += __shfl_xor_sync(kFull, gsum, 2);
            usum += __shfl_xor_sync(kFull, usum, 1);
            usum += __shfl_xor_sync(kFull, usum, 2);
            const float h = gsum / (1.0f + expf(-gsum)) * usum;  // the four lanes of a row agree
            // pair word c = (h_c, h_{c+4}) is formed in lane 4c from lane 4c+16
            const float h4 = __shfl_down_sync(kFull, h, 16);
            float part = h;
            part += __shfl_xor_sync(kFull, part, 4);
            part += __shfl_xor_sync(kFull, part, 8);
            part += __shfl_xor_sync(kFull, part, 16);
            uint8_t* hr = ws.h_perm + static_cast<size_t>(pl.route[pos]) * hps;
            if (lane < 16 && sl == 0) {
                const uint32_t c = lane >> 2;
                const uint32_t hi = f2_to_bf16x2(h, h4);
                const uint32_t lo = f2_to_bf16x2(h - __uint_as_float(hi << 16), h4 - __uint_as_float(hi & 0xffff0000u));
                reinterpret_cast<uint32_t*>(hr)[ti * 4 + c] = hi;
                reinterpret_cast<uint32_t*>(hr + tiles * 16)[ti * 4 + c] = lo;
            }
            if (lane == 0) reinterpret_cast<float*>(hr + 2 * tiles * 16)[ti] = part;
        }
    }
}

// ---------------------------------------------------------------- down
template <uint32_t H, uint32_t I>
__global__ void __launch_bounds__(kPipeThreads, 2)
moe_down_pipe_kernel(uint32_t E, const uint8_t* __restrict__ experts, const uint8_t* __restrict__ shared_slot,
                     MoeLayoutDev Ld, MoeWs ws, uint32_t cap_g, uint32_t cap_r) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const DownStage SL = down_stage(I);
    unsigned char* stages = smem_raw;
    uint32_t* flags = reinterpret_cast<uint32_t*>(stages + kDownStages * SL.bytes);
    uint64_t* bar = reinterpret_cast<uint64_t*>(flags + 4);
    const PlanSmem pl = plan_at(bar + kDownStages, cap_g, cap_r);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    constexpr uint32_t tiles = H / 64;
    constexpr uint32_t gpr = I / kMmaGroup;
    constexpr uint32_t wslots = I / 8;
    const size_t hps = hperm_stride(I);

    // The group plan was written by the router kernel, which completed before
    // the up kernel passed its own wait; it is safe to read before this
    // kernel's wait (through L2).
    const uint32_t ng = min(__ldcg(ws.num_groups), cap_g);
    const uint32_t total = ng * tiles;
    // a contiguous run of items per CTA (consecutive tiles of one expert)
    const uint32_t k0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * total / gridDim.x);
    const uint32_t k1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * total / gridDim.x);
    if (k0 >= k1) {
        pdl_wait();
        return;
    }
    const uint32_t my_items = k1 - k0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kDownStages; ++s) mbar_init(&bar[s], 32);  // the producer's lanes
        flags[0] = 0;
        fence_mbar_init();
    }
    load_plan(ws, ng, cap_r, pl);
    __syncthreads();

    if (warp == kWarps) {
        // producer: item k's 64 weight rows (contiguous in the slot; warp
        // iteration i copies rows 2i, 2i+1) and scale/bias blocks ...
        constexpr uint32_t kRowBytes = I / 2;
        static_assert(kRowBytes == 256, "two rows per 512-byte warp copy");
        constexpr uint32_t kScaleBytes = 64 * (I / 32);
        auto issue_weights = [&](uint32_t k, int s) {
            const uint32_t gi = k / tiles, r0 = (k % tiles) * 64;
            const uint32_t e = pl.expert[gi];
            const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * Ld.expert_bytes;
            unsigned char* st = stages + s * SL.bytes;
            const uint8_t* wsrc = slot + Ld.off[6] + static_cast<size_t>(r0) * kRowBytes + lane * 16;
            unsigned char* wdst = st + SL.w + (lane >> 4) * SL.rs + (lane & 15) * 16;
#pragma unroll
            for (uint32_t i = 0; i < 32; ++i) cp_async16(wdst + 2 * i * SL.rs, wsrc + i * 512);
            const size_t so = static_cast<size_t>(r0) * (I / 32) + lane * 16;
#pragma unroll
            for (uint32_t c = 0; c < kScaleBytes; c += 512) {
                cp_async16(st + SL.s + lane * 16 + c, slot + Ld.off[7] + so + c);
                cp_async16(st + SL.b + lane * 16 + c, slot + Ld.off[8] + so + c);
            }
        };
        // ... and the group's routed activations: hi and lo bf16 rows of h
        // (pair order) and the per-8 partial sums of each route
        auto issue_h = [&](uint32_t k, int s) {
            const uint32_t gi = k / tiles;
            const uint32_t start = pl.start[gi], n = pl.count[gi];
            unsigned char* st = stages + s * SL.bytes;
            const ActTile tile = act_tile_at(st + SL.act, I, 16);
            for (uint32_t p = 0; p < n; ++p) {
                const uint8_t* hr = ws.h_perm + static_cast<size_t>(pl.route[start + p]) * hps + lane * 16;
#pragma unroll
                for (uint32_t c = 0; c < wslots; c += 32) {
                    cp_async16(tile.act + p * tile.stride + c + lane, hr + c * 16);
                    cp_async16(tile.act + (p + 8) * tile.stride + c + lane, hr + (wslots + c) * 16);
                }
                if (lane < wslots / 4)
                    cp_async16(st + SL.part + p * SL.part_stride + lane * 16, hr + 2 * wslots * 16);
            }
        };
        for (int j = 0; j < kDownStages && static_cast<uint32_t>(j) < my_items; ++j) issue_weights(k0 + j, j);
        pdl_wait();  // h_perm comes from the up kernel
        for (int j = 0; j < kDownStages && static_cast<uint32_t>(j) < my_items; ++j) {
            issue_h(k0 + j, j);
            cp_async_arrive(&bar[j]);
        }
        for (uint32_t j = 0; j + kDownStages < my_items; ++j) {
            const int s = static_cast<int>(j % kDownStages);
            named_sync(bar_empty(s), kPipeThreads);  // every compute warp has released item j's stage
            if (*reinterpret_cast<volatile uint32_t*>(&flags[0])) break;
            issue_weights(k0 + j + kDownStages, s);
            issue_h(k0 + j + kDownStages, s);
            cp_async_arrive(&bar[s]);
        }
        cp_async_wait_all();  // no copy of this CTA outlives it
        return;
    }

    pdl_wait();
    pdl_launch_dependents();  // the combine kernel waits for this whole grid
    const uint32_t rw0 = warp * 8;  // this warp's 8 rows within the 64-row tile
    for (uint32_t j = 0; j < my_items; ++j) {
        const int s = static_cast<int>(j % kDownStages);
        const uint32_t k = k0 + j;
        const bool ok = mbar_wait_bounded(&bar[s], (j / kDownStages) & 1u, kPipeWaitNs);
        if (ok) {
            const uint32_t gi = k / tiles, r0 = (k % tiles) * 64;
            const uint32_t start = pl.start[gi], n = pl.count[gi];
            const unsigned char* st = stages + s * SL.bytes;
            const ActTile tile = act_tile_at(const_cast<unsigned char*>(st) + SL.act, I, 16);
            const uint16_t* ds = reinterpret_cast<const uint16_t*>(st + SL.s) + (rw0 + 2 * t) * gpr;
            const uint16_t* db = reinterpret_cast<const uint16_t*>(st + SL.b) + (rw0 + 2 * t) * gpr;
            const float* prow = reinterpret_cast<const float*>(st + SL.part + g * SL.part_stride);
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (uint32_t b = 0; b < gpr; b += 4) {
                // route g's activation sums of groups b..b+3: each lane adds two of the
                // eight per-8 partials of a group, the quad finishes the sum
                float X[4], X2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const float2 pv = *reinterpret_cast<const float2*>(prow + (b + jj) * 8 + 2 * t);
                    float v = pv.x + pv.y;
                    v += __shfl_xor_sync(kFull, v, 1);
                    v += __shfl_xor_sync(kFull, v, 2);
                    X[jj] = v;
                }
                Q4MmaFrag4 f;
                f.load_smem(st + SL.w + (rw0 + g) * SL.rs, ds, db, gpr, b, t);
                f.compute_x<true, false>(tile, b, g, t, X, X2, acc);
            }
            if (j + kDownStages < my_items) named_arrive(bar_empty(s), kPipeThreads);  // stage s released
            if (static_cast<uint32_t>(g) < n) {
                const uint32_t route = pl.route[start + g];
                *reinterpret_cast<float2*>(ws.y + static_cast<size_t>(route) * H + r0 + rw0 + 2 * t) =
                    make_float2(acc[0], acc[1]);
            }
        } else {
            // the producer stops at this item (it reads the flag after the release)
            if (lane == 0) {
                atomicOr(&flags[0], 1u);
                latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
            }
            __syncwarp();
            if (j + kDownStages < my_items) named_arrive(bar_empty(s), kPipeThreads);
            break;
        }
    }
}

// ---------------------------------------------------------------- launch
static cudaError_t launch_pipe(const void* fn, dim3 grid, size_t smem, cudaStream_t s, void** args, bool pdl) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kPipeThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

static void plan_caps(const MoeLaunch& a, uint32_t& cap_g, uint32_t& cap_r) {
    const uint32_t routed = a.tokens * a.top_k;
    cap_g = (routed < a.num_experts ? routed : a.num_experts) + 1;
    cap_r = routed + a.tokens;
}

bool moe_pipe_supported(const MoeLaunch& a) {
    const MoeLayoutDev& L = a.layout;
    // the pipelined kernels are specialised for the expert shape of every
    // configuration the runtime ships (hidden 2048, intermediate 512)
    if (!moe_mma_supported(L) || a.tokens > 8 || L.hidden != kPipeH || L.inter != kPipeI) return false;
    for (int i = 0; i < 9; ++i)
        if (L.off[i] % 16) return false;
    uint32_t cg, cr;
    plan_caps(a, cg, cr);
    const bool lo = a.x_dtype == PBMOE_F32;
    // two CTAs per SM for the bf16 up kernel and the down kernel
    return up_pipe_smem(L.hidden, lo, cg, cr) <= (lo ? 220u : 112u) * 1024 &&
           down_pipe_smem(L.inter, cg, cr) <= 112u * 1024;
}

cudaError_t moe_up_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts, T = a.tokens;
    uint32_t cg, cr;
    plan_caps(a, cg, cr);
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    if (a.x_dtype == PBMOE_BF16) {
        const dim3 grid(device_sm_count() * UpCfg<uint16_t>::kCtasPerSm);
        const uint16_t* x = static_cast<const uint16_t*>(a.x);
        void* args[] = {(void*)&x,       (void*)&T,  (void*)&E,  (void*)&experts, (void*)&shared,
                        (void*)&L,       (void*)&ws, (void*)&cg, (void*)&cr};
        return launch_pipe(reinterpret_cast<const void*>(moe_up_pipe_kernel<uint16_t, kPipeH, kPipeI>), grid,
                           up_pipe_smem(L.hidden, false, cg, cr), s, args, pdl);
    }
    const float* x = static_cast<const float*>(a.x);
    const dim3 grid(device_sm_count() * UpCfg<float>::kCtasPerSm);
    void* args[] = {(void*)&x, (void*)&T, (void*)&E, (void*)&experts, (void*)&shared,
                    (void*)&L, (void*)&ws, (void*)&cg, (void*)&cr};
    return launch_pipe(reinterpret_cast<const void*>(moe_up_pipe_kernel<float, kPipeH, kPipeI>), grid,
                       up_pipe_smem(L.hidden, true, cg, cr), s, args, pdl);
}

cudaError_t moe_down_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    uint32_t cg, cr;
    plan_caps(a, cg, cr);
    void* args[] = {(void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws, (void*)&cg, (void*)&cr};
    return launch_pipe(reinterpret_cast<const void*>(moe_down_pipe_kernel<kPipeH, kPipeI>), dim3(2 * device_sm_count()),
                       down_pipe_smem(L.inter, cg, cr), s, args, pdl);
}

}  // namespace pbmoe
