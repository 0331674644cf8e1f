// moe_pipe.cu — persistent, asynchronously pipelined MoE expert kernels for
// decode batches of at most 8 tokens (group-64 Q4 experts).
//
// One CTA per SM walks a strided list of work items. The weight bytes of each
// item are moved by the SM's TMA engine (1-D cp.async.bulk, no multicast) into
// one of several shared-memory stages, completing on that stage's mbarrier;
// warp 0 refills a stage as soon as every warp has finished reading it, so
// several items' bytes are always in flight per SM while the tensor cores
// (mma.sync, q4_mma.cuh) consume the current one. Rows land in padded shared
// rows so fragment loads are bank-conflict free.
//
//   moe_up_pipe_kernel    item = (group, 8 intermediate rows): gate and up
//       rows + their scales/biases; the batch's tokens stay resident in shared
//       memory for the whole kernel. 8 warps = 8 K-slices, summed in shared
//       memory; SwiGLU (silu(g)*u, shaders.metal:1699-1708) is written as bf16
//       hi/lo pair slots + per-8 partial sums (MoeWs::h_perm), the down
//       kernel's input layout.
//   moe_down_pipe_kernel  item = (group, 64 down rows): rows, scales, and the
//       group's routes' h_perm rows. Weights of the first stages are requested
//       before the programmatic-dependent-launch wait (they do not depend on
//       the up kernel).
//
// Every mbarrier wait is bounded (kPipeWaitNs); on expiry the kernel latches
// PBMOE_DEV_ERR_PIPE_TIMEOUT, waits (bounded) for its own copies, and returns.

#include "kernels.h"
#include "pipe.cuh"
#include "q4_mma.cuh"

namespace pbmoe {

// Stage counts: bf16 activations run two CTAs per SM (3 stages each, 18 warps
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

// ---------------------------------------------------------------- layouts
struct UpStage {
    uint32_t rs;     // padded row stride (bytes) = H/2 + 32
    uint32_t gate, up, gs, gb, us, ub;
    uint32_t bytes;  // stage size, multiple of 128
    uint32_t tx;     // bytes delivered per item
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
    L.tx = 16 * (H / 2) + 4 * sb;
    return L;
}

__host__ __device__ inline size_t up_pipe_smem(uint32_t H, bool lo) {
    const UpStage L = up_stage(H);
    const int stages = lo ? kUpStagesF32 : kUpStagesBf16;
    // stages, token tile, 2 x 8 warps x 128 partial sums, 64-entry h buffer, flags, mbarriers
    return size_t(stages) * L.bytes + act_tile_bytes(H, lo ? 16 : 8) + 2 * 8 * 128 * 4 + 64 * 4 + 16 + stages * 8;
}

struct DownStage {
    uint32_t rs;  // padded row stride = I/2 + 32
    uint32_t w, s, b, act, part;
    uint32_t part_stride;  // padded stride of the per-route partial-sum rows
    uint32_t bytes;
    uint32_t tx_w;     // weight + scale bytes per item
    uint32_t tx_route; // h bytes per route
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
    L.tx_w = 64 * (I / 2) + 2 * sb;
    L.tx_route = 2 * (I / 8) * 16 + (I / 8) * 4;
    return L;
}

__host__ __device__ inline size_t down_pipe_smem(uint32_t I) {
    return size_t(kDownStages) * down_stage(I).bytes + 16 + kDownStages * 8;
}

// Bounded drain of every stage's outstanding phase after a failure.
__device__ void drain_stages(uint64_t* bar, int stages, const uint32_t* pending_parity, const bool* pending) {
    for (int s = 0; s < stages; ++s)
        if (pending[s]) mbar_wait_bounded(&bar[s], pending_parity[s], 100000000ull);
}

// Warp roles: warps 0..7 compute, warp 8 ("PE") produces copies and runs
// the epilogue. Compute warps never wait on a CTA-wide barrier: they wait on
// the stage's mbarrier (data), arrive on named barrier READY(s) once they have
// finished reading stage s (and, for the up kernel, written their partial
// sums), and - up kernel only - sync on FREE(p) before overwriting the
// double-buffered partial-sum area p that the PE warp reads.
constexpr int kComputeWarps = 8;
constexpr int kPipeCtaThreads = (kComputeWarps + 1) * 32;
__device__ __forceinline__ int bar_ready(int s) { return 1 + s; }   // ids 1..stages (<= 6)
__device__ __forceinline__ int bar_free(int p) { return 7 + p; }    // ids 7, 8

// ---------------------------------------------------------------- up
template <typename XT>
__global__ void __launch_bounds__(kPipeCtaThreads, UpCfg<XT>::kCtasPerSm)
moe_up_pipe_kernel(const XT* __restrict__ x, uint32_t T, uint32_t E, const uint8_t* __restrict__ experts,
                   const uint8_t* __restrict__ shared_slot, MoeLayoutDev Ld, MoeWs ws) {
    constexpr bool kLo = sizeof(XT) == 4;
    constexpr int kUpStages = UpCfg<XT>::kStages;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const uint32_t H = Ld.hidden, I = Ld.inter;
    const UpStage SL = up_stage(H);
    unsigned char* stages = smem_raw;
    const ActTile tile = act_tile_at(stages + kUpStages * SL.bytes, H, kLo ? 16 : 8);
    float* red = reinterpret_cast<float*>(stages + kUpStages * SL.bytes + act_tile_bytes(H, kLo ? 16 : 8));
    float* hbuf = red + 2 * kComputeWarps * 2 * 64;  // [8 routes][8 rows]
    uint32_t* flags = reinterpret_cast<uint32_t*>(hbuf + 64);  // [0] error, [1] stop
    uint64_t* bar = reinterpret_cast<uint64_t*>(flags + 4);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t tiles = I / 8;
    const uint32_t gpr = H / kMmaGroup;
    const uint32_t gps = gpr / kComputeWarps;  // groups per warp K-slice (multiple of 4)
    const size_t hps = hperm_stride(I);

    pdl_wait();
    const uint32_t total = __ldcg(ws.num_groups) * tiles;
    if (blockIdx.x >= total) return;
    const uint32_t my_items = (total - blockIdx.x + gridDim.x - 1) / gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kUpStages; ++s) mbar_init(&bar[s], 1);
        flags[0] = 0;
        flags[1] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    auto slot_of = [&](uint32_t gi) -> const uint8_t* {
        const uint32_t e = __ldcg(ws.group_expert + gi);
        return e >= E ? shared_slot : experts + static_cast<size_t>(e) * Ld.expert_bytes;
    };
    // PE warp: request item k into stage s
    auto issue = [&](uint32_t k, int s) {
        const uint32_t gi = k / tiles, i0 = (k % tiles) * 8;
        const uint8_t* slot = slot_of(gi);
        unsigned char* st = stages + s * SL.bytes;
        if (lane == 0) mbar_arrive_expect_tx(&bar[s], SL.tx);
        __syncwarp();
        if (lane < 8) {
            bulk_g2s(st + SL.gate + lane * SL.rs, slot + Ld.off[0] + static_cast<size_t>(i0 + lane) * (H / 2), H / 2,
                     &bar[s]);
        } else if (lane < 16) {
            const int r = lane - 8;
            bulk_g2s(st + SL.up + r * SL.rs, slot + Ld.off[3] + static_cast<size_t>(i0 + r) * (H / 2), H / 2, &bar[s]);
        } else if (lane < 20) {
            const int c = lane - 16;  // gs, gb, us, ub
            const uint32_t dst[4] = {SL.gs, SL.gb, SL.us, SL.ub};
            const uint64_t off[4] = {Ld.off[1], Ld.off[2], Ld.off[4], Ld.off[5]};
            bulk_g2s(st + dst[c], slot + off[c] + static_cast<size_t>(i0) * (H / 32), 8 * (H / 32), &bar[s]);
        }
    };

    if (warp == kComputeWarps) {
        for (int j = 0; j < kUpStages && static_cast<uint32_t>(j) < my_items; ++j) issue(blockIdx.x + j * gridDim.x, j);
    }
    // the batch's tokens stay resident for the whole kernel (all 288 threads stage them)
    if constexpr (kLo)
        stage_act_mma<XT>(x, H, nullptr, static_cast<int>(T), H, tile);
    else
        stage_act_rows8_tok<XT>(x, H, static_cast<int>(T), H, tile);
    // Every CTA of this grid is resident (one per SM), so the down kernel may
    // be scheduled now: its CTAs take SMs as these exit and prefetch weights
    // while the rest of this grid finishes (it waits for all of it before
    // reading h_perm).
    pdl_launch_dependents();

    if (warp < kComputeWarps) {
        const uint32_t grp0 = warp * gps;
        for (uint32_t j = 0; j < my_items; ++j) {
            const int s = static_cast<int>(j % kUpStages);
            const int p = static_cast<int>(j & 1u);
            if (j >= 2) {
                named_sync(bar_free(p), kPipeCtaThreads);  // PE has consumed red[p] of item j-2
                if (*reinterpret_cast<volatile uint32_t*>(&flags[1])) break;
            }
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
                    fg.compute<kLo, false>(tile, grp0 + b, g, t, ag);
                    fu.compute<kLo, false>(tile, grp0 + b, g, t, au);
                }
            } else if (lane == 0) {
                atomicOr(&flags[0], 1u);
            }
            float* rw = red + (p * kComputeWarps + warp) * 128;
            rw[g * 8 + 2 * t] = ag[0];
            rw[g * 8 + 2 * t + 1] = ag[1];
            rw[64 + g * 8 + 2 * t] = au[0];
            rw[64 + g * 8 + 2 * t + 1] = au[1];
            named_arrive(bar_ready(s), kPipeCtaThreads);
        }
    } else {
        // PE warp: refill + epilogue
        for (uint32_t j = 0; j < my_items; ++j) {
            const int s = static_cast<int>(j % kUpStages);
            const int p = static_cast<int>(j & 1u);
            named_sync(bar_ready(s), kPipeCtaThreads);  // stage s read, red[p] written by every compute warp
            if (*reinterpret_cast<volatile uint32_t*>(&flags[0])) {
                if (lane == 0) {
                    latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
                    flags[1] = 1;
                    uint32_t pp[kUpStages];
                    bool pend[kUpStages];
                    for (int q = 0; q < kUpStages; ++q) {
                        const uint32_t jj = j + ((q - s + kUpStages) % kUpStages);
                        pend[q] = jj < my_items && jj != j;
                        pp[q] = (jj / kUpStages) & 1u;
                    }
                    drain_stages(bar, kUpStages, pp, pend);
                }
                __syncwarp();
                if (j + 2 < my_items) named_arrive(bar_free(p), kPipeCtaThreads);
                break;
            }
            const uint32_t k = blockIdx.x + j * gridDim.x;
            if (j + kUpStages < my_items) issue(k + kUpStages * gridDim.x, s);
            const uint32_t gi = k / tiles, ti = k % tiles;
            const uint32_t start = __ldcg(ws.group_start + gi), n = __ldcg(ws.group_count + gi);
            // lane (route q0 = lane/4, rows 2(lane%4), 2(lane%4)+1)
            const uint32_t q0 = lane >> 2, rr = 2 * (lane & 3);
            const float* rb = red + p * kComputeWarps * 128;
            if (q0 < n) {
                const uint32_t tok = __ldcg(ws.group_tokens + start + q0);
                float g0 = 0.f, g1 = 0.f, u0 = 0.f, u1 = 0.f;
#pragma unroll
                for (int w = 0; w < kComputeWarps; ++w) {
                    g0 += rb[w * 128 + tok * 8 + rr];
                    g1 += rb[w * 128 + tok * 8 + rr + 1];
                    u0 += rb[w * 128 + 64 + tok * 8 + rr];
                    u1 += rb[w * 128 + 64 + tok * 8 + rr + 1];
                }
                hbuf[q0 * 8 + rr] = g0 / (1.0f + expf(-g0)) * u0;
                hbuf[q0 * 8 + rr + 1] = g1 / (1.0f + expf(-g1)) * u1;
            }
            __syncwarp();
            // red[p] fully read: the compute warps may overwrite it (item j+2)
            if (j + 2 < my_items) named_arrive(bar_free(p), kPipeCtaThreads);
            if (q0 < n) {
                // lane writes bf16 pair word c = lane%4: (h_c, h_{c+4}) as hi and lo
                const uint32_t c = lane & 3;
                const float a = hbuf[q0 * 8 + c], bv = hbuf[q0 * 8 + c + 4];
                const uint32_t hi = f2_to_bf16x2(a, bv);
                const uint32_t lo = f2_to_bf16x2(a - __uint_as_float(hi << 16), bv - __uint_as_float(hi & 0xffff0000u));
                const uint32_t route = __ldcg(ws.group_routes + start + q0);
                uint8_t* hr = ws.h_perm + static_cast<size_t>(route) * hps;
                reinterpret_cast<uint32_t*>(hr)[ti * 4 + c] = hi;
                reinterpret_cast<uint32_t*>(hr + tiles * 16)[ti * 4 + c] = lo;
                if (c == 0) {
                    float part = 0.f;
#pragma unroll
                    for (int r = 0; r < 8; ++r) part += hbuf[q0 * 8 + r];
                    reinterpret_cast<float*>(hr + 2 * tiles * 16)[ti] = part;
                }
            }
            __syncwarp();
        }
    }
}

// ---------------------------------------------------------------- down
__global__ void __launch_bounds__(kPipeCtaThreads, 2)
moe_down_pipe_kernel(uint32_t E, const uint8_t* __restrict__ experts, const uint8_t* __restrict__ shared_slot,
                     MoeLayoutDev Ld, MoeWs ws) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const uint32_t H = Ld.hidden, I = Ld.inter;
    const DownStage SL = down_stage(I);
    unsigned char* stages = smem_raw;
    uint32_t* flags = reinterpret_cast<uint32_t*>(stages + kDownStages * SL.bytes);
    uint64_t* bar = reinterpret_cast<uint64_t*>(flags + 4);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t tiles = H / 64;
    const uint32_t gpr = I / kMmaGroup;  // 4 or 8
    const uint32_t wslots = I / 8;
    const size_t hps = hperm_stride(I);

    // The group plan was written by the router kernel, which completed before
    // the up kernel passed its own wait; it is safe to read before this
    // kernel's wait (through L2).
    const uint32_t total = __ldcg(ws.num_groups) * tiles;
    if (blockIdx.x >= total) {
        pdl_wait();
        return;
    }
    const uint32_t my_items = (total - blockIdx.x + gridDim.x - 1) / gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kDownStages; ++s) mbar_init(&bar[s], 1);
        flags[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    auto slot_of = [&](uint32_t gi) -> const uint8_t* {
        const uint32_t e = __ldcg(ws.group_expert + gi);
        return e >= E ? shared_slot : experts + static_cast<size_t>(e) * Ld.expert_bytes;
    };
    auto issue_weights = [&](uint32_t k, int s) {
        const uint32_t gi = k / tiles, r0 = (k % tiles) * 64;
        const uint32_t n = __ldcg(ws.group_count + gi);
        const uint8_t* slot = slot_of(gi);
        unsigned char* st = stages + s * SL.bytes;
        if (lane == 0) mbar_arrive_expect_tx(&bar[s], SL.tx_w + n * SL.tx_route);
        __syncwarp();
        for (int r = lane; r < 64; r += 32)
            bulk_g2s(st + SL.w + r * SL.rs, slot + Ld.off[6] + static_cast<size_t>(r0 + r) * (I / 2), I / 2, &bar[s]);
        if (lane == 0) bulk_g2s(st + SL.s, slot + Ld.off[7] + static_cast<size_t>(r0) * (I / 32), 64 * (I / 32), &bar[s]);
        if (lane == 1) bulk_g2s(st + SL.b, slot + Ld.off[8] + static_cast<size_t>(r0) * (I / 32), 64 * (I / 32), &bar[s]);
    };
    auto issue_h = [&](uint32_t k, int s) {
        const uint32_t gi = k / tiles;
        const uint32_t start = __ldcg(ws.group_start + gi), n = __ldcg(ws.group_count + gi);
        unsigned char* st = stages + s * SL.bytes;
        const ActTile tile = act_tile_at(st + SL.act, I, 16);
        for (uint32_t c = lane; c < 3 * n; c += 32) {
            const uint32_t p = c / 3, part = c % 3;
            const uint8_t* hr = ws.h_perm + static_cast<size_t>(__ldcg(ws.group_routes + start + p)) * hps;
            if (part == 0)
                bulk_g2s(tile.act + p * tile.stride, hr, wslots * 16, &bar[s]);
            else if (part == 1)
                bulk_g2s(tile.act + (p + 8) * tile.stride, hr + wslots * 16, wslots * 16, &bar[s]);
            else
                bulk_g2s(st + SL.part + p * SL.part_stride, hr + 2 * wslots * 16, wslots * 4, &bar[s]);
        }
    };

    if (warp == kComputeWarps) {
        for (int j = 0; j < kDownStages && static_cast<uint32_t>(j) < my_items; ++j)
            issue_weights(blockIdx.x + j * gridDim.x, j);
    }
    pdl_wait();  // h_perm comes from the up kernel
    pdl_launch_dependents();  // the combine kernel waits for this whole grid
    if (warp == kComputeWarps) {
        for (int j = 0; j < kDownStages && static_cast<uint32_t>(j) < my_items; ++j)
            issue_h(blockIdx.x + j * gridDim.x, j);
    }

    if (warp < kComputeWarps) {
        const uint32_t rw0 = warp * 8;  // this warp's 8 rows within the 64-row tile
        for (uint32_t j = 0; j < my_items; ++j) {
            const int s = static_cast<int>(j % kDownStages);
            const bool ok = mbar_wait_bounded(&bar[s], (j / kDownStages) & 1u, kPipeWaitNs);
            if (ok) {
                const uint32_t k = blockIdx.x + j * gridDim.x;
                const uint32_t gi = k / tiles, r0 = (k % tiles) * 64;
                const uint32_t start = __ldcg(ws.group_start + gi), n = __ldcg(ws.group_count + gi);
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
                if (static_cast<uint32_t>(g) < n) {
                    const uint32_t route = __ldcg(ws.group_routes + start + g);
                    *reinterpret_cast<float2*>(ws.y + static_cast<size_t>(route) * H + r0 + rw0 + 2 * t) =
                        make_float2(acc[0], acc[1]);
                }
            } else if (lane == 0) {
                atomicOr(&flags[0], 1u);
            }
            named_arrive(bar_ready(s), kPipeCtaThreads);
            if (!ok) break;
        }
    } else {
        for (uint32_t j = 0; j < my_items; ++j) {
            const int s = static_cast<int>(j % kDownStages);
            named_sync(bar_ready(s), kPipeCtaThreads);  // stage s consumed by every compute warp
            if (*reinterpret_cast<volatile uint32_t*>(&flags[0])) {
                if (lane == 0) {
                    latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
                    uint32_t pp[kDownStages];
                    bool pend[kDownStages];
                    for (int q = 0; q < kDownStages; ++q) {
                        const uint32_t jj = j + ((q - s + kDownStages) % kDownStages);
                        pend[q] = jj < my_items && jj != j;
                        pp[q] = (jj / kDownStages) & 1u;
                    }
                    drain_stages(bar, kDownStages, pp, pend);
                }
                break;
            }
            if (j + kDownStages < my_items) {
                const uint32_t kn = blockIdx.x + (j + kDownStages) * gridDim.x;
                issue_weights(kn, s);
                issue_h(kn, s);
            }
        }
    }
}

// ---------------------------------------------------------------- launch
static cudaError_t launch_pipe(const void* fn, dim3 grid, size_t smem, cudaStream_t s, void** args, bool pdl) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kPipeCtaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

bool moe_pipe_supported(const MoeLaunch& a) {
    const MoeLayoutDev& L = a.layout;
    if (!moe_mma_supported(L) || a.tokens > 8) return false;
    for (int i = 0; i < 9; ++i)
        if (L.off[i] % 16) return false;
    const bool lo = a.x_dtype == PBMOE_F32;
    // two CTAs per SM for the bf16 up kernel and the down kernel
    return up_pipe_smem(L.hidden, lo) <= (lo ? 220u : 112u) * 1024 && down_pipe_smem(L.inter) <= 112u * 1024;
}

cudaError_t moe_up_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts, T = a.tokens;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    if (a.x_dtype == PBMOE_BF16) {
        const dim3 grid(device_sm_count() * UpCfg<uint16_t>::kCtasPerSm);
        const uint16_t* x = static_cast<const uint16_t*>(a.x);
        void* args[] = {(void*)&x, (void*)&T, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
        return launch_pipe(reinterpret_cast<const void*>(moe_up_pipe_kernel<uint16_t>), grid,
                           up_pipe_smem(L.hidden, false), s, args, pdl);
    }
    const float* x = static_cast<const float*>(a.x);
    const dim3 grid(device_sm_count() * UpCfg<float>::kCtasPerSm);
    void* args[] = {(void*)&x, (void*)&T, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    return launch_pipe(reinterpret_cast<const void*>(moe_up_pipe_kernel<float>), grid, up_pipe_smem(L.hidden, true),
                       s, args, pdl);
}

cudaError_t moe_down_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    void* args[] = {(void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    return launch_pipe(reinterpret_cast<const void*>(moe_down_pipe_kernel), dim3(2 * device_sm_count()),
                       down_pipe_smem(L.inter), s, args, pdl);
}

}  // namespace pbmoe
