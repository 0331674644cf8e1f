// moe_pipe.cu — persistent, asynchronously pipelined MoE expert kernels for
// decode batches of at most 32 tokens (group-64 Q4 experts, hidden 2048,
// intermediate 512: the expert shape of every configuration the runtime
// ships; other shapes use the non-pipelined kernels of moe_mma.cu).
//
// Each CTA walks a contiguous run of work items (consecutive tiles of one or
// two experts). Warp roles:
//   compute warps (8)  tensor-core math (mma.sync, q4_mma.cuh) on one stage
//   producer warp (1)  issues the 16-byte cp.async copies of the items
//                      `stages` ahead and does nothing else: a thread's
//                      cp.async may stall at issue until the SM's request
//                      queue has room, and only this warp ever waits there
//   epilogue warps (2) up kernel only: sum the compute warps' K-slice
//                      partials and write SwiGLU output (one 8-row tile of
//                      the item each), off the compute warps' critical path
// Handshakes: a stage is full when its mbarrier has the producer's 32 lane
// arrivals (cp.async completion, no pending-count increment); compute warps
// release it with bar.arrive EMPTY(s), on which the producer bar.syncs before
// refilling it. Partial sums go through 2 rotating buffers (RED(p) arrive /
// sync towards the epilogue warps, FREE(p) back; the down kernel's activation
// buffers are handed back with ACT_FREE). An arrival is made exactly
// when the matching sync will be made, and no role leaves its item loop
// early: after a failure (a bounded wait expired, PBMOE_DEV_ERR_PIPE_TIMEOUT
// latched) the roles keep the handshakes but skip waits, copies and math, so
// every named barrier completes and the kernel returns.
//
//   moe_up_pipe_kernel    item = (group, 16 intermediate rows), fetched and
//       computed as two steps of half the hidden dimension each: gate and up
//       half-rows + their scales/biases. The 16 rows are the M operand of the
//       mma and the batch's tokens the N operand (q4_mma_rows16); the tokens
//       stay resident in shared memory (staged before the programmatic-
//       dependent-launch wait, as they do not depend on the router). Batches
//       above 8 tokens keep all 32 token rows and gather the N operand from
//       the item's group, which the group plan caps at 8 routes (an
//       expert's routes and the shared expert's tokens split into groups of
//       8, consecutive in the plan, so their weights stream together). 8 compute
//       warps = 8 K-slices of each step; SwiGLU (silu(g)*u,
//       shaders.metal:1699-1708) is written as bf16 hi/lo pair slots +
//       per-8 partial sums (MoeWs::h_perm), the down kernel's input.
//   moe_down_pipe_kernel  item = (group, 64 down rows): warp w takes the
//       16-row block w%4 (the mma's M operand; the group's routes are N) over
//       K-half w/4, and the two halves are summed through shared memory.
//       Weight stages hold only weights: the routed activations of each
//       group of the CTA's run are copied once into one of two buffers (the
//       first two after the programmatic-dependent-launch wait, while the
//       first weight stages are requested before it; a later group's once the
//       compute warps have left the group that held its buffer).

#include "kernels.h"
#include "pipe.cuh"
#include "plan.cuh"
#include "q4_mma.cuh"

namespace pbmoe {

constexpr uint32_t kPipeH = 2048, kPipeI = 512;
constexpr int kWarps = 8;  // compute warps
constexpr int kComputeThreads = kWarps * 32;
constexpr int kHandshake = kComputeThreads + 32;  // compute warps + producer
constexpr int kEpiWarps = 2;                      // up kernel: one epilogue warp per 8-row tile of an item
constexpr int kRedHandshake = kComputeThreads + 32 * kEpiWarps;  // compute warps + epilogue warps
constexpr int kUpThreads = (kWarps + 1 + kEpiWarps) * 32;       // + producer + epilogue
constexpr int kDownThreads = (kWarps + 1) * 32;   // + producer
constexpr int kRedBufs = 2;

// Stage counts: bf16 activations of at most 8 tokens run two CTAs per SM
// (3 stages each); f32 activations keep a 16-row token tile and run one CTA
// per SM; batches of 9..32 bf16 tokens (kGather) keep all 32 token rows
// resident and run one CTA per SM.
constexpr int kUpStagesBf16 = 3;
constexpr int kUpStagesF32 = 5;
constexpr int kUpStagesGather = 3;
constexpr int kDownStages = 3;
constexpr uint32_t kPipeMaxTokens = 32;  // tokens of one launch (8 without kGather)

template <typename XT, bool kGather>
struct UpCfg {
    static constexpr int kStages = kGather ? kUpStagesGather : sizeof(XT) == 4 ? kUpStagesF32 : kUpStagesBf16;
    static constexpr int kCtasPerSm = kGather || sizeof(XT) == 4 ? 1 : 2;
    static constexpr uint32_t kTileRows = kGather ? kPipeMaxTokens : sizeof(XT) == 4 ? 16 : 8;
};

// Named barrier ids (0 is __syncthreads).
constexpr int kBarStage = 1;                                        // compute warps only
__device__ __forceinline__ int bar_empty(int s) { return 2 + s; }  // 2..6
__device__ __forceinline__ int bar_red(int p) { return 7 + p; }    // 7, 8 (up)
__device__ __forceinline__ int bar_free(int p) { return 9 + p; }   // 9, 10 (up)
__device__ __forceinline__ int bar_pair(int rb) { return 5 + rb; }       // 5..8 (down)
__device__ __forceinline__ int bar_pair_free(int rb) { return 9 + rb; }  // 9..12 (down)
__device__ __forceinline__ int bar_act_free(int hb) { return 13 + hb; }  // 13, 14 (down)

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

// The layer-major group plan in shared memory, built by every CTA from the
// router's route ids (build_plan below), so that per-item lookups are
// shared-memory loads instead of dependent L2 round trips. `cap_g` groups and
// `cap_r` grouped positions fit (plan_caps: min(T*K, E) + 1 groups, or T*K +
// ceil(T/8) when groups are split at 8 routes; T*K + T positions).
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

// What a pipelined expert kernel needs to build the group plan itself from
// the router's route ids (plan_rank, into its PlanSmem).
struct PlanArgs {
    uint32_t T, K, e_lo, e_hi, has_shared, max_group;
};

// All threads: the layer-major plan from ws.route_ids into pl, with `scratch`
// (plan_scratch_bytes) as working space; returns the group count. Up to
// kPlanRankRoutes routes the O(R)-per-thread ranking is the faster build,
// above it the block scans (at 320 routes the ranking made the batch-32
// decode step 0.9 ms slower).
constexpr uint32_t kPlanRankRoutes = 128;
__host__ __device__ inline size_t plan_scratch_bytes(uint32_t T, uint32_t K, uint32_t E) {
    return 4 * (T * K <= kPlanRankRoutes ? plan_rank_scratch_words(T, K) : plan_block_scratch_words(T, K, E));
}
__device__ inline uint32_t build_plan(const PlanArgs& pa, uint32_t E, const MoeWs& ws, const PlanSmem& pl,
                                      uint32_t cap_g, uint32_t* scratch, uint32_t* ng_smem) {
    const PlanOut out{pl.expert, pl.start, pl.count, pl.token, pl.route, ng_smem};
    if (pa.T * pa.K <= kPlanRankRoutes)
        plan_rank(pa.T, pa.K, E, pa.e_lo, pa.e_hi, pa.has_shared != 0, pa.max_group, ws.route_ids, out, scratch);
    else
        plan_block(pa.T, pa.K, E, pa.e_lo, pa.e_hi, pa.has_shared != 0, pa.max_group, ws.route_ids, out, scratch);
    __syncthreads();
    return min(*ng_smem, cap_g);
}

// Contiguous run [k0, k1) of the `total` items for this CTA (sizes differ by
// at most one).
__device__ __forceinline__ void item_run(uint32_t total, uint32_t& k0, uint32_t& k1) {
    k0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * total / gridDim.x);
    k1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * total / gridDim.x);
}

__device__ __forceinline__ bool pipe_failed(const uint32_t* flags) {
    return *reinterpret_cast<const volatile uint32_t*>(flags) != 0;
}

// ---------------------------------------------------------------- layouts
// One up step: 16 rows x half of the hidden dimension of gate and of up
// (padded rows), and the matching half of each row's scales/biases.
struct UpStage {
    uint32_t rs;     // padded half-row stride (bytes) = H/4 + 32
    uint32_t srs;    // padded scale-row stride (bytes): H/128 bf16 + pad, 48 for H = 2048
    uint32_t gate, up, sc;  // sc: gs, gb, us, ub blocks of 16 rows each
    uint32_t bytes;  // stage size, multiple of 128
};

__host__ __device__ constexpr UpStage up_stage(uint32_t H) {
    return {H / 4 + 32, H / 64 + 16, 0, 16 * (H / 4 + 32), 32 * (H / 4 + 32),
            (32 * (H / 4 + 32) + 4 * 16 * (H / 64 + 16) + 127) / 128 * 128};
}

__host__ __device__ inline size_t up_pipe_smem(uint32_t H, int stages, uint32_t tile_rows, uint32_t cap_g,
                                              uint32_t cap_r) {
    const UpStage L = up_stage(H);
    // stages, token tile, partial-sum buffers, flags, mbarriers, plan
    return size_t(stages) * L.bytes + act_tile_bytes(H, tile_rows) + size_t(kRedBufs) * kWarps * 256 * 4 + 16 +
           stages * 8 + plan_smem_bytes(cap_g, cap_r);
}
template <typename XT, bool kGather>
inline size_t up_pipe_smem_for(uint32_t H, uint32_t cap_g, uint32_t cap_r) {
    return up_pipe_smem(H, UpCfg<XT, kGather>::kStages, UpCfg<XT, kGather>::kTileRows, cap_g, cap_r);
}

struct DownStage {
    uint32_t rs;  // padded row stride = I/2 + 32
    uint32_t w, s, b;
    uint32_t bytes;
};

__host__ __device__ constexpr DownStage down_stage(uint32_t I) {
    return {I / 2 + 32, 0, 64 * (I / 2 + 32), 64 * (I / 2 + 32) + 64 * (I / 32),
            (64 * (I / 2 + 32) + 128 * (I / 32) + 127) / 128 * 128};
}

// One group's routed activations: 16-row pair-order tile (hi rows 0..7, lo
// rows 8..15) and the per-8 partial sums of each route (padded rows).
struct DownAct {
    uint32_t act, part, part_stride, bytes;
};

__host__ __device__ inline DownAct down_act(uint32_t I) {
    const uint32_t act_bytes = static_cast<uint32_t>(act_tile_bytes(I, 16));
    const uint32_t part = (act_bytes + 15) / 16 * 16;
    const uint32_t ps = (I / 8) * 4 + 32;
    return {0, part, ps, (part + 8 * ps + 127) / 128 * 128};
}

// stages, two activation buffers, K-half partial sums [4 row blocks][32 lanes][4], flags, mbarriers, plan
constexpr uint32_t kDownRedBytes = 4 * 32 * 4 * 4;
__host__ __device__ inline size_t down_pipe_smem(uint32_t I, uint32_t cap_g, uint32_t cap_r) {
    return size_t(kDownStages) * down_stage(I).bytes + 2 * size_t(down_act(I).bytes) + kDownRedBytes + 16 +
           (kDownStages + 2) * 8 + plan_smem_bytes(cap_g, cap_r);
}

// ---------------------------------------------------------------- up
// kGather (batches of 9..32 bf16 tokens): the tile holds every token of the
// batch and an item's N operand is its group's (at most 8) tokens, gathered
// by row index from the tile; without it the N operand is the tile's 8 rows,
// i.e. every token of the batch, and the epilogue picks the group's columns.
template <typename XT, uint32_t H, uint32_t I, bool kGather>
__global__ void __launch_bounds__(kUpThreads, (UpCfg<XT, kGather>::kCtasPerSm))
moe_up_pipe_kernel(const XT* __restrict__ x, uint32_t T, uint32_t E, const uint8_t* __restrict__ experts,
                   const uint8_t* __restrict__ shared_slot, MoeLayoutDev Ld, MoeWs ws, uint32_t cap_g,
                   uint32_t cap_r, int x_from_router, PlanArgs pa) {
    using Cfg = UpCfg<XT, kGather>;
    constexpr bool kLo = sizeof(XT) == 4;
    static_assert(!(kGather && kLo), "gathered token rows are bf16");
    constexpr int S = Cfg::kStages;
    constexpr UpStage SL = up_stage(H);
    constexpr uint32_t kTiles = I / 16;          // 16-row tiles per expert
    constexpr uint32_t kTiles8 = I / 8;          // 8-row tiles of the h_perm layout
    constexpr uint32_t kHalfGroups = H / 128;    // scale groups per step
    constexpr uint32_t kGpw = kHalfGroups / kWarps;  // groups per warp per step
    static_assert(kGpw == 2, "two groups per warp per step");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* stages = smem_raw;
    const ActTile tile = act_tile_at(stages + S * SL.bytes, H, Cfg::kTileRows);
    // partial sums: [kRedBufs][8 warps][gate | up][16 rows][8 columns]
    float* red = reinterpret_cast<float*>(stages + S * SL.bytes + act_tile_bytes(H, Cfg::kTileRows));
    uint32_t* flags = reinterpret_cast<uint32_t*>(red + kRedBufs * kWarps * 256);  // [0] failure
    uint64_t* bar = reinterpret_cast<uint64_t*>(flags + 4);
    const PlanSmem pl = plan_at(bar + S, cap_g, cap_r);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t hps = hperm_stride(I);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bar[s], 32);  // the producer's lanes
        flags[0] = 0;
        fence_mbar_init();
    }
    // The batch's tokens are the layer input, complete before the router
    // started: stage them before waiting for the router, unless the router
    // writes them (the normalised input, x_from_router), in which case they
    // are read only after the wait.
    auto stage_tokens = [&]() {
        if (warp < kWarps) {
            if constexpr (kLo) {
                stage_act_mma<XT>(x, H, nullptr, static_cast<int>(T), H, tile, kBarStage, kComputeThreads);
            } else if constexpr (kGather) {
                for (uint32_t t0 = 0; t0 < T; t0 += 8) {  // 8-row blocks of the tile
                    ActTile sub = tile;
                    sub.act += static_cast<size_t>(t0) * tile.stride;
                    sub.gsum += static_cast<size_t>(t0) * tile.groups;
                    stage_act_rows8_tok<XT>(x + static_cast<size_t>(t0) * H, H, static_cast<int>(min(8u, T - t0)), H,
                                            sub, kBarStage, kComputeThreads);
                }
            } else {
                stage_act_rows8_tok<XT>(x, H, static_cast<int>(T), H, tile, kBarStage, kComputeThreads);
            }
        }
    };
    if (!x_from_router) stage_tokens();
    pdl_wait();
    // the plan first, built from the route ids with the stage area as
    // scratch: the producer's first weight copies are then in flight while
    // the compute warps stage tokens written by the router
    __shared__ uint32_t s_ng;
    const uint32_t ng = build_plan(pa, E, ws, pl, cap_g, reinterpret_cast<uint32_t*>(stages), &s_ng);
    uint32_t k0, k1;
    item_run(ng * kTiles, k0, k1);
    if (k0 >= k1) return;
    const uint32_t my_items = k1 - k0;
    const uint32_t steps = 2 * my_items;
    // Every CTA of this grid is resident, so the down kernel may be scheduled
    // now: its CTAs take SMs as these exit and prefetch weights while the
    // rest of this grid finishes (it waits for all of it before reading h_perm).
    pdl_launch_dependents();

    if (warp == kWarps) {
        // producer: step u = (item k0 + u/2, half u%2): 16 gate and 16 up
        // half-rows (one 512-byte warp copy each) and the four 16-row
        // scale/bias half-blocks (lane = row/2, 16-byte chunk), then each
        // lane's completion arrival
        constexpr uint32_t kRowBytes = H / 2, kHalfBytes = H / 4, kScaleRow = H / 32;
        static_assert(kHalfBytes == 512 && kScaleRow / 2 == 32, "one warp copy per half-row, two chunks per scale half-row");
        auto issue = [&](uint32_t u, int s) {
            const uint32_t k = k0 + u / 2, half = u & 1u;
            const uint32_t gi = k / kTiles, r0 = (k % kTiles) * 16;
            const uint32_t e = pl.expert[gi];
            const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * Ld.expert_bytes;
            unsigned char* st = stages + s * SL.bytes;
            const size_t wo = static_cast<size_t>(r0) * kRowBytes + half * kHalfBytes + lane * 16;
            const uint8_t* gsrc = slot + Ld.off[0] + wo;
            const uint8_t* usrc = slot + Ld.off[3] + wo;
#pragma unroll
            for (uint32_t r = 0; r < 16; ++r) {
                cp_async16(st + SL.gate + r * SL.rs + lane * 16, gsrc + r * kRowBytes);
                cp_async16(st + SL.up + r * SL.rs + lane * 16, usrc + r * kRowBytes);
            }
            const uint32_t row = lane >> 1, chunk = lane & 1;
            const size_t so = static_cast<size_t>(r0 + row) * kScaleRow + half * (kScaleRow / 2) + chunk * 16;
            unsigned char* sd = st + SL.sc + row * SL.srs + chunk * 16;
            cp_async16(sd + 0 * 16 * SL.srs, slot + Ld.off[1] + so);
            cp_async16(sd + 1 * 16 * SL.srs, slot + Ld.off[2] + so);
            cp_async16(sd + 2 * 16 * SL.srs, slot + Ld.off[4] + so);
            cp_async16(sd + 3 * 16 * SL.srs, slot + Ld.off[5] + so);
            cp_async_arrive(&bar[s]);
        };
        for (int u = 0; u < S && static_cast<uint32_t>(u) < steps; ++u) issue(u, u);
        for (uint32_t u = 0; u + S < steps; ++u) {
            const int s = static_cast<int>(u % S);
            named_sync(bar_empty(s), kHandshake);  // every compute warp has released step u's stage
            if (!pipe_failed(flags)) issue(u + S, s);
        }
        cp_async_wait_all();  // no copy of this CTA outlives it
        return;
    }
    if (x_from_router) stage_tokens();

    if (warp > kWarps) {
        // epilogue warp ew = 0, 1 takes the item's 8-row tile ew: lane
        // (q = lane/4, c = lane%4) finishes route q of the group (q < n <= 8)
        // for rows 8ew+c and 8ew+c+4: it sums the 8 K-slice partials of each
        // row for gate and up (slice order 0..7), applies SwiGLU and writes
        // pair word c of the tile as bf16 hi and lo; the quad sums the tile's
        // per-8 partial.
        const uint32_t ew = static_cast<uint32_t>(warp - kWarps - 1);
        const uint32_t q = static_cast<uint32_t>(lane >> 2), c = static_cast<uint32_t>(lane & 3);
        for (uint32_t j = 0; j < my_items; ++j) {
            const int p = static_cast<int>(j % kRedBufs);
            named_sync(bar_red(p), kRedHandshake);  // red[p] holds item j's partials
            if (!pipe_failed(flags)) {
                const uint32_t k = k0 + j;
                const uint32_t gi = k / kTiles, ti = k % kTiles;
                const uint32_t start = pl.start[gi], n = pl.count[gi];
                const bool active = q < n;
                const uint32_t tok = active ? pl.token[start + q] : 0u;
                const float* rb = red + p * kWarps * 256 + (8 * ew + c) * 8 + (kGather ? q : tok);
                float gs[2] = {0.f, 0.f}, us[2] = {0.f, 0.f};  // rows 8ew+c, 8ew+c+4
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        gs[r] += rb[w * 256 + r * 32];
                        us[r] += rb[w * 256 + 128 + r * 32];
                    }
                }
                float h[2];
#pragma unroll
                for (int r = 0; r < 2; ++r) h[r] = gs[r] / (1.0f + expf(-gs[r])) * us[r];
                float part = h[0] + h[1];
                part += __shfl_xor_sync(kFull, part, 1);
                part += __shfl_xor_sync(kFull, part, 2);
                if (active) {
                    uint8_t* hr = ws.h_perm + static_cast<size_t>(pl.route[start + q]) * hps;
                    uint32_t* hw = reinterpret_cast<uint32_t*>(hr);
                    uint32_t* lw = reinterpret_cast<uint32_t*>(hr + kTiles8 * 16);
                    const uint32_t hi = f2_to_bf16x2(h[0], h[1]);
                    const uint32_t lo = f2_to_bf16x2(h[0] - __uint_as_float(hi << 16), h[1] - __uint_as_float(hi & 0xffff0000u));
                    hw[(2 * ti + ew) * 4 + c] = hi;
                    lw[(2 * ti + ew) * 4 + c] = lo;
                    if (c == 0) reinterpret_cast<float*>(hr + 2 * kTiles8 * 16)[2 * ti + ew] = part;
                }
            }
            __syncwarp();
            if (j + kRedBufs < my_items) named_arrive(bar_free(p), kRedHandshake);  // red[p] may be rewritten
        }
        return;
    }

    // compute warps: warp w takes groups 2w, 2w+1 of each half
    const int g = lane >> 2, t = lane & 3;
    const uint32_t gl0 = warp * kGpw;  // first group of this warp within a half
    // tile rows of the lane's B-operand column g and of its output columns
    // 2t, 2t+1 (their activation sums): the columns themselves, or with
    // kGather the tokens of the item's group (columns past the group repeat
    // its last token; the epilogue drops them)
    uint32_t brow = static_cast<uint32_t>(g), xr0 = 2u * t, xr1 = 2u * t + 1u;
    // bf16 activations: the B fragments and activation sums of the warp's
    // groups (both halves) stay in registers while the item's tokens are
    // unchanged (the whole run without kGather, the item's group with it):
    // the shared-memory traffic of a step is then the weight stage alone.
    constexpr bool kCacheX = !kLo;
    uint4 xc[2][kGpw][2];
    float xs[2][kGpw][2];
    uint32_t cur_gi = 0xffffffffu;
    float ag[4], au[4];
    for (uint32_t j = 0; j < my_items; ++j) {
        if constexpr (kCacheX) {
            const uint32_t gi = kGather ? (k0 + j) / kTiles : 0u;
            if (gi != cur_gi) {
                cur_gi = gi;
                if constexpr (kGather) {
                    const uint32_t p0 = pl.start[gi], n = pl.count[gi], last = n ? n - 1 : 0u;
                    brow = min(pl.token[p0 + min(static_cast<uint32_t>(g), last)], Cfg::kTileRows - 1);
                    xr0 = min(pl.token[p0 + min(2u * t, last)], Cfg::kTileRows - 1);
                    xr1 = min(pl.token[p0 + min(2u * t + 1u, last)], Cfg::kTileRows - 1);
                }
#pragma unroll
                for (uint32_t hf = 0; hf < 2; ++hf) {
#pragma unroll
                    for (uint32_t gl = 0; gl < kGpw; ++gl) {
                        const uint32_t grp = hf * kHalfGroups + gl0 + gl;
                        const uint32_t wd = grp * 8 + 2 * t;
                        xc[hf][gl][0] = tile.act[brow * tile.stride + wd];
                        xc[hf][gl][1] = tile.act[brow * tile.stride + wd + 1];
                        xs[hf][gl][0] = tile.gsum[xr0 * tile.groups + grp];
                        xs[hf][gl][1] = tile.gsum[xr1 * tile.groups + grp];
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) ag[i] = au[i] = 0.f;
#pragma unroll
        for (uint32_t half = 0; half < 2; ++half) {
            const uint32_t u = 2 * j + half;
            const int s = static_cast<int>(u % S);
            if (!pipe_failed(flags)) {
                if (mbar_wait_bounded(&bar[s], (u / S) & 1u, kPipeWaitNs)) {
                    const unsigned char* st = stages + s * SL.bytes;
                    // scale / bias pairs of rows g and g+8 for groups gl0, gl0+1
                    const unsigned char* sc = st + SL.sc + gl0 * 2;
                    const uint32_t sgw = *reinterpret_cast<const uint32_t*>(sc + 0 * 16 * SL.srs + g * SL.srs);
                    const uint32_t shw = *reinterpret_cast<const uint32_t*>(sc + 0 * 16 * SL.srs + (g + 8) * SL.srs);
                    const uint32_t bgw = *reinterpret_cast<const uint32_t*>(sc + 1 * 16 * SL.srs + g * SL.srs);
                    const uint32_t bhw = *reinterpret_cast<const uint32_t*>(sc + 1 * 16 * SL.srs + (g + 8) * SL.srs);
                    const uint32_t sgu = *reinterpret_cast<const uint32_t*>(sc + 2 * 16 * SL.srs + g * SL.srs);
                    const uint32_t shu = *reinterpret_cast<const uint32_t*>(sc + 2 * 16 * SL.srs + (g + 8) * SL.srs);
                    const uint32_t bgu = *reinterpret_cast<const uint32_t*>(sc + 3 * 16 * SL.srs + g * SL.srs);
                    const uint32_t bhu = *reinterpret_cast<const uint32_t*>(sc + 3 * 16 * SL.srs + (g + 8) * SL.srs);
#pragma unroll
                    for (uint32_t gl = 0; gl < kGpw; ++gl) {
                        const uint32_t grp = half * kHalfGroups + gl0 + gl;  // group index along H
                        const uint32_t wd = grp * 8 + 2 * t;
                        uint4 xb[2], xl[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
                        float X0, X1;
                        if constexpr (kCacheX) {
                            xb[0] = xc[half][gl][0];
                            xb[1] = xc[half][gl][1];
                            X0 = xs[half][gl][0];
                            X1 = xs[half][gl][1];
                        } else {
                            xb[0] = tile.act[brow * tile.stride + wd];
                            xb[1] = tile.act[brow * tile.stride + wd + 1];
                            if (kLo) {
                                xl[0] = tile.act[(g + 8) * tile.stride + wd];
                                xl[1] = tile.act[(g + 8) * tile.stride + wd + 1];
                            }
                            X0 = tile.gsum[xr0 * tile.groups + grp];
                            X1 = tile.gsum[xr1 * tile.groups + grp];
                        }
                        const uint32_t wo = (gl0 + gl) * 32 + 8 * t;
                        const uint2 gg = *reinterpret_cast<const uint2*>(st + SL.gate + g * SL.rs + wo);
                        const uint2 gh = *reinterpret_cast<const uint2*>(st + SL.gate + (g + 8) * SL.rs + wo);
                        const uint2 ug = *reinterpret_cast<const uint2*>(st + SL.up + g * SL.rs + wo);
                        const uint2 uh = *reinterpret_cast<const uint2*>(st + SL.up + (g + 8) * SL.rs + wo);
                        auto bf = [&](uint32_t wv) {
                            return gl ? __uint_as_float(wv & 0xffff0000u) : __uint_as_float(wv << 16);
                        };
                        q4_mma_rows16<kLo>(gg, gh, xb, xl, bf(sgw), bf(shw), bf(bgw), bf(bhw), X0, X1, ag);
                        q4_mma_rows16<kLo>(ug, uh, xb, xl, bf(sgu), bf(shu), bf(bgu), bf(bhu), X0, X1, au);
                    }
                } else if (lane == 0) {
                    atomicOr(&flags[0], 1u);
                    latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
                }
            }
            if (u + S < steps) named_arrive(bar_empty(s), kHandshake);  // stage s released
        }
        const int p = static_cast<int>(j % kRedBufs);
        if (j >= kRedBufs) named_sync(bar_free(p), kRedHandshake);  // the epilogue is done with red[p]
        float* rw = red + (p * kWarps + warp) * 256;
        *reinterpret_cast<float2*>(rw + g * 8 + 2 * t) = make_float2(ag[0], ag[1]);
        *reinterpret_cast<float2*>(rw + (g + 8) * 8 + 2 * t) = make_float2(ag[2], ag[3]);
        *reinterpret_cast<float2*>(rw + 128 + g * 8 + 2 * t) = make_float2(au[0], au[1]);
        *reinterpret_cast<float2*>(rw + 128 + (g + 8) * 8 + 2 * t) = make_float2(au[2], au[3]);
        named_arrive(bar_red(p), kRedHandshake);
    }
}

// ---------------------------------------------------------------- down
template <uint32_t H, uint32_t I>
__global__ void __launch_bounds__(kDownThreads, 2)
moe_down_pipe_kernel(uint32_t E, const uint8_t* __restrict__ experts, const uint8_t* __restrict__ shared_slot,
                     MoeLayoutDev Ld, MoeWs ws, uint32_t cap_g, uint32_t cap_r, PlanArgs pa) {
    constexpr int S = kDownStages;
    constexpr DownStage SL = down_stage(I);
    constexpr uint32_t tiles = H / 64;
    constexpr uint32_t gpr = I / kMmaGroup;
    constexpr uint32_t wslots = I / 8;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const DownAct AL = down_act(I);
    unsigned char* stages = smem_raw;
    unsigned char* abuf = stages + S * SL.bytes;  // [2][AL.bytes]
    float4* kred = reinterpret_cast<float4*>(abuf + 2 * AL.bytes);  // [4 row blocks][32 lanes]
    uint32_t* flags = reinterpret_cast<uint32_t*>(abuf + 2 * AL.bytes + kDownRedBytes);
    uint64_t* bar = reinterpret_cast<uint64_t*>(flags + 4);  // [S] weight stages, [2] activation buffers
    const PlanSmem pl = plan_at(bar + S + 2, cap_g, cap_r);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t hps = hperm_stride(I);

    // The route ids were written by the router kernel, which completed before
    // the up kernel passed its own wait (and this kernel launched only after
    // that): the plan is built from them before this kernel's wait, with the
    // stage area as scratch.
    __shared__ uint32_t s_ng;
    const uint32_t ng = build_plan(pa, E, ws, pl, cap_g, reinterpret_cast<uint32_t*>(stages), &s_ng);
    uint32_t k0, k1;
    item_run(ng * tiles, k0, k1);
    if (k0 >= k1) {
        pdl_wait();
        return;
    }
    const uint32_t my_items = k1 - k0;
    const uint32_t g_first = k0 / tiles, g_last = (k1 - 1) / tiles;  // the run's groups
    if (threadIdx.x == 0) {
        for (int s = 0; s < S + 2; ++s) mbar_init(&bar[s], 32);  // the producer's lanes
        flags[0] = 0;
        fence_mbar_init();
    }
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
            cp_async_arrive(&bar[s]);
        };
        // ... and, once per group of the run, the group's routed activations:
        // hi and lo bf16 rows of h (pair order) and the per-8 partial sums
        auto issue_act = [&](uint32_t gi, int hb) {
            const uint32_t start = pl.start[gi], n = min(pl.count[gi], 8u);
            unsigned char* ab = abuf + hb * AL.bytes;
            const ActTile tile = act_tile_at(ab + AL.act, I, 16);
            for (uint32_t p = 0; p < n; ++p) {
                const uint8_t* hr = ws.h_perm + static_cast<size_t>(pl.route[start + p]) * hps + lane * 16;
#pragma unroll
                for (uint32_t c = 0; c < wslots; c += 32) {
                    cp_async16(tile.act + p * tile.stride + c + lane, hr + c * 16);
                    cp_async16(tile.act + (p + 8) * tile.stride + c + lane, hr + (wslots + c) * 16);
                }
                if (lane < wslots / 4) cp_async16(ab + AL.part + p * AL.part_stride + lane * 16, hr + 2 * wslots * 16);
            }
            cp_async_arrive(&bar[S + hb]);
        };
        for (int j = 0; j < S && static_cast<uint32_t>(j) < my_items; ++j) issue_weights(k0 + j, j);
        pdl_wait();  // h_perm comes from the up kernel
        issue_act(g_first, 0);
        if (g_last != g_first) issue_act(g_first + 1, 1);
        for (uint32_t j = 0; j + S < my_items; ++j) {
            const int s = static_cast<int>(j % S);
            named_sync(bar_empty(s), kHandshake);  // every compute warp has released item j's stage
            const uint32_t k = k0 + j + S;
            if (k % tiles == 0 && k / tiles >= g_first + 2) {
                // the first item of the run's third or later group m: its
                // activations go into the buffer of group m - 2, which the
                // compute warps left when they entered group m - 1
                const int hb = static_cast<int>((k / tiles - g_first) & 1u);
                named_sync(bar_act_free(hb), kHandshake);
                if (!pipe_failed(flags)) issue_act(k / tiles, hb);
            }
            if (!pipe_failed(flags)) issue_weights(k, s);
        }
        cp_async_wait_all();  // no copy of this CTA outlives it
        return;
    }

    pdl_launch_dependents();  // the combine kernel waits for this whole grid
    const int g = lane >> 2, t = lane & 3;
    const int rb = warp & 3, kh = warp >> 2;  // 16-row block, K-half
    constexpr uint32_t kHalfGroups = gpr / 2;
    static_assert(kHalfGroups == 4, "four groups per K-half");
    uint32_t cur_group = 0xffffffffu;
    ActTile tile{};
    float X0[kHalfGroups], X1[kHalfGroups];  // activation sums of routes 2t, 2t+1 over this K-half's groups
    for (uint32_t j = 0; j < my_items; ++j) {
        const int s = static_cast<int>(j % S);
        const uint32_t k = k0 + j;
        const uint32_t gi = k / tiles, r0 = (k % tiles) * 64;
        bool ok = !pipe_failed(flags);
        if (gi != cur_group) {
            // group m of the run lives in activation buffer m % 2, its
            // (m / 2)-th fill
            const uint32_t m = gi - g_first;
            const int hb = static_cast<int>(m & 1u);
            if (ok) ok = mbar_wait_bounded(&bar[S + hb], (m >> 1) & 1u, kPipeWaitNs);
            if (ok) {
                unsigned char* ab = abuf + hb * AL.bytes;
                tile = act_tile_at(ab + AL.act, I, 16);
                const float* p0 = reinterpret_cast<const float*>(ab + AL.part + (2 * t) * AL.part_stride);
                const float* p1 = reinterpret_cast<const float*>(ab + AL.part + (2 * t + 1) * AL.part_stride);
#pragma unroll
                for (uint32_t i = 0; i < kHalfGroups; ++i) {
                    const uint32_t o = (kh * kHalfGroups + i) * 8;
                    const float4 a0 = *reinterpret_cast<const float4*>(p0 + o), a1 = *reinterpret_cast<const float4*>(p0 + o + 4);
                    const float4 c0 = *reinterpret_cast<const float4*>(p1 + o), c1 = *reinterpret_cast<const float4*>(p1 + o + 4);
                    X0[i] = ((a0.x + a0.y) + (a0.z + a0.w)) + ((a1.x + a1.y) + (a1.z + a1.w));
                    X1[i] = ((c0.x + c0.y) + (c0.z + c0.w)) + ((c1.x + c1.y) + (c1.z + c1.w));
                }
            }
            // group m - 1's buffer is free for group m + 1 (made after the
            // wait above, so after the producer's sync for group m)
            if (m >= 1 && gi + 1 <= g_last) named_arrive(bar_act_free(static_cast<int>((m + 1) & 1u)), kHandshake);
            cur_group = gi;
        }
        if (ok) ok = mbar_wait_bounded(&bar[s], (j / S) & 1u, kPipeWaitNs);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows (g, g+8) x routes (2t, 2t+1)
        if (ok) {
            const unsigned char* st = stages + s * SL.bytes;
            const uint32_t rg = rb * 16 + g;
            // scale / bias of rows rg, rg+8 for the four groups of this K-half
            const uint2 sg = *reinterpret_cast<const uint2*>(st + SL.s + rg * (gpr * 2) + kh * 8);
            const uint2 sh = *reinterpret_cast<const uint2*>(st + SL.s + (rg + 8) * (gpr * 2) + kh * 8);
            const uint2 bg = *reinterpret_cast<const uint2*>(st + SL.b + rg * (gpr * 2) + kh * 8);
            const uint2 bh = *reinterpret_cast<const uint2*>(st + SL.b + (rg + 8) * (gpr * 2) + kh * 8);
#pragma unroll
            for (uint32_t i = 0; i < kHalfGroups; ++i) {
                const uint32_t grp = kh * kHalfGroups + i;
                const uint32_t wd = grp * 8 + 2 * t;
                const uint4 xb[2] = {tile.act[g * tile.stride + wd], tile.act[g * tile.stride + wd + 1]};
                const uint4 xl[2] = {tile.act[(g + 8) * tile.stride + wd], tile.act[(g + 8) * tile.stride + wd + 1]};
                const uint32_t wo = grp * 32 + 8 * t;
                const uint2 wg = *reinterpret_cast<const uint2*>(st + SL.w + rg * SL.rs + wo);
                const uint2 wh = *reinterpret_cast<const uint2*>(st + SL.w + (rg + 8) * SL.rs + wo);
                q4_mma_rows16<true>(wg, wh, xb, xl, Q4MmaFrag4::pick(sg, i), Q4MmaFrag4::pick(sh, i),
                                    Q4MmaFrag4::pick(bg, i), Q4MmaFrag4::pick(bh, i), X0[i], X1[i], acc);
            }
        } else if (lane == 0 && !pipe_failed(flags)) {
            atomicOr(&flags[0], 1u);
            latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
        }
        if (j + S < my_items) named_arrive(bar_empty(s), kHandshake);  // stage s released
        // the K-halves meet: half 1 hands its partials to half 0, which stores y
        if (kh == 1) {
            if (j > 0) named_sync(bar_pair_free(rb), 64);
            kred[rb * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            named_arrive(bar_pair(rb), 64);
        } else {
            named_sync(bar_pair(rb), 64);
            const float4 o = kred[rb * 32 + lane];
            if (j + 1 < my_items) named_arrive(bar_pair_free(rb), 64);
            if (ok && !pipe_failed(flags)) {
                const uint32_t start = pl.start[gi], n = pl.count[gi];
                const uint32_t row = r0 + rb * 16 + g;
                const float v[4] = {acc[0] + o.x, acc[1] + o.y, acc[2] + o.z, acc[3] + o.w};
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t q = 2 * t + c;
                    if (q < n) {
                        float* yr = ws.y + static_cast<size_t>(pl.route[start + q]) * H;
                        yr[row] = v[c];
                        yr[row + 8] = v[2 + c];
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------- launch
static cudaError_t launch_pipe(const void* fn, dim3 grid, int threads, size_t smem, cudaStream_t s, void** args,
                               bool pdl) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
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
    if (a.tokens <= 8)
        cap_g = (routed < a.num_experts ? routed : a.num_experts) + 1;
    else  // groups of at most 8 routes: at most one per route, plus the shared expert's
        cap_g = routed + (a.tokens + 7) / 8;
    cap_r = routed + a.tokens;
}

static uint32_t down_grid() { return 2u * static_cast<uint32_t>(device_sm_count()); }

static PlanArgs plan_args(const MoeLaunch& a) {
    PlanArgs p;
    p.T = a.tokens;
    p.K = a.top_k;
    p.e_lo = a.expert_count ? a.expert_lo : 0u;
    p.e_hi = a.expert_count ? a.expert_lo + a.expert_count : a.num_experts;
    p.has_shared = a.shared_slot != nullptr;
    p.max_group = a.tokens > 8 ? 8u : 0u;
    return p;
}

bool moe_pipe_supported(const MoeLaunch& a) {
    const MoeLayoutDev& L = a.layout;
    if (!moe_mma_supported(L) || a.tokens > kPipeMaxTokens || L.hidden != kPipeH || L.inter != kPipeI) return false;
    for (int i = 0; i < 9; ++i)
        if (L.off[i] % 16) return false;
    const bool gather = a.tokens > 8;
    // gathered batches take bf16 token rows; the expert-parallel exchange
    // keeps its launches at 8 tokens
    if (gather && (a.x_dtype != PBMOE_BF16 || a.ep)) return false;
    uint32_t cg, cr;
    plan_caps(a, cg, cr);
    const bool lo = a.x_dtype == PBMOE_F32;
    const size_t up = gather ? up_pipe_smem_for<uint16_t, true>(L.hidden, cg, cr)
                      : lo   ? up_pipe_smem_for<float, false>(L.hidden, cg, cr)
                             : up_pipe_smem_for<uint16_t, false>(L.hidden, cg, cr);
    // the plan's scratch lives in the stage area of both kernels
    const size_t scratch = plan_scratch_bytes(a.tokens, a.top_k, a.num_experts);
    const int up_stages = gather ? kUpStagesGather : lo ? kUpStagesF32 : kUpStagesBf16;
    if (scratch > size_t(up_stages) * up_stage(L.hidden).bytes || scratch > size_t(kDownStages) * down_stage(L.inter).bytes)
        return false;
    // one CTA per SM for the gathered and f32 up kernels, two for the 8-token
    // bf16 one and the down kernel
    return up <= (gather || lo ? 227u : 112u) * 1024 && down_pipe_smem(L.inter, cg, cr) <= 112u * 1024;
}

template <typename XT, bool kGather>
static cudaError_t up_pipe_launch_t(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts, T = a.tokens;
    uint32_t cg, cr;
    plan_caps(a, cg, cr);
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    int from_router = a.in_norm_w != nullptr;
    PlanArgs pa = plan_args(a);
    const XT* x = static_cast<const XT*>(a.x);
    const dim3 grid(device_sm_count() * UpCfg<XT, kGather>::kCtasPerSm);
    void* args[] = {(void*)&x, (void*)&T,  (void*)&E,  (void*)&experts, (void*)&shared,
                    (void*)&L, (void*)&ws, (void*)&cg, (void*)&cr,      (void*)&from_router, (void*)&pa};
    return launch_pipe(reinterpret_cast<const void*>(moe_up_pipe_kernel<XT, kPipeH, kPipeI, kGather>), grid,
                       kUpThreads, up_pipe_smem_for<XT, kGather>(L.hidden, cg, cr), s, args, pdl);
}

cudaError_t moe_up_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    if (a.x_dtype == PBMOE_BF16)
        return a.tokens > 8 ? up_pipe_launch_t<uint16_t, true>(a, s, pdl) : up_pipe_launch_t<uint16_t, false>(a, s, pdl);
    return up_pipe_launch_t<float, false>(a, s, pdl);
}

cudaError_t moe_down_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl) {
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    uint32_t E = a.num_experts;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    uint32_t cg, cr;
    plan_caps(a, cg, cr);
    PlanArgs pa = plan_args(a);
    void* args[] = {(void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws, (void*)&cg, (void*)&cr, (void*)&pa};
    return launch_pipe(reinterpret_cast<const void*>(moe_down_pipe_kernel<kPipeH, kPipeI>), dim3(down_grid()),
                       kDownThreads, down_pipe_smem(L.inter, cg, cr), s, args, pdl);
}

}  // namespace pbmoe
