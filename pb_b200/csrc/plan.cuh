// plan.cuh — the layer-major group plan of a MoE layer's routes: unique
// experts ascending (the shared expert first), each expert's routes in route
// order, built from the router's route ids by one CTA. Shared by the router
// kernel (moe_decode.cu) and the pipelined expert kernels (moe_pipe.cu).
#pragma once

#include "common.cuh"
#include "routing.cuh"

namespace pbmoe {

// Where a plan goes: the MoeWs arrays, or a CTA's shared-memory copy.
struct PlanOut {
    uint32_t* expert;      // [groups] expert slot index (e - e_lo), E = shared expert
    uint32_t* start;       // [groups] first grouped position
    uint32_t* count;       // [groups]
    uint32_t* token;       // [positions] token index per grouped position
    uint32_t* route;       // [positions] route index per grouped position
    uint32_t* num_groups;  // [1]
};

__host__ __device__ inline size_t plan_block_scratch_words(uint32_t T, uint32_t K, uint32_t E) {
    return size_t(3) * E + size_t(2) * T * K + 32;
}

// The same plan by the whole CTA, for any number of routes: per-expert counts
// and two block scans, ranks inside each expert from __match_any_sync. With
// max_group = m > 0 an expert's routes (and the shared expert's T) form
// ceil(count / m) consecutive groups of at most m routes each, in the same
// grouped positions: the pipelined expert kernels take at most 8 routes per
// group as their MMA's N operand. Built by the router kernel into the
// workspace for the non-pipelined expert kernels, and by each pipelined
// expert kernel's CTA into its own shared memory (out.* there). `smem` is
// scratch of 3 E + 2 T K + 32 words (plan_block_scratch_words).
static __device__ __noinline__ void plan_block(uint32_t T, uint32_t K, uint32_t E, uint32_t e_lo, uint32_t e_hi,
                                               bool has_shared, uint32_t max_group,
                                               const uint32_t* __restrict__ route_ids, const PlanOut& out,
                                               uint32_t* smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* cnt = smem;             // [E] counts -> starts
    uint32_t* gidx = cnt + E;         // [E] used flags -> group index
    uint32_t* run = gidx + E;         // [E] routes of each expert placed so far
    uint32_t* ids = run + E;          // [T*K]
    uint32_t* rnk = ids + T * K;      // [T*K] rank of each route inside its group
    uint32_t* tmp = rnk + T * K;      // [32]
    const uint32_t R = T * K;
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = run[e] = 0;
    __syncthreads();
    // only the experts of this rank's range [e_lo, e_hi) form groups (all of
    // them on a single GPU); group_expert holds the slot index e - e_lo
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = __ldcg(route_ids + r);
        ids[r] = e;
        if (e >= e_lo && e < e_hi) atomicAdd(&cnt[e], 1u);
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x)
        gidx[e] = max_group ? (cnt[e] + max_group - 1) / max_group : (cnt[e] ? 1u : 0u);
    __syncthreads();
    const uint32_t U = block_exclusive_scan(gidx, E, tmp);
    const uint32_t RL = block_exclusive_scan(cnt, E, tmp);  // cnt[e] = start of expert e; RL local routes
    // rank of each route among the earlier routes of its expert: warp 0 walks
    // the routes 32 at a time; lanes with the same expert find each other with
    // __match_any_sync and a per-expert running count carries across chunks
    if (warp == 0) {
        for (uint32_t r0 = 0; r0 < R; r0 += 32) {
            const uint32_t r = r0 + lane;
            const uint32_t e = r < R ? ids[r] : 0xffffffffu;
            const uint32_t peers = __match_any_sync(kFull, e);
            const uint32_t below = peers & ((1u << lane) - 1u);
            if (r < R && e < E) {
                rnk[r] = run[e] + __popc(below);
                if ((peers >> lane) == 1u) run[e] += __popc(peers);  // the group's highest lane
            }
            __syncwarp();
        }
    }
    __syncthreads();
    const uint32_t mg = max_group ? max_group : 0xffffffffu;
    const uint32_t shared_groups = !has_shared ? 0u : max_group ? (T + max_group - 1) / max_group : 1u;
    const uint32_t routed_base = has_shared ? T : 0u;  // grouped positions taken by the shared groups
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = ids[r];
        if (e < e_lo || e >= e_hi) continue;
        const uint32_t rank = rnk[r];
        const uint32_t pos = routed_base + cnt[e] + rank;
        out.route[pos] = r;
        out.token[pos] = r / K;
        if (rank % mg == 0) {
            // exclusive-scan property: the expert's size is the next start minus this one
            const uint32_t total = (e + 1 < E ? cnt[e + 1] : RL) - cnt[e];
            const uint32_t g = shared_groups + gidx[e] + rank / mg;
            out.expert[g] = e - e_lo;
            out.start[g] = pos;
            out.count[g] = min(total - rank, mg);
        }
    }
    if (has_shared) {
        for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) {
            out.route[t] = R + t;
            out.token[t] = t;
        }
        for (uint32_t j = threadIdx.x; j < shared_groups; j += blockDim.x) {
            out.expert[j] = E;
            out.start[j] = j * mg;
            out.count[j] = min(T - j * mg, mg);
        }
    }
    if (threadIdx.x == 0) *out.num_groups = U + shared_groups;
}

// The same plan by ranking, for the pipelined expert kernels (every CTA
// builds its own copy, so its cost is on their critical path): each route's
// grouped position is the number of local routes with a smaller expert id
// plus the earlier routes of its own expert, found by one pass over the R
// route ids in shared memory per thread; a second pass counts the groups of
// the smaller experts. O(R) per thread and independent of E. `smem` is
// scratch of 5 R + 1 words (plan_rank_scratch_words).
__host__ __device__ inline size_t plan_rank_scratch_words(uint32_t T, uint32_t K) { return size_t(5) * T * K + 1; }

static __device__ __noinline__ void plan_rank(uint32_t T, uint32_t K, uint32_t E, uint32_t e_lo, uint32_t e_hi,
                                              bool has_shared, uint32_t max_group,
                                              const uint32_t* __restrict__ route_ids, const PlanOut& out,
                                              uint32_t* smem) {
    constexpr uint32_t kNone = 0xffffffffu;
    const uint32_t R = T * K;
    uint32_t* ids = smem;         // [R] expert id, or kNone for routes of other ranks' experts
    uint32_t* before = ids + R;   // [R] earlier routes of the same expert
    uint32_t* cnt = before + R;   // [R] routes of the route's expert
    uint32_t* pos = cnt + R;      // [R] grouped position
    uint32_t* ngrp = pos + R;     // [R] the expert's group count on its first route, else 0
    uint32_t* total = ngrp + R;   // [1] local groups
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = __ldcg(route_ids + r);
        ids[r] = (e >= e_lo && e < e_hi) ? e : kNone;
    }
    __syncthreads();
    const uint32_t mg = max_group ? max_group : 0xffffffffu;
    const uint32_t shared_groups = !has_shared ? 0u : max_group ? (T + max_group - 1) / max_group : 1u;
    const uint32_t routed_base = has_shared ? T : 0u;  // grouped positions taken by the shared groups
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = ids[r];
        uint32_t less = 0, same = 0, same_before = 0;
        for (uint32_t q = 0; q < R; ++q) {
            const uint32_t f = ids[q];
            less += f < e ? 1u : 0u;
            same += f == e ? 1u : 0u;
            same_before += (f == e && q < r) ? 1u : 0u;
        }
        before[r] = same_before;
        cnt[r] = same;
        pos[r] = routed_base + less + same_before;
        ngrp[r] = (e != kNone && same_before == 0) ? (max_group ? (same + max_group - 1) / max_group : 1u) : 0u;
    }
    __syncthreads();
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = ids[r], b = before[r];
        if (e == kNone) continue;
        out.route[pos[r]] = r;
        out.token[pos[r]] = r / K;
        if (b % mg != 0) continue;
        uint32_t gless = 0;  // groups of the smaller experts
        for (uint32_t q = 0; q < R; ++q) gless += ids[q] < e ? ngrp[q] : 0u;
        const uint32_t g = shared_groups + gless + b / mg;
        out.expert[g] = e - e_lo;
        out.start[g] = pos[r];
        out.count[g] = min(cnt[r] - b, mg);
    }
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (uint32_t q = 0; q < R; ++q) t += ngrp[q];
        *total = t;
    }
    if (has_shared) {
        for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) {
            out.route[t] = R + t;
            out.token[t] = t;
        }
        for (uint32_t j = threadIdx.x; j < shared_groups; j += blockDim.x) {
            out.expert[j] = E;
            out.start[j] = j * mg;
            out.count[j] = min(T - j * mg, mg);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *out.num_groups = shared_groups + *total;
}

}  // namespace pbmoe
