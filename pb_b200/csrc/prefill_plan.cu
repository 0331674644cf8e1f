// prefill_plan.cu — the layer-major prefill's expert grouping, on the device.
//
// Reference: the scheduler turns each row's K routes into slots of the
// ascending union of selected experts (ScheduledLayerMajorExperts,
// scheduler/mod.rs:720-765), then qwen_layer_major_group_plan
// (metal/mod.rs:3197-3233) buckets the routes by slot, keeping route order
// inside a slot: source_rows[j] = route / K for grouped row j,
// output_indices[route] = j, groups[slot] = (start, count). Both run on the
// host there after the routing read-back; here one CTA does both on the
// device so the grouped GEMM can follow the routing kernel without a sync.
//
// One CTA of 1024 threads. Route r belongs to warp r / C (C = ceil(routes /
// 32)). Each warp counts its routes per slot (cnt[warp][slot]), a scan over
// warps then slots gives every (warp, slot) its first grouped row, and each
// warp walks its routes in order 32 at a time, ranking equal slots with
// __match_any_sync, so grouped rows keep route order exactly as the stable
// host bucketing does.

#include "kernels.h"
#include "common.cuh"

namespace pbmoe {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;

size_t prefill_plan_smem(uint32_t E) {
    // slot_of[E], cnt[32][E], count[E]
    return (size_t(E) * (kPlanWarps + 2)) * sizeof(uint32_t);
}

// Exclusive block scan of one value per thread (1024 threads).
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* warp_tot, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += u;
    }
    __syncthreads();
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    uint32_t before = 0, tot = 0;
#pragma unroll 4
    for (int w = 0; w < kPlanWarps; ++w) {
        const uint32_t t = warp_tot[w];
        before += w < warp ? t : 0u;
        tot += t;
    }
    total = tot;
    return before + incl - v;
}

__global__ void __launch_bounds__(kPlanThreads, 1) prefill_plan_kernel(PrefillPlanArgs a) {
    extern __shared__ uint32_t psm[];
    const uint32_t E = a.num_experts;
    uint32_t* slot_of = psm;                 // [E]: seen flag, then slot
    uint32_t* cnt = psm + E;                 // [32][E]
    uint32_t* count = cnt + kPlanWarps * E;  // [E]
    __shared__ uint32_t warp_tot[kPlanWarps], bad;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t routes = a.rows * a.top_k;

    for (uint32_t i = tid; i < E * (kPlanWarps + 2); i += kPlanThreads) psm[i] = 0;
    if (tid == 0) bad = 0;
    __syncthreads();
    for (uint32_t r = tid; r < routes; r += kPlanThreads) {
        const uint32_t id = __ldg(a.route_ids + r);
        if (id < E)
            slot_of[id] = 1;
        else
            bad = 1;
    }
    __syncthreads();
    if (bad) {
        if (tid == 0) {
            if (a.status) atomicOr(a.status, PBMOE_DEV_ERR_EXPERT_ID);
            *a.unique_count = 0;
        }
        return;
    }
    // slots: rank of each selected expert among the selected, ascending id
    uint32_t unique = 0;
    for (uint32_t e0 = 0; e0 < E; e0 += kPlanThreads) {  // E <= 1024: one pass
        const uint32_t e = e0 + tid;
        const uint32_t f = e < E ? slot_of[e] : 0u;
        uint32_t tot;
        const uint32_t s = block_excl_scan(f, warp_tot, tot) + unique;
        if (f) a.slot_experts[s] = e;
        __syncthreads();
        if (e < E) slot_of[e] = f ? s : 0xffffffffu;
        unique += tot;
    }
    if (tid == 0) *a.unique_count = unique;
    __syncthreads();

    // per-warp slot counts over the warp's contiguous run of routes
    const uint32_t chunk = (routes + kPlanWarps - 1) / kPlanWarps;
    const uint32_t r0 = min(routes, warp * chunk), r1 = min(routes, r0 + chunk);
    for (uint32_t r = r0 + lane; r < r1; r += 32) atomicAdd(&cnt[warp * E + slot_of[__ldg(a.route_ids + r)]], 1u);
    __syncthreads();
    // per slot: exclusive scan over warps, total count, then over slots
    for (uint32_t s0 = 0; s0 < E; s0 += kPlanThreads) {
        const uint32_t s = s0 + tid;
        uint32_t run = 0;
        if (s < E)
            for (int w = 0; w < kPlanWarps; ++w) {
                const uint32_t v = cnt[w * E + s];
                cnt[w * E + s] = run;
                run += v;
            }
        if (s < E) count[s] = run;
    }
    __syncthreads();
    uint32_t start_base = 0;
    for (uint32_t s0 = 0; s0 < E; s0 += kPlanThreads) {
        const uint32_t s = s0 + tid;
        const uint32_t c = s < unique ? count[s] : 0u;
        uint32_t tot;
        const uint32_t start = block_excl_scan(c, warp_tot, tot) + start_base;
        if (s < unique) {
            for (int w = 0; w < kPlanWarps; ++w) cnt[w * E + s] += start;
            a.groups[2 * s] = start;
            a.groups[2 * s + 1] = c;
        }
        start_base += tot;
    }
    __syncthreads();
    // stable placement, 32 routes of this warp's run at a time
    for (uint32_t b = r0; b < r1; b += 32) {
        const uint32_t r = b + lane;
        const bool ok = r < r1;
        const uint32_t s = ok ? slot_of[__ldg(a.route_ids + r)] : 0xffffffffu;
        const uint32_t same = __match_any_sync(kFull, s);
        if (ok) {
            const uint32_t pos = cnt[warp * E + s] + __popc(same & ((1u << lane) - 1u));
            a.source_rows[pos] = r / a.top_k;
            a.output_indices[r] = pos;
            if (a.route_slots) a.route_slots[r] = s;
        }
        __syncwarp();
        if (ok && lane == __ffs(same) - 1) cnt[warp * E + s] += __popc(same);
        __syncwarp();
    }
}

cudaError_t prefill_plan_launch(const PrefillPlanArgs& a, cudaStream_t s) {
    const size_t smem = prefill_plan_smem(a.num_experts);
    cudaError_t e = cudaFuncSetAttribute(prefill_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    prefill_plan_kernel<<<1, kPlanThreads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace pbmoe
