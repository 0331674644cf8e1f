// routing.cuh — on-device routing softmax/top-K with the reference's exact
// selection semantics, and the layer-major group plan.
#pragma once

#include "common.cuh"

namespace pbmoe {

// Order-preserving map of a non-NaN float to u32 (IEEE order; -0.0 and +0.0
// map to the same key because they compare equal in the reference's `<`).
__device__ __forceinline__ uint32_t float_order_key(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) == 0) u = 0;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr uint32_t kMaxTopK = 32;

// 1 / (1 + exp(-x)) in f32 as the reference computes it (f32 exp, add,
// divide). The exponential is the double-precision exp rounded once to f32,
// which is the correctly rounded f32 exp (the double result is far closer to
// the exact value than any f32 rounding boundary it could straddle, except
// on a set of inputs too small to meet); the host reference's f32 exp is
// correctly rounded too, so biased scores, and the ids selected on them,
// match it bit for bit.
__device__ __forceinline__ float router_sigmoid(float x) {
    const float e = static_cast<float>(exp(-static_cast<double>(x)));
    return 1.0f / (1.0f + e);
}

// Copy one token's E logits from global memory (written by an earlier kernel
// or CTA: read through L2) into shared memory, with every load of the lane in
// flight at once. `s` must be 16-byte aligned; ends with __syncwarp.
__device__ __forceinline__ void stage_logits_warp(const float* __restrict__ lg, uint32_t E, float* s) {
    const int lane = threadIdx.x & 31;
    if ((reinterpret_cast<uintptr_t>(lg) & 15u) == 0) {
        const uint32_t n4 = E >> 2;
        constexpr int kMax = 8;  // 8 x 128 floats per pass
        for (uint32_t base = 0; base < n4; base += 32 * kMax) {
            float4 v[kMax];
#pragma unroll
            for (int i = 0; i < kMax; ++i) {
                const uint32_t q = base + i * 32 + lane;
                if (q < n4) v[i] = __ldcg(reinterpret_cast<const float4*>(lg) + q);
            }
#pragma unroll
            for (int i = 0; i < kMax; ++i) {
                const uint32_t q = base + i * 32 + lane;
                if (q < n4) reinterpret_cast<float4*>(s)[q] = v[i];
            }
        }
        for (uint32_t e = (n4 << 2) + lane; e < E; e += 32) s[e] = __ldcg(lg + e);
    } else {
        for (uint32_t base = 0; base < E; base += 32 * 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t e = base + i * 32 + lane;
                if (e < E) v[i] = __ldcg(lg + e);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t e = base + i * 32 + lane;
                if (e < E) s[e] = v[i];
            }
        }
    }
    __syncwarp();
}

// Weights of the K selected slots (lane k = slot k holds its score `sval` and
// expert `sid`), given the token's logit maximum m and softmax denominator sum:
// the normalisation over the K selected (summed in slot order,
// scheduler/expert_access.rs:80-133) and the routed scaling factor. Invalid
// sums latch PBMOE_DEV_ERR_ROUTE_WEIGHTS (where the reference bails) and
// write zero weights.
// With `raw` (sigmoid/noaux scoring) the slot's probability is instead the
// raw sigmoid of its expert's logit, raw[sid] (routing_sigmoid_noaux_top_k).
__device__ __forceinline__ void route_weights_lanes(float sval, uint32_t sid, float m, float sum, uint32_t K,
                                                    uint32_t normalization, float routed_scale, uint32_t* ids_out,
                                                    float* w_out, uint32_t* status, const float* raw = nullptr) {
    const int lane = threadIdx.x & 31;
    const bool is_slot = static_cast<uint32_t>(lane) < K;
    // softmax probability of each selected slot
    const bool have_inverse = sum > 0.f && isfinite(sum);
    const float inverse_sum = have_inverse ? 1.0f / sum : 0.f;
    float p = 0.f;
    if (is_slot) {
        if (raw) {
            p = router_sigmoid(__ldcg(raw + sid));
        } else {
            p = expf(sval - m);
            if (have_inverse) p *= inverse_sum;
        }
    }
    // normalisation over the K selected, summed in slot order
    float ssum = 0.f;
    for (uint32_t k = 0; k < K; ++k) ssum += __shfl_sync(kFull, p, k);
    bool ok;
    float inv;
    if (normalization == PBMOE_ROUTE_DEEPSEEK_RENORMALIZE_WITH_FLOOR) {
        ok = isfinite(ssum) && ssum >= 0.f;
        inv = 1.0f / fmaxf(ssum, 6.103515625e-5f);
    } else {
        ok = isfinite(ssum) && ssum > 0.f;
        inv = 1.0f / ssum;
    }
    float w = p * inv;
    ok = ok && __all_sync(kFull, !is_slot || p >= 0.f);
    w *= routed_scale;
    if (!ok) {
        w = 0.f;
        if (lane == 0) latch_status(status, PBMOE_DEV_ERR_ROUTE_WEIGHTS);
    }
    if (is_slot) {
        ids_out[lane] = sid;
        w_out[lane] = w;
    }
    __syncwarp();
}

// One warp routes one token whose E logits are in shared memory `s` (K <= 32):
// softmax top-k, or with `bias` (f32 [E]) sigmoid/noaux top-k, whose weights
// are the raw sigmoid of the token's logits `raw` (global, [E]); `s` is
// overwritten with the biased scores then.
//
// The selection replays routing_top_k_iter (math.rs:746-765) exactly: K slots
// start as (expert 0, -inf); experts are visited in index order and an expert
// replaces the FIRST slot holding the minimum value when its score is strictly
// greater. The slots are kept sorted across the warp by (value, slot index):
// lane i holds the i-th entry, so lane 0 holds the first minimum slot, the one
// the next admission replaces. Lanes K..31 hold sentinels (+inf, slot >= K)
// that sort after every real slot and never move. An admission of score v
// evicts lane 0's entry and inserts (v, expert, evicted slot) at its ordered
// place: lanes whose entry sorts below the new one take their upper
// neighbour's entry (one shuffle each of value, expert, slot), the lane at the
// insertion point takes the new entry. Experts are examined 32 at a time:
// lanes whose score beats the current minimum are candidates, replayed in
// ascending expert order, and re-pruned against the new minimum after each
// admission. An expert whose score does not beat the minimum is skipped, as
// the sequential loop skips it.
//
// Weights follow routing_softmax_top_k (math.rs:771-783): p_k = exp(s_k - max)
// * (1/sum_e exp(s_e - max)); then the configured normalisation over the K
// selected p_k (summed in slot order, scheduler/expert_access.rs:80-133) and
// the routed scaling factor (route_weights_lanes).
static __device__ __noinline__ void route_token(float* s, uint32_t E, uint32_t K, uint32_t normalization,
                                                float routed_scale, uint32_t* ids_out, float* w_out,
                                                uint32_t* status, const float* bias = nullptr,
                                                const float* raw = nullptr) {
    const int lane = threadIdx.x & 31;
    const float NEG_INF = -__int_as_float(0x7f800000), POS_INF = __int_as_float(0x7f800000);
    float m = NEG_INF;
    float sum = 0.f;
    if (bias) {
        // sigmoid/noaux (math.rs:788-819): select on sigmoid(logit) + bias
        for (uint32_t e = lane; e < E; e += 32) s[e] = router_sigmoid(s[e]) + __ldg(bias + e);
        __syncwarp();
    } else {
        // max and softmax denominator (rolled loops: this code runs once per
        // token and launch, so its size costs more than its loop overhead)
#pragma unroll 4
        for (uint32_t e = lane; e < E; e += 32) m = fmaxf(m, s[e]);
        m = warp_max(m);
#pragma unroll 4
        for (uint32_t e = lane; e < E; e += 32) sum += expf(s[e] - m);
        sum = warp_sum(sum);
    }

    const uint32_t ulane = static_cast<uint32_t>(lane);
    float ov = ulane < K ? NEG_INF : POS_INF;  // this lane's entry: value, expert, slot
    uint32_t oi = 0, os = ulane;
    float mv = NEG_INF;  // lane 0's entry (uniform): the current minimum and its slot
    uint32_t ms = 0;
    for (uint32_t base = 0; base < E; base += 32) {
        const uint32_t e = base + ulane;
        const float vc = e < E ? s[e] : NEG_INF;
        uint32_t cand = __ballot_sync(kFull, vc > mv);
        while (cand) {
            const int src = __ffs(cand) - 1;
            const float v = __shfl_sync(kFull, vc, src);  // > mv: stale candidates were pruned
            const bool below = lane >= 1 && (ov < v || (ov == v && os < ms));
            const bool up_below = __shfl_down_sync(kFull, below ? 1 : 0, 1) != 0 && lane < 31;
            const float uv = __shfl_down_sync(kFull, ov, 1);
            const uint32_t ui = __shfl_down_sync(kFull, oi, 1);
            const uint32_t us = __shfl_down_sync(kFull, os, 1);
            const bool here = lane == 0 || below;
            const uint32_t slot = ms;
            ov = up_below ? uv : (here ? v : ov);
            oi = up_below ? ui : (here ? base + static_cast<uint32_t>(src) : oi);
            os = up_below ? us : (here ? slot : os);
            mv = __shfl_sync(kFull, ov, 0);
            ms = __shfl_sync(kFull, os, 0);
            cand &= __ballot_sync(kFull, vc > mv) & ~((2u << src) - 1u);
        }
    }
    // lane k takes slot k
    float my_val = NEG_INF;
    uint32_t my_id = 0;
    for (uint32_t j = 0; j < K; ++j) {
        const float v = __shfl_sync(kFull, ov, j);
        const uint32_t id = __shfl_sync(kFull, oi, j);
        const uint32_t sl = __shfl_sync(kFull, os, j);
        if (sl == ulane) {
            my_val = v;
            my_id = id;
        }
    }
    route_weights_lanes(my_val, my_id, m, sum, K, normalization, routed_scale, ids_out, w_out, status,
                        bias ? raw : nullptr);
}

// Block-wide exclusive scan of n <= 4096 u32 values in shared memory, in
// place; returns the total. Uses `tmp` (>= 32 words of shared memory).
__device__ inline uint32_t block_exclusive_scan(uint32_t* a, uint32_t n, uint32_t* tmp) {
    const uint32_t tid = threadIdx.x, nt = blockDim.x;
    const uint32_t per = (n + nt - 1) / nt;
    const uint32_t lo = tid * per, hi = min(lo + per, n);
    uint32_t local = 0;
    for (uint32_t i = lo; i < hi; ++i) local += a[i];
    // warp inclusive scan of local
    const int lane = tid & 31, warp = tid >> 5;
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) tmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t nw = nt >> 5;
        uint32_t v = lane < static_cast<int>(nw) ? tmp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t u = __shfl_up_sync(kFull, v, o);
            if (lane >= o) v += u;
        }
        if (lane < static_cast<int>(nw)) tmp[lane] = v;  // inclusive per warp
    }
    __syncthreads();
    uint32_t run = (warp > 0 ? tmp[warp - 1] : 0) + incl - local;
    const uint32_t total = tmp[(nt >> 5) - 1];
    for (uint32_t i = lo; i < hi; ++i) {
        uint32_t v = a[i];
        a[i] = run;
        run += v;
    }
    __syncthreads();
    return total;
}

}  // namespace pbmoe
