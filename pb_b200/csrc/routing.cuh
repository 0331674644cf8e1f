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

// One warp routes one token whose E logits are in shared memory `s` (K <= 32).
//
// Selection reproduces routing_top_k_iter (math.rs:746-765) exactly: K slots
// start as (expert 0, -inf); experts are visited in index order and an expert
// replaces the FIRST slot holding the minimum value when its score is strictly
// greater. Slots live in lanes 0..K-1 (slot index = lane). Experts are examined
// 32 at a time: only lanes whose score beats the current minimum are
// candidates, and they are replayed one by one in ascending expert order; after
// each replacement the minimum slot is found again (__reduce_min_sync on an
// order-preserving key, lowest slot on ties) and the remaining candidates are
// pruned against it. Experts that could not have been inserted (score <= the
// current minimum) are skipped, as the sequential loop would have skipped them.
//
// Weights follow routing_softmax_top_k (math.rs:771-783): p_k = exp(s_k - max)
// * (1/sum_e exp(s_e - max)); then the configured normalisation over the K
// selected p_k (summed in slot order, scheduler/expert_access.rs:80-133) and
// the routed scaling factor. Invalid sums latch PBMOE_DEV_ERR_ROUTE_WEIGHTS
// (where the reference bails) and write zero weights.
// Weights of the K selected slots (lane k = slot k holds its score `sval` and
// expert `sid`), given the token's logit maximum m and softmax denominator sum.
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

// Inverse of float_order_key (the zero key maps back to +0.0, which compares
// equal to -0.0 as the reference's comparisons do).
__device__ __forceinline__ float float_from_order_key(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ inline void route_token_smem(const float* s, uint32_t E, uint32_t K, uint32_t normalization,
                                 float routed_scale, uint32_t* ids_out, float* w_out, uint32_t* status) {
    const int lane = threadIdx.x & 31;
    const float NEG_INF = -__int_as_float(0x7f800000);
    // the lane's scores stay in registers for the max, the sum and the scan
    constexpr int kRegChunks = 16;
    const bool in_regs = E <= 32u * kRegChunks;
    float v[kRegChunks];
    float m = NEG_INF;
    float sum = 0.f;
    if (in_regs) {
#pragma unroll
        for (int c = 0; c < kRegChunks; ++c) {
            const uint32_t e = c * 32 + lane;
            v[c] = e < E ? s[e] : NEG_INF;
        }
#pragma unroll
        for (int c = 0; c < kRegChunks; ++c) m = fmaxf(m, v[c]);
        m = warp_max(m);
#pragma unroll
        for (int c = 0; c < kRegChunks; ++c)
            if (static_cast<uint32_t>(c * 32 + lane) < E) sum += expf(v[c] - m);
    } else {
        for (uint32_t e = lane; e < E; e += 32) m = fmaxf(m, s[e]);
        m = warp_max(m);
        for (uint32_t e = lane; e < E; e += 32) sum += expf(s[e] - m);
    }
    sum = warp_sum(sum);

    const bool is_slot = static_cast<uint32_t>(lane) < K;
    float sval = NEG_INF;
    uint32_t sid = 0;
    uint32_t key = is_slot ? float_order_key(NEG_INF) : 0xffffffffu;
    // current minimum slot (value mv, index mslot); all slots start at -inf
    float mv = NEG_INF;
    int mslot = 0;
    // One dependent chain per replacement: select in the slot lane, min-reduce
    // the slot keys, then (in parallel) the new minimum's value from its key
    // and its first slot from a ballot. Candidates are tested against the
    // exact current minimum; stale ones are simply rejected.
    auto scan_chunk = [&](uint32_t base, float vc) {
        uint32_t cand = __ballot_sync(kFull, vc > mv);
        while (cand) {
            const int src = __ffs(cand) - 1;
            cand &= cand - 1;
            const float ve = __shfl_sync(kFull, vc, src);
            if (ve > mv) {  // warp-uniform
                const uint32_t kn = float_order_key(ve);
                if (lane == mslot) {
                    sval = ve;
                    sid = base + static_cast<uint32_t>(src);
                    key = kn;
                }
                const uint32_t mk = __reduce_min_sync(kFull, key);
                mslot = __ffs(__ballot_sync(kFull, key == mk)) - 1;
                mv = float_from_order_key(mk);
            }
        }
    };
    if (in_regs) {
#pragma unroll
        for (int c = 0; c < kRegChunks; ++c)
            if (static_cast<uint32_t>(c * 32) < E) scan_chunk(c * 32, v[c]);
    } else {
        for (uint32_t base = 0; base < E; base += 32) scan_chunk(base, base + lane < E ? s[base + lane] : NEG_INF);
    }
    route_weights_lanes(sval, sid, m, sum, K, normalization, routed_scale, ids_out, w_out, status);
}

// route_token_smem with the K slots replicated in registers of every lane.
// The selection is the same replay of routing_top_k_iter (math.rs:746-765):
// experts in index order, 32 at a time; lanes whose score beats the current
// minimum are candidates, replayed in ascending order; an admitted expert
// replaces the first minimum slot. Here every lane holds all KMAX slots
// (slots >= K hold +inf and are never a minimum, since real slots come first
// and ties go to the lower slot), so an admission is a register select and a
// min tree over the slots instead of warp-wide reductions; after each
// admission one ballot drops the chunk's candidates that no longer beat the
// minimum. When the first K scores are all finite and above -inf, the replay
// would put expert k into slot k for k < K (each fills the first -inf slot),
// so those slots are filled directly. The chunk loop stays rolled (the
// admission code is emitted once).
template <int KMAX>
__device__ __noinline__ void route_token_regs(float* s, uint32_t E, uint32_t K, uint32_t normalization,
                                              float routed_scale, uint32_t* ids_out, float* w_out,
                                              uint32_t* status, const float* bias, const float* raw) {
    const int lane = threadIdx.x & 31;
    const float NEG_INF = -__int_as_float(0x7f800000), POS_INF = __int_as_float(0x7f800000);
    float m = NEG_INF;
    float sum = 0.f;
    if (bias) {
        // sigmoid/noaux (math.rs:788-819): select on sigmoid(logit) + bias
        for (uint32_t e = lane; e < E; e += 32) s[e] = router_sigmoid(s[e]) + __ldg(bias + e);
        __syncwarp();
    } else {
        for (uint32_t e = lane; e < E; e += 32) m = fmaxf(m, s[e]);
        m = warp_max(m);
        for (uint32_t e = lane; e < E; e += 32) sum += expf(s[e] - m);
        sum = warp_sum(sum);
    }

    float sval[KMAX];
    uint32_t sid[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        sval[k] = static_cast<uint32_t>(k) < K ? NEG_INF : POS_INF;
        sid[k] = 0;
    }
    float mv = NEG_INF;  // current minimum value and its (first) slot, one-hot
    uint32_t mslot = 1u;
    auto new_min = [&]() {
        // minimum over the slots, the lowest slot among equals: pairs (a, b)
        // with every index of a below b's keep a unless b is strictly smaller
        float tv[KMAX];
        uint32_t ti[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
            tv[k] = sval[k];
            ti[k] = 1u << k;
        }
#pragma unroll
        for (int w = 1; w < KMAX; w *= 2) {
#pragma unroll
            for (int k = 0; k + w < KMAX; k += 2 * w) {
                const bool b = tv[k + w] < tv[k];
                tv[k] = b ? tv[k + w] : tv[k];
                ti[k] = b ? ti[k + w] : ti[k];
            }
        }
        mv = tv[0];
        mslot = ti[0];  // one-hot: the slot an admission replaces
    };
    uint32_t start = 0;
    {  // the first K experts straight into slots 0..K-1 when all of them are admitted in turn
        const float f = static_cast<uint32_t>(lane) < K ? s[lane] : 0.f;
        if (__all_sync(kFull, static_cast<uint32_t>(lane) >= K || f > NEG_INF)) {
#pragma unroll
            for (int k = 0; k < KMAX; ++k) {
                const float fk = __shfl_sync(kFull, f, k);
                if (static_cast<uint32_t>(k) < K) {
                    sval[k] = fk;
                    sid[k] = static_cast<uint32_t>(k);
                }
            }
            new_min();
            start = K;
        }
    }
    for (uint32_t base = start & ~31u; base < E; base += 32) {
        const uint32_t e = base + lane;
        const float vc = (e < E && e >= start) ? s[e] : NEG_INF;
        uint32_t cand = __ballot_sync(kFull, vc > mv);
        while (cand) {
            const int src = __ffs(cand) - 1;
            const float ve = __shfl_sync(kFull, vc, src);
            // admit (ve > mv holds: stale candidates were dropped below)
            const uint32_t e_new = base + static_cast<uint32_t>(src);
#pragma unroll
            for (int k = 0; k < KMAX; ++k) {
                const bool hit = (mslot >> k) & 1u;
                sval[k] = hit ? ve : sval[k];
                sid[k] = hit ? e_new : sid[k];
            }
            new_min();
            cand &= __ballot_sync(kFull, vc > mv) & ~((2u << src) - 1u);
        }
    }
    // lane k takes slot k
    float my_val = NEG_INF;
    uint32_t my_id = 0;
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
        if (k == lane) {
            my_val = sval[k];
            my_id = sid[k];
        }
    route_weights_lanes(my_val, my_id, m, sum, K, normalization, routed_scale, ids_out, w_out, status,
                        bias ? raw : nullptr);
}

// One warp routes one token whose logits are in shared memory `s` (K <= 32):
// softmax top-k, or with `bias` (f32 [E]) sigmoid/noaux top-k, whose weights
// are the raw sigmoid of the token's logits `raw` (global, [E]); `s` is
// overwritten with the biased scores then.
__device__ inline void route_token(float* s, uint32_t E, uint32_t K, uint32_t normalization, float routed_scale,
                                   uint32_t* ids_out, float* w_out, uint32_t* status, const float* bias = nullptr,
                                   const float* raw = nullptr) {
    // slot counts instantiated: the smallest that holds K (10 is the
    // 512-expert top-10 configuration's)
    if (K <= 4)
        route_token_regs<4>(s, E, K, normalization, routed_scale, ids_out, w_out, status, bias, raw);
    else if (K <= 8)
        route_token_regs<8>(s, E, K, normalization, routed_scale, ids_out, w_out, status, bias, raw);
    else if (K <= 10)
        route_token_regs<10>(s, E, K, normalization, routed_scale, ids_out, w_out, status, bias, raw);
    else if (K <= 16)
        route_token_regs<16>(s, E, K, normalization, routed_scale, ids_out, w_out, status, bias, raw);
    else
        route_token_regs<32>(s, E, K, normalization, routed_scale, ids_out, w_out, status, bias, raw);
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
