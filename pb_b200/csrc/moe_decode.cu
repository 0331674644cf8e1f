// moe_decode.cu — one MoE FFN decode layer on sm_100a, four stream-ordered
// kernels:
//
//   1. moe_router_kernel   router GEMV (bf16 [E x H]) + shared-expert gate
//                          logit; the first CTAs route the tokens once every
//                          CTA's logits are written (route_token) and build the
//                          layer-major group plan (unique experts in ascending
//                          id order, routes in route order inside each group,
//                          shared expert as group 0 with every token).
//   2. moe_expert_up_kernel   gate and up rows of one group's expert for the
//                          group's tokens, SwiGLU fused: h = silu(g) * u.
//   3. moe_expert_down_kernel down rows of the group's expert on h -> y.
//   4. moe_combine_kernel  out = residual + sum_k w_k y_k + sigma(gate.x) y_shared,
//                          optional next-layer RMSNorm.
//
// Reference counterparts: the router projection and CPU top-k
// (runtime/mod.rs:1065, math.rs:771-783), the grouping plan
// (metal/mod.rs:3197-3233), the per-expert CMD3 dispatches
// (metal/mod.rs:4289-4470: q4 gate :4365, up :4375, silu_product :4389,
// down :4396), the shared phase (metal/mod.rs:4609-4716) and the combine
// (shaders.metal:1723-1786) with the next-layer rms_norm_reduced
// (shaders.metal:1176-1213).
//
// Kernels 2-4 are launched with programmatic dependent launch: each waits on
// griddepcontrol.wait before touching its predecessor's outputs.

#include <cooperative_groups.h>

#include "kernels.h"
#include "pipe.cuh"
#include "q4_rows.cuh"
#include "plan.cuh"
#include "routing.cuh"

namespace pbmoe {

namespace cg = cooperative_groups;

// ---------------------------------------------------------------- kernel 1
// Router logits in exactly the reference's arithmetic. dense_mmap_fma_matvec_bf16
// (shaders.metal:1059-1075), restated on the CPU as the oracle's router, runs one
// sequential fp32 fma chain per (row, token): acc = fma(w[c], x[c], acc) for
// c = 0, 1, ..., H-1. Route ids are integer outputs and must match bit for bit,
// so every (row, token) chain here is one thread walking the columns in that
// order: the sum is never split or reassociated, and identical inputs give
// identical logits, hence identical top-k ids. A chain of H dependent fmas is
// the kernel's floor (H x the fma latency); everything else is arranged around
// it.
//
// A CTA owns rpc consecutive rows (kRtRows, or fewer when rows of a wide
// hidden size would not fit in shared memory; row E is the shared-expert
// gate) and runs their chains for a pass of up to kRtTokPass tokens, a warp
// covering 4 rows x 8 tokens so that each shared-memory read serves 8 or 4
// chains.
// The rows' bf16 weights arrive in shared memory by bulk copies issued before
// the programmatic-dependent-launch wait (they do not depend on the previous
// kernel).
//
// Staged rows (bf16 input, or an input normalised here): one warp per token
// reads the token's row with all of a lane's loads in flight, and writes it
// to shared memory as f32, [pass][H + 4] (the pad puts consecutive tokens'
// 16-byte reads in distinct banks). With in_norm_w the layer input x is the
// un-normalised hidden state: the warp first computes the token's RMSNorm
// scale, the staged values are bf16(x * scale * w) (the post-attention norm
// the reference runs ahead of the router, rms_norm_reduced,
// shaders.metal:1176-1213), and the CTAs together write those rows to ws.xn,
// the expert kernels' input. The weights are converted once to f32 rows in
// shared memory when they fit (else read as bf16, chunk by chunk as they
// land), padded so that a warp's 4 weight rows and 8 token rows fall in
// distinct banks; a chain step is 16 columns, the next step's reads issued
// before the current fmas.
// f32 input without a norm is staged per 256-column chunk instead,
// double-buffered.
//
// Routing and the group plan: each CTA counts itself in ticket[0] (a release
// add) once its logits are written; the first NR = ceil(T / kRtRows) CTAs (at
// most kRtRouteCtas, so the other CTAs always find SM slots) wait, bounded,
// for ticket[0] == gridDim.x, route one token per warp (route_token: the
// exact slot order of routing_top_k_iter, math.rs:746-765), and build the
// layer-major plan (unique experts ascending, routes in route order inside
// each group, the shared expert as group 0): directly when NR is 1, else the
// last of them (counted in ticket[1]); with the pipelined expert kernels,
// which build the plan themselves from the route ids (plan.cuh), there is no
// plan here. The last routing CTA resets both counters for the next launch.
constexpr int kRtRows = 8;
constexpr int kRtThreads = 32 * kRtRows;
constexpr uint32_t kRtTokPass = 32;
constexpr uint32_t kRtChunk = 256;
constexpr uint32_t kRtXStride = kRtChunk + 4;  // padded f32 row of a staged chunk
constexpr uint32_t kRtMaxChunks = 64;          // hidden <= 16384
constexpr uint32_t kRtRouteCtas = 64;
constexpr size_t kRtStageBudget = 216 * 1024;  // weights + staged token rows of one pass
constexpr int kRtVecs = static_cast<int>(kRtTokPass * kRtChunk / 4 / kRtThreads);  // float4 per thread per chunk
constexpr uint32_t kRtWarpPlanRoutes = 256;    // plans of at most this many routes are built by one warp
constexpr uint32_t kRtBlk = 2048;              // columns of a token row held in registers while staging

// router rows per CTA for hidden size H: all kRtRows warps when their bf16
// rows leave room for a staged token row, else half
__host__ __device__ inline uint32_t rt_rows_per_cta(uint32_t H) { return H <= 8192 ? kRtRows : kRtRows / 2; }

struct RtSmem {
    size_t w_bytes, wf_bytes, x_bytes, nw_bytes, total;
    uint32_t pass;    // tokens per pass
    uint32_t stride;  // floats per staged row (staged rows)
};
__host__ __device__ inline RtSmem rt_smem_layout(uint32_t T, uint32_t H, uint32_t E, uint32_t K, bool staged_rows,
                                                  bool norm) {
    RtSmem s;
    s.nw_bytes = norm ? static_cast<size_t>(H) * 4 : 0;  // the input norm's weights
    const size_t rpc = rt_rows_per_cta(H);
    s.w_bytes = (rpc * (H + 8) * 2 + 127) / 128 * 128;
    s.wf_bytes = 0;
    if (staged_rows) {
        if (rpc * (H + 4) * 4 + s.w_bytes <= 100 * 1024) s.wf_bytes = rpc * (H + 4) * 4;
        s.stride = H + 4;
        const size_t row = static_cast<size_t>(s.stride) * 4;
        const size_t used = s.w_bytes + s.wf_bytes + s.nw_bytes;
        size_t pass = used < kRtStageBudget ? (kRtStageBudget - used) / row : 1;
        if (pass < 1) pass = 1;
        if (pass > kRtTokPass) pass = kRtTokPass;
        if (pass > T) pass = T;
        s.pass = static_cast<uint32_t>(pass);
        s.x_bytes = pass * row;
    } else {
        s.stride = 0;
        s.pass = kRtTokPass;
        s.x_bytes = static_cast<size_t>(2) * kRtTokPass * kRtXStride * 4;
    }
    const size_t stage = s.w_bytes + s.wf_bytes + s.x_bytes + s.nw_bytes;
    const size_t plan = (3ull * E + 2ull * T * K + 32) * 4;
    const size_t route = static_cast<size_t>(kRtRows) * ((E + 3) & ~3u) * 4;
    size_t m = stage > plan ? stage : plan;
    s.total = m > route ? m : route;
    return s;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// atomic adds at gpu scope: release (the CTA's writes ordered before it by
// the preceding __syncthreads are visible to an acquirer that reads the
// count), and acquire-release (also sees the writes of the CTAs that counted
// before)
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

template <typename T>
__device__ __forceinline__ float4 rt_load4(const T* p, size_t i);
template <>
__device__ __forceinline__ float4 rt_load4<float>(const float* p, size_t i) {
    return *reinterpret_cast<const float4*>(p + i);
}
template <>
__device__ __forceinline__ float4 rt_load4<uint16_t>(const uint16_t* p, size_t i) {
    const uint2 u = *reinterpret_cast<const uint2*>(p + i);
    return make_float4(bf16_bits_to_f32(u.x & 0xffffu), bf16_bits_to_f32(u.x >> 16), bf16_bits_to_f32(u.y & 0xffffu),
                       bf16_bits_to_f32(u.y >> 16));
}

__device__ __forceinline__ float bf16_round(float v) { return bf16_bits_to_f32(f32_to_bf16_bits(v)); }

// acc = fma(w[c], x[c], acc) for c = 0..H-1 in order, f32 weights and
// activations in shared memory (H a multiple of 16). A step is 16 columns;
// the next step's reads are issued before the current 16 fmas, which take
// longer than a shared-memory read's latency.
__device__ __forceinline__ float rt_chain_f32(const float* __restrict__ wr, const float* __restrict__ xr, uint32_t H) {
    float acc = 0.f;
    float4 a[4], b[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        a[q] = *reinterpret_cast<const float4*>(wr + 4 * q);
        b[q] = *reinterpret_cast<const float4*>(xr + 4 * q);
    }
    for (uint32_t c = 16;; c += 16) {
        const uint32_t cn = c < H ? c : 0u;  // the last step re-reads column 0, unused
        float4 na[4], nb[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            na[q] = *reinterpret_cast<const float4*>(wr + cn + 4 * q);
            nb[q] = *reinterpret_cast<const float4*>(xr + cn + 4 * q);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            acc = fmaf(a[q].x, b[q].x, acc);
            acc = fmaf(a[q].y, b[q].y, acc);
            acc = fmaf(a[q].z, b[q].z, acc);
            acc = fmaf(a[q].w, b[q].w, acc);
        }
        if (c >= H) break;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            a[q] = na[q];
            b[q] = nb[q];
        }
    }
    return acc;
}

// the same chain over columns [c0, ce) with bf16 weights
__device__ __forceinline__ float rt_chain_bf16w(const uint16_t* __restrict__ wr, const float* __restrict__ xr,
                                                uint32_t c0, uint32_t ce, float acc) {
#pragma unroll 4
    for (uint32_t c = c0; c < ce; c += 8) {
        const uint4 q = *reinterpret_cast<const uint4*>(wr + c);
        const float4 a = *reinterpret_cast<const float4*>(xr + c);
        const float4 b = *reinterpret_cast<const float4*>(xr + c + 4);
        acc = fmaf(__uint_as_float(q.x << 16), a.x, acc);
        acc = fmaf(__uint_as_float(q.x & 0xffff0000u), a.y, acc);
        acc = fmaf(__uint_as_float(q.y << 16), a.z, acc);
        acc = fmaf(__uint_as_float(q.y & 0xffff0000u), a.w, acc);
        acc = fmaf(__uint_as_float(q.z << 16), b.x, acc);
        acc = fmaf(__uint_as_float(q.z & 0xffff0000u), b.y, acc);
        acc = fmaf(__uint_as_float(q.w << 16), b.z, acc);
        acc = fmaf(__uint_as_float(q.w & 0xffff0000u), b.w, acc);
    }
    return acc;
}

// Layer-major group plan of the R = T*K routes, built by one warp: per-expert
// counts in shared memory, an exclusive scan over the experts (a lane owns a
// contiguous block of them), then the routes placed 32 at a time in route
// order, lanes of the same expert ranked by __match_any_sync and a running
// count per expert. Experts come out ascending and each expert's routes in
// route order, the plan the block version builds. Loops stay rolled: the plan
// runs once per launch, so its code size is its cost. `gs` is shared scratch
// of 2 * (e_hi - e_lo) + 1 words.
__device__ __noinline__ void plan_warp(uint32_t T, uint32_t K, uint32_t E, uint32_t e_lo, uint32_t e_hi,
                                       bool has_shared, const MoeWs& ws, uint32_t* gs) {
    const int lane = threadIdx.x & 31;
    const uint32_t R = T * K, EL = e_hi - e_lo;
    uint32_t* cnt = gs;       // [EL] counts, then starts
    uint32_t* run = gs + EL;  // [EL] routes of each expert placed so far
#pragma unroll 1
    for (uint32_t e = lane; e < EL; e += 32) cnt[e] = run[e] = 0;
    __syncwarp();
#pragma unroll 1
    for (uint32_t r = lane; r < R; r += 32) {
        const uint32_t e = __ldcg(ws.route_ids + r);
        if (e >= e_lo && e < e_hi) atomicAdd(&cnt[e - e_lo], 1u);
    }
    __syncwarp();
    // exclusive scans of the counts and of the used flags over the experts
    const uint32_t per = (EL + 31) / 32, lo = min(lane * per, EL), hi = min(lo + per, EL);
    uint32_t routes = 0, used = 0;
#pragma unroll 1
    for (uint32_t e = lo; e < hi; ++e) {
        routes += cnt[e];
        used += cnt[e] ? 1u : 0u;
    }
    uint32_t r_incl = routes, u_incl = used;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t a = __shfl_up_sync(kFull, r_incl, o), b = __shfl_up_sync(kFull, u_incl, o);
        if (lane >= o) {
            r_incl += a;
            u_incl += b;
        }
    }
    const uint32_t U = __shfl_sync(kFull, u_incl, 31);
    const uint32_t shared_groups = has_shared ? 1u : 0u;
    const uint32_t routed_base = has_shared ? T : 0u;  // grouped positions taken by the shared group
    uint32_t start = r_incl - routes, g = u_incl - used;
#pragma unroll 1
    for (uint32_t e = lo; e < hi; ++e) {
        const uint32_t c = cnt[e];
        if (c) {
            ws.group_expert[shared_groups + g] = e;
            ws.group_start[shared_groups + g] = routed_base + start;
            ws.group_count[shared_groups + g] = c;
            ++g;
        }
        cnt[e] = start;
        start += c;
    }
    __syncwarp();
#pragma unroll 1
    for (uint32_t r0 = 0; r0 < R; r0 += 32) {
        const uint32_t r = r0 + lane;
        const uint32_t e = r < R ? __ldcg(ws.route_ids + r) : 0xffffffffu;
        const bool mine = e >= e_lo && e < e_hi;
        const uint32_t peers = __match_any_sync(kFull, mine ? e : 0xffffffffu);
        if (mine) {
            const uint32_t el = e - e_lo;
            const uint32_t pos = routed_base + cnt[el] + run[el] + __popc(peers & ((1u << lane) - 1u));
            ws.group_routes[pos] = r;
            ws.group_tokens[pos] = r / K;
        }
        __syncwarp();
        if (mine && (peers >> lane) == 1u) run[e - e_lo] += __popc(peers);  // the group's highest lane
        __syncwarp();
    }
    if (has_shared) {
#pragma unroll 1
        for (uint32_t t = lane; t < T; t += 32) {
            ws.group_routes[t] = R + t;
            ws.group_tokens[t] = t;
        }
        if (lane == 0) {
            ws.group_expert[0] = E;
            ws.group_start[0] = 0;
            ws.group_count[0] = T;
        }
    }
    if (lane == 0) *ws.num_groups = U + shared_groups;
}

template <typename XT>
__global__ void __launch_bounds__(kRtThreads)
moe_router_kernel(const XT* __restrict__ x, uint32_t T, uint32_t H, uint32_t E, uint32_t K,
                  uint32_t normalization, float routed_scale, const uint16_t* __restrict__ router_w,
                  const uint16_t* __restrict__ shared_gate_w, int has_shared, uint32_t e_lo, uint32_t e_hi,
                  uint32_t* ep_epoch, const float* __restrict__ in_norm_w, float in_eps,
                  const float* __restrict__ router_bias, uint32_t max_group, uint32_t build_plan, MoeWs ws) {
    extern __shared__ __align__(128) unsigned char rt_smem[];
    __shared__ __align__(8) uint64_t bars[kRtMaxChunks];
    __shared__ __align__(8) uint64_t nbar;  // the norm weights
    __shared__ uint32_t cta_flag;  // plan CTA selection
    __shared__ uint32_t failed;    // a bounded wait expired
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool staged_rows = sizeof(XT) == 2 || in_norm_w != nullptr;
    const RtSmem SL = rt_smem_layout(T, H, E, K, staged_rows, in_norm_w != nullptr);
    uint16_t* w_s = reinterpret_cast<uint16_t*>(rt_smem);
    float* wf_s = reinterpret_cast<float*>(rt_smem + SL.w_bytes);
    float* x_s = reinterpret_cast<float*>(rt_smem + SL.w_bytes + SL.wf_bytes);
    float* nw_s = reinterpret_cast<float*>(rt_smem + SL.w_bytes + SL.wf_bytes + SL.x_bytes);
    const uint32_t nrows = E + (shared_gate_w ? 1u : 0u);
    const uint32_t rpc = rt_rows_per_cta(H);
    const uint32_t row0 = blockIdx.x * rpc;
    const uint32_t rows_here = min(nrows - row0, rpc);
    const uint32_t nchunks = (H + kRtChunk - 1) / kRtChunk;

    // weights: the CTA's router rows (contiguous) in one bulk copy, the gate
    // row in another; with f32 weight rows the chains start once all have
    // landed (bars[0]), otherwise chunk by chunk (bars[k] per 256 columns).
    // The input norm's weights land on nbar.
    if (threadIdx.x == 0) {
        failed = 0;
        if (in_norm_w) {
            mbar_init(&nbar, 1);
            fence_mbar_init();
            mbar_arrive_expect_tx(&nbar, H * 4);
            bulk_load(nw_s, in_norm_w, H * 4, &nbar);
        }
        const uint32_t router_rows = row0 < E ? min(E - row0, rows_here) : 0u;
        if (SL.wf_bytes) {
            mbar_init(&bars[0], 1);
            fence_mbar_init();
            mbar_arrive_expect_tx(&bars[0], rows_here * H * 2);
            if (router_rows) bulk_load(w_s, router_w + static_cast<size_t>(row0) * H, router_rows * H * 2, &bars[0]);
            if (router_rows < rows_here)
                bulk_load(w_s + static_cast<size_t>(router_rows) * H, shared_gate_w, H * 2, &bars[0]);
        } else {
            for (uint32_t k = 0; k < nchunks; ++k) mbar_init(&bars[k], 1);
            fence_mbar_init();
            for (uint32_t k = 0; k < nchunks; ++k) {
                const uint32_t c0 = k * kRtChunk, cw = min(kRtChunk, H - c0);
                mbar_arrive_expect_tx(&bars[k], rows_here * cw * 2);
                for (uint32_t r = 0; r < rows_here; ++r) {
                    const uint32_t row = row0 + r;
                    const uint16_t* src = (row < E ? router_w + static_cast<size_t>(row) * H : shared_gate_w) + c0;
                    bulk_load(w_s + static_cast<size_t>(r) * (H + 8) + c0, src, cw * 2, &bars[k]);
                }
            }
        }
    }
    pdl_wait();
    __syncthreads();  // `failed` initialised

    auto wait_chunk = [&](uint32_t k) {
        if (!failed && !mbar_wait_bounded(&bars[k], 0, kPipeWaitNs)) {
            failed = 1;
            latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
        }
    };
    auto write_logit = [&](uint32_t t, uint32_t r, float acc) {
        const uint32_t row = row0 + r;
        if (row < E)
            ws.logits[static_cast<size_t>(t) * E + row] = acc;
        else
            ws.shared_logit[t] = acc;
    };

    if (staged_rows) {
        if (in_norm_w && !failed && !mbar_wait_bounded(&nbar, 0, kPipeWaitNs)) {
            failed = 1;
            latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
        }
        for (uint32_t t0 = 0; t0 < T; t0 += SL.pass) {
            const uint32_t tp = min(T - t0, SL.pass);
            if (t0 > 0) __syncthreads();  // the previous pass's chains are done with the rows
            // One warp per token reads the row once per kRtBlk columns into
            // registers (a whole row at hidden sizes up to kRtBlk), takes the
            // RMSNorm scale from them (the formula of rms_norm_rows_kernel:
            // 1 / sqrt(mean(x^2) + eps)) and writes the row as f32
            // (bf16-rounded when normalised here); the normalised row also
            // goes to ws.xn from CTA t mod grid.
            for (uint32_t tt = warp; tt < tp; tt += kRtRows) {
                const uint32_t t = t0 + tt;
                const XT* xr = x + static_cast<size_t>(t) * H;
                float* dst = x_s + static_cast<size_t>(tt) * SL.stride;
                const bool owner = in_norm_w && t % gridDim.x == blockIdx.x;
                float4 v[kRtBlk / 128];
                auto load_blk = [&](uint32_t c0) {
#pragma unroll
                    for (int j = 0; j < static_cast<int>(kRtBlk / 128); ++j) {
                        const uint32_t c = c0 + j * 128 + lane * 4;
                        v[j] = c < H ? rt_load4<XT>(xr, c) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                };
                float sc = 1.f;
                if (in_norm_w) {
                    float ss = 0.f;
                    for (uint32_t c0 = 0; c0 < H; c0 += kRtBlk) {
                        load_blk(c0);
#pragma unroll
                        for (int j = 0; j < static_cast<int>(kRtBlk / 128); ++j)
                            ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
                    }
                    ss = warp_sum(ss);
                    sc = 1.0f / sqrtf(ss / static_cast<float>(H) + in_eps);
                }
                for (uint32_t c0 = 0; c0 < H; c0 += kRtBlk) {
                    if (!in_norm_w || H > kRtBlk) load_blk(c0);  // else the row is still in v
#pragma unroll
                    for (int j = 0; j < static_cast<int>(kRtBlk / 128); ++j) {
                        const uint32_t c = c0 + j * 128 + lane * 4;
                        if (c >= H) continue;
                        float4 o = v[j];
                        if (in_norm_w) {
                            const float4 n = *reinterpret_cast<const float4*>(nw_s + c);
                            o = make_float4(bf16_round(o.x * sc * n.x), bf16_round(o.y * sc * n.y),
                                            bf16_round(o.z * sc * n.z), bf16_round(o.w * sc * n.w));
                            if (owner) {
                                const uint2 pk = make_uint2(f32_to_bf16_bits(o.x) | (f32_to_bf16_bits(o.y) << 16),
                                                            f32_to_bf16_bits(o.z) | (f32_to_bf16_bits(o.w) << 16));
                                *reinterpret_cast<uint2*>(ws.xn + static_cast<size_t>(t) * H + c) = pk;
                            }
                        }
                        *reinterpret_cast<float4*>(dst + c) = o;
                    }
                }
            }
            if (SL.wf_bytes && t0 == 0) {
                // the weights have landed: f32 copy of the rows, once
                wait_chunk(0);
                const uint32_t vpr = H / 8, nvec = rows_here * vpr;
                for (uint32_t i = threadIdx.x; i < nvec; i += kRtThreads) {
                    const uint32_t r = i / vpr, c = (i - r * vpr) * 8;
                    const uint4 q = *reinterpret_cast<const uint4*>(w_s + static_cast<size_t>(i) * 8);
                    float4* d = reinterpret_cast<float4*>(wf_s + static_cast<size_t>(r) * (H + 4) + c);
                    d[0] = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xffff0000u),
                                       __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xffff0000u));
                    d[1] = make_float4(__uint_as_float(q.z << 16), __uint_as_float(q.z & 0xffff0000u),
                                       __uint_as_float(q.w << 16), __uint_as_float(q.w & 0xffff0000u));
                }
            }
            __syncthreads();
            // a warp runs 4 rows x 8 tokens (its weight reads are 4 distinct
            // 16-byte words, its activation reads 8): row group rg, token group tg
            const uint32_t rgroups = rpc / 4, rg = warp % rgroups, tg = warp / rgroups;
            const uint32_t r = rg * 4 + (lane >> 3), tt = tg * 8 + (lane & 7);
            if (r < rows_here && tt < tp) {
                const float* xr = x_s + static_cast<size_t>(tt) * SL.stride;
                float acc;
                if (SL.wf_bytes) {
                    acc = rt_chain_f32(wf_s + static_cast<size_t>(r) * (H + 4), xr, H);
                } else {
                    acc = 0.f;
                    const uint16_t* wrow = w_s + static_cast<size_t>(r) * (H + 8);
                    for (uint32_t k = 0; k < nchunks; ++k) {
                        wait_chunk(k);
                        acc = rt_chain_bf16w(wrow, xr, k * kRtChunk, min(H, (k + 1) * kRtChunk), acc);
                    }
                }
                write_logit(t0 + tt, r, acc);
            }
        }
    } else {
        // ---- f32 token rows (f32 input, no norm): 256-column chunks, double-buffered
        const uint16_t* wrow = w_s + static_cast<size_t>(warp) * (H + 8);
        float4 reg[kRtVecs];
        auto load_regs = [&](uint32_t t0, uint32_t tp, uint32_t k) {
            const uint32_t c0 = k * kRtChunk, cw = min(kRtChunk, H - c0);
            const uint32_t vpr = cw / 4, total = tp * vpr;
#pragma unroll
            for (int j = 0; j < kRtVecs; ++j) {
                const uint32_t i = threadIdx.x + j * kRtThreads;
                if (i < total) {
                    const uint32_t tt = i / vpr, cc = (i - tt * vpr) * 4;
                    reg[j] = rt_load4<XT>(x, static_cast<size_t>(t0 + tt) * H + c0 + cc);
                }
            }
        };
        auto store_regs = [&](uint32_t tp, uint32_t k, float* dst) {
            const uint32_t c0 = k * kRtChunk, cw = min(kRtChunk, H - c0);
            const uint32_t vpr = cw / 4, total = tp * vpr;
#pragma unroll
            for (int j = 0; j < kRtVecs; ++j) {
                const uint32_t i = threadIdx.x + j * kRtThreads;
                if (i < total) {
                    const uint32_t tt = i / vpr, cc = (i - tt * vpr) * 4;
                    *reinterpret_cast<float4*>(dst + tt * kRtXStride + cc) = reg[j];
                }
            }
        };
        const uint32_t xbuf = kRtTokPass * kRtXStride;  // floats per staging buffer
        for (uint32_t t0 = 0; t0 < T; t0 += kRtTokPass) {
            const uint32_t tp = min(T - t0, kRtTokPass);
            const bool mine = static_cast<uint32_t>(warp) < rows_here && static_cast<uint32_t>(lane) < tp;
            if (t0 > 0) __syncthreads();
            load_regs(t0, tp, 0);
            store_regs(tp, 0, x_s);
            __syncthreads();
            float acc = 0.f;
            for (uint32_t k = 0; k < nchunks; ++k) {
                if (k + 1 < nchunks) load_regs(t0, tp, k + 1);
                if (mine) {
                    wait_chunk(k);
                    const uint32_t c0 = k * kRtChunk, cw = min(kRtChunk, H - c0);
                    const uint16_t* wr = wrow + c0;
                    const float* xr = x_s + (k & 1u) * xbuf + lane * kRtXStride;
#pragma unroll 4
                    for (uint32_t c = 0; c < cw; c += 8) {
                        const uint4 q = *reinterpret_cast<const uint4*>(wr + c);
                        const float4 a = *reinterpret_cast<const float4*>(xr + c);
                        const float4 b = *reinterpret_cast<const float4*>(xr + c + 4);
                        acc = fmaf(__uint_as_float(q.x << 16), a.x, acc);
                        acc = fmaf(__uint_as_float(q.x & 0xffff0000u), a.y, acc);
                        acc = fmaf(__uint_as_float(q.y << 16), a.z, acc);
                        acc = fmaf(__uint_as_float(q.y & 0xffff0000u), a.w, acc);
                        acc = fmaf(__uint_as_float(q.z << 16), b.x, acc);
                        acc = fmaf(__uint_as_float(q.z & 0xffff0000u), b.y, acc);
                        acc = fmaf(__uint_as_float(q.w << 16), b.z, acc);
                        acc = fmaf(__uint_as_float(q.w & 0xffff0000u), b.w, acc);
                    }
                }
                if (k + 1 < nchunks) store_regs(tp, k + 1, x_s + ((k + 1) & 1u) * xbuf);
                __syncthreads();
            }
            if (mine) write_logit(t0 + lane, warp, acc);
        }
    }

    // ---- arrival; the routing CTAs wait for every CTA's logits
    __syncthreads();
    if (threadIdx.x == 0) red_add_release_gpu(&ws.ticket[0], 1u);
    const uint32_t route_ctas = min(min(gridDim.x, kRtRouteCtas), (T + kRtRows - 1) / kRtRows);
    auto drain = [&]() {  // after an expired wait, let this CTA's own copies land (bounded) before it exits
        if (threadIdx.x == 0 && failed) {
            for (uint32_t k = 0; k < (SL.wf_bytes ? 1u : nchunks); ++k) mbar_wait_bounded(&bars[k], 0, kPipeWaitNs);
            if (in_norm_w) mbar_wait_bounded(&nbar, 0, kPipeWaitNs);
        }
    };
    if (blockIdx.x >= route_ctas) {
        drain();
        return;
    }
    if (threadIdx.x == 0) {
        const uint64_t t_start = global_ns();
        while (ld_acquire_gpu(&ws.ticket[0]) < gridDim.x) {
            if (global_ns() - t_start > kPipeWaitNs) {
                latch_status(ws.status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
    // every CTA of this grid has started: the expert kernel may be scheduled
    // now and run its prologue under the routing; it reads the plan only after
    // griddepcontrol.wait, i.e. after this grid completes
    pdl_launch_dependents();
    {
        const uint32_t Ep = (E + 3) & ~3u;
        float* s = reinterpret_cast<float*>(rt_smem) + warp * Ep;  // the staging area is free now
        for (uint32_t t = blockIdx.x * kRtRows + warp; t < T; t += route_ctas * kRtRows) {
            stage_logits_warp(ws.logits + static_cast<size_t>(t) * E, E, s);
            route_token(s, E, K, normalization, routed_scale, ws.route_ids + static_cast<size_t>(t) * K,
                        ws.route_w + static_cast<size_t>(t) * K, ws.status, router_bias,
                        ws.logits + static_cast<size_t>(t) * E);
        }
    }
    __syncthreads();
    if (route_ctas > 1) {
        if (threadIdx.x == 0) cta_flag = (atom_add_acq_rel_gpu(&ws.ticket[1], 1u) == route_ctas - 1) ? 1u : 0u;
        __syncthreads();
        if (!cta_flag) {
            drain();
            return;
        }
    }

    // group plan (unless the pipelined expert kernels build their own from
    // the route ids); shared memory reuses the staging area
    uint32_t* plan_smem = reinterpret_cast<uint32_t*>(rt_smem);
    if (!build_plan) {
    } else if (T * K <= kRtWarpPlanRoutes && max_group == 0) {
        if (warp == 0) plan_warp(T, K, E, e_lo, e_hi, has_shared != 0, ws, plan_smem);
    } else {
        plan_block(T, K, E, e_lo, e_hi, has_shared != 0, max_group, ws.route_ids,
                   PlanOut{ws.group_expert, ws.group_start, ws.group_count, ws.group_tokens, ws.group_routes,
                           ws.num_groups},
                   plan_smem);
    }
    if (threadIdx.x == 0) {
        ws.ticket[0] = 0;  // ready for the next launch
        ws.ticket[1] = 0;
        if (ep_epoch) *ep_epoch += 1u;  // this layer's expert-parallel exchange epoch
    }
    drain();
}

// ---------------------------------------------------------------- kernel 2
constexpr int kUpThreads = 128;
constexpr int kUpRowsPerWarp = 2;  // intermediate indices per warp (gate+up = 4 rows)
constexpr int kUpRowsPerCta = kUpRowsPerWarp * (kUpThreads / 32);

template <typename XT, int NT>
__global__ void __launch_bounds__(kUpThreads, 3)
moe_expert_up_kernel(const XT* __restrict__ x, uint32_t E, const uint8_t* __restrict__ experts,
                     const uint8_t* __restrict__ shared_slot, MoeLayoutDev L, MoeWs ws) {
    extern __shared__ __align__(16) float smem[];
    const uint32_t g = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    pdl_wait();
    if (g >= *ws.num_groups) return;
    const uint32_t e = ws.group_expert[g];
    const uint32_t start = ws.group_start[g], n = ws.group_count[g];
    const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * L.expert_bytes;
    const uint32_t H = L.hidden, I = L.inter;
    const uint32_t chunks = H >> 5;
    float* xs = smem;
    float* xe = xs + NT * H;
    float* xo = xe + NT * chunks;

    const Q4Geom geom{I, H, (H + L.group - 1) / L.group, chunks, L.cpg_shift_h};
    const uint32_t i0 = blockIdx.x * kUpRowsPerCta + warp * kUpRowsPerWarp;
    const uint8_t* pk[2 * kUpRowsPerWarp];
    const uint16_t* ps[2 * kUpRowsPerWarp];
    const uint16_t* pb[2 * kUpRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kUpRowsPerWarp; ++r) {
        const uint32_t i = i0 + r;
        const bool ok = i < I;
        const size_t prow = static_cast<size_t>(i) * (H / 2);
        const size_t srow = static_cast<size_t>(i) * geom.gpr;
        pk[r] = ok ? slot + L.off[0] + prow : nullptr;
        ps[r] = reinterpret_cast<const uint16_t*>(slot + L.off[1]) + srow;
        pb[r] = reinterpret_cast<const uint16_t*>(slot + L.off[2]) + srow;
        pk[kUpRowsPerWarp + r] = ok ? slot + L.off[3] + prow : nullptr;
        ps[kUpRowsPerWarp + r] = reinterpret_cast<const uint16_t*>(slot + L.off[4]) + srow;
        pb[kUpRowsPerWarp + r] = reinterpret_cast<const uint16_t*>(slot + L.off[5]) + srow;
    }
    Q4RowFrag<32, 2 * kUpRowsPerWarp, 2> frag;
    for (uint32_t p0 = 0; p0 < n; p0 += NT) {
        const int nt = static_cast<int>(min(n - p0, static_cast<uint32_t>(NT)));
        frag.load(pk, ps, pb, geom, 0);  // weights in flight while x is staged
        __syncthreads();
        stage_x_fast<XT>(x, H, ws.group_tokens + start + p0, nt, H, xs, xe, xo);
        float acc[2 * kUpRowsPerWarp][NT];
        q4_rows_finish<32, 2 * kUpRowsPerWarp, 2, NT>(frag, pk, ps, pb, geom, xs, xe, xo, nt, acc);
#pragma unroll
        for (int r = 0; r < kUpRowsPerWarp; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float gs = warp_sum(acc[r][t]);
                const float us = warp_sum(acc[kUpRowsPerWarp + r][t]);
                if (lane == 0 && t < nt && i0 + r < I) {
                    const uint32_t route = ws.group_routes[start + p0 + t];
                    ws.h[static_cast<size_t>(route) * I + i0 + r] = gs / (1.0f + expf(-gs)) * us;
                }
            }
        }
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------- kernel 3
constexpr int kDownThreads = 128;
constexpr int kDownRowsPerGroup = 4;  // rows per lane group

template <int LPR, int NT>
__global__ void __launch_bounds__(kDownThreads, 4)
moe_expert_down_kernel(uint32_t E, const uint8_t* __restrict__ experts, const uint8_t* __restrict__ shared_slot,
                       MoeLayoutDev L, MoeWs ws) {
    extern __shared__ __align__(16) float smem[];
    constexpr int kGroups = 32 / LPR;
    constexpr int kRowsPerCta = kDownRowsPerGroup * kGroups * (kDownThreads / 32);
    const uint32_t g = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane / LPR;
    const uint32_t H = L.hidden, I = L.inter;
    const uint32_t chunks = I >> 5;
    const Q4Geom geom{H, I, (I + L.group - 1) / L.group, chunks, L.cpg_shift_i};

    // The group plan was written by the router kernel, which completed before
    // the up kernel could start; weights do not depend on the up kernel.
    const uint32_t ng = *ws.num_groups;
    if (g >= ng) {
        pdl_wait();
        return;
    }
    const uint32_t e = ws.group_expert[g];
    const uint32_t start = ws.group_start[g], n = ws.group_count[g];
    const uint8_t* slot = e >= E ? shared_slot : experts + static_cast<size_t>(e) * L.expert_bytes;
    float* xs = smem;
    float* xe = xs + NT * I;
    float* xo = xe + NT * chunks;
    const uint32_t r0 = blockIdx.x * kRowsPerCta + (warp * kGroups + sub) * kDownRowsPerGroup;
    const uint8_t* pk[kDownRowsPerGroup];
    const uint16_t* ps[kDownRowsPerGroup];
    const uint16_t* pb[kDownRowsPerGroup];
#pragma unroll
    for (int r = 0; r < kDownRowsPerGroup; ++r) {
        const uint32_t row = r0 + r;
        pk[r] = row < H ? slot + L.off[6] + static_cast<size_t>(row) * (I / 2) : nullptr;
        ps[r] = reinterpret_cast<const uint16_t*>(slot + L.off[7]) + static_cast<size_t>(row) * geom.gpr;
        pb[r] = reinterpret_cast<const uint16_t*>(slot + L.off[8]) + static_cast<size_t>(row) * geom.gpr;
    }
    Q4RowFrag<LPR, kDownRowsPerGroup, 1> frag;
    frag.load(pk, ps, pb, geom, 0);  // down weights do not depend on the up kernel
    pdl_wait();
    for (uint32_t p0 = 0; p0 < n; p0 += NT) {
        const int nt = static_cast<int>(min(n - p0, static_cast<uint32_t>(NT)));
        if (p0 > 0) frag.load(pk, ps, pb, geom, 0);
        __syncthreads();
        stage_x_fast<float>(ws.h, I, ws.group_routes + start + p0, nt, I, xs, xe, xo);
        float acc[kDownRowsPerGroup][NT];
        q4_rows_finish<LPR, kDownRowsPerGroup, 1, NT>(frag, pk, ps, pb, geom, xs, xe, xo, nt, acc);
#pragma unroll
        for (int r = 0; r < kDownRowsPerGroup; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float s = group_sum<LPR>(acc[r][t]);
                if ((lane & (LPR - 1)) == 0 && t < nt && r0 + r < H) {
                    const uint32_t route = ws.group_routes[start + p0 + t];
                    ws.y[static_cast<size_t>(route) * H + r0 + r] = s;
                }
            }
        }
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------- kernel 4
constexpr int kCombineMaxThreads = 256;
constexpr int kCombineVec = 4;  // float4 groups per thread: a piece is at most 4 * 256 * 4 columns

template <typename T>
__device__ __forceinline__ float4 load_act4(const T* p, size_t i);
template <>
__device__ __forceinline__ float4 load_act4<float>(const float* p, size_t i) {
    return *reinterpret_cast<const float4*>(p + i);
}
template <>
__device__ __forceinline__ float4 load_act4<uint16_t>(const uint16_t* p, size_t i) {
    const uint2 u = *reinterpret_cast<const uint2*>(p + i);
    return make_float4(bf16_bits_to_f32(u.x & 0xffffu), bf16_bits_to_f32(u.x >> 16), bf16_bits_to_f32(u.y & 0xffffu),
                       bf16_bits_to_f32(u.y >> 16));
}
template <typename T>
__device__ __forceinline__ void store_act4(T* p, size_t i, float4 v);
template <>
__device__ __forceinline__ void store_act4<float>(float* p, size_t i, float4 v) {
    *reinterpret_cast<float4*>(p + i) = v;
}
template <>
__device__ __forceinline__ void store_act4<uint16_t>(uint16_t* p, size_t i, float4 v) {
    uint2 u;
    u.x = f32_to_bf16_bits(v.x) | (static_cast<uint32_t>(f32_to_bf16_bits(v.y)) << 16);
    u.y = f32_to_bf16_bits(v.z) | (static_cast<uint32_t>(f32_to_bf16_bits(v.w)) << 16);
    *reinterpret_cast<uint2*>(p + i) = u;
}
__device__ __forceinline__ void fma4(float4& a, float w, const float4& b) {
    a.x += w * b.x;
    a.y += w * b.y;
    a.z += w * b.z;
    a.w += w * b.w;
}
__device__ __forceinline__ void add4(float4& a, const float4& b) {
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// CTA (t, y) combines columns [y*piece, (y+1)*piece) of token t, four
// consecutive columns per thread (float4). Per element the K routed outputs
// (weighted, in slot order) and the gated shared output are summed as the
// reference does, then the residual is added. Routes whose expert lies
// outside [e_lo, e_hi) belong to another rank and are skipped (their y rows
// were not written). With a next-layer norm the token's pieces form one
// thread-block cluster: each CTA's sum of squares is read by every CTA of the
// cluster over distributed shared memory, in piece order.
//
// kEP: expert-parallel combine. A CTA's partial (local routes plus, on the
// rank that holds it, the shared expert) goes to every other rank's receive
// buffer over peer memory (16-byte NVLink stores); after a CTA barrier
// thread d publishes it with a system-scope release of the epoch flag of
// (rank, token, piece) in rank d's flag array, then waits, bounded, for rank
// d's flag of this piece (relaxed polling, then an acquire fence); the output is
// residual + the world partials summed in rank order, identical on every
// rank. A wait that expires latches PBMOE_DEV_ERR_PEER_TIMEOUT and the
// missing partial counts as zero. Receive buffers alternate by epoch parity:
// a rank can run at most one layer ahead of another (its next partial waits
// for everyone's flags), so the parity a rank writes is never the one a
// slower rank is still reading.
template <typename OT, int KMAX, bool kEP>
__global__ void __launch_bounds__(kCombineMaxThreads)
moe_combine_kernel(uint32_t T, uint32_t H, uint32_t K, int has_shared, int has_gate, const OT* __restrict__ residual,
                   OT* __restrict__ out, const float* __restrict__ norm_w, OT* __restrict__ next_normed, float eps,
                   uint32_t e_lo, uint32_t e_hi, uint32_t piece, MoeWs ws, EpPeers ep) {
    __shared__ float red[kCombineMaxThreads / 32];
    __shared__ float wsh[KMAX];
    __shared__ float piece_ss;
    __shared__ uint32_t missing;
    const uint32_t t = blockIdx.x;
    const uint32_t cb = blockIdx.y * piece, ce = min(H, cb + piece);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    // Before the dependency wait: the routes, their weights and the shared
    // gate's logit (router outputs), the residual and the norm weights. This
    // grid is launched only after the up kernel passed its own wait, i.e.
    // after the router (and whatever wrote the residual before it)
    // completed; only the expert outputs y come from the grids still running.
    if (threadIdx.x < K) {
        const uint32_t e = __ldcg(ws.route_ids + static_cast<size_t>(t) * K + threadIdx.x);
        wsh[threadIdx.x] = (e >= e_lo && e < e_hi) ? __ldcg(ws.route_w + static_cast<size_t>(t) * K + threadIdx.x)
                                                   : 0.f;  // another rank's route
    }
    if (threadIdx.x == 0) missing = 0;
    float sw = 0.f;
    if (has_shared) sw = has_gate ? 1.0f / (1.0f + expf(-__ldcg(ws.shared_logit + t))) : 1.0f;
    float4 res[kCombineVec], nwv[kCombineVec];
#pragma unroll
    for (int j = 0; j < kCombineVec; ++j) {
        const uint32_t c = cb + 4 * (threadIdx.x + j * blockDim.x);
        res[j] = (c < ce && residual) ? load_act4<OT>(residual, static_cast<size_t>(t) * H + c) : zero;
        nwv[j] = (c < ce && norm_w) ? *reinterpret_cast<const float4*>(norm_w + c) : zero;
    }
    pdl_wait();
    // every CTA of this grid is resident: the next layer's first kernel may be
    // scheduled now and prefetch its weights while the combine runs (it reads
    // this kernel's outputs only after its own griddepcontrol.wait)
    pdl_launch_dependents();
    __syncthreads();
    const float* yt = ws.y + static_cast<size_t>(t) * K * H;
    const float* ysh = ws.y + (static_cast<size_t>(T) * K + t) * H;
    float4 v[kCombineVec];
#pragma unroll
    for (int j = 0; j < kCombineVec; ++j) {
        const uint32_t c = cb + 4 * (threadIdx.x + j * blockDim.x);
        float4 acc = zero;
        if (c < ce) {
            float4 yv[KMAX];
#pragma unroll
            for (int k = 0; k < KMAX; ++k)
                yv[k] = (static_cast<uint32_t>(k) < K && wsh[k] != 0.f)
                            ? __ldcg(reinterpret_cast<const float4*>(yt + static_cast<size_t>(k) * H + c))
                            : zero;
            const float4 sh = has_shared ? __ldcg(reinterpret_cast<const float4*>(ysh + c)) : zero;
#pragma unroll
            for (int k = 0; k < KMAX; ++k)
                if (static_cast<uint32_t>(k) < K) fma4(acc, wsh[k], yv[k]);
            fma4(acc, sw, sh);
        }
        v[j] = acc;
    }
    if constexpr (kEP) {
        const uint32_t epoch = __ldcg(ep.epoch);
        const uint32_t par = epoch & 1u;
        auto recv_row = [&](uint32_t rank_buf, uint32_t src) {  // partial of `src` in rank `rank_buf`'s buffer
            return ep.recv[rank_buf] + ((static_cast<size_t>(par) * ep.world + src) * ep.max_tokens + t) * H;
        };
        auto flag = [&](uint32_t rank_buf, uint32_t src) {
            return ep.flags[rank_buf] + (static_cast<size_t>(src) * ep.max_tokens + t) * kCombinePieces + blockIdx.y;
        };
        // 1. this rank's partial to every other rank
#pragma unroll
        for (int j = 0; j < kCombineVec; ++j) {
            const uint32_t c = cb + 4 * (threadIdx.x + j * blockDim.x);
            if (c < ce)
                for (uint32_t d = 0; d < ep.world; ++d)
                    if (d != ep.rank) *reinterpret_cast<float4*>(recv_row(d, ep.rank) + c) = v[j];
        }
        __syncthreads();
        // 2. thread d (d != rank) publishes to rank d and then waits for rank
        // d's partial of this piece: one system-scope release and one acquire
        // fence per peer, all peers in parallel
        if (threadIdx.x < ep.world && threadIdx.x != ep.rank) {
            st_release_sys(flag(threadIdx.x, ep.rank), epoch);
            const uint32_t* f = flag(ep.rank, threadIdx.x);
            const uint64_t t0 = global_ns();
            while (static_cast<int32_t>(ld_relaxed_sys(f) - epoch) < 0) {
                if (global_ns() - t0 > ep.timeout_ns) {
                    atomicOr(&missing, 1u << threadIdx.x);
                    if (ws.status) atomicOr(ws.status, PBMOE_DEV_ERR_PEER_TIMEOUT);
                    break;
                }
                __nanosleep(64);
            }
            fence_acq_rel_sys();
        }
        __syncthreads();
        // every rank's partial in rank order (peer data not cached: peers wrote it)
#pragma unroll
        for (int j = 0; j < kCombineVec; ++j) {
            const uint32_t c = cb + 4 * (threadIdx.x + j * blockDim.x);
            float4 m = zero;
            if (c < ce)
                for (uint32_t src = 0; src < ep.world; ++src) {
                    if (src == ep.rank)
                        add4(m, v[j]);
                    else if (!(missing & (1u << src)))
                        add4(m, __ldcv(reinterpret_cast<const float4*>(recv_row(ep.rank, src) + c)));
                }
            v[j] = m;
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kCombineVec; ++j) {
        const uint32_t c = cb + 4 * (threadIdx.x + j * blockDim.x);
        if (c < ce) {
            float4 o = res[j];
            add4(o, v[j]);
            store_act4<OT>(out, static_cast<size_t>(t) * H + c, o);
            ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
            v[j] = o;
        }
    }
    if (!norm_w) return;
    // the token's sum of squares: warps, then the CTA, then the cluster
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (uint32_t w = 0; w < blockDim.x / 32; ++w) s += red[w];
        piece_ss = s;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    float tot = 0.f;
    for (uint32_t r = 0; r < gridDim.y; ++r) tot += *cluster.map_shared_rank(&piece_ss, r);
    cluster.sync();  // no CTA leaves while another still reads its piece_ss
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(H) + eps);
#pragma unroll
    for (int j = 0; j < kCombineVec; ++j) {
        const uint32_t c = cb + 4 * (threadIdx.x + j * blockDim.x);
        if (c < ce) {
            const float4 nw = nwv[j];
            store_act4<OT>(next_normed, static_cast<size_t>(t) * H + c,
                           make_float4(v[j].x * scale * nw.x, v[j].y * scale * nw.y, v[j].z * scale * nw.z,
                                       v[j].w * scale * nw.w));
        }
    }
}

// ---------------------------------------------------------------- routing only
__global__ void route_topk_kernel(const float* __restrict__ logits, uint32_t T, uint32_t E, uint32_t K,
                                  uint32_t normalization, float routed_scale, uint32_t* ids, float* w,
                                  uint32_t* status, const float* __restrict__ bias) {
    extern __shared__ __align__(16) float rsm[];  // per warp: E logits (padded to 4)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t = blockIdx.x * (blockDim.x / 32) + warp;
    if (t >= T) return;
    const uint32_t Ep = (E + 3) & ~3u;
    float* s = rsm + warp * Ep;
    stage_logits_warp(logits + static_cast<size_t>(t) * E, E, s);
    route_token(s, E, K, normalization, routed_scale, ids + static_cast<size_t>(t) * K,
                w + static_cast<size_t>(t) * K, status, bias, logits + static_cast<size_t>(t) * E);
}

// ---------------------------------------------------------------- host side
cudaError_t moe_launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args,
                           bool pdl) {
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

size_t moe_router_smem(uint32_t T, uint32_t H, uint32_t E, uint32_t K) {
    const size_t a = rt_smem_layout(T, H, E, K, true, true).total, b = rt_smem_layout(T, H, E, K, false, false).total;
    return a > b ? a : b;
}

template <typename F>
static cudaError_t set_smem(F* fn, size_t bytes) {
    return cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bytes));
}

// CUDA-core gate/up kernel for layouts the tensor-core kernels do not take.
template <typename XT>
static cudaError_t moe_up_fallback_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl) {
    cudaError_t err;
    const uint32_t T = a.tokens, H = a.layout.hidden, I = a.layout.inter;
    uint32_t E = a.num_experts;
    MoeLayoutDev L = a.layout;
    MoeWs ws = a.ws;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    const uint32_t chunks = H >> 5;
    dim3 grid((I + kUpRowsPerCta - 1) / kUpRowsPerCta, gmax);
    const XT* x = static_cast<const XT*>(a.x);
    void* args[] = {(void*)&x, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
    if (T == 1) {
        const size_t smem = (1ull * H + 2ull * chunks) * sizeof(float);
        auto fn = moe_expert_up_kernel<XT, 1>;
        if ((err = set_smem(fn, smem)) != cudaSuccess) return err;
        return moe_launch_pdl(reinterpret_cast<const void*>(fn), grid, dim3(kUpThreads), smem, s, args, pdl);
    }
    const size_t smem = 4ull * (H + 2ull * chunks) * sizeof(float);
    auto fn = moe_expert_up_kernel<XT, 4>;
    if ((err = set_smem(fn, smem)) != cudaSuccess) return err;
    return moe_launch_pdl(reinterpret_cast<const void*>(fn), grid, dim3(kUpThreads), smem, s, args, pdl);
}

template <typename XT, typename OT>
static cudaError_t moe_layer_launch_t(const MoeLaunch& a, cudaStream_t s) {
    cudaError_t err;
    const uint32_t T = a.tokens, H = a.layout.hidden, I = a.layout.inter, E = a.num_experts, K = a.top_k;
    const int has_shared = a.shared_slot != nullptr;
    const int has_gate = a.shared_gate != nullptr;
    const uint32_t e_lo = a.expert_count ? a.expert_lo : 0u;
    const uint32_t e_hi = a.expert_count ? a.expert_lo + a.expert_count : E;
    MoeWs ws = a.ws;
    auto mark = [&](int i) -> cudaError_t {
        return a.phase_events ? cudaEventRecord(static_cast<cudaEvent_t>(a.phase_events[i]), s) : cudaSuccess;
    };
    const bool pdl = a.phase_events == nullptr;
    // the experts' input: x itself, or the router's normalised rows
    MoeLaunch ex = a;
    if (a.in_norm_w) {
        ex.x = ws.xn;
        ex.x_dtype = PBMOE_BF16;
    }
    const bool mx = a.layout.mxfp4 != 0;
    const bool mma = !mx && moe_mma_supported(a.layout);
    const bool pipe = mma && moe_pipe_supported(ex);
    // the pipelined kernels take at most 8 routes per group: larger batches
    // split each expert's routes into groups of 8; they build the plan
    // themselves from the route ids, the other expert kernels read the
    // router's
    uint32_t max_group = pipe && T > 8 ? 8u : 0u;
    uint32_t build_plan = pipe ? 0u : 1u;
    if ((err = mark(0)) != cudaSuccess) return err;
    // 1. router + routing + plan
    {
        const uint32_t nrows = E + (has_gate ? 1u : 0u);
        const uint32_t rpc = rt_rows_per_cta(H);
        dim3 grid((nrows + rpc - 1) / rpc);
        const size_t smem =
            rt_smem_layout(T, H, E, K, sizeof(XT) == 2 || a.in_norm_w != nullptr, a.in_norm_w != nullptr).total;
        auto fn = moe_router_kernel<XT>;
        if ((err = set_smem(fn, smem)) != cudaSuccess) return err;
        const XT* x = static_cast<const XT*>(a.x);
        uint32_t norm = a.normalization;
        float scale = a.routed_scale;
        const uint16_t* rw = a.router_w;
        const uint16_t* sg = a.shared_gate;
        uint32_t* ep_epoch = a.ep ? a.ep->epoch : nullptr;
        const float* inw = a.in_norm_w;
        float ineps = a.in_eps;
        const float* rbias = a.router_bias;
        void* args[] = {(void*)&x,    (void*)&T,     (void*)&H,  (void*)&E,  (void*)&K,
                        (void*)&norm, (void*)&scale, (void*)&rw, (void*)&sg, (void*)&has_shared,
                        (void*)&e_lo, (void*)&e_hi,  (void*)&ep_epoch, (void*)&inw, (void*)&ineps, (void*)&rbias,
                        (void*)&max_group, (void*)&build_plan, (void*)&ws};
        if ((err = moe_launch_pdl(reinterpret_cast<const void*>(fn), grid, dim3(kRtThreads), smem, s, args,
                              a.pdl && pdl)) != cudaSuccess)
            return err;
    }
    if ((err = mark(1)) != cudaSuccess) return err;
    const uint32_t gmax = (T * K < E ? T * K : E) + (has_shared ? 1u : 0u);
    MoeLayoutDev L = a.layout;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    // 2. gate/up/SwiGLU
    if (mx) {
        if ((err = moe_up_mxfp4_launch(ex, gmax, s, pdl)) != cudaSuccess) return err;
    } else if (pipe) {
        if ((err = moe_up_pipe_launch(ex, s, pdl)) != cudaSuccess) return err;
    } else if (mma) {
        if ((err = moe_up_mma_launch(ex, gmax, s, pdl)) != cudaSuccess) return err;
    } else {
        err = ex.x_dtype == PBMOE_BF16 ? moe_up_fallback_launch<uint16_t>(ex, gmax, s, pdl)
                                       : moe_up_fallback_launch<float>(ex, gmax, s, pdl);
        if (err != cudaSuccess) return err;
    }
    if ((err = mark(2)) != cudaSuccess) return err;
    // 3. down
    if (mx) {
        if ((err = moe_down_mxfp4_launch(a, gmax, s, pdl)) != cudaSuccess) return err;
    } else if (pipe) {
        if ((err = moe_down_pipe_launch(a, s, pdl)) != cudaSuccess) return err;
    } else if (mma) {
        if ((err = moe_down_mma_launch(a, gmax, s, pdl)) != cudaSuccess) return err;
    } else {
        const uint32_t chunks = I >> 5;
        void* args[] = {(void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
        const int lpr = chunks >= 32 ? 32 : (chunks >= 16 ? 16 : 8);
        const int groups = 32 / lpr;
        const uint32_t rows_per_cta = kDownRowsPerGroup * groups * (kDownThreads / 32);
        dim3 grid((H + rows_per_cta - 1) / rows_per_cta, gmax);
        const int nt = T == 1 ? 1 : 4;
        const size_t smem = static_cast<size_t>(nt) * (I + 2ull * chunks) * sizeof(float);
        const void* fn = nullptr;
        if (lpr == 32)
            fn = nt == 1 ? reinterpret_cast<const void*>(moe_expert_down_kernel<32, 1>)
                         : reinterpret_cast<const void*>(moe_expert_down_kernel<32, 4>);
        else if (lpr == 16)
            fn = nt == 1 ? reinterpret_cast<const void*>(moe_expert_down_kernel<16, 1>)
                         : reinterpret_cast<const void*>(moe_expert_down_kernel<16, 4>);
        else
            fn = nt == 1 ? reinterpret_cast<const void*>(moe_expert_down_kernel<8, 1>)
                         : reinterpret_cast<const void*>(moe_expert_down_kernel<8, 4>);
        if ((err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))) !=
            cudaSuccess)
            return err;
        if ((err = moe_launch_pdl(fn, grid, dim3(kDownThreads), smem, s, args, pdl)) != cudaSuccess) return err;
    }
    if ((err = mark(3)) != cudaSuccess) return err;
    // 4. combine (+ next-layer norm)
    {
        const OT* res = static_cast<const OT*>(a.residual);
        OT* out = static_cast<OT*>(a.out);
        OT* nn = static_cast<OT*>(a.next_normed);
        const float* nw = a.next_norm_w;
        float eps = a.eps;
        EpPeers ep{};
        if (a.ep) ep = *a.ep;
        uint32_t lo = e_lo, hi = e_hi;
        const void* fn;
        if (a.ep)
            fn = K <= 8    ? reinterpret_cast<const void*>(moe_combine_kernel<OT, 8, true>)
                 : K <= 16 ? reinterpret_cast<const void*>(moe_combine_kernel<OT, 16, true>)
                           : reinterpret_cast<const void*>(moe_combine_kernel<OT, 32, true>);
        else
            fn = K <= 8    ? reinterpret_cast<const void*>(moe_combine_kernel<OT, 8, false>)
                 : K <= 16 ? reinterpret_cast<const void*>(moe_combine_kernel<OT, 16, false>)
                           : reinterpret_cast<const void*>(moe_combine_kernel<OT, 32, false>);
        // T x Y CTAs of `piece` columns each; with a next-layer norm the Y
        // pieces of a token form one cluster (row-wide sum of squares)
        uint32_t Y = (H + 255) / 256;
        if (Y > kCombinePieces) Y = kCombinePieces;
        uint32_t piece = ((H + Y - 1) / Y + 3) & ~3u;
        Y = (H + piece - 1) / piece;
        const uint32_t vecs = piece / 4;
        uint32_t threads = vecs < static_cast<uint32_t>(kCombineMaxThreads) ? (vecs + 31) & ~31u
                                                                            : static_cast<uint32_t>(kCombineMaxThreads);
        if ((H & 3u) != 0 || vecs > threads * kCombineVec) return cudaErrorInvalidValue;
        void* args[] = {(void*)&T,   (void*)&H,   (void*)&K,     (void*)&has_shared, (void*)&has_gate,
                        (void*)&res, (void*)&out, (void*)&nw,    (void*)&nn,         (void*)&eps,
                        (void*)&lo,  (void*)&hi,  (void*)&piece, (void*)&ws,         (void*)&ep};
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(T, Y);
        cfg.blockDim = dim3(threads);
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        unsigned na = 0;
        if (pdl) {
            attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[na].val.programmaticStreamSerializationAllowed = 1;
            ++na;
        }
        if (nw) {
            attr[na].id = cudaLaunchAttributeClusterDimension;
            attr[na].val.clusterDim.x = 1;
            attr[na].val.clusterDim.y = Y;
            attr[na].val.clusterDim.z = 1;
            ++na;
        }
        cfg.attrs = attr;
        cfg.numAttrs = na;
        if ((err = cudaLaunchKernelExC(&cfg, fn, args)) != cudaSuccess) return err;
    }
    return mark(4);
}

cudaError_t moe_layer_launch(const MoeLaunch& a, cudaStream_t s) {
    if (a.x_dtype == PBMOE_BF16) {
        return a.out_dtype == PBMOE_BF16 ? moe_layer_launch_t<uint16_t, uint16_t>(a, s)
                                         : moe_layer_launch_t<uint16_t, float>(a, s);
    }
    return a.out_dtype == PBMOE_BF16 ? moe_layer_launch_t<float, uint16_t>(a, s) : moe_layer_launch_t<float, float>(a, s);
}

cudaError_t route_topk_launch(const float* logits, uint32_t T, uint32_t E, uint32_t K, uint32_t normalization,
                              float routed_scale, uint32_t* ids, float* w, uint32_t* status, cudaStream_t s,
                              const float* bias) {
    const int warps = 4;
    const size_t smem = warps * ((E + 3) & ~3u) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(route_topk_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    route_topk_kernel<<<(T + warps - 1) / warps, warps * 32, smem, s>>>(logits, T, E, K, normalization,
                                                                          routed_scale, ids, w, status, bias);
    return cudaGetLastError();
}

}  // namespace pbmoe
