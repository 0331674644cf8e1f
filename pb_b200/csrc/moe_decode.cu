// moe_decode.cu — one MoE FFN decode layer on sm_100a, four stream-ordered
// kernels:
//
//   1. moe_router_kernel   router GEMV (bf16 [E x H]) + shared-expert gate
//                          logit; the last CTA to finish routes every token
//                          (route_token_smem) and builds the layer-major group
//                          plan (unique experts in ascending id order, routes
//                          in route order inside each group, shared expert as
//                          group 0 with every token).
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
#include "routing.cuh"

namespace pbmoe {

namespace cg = cooperative_groups;

// ---------------------------------------------------------------- kernel 1
constexpr int kRouterThreads = 256;
constexpr int kRouterRowsPerWarp = 1;
constexpr int kRouterTokPass = 8;
constexpr int kRouterVec = 8;  // 16-byte weight vectors per lane loaded before use

template <typename XT>
__global__ void __launch_bounds__(kRouterThreads)
moe_router_kernel(const XT* __restrict__ x, uint32_t T, uint32_t H, uint32_t E, uint32_t K,
                  uint32_t normalization, float routed_scale, const uint16_t* __restrict__ router_w,
                  const uint16_t* __restrict__ shared_gate_w, int has_shared, uint32_t e_lo, uint32_t e_hi,
                  uint32_t* ep_epoch, MoeWs ws) {
    extern __shared__ __align__(16) float smem[];
    XT* xs = reinterpret_cast<XT*>(smem);  // [kRouterTokPass][H], in x's own type
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nrows = E + (shared_gate_w ? 1u : 0u);
    const uint32_t row0 = (blockIdx.x * (kRouterThreads / 32) + warp) * kRouterRowsPerWarp;
    const uint32_t vec_per_row = H / 8;  // 16-byte vectors of 8 bf16

    // The router row does not depend on earlier kernels: start its loads
    // before waiting for the previous kernel (programmatic dependent launch).
    const uint32_t row = row0;
    const bool has_row = row < nrows;
    const uint16_t* wrow = !has_row ? nullptr : (row < E ? router_w + static_cast<size_t>(row) * H : shared_gate_w);
    uint4 w4[kRouterVec];
    auto load_block = [&](uint32_t vb) {
#pragma unroll
        for (int i = 0; i < kRouterVec; ++i) {
            const uint32_t v = vb + i * 32 + lane;
            w4[i] = (has_row && v < vec_per_row) ? ld_stream_u4(wrow + static_cast<size_t>(v) * 8)
                                                 : make_uint4(0, 0, 0, 0);
        }
    };
    load_block(0);
    pdl_wait();
    for (uint32_t t0 = 0; t0 < T; t0 += kRouterTokPass) {
        const uint32_t nt = min(T - t0, static_cast<uint32_t>(kRouterTokPass));
        __syncthreads();
        {  // stage x (a copy): every 16-byte load issued before any store
            constexpr uint32_t kPerVec = 16 / sizeof(XT);
            const uint32_t vpr = H / kPerVec, total = nt * vpr;
            const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0) * H);
            uint4* dst = reinterpret_cast<uint4*>(xs);
            for (uint32_t base = 0; base < total; base += 8 * blockDim.x) {
                uint4 v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t idx = base + i * blockDim.x + threadIdx.x;
                    if (idx < total) v[i] = src[idx];
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t idx = base + i * blockDim.x + threadIdx.x;
                    if (idx < total) dst[idx] = v[i];
                }
            }
        }
        __syncthreads();
        if (has_row) {
            float acc[kRouterTokPass];
#pragma unroll
            for (int t = 0; t < kRouterTokPass; ++t) acc[t] = 0.f;
            for (uint32_t vb = 0; vb < vec_per_row; vb += 32 * kRouterVec) {
                if (vb > 0 || t0 > 0) load_block(vb);
#pragma unroll
                for (int i = 0; i < kRouterVec; ++i) {
                    const uint32_t v = vb + i * 32 + lane;
                    if (v >= vec_per_row) break;
                    const uint32_t wv[4] = {w4[i].x, w4[i].y, w4[i].z, w4[i].w};
                    float wf[8];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        wf[2 * q] = __uint_as_float(wv[q] << 16);
                        wf[2 * q + 1] = __uint_as_float(wv[q] & 0xffff0000u);
                    }
#pragma unroll
                    for (int t = 0; t < kRouterTokPass; ++t) {
                        if (static_cast<uint32_t>(t) < nt) {
                            float4 a, b;
                            if constexpr (sizeof(XT) == 2) {  // bf16: one 16-byte read, widened exactly
                                const uint4 q = *reinterpret_cast<const uint4*>(xs + t * H + v * 8);
                                a = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xffff0000u),
                                                __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xffff0000u));
                                b = make_float4(__uint_as_float(q.z << 16), __uint_as_float(q.z & 0xffff0000u),
                                                __uint_as_float(q.w << 16), __uint_as_float(q.w & 0xffff0000u));
                            } else {
                                const float4* xp = reinterpret_cast<const float4*>(xs + t * H + v * 8);
                                a = xp[0];
                                b = xp[1];
                            }
                            acc[t] = fmaf(wf[0], a.x, acc[t]);
                            acc[t] = fmaf(wf[1], a.y, acc[t]);
                            acc[t] = fmaf(wf[2], a.z, acc[t]);
                            acc[t] = fmaf(wf[3], a.w, acc[t]);
                            acc[t] = fmaf(wf[4], b.x, acc[t]);
                            acc[t] = fmaf(wf[5], b.y, acc[t]);
                            acc[t] = fmaf(wf[6], b.z, acc[t]);
                            acc[t] = fmaf(wf[7], b.w, acc[t]);
                        }
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < kRouterTokPass; ++t) {
                if (static_cast<uint32_t>(t) < nt) {
                    const float sum = warp_sum(acc[t]);
                    if (lane == 0) {
                        if (row < E)
                            ws.logits[static_cast<size_t>(t0 + t) * E + row] = sum;
                        else
                            ws.shared_logit[t0 + t] = sum;
                    }
                }
            }
        }
    }

    // ---- last CTA: routing + group plan
    __shared__ uint32_t is_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(ws.ticket, 1u);
        is_last = (prev == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // Every other CTA has exited: let the expert kernel be scheduled now, so
    // its prologue (barrier setup, activation staging) runs under this CTA's
    // routing and plan; it reads the plan only after griddepcontrol.wait,
    // i.e. after this grid completes.
    pdl_launch_dependents();

    {
        const uint32_t Ep = (E + 3) & ~3u;
        float* s = smem + warp * Ep;  // the x staging area is free now
        for (uint32_t t = warp; t < T; t += blockDim.x / 32) {
            stage_logits_warp(ws.logits + static_cast<size_t>(t) * E, E, s);
            route_token_smem(s, E, K, normalization, routed_scale, ws.route_ids + static_cast<size_t>(t) * K,
                             ws.route_w + static_cast<size_t>(t) * K, ws.status);
        }
    }
    __syncthreads();

    // group plan; shared memory reuses the activation staging area
    uint32_t* cnt = reinterpret_cast<uint32_t*>(smem);  // [E] counts -> starts
    uint32_t* gidx = cnt + E;                           // [E] used flags -> group index
    uint32_t* ids = gidx + E;                           // [T*K]
    uint32_t* tmp = ids + T * K;                        // [32]
    const uint32_t R = T * K;
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    // only the experts of this rank's range [e_lo, e_hi) form groups (all of
    // them on a single GPU); group_expert holds the slot index e - e_lo
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = __ldcg(ws.route_ids + r);
        ids[r] = e;
        if (e >= e_lo && e < e_hi) atomicAdd(&cnt[e], 1u);
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) gidx[e] = cnt[e] ? 1u : 0u;
    __syncthreads();
    const uint32_t U = block_exclusive_scan(gidx, E, tmp);
    const uint32_t RL = block_exclusive_scan(cnt, E, tmp);  // cnt[e] = start of expert e; RL local routes
    const uint32_t shared_groups = has_shared ? 1u : 0u;
    const uint32_t routed_base = has_shared ? T : 0u;  // grouped positions taken by the shared group
    for (uint32_t r = threadIdx.x; r < R; r += blockDim.x) {
        const uint32_t e = ids[r];
        if (e < e_lo || e >= e_hi) continue;
        uint32_t rank = 0;
        for (uint32_t q = 0; q < r; ++q) rank += (ids[q] == e) ? 1u : 0u;
        const uint32_t pos = routed_base + cnt[e] + rank;
        ws.group_routes[pos] = r;
        ws.group_tokens[pos] = r / K;
        if (rank == 0) {
            // exclusive-scan property: the group's size is the next start minus this one
            const uint32_t g = shared_groups + gidx[e];
            ws.group_expert[g] = e - e_lo;
            ws.group_start[g] = routed_base + cnt[e];
            ws.group_count[g] = (e + 1 < E ? cnt[e + 1] : RL) - cnt[e];
        }
    }
    if (has_shared) {
        for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) {
            ws.group_routes[t] = R + t;
            ws.group_tokens[t] = t;
        }
        if (threadIdx.x == 0) {
            ws.group_expert[0] = E;
            ws.group_start[0] = 0;
            ws.group_count[0] = T;
        }
    }
    if (threadIdx.x == 0) {
        *ws.num_groups = U + shared_groups;
        *ws.ticket = 0;  // ready for the next launch
        if (ep_epoch) *ep_epoch += 1u;  // this layer's expert-parallel exchange epoch
    }
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
    pdl_wait();
    if (threadIdx.x < K) {
        const uint32_t e = __ldcg(ws.route_ids + static_cast<size_t>(t) * K + threadIdx.x);
        wsh[threadIdx.x] = (e >= e_lo && e < e_hi) ? __ldcg(ws.route_w + static_cast<size_t>(t) * K + threadIdx.x)
                                                   : 0.f;  // another rank's route
    }
    if (threadIdx.x == 0) missing = 0;
    float sw = 0.f;
    if (has_shared) sw = has_gate ? 1.0f / (1.0f + expf(-__ldcg(ws.shared_logit + t))) : 1.0f;
    __syncthreads();
    const float* yt = ws.y + static_cast<size_t>(t) * K * H;
    const float* ysh = ws.y + (static_cast<size_t>(T) * K + t) * H;
    const uint32_t cb = blockIdx.y * piece, ce = min(H, cb + piece);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
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
            float4 o = residual ? load_act4<OT>(residual, static_cast<size_t>(t) * H + c) : zero;
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
            const float4 nw = *reinterpret_cast<const float4*>(norm_w + c);
            store_act4<OT>(next_normed, static_cast<size_t>(t) * H + c,
                           make_float4(v[j].x * scale * nw.x, v[j].y * scale * nw.y, v[j].z * scale * nw.z,
                                       v[j].w * scale * nw.w));
        }
    }
}

// ---------------------------------------------------------------- routing only
__global__ void route_topk_kernel(const float* __restrict__ logits, uint32_t T, uint32_t E, uint32_t K,
                                  uint32_t normalization, float routed_scale, uint32_t* ids, float* w,
                                  uint32_t* status) {
    extern __shared__ __align__(16) float rsm[];  // per warp: E logits (padded to 4)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t = blockIdx.x * (blockDim.x / 32) + warp;
    if (t >= T) return;
    const uint32_t Ep = (E + 3) & ~3u;
    float* s = rsm + warp * Ep;
    stage_logits_warp(logits + static_cast<size_t>(t) * E, E, s);
    route_token_smem(s, E, K, normalization, routed_scale, ids + static_cast<size_t>(t) * K,
                     w + static_cast<size_t>(t) * K, status);
}

// ---------------------------------------------------------------- host side
static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args,
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
    const size_t stage = static_cast<size_t>(kRouterTokPass) * H * sizeof(float);
    const size_t plan = (2ull * E + static_cast<size_t>(T) * K + 32) * sizeof(uint32_t);
    const size_t route = static_cast<size_t>(kRouterThreads / 32) * ((E + 3) & ~3u) * sizeof(float);
    size_t m = stage > plan ? stage : plan;
    return m > route ? m : route;
}

template <typename F>
static cudaError_t set_smem(F* fn, size_t bytes) {
    return cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bytes));
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
    if ((err = mark(0)) != cudaSuccess) return err;
    // 1. router + routing + plan
    {
        const uint32_t nrows = E + (has_gate ? 1u : 0u);
        const uint32_t rows_per_cta = (kRouterThreads / 32) * kRouterRowsPerWarp;
        dim3 grid((nrows + rows_per_cta - 1) / rows_per_cta);
        const size_t smem = moe_router_smem(T, H, E, K);
        auto fn = moe_router_kernel<XT>;
        if ((err = set_smem(fn, smem)) != cudaSuccess) return err;
        const XT* x = static_cast<const XT*>(a.x);
        uint32_t norm = a.normalization;
        float scale = a.routed_scale;
        const uint16_t* rw = a.router_w;
        const uint16_t* sg = a.shared_gate;
        uint32_t* ep_epoch = a.ep ? a.ep->epoch : nullptr;
        void* args[] = {(void*)&x,  (void*)&T,          (void*)&H,    (void*)&E,    (void*)&K,
                        (void*)&norm, (void*)&scale,    (void*)&rw,   (void*)&sg,   (void*)&has_shared,
                        (void*)&e_lo, (void*)&e_hi,     (void*)&ep_epoch, (void*)&ws};
        if ((err = launch_pdl(reinterpret_cast<const void*>(fn), grid, dim3(kRouterThreads), smem, s, args,
                              a.pdl && pdl)) != cudaSuccess)
            return err;
    }
    if ((err = mark(1)) != cudaSuccess) return err;
    const uint32_t gmax = (T * K < E ? T * K : E) + (has_shared ? 1u : 0u);
    MoeLayoutDev L = a.layout;
    const uint8_t* experts = a.experts;
    const uint8_t* shared = a.shared_slot;
    const bool mma = moe_mma_supported(a.layout);
    const bool pipe = moe_pipe_supported(a);
    // 2. gate/up/SwiGLU
    if (pipe) {
        if ((err = moe_up_pipe_launch(a, s, pdl)) != cudaSuccess) return err;
    } else if (mma) {
        if ((err = moe_up_mma_launch(a, gmax, s, pdl)) != cudaSuccess) return err;
    } else {
        const uint32_t chunks = H >> 5;
        dim3 grid((I + kUpRowsPerCta - 1) / kUpRowsPerCta, gmax);
        const XT* x = static_cast<const XT*>(a.x);
        void* args[] = {(void*)&x, (void*)&E, (void*)&experts, (void*)&shared, (void*)&L, (void*)&ws};
        if (T == 1) {
            const size_t smem = (1ull * H + 2ull * chunks) * sizeof(float);
            auto fn = moe_expert_up_kernel<XT, 1>;
            if ((err = set_smem(fn, smem)) != cudaSuccess) return err;
            err = launch_pdl(reinterpret_cast<const void*>(fn), grid, dim3(kUpThreads), smem, s, args, pdl);
        } else {
            const size_t smem = 4ull * (H + 2ull * chunks) * sizeof(float);
            auto fn = moe_expert_up_kernel<XT, 4>;
            if ((err = set_smem(fn, smem)) != cudaSuccess) return err;
            err = launch_pdl(reinterpret_cast<const void*>(fn), grid, dim3(kUpThreads), smem, s, args, pdl);
        }
        if (err != cudaSuccess) return err;
    }
    if ((err = mark(2)) != cudaSuccess) return err;
    // 3. down
    if (pipe) {
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
        if ((err = launch_pdl(fn, grid, dim3(kDownThreads), smem, s, args, pdl)) != cudaSuccess) return err;
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
                              float routed_scale, uint32_t* ids, float* w, uint32_t* status, cudaStream_t s) {
    const int warps = 4;
    const size_t smem = warps * ((E + 3) & ~3u) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(route_topk_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    route_topk_kernel<<<(T + warps - 1) / warps, warps * 32, smem, s>>>(logits, T, E, K, normalization,
                                                                          routed_scale, ids, w, status);
    return cudaGetLastError();
}

}  // namespace pbmoe
