// mla.cu — MLA absorbed decode attention (split-KV, tensor cores).
//
// Reference semantics (mla_absorbed_attention, weights/store.rs:1179-1327;
// Metal glm_mla_absorbed_scores / glm_mla_softmax / glm_mla_context,
// shaders.metal:1603-1682), per sequence and head h:
//   q_lat[c] = sum_d q_nope[h,d] * W_UK[h,d,c]                 (absorb)
//   s_t      = (q_lat . c_kv[t] + q_rope[h] . k_rope[t]) * scale
//   p        = softmax_t(s)
//   ctx[c]   = sum_t p_t * c_kv[t,c]
//   out[h,d] = sum_c ctx[c] * W_UV[h,d,c]
// with scale = 1/sqrt(nope + rope) (store.rs:1262) and k_rope already rotated
// when the cache was written (runtime/mod.rs:2906-2913).
//
// Three launches:
//   1. mla_absorb_kernel   q_lat for every (sequence, head), W_UK read once;
//                          writes Q' = [q_lat | q_rope] * scale * log2(e) (f32).
//   2. mla_attn_kernel     one CTA per (KV split, sequence): every 64-token
//                          tile of the split's latent cache is read from HBM
//                          once (cp.async, double-buffered) and serves all 16
//                          heads. S = Q' K^T (16 heads = the mma's M; Q' as
//                          bf16 hi + lo so scores keep ~16 mantissa bits),
//                          online softmax in base 2, O += P C with P in bf16.
//                          Writes the split's (max, sum, O[16 x 512]).
//   3. mla_out_kernel      one CTA per (head, sequence): merges the splits'
//                          partials into ctx (in shared memory), then
//                          out = W_UV[h] ctx.
// The split plan keeps batch x splits within one wave of SMs (the attention
// kernel runs one CTA per SM).
// Shapes: 16 heads, latent 512, rope 64, v 128, nope <= 128, batch <= 32.

#include "common.cuh"
#include "kernels.h"

namespace pbmoe {

constexpr uint32_t kMlaHeads = 16, kMlaLatent = 512, kMlaRope = 64, kMlaV = 128;
constexpr uint32_t kMlaK = kMlaLatent + kMlaRope;  // 576: score dimension
constexpr uint32_t kMlaTile = 64;                  // tokens per tile
constexpr uint32_t kMlaWarps = 4;
// shared-memory row strides (bytes), padded by 16 against ldmatrix bank conflicts
constexpr uint32_t kQRow = kMlaK * 2 + 16;        // Q' hi / lo rows
constexpr uint32_t kCRow = kMlaLatent * 2 + 16;   // c_kv rows
constexpr uint32_t kRRow = kMlaRope * 2 + 16;     // k_rope rows
constexpr uint32_t kPRow = kMlaTile * 2 + 16;     // P rows
constexpr uint32_t kStageBytes = kMlaTile * (kCRow + kRRow);
constexpr uint32_t kMlaPartialFloats = 2 + kMlaLatent;  // max, sum, O
constexpr size_t kMlaSmem = 2 * size_t(kMlaHeads) * kQRow + 2 * size_t(kStageBytes) + kMlaHeads * kPRow +
                            kMlaWarps * kMlaHeads * 4 * 2;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte global -> shared async copy; src_bytes = 0 zero-fills the chunk.
__device__ __forceinline__ void cp16_zfill(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
}

// ---------------------------------------------------------------- 1. absorb
// grid (heads, latent/64), 256 threads: thread (quarter = tid/64, column
// c = 64*blockIdx.y + tid%64) sums a quarter of the nope dims for every
// sequence, with all its W_UK loads in flight at once; the quarters meet in
// shared memory. Writes Q'[b][h][0..511] = q_lat * k and Q'[b][h][512..575] =
// q_rope * k, k = scale * log2(e). nope <= 128 (host-checked).
constexpr uint32_t kAbsorbMaxNope = 128;
template <typename QT>
__global__ void __launch_bounds__(256) mla_absorb_kernel(const QT* __restrict__ q, uint32_t batch, uint32_t nope,
                                                         const uint16_t* __restrict__ w_uk, float k,
                                                         float* __restrict__ qp) {
    __shared__ float qs[kMlaMaxBatch * kAbsorbMaxNope];
    __shared__ float red[4][8][64];
    const uint32_t h = blockIdx.x, tid = threadIdx.x;
    const uint32_t quarter = tid >> 6, cc = tid & 63, c = blockIdx.y * 64 + cc;
    const uint32_t qdim = nope + kMlaRope;
    // W_UK does not depend on the earlier kernels: its loads are issued before
    // waiting for them
    const uint32_t dq = (nope + 3) / 4, d0 = quarter * dq;
    float w[kAbsorbMaxNope / 4];
    const uint16_t* wcol = w_uk + static_cast<size_t>(h) * nope * kMlaLatent + c;
#pragma unroll
    for (uint32_t i = 0; i < kAbsorbMaxNope / 4; ++i)
        w[i] = (i < dq && d0 + i < nope) ? bf16_bits_to_f32(wcol[static_cast<size_t>(d0 + i) * kMlaLatent]) : 0.f;
    pdl_wait();
    pdl_launch_dependents();
    for (uint32_t i = tid; i < batch * nope; i += blockDim.x) {
        const uint32_t b = i / nope, d = i % nope;
        qs[i] = load_act(q, (static_cast<size_t>(b) * kMlaHeads + h) * qdim + d);
    }
    __syncthreads();
    for (uint32_t b0 = 0; b0 < batch; b0 += 8) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            acc[j] = 0.f;
            if (b0 + j < batch) {
                const float* qb = qs + (b0 + j) * nope + d0;
#pragma unroll
                for (uint32_t i = 0; i < kAbsorbMaxNope / 4; ++i)
                    if (i < dq && d0 + i < nope) acc[j] = fmaf(qb[i], w[i], acc[j]);
            }
            red[quarter][j][cc] = acc[j];
        }
        __syncthreads();
        if (quarter == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (b0 + j < batch) {
                    const float v = red[0][j][cc] + red[1][j][cc] + red[2][j][cc] + red[3][j][cc];
                    qp[(static_cast<size_t>(b0 + j) * kMlaHeads + h) * kMlaK + c] = v * k;
                }
        }
        __syncthreads();
    }
    if (blockIdx.y == 0 && tid < kMlaRope) {
        for (uint32_t b = 0; b < batch; ++b)
            qp[(static_cast<size_t>(b) * kMlaHeads + h) * kMlaK + kMlaLatent + tid] =
                load_act(q, (static_cast<size_t>(b) * kMlaHeads + h) * qdim + nope + tid) * k;
    }
}

// ---------------------------------------------------------------- 2. attention
// grid (splits, batch), 128 threads (4 warps). Warp w computes the scores of
// tokens 16w..16w+15 of each tile (two n-tiles, all 576 dims) and owns the
// context columns 128w..128w+127.
__global__ void __launch_bounds__(kMlaWarps * 32, 1) mla_attn_kernel(const float* __restrict__ qp, MlaSeqs seqs,
                                                                      uint32_t split_tokens, uint32_t splits,
                                                                      float* __restrict__ partial) {
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_wait();
    pdl_launch_dependents();
    unsigned char* qhi = smem;
    unsigned char* qlo = qhi + kMlaHeads * kQRow;
    unsigned char* stage0 = qlo + kMlaHeads * kQRow;
    unsigned char* pbuf = stage0 + 2 * kStageBytes;
    float* wmax = reinterpret_cast<float*>(pbuf + kMlaHeads * kPRow);  // [warps][16]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t b = blockIdx.y, sp = blockIdx.x;
    const uint32_t L = seqs.len[b];
    const uint32_t t0 = sp * split_tokens, t1 = min(L, t0 + split_tokens);
    float* out = partial + (static_cast<size_t>(b) * splits + sp) * kMlaHeads * kMlaPartialFloats;
    const float NEG_INF = -__int_as_float(0x7f800000);
    if (t0 >= t1) {  // empty split: contributes nothing
        for (uint32_t i = threadIdx.x; i < kMlaHeads * kMlaPartialFloats; i += blockDim.x)
            out[i] = (i % kMlaPartialFloats == 0) ? NEG_INF : 0.f;
        return;
    }
    const uint16_t* ckv = seqs.c_kv[b];
    const uint16_t* krope = seqs.k_rope[b];
    const uint32_t ntiles = (t1 - t0 + kMlaTile - 1) / kMlaTile;

    auto issue_tile = [&](uint32_t tile, int buf) {
        unsigned char* st = stage0 + buf * kStageBytes;
        const uint32_t tb = t0 + tile * kMlaTile;
        // c_kv: 64 rows x 64 chunks; k_rope: 64 rows x 8 chunks
        for (uint32_t i = threadIdx.x; i < kMlaTile * 64; i += blockDim.x) {
            const uint32_t r = i >> 6, ch = i & 63;
            const uint32_t tok = tb + r;
            const bool ok = tok < t1;
            cp16_zfill(st + r * kCRow + ch * 16, ckv + static_cast<size_t>(ok ? tok : t0) * kMlaLatent + ch * 8,
                       ok ? 16u : 0u);
        }
        unsigned char* rt = st + kMlaTile * kCRow;
        for (uint32_t i = threadIdx.x; i < kMlaTile * 8; i += blockDim.x) {
            const uint32_t r = i >> 3, ch = i & 7;
            const uint32_t tok = tb + r;
            const bool ok = tok < t1;
            cp16_zfill(rt + r * kRRow + ch * 16, krope + static_cast<size_t>(ok ? tok : t0) * kMlaRope + ch * 8,
                       ok ? 16u : 0u);
        }
    };
    issue_tile(0, 0);
    cp_commit();

    // Q' of this sequence as bf16 hi and lo (residue) rows; every load of the
    // thread is issued before any conversion
    {
        const float4* q4 = reinterpret_cast<const float4*>(qp + static_cast<size_t>(b) * kMlaHeads * kMlaK);
        constexpr uint32_t kVec = kMlaHeads * kMlaK / 4;  // 2304 float4
        constexpr uint32_t kPer = kVec / (kMlaWarps * 32);
        static_assert(kVec % (kMlaWarps * 32) == 0, "whole float4 per thread");
        float4 v[kPer];
#pragma unroll
        for (uint32_t j = 0; j < kPer; ++j) v[j] = __ldcg(q4 + j * kMlaWarps * 32 + threadIdx.x);
#pragma unroll
        for (uint32_t j = 0; j < kPer; ++j) {
            const uint32_t i = j * kMlaWarps * 32 + threadIdx.x;
            const uint32_t h = i / (kMlaK / 4), c4 = i % (kMlaK / 4);
            const uint32_t h0 = pack_bf16x2(v[j].x, v[j].y), h1 = pack_bf16x2(v[j].z, v[j].w);
            const uint32_t l0 = pack_bf16x2(v[j].x - bf16_bits_to_f32(h0 & 0xffffu), v[j].y - bf16_bits_to_f32(h0 >> 16));
            const uint32_t l1 = pack_bf16x2(v[j].z - bf16_bits_to_f32(h1 & 0xffffu), v[j].w - bf16_bits_to_f32(h1 >> 16));
            *reinterpret_cast<uint2*>(qhi + h * kQRow + c4 * 8) = make_uint2(h0, h1);
            *reinterpret_cast<uint2*>(qlo + h * kQRow + c4 * 8) = make_uint2(l0, l1);
        }
    }

    // running state: heads g and g+8 (per lane), context columns of this warp
    float m_run[2] = {NEG_INF, NEG_INF}, l_run[2] = {0.f, 0.f};
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    // ldmatrix lane addressing: A (16 x 16 block): lane -> row (lane & 15), col half (lane >> 4)
    const uint32_t a_row = lane & 15, a_col = (lane >> 4) * 8;
    // B (n8 x k16) from [n][k] rows: lane -> row (lane & 7) + 8 * ((lane >> 4) & 1) for x4 over 2 n-tiles,
    // k half ((lane >> 3) & 1)
    const uint32_t b_row = (lane & 7) + ((lane >> 4) << 3), b_k = ((lane >> 3) & 1) * 8;

    for (uint32_t tile = 0; tile < ntiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < ntiles) issue_tile(tile + 1, buf ^ 1);
        cp_commit();
        cp_wait<1>();
        __syncthreads();  // tile `tile` landed (and, on the first pass, Q')
        const unsigned char* st = stage0 + buf * kStageBytes;
        const unsigned char* rt = st + kMlaTile * kCRow;

        // ---- scores of tokens 16w .. 16w+15: two n-tiles, hi and lo accumulators
        float sh[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float sl[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const uint32_t tok0 = warp * 16;
#pragma unroll
        for (uint32_t kk = 0; kk < kMlaK / 16; ++kk) {
            uint32_t ah[4], al[4], bb[4];
            ldsm_x4(ah, qhi + a_row * kQRow + (kk * 16 + a_col) * 2);
            ldsm_x4(al, qlo + a_row * kQRow + (kk * 16 + a_col) * 2);
            const uint32_t kc = kk * 16 + b_k;
            if (kk < kMlaLatent / 16)
                ldsm_x4(bb, st + (tok0 + b_row) * kCRow + kc * 2);
            else
                ldsm_x4(bb, rt + (tok0 + b_row) * kRRow + (kc - kMlaLatent) * 2);
            mma16816(sh[0], ah, bb[0], bb[1]);
            mma16816(sl[0], al, bb[0], bb[1]);
            mma16816(sh[1], ah, bb[2], bb[3]);
            mma16816(sl[1], al, bb[2], bb[3]);
        }
        // s[n][i]: n-tile n, (head g | g+8) x (token 2t | 2t+1)
        float s[2][4];
        const uint32_t tbase = t0 + tile * kMlaTile + tok0;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t tok = tbase + n * 8 + 2 * t + (i & 1);
                s[n][i] = tok < t1 ? sh[n][i] + sl[n][i] : NEG_INF;
            }
        // per-head maximum over the tile: warp's 16 tokens, then across warps
        float mx[2];
        mx[0] = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
        mx[1] = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(kFull, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(kFull, mx[r], 2));
        }
        if (t == 0) {
            wmax[warp * kMlaHeads + g] = mx[0];
            wmax[warp * kMlaHeads + g + 8] = mx[1];
        }
        __syncthreads();
        float alpha[2], m_new[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float m = m_run[r];
#pragma unroll
            for (int w = 0; w < kMlaWarps; ++w) m = fmaxf(m, wmax[w * kMlaHeads + g + 8 * r]);
            m_new[r] = m;
            alpha[r] = (m_run[r] == NEG_INF) ? 0.f : exp2f(m_run[r] - m);
            m_run[r] = m;
        }
        // p = 2^(s - m) rounded to bf16; the row sums use the rounded values
        float lsum[2] = {0.f, 0.f};
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            uint32_t pw[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const float p0 = (m_new[r] == NEG_INF) ? 0.f : exp2f(s[n][2 * r] - m_new[r]);
                const float p1 = (m_new[r] == NEG_INF) ? 0.f : exp2f(s[n][2 * r + 1] - m_new[r]);
                pw[r] = pack_bf16x2(p0, p1);
                lsum[r] += bf16_bits_to_f32(pw[r] & 0xffffu) + bf16_bits_to_f32(pw[r] >> 16);
            }
            const uint32_t col = (tok0 + n * 8 + 2 * t) * 2;
            *reinterpret_cast<uint32_t*>(pbuf + g * kPRow + col) = pw[0];
            *reinterpret_cast<uint32_t*>(pbuf + (g + 8) * kPRow + col) = pw[1];
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            lsum[r] += __shfl_xor_sync(kFull, lsum[r], 1);
            lsum[r] += __shfl_xor_sync(kFull, lsum[r], 2);
            l_run[r] = l_run[r] * alpha[r] + lsum[r];  // this warp's tokens only; summed over warps at the end
        }
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        __syncthreads();  // P complete
        // ---- O[:, 128w .. 128w+127] += P (16 x 64) C (64 x 128)
#pragma unroll
        for (uint32_t kk = 0; kk < kMlaTile / 16; ++kk) {
            uint32_t pa[4];
            ldsm_x4(pa, pbuf + a_row * kPRow + (kk * 16 + a_col) * 2);
            // trans loads: rows = tokens kk*16 + (lane & 15), columns 8-wide blocks
            const unsigned char* crow = st + (kk * 16 + (lane & 15)) * kCRow;
#pragma unroll
            for (int n = 0; n < 16; n += 2) {
                uint32_t bb[4];
                ldsm_x4_t(bb, crow + (warp * 128 + n * 8 + (lane >> 4) * 8) * 2);
                mma16816(o[n], pa, bb[0], bb[1]);
                mma16816(o[n + 1], pa, bb[2], bb[3]);
            }
        }
        __syncthreads();  // stage `buf` and P free for reuse
    }
    cp_wait<0>();

    // split partial: max, sum over all warps' tokens, O
    __syncthreads();
    float* lsh = wmax;  // reuse: [warps][16] partial sums
    if (t == 0) {
        lsh[warp * kMlaHeads + g] = l_run[0];
        lsh[warp * kMlaHeads + g + 8] = l_run[1];
    }
    __syncthreads();
    if (threadIdx.x < kMlaHeads) {
        float l = 0.f;
#pragma unroll
        for (int w = 0; w < kMlaWarps; ++w) l += lsh[w * kMlaHeads + threadIdx.x];
        out[threadIdx.x * kMlaPartialFloats + 1] = l;
    }
    if (warp == 0 && t == 0) {
        out[g * kMlaPartialFloats] = m_run[0];
        out[(g + 8) * kMlaPartialFloats] = m_run[1];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
        const uint32_t col = warp * 128 + n * 8 + 2 * t;
        *reinterpret_cast<float2*>(out + g * kMlaPartialFloats + 2 + col) = make_float2(o[n][0], o[n][1]);
        *reinterpret_cast<float2*>(out + (g + 8) * kMlaPartialFloats + 2 + col) = make_float2(o[n][2], o[n][3]);
    }
}

// ---------------------------------------------------------------- 3. merge + output
// grid (heads, batch), 256 threads. The splits of (sequence b, head h) are
// merged as ctx[c] = sum_s 2^(m_s - M) O_s[c] / sum_s 2^(m_s - M) l_s into
// shared memory, then warp w computes out rows d = w, w + 8, ... of
// W_UV[h] ctx (16 rows per warp, 16-byte weight loads; W_UV[h] is read from
// L2 by the batch's CTAs of head h after the first brings it in).
constexpr uint32_t kOutThreads = 256;
constexpr uint32_t kOutMaxSplits = 1024;
template <typename OT>
__global__ void __launch_bounds__(kOutThreads) mla_merge_out_kernel(const float* __restrict__ partial,
                                                                     uint32_t splits, const uint16_t* __restrict__ w_uv,
                                                                     OT* __restrict__ out) {
    __shared__ float wsc[kOutMaxSplits];
    __shared__ __align__(16) float cs[kMlaLatent];
    __shared__ float red[kOutThreads / 32];
    const uint32_t h = blockIdx.x, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // W_UV rows do not depend on the earlier kernels: the first rows' loads
    // are issued before waiting for them
    constexpr uint32_t kRowsPerWarp = kMlaV / (kOutThreads / 32);  // 16
    const uint16_t* wrow0 = w_uv + (static_cast<size_t>(h) * kMlaV + warp) * kMlaLatent + lane * 16;
    uint4 wa[2] = {__ldg(reinterpret_cast<const uint4*>(wrow0)), __ldg(reinterpret_cast<const uint4*>(wrow0 + 8))};
    pdl_wait();
    pdl_launch_dependents();
    const float* base = partial + static_cast<size_t>(b) * splits * kMlaHeads * kMlaPartialFloats +
                        h * kMlaPartialFloats;
    const size_t stride = static_cast<size_t>(kMlaHeads) * kMlaPartialFloats;
    const float NEG_INF = -__int_as_float(0x7f800000);
    float M = NEG_INF;
    for (uint32_t sp = threadIdx.x; sp < splits; sp += blockDim.x) M = fmaxf(M, __ldcg(base + sp * stride));
    M = warp_max(M);
    if (lane == 0) red[warp] = M;
    __syncthreads();
    M = red[0];
#pragma unroll
    for (int w = 1; w < kOutThreads / 32; ++w) M = fmaxf(M, red[w]);
    float tot = 0.f;
    for (uint32_t sp = threadIdx.x; sp < splits; sp += blockDim.x) {
        const float m = __ldcg(base + sp * stride);
        const float w = (m == NEG_INF) ? 0.f : exp2f(m - M);
        wsc[sp] = w;
        tot += w * __ldcg(base + sp * stride + 1);
    }
    tot = warp_sum(tot);
    __syncthreads();  // everyone has read red[] (M) and written wsc[]
    if (lane == 0) red[warp] = tot;
    __syncthreads();
    tot = 0.f;
#pragma unroll
    for (int w = 0; w < kOutThreads / 32; ++w) tot += red[w];
    const float inv = tot > 0.f ? 1.0f / tot : 0.f;
    // context: thread c of 256 takes columns c and c + 256
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const uint32_t c = threadIdx.x + half * kOutThreads;
        const float* oc = base + 2 + c;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t sp = 0;
        for (; sp + 8 <= splits; sp += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldcg(oc + (sp + j) * stride);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j & 3] = fmaf(wsc[sp + j], v[j], acc[j & 3]);
        }
        for (; sp < splits; ++sp) acc[0] = fmaf(wsc[sp], __ldcg(oc + sp * stride), acc[0]);
        cs[c] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * inv;
    }
    __syncthreads();
    // out rows: warp w takes d = w + 8 i; lane covers 16 latent columns
    float cv[16];
    {
        const float4* c4 = reinterpret_cast<const float4*>(cs + lane * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = c4[i];
            cv[4 * i] = v.x, cv[4 * i + 1] = v.y, cv[4 * i + 2] = v.z, cv[4 * i + 3] = v.w;
        }
    }
    for (uint32_t i = 0; i < kRowsPerWarp; ++i) {
        const uint32_t d = warp + i * (kOutThreads / 32);
        uint4 wn[2] = {wa[0], wa[1]};
        if (i + 1 < kRowsPerWarp) {  // next row in flight
            const uint16_t* wr = w_uv + (static_cast<size_t>(h) * kMlaV + d + kOutThreads / 32) * kMlaLatent + lane * 16;
            wn[0] = __ldg(reinterpret_cast<const uint4*>(wr));
            wn[1] = __ldg(reinterpret_cast<const uint4*>(wr + 8));
        }
        const uint32_t wv[8] = {wa[0].x, wa[0].y, wa[0].z, wa[0].w, wa[1].x, wa[1].y, wa[1].z, wa[1].w};
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            acc = fmaf(bf16_bits_to_f32(wv[q] & 0xffffu), cv[2 * q], acc);
            acc = fmaf(bf16_bits_to_f32(wv[q] >> 16), cv[2 * q + 1], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) store_act(out, (static_cast<size_t>(b) * kMlaHeads + h) * kMlaV + d, acc);
        wa[0] = wn[0];
        wa[1] = wn[1];
    }
}

// ---------------------------------------------------------------- launch
size_t mla_smem_bytes() { return kMlaSmem; }

bool mla_shape_supported(uint32_t heads, uint32_t rope, uint32_t latent, uint32_t v_dim) {
    return heads == kMlaHeads && rope == kMlaRope && latent == kMlaLatent && v_dim == kMlaV;
}

// Splits of the longest cache such that batch x splits CTAs fill at most one
// wave of SMs (one attention CTA per SM), each split at least one 64-token
// tile; a split need not be a whole number of tiles (the last tile of a
// split is masked).
void mla_plan_splits(const MlaLaunch& a, int num_sms, uint32_t& split_tokens, uint32_t& splits) {
    uint32_t lmax = 1;
    for (uint32_t b = 0; b < a.batch; ++b) lmax = a.seqs.len[b] > lmax ? a.seqs.len[b] : lmax;
    uint32_t want = static_cast<uint32_t>(num_sms) / (a.batch ? a.batch : 1);
    if (want < 1) want = 1;
    uint32_t st = (lmax + want - 1) / want;
    if (st < kMlaTile) st = kMlaTile;
    split_tokens = st;
    splits = (lmax + st - 1) / st;
}

uint32_t mla_max_splits(uint32_t max_batch, int num_sms) {
    return static_cast<uint32_t>(num_sms) / (max_batch ? max_batch : 1) + 1;
}

cudaError_t mla_decode_launch(const MlaLaunch& a, cudaStream_t s) {
    const float k = a.scale * 1.4426950408889634f;  // scores in base 2
    cudaError_t e;
    {
        const dim3 grid(kMlaHeads, kMlaLatent / 64);
        if (a.q_dtype == PBMOE_F32)
            e = launch_pdl_kernel(mla_absorb_kernel<float>, grid, dim3(256), 0, s, static_cast<const float*>(a.q),
                                  a.batch, a.nope, a.w_uk, k, a.qp);
        else
            e = launch_pdl_kernel(mla_absorb_kernel<uint16_t>, grid, dim3(256), 0, s,
                                  static_cast<const uint16_t*>(a.q), a.batch, a.nope, a.w_uk, k, a.qp);
        if (e != cudaSuccess) return e;
    }
    if ((e = cudaFuncSetAttribute(mla_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kMlaSmem))) != cudaSuccess)
        return e;
    if ((e = launch_pdl_kernel(mla_attn_kernel, dim3(a.splits, a.batch), dim3(kMlaWarps * 32), kMlaSmem, s, a.qp,
                               a.seqs, a.split_tokens, a.splits, a.partial)) != cudaSuccess)
        return e;
    if (a.splits > kOutMaxSplits) return cudaErrorInvalidValue;
    const dim3 og(kMlaHeads, a.batch);
    if (a.out_dtype == PBMOE_F32)
        return launch_pdl_kernel(mla_merge_out_kernel<float>, og, dim3(kOutThreads), 0, s, a.partial, a.splits, a.w_uv,
                                 static_cast<float*>(a.out));
    return launch_pdl_kernel(mla_merge_out_kernel<uint16_t>, og, dim3(kOutThreads), 0, s, a.partial, a.splits, a.w_uv,
                             static_cast<uint16_t*>(a.out));
}

}  // namespace pbmoe
