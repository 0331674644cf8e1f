// q4_mma.cuh — decode-GEMV building blocks on the tensor cores (mma.sync
// m16n8k16, bf16 inputs, f32 accumulate) for group-64 Q4 weights.
//
// Why tensor cores for a matvec: the decode path is HBM-bound, and at B200
// bandwidth the SM has ~2.8 instruction issues per weight nibble to spend.
// Dequantising on the CUDA cores costs ~3.3 (shift, mask, convert, FMA per
// nibble) and leaves the kernel issue-bound. Here a nibble costs one mask-OR
// (two nibbles per instruction) plus a quarter of an mma.
//
// Exact nibble → bf16: OR-ing a nibble into the mantissa of 128.0 (0x4300)
// gives the bf16 value 128 + q exactly, so one LOP3 turns a shifted u32 word
// into a bf16x2 pair (128 + q_a, 128 + q_b). The mma then accumulates
//     D = sum_c (128 + q_c) x_c = 128 * X + sum_c q_c x_c,   X = sum_c x_c
// in fp32 over one quantisation group (products are exact; the 128*X offset
// costs ~2^-17 relative), and each group is finished on the CUDA cores as
//     y += s * D + (b - 128 s) * X
// which equals sum_c (q_c s + b) x_c (math.rs:861-911 up to summation order).
//
// Fragment mapping (PTX ISA m16n8k16 .row.col): lane = 4*g + t.
//   A (16x16 activations): row g = token g, row g+8 = token g+8 (or the low
//     part of token g when activations are f32, see stage_act_mma);
//     a0/a2 hold k = {2t,2t+1} / {2t+8,2t+9} of row g, a1/a3 of row g+8.
//   B (16x8 weights, k x n): column n = weight row r0+n, supplied by lanes
//     with g = n; b0/b1 hold k = {2t,2t+1} / {2t+8,2t+9}.
//   D: d0/d1 = token g x weight rows r0+2t / r0+2t+1; d2/d3 = token g+8.
// The contraction index k is a free permutation of the group's 64 columns:
// for word step m in {0,1} lane t contributes packed word w = 2t+m of the
// group (columns 8w..8w+7). mma "P" takes nibble pairs (0,4) and (1,5), mma
// "Q" takes (2,6) and (3,7); the activations are staged in shared memory in
// the same pair order, so one 16-byte load yields all four A registers.
#pragma once

#include "common.cuh"

namespace pbmoe {

constexpr uint32_t kMmaGroup = 64;       // the fast path's quantisation group
constexpr uint32_t kBf16Offset = 0x43004300u;  // bf16x2 (128.0, 128.0)

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}


// Shared-memory activation tile for the mma path:
//   act  : [rows][K/8 + 1 slots] of uint4, slot = 8 activations of one packed
//          word in pair order (x0,x4),(x1,x5),(x2,x6),(x3,x7) as bf16x2; the
//          extra slot pads each row so that lanes reading the same word of
//          consecutive rows hit different banks (rows can then also be filled
//          by contiguous bulk copies)
//   gsum : [rows][K/64] f32 group sums of the (full precision) activations
// Rows >= the token count are zero. With LO (f32 inputs), row t+8 holds the
// bf16 rounding residue of token t, so hi + lo carries ~16 mantissa bits.
struct ActTile {
    uint4* act;
    float* gsum;
    uint32_t slots;   // K / 8
    uint32_t groups;  // row stride of gsum in floats (K / 64 + 1: padded against bank conflicts)
    uint32_t stride;  // slots per row including the pad (K / 8 + 1)
};

__host__ __device__ inline uint32_t act_stride(uint32_t K) { return K / 8 + 1; }

__host__ __device__ inline size_t act_tile_bytes(uint32_t K, uint32_t rows) {
    return size_t(rows) * act_stride(K) * 16 + (size_t(rows) * (K / 64 + 1) * 4 + 15) / 16 * 16;
}

__host__ __device__ inline ActTile act_tile_at(void* base, uint32_t K, uint32_t rows) {
    ActTile t;
    t.act = reinterpret_cast<uint4*>(base);
    t.gsum = reinterpret_cast<float*>(reinterpret_cast<char*>(base) + size_t(rows) * act_stride(K) * 16);
    t.slots = K / 8;
    t.groups = K / 64 + 1;
    t.stride = act_stride(K);
    return t;
}

__device__ __forceinline__ uint32_t pack_pairs_lo(uint32_t a, uint32_t b) {  // (a.lo, b.lo)
    return __byte_perm(a, b, 0x5410);
}
__device__ __forceinline__ uint32_t pack_pairs_hi(uint32_t a, uint32_t b) {  // (a.hi, b.hi)
    return __byte_perm(a, b, 0x7632);
}

// Round two floats to a bf16x2 (round to nearest even), low half = a.
__device__ __forceinline__ uint32_t f2_to_bf16x2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}

// Barrier that ends a staging pass: the whole CTA (nthreads == 0) or the
// `nthreads` threads of named barrier `bar_id`.
__device__ __forceinline__ void tile_sync(int bar_id, uint32_t nthreads) {
    if (nthreads == 0)
        __syncthreads();
    else
        asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
}

// Stage `ntok` activation rows (<= 16 for bf16, <= 8 for f32) into `tile`.
// x rows are `x_stride` elements apart; rows_idx maps local token t to its
// source row (NULL = identity). All global loads of a thread are issued before
// its shared stores. Run by threads 0..nthreads-1 (the whole CTA when
// nthreads == 0) and ends with their barrier (tile_sync).
//
// f32 rows may be normalised on the way in: with norm_w, activation c of token
// t is staged as x * nscale[t] * norm_w[c] (nscale: the tokens' 1/rms, in
// shared memory, computed by the caller).
template <typename XT, uint32_t kBatch = 4>
__device__ void stage_act_mma(const XT* __restrict__ x, size_t x_stride, const uint32_t* rows_idx, int ntok,
                              uint32_t K, const ActTile& tile, int bar_id = 0, uint32_t nthreads = 0,
                              const float* __restrict__ norm_w = nullptr, const float* nscale = nullptr) {
    constexpr bool kLo = sizeof(XT) == 4;
    const uint32_t nthr = nthreads ? nthreads : blockDim.x;
    const uint32_t slots = K / 8;
    const uint32_t nt = static_cast<uint32_t>(ntok);
    // zero the unused rows (and, for bf16, rows ntok..15; for f32, rows ntok..7
    // and 8+ntok..15) and their group sums (for f32 also rows 8..15), row by
    // row: no division by the row length
    for (uint32_t row = 0; row < 16; ++row) {
        const uint32_t tok = kLo ? (row & 7u) : row;
        if (tok >= nt)
            for (uint32_t w = threadIdx.x; w < slots; w += nthr) tile.act[row * tile.stride + w] = make_uint4(0, 0, 0, 0);
        if (tok >= nt || (kLo && row >= 8))
            for (uint32_t gi = threadIdx.x; gi < tile.groups; gi += nthr) tile.gsum[row * tile.groups + gi] = 0.f;
    }
    // a thread keeps word w = w0 + threadIdx.x of every token (8 activations):
    // kBatch tokens' loads in flight at once (1 for register-heavy callers),
    // the word's norm weights loaded once; the 8 words of a 64-column group
    // are 8 consecutive lanes
    for (uint32_t w0 = 0; w0 < slots; w0 += nthr) {
        const uint32_t w = w0 + threadIdx.x;
        const bool okw = w < slots;
        float nn[8];
        if constexpr (kLo) {
            if (norm_w && okw) {
                const float4 n0 = *reinterpret_cast<const float4*>(norm_w + static_cast<size_t>(w) * 8);
                const float4 n1 = *reinterpret_cast<const float4*>(norm_w + static_cast<size_t>(w) * 8 + 4);
                nn[0] = n0.x, nn[1] = n0.y, nn[2] = n0.z, nn[3] = n0.w, nn[4] = n1.x, nn[5] = n1.y, nn[6] = n1.z,
                nn[7] = n1.w;
            }
        }
        for (uint32_t t0 = 0; t0 < nt; t0 += kBatch) {
            uint4 v[kBatch][kLo ? 2 : 1];
#pragma unroll
            for (uint32_t i = 0; i < kBatch; ++i) {
                const uint32_t t = t0 + i;
                if (okw && t < nt) {
                    const size_t src = rows_idx ? rows_idx[t] : static_cast<size_t>(t);
                    const uint4* p = reinterpret_cast<const uint4*>(x + src * x_stride + static_cast<size_t>(w) * 8);
                    v[i][0] = p[0];
                    if constexpr (kLo) v[i][1] = p[1];
                }
            }
#pragma unroll
            for (uint32_t i = 0; i < kBatch; ++i) {
                const uint32_t t = t0 + i;
                if (t >= nt) break;  // uniform: every lane has the same token
                const bool ok = okw;
                float sum = 0.f;
                if (ok) {
                    if constexpr (!kLo) {
                        const uint4 r = v[i][0];  // (x0,x1) (x2,x3) (x4,x5) (x6,x7)
                        tile.act[t * tile.stride + w] =
                            make_uint4(pack_pairs_lo(r.x, r.z), pack_pairs_hi(r.x, r.z), pack_pairs_lo(r.y, r.w),
                                       pack_pairs_hi(r.y, r.w));
                        const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            sum += __uint_as_float(rr[q] << 16) + __uint_as_float(rr[q] & 0xffff0000u);
                    } else {
                        float f[8] = {__uint_as_float(v[i][0].x), __uint_as_float(v[i][0].y),
                                      __uint_as_float(v[i][0].z), __uint_as_float(v[i][0].w),
                                      __uint_as_float(v[i][1].x), __uint_as_float(v[i][1].y),
                                      __uint_as_float(v[i][1].z), __uint_as_float(v[i][1].w)};
                        if (norm_w) {
                            const float sc = nscale[t];
#pragma unroll
                            for (int q = 0; q < 8; ++q) f[q] = f[q] * sc * nn[q];
                        }
                        uint32_t hi[4], lo[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            // pair order (x_q, x_{q+4})
                            const uint32_t h = f2_to_bf16x2(f[q], f[q + 4]);
                            const float h0 = __uint_as_float(h << 16), h1 = __uint_as_float(h & 0xffff0000u);
                            hi[q] = h;
                            lo[q] = f2_to_bf16x2(f[q] - h0, f[q + 4] - h1);
                            sum += f[q] + f[q + 4];
                        }
                        tile.act[t * tile.stride + w] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        tile.act[(t + 8) * tile.stride + w] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
                sum += __shfl_xor_sync(kFull, sum, 1);
                sum += __shfl_xor_sync(kFull, sum, 2);
                sum += __shfl_xor_sync(kFull, sum, 4);
                if (ok && (w & 7u) == 0) tile.gsum[t * tile.groups + (w >> 3)] = sum;
            }
        }
    }
    tile_sync(bar_id, nthreads);
}

// stage_act_mma for bf16 tiles with only 8 token rows (tokens <= 8) and
// contiguous token rows.
template <typename XT>
__device__ void stage_act_rows8_tok(const XT* __restrict__ x, size_t x_stride, int ntok, uint32_t K,
                                    const ActTile& tile, int bar_id = 0, uint32_t nthreads = 0) {
    const uint32_t nthr = nthreads ? nthreads : blockDim.x;
    static_assert(sizeof(XT) == 2, "8-row tiles hold bf16 activations");
    const uint32_t slots = K / 8;
    const uint32_t nt = static_cast<uint32_t>(ntok);
    for (uint32_t row = nt; row < 8; ++row) {  // absent tokens: zero rows and group sums
        for (uint32_t w = threadIdx.x; w < slots; w += nthr) tile.act[row * tile.stride + w] = make_uint4(0, 0, 0, 0);
        for (uint32_t gi = threadIdx.x; gi < tile.groups; gi += nthr) tile.gsum[row * tile.groups + gi] = 0.f;
    }
    // a thread keeps word w = w0 + threadIdx.x of every token, all tokens'
    // loads in flight at once; the 8 words of a group are 8 consecutive lanes
    for (uint32_t w0 = 0; w0 < slots; w0 += nthr) {
        const uint32_t w = w0 + threadIdx.x;
        const bool okw = w < slots;
        uint4 v[8];
#pragma unroll
        for (uint32_t t = 0; t < 8; ++t)
            if (okw && t < nt) v[t] = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * x_stride + static_cast<size_t>(w) * 8);
#pragma unroll
        for (uint32_t t = 0; t < 8; ++t) {
            if (t >= nt) break;  // uniform
            float sum = 0.f;
            if (okw) {
                const uint4 r = v[t];
                tile.act[t * tile.stride + w] = make_uint4(pack_pairs_lo(r.x, r.z), pack_pairs_hi(r.x, r.z),
                                                           pack_pairs_lo(r.y, r.w), pack_pairs_hi(r.y, r.w));
                const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) sum += __uint_as_float(rr[q] << 16) + __uint_as_float(rr[q] & 0xffff0000u);
            }
            sum += __shfl_xor_sync(kFull, sum, 1);
            sum += __shfl_xor_sync(kFull, sum, 2);
            sum += __shfl_xor_sync(kFull, sum, 4);
            if (okw && (w & 7u) == 0) tile.gsum[t * tile.groups + (w >> 3)] = sum;
        }
    }
    tile_sync(bar_id, nthreads);
}

// Register fragment of one 8-row tile over a block of 4 consecutive groups:
// lane (g,t) holds words 2t, 2t+1 of row r0+g for each group, and the bf16
// scales/biases of rows r0+2t and r0+2t+1 for the four groups (8 bytes each).
// load() only issues global loads, so it can run before activation staging
// or before a programmatic-dependent-launch wait.
struct Q4MmaFrag4 {
    uint2 w[4];
    uint2 sa, sb, ba, bb;  // 4 bf16 each: scale/bias of row 2t (a) and 2t+1 (b)

    __device__ __forceinline__ void load(const uint8_t* row_g, const uint16_t* s_row_2t, const uint16_t* b_row_2t,
                                         uint32_t gpr, uint32_t grp0, int t) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = ld_stream_u2(row_g + (grp0 + j) * (kMmaGroup / 2) + 8 * t);
        sa = *reinterpret_cast<const uint2*>(s_row_2t + grp0);
        sb = *reinterpret_cast<const uint2*>(s_row_2t + gpr + grp0);
        ba = *reinterpret_cast<const uint2*>(b_row_2t + grp0);
        bb = *reinterpret_cast<const uint2*>(b_row_2t + gpr + grp0);
    }

    // Same fragment from a shared-memory copy of the tile: row_g is row r0+g,
    // s_row_2t / b_row_2t are rows r0+2t of the scale / bias blocks, and
    // `sstride` elements separate consecutive scale rows.
    __device__ __forceinline__ void load_smem(const uint8_t* row_g, const uint16_t* s_row_2t, const uint16_t* b_row_2t,
                                              uint32_t sstride, uint32_t grp0, int t) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = *reinterpret_cast<const uint2*>(row_g + (grp0 + j) * (kMmaGroup / 2) + 8 * t);
        sa = *reinterpret_cast<const uint2*>(s_row_2t + grp0);
        sb = *reinterpret_cast<const uint2*>(s_row_2t + sstride + grp0);
        ba = *reinterpret_cast<const uint2*>(b_row_2t + grp0);
        bb = *reinterpret_cast<const uint2*>(b_row_2t + sstride + grp0);
    }

    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = make_uint2(0, 0);
        sa = sb = ba = bb = make_uint2(0, 0);
    }

    static __device__ __forceinline__ float pick(const uint2& v, int j) {
        const uint32_t word = (j < 2) ? v.x : v.y;
        return (j & 1) ? __uint_as_float(word & 0xffff0000u) : __uint_as_float(word << 16);
    }

    // acc[0..1]: token g x rows 2t / 2t+1; acc[2..3]: token g+8 (kTok16).
    // With kLo the residue rows g+8 are folded into acc[0..1].
    template <bool kLo, bool kTok16>
    __device__ __forceinline__ void compute(const ActTile& tile, uint32_t grp0, int g, int t, float (&acc)[4]) const {
        float X[4], X2[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            X[j] = tile.gsum[g * tile.groups + grp0 + j];
            X2[j] = kTok16 ? tile.gsum[(g + 8) * tile.groups + grp0 + j] : 0.f;
        }
        compute_x<kLo, kTok16>(tile, grp0, g, t, X, X2, acc);
    }

    // Same with the activation group sums supplied by the caller (X: token g,
    // X2: token g+8).
    template <bool kLo, bool kTok16>
    __device__ __forceinline__ void compute_x(const ActTile& tile, uint32_t grp0, int g, int t, const float (&X)[4],
                                              const float (&X2)[4], float (&acc)[4]) const {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t wd = (grp0 + j) * 8 + 2 * t;
            const uint4 xa0 = tile.act[g * tile.stride + wd];
            const uint4 xa1 = tile.act[g * tile.stride + wd + 1];
            uint4 xb0 = make_uint4(0, 0, 0, 0), xb1 = make_uint4(0, 0, 0, 0);
            if (kLo || kTok16) {
                xb0 = tile.act[(g + 8) * tile.stride + wd];
                xb1 = tile.act[(g + 8) * tile.stride + wd + 1];
            }
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t words[2] = {w[j].x, w[j].y};
            const uint4 xa[2] = {xa0, xa1}, xb[2] = {xb0, xb1};
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const uint32_t q = words[m];
                const uint32_t b0p = (q & 0x000F000Fu) | kBf16Offset;
                const uint32_t b1p = ((q >> 4) & 0x000F000Fu) | kBf16Offset;
                const uint32_t b0q = ((q >> 8) & 0x000F000Fu) | kBf16Offset;
                const uint32_t b1q = ((q >> 12) & 0x000F000Fu) | kBf16Offset;
                mma_bf16_16816(d, xa[m].x, xb[m].x, xa[m].y, xb[m].y, b0p, b1p);
                mma_bf16_16816(d, xa[m].z, xb[m].z, xa[m].w, xb[m].w, b0q, b1q);
            }
            const float s0 = pick(sa, j), s1 = pick(sb, j);
            const float c0 = fmaf(-128.f, s0, pick(ba, j));
            const float c1 = fmaf(-128.f, s1, pick(bb, j));
            if (kLo) {
                acc[0] = fmaf(s0, d[0] + d[2], fmaf(c0, X[j], acc[0]));
                acc[1] = fmaf(s1, d[1] + d[3], fmaf(c1, X[j], acc[1]));
            } else {
                acc[0] = fmaf(s0, d[0], fmaf(c0, X[j], acc[0]));
                acc[1] = fmaf(s1, d[1], fmaf(c1, X[j], acc[1]));
                if (kTok16) {
                    acc[2] = fmaf(s0, d[2], fmaf(c0, X2[j], acc[2]));
                    acc[3] = fmaf(s1, d[3], fmaf(c1, X2[j], acc[3]));
                }
            }
        }
    }
};

// Gate and up fragments of the same rows and groups on one activation tile:
// the activation fragments and group sums are loaded once for both.
template <bool kLo>
__device__ __forceinline__ void q4_mma_pair(const Q4MmaFrag4& fa, const Q4MmaFrag4& fb, const ActTile& tile,
                                            uint32_t grp0, int g, int t, float (&acc_a)[4], float (&acc_b)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t wd = (grp0 + j) * 8 + 2 * t;
        const uint4 xa0 = tile.act[g * tile.stride + wd];
        const uint4 xa1 = tile.act[g * tile.stride + wd + 1];
        uint4 xb0 = make_uint4(0, 0, 0, 0), xb1 = make_uint4(0, 0, 0, 0);
        if (kLo) {
            xb0 = tile.act[(g + 8) * tile.stride + wd];
            xb1 = tile.act[(g + 8) * tile.stride + wd + 1];
        }
        const float X = tile.gsum[g * tile.groups + grp0 + j];
        const uint4 xa[2] = {xa0, xa1}, xb[2] = {xb0, xb1};
        const Q4MmaFrag4* fr[2] = {&fa, &fb};
        float (*ac[2])[4] = {&acc_a, &acc_b};
#pragma unroll
        for (int f = 0; f < 2; ++f) {
            const Q4MmaFrag4& F = *fr[f];
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t words[2] = {F.w[j].x, F.w[j].y};
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const uint32_t q = words[m];
                const uint32_t b0p = (q & 0x000F000Fu) | kBf16Offset;
                const uint32_t b1p = ((q >> 4) & 0x000F000Fu) | kBf16Offset;
                const uint32_t b0q = ((q >> 8) & 0x000F000Fu) | kBf16Offset;
                const uint32_t b1q = ((q >> 12) & 0x000F000Fu) | kBf16Offset;
                mma_bf16_16816(d, xa[m].x, xb[m].x, xa[m].y, xb[m].y, b0p, b1p);
                mma_bf16_16816(d, xa[m].z, xb[m].z, xa[m].w, xb[m].w, b0q, b1q);
            }
            const float s0 = Q4MmaFrag4::pick(F.sa, j), s1 = Q4MmaFrag4::pick(F.sb, j);
            const float c0 = fmaf(-128.f, s0, Q4MmaFrag4::pick(F.ba, j));
            const float c1 = fmaf(-128.f, s1, Q4MmaFrag4::pick(F.bb, j));
            float(&acc)[4] = *ac[f];
            if (kLo) {
                acc[0] = fmaf(s0, d[0] + d[2], fmaf(c0, X, acc[0]));
                acc[1] = fmaf(s1, d[1] + d[3], fmaf(c1, X, acc[1]));
            } else {
                acc[0] = fmaf(s0, d[0], fmaf(c0, X, acc[0]));
                acc[1] = fmaf(s1, d[1], fmaf(c1, X, acc[1]));
            }
        }
    }
}

// Weight-stationary form for batches of at most 8 tokens: 16 weight rows are
// the M operand (rows g and g+8 of lane (g,t)) and the tokens the N operand,
// so every product of the m16n8k16 is useful. For one group the lane holds
// words 2t, 2t+1 of both rows (wg, wh); xb[m] is token g's staged slot for
// word 2t+m (xl[m]: its lo residue when activations are f32, folded into the
// same accumulator). d = [row g | row g+8] x [token 2t | token 2t+1], finished
// as acc += s * d + (b - 128 s) * X with the tokens' group sums X0, X1.
// One word pair (word m of rows g and g+8, 8 nibbles each) unpacked and
// multiplied in a single asm block: the four unpacked bf16x2 registers of an
// mma's A operand are produced in place, so no operand-marshalling moves are
// needed between the unpack and the two (four with a lo residue) mma.sync.
__device__ __forceinline__ void q4_rows16_word(float (&d)[4], uint32_t q, uint32_t r, uint4 xb) {
    asm("{\n"
        " .reg .b32 qa, qb, qc, qd, ra, rb, rc, rd, t;\n"
        " lop3.b32 qa, %4, 0x000F000F, 0x43004300, 0xea;\n"
        " lop3.b32 ra, %5, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %4, 4;\n lop3.b32 qb, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %5, 4;\n lop3.b32 rb, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %4, 8;\n lop3.b32 qc, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %5, 8;\n lop3.b32 rc, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %4, 12;\n lop3.b32 qd, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %5, 12;\n lop3.b32 rd, t, 0x000F000F, 0x43004300, 0xea;\n"
        " mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {qa,ra,qb,rb}, {%6,%7}, {%0,%1,%2,%3};\n"
        " mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {qc,rc,qd,rd}, {%8,%9}, {%0,%1,%2,%3};\n"
        "}\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(q), "r"(r), "r"(xb.x), "r"(xb.y), "r"(xb.z), "r"(xb.w));
}

// Same with the hi and lo parts of f32 activations accumulated together.
__device__ __forceinline__ void q4_rows16_word_lo(float (&d)[4], uint32_t q, uint32_t r, uint4 xb, uint4 xl) {
    asm("{\n"
        " .reg .b32 qa, qb, qc, qd, ra, rb, rc, rd, t;\n"
        " lop3.b32 qa, %4, 0x000F000F, 0x43004300, 0xea;\n"
        " lop3.b32 ra, %5, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %4, 4;\n lop3.b32 qb, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %5, 4;\n lop3.b32 rb, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %4, 8;\n lop3.b32 qc, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %5, 8;\n lop3.b32 rc, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %4, 12;\n lop3.b32 qd, t, 0x000F000F, 0x43004300, 0xea;\n"
        " shr.b32 t, %5, 12;\n lop3.b32 rd, t, 0x000F000F, 0x43004300, 0xea;\n"
        " mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {qa,ra,qb,rb}, {%6,%7}, {%0,%1,%2,%3};\n"
        " mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {qc,rc,qd,rd}, {%8,%9}, {%0,%1,%2,%3};\n"
        " mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {qa,ra,qb,rb}, {%10,%11}, {%0,%1,%2,%3};\n"
        " mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {qc,rc,qd,rd}, {%12,%13}, {%0,%1,%2,%3};\n"
        "}\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(q), "r"(r), "r"(xb.x), "r"(xb.y), "r"(xb.z), "r"(xb.w), "r"(xl.x), "r"(xl.y), "r"(xl.z), "r"(xl.w));
}

template <bool kLo>
__device__ __forceinline__ void q4_mma_rows16(uint2 wg, uint2 wh, const uint4 (&xb)[2], const uint4 (&xl)[2],
                                              float s_g, float s_h, float b_g, float b_h, float X0, float X1,
                                              float (&acc)[4]) {
    static_assert(kBf16Offset == 0x43004300u, "unpack constant of q4_rows16_word");
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    if (kLo) {
        q4_rows16_word_lo(d, wg.x, wh.x, xb[0], xl[0]);
        q4_rows16_word_lo(d, wg.y, wh.y, xb[1], xl[1]);
    } else {
        q4_rows16_word(d, wg.x, wh.x, xb[0]);
        q4_rows16_word(d, wg.y, wh.y, xb[1]);
    }
    const float c_g = fmaf(-128.f, s_g, b_g), c_h = fmaf(-128.f, s_h, b_h);
    acc[0] = fmaf(s_g, d[0], fmaf(c_g, X0, acc[0]));
    acc[1] = fmaf(s_g, d[1], fmaf(c_g, X1, acc[1]));
    acc[2] = fmaf(s_h, d[2], fmaf(c_h, X0, acc[2]));
    acc[3] = fmaf(s_h, d[3], fmaf(c_h, X1, acc[3]));
}

}  // namespace pbmoe
