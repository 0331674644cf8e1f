// q4_rows.cuh — warp-level Q4 row-dot building blocks shared by the decode
// kernels (pbmoe_q4_matvec, the MoE expert kernels).
#pragma once

#include "common.cuh"

namespace pbmoe {

// Geometry of one Q4 matrix as the fast path sees it.
struct Q4Geom {
    uint32_t rows;
    uint32_t cols;
    uint32_t gpr;        // groups per row = ceil(cols / group)
    uint32_t chunks;     // cols / 32
    uint32_t cpg_shift;  // log2(group / 32): chunk j lives in group j >> cpg_shift
};

// Fast path: cols % 32 == 0, group a power of two >= 32, packed rows 16-byte
// aligned (cols/2 % 16 == 0 and a 16-byte aligned base).
__host__ __device__ inline bool q4_fast_ok(uint32_t cols, uint32_t group, const void* packed) {
    bool pow2 = group >= 32 && (group & (group - 1)) == 0;
    return cols % 32 == 0 && pow2 && (reinterpret_cast<uintptr_t>(packed) % 16 == 0);
}

__host__ __device__ inline uint32_t ilog2_u32(uint32_t v) {
    uint32_t r = 0;
    while (v > 1) {
        v >>= 1;
        ++r;
    }
    return r;
}

// Stage `ntok` activation rows (row stride `x_stride` elements) into shared
// memory as f32, plus each 32-column chunk's even/odd sums. Layout per token:
// xs[t * cols + xs_index(j, c)], xe[t * chunks + j], xo[t * chunks + j].
// Needs cols % 32 == 0 and 16-byte aligned rows. `rows_idx` maps local token t
// to the source row (NULL = identity).
//
// Phase 1 issues every 16-byte load of the thread before storing any of them
// (one memory round trip for the whole staging); phase 2 forms the chunk sums
// from shared memory. Ends with __syncthreads.
//
// With norm_w, each staged row is replaced by its RMSNorm times norm_w
// (x * (1 / sqrt(mean(x^2) + eps)) * w, rms_norm_reduced, shaders.metal:
// 1176-1213) before the chunk sums; `nscale` is shared memory for ntok floats.
template <typename XT>
__device__ void stage_x_fast(const XT* __restrict__ x, size_t x_stride, const uint32_t* rows_idx,
                             int ntok, uint32_t cols, float* xs, float* xe, float* xo,
                             const float* __restrict__ norm_w = nullptr, float eps = 0.f, float* nscale = nullptr) {
    constexpr uint32_t kPerVec = 16 / sizeof(XT);  // elements per 16-byte vector
    constexpr int kBatch = 8;                       // vectors in flight per thread
    const uint32_t chunks = cols >> 5;
    const uint32_t vec_per_row = cols / kPerVec;
    const uint32_t total = static_cast<uint32_t>(ntok) * vec_per_row;
    for (uint32_t base = 0; base < total; base += kBatch * blockDim.x) {
        uint4 v[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const uint32_t idx = base + i * blockDim.x + threadIdx.x;
            if (idx < total) {
                const uint32_t t = idx / vec_per_row, q = idx - t * vec_per_row;
                const size_t src = rows_idx ? rows_idx[t] : static_cast<size_t>(t);
                v[i] = *reinterpret_cast<const uint4*>(x + src * x_stride + static_cast<size_t>(q) * kPerVec);
            }
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const uint32_t idx = base + i * blockDim.x + threadIdx.x;
            if (idx < total) {
                const uint32_t t = idx / vec_per_row, q = idx - t * vec_per_row;
                const uint32_t c0 = q * kPerVec;
                float* dst = xs + static_cast<size_t>(t) * cols;
                const uint32_t j = c0 >> 5;
                if constexpr (sizeof(XT) == 2) {
                    // eight bf16 columns = two swizzled float4
                    *reinterpret_cast<float4*>(dst + xs_index(j, c0 & 31u)) =
                        make_float4(__uint_as_float(v[i].x << 16), __uint_as_float(v[i].x & 0xffff0000u),
                                    __uint_as_float(v[i].y << 16), __uint_as_float(v[i].y & 0xffff0000u));
                    *reinterpret_cast<float4*>(dst + xs_index(j, (c0 & 31u) + 4)) =
                        make_float4(__uint_as_float(v[i].z << 16), __uint_as_float(v[i].z & 0xffff0000u),
                                    __uint_as_float(v[i].w << 16), __uint_as_float(v[i].w & 0xffff0000u));
                } else {
                    // four consecutive f32 columns = one swizzled float4
                    *reinterpret_cast<float4*>(dst + xs_index(j, c0 & 31u)) =
                        make_float4(__uint_as_float(v[i].x), __uint_as_float(v[i].y), __uint_as_float(v[i].z),
                                    __uint_as_float(v[i].w));
                }
            }
        }
    }
    __syncthreads();
    if (norm_w) {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
        for (int t = warp; t < ntok; t += nw) {
            const float* row = xs + static_cast<size_t>(t) * cols;
            float ss = 0.f;
            for (uint32_t i = lane * 4; i < cols; i += 128) {
                const float4 v = *reinterpret_cast<const float4*>(row + i);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
            ss = warp_sum(ss);
            if (lane == 0) nscale[t] = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
        }
        __syncthreads();
        const uint32_t n = static_cast<uint32_t>(ntok) * cols;
        for (uint32_t p = threadIdx.x; p < n; p += blockDim.x) {
            const uint32_t t = p / cols, q = p - t * cols, j = q >> 5, pp = q & 31u;
            const uint32_t c = ((((pp >> 2) ^ (j & 7u)) << 2) | (pp & 3u));  // logical column of slot pp
            xs[p] = xs[p] * nscale[t] * norm_w[(j << 5) + c];
        }
        __syncthreads();
    }
    const uint32_t nsum = static_cast<uint32_t>(ntok) * chunks;
    for (uint32_t i = threadIdx.x; i < nsum; i += blockDim.x) {
        const uint32_t t = i / chunks, j = i - t * chunks;
        const float4* c4 = reinterpret_cast<const float4*>(xs + static_cast<size_t>(t) * cols + (j << 5));
        float e = 0.f, o = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 f = c4[k];
            e += f.x + f.z;
            o += f.y + f.w;
        }
        xe[i] = e;
        xo[i] = o;
    }
    __syncthreads();
}

// Generic staging (any cols): f32 copy only.
template <typename XT>
__device__ void stage_x_generic(const XT* __restrict__ x, size_t x_stride, const uint32_t* rows_idx,
                                int ntok, uint32_t cols, float* xs) {
    for (int t = 0; t < ntok; ++t) {
        const size_t src = rows_idx ? rows_idx[t] : static_cast<size_t>(t);
        for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x)
            xs[static_cast<size_t>(t) * cols + c] = load_act<XT>(x, src * x_stride + c);
    }
}

// Fast-path partial dot products of NR rows with NT staged tokens.
//
// The warp is split into 32/LPR lane groups; a lane group owns one row at a
// time and its LPR lanes stride over the row's 16-byte chunks (chunk j goes to
// lane j % LPR), so every warp-wide load instruction reads 16*32 contiguous
// bytes per row group. A fragment holds one block of LPR*CPL chunks of NR rows
// in registers: load() issues all of the block's loads at once, accumulate()
// consumes them, so a kernel can start the weight loads before it stages the
// activations.
//
// row_packed[r] / row_scale[r] / row_bias[r] are this lane group's row r
// (NULL packed = absent row, contributes 0). acc[r][t] receives the lane's
// partial sum_c (q*s+b)*x_t[c]; reduce across the LPR lanes afterwards.
template <int LPR, int NR, int CPL>
struct Q4RowFrag {
    uint4 w[NR][CPL];
    float sc[NR][CPL], bi[NR][CPL];

    __device__ __forceinline__ void load(const uint8_t* const (&row_packed)[NR], const uint16_t* const (&row_scale)[NR],
                                         const uint16_t* const (&row_bias)[NR], const Q4Geom& g, uint32_t jb) {
        const int li = threadIdx.x & (LPR - 1);
#pragma unroll
        for (int r = 0; r < NR; ++r) {
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const uint32_t j = jb + c * LPR + li;
                if (row_packed[r] != nullptr && j < g.chunks) {
                    w[r][c] = ld_stream_u4(row_packed[r] + (static_cast<size_t>(j) << 4));
                    const uint32_t gi = j >> g.cpg_shift;
                    sc[r][c] = bf16_bits_to_f32(ld_nc_u16(row_scale[r] + gi));
                    bi[r][c] = bf16_bits_to_f32(ld_nc_u16(row_bias[r] + gi));
                } else {
                    w[r][c] = make_uint4(0, 0, 0, 0);
                    sc[r][c] = 0.f;
                    bi[r][c] = 0.f;
                }
            }
        }
    }

    template <int NT>
    __device__ __forceinline__ void accumulate(const Q4Geom& g, uint32_t jb, const float* xs, const float* xe,
                                               const float* xo, int ntok, float (&acc)[NR][NT]) const {
        const int li = threadIdx.x & (LPR - 1);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const uint32_t j = jb + c * LPR + li;
            if (j >= g.chunks) continue;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                ChunkF f;
                decode_chunk(w[r][c], f);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t < ntok) {
                        const float e = xe[t * g.chunks + j];
                        const float o = xo[t * g.chunks + j];
                        const float qd =
                            chunk_qdot(f, xs + static_cast<size_t>(t) * g.cols + (j << 5), j & 7u, e, o);
                        acc[r][t] = fmaf(sc[r][c], qd, fmaf(bi[r][c], e + o, acc[r][t]));
                    }
                }
            }
        }
    }
};

// Runs the fragment over all chunk blocks of the rows; `frag` must already
// hold block 0 (frag.load(..., 0)).
template <int LPR, int NR, int CPL, int NT>
__device__ __forceinline__ void q4_rows_finish(Q4RowFrag<LPR, NR, CPL>& frag, const uint8_t* const (&row_packed)[NR],
                                               const uint16_t* const (&row_scale)[NR],
                                               const uint16_t* const (&row_bias)[NR], const Q4Geom& g,
                                               const float* xs, const float* xe, const float* xo, int ntok,
                                               float (&acc)[NR][NT]) {
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (uint32_t jb = 0; jb < g.chunks; jb += LPR * CPL) {
        if (jb > 0) frag.load(row_packed, row_scale, row_bias, g, jb);
        frag.template accumulate<NT>(g, jb, xs, xe, xo, ntok, acc);
    }
}

// Generic partial dot of one row (any cols / group): lanes stride over
// columns and accumulate fma(q, s*x, b*x) as math.rs:861-911 does per element.
__device__ __forceinline__ float q4_row_partial_generic(const uint8_t* packed_row, const uint16_t* s_row,
                                                        const uint16_t* b_row, uint32_t cols, uint32_t group,
                                                        const float* xs, int lane, int nl) {
    float acc = 0.f;
    for (uint32_t c = lane; c < cols; c += nl) {
        const uint8_t byte = packed_row[c >> 1];
        const float q = static_cast<float>((c & 1) ? (byte >> 4) : (byte & 0x0f));
        const uint32_t gi = c / group;
        const float s = bf16_bits_to_f32(s_row[gi]);
        const float b = bf16_bits_to_f32(b_row[gi]);
        const float x = xs[c];
        acc += fmaf(q, s * x, b * x);
    }
    return acc;
}

}  // namespace pbmoe
