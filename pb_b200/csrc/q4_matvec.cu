// q4_matvec.cu — decode Q4 matvec y[b] = W x[b] (pbmoe_q4_matvec).
//
// Replaces q4_fma_matvec_bf16_scale_bias (shaders.metal:164-199), which gives
// each Apple SIMD group one row and stages x in an 8192-float threadgroup
// cache. Here each warp owns kRows rows per lane group; every lane streams
// 16-byte chunks of packed nibbles with ld.global.nc.L1::no_allocate (all of a
// warp's chunk loads are issued before its arithmetic), x is staged once per
// CTA in shared memory (swizzled, with per-chunk sums), and the row sums are
// finished with warp shuffles. Shapes outside the fast path (cols % 32 != 0,
// non power-of-two groups, unaligned rows) run a per-element kernel with the
// reference's own per-element arithmetic.
//
// The fast and tensor-core kernels are launched with programmatic dependent
// launch: a kernel issues its weight loads (which no earlier kernel writes),
// lets the next kernel in the stream be scheduled and only then waits for its
// predecessor (griddepcontrol.wait) before reading x or writing y, so
// back-to-back matvecs stream weights without a gap between launches.

#include <algorithm>

#include "kernels.h"
#include "pipe.cuh"
#include "q4_mma.cuh"
#include "q4_rows.cuh"

namespace pbmoe {

static cudaError_t launch_with_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

constexpr int kMvThreads = 128;
constexpr int kMvRows = 4;  // rows per lane group per pass

// One matrix of a launch: weights, output and row count. A launch covers up
// to kQ4MaxMats matrices on the same x, each one's CTAs after the previous
// one's: the MLA chain's q_a and kv_a projections, which read the same normed
// hidden state (execute_glm_mla_input_projection_chain,
// metal/qwen_execution.rs:289-480), or a batch of resident projections on one
// input (resident_mmap_matvec_batch, runtime/mod.rs:1184).
struct MvMat {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* biases;
    void* y;
    uint32_t rows;
};
struct MvSet {
    MvMat m[kQ4MaxMats];
    uint32_t first[kQ4MaxMats];  // first CTA of matrix i
    uint32_t count;
};

// The matrix of this CTA and the CTA's index within it.
__device__ __forceinline__ const MvMat& mv_pick(const MvSet& set, uint32_t& bx) {
    uint32_t i = 0;
    while (i + 1 < set.count && blockIdx.x >= set.first[i + 1]) ++i;
    bx = blockIdx.x - set.first[i];
    return set.m[i];
}

// Optional fusions: the input RMSNorm (norm_w, eps) and a residual added to y.
struct MvFuse {
    const float* norm_w;
    float eps;
    const void* residual;
};

template <typename YT>
__device__ __forceinline__ void store_y(const MvFuse& fz, YT* y, size_t i, float v) {
    if (fz.residual) v += load_act<YT>(static_cast<const YT*>(fz.residual), i);
    store_act<YT>(y, i, v);
}

template <typename XT, typename YT, int LPR, int CPL, int NT>
__global__ void __launch_bounds__(kMvThreads, 3)
q4_matvec_fast_kernel(const __grid_constant__ MvSet set, Q4Geom g0, const XT* __restrict__ x, uint32_t batch,
                      MvFuse fz) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float nscale[NT];
    constexpr int kGroups = 32 / LPR;
    constexpr int kRowsPerCta = kMvRows * kGroups * (kMvThreads / 32);
    uint32_t bx;
    const MvMat m = mv_pick(set, bx);
    Q4Geom g = g0;
    g.rows = m.rows;
    YT* y = static_cast<YT*>(m.y);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane / LPR;
    float* xs = smem;
    float* xe = xs + NT * g.cols;
    float* xo = xe + NT * g.chunks;
    const uint32_t r0 = bx * kRowsPerCta + (warp * kGroups + sub) * kMvRows;
    const uint8_t* pk[kMvRows];
    const uint16_t* ps[kMvRows];
    const uint16_t* pb[kMvRows];
#pragma unroll
    for (int r = 0; r < kMvRows; ++r) {
        const uint32_t row = r0 + r;
        pk[r] = row < g.rows ? m.packed + static_cast<size_t>(row) * (g.cols / 2) : nullptr;
        ps[r] = m.scales + static_cast<size_t>(row) * g.gpr;
        pb[r] = m.biases + static_cast<size_t>(row) * g.gpr;
    }
    Q4RowFrag<LPR, kMvRows, CPL> frag;
    for (uint32_t b0 = 0; b0 < batch; b0 += NT) {
        const int nt = static_cast<int>(min(batch - b0, static_cast<uint32_t>(NT)));
        frag.load(pk, ps, pb, g, 0);  // weights in flight while x is staged
        if (b0 == 0) {
            pdl_launch_dependents();
            pdl_wait();
        }
        __syncthreads();
        stage_x_fast<XT>(x + static_cast<size_t>(b0) * g.cols, g.cols, nullptr, nt, g.cols, xs, xe, xo, fz.norm_w,
                         fz.eps, nscale);
        float acc[kMvRows][NT];
        q4_rows_finish<LPR, kMvRows, CPL, NT>(frag, pk, ps, pb, g, xs, xe, xo, nt, acc);
#pragma unroll
        for (int r = 0; r < kMvRows; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float s = group_sum<LPR>(acc[r][t]);
                if ((lane & (LPR - 1)) == 0 && t < nt && r0 + r < g.rows)
                    store_y<YT>(fz, y, static_cast<size_t>(b0 + t) * g.rows + r0 + r, s);
            }
        }
    }
}

// Persistent, cp.async-pipelined form for launches of many rows (a
// projection batch): a CTA stages x once, then walks 32-row blocks
// `gridDim.x` apart over every matrix of the set. A block's nibbles, scales
// and biases are copied into one of kSmStages shared-memory stages by every
// thread (16-byte cp.async), kSmStages - 1 blocks ahead of the one being
// computed, so each SM keeps ~100 KB of weights in flight. Warp w computes
// rows 4w..4w+3 of the block; a lane takes chunks lane, lane + 32, ... of each
// row (the fast kernel's chunk arithmetic, weights read from shared memory).
// Rows of up to kSmMaxCols columns (a block's bytes fit a stage).
constexpr int kSmThreads = 256;
constexpr int kSmRows = 32;       // rows per block
constexpr int kSmStages = 4;
constexpr uint32_t kSmMaxCols = 2048;

__device__ __forceinline__ const MvMat& mv_pick_block(const MvSet& set, uint32_t blk, uint32_t& bx) {
    uint32_t i = 0;
    while (i + 1 < set.count && blk >= set.first[i + 1]) ++i;
    bx = blk - set.first[i];
    return set.m[i];
}

template <typename XT, typename YT, int NT>
__global__ void __launch_bounds__(kSmThreads, 1)
q4_matvec_stream_kernel(const __grid_constant__ MvSet set, uint32_t nblocks, Q4Geom g0, const XT* __restrict__ x,
                        uint32_t batch) {
    extern __shared__ __align__(16) unsigned char sm_raw[];
    const uint32_t cols = g0.cols, chunks = g0.chunks, gpr = g0.gpr, rb = cols / 2;
    float* xs = reinterpret_cast<float*>(sm_raw);
    float* xe = xs + NT * cols;
    float* xo = xe + NT * chunks;
    unsigned char* stage0 = sm_raw + ((NT * (cols + 2 * chunks) * 4 + 127) / 128) * 128;
    const uint32_t sbytes = kSmRows * rb + 2 * kSmRows * gpr * 2;  // nibbles, then scales, then biases
    const uint32_t sstride = (sbytes + 127) / 128 * 128;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nt = static_cast<int>(batch);

    auto issue = [&](uint32_t blk, int st) {
        uint32_t bx;
        const MvMat& m = mv_pick_block(set, blk, bx);
        const uint32_t r0 = bx * kSmRows;
        const uint32_t nr = min(static_cast<uint32_t>(kSmRows), m.rows - r0);
        unsigned char* d = stage0 + st * sstride;
        // nibbles: nr rows of rb bytes, contiguous in the matrix
        const uint32_t nvec = nr * rb / 16;
        const unsigned char* src = m.packed + static_cast<size_t>(r0) * rb;
        for (uint32_t i = threadIdx.x; i < nvec; i += kSmThreads) cp_async16(d + i * 16, src + i * 16);
        // scales and biases: nr * gpr bf16 each (gpr * 2 bytes per row)
        const uint32_t sb = nr * gpr * 2;
        const unsigned char* ssrc = reinterpret_cast<const unsigned char*>(m.scales + static_cast<size_t>(r0) * gpr);
        const unsigned char* bsrc = reinterpret_cast<const unsigned char*>(m.biases + static_cast<size_t>(r0) * gpr);
        for (uint32_t i = threadIdx.x * 4; i < sb; i += kSmThreads * 4) {
            cp_async4(d + kSmRows * rb + i, ssrc + i);
            cp_async4(d + kSmRows * rb + kSmRows * gpr * 2 + i, bsrc + i);
        }
    };
    uint32_t blk = blockIdx.x;
    for (int st = 0; st < kSmStages - 1; ++st) {
        const uint32_t b = blk + st * gridDim.x;
        if (b < nblocks) issue(b, st);
        cp_async_commit();
    }
    pdl_launch_dependents();
    pdl_wait();
    stage_x_fast<XT>(x, cols, nullptr, nt, cols, xs, xe, xo);
    for (int it = 0; blk < nblocks; ++it, blk += gridDim.x) {
        const int st = it % kSmStages;
        {  // the block kSmStages - 1 ahead goes into the stage freed last iteration
            const uint32_t b = blk + (kSmStages - 1) * gridDim.x;
            if (b < nblocks) issue(b, (it + kSmStages - 1) % kSmStages);
            cp_async_commit();
        }
        cp_async_wait_group<kSmStages - 1>();
        __syncthreads();
        uint32_t bx;
        const MvMat& m = mv_pick_block(set, blk, bx);
        const unsigned char* d = stage0 + st * sstride;
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(d + kSmRows * rb);
        const uint16_t* bi = sc + kSmRows * gpr;
        float acc[4][NT];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
        for (uint32_t j = lane; j < chunks; j += 32) {
            const uint32_t gi = j >> g0.cpg_shift;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t row = warp * 4 + r;
                const uint4 w = *reinterpret_cast<const uint4*>(d + row * rb + j * 16);
                const float s = bf16_bits_to_f32(sc[row * gpr + gi]);
                const float bv = bf16_bits_to_f32(bi[row * gpr + gi]);
                ChunkF f;
                decode_chunk(w, f);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    if (t < nt) {
                        const float e = xe[t * chunks + j], o = xo[t * chunks + j];
                        const float qd = chunk_qdot(f, xs + static_cast<size_t>(t) * cols + (j << 5), j & 7u, e, o);
                        acc[r][t] = fmaf(s, qd, fmaf(bv, e + o, acc[r][t]));
                    }
                }
            }
        }
        YT* y = static_cast<YT*>(m.y);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = warp_sum(acc[r][t]);
                const uint32_t row = bx * kSmRows + warp * 4 + r;
                if (lane == 0 && t < nt && row < m.rows) store_act<YT>(y, static_cast<size_t>(t) * m.rows + row, v);
            }
        }
        __syncthreads();  // stage st is read: the next iteration refills it
    }
    cp_async_wait_group<0>();
}

template <typename XT, typename YT>
__global__ void __launch_bounds__(kMvThreads)
q4_matvec_generic_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                         const uint16_t* __restrict__ biases, uint32_t rows, uint32_t cols, uint32_t group,
                         const XT* __restrict__ x, YT* __restrict__ y, uint32_t batch) {
    extern __shared__ __align__(16) float smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t gpr = (cols + group - 1) / group;
    const uint32_t row = blockIdx.x * (kMvThreads / 32) + warp;
    for (uint32_t b = 0; b < batch; ++b) {
        __syncthreads();
        stage_x_generic<XT>(x + static_cast<size_t>(b) * cols, cols, nullptr, 1, cols, smem);
        __syncthreads();
        if (row < rows) {
            const float p = q4_row_partial_generic(packed + static_cast<size_t>(row) * ((cols + 1) / 2),
                                                   scales + static_cast<size_t>(row) * gpr,
                                                   biases + static_cast<size_t>(row) * gpr, cols, group, smem, lane,
                                                   32);
            const float s = warp_sum(p);
            if (lane == 0) store_act<YT>(y, static_cast<size_t>(b) * rows + row, s);
        }
    }
}

// Tensor-core matvec for group-64 weights (q4_mma.cuh): CTA = 8 warps =
// (8/KS) tiles of 8 rows x KS K-slices; slices are summed in shared memory.
// kTok16: bf16 activations, up to 16 tokens per pass; f32 activations use
// hi/lo rows (8 tokens per pass). With fz.norm_w (f32 activations) the CTA
// computes each token's 1/rms from x first and stages the normalised rows.
// NB > 1: each warp's K-slice is exactly NB 4-group blocks, all held in
// registers and loaded before the dependency wait (one CTA per SM for the
// registers); NB = 1 streams the blocks one at a time.
template <typename XT, typename YT, int KS, bool kTok16, int NB = 1>
__global__ void __launch_bounds__(256, NB > 1 ? 1 : 2)
q4_matvec_mma_kernel(const __grid_constant__ MvSet set, uint32_t cols, const XT* __restrict__ x, uint32_t batch,
                     MvFuse fz) {
    constexpr bool kLo = sizeof(XT) == 4;
    constexpr bool kRows16 = kLo || kTok16;
    constexpr int kPass = kTok16 ? 16 : 8;
    constexpr int kTiles = 8 / KS;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ float nscale[kPass];
    uint32_t bx;
    const MvMat m = mv_pick(set, bx);
    const uint32_t rows = m.rows;
    YT* y = static_cast<YT*>(m.y);
    const uint32_t trows = kRows16 ? 16 : 8;
    const ActTile tile = act_tile_at(smem_raw, cols, trows);
    float* red = reinterpret_cast<float*>(smem_raw + act_tile_bytes(cols, trows));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int tl = warp / KS, ks = warp % KS;
    const uint32_t gpr = cols / kMmaGroup;
    const uint32_t gps = gpr / KS;
    const uint32_t r0 = bx * (8 * kTiles) + tl * 8;
    // rows past the end read the last row and are never stored
    const uint32_t rg = min(r0 + g, rows - 1), ra = min(r0 + 2 * t, rows - 1), rb = min(r0 + 2 * t + 1, rows - 1);
    const uint8_t* wrow = m.packed + static_cast<size_t>(rg) * (cols / 2);
    const uint32_t grp0 = ks * gps;
    Q4MmaFrag4 f[NB];
    // scale rows ra and rb = ra + 1 unless clamped; load them through the
    // (row 2t, row 2t+1) pair when both exist, else clamp both to ra
    const uint16_t* sa = m.scales + static_cast<size_t>(ra) * gpr;
    const uint16_t* ba = m.biases + static_cast<size_t>(ra) * gpr;
    const uint32_t pair_gpr = (rb == ra + 1) ? gpr : 0;
#pragma unroll
    for (int j = 0; j < NB; ++j) f[j].load(wrow, sa, ba, pair_gpr, grp0 + 4 * j, t);
    pdl_launch_dependents();
    pdl_wait();
    for (uint32_t b0 = 0; b0 < batch; b0 += kPass) {
        const int nt = static_cast<int>(min(batch - b0, static_cast<uint32_t>(kPass)));
        __syncthreads();
        if constexpr (kLo) {
            if (fz.norm_w) {  // 1/rms of each token of the pass, one warp per token
                for (int tok = warp; tok < nt; tok += 8) {
                    const float* xr = reinterpret_cast<const float*>(x) + static_cast<size_t>(b0 + tok) * cols;
                    float ss = 0.f;
                    // the lane's float4 of the row 8 at a time, each batch's loads in
                    // flight together (two round trips at 1536 columns), summed in order
                    for (uint32_t c0 = 0; c0 < cols; c0 += 8 * 128) {
                        float4 v[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const uint32_t i = c0 + lane * 4 + j * 128;
                            v[j] = i < cols ? *reinterpret_cast<const float4*>(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
                    }
                    ss = warp_sum(ss);
                    if (lane == 0) nscale[tok] = 1.0f / sqrtf(ss / static_cast<float>(cols) + fz.eps);
                }
                __syncthreads();
            }
        }
        if constexpr (kRows16)
            stage_act_mma<XT>(x + static_cast<size_t>(b0) * cols, cols, nullptr, nt, cols, tile, 0, 0, fz.norm_w,
                              nscale);
        else
            stage_act_rows8_tok<XT>(x + static_cast<size_t>(b0) * cols, cols, nt, cols, tile);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (NB > 1) {
#pragma unroll
            for (int j = 0; j < NB; ++j) f[j].template compute<kLo, kTok16>(tile, grp0 + 4 * j, g, t, acc);
        } else {
            for (uint32_t b = 0; b < gps; b += 4) {
                if (b > 0) f[0].load(wrow, sa, ba, pair_gpr, grp0 + b, t);
                f[0].template compute<kLo, kTok16>(tile, grp0 + b, g, t, acc);
            }
            if (gps > 4) f[0].load(wrow, sa, ba, pair_gpr, grp0, t);  // block 0 again for the next pass
        }
        float* rw = red + warp * (16 * 8);
        rw[g * 8 + 2 * t] = acc[0];
        rw[g * 8 + 2 * t + 1] = acc[1];
        if (kTok16) {
            rw[(g + 8) * 8 + 2 * t] = acc[2];
            rw[(g + 8) * 8 + 2 * t + 1] = acc[3];
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < kTiles * 16 * 8; i += blockDim.x) {
            const uint32_t tile_i = i / 128, tok = (i / 8) % 16, r = i % 8;
            const uint32_t row = bx * (8 * kTiles) + tile_i * 8 + r;
            if (tok < static_cast<uint32_t>(nt) && row < rows) {
                float sum = 0.f;
#pragma unroll
                for (int k = 0; k < KS; ++k) sum += red[(tile_i * KS + k) * 128 + tok * 8 + r];
                store_y<YT>(fz, y, static_cast<size_t>(b0 + tok) * rows + row, sum);
            }
        }
    }
}

static int mv_sm_count() {
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

// The launch's matrices (the set, or packed [+ packed2]) with each one's
// first CTA for `rows_per_cta`; returns the total CTA count.
static uint32_t set_of(const Q4MatvecArgs& a, uint32_t rows_per_cta, MvSet& set) {
    set = MvSet{};
    if (a.set_count) {
        set.count = a.set_count;
        for (uint32_t i = 0; i < a.set_count; ++i)
            set.m[i] = MvMat{a.set[i].packed, a.set[i].scales, a.set[i].biases, a.set[i].y, a.set[i].rows};
    } else {
        set.count = a.packed2 ? 2u : 1u;
        set.m[0] = MvMat{a.packed, a.scales, a.biases, a.y, a.rows};
        if (a.packed2) set.m[1] = MvMat{a.packed2, a.scales2, a.biases2, a.y2, a.rows2};
    }
    uint32_t ctas = 0;
    for (uint32_t i = 0; i < set.count; ++i) {
        set.first[i] = ctas;
        ctas += (set.m[i].rows + rows_per_cta - 1) / rows_per_cta;
    }
    return ctas;
}

template <typename XT, typename YT, int KS>
static cudaError_t launch_mma_ks(const Q4MatvecArgs& a, cudaStream_t s) {
    constexpr int kTiles = 8 / KS;
    const bool lo = sizeof(XT) == 4;
    const bool tok16 = !lo && a.batch > 8;
    const size_t trows = (lo || tok16) ? 16 : 8;
    const size_t smem = act_tile_bytes(a.cols, static_cast<uint32_t>(trows)) + 8 * 16 * 8 * 4;
    if (smem > 200 * 1024) return cudaErrorNotSupported;
    // f32 activations whose warp slices are 2 or 3 blocks: every block in
    // registers before the wait (the decode step's q_b: 1536 columns, KS 2)
    const uint32_t nb = a.cols / 256 / KS;
    const void* fn = tok16 ? reinterpret_cast<const void*>(q4_matvec_mma_kernel<XT, YT, KS, true>)
                           : reinterpret_cast<const void*>(q4_matvec_mma_kernel<XT, YT, KS, false>);
    if (lo && nb == 2) fn = reinterpret_cast<const void*>(q4_matvec_mma_kernel<XT, YT, KS, false, 2>);
    if (lo && nb == 3) fn = reinterpret_cast<const void*>(q4_matvec_mma_kernel<XT, YT, KS, false, 3>);
    cudaError_t err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    MvSet set;
    const uint32_t ctas = set_of(a, 8 * kTiles, set);
    MvFuse fz{a.norm_w, a.eps, a.residual};
    uint32_t cols = a.cols, batch = a.batch;
    const XT* x = static_cast<const XT*>(a.x);
    void* args[] = {(void*)&set, (void*)&cols, (void*)&x, (void*)&batch, (void*)&fz};
    return launch_with_pdl(fn, dim3(ctas), dim3(256), smem, s, args);
}

// Group-64 weights whose row length is a multiple of 256 columns.
template <typename XT, typename YT>
static cudaError_t launch_mma(const Q4MatvecArgs& a, cudaStream_t s) {
    const uint32_t blocks = a.cols / 256;  // 4-group blocks per row
    if (blocks % 8 == 0) return launch_mma_ks<XT, YT, 8>(a, s);
    if (blocks % 4 == 0) return launch_mma_ks<XT, YT, 4>(a, s);
    if (blocks % 2 == 0) return launch_mma_ks<XT, YT, 2>(a, s);
    return launch_mma_ks<XT, YT, 1>(a, s);
}

template <typename XT, typename YT, int LPR, int CPL, int NT>
static cudaError_t launch_fast(const Q4MatvecArgs& a, const Q4Geom& g, cudaStream_t s) {
    constexpr int kGroups = 32 / LPR;
    constexpr int kRowsPerCta = kMvRows * kGroups * (kMvThreads / 32);
    bool stream_aligned = a.set_count > 1;
    for (uint32_t i = 0; i < a.set_count; ++i)
        stream_aligned = stream_aligned && reinterpret_cast<uintptr_t>(a.set[i].packed) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(a.set[i].scales) % 4 == 0 &&
                         reinterpret_cast<uintptr_t>(a.set[i].biases) % 4 == 0;
    if (stream_aligned && !a.norm_w && !a.residual && a.batch <= static_cast<uint32_t>(NT) &&
        g.cols <= kSmMaxCols && (g.cols / 2) % 16 == 0 && g.gpr % 2 == 0) {
        // a projection batch: the persistent pipelined kernel (weights 16-byte
        // aligned per row: packed base 16-byte aligned and cols/2 a multiple of 16)
        const size_t xbytes = (static_cast<size_t>(NT) * (g.cols + 2ull * g.chunks) * 4 + 127) / 128 * 128;
        const size_t sstride = ((size_t(kSmRows) * (g.cols / 2) + 2ull * kSmRows * g.gpr * 2) + 127) / 128 * 128;
        const size_t smem = xbytes + kSmStages * sstride;
        auto fn = q4_matvec_stream_kernel<XT, YT, NT>;
        cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err != cudaSuccess) return err;
        MvSet set;
        uint32_t nblocks = set_of(a, kSmRows, set);
        const uint32_t grid = std::min(nblocks, static_cast<uint32_t>(mv_sm_count()));
        Q4Geom gg = g;
        const XT* x = static_cast<const XT*>(a.x);
        uint32_t batch = a.batch;
        void* args[] = {(void*)&set, (void*)&nblocks, (void*)&gg, (void*)&x, (void*)&batch};
        return launch_with_pdl(reinterpret_cast<const void*>(fn), dim3(grid), dim3(kSmThreads), smem, s, args);
    }
    const size_t smem = static_cast<size_t>(NT) * (g.cols + 2ull * g.chunks) * sizeof(float);
    auto fn = q4_matvec_fast_kernel<XT, YT, LPR, CPL, NT>;
    cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    MvSet set;
    const uint32_t ctas = set_of(a, kRowsPerCta, set);
    MvFuse fz{a.norm_w, a.eps, a.residual};
    Q4Geom gg = g;
    const XT* x = static_cast<const XT*>(a.x);
    uint32_t batch = a.batch;
    void* args[] = {(void*)&set, (void*)&gg, (void*)&x, (void*)&batch, (void*)&fz};
    return launch_with_pdl(reinterpret_cast<const void*>(fn), dim3(ctas), dim3(kMvThreads), smem, s, args);
}

static bool weights_aligned(const uint8_t* p, const uint16_t* sc, const uint16_t* bi) {
    return reinterpret_cast<uintptr_t>(p) % 16 == 0 && reinterpret_cast<uintptr_t>(sc) % 8 == 0 &&
           reinterpret_cast<uintptr_t>(bi) % 8 == 0;
}

template <typename XT, typename YT>
static cudaError_t q4_matvec_launch_t(const Q4MatvecArgs& a, cudaStream_t s) {
    constexpr size_t kSmemLimit = 200 * 1024;
    const size_t xelem = a.x_dtype == PBMOE_BF16 ? 2 : 4;
    const bool fused = a.norm_w || a.residual || a.packed2 || a.set_count > 1;
    // every matrix of the launch must suit the kernel
    bool all_aligned = true, all_fast = true;
    auto visit = [&](const uint8_t* p, const uint16_t* sc, const uint16_t* bi) {
        all_aligned = all_aligned && weights_aligned(p, sc, bi);
        all_fast = all_fast && q4_fast_ok(a.cols, a.group, p);
    };
    if (a.set_count) {
        for (uint32_t i = 0; i < a.set_count; ++i) visit(a.set[i].packed, a.set[i].scales, a.set[i].biases);
    } else {
        visit(a.packed, a.scales, a.biases);
        if (a.packed2) visit(a.packed2, a.scales2, a.biases2);
    }
    // plain calls of one or two tokens: the CUDA-core kernel (more weight
    // bytes in flight per warp, one wave of CTAs; a matrix set streams
    // through the persistent kernel); larger batches and the fused forms
    // (input norm, residual, a second matrix): the tensor-core kernel, whose
    // shorter instruction stream after the dependency wait wins on the
    // latency-bound decode projections
    const bool fused_single = a.norm_w || a.residual || a.packed2;
    if ((a.batch > 2 || fused_single) && a.group == kMmaGroup && a.cols % 256 == 0 && all_aligned &&
        reinterpret_cast<uintptr_t>(a.x) % 16 == 0) {
        cudaError_t e = launch_mma<XT, YT>(a, s);
        if (e != cudaErrorNotSupported) return e;
    }
    if (all_fast && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && (a.cols * xelem) % 16 == 0) {
        Q4Geom g{a.rows, a.cols, (a.cols + a.group - 1) / a.group, a.cols / 32, ilog2_u32(a.group / 32)};
        const size_t per_tok = (g.cols + 2ull * g.chunks) * sizeof(float);
        const bool multi = a.batch > 1 && 4 * per_tok <= kSmemLimit;
        if (per_tok <= kSmemLimit) {
            if (g.chunks >= 32) {
                return multi ? launch_fast<XT, YT, 32, 2, 4>(a, g, s) : launch_fast<XT, YT, 32, 2, 1>(a, g, s);
            } else if (g.chunks >= 16) {
                return multi ? launch_fast<XT, YT, 16, 1, 4>(a, g, s) : launch_fast<XT, YT, 16, 1, 1>(a, g, s);
            } else if (g.chunks >= 8) {
                return multi ? launch_fast<XT, YT, 8, 1, 4>(a, g, s) : launch_fast<XT, YT, 8, 1, 1>(a, g, s);
            }
        }
    }
    if (fused) return cudaErrorNotSupported;  // the per-element kernel has no fused forms
    const size_t smem = static_cast<size_t>(a.cols) * sizeof(float);
    if (smem > kSmemLimit) return cudaErrorNotSupported;
    auto fn = q4_matvec_generic_kernel<XT, YT>;
    cudaError_t err = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const dim3 grid((a.rows + (kMvThreads / 32) - 1) / (kMvThreads / 32));
    fn<<<grid, kMvThreads, smem, s>>>(a.packed, a.scales, a.biases, a.rows, a.cols, a.group,
                                      static_cast<const XT*>(a.x), static_cast<YT*>(a.y), a.batch);
    return cudaGetLastError();
}

cudaError_t q4_matvec_launch(const Q4MatvecArgs& a, cudaStream_t s) {
    if (a.x_dtype == PBMOE_BF16)
        return a.y_dtype == PBMOE_BF16 ? q4_matvec_launch_t<uint16_t, uint16_t>(a, s)
                                       : q4_matvec_launch_t<uint16_t, float>(a, s);
    return a.y_dtype == PBMOE_BF16 ? q4_matvec_launch_t<float, uint16_t>(a, s) : q4_matvec_launch_t<float, float>(a, s);
}

}  // namespace pbmoe
