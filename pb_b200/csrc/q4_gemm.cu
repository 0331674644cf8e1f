// q4_gemm.cu — prefill Q4 GEMM: Y[m, n] = sum_k X[m, k] * (q[n, k] * s[n, g(k)] + b[n, g(k)])
// for a dense weight (config 2: X bf16 [2048 x 2048], W Q4 [5120 x 2048]) and,
// grouped, for per-expert weights with the routes bucketed by expert.
//
// Reference: the layer-major prefill path (qwen_layer_major_group_plan,
// metal/mod.rs:3197-3233; qwen_layer_major_gather, shaders.metal:1743-1754;
// q4_mmap_fma_matvec_batch_bf16_scale_bias, shaders.metal:973-1057), which
// re-streams every weight row for each pair of input rows. Here a CTA holds a
// 128-row weight tile against 64 or 128 tokens: each weight is read from L2
// once per CTA, dequantised once in registers and used by up to 16 mma.sync
// (16 weight rows x 8 tokens x 16 k each), accumulating in fp32.
//
// Operands are fp16: w = q*s + b is rounded once to fp16 (exact q from the
// 1024+q bit trick, then fma.rn.f16x2), and the bf16 activations convert to
// fp16 exactly while they are staged. bf16 weights would carry 2^-9 relative
// rounding per weight (up to ~0.9% max-relative error against the f32
// reference on config-2 shapes); fp16 keeps 11 bits (errors ~1e-6 before the
// output rounding). An activation of magnitude >= 65536 (or non-finite) has
// no fp16 value: the tile latches PBMOE_DEV_ERR_F16_RANGE.
//
// Layout per CTA: 8 warps = 4 (32 weight rows: two 16-row A tiles) x 2 (64
// tokens: eight 8-token B tiles). K advances one 64-wide scale group per
// stage: the group's 128 x 32-byte nibble rows arrive by cp.async, the
// tokens' 128 x 64 activations are staged through registers into pair order
// (x0,x4),(x1,x5),(x2,x6),(x3,x7) per 8-k slot, the order in which the
// unpacked nibble pairs feed the mma.

#include "kernels.h"
#include "pipe.cuh"
#include "q4_mma.cuh"

namespace pbmoe {

constexpr int kGemmRows = 128;  // weight rows (output columns) per CTA
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 256;
constexpr uint32_t kXSlotStride = 9;  // 8 slots of 16 bytes + 1 pad per token row (bank-conflict free)
constexpr uint32_t kWStage = kGemmRows * 32;  // one group of nibbles per weight row
constexpr uint32_t kYStride = kGemmRows + 4;  // f32 epilogue tile row (bank-conflict free)

// CTA shape: 8 warps = WR (row warps, AT 16-row A tiles each) x WT (token
// warps, 64 tokens = eight 8-token B tiles each); WR * AT * 16 = 128 rows.
template <int WR, int AT, int WT>
struct GemmShape {
    static_assert(WR * WT == kGemmThreads / 32 && WR * AT * 16 == kGemmRows, "CTA shape");
    static constexpr int kToks = WT * 64;
    static constexpr uint32_t kXStage = kToks * kXSlotStride * 16;
    static constexpr size_t kStageBytes = size_t(kGemmStages) * (kWStage + kXStage);
    static_assert(kStageBytes >= size_t(kToks) * kYStride * 4, "epilogue tile fits in the stages");
    // W stages, X stages, the tile's scales and biases for every group
    static constexpr size_t smem(uint32_t groups) { return kStageBytes + 2 * size_t(kGemmRows) * groups * 2; }
};
using DenseShape = GemmShape<4, 2, 2>;    // 128 rows x 128 tokens
using GroupedShape = GemmShape<8, 1, 1>;  // 128 rows x 64 tokens (about 40 routes per expert)

constexpr uint32_t kF16Offset = 0x64006400u;  // f16x2 (1024.0, 1024.0): 1024 + q is exact for q < 16

__device__ __forceinline__ uint32_t f16x2_dequant(uint32_t nib_pair, uint32_t s2, uint32_t b2) {
    // (1024 + q) - 1024 = q exactly in fp16, then q * s + b rounded once
    uint32_t q, w;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(nib_pair | kF16Offset), "r"(kF16Offset));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(w) : "r"(q), "r"(s2), "r"(b2));
    return w;
}

// bf16x2 -> f16x2, exact for |v| < 65536 (f16 keeps bf16's 8 mantissa bits)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t u) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(u & 0xffff0000u)), "f"(__uint_as_float(u << 16)));
    return r;
}

__device__ __forceinline__ uint16_t bf16_to_f16_bits(uint16_t v) {
    return __half_as_ushort(__float2half_rn(__uint_as_float(static_cast<uint32_t>(v) << 16)));
}

// A fragments (rows g, g+8 of a 16-row tile) of one word pair, dequantised:
// a_lo feeds the mma of pairs 0/1 of the word, a_hi of pairs 2/3.
__device__ __forceinline__ void dequant_word_pair(uint32_t q, uint32_t r, uint32_t sg2, uint32_t bg2, uint32_t sh2,
                                                  uint32_t bh2, uint32_t (&a_lo)[4], uint32_t (&a_hi)[4]) {
    a_lo[0] = f16x2_dequant(q & 0x000F000Fu, sg2, bg2);
    a_lo[1] = f16x2_dequant(r & 0x000F000Fu, sh2, bh2);
    a_lo[2] = f16x2_dequant((q >> 4) & 0x000F000Fu, sg2, bg2);
    a_lo[3] = f16x2_dequant((r >> 4) & 0x000F000Fu, sh2, bh2);
    a_hi[0] = f16x2_dequant((q >> 8) & 0x000F000Fu, sg2, bg2);
    a_hi[1] = f16x2_dequant((r >> 8) & 0x000F000Fu, sh2, bh2);
    a_hi[2] = f16x2_dequant((q >> 12) & 0x000F000Fu, sg2, bg2);
    a_hi[3] = f16x2_dequant((r >> 12) & 0x000F000Fu, sh2, bh2);
}

__device__ __forceinline__ void mma_a4(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pair_of(uint16_t v) { return static_cast<uint32_t>(v) * 0x10001u; }

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes)
                 : "memory");
}

// One CTA tile: weight rows n0 .. n0+127 of a [N x K] Q4 matrix (rows beyond
// N are skipped) against token rows xrow(i), i < mcount <= kToks, written to
// output rows yrow(i). packed / scales / biases point at the whole matrix.
template <typename Shape, int WR, int AT, int WT, typename YT, typename XRow, typename YRow>
__device__ __forceinline__ void q4_gemm_tile(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                                             const uint16_t* __restrict__ biases, uint32_t N, uint32_t K,
                                             uint32_t n0, const uint16_t* __restrict__ x, uint32_t mcount,
                                             XRow xrow, YT* __restrict__ y, YRow yrow, uint32_t* status) {
    constexpr int kToks = Shape::kToks;
    constexpr int kXPerThread = kToks * 8 / kGemmThreads;  // 16-byte activation chunks per thread per group
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* wst = smem;                                              // [S][128 rows][32 B]
    uint4* xst = reinterpret_cast<uint4*>(smem + kGemmStages * kWStage);  // [S][toks][9 slots]
    const uint32_t G = K / 64;
    uint16_t* ssh = reinterpret_cast<uint16_t*>(smem + Shape::kStageBytes);  // [128][G]
    uint16_t* bsh = ssh + kGemmRows * G;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t rows_here = N - n0 < static_cast<uint32_t>(kGemmRows) ? N - n0 : kGemmRows;
    const size_t prow = K / 2;  // bytes per nibble row

    // scales and biases of the tile's rows, all groups (rows are contiguous;
    // the chunk holding the last row is cut at the matrix end)
    {
        const uint32_t avail = rows_here * G;  // entries that exist
        for (uint32_t i = tid; i < kGemmRows * G / 8; i += kGemmThreads) {
            const uint32_t bytes = i * 8 >= avail ? 0u : (avail - i * 8 >= 8 ? 16u : (avail - i * 8) * 2);
            const size_t src = static_cast<size_t>(n0) * G + (bytes ? i * 8 : 0);
            cp_async16_zfill(ssh + i * 8, scales + src, bytes);
            cp_async16_zfill(bsh + i * 8, biases + src, bytes);
        }
    }
    auto issue_w = [&](uint32_t grp, int s) {
        // 128 rows x 32 bytes = 256 chunks: one per thread
        const uint32_t r = tid >> 1, c = tid & 1;
        const bool ok = r < rows_here;
        const uint8_t* src = packed + (static_cast<size_t>(n0 + (ok ? r : 0)) * prow + grp * 32 + c * 16);
        cp_async16_zfill(wst + s * kWStage + r * 32 + c * 16, src, ok ? 16u : 0u);
    };
    // activations of group grp: toks x 8 slots of 16 bytes
    uint4 xr[kXPerThread];
    uint32_t xmax = 0;  // per-half max of |x| bits: the fp16 range check
    auto load_x = [&](uint32_t grp) {
#pragma unroll
        for (int j = 0; j < kXPerThread; ++j) {
            const uint32_t i = j * kGemmThreads + tid, tok = i >> 3, slot = i & 7;
            xr[j] = tok < mcount ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(xrow(tok)) * K +
                                                                       grp * 64 + slot * 8))
                                 : make_uint4(0, 0, 0, 0);
        }
    };
    auto store_x = [&](int s) {
#pragma unroll
        for (int j = 0; j < kXPerThread; ++j) {
            const uint32_t i = j * kGemmThreads + tid, tok = i >> 3, slot = i & 7;
            const uint4 r = xr[j];
            xmax = __vmaxu2(xmax, __vmaxu2(__vmaxu2(r.x & 0x7fff7fffu, r.y & 0x7fff7fffu),
                                           __vmaxu2(r.z & 0x7fff7fffu, r.w & 0x7fff7fffu)));
            xst[s * (kToks * kXSlotStride) + tok * kXSlotStride + slot] =
                make_uint4(bf16x2_to_f16x2(pack_pairs_lo(r.x, r.z)), bf16x2_to_f16x2(pack_pairs_hi(r.x, r.z)),
                           bf16x2_to_f16x2(pack_pairs_lo(r.y, r.w)), bf16x2_to_f16x2(pack_pairs_hi(r.y, r.w)));
        }
    };

    asm volatile("cp.async.commit_group;" ::: "memory");  // scales and biases: their own group
#pragma unroll
    for (int s = 0; s < kGemmStages - 1; ++s) {
        if (static_cast<uint32_t>(s) < G) {
            issue_w(s, s);
            load_x(s);
            store_x(s);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // scales and biases to fp16 in place (bf16 values in the fp16 normal
    // range convert exactly)
    asm volatile("cp.async.wait_group %0;" ::"n"(kGemmStages - 1) : "memory");
    __syncthreads();
    for (uint32_t i = tid; i < 2 * kGemmRows * G; i += kGemmThreads) ssh[i] = bf16_to_f16_bits(ssh[i]);

    const uint32_t rs = (warp % WR) * (16 * AT);  // this warp's weight rows within the tile
    const uint32_t ts = (warp / WR) * 64;         // this warp's tokens within the tile
    // 8-token B tiles that hold a token of this warp (warp-uniform)
    const int ntiles = mcount > ts ? min(8, static_cast<int>((mcount - ts + 7) / 8)) : 0;
    float acc[AT][8][4];
#pragma unroll
    for (int a = 0; a < AT; ++a)
#pragma unroll
        for (int n = 0; n < 8; ++n) acc[a][n][0] = acc[a][n][1] = acc[a][n][2] = acc[a][n][3] = 0.f;

    for (uint32_t grp = 0; grp < G; ++grp) {
        const int s = static_cast<int>(grp % kGemmStages);
        const uint32_t nxt = grp + kGemmStages - 1;
        if (nxt < G) load_x(nxt);  // global loads in flight during this group's math
        asm volatile("cp.async.wait_group %0;" ::"n"(kGemmStages - 2) : "memory");
        __syncthreads();  // group grp's nibbles and activations visible; stage (grp-1) free
        const unsigned char* ws = wst + s * kWStage;
        const uint4* xs = xst + s * (kToks * kXSlotStride);
        uint32_t sg2[AT], bg2[AT], sh2[AT], bh2[AT];
        uint2 wg[AT], wh[AT];
#pragma unroll
        for (int a = 0; a < AT; ++a) {
            const uint32_t r = rs + a * 16 + g;
            sg2[a] = pair_of(ssh[r * G + grp]);
            bg2[a] = pair_of(bsh[r * G + grp]);
            sh2[a] = pair_of(ssh[(r + 8) * G + grp]);
            bh2[a] = pair_of(bsh[(r + 8) * G + grp]);
            wg[a] = *reinterpret_cast<const uint2*>(ws + r * 32 + 8 * t);
            wh[a] = *reinterpret_cast<const uint2*>(ws + (r + 8) * 32 + 8 * t);
        }
        // per word m (2t, then 2t+1): dequantised A fragments, then the B tiles
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            uint32_t alo[AT][4], ahi[AT][4];
#pragma unroll
            for (int a = 0; a < AT; ++a)
                dequant_word_pair(m ? wg[a].y : wg[a].x, m ? wh[a].y : wh[a].x, sg2[a], bg2[a], sh2[a], bh2[a],
                                  alo[a], ahi[a]);
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                if (n < ntiles) {
                    const uint4 xb = xs[(ts + n * 8 + g) * kXSlotStride + 2 * t + m];
#pragma unroll
                    for (int a = 0; a < AT; ++a) {
                        mma_a4(acc[a][n], alo[a], xb.x, xb.y);
                        mma_a4(acc[a][n], ahi[a], xb.z, xb.w);
                    }
                }
            }
        }
        if (nxt < G) {
            const int sn = static_cast<int>(nxt % kGemmStages);
            issue_w(nxt, sn);
            store_x(sn);  // stage sn = (grp-1) % S, released by the barrier above
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (((xmax & 0xffffu) >= 0x4780u || (xmax >> 16) >= 0x4780u) && status)
        atomicOr(status, PBMOE_DEV_ERR_F16_RANGE);  // some |x| >= 65536 or non-finite
    __syncthreads();  // every warp is done with the stages: reuse them for the output tile

    // epilogue: acc[a][n] = rows (r, r+8) x tokens (2t, 2t+1) -> f32 tile
    // [toks][128], then whole 16-byte runs of each output row
    float* ytile = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int a = 0; a < AT; ++a) {
        const uint32_t r = rs + a * 16 + g;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            if (n < ntiles) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t tok = ts + n * 8 + 2 * t + c;
                    ytile[tok * kYStride + r] = acc[a][n][c];
                    ytile[tok * kYStride + r + 8] = acc[a][n][2 + c];
                }
            }
        }
    }
    __syncthreads();
    constexpr int kPerChunk = 16 / sizeof(YT);  // outputs per 16-byte store
    constexpr int kChunks = kGemmRows / kPerChunk;
    const bool vec_ok = (N % kPerChunk) == 0;  // row starts stay 16-byte aligned
    for (uint32_t i = tid; i < mcount * kChunks; i += kGemmThreads) {
        const uint32_t tok = i / kChunks, col = (i % kChunks) * kPerChunk;
        if (col >= rows_here) continue;
        const float* src = ytile + tok * kYStride + col;
        YT* dst = y + static_cast<size_t>(yrow(tok)) * N + n0 + col;
        if (vec_ok && col + kPerChunk <= rows_here) {
            if constexpr (sizeof(YT) == 4) {
                *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
            } else {
                const float4 lo = *reinterpret_cast<const float4*>(src);
                const float4 hi = *reinterpret_cast<const float4*>(src + 4);
                *reinterpret_cast<uint4*>(dst) = make_uint4(f2_to_bf16x2(lo.x, lo.y), f2_to_bf16x2(lo.z, lo.w),
                                                            f2_to_bf16x2(hi.x, hi.y), f2_to_bf16x2(hi.z, hi.w));
            }
        } else {
            for (int j = 0; j < kPerChunk && col + j < rows_here; ++j) store_act(dst, j, src[j]);
        }
    }
}

// Dense: grid (ceil(N/128), ceil(M/toks)).
template <typename YT>
__global__ void __launch_bounds__(kGemmThreads, 1)
q4_gemm_dense_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                     const uint16_t* __restrict__ biases, uint32_t N, uint32_t K, const uint16_t* __restrict__ x,
                     uint32_t M, YT* __restrict__ y, uint32_t* status) {
    constexpr int kToks = DenseShape::kToks;
    const uint32_t n0 = blockIdx.x * kGemmRows, m0 = blockIdx.y * kToks;
    const uint32_t mcount = M - m0 < static_cast<uint32_t>(kToks) ? M - m0 : kToks;
    q4_gemm_tile<DenseShape, 4, 2, 2, YT>(packed, scales, biases, N, K, n0, x, mcount,
                                          [m0](uint32_t i) { return m0 + i; }, y,
                                          [m0](uint32_t i) { return m0 + i; }, status);
}

// Grouped (layer-major prefill): grid (ceil(N/128), tile bound). Tile j of
// the y dimension is the j-th 64-route run over the groups in slot order;
// the CTA finds its (slot, first route) by a block scan of the group sizes.
// Rows are gathered from x by source_rows and written to y in grouped order.
template <typename YT>
__global__ void __launch_bounds__(kGemmThreads, 2)
q4_gemm_grouped_kernel(Q4GroupedArgs a) {
    constexpr int kToks = GroupedShape::kToks;
    __shared__ uint32_t found_slot, found_tok0, warp_tot[kGemmThreads / 32];
    const uint32_t unique = min(*a.unique_count, a.max_unique);
    const uint32_t j = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) found_slot = 0xffffffffu;
    uint32_t base = 0;  // tiles of the slots before this chunk
    for (uint32_t c0 = 0; c0 < unique; c0 += kGemmThreads) {
        const uint32_t slot = c0 + tid;
        const uint32_t cnt = slot < unique ? a.groups[2 * slot + 1] : 0u;
        const uint32_t tiles = (cnt + kToks - 1) / kToks;
        uint32_t incl = tiles;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += v;
        }
        __syncthreads();  // warp_tot of the previous chunk consumed
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        uint32_t before = base, total = 0;
        for (int w = 0; w < kGemmThreads / 32; ++w) {
            if (w < warp) before += warp_tot[w];
            total += warp_tot[w];
        }
        const uint32_t lo = before + incl - tiles;
        if (tiles && j >= lo && j < lo + tiles) {
            found_slot = slot;
            found_tok0 = (j - lo) * kToks;
        }
        base += total;
    }
    __syncthreads();
    const uint32_t slot = found_slot;
    if (slot == 0xffffffffu) return;  // beyond the last tile
    const uint32_t start = a.groups[2 * slot], cnt = a.groups[2 * slot + 1];
    const uint32_t first = start + found_tok0;
    const uint32_t mcount = min(cnt - found_tok0, static_cast<uint32_t>(kToks));
    const uint32_t expert = a.slot_experts[slot];
    if (expert >= a.num_experts || first + mcount > a.routes) {
        if (tid == 0 && a.status) atomicOr(a.status, PBMOE_DEV_ERR_EXPERT_ID);
        return;
    }
    const uint8_t* e = a.experts + static_cast<size_t>(expert) * a.expert_bytes;
    const uint32_t* src_rows = a.source_rows + first;
    q4_gemm_tile<GroupedShape, 8, 1, 1, YT>(
        e + a.packed_offset, reinterpret_cast<const uint16_t*>(e + a.scales_offset),
        reinterpret_cast<const uint16_t*>(e + a.biases_offset), a.rows, a.cols, blockIdx.x * kGemmRows,
        static_cast<const uint16_t*>(a.x), mcount, [src_rows](uint32_t i) { return __ldg(src_rows + i); },
        static_cast<YT*>(a.y), [first](uint32_t i) { return first + i; }, a.status);
}

bool q4_gemm_supported(uint32_t N, uint32_t K, uint32_t group) {
    return group == 64 && K % 64 == 0 && K >= 64 && N > 0 && DenseShape::smem(K / 64) <= 200 * 1024 &&
           GroupedShape::smem(K / 64) <= 110 * 1024;
}

template <typename KernelT>
static cudaError_t set_smem(KernelT* k, size_t smem) {
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
}

cudaError_t q4_gemm_launch(const Q4GemmArgs& a, cudaStream_t s) {
    const dim3 grid((a.rows + kGemmRows - 1) / kGemmRows, (a.m + DenseShape::kToks - 1) / DenseShape::kToks);
    const size_t smem = DenseShape::smem(a.cols / 64);
    cudaError_t e;
    if (a.y_dtype == PBMOE_F32) {
        if ((e = set_smem(q4_gemm_dense_kernel<float>, smem)) != cudaSuccess) return e;
        q4_gemm_dense_kernel<float><<<grid, kGemmThreads, smem, s>>>(a.packed, a.scales, a.biases, a.rows, a.cols,
                                                                     static_cast<const uint16_t*>(a.x), a.m,
                                                                     static_cast<float*>(a.y), a.status);
    } else {
        if ((e = set_smem(q4_gemm_dense_kernel<uint16_t>, smem)) != cudaSuccess) return e;
        q4_gemm_dense_kernel<uint16_t><<<grid, kGemmThreads, smem, s>>>(a.packed, a.scales, a.biases, a.rows,
                                                                        a.cols, static_cast<const uint16_t*>(a.x),
                                                                        a.m, static_cast<uint16_t*>(a.y), a.status);
    }
    return cudaGetLastError();
}

uint32_t q4_grouped_tile_bound(uint32_t routes, uint32_t max_unique) {
    // sum over slots of ceil(count / toks) <= routes / toks + slots
    return (routes + GroupedShape::kToks - 1) / GroupedShape::kToks + max_unique;
}

cudaError_t q4_gemm_grouped_launch(const Q4GroupedArgs& a, cudaStream_t s) {
    const dim3 grid((a.rows + kGemmRows - 1) / kGemmRows, q4_grouped_tile_bound(a.routes, a.max_unique));
    const size_t smem = GroupedShape::smem(a.cols / 64);
    cudaError_t e;
    if (a.y_dtype == PBMOE_F32) {
        if ((e = set_smem(q4_gemm_grouped_kernel<float>, smem)) != cudaSuccess) return e;
        q4_gemm_grouped_kernel<float><<<grid, kGemmThreads, smem, s>>>(a);
    } else {
        if ((e = set_smem(q4_gemm_grouped_kernel<uint16_t>, smem)) != cudaSuccess) return e;
        q4_gemm_grouped_kernel<uint16_t><<<grid, kGemmThreads, smem, s>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace pbmoe
