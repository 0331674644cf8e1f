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
//   2. mla_attn_kernel     one CTA per (KV split, sequence): every 32-token
//                          tile of the split's latent cache is read from HBM
//                          once (cp.async, double-buffered) and serves all 16
//                          heads. S = Q' K^T (16 heads = the mma's M; Q' as
//                          bf16 hi + lo so scores keep ~16 mantissa bits),
//                          online softmax in base 2, O += P C with P in bf16.
//                          Writes the split's (max, sum, O[16 x 512]).
//   3. mla_merge_out_kernel one CTA per (head, sequence): merges the splits'
//                          partials into ctx (in shared memory), then
//                          out = W_UV[h] ctx.
// The split plan keeps batch x splits within one wave (the attention kernel
// runs two CTAs per SM).
// Shapes: 16 heads, latent 512, rope 64, v 128, nope <= 128, batch <= 32.

#include "common.cuh"
#include "kernels.h"
#include "rope.cuh"

namespace pbmoe {

constexpr uint32_t kMlaHeads = 16, kMlaLatent = 512, kMlaRope = 64, kMlaV = 128;
constexpr uint32_t kMlaK = kMlaLatent + kMlaRope;  // 576: score dimension
constexpr uint32_t kMlaTile = 32;                  // tokens per tile
constexpr uint32_t kMlaWarps = 4;
constexpr uint32_t kMlaThreads = kMlaWarps * 32;
// shared-memory row strides (bytes), padded by 16 against ldmatrix bank conflicts
constexpr uint32_t kCRow = kMlaLatent * 2 + 16;   // c_kv rows
constexpr uint32_t kRRow = kMlaRope * 2 + 16;     // k_rope rows
constexpr uint32_t kPRow = kMlaTile * 2 + 16;     // P rows
constexpr uint32_t kStageBytes = kMlaTile * (kCRow + kRRow);
constexpr uint32_t kMlaPartialFloats = 2 + kMlaLatent;  // max, sum, O
// Scores: warp w sums k-steps 9w .. 9w+8 of the 36 for every token of the tile
constexpr uint32_t kKSteps = kMlaK / 16;                   // 36 k-steps of the score MMAs
constexpr uint32_t kKStepsPerWarp = kKSteps / kMlaWarps;   // 9
constexpr uint32_t kColsPerWarp = kMlaLatent / kMlaWarps;  // 128 context columns per warp
constexpr uint32_t kTokNt = kMlaTile / 8;                  // 4 n-tiles of tokens per tile
static_assert(kKSteps % kMlaWarps == 0, "score k-steps split evenly over the warps");
static_assert(kMlaTile == 8 * kMlaWarps, "one n-tile of tokens per warp in the softmax");
constexpr uint32_t kSRow = kMlaTile + 8;  // partial-score rows (floats), padded against bank conflicts
constexpr size_t kMlaSmem = 2 * size_t(kStageBytes) + kMlaHeads * kPRow + kMlaWarps * kMlaHeads * 4 * 2 +
                            size_t(kMlaWarps) * kMlaHeads * kSRow * 4;
static_assert(kMlaCtasPerSm * (kMlaSmem + 1024) <= 228 * 1024, "two attention CTAs per SM");

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
// 16-byte global -> shared async copy of a chunk known to be in range.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return static_cast<uint32_t>(f32_to_bf16_bits(lo)) | (static_cast<uint32_t>(f32_to_bf16_bits(hi)) << 16);
}

// ---------------------------------------------------------------- 1. absorb
// grid (heads, latent/64), 256 threads. Thread (rg = tid/8, cb = tid%8) holds
// W_UK[h][d][64*blockIdx.y + 8cb .. +7] for d = rg, rg+32, rg+64, rg+96 (four
// 16-byte loads issued before the dependency wait) and sums those rows'
// contributions for 8 sequences at a time; the 4 lanes of a warp that share
// cb add theirs with shuffles, the 8 warps theirs in shared memory. Writes
// Q'[b][h][0..511] = q_lat * k and Q'[b][h][512..575] = q_rope * k,
// k = scale * log2(e). nope <= 128 (host-checked).
//
// kRope (f32 queries): the call also does the RoPE + cache append of
// mla_rope_append_kernel on the way. The first column block's rope threads
// rotate each sequence's rope part of head h in place (as that kernel does) and
// scale the rotated values into Q'; grid rows past latent/64 append the key
// and latent rows, one token per CTA (rope_append_kv). A token whose position
// is past its cache or the RoPE table is left unrotated and unwritten, with
// PBMOE_DEV_ERR_POSITION latched.
constexpr uint32_t kAbsorbMaxNope = 128;
template <typename QT, bool kRope = false>
__global__ void __launch_bounds__(256) mla_absorb_kernel(const QT* __restrict__ q, uint32_t batch, uint32_t nope,
                                                         const uint16_t* __restrict__ w_uk, float k,
                                                         float* __restrict__ qp, RopeAppendArgs ra) {
    __shared__ float qs[kMlaMaxBatch * kAbsorbMaxNope];
    __shared__ float red[8][8][64];  // [warp][sequence of the pass][column]
    const uint32_t h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if constexpr (kRope) {
        if (blockIdx.y >= kMlaLatent / 64) {  // the cache append of token (row - 8) * 16 + h
            pdl_wait();
            pdl_launch_dependents();
            const uint32_t b = (blockIdx.y - kMlaLatent / 64) * kMlaHeads + blockIdx.x;
            uint32_t pos;
            if (b < batch && rope_token_position(ra, b, pos)) rope_append_kv(ra, b, pos, &red[0][0][0]);
            return;
        }
    }
    const uint32_t cb = tid & 7, rg = tid >> 3;
    const uint32_t qdim = nope + kMlaRope;
    // W_UK does not depend on the earlier kernels: its loads are issued before
    // waiting for them
    uint4 wv[kAbsorbMaxNope / 32];
#pragma unroll
    for (uint32_t i = 0; i < kAbsorbMaxNope / 32; ++i) {
        const uint32_t d = rg + 32 * i;
        wv[i] = d < nope ? __ldg(reinterpret_cast<const uint4*>(w_uk + (static_cast<size_t>(h) * nope + d) * kMlaLatent +
                                                                blockIdx.y * 64 + cb * 8))
                         : make_uint4(0, 0, 0, 0);
    }
    pdl_wait();
    pdl_launch_dependents();
    // the query of every sequence (and, in the first column block, its rope
    // part), 4 and 8 values per thread in flight at a time: one L2 round
    // trip each at batch <= 8
    const bool rope_cta = blockIdx.y == 0 && tid < kMlaRope;
    for (uint32_t i0 = 0; i0 < batch * nope; i0 += 4 * 256) {
        float qv[4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t i = i0 + tid + j * 256;
            qv[j] = i < batch * nope ? load_act(q, (static_cast<size_t>(i / nope) * kMlaHeads + h) * qdim + i % nope)
                                     : 0.f;
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t i = i0 + tid + j * 256;
            if (i < batch * nope) qs[i] = qv[j];
        }
    }
    if (rope_cta) {
        if constexpr (kRope) {
            // thread tid writes split-half element tid of head h's rope part: from
            // pair p = tid % 32, cos/sin of the token's position
            float* qf = reinterpret_cast<float*>(const_cast<QT*>(q));
            const uint32_t p = tid & 31u, half = kMlaRope / 2;
            for (uint32_t b0 = 0; b0 < batch; b0 += 8) {
                float x0[8], x1[8], xs[8];
                float2 c[8];
                bool ok[8];
#pragma unroll
                for (uint32_t j = 0; j < 8; ++j) {
                    const uint32_t b = b0 + j;
                    ok[j] = false;
                    x0[j] = x1[j] = xs[j] = 0.f;
                    c[j] = make_float2(0.f, 0.f);
                    if (b < batch) {
                        const float* qr = qf + (static_cast<size_t>(b) * kMlaHeads + h) * qdim + nope;
                        const uint32_t pos = ra.positions[b];
                        ok[j] = pos < ra.max_positions && pos < ra.cache_len;
                        x0[j] = qr[2 * p];
                        x1[j] = qr[2 * p + 1];
                        xs[j] = qr[tid];
                        if (ok[j]) c[j] = ra.table[static_cast<size_t>(pos) * half + p];
                    }
                }
                asm volatile("bar.sync 1, 64;" ::: "memory");  // the 64 rope threads: every read before any write
#pragma unroll
                for (uint32_t j = 0; j < 8; ++j) {
                    const uint32_t b = b0 + j;
                    if (b < batch) {
                        const float r = !ok[j] ? xs[j]
                                        : tid < half ? __fsub_rn(__fmul_rn(x0[j], c[j].x), __fmul_rn(x1[j], c[j].y))
                                                     : __fadd_rn(__fmul_rn(x1[j], c[j].x), __fmul_rn(x0[j], c[j].y));
                        if (ok[j]) qf[(static_cast<size_t>(b) * kMlaHeads + h) * qdim + nope + tid] = r;
                        qp[(static_cast<size_t>(b) * kMlaHeads + h) * kMlaK + kMlaLatent + tid] = r * k;
                    }
                }
            }
        } else {
            for (uint32_t b0 = 0; b0 < batch; b0 += 8) {
                float rv[8];
#pragma unroll
                for (uint32_t j = 0; j < 8; ++j)
                    rv[j] = b0 + j < batch ? load_act(q, (static_cast<size_t>(b0 + j) * kMlaHeads + h) * qdim + nope + tid)
                                           : 0.f;
#pragma unroll
                for (uint32_t j = 0; j < 8; ++j)
                    if (b0 + j < batch) qp[(static_cast<size_t>(b0 + j) * kMlaHeads + h) * kMlaK + kMlaLatent + tid] = rv[j] * k;
            }
        }
    }
    __syncthreads();
    for (uint32_t b0 = 0; b0 < batch; b0 += 8) {
        float acc[8][8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[j][c] = 0.f;
#pragma unroll
        for (uint32_t i = 0; i < kAbsorbMaxNope / 32; ++i) {
            const uint32_t d = rg + 32 * i;
            if (d < nope) {
                const uint32_t wq[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
                float wf[8];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    wf[2 * c] = bf16_bits_to_f32(wq[c] & 0xffffu);
                    wf[2 * c + 1] = bf16_bits_to_f32(wq[c] >> 16);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float qv = b0 + j < batch ? qs[(b0 + j) * nope + d] : 0.f;
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[j][c] = fmaf(qv, wf[c], acc[j][c]);
                }
            }
        }
        // the warp's 4 row groups of column block cb: lanes cb, cb+8, cb+16, cb+24
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                acc[j][c] += __shfl_xor_sync(kFull, acc[j][c], 8);
                acc[j][c] += __shfl_xor_sync(kFull, acc[j][c], 16);
            }
        if (lane < 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int c = 0; c < 8; ++c) red[warp][j][lane * 8 + c] = acc[j][c];
        }
        __syncthreads();
        for (uint32_t o = tid; o < 8 * 64; o += 256) {
            const uint32_t j = o / 64, col = o % 64;
            if (b0 + j < batch) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) v += red[w][j][col];
                qp[(static_cast<size_t>(b0 + j) * kMlaHeads + h) * kMlaK + blockIdx.y * 64 + col] = v * k;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- 2. attention
// grid (splits, batch), 128 threads (4 warps), two CTAs per SM so that one
// CTA's softmax and barriers overlap the other's MMAs. Per 32-token tile
// (double-buffered cp.async): warp w computes partial scores of every token
// of the tile over score dims 144w .. 144w+143 (its Q' hi and lo fragments
// held in registers for the whole split: four independent n-tile
// accumulators per half), the partials meet in shared memory, summed in warp
// order; warp w then owns tokens 8w .. 8w+7 for the online softmax and
// context columns 128w .. 128w+127 for O += P C. Fragment loads run one step
// ahead of the MMAs that use them.
// fresh_pos (nullable): per sequence, the cache row the absorb launch of the
// same call appends while this kernel may already run; every other attended
// row was written before the call (the absorb launch passed its own
// dependency wait before this grid launched), so a first tile without that
// row is requested before this kernel's wait.
__global__ void __launch_bounds__(kMlaThreads, kMlaCtasPerSm) mla_attn_kernel(const float* __restrict__ qp,
                                                                               MlaSeqs seqs, uint32_t split_tokens,
                                                                               uint32_t splits,
                                                                               float* __restrict__ partial,
                                                                               const uint32_t* __restrict__ fresh_pos) {
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* stage0 = smem;
    unsigned char* pbuf = stage0 + 2 * kStageBytes;
    float* wmax = reinterpret_cast<float*>(pbuf + kMlaHeads * kPRow);  // [warps][16]
    float* spart = wmax + kMlaWarps * kMlaHeads * 2;                     // [warps][16 heads][kSRow]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t b = blockIdx.y, sp = blockIdx.x;
    const uint32_t L = seqs.len[b];
    const uint32_t t0 = sp * split_tokens, t1 = min(L, t0 + split_tokens);
    float* out = partial + (static_cast<size_t>(b) * splits + sp) * kMlaHeads * kMlaPartialFloats;
    const float NEG_INF = -__int_as_float(0x7f800000);
    if (t0 >= t1) {  // empty split: contributes nothing
        pdl_wait();
        pdl_launch_dependents();
        for (uint32_t i = threadIdx.x; i < kMlaHeads * kMlaPartialFloats; i += blockDim.x)
            out[i] = (i % kMlaPartialFloats == 0) ? NEG_INF : 0.f;
        return;
    }
    const uint16_t* ckv = seqs.c_kv[b];
    const uint16_t* krope = seqs.k_rope[b];
    const uint32_t ntiles = (t1 - t0 + kMlaTile - 1) / kMlaTile;

    // Thread i copies 16-byte chunk (i % 64) of tile rows i / 64 + 2j (c_kv)
    // and chunk (i % 8) of rows i / 8 + 16j (k_rope); a whole tile takes
    // fixed offsets from two base pointers, the split's last tile zero-fills
    // rows past its end.
    static_assert(kMlaThreads == 128 && kMlaTile == 32, "copy mapping assumes 128 threads, 32-token tiles");
    const uint32_t c_row = threadIdx.x >> 6, c_ch = threadIdx.x & 63;
    const uint32_t r_row = threadIdx.x >> 3, r_ch = threadIdx.x & 7;
    auto issue_tile = [&](uint32_t tile, int buf) {
        unsigned char* st = stage0 + buf * kStageBytes;
        unsigned char* rt = st + kMlaTile * kCRow;
        const uint32_t tb = t0 + tile * kMlaTile;
        const uint16_t* csrc = ckv + static_cast<size_t>(tb + c_row) * kMlaLatent + c_ch * 8;
        const uint16_t* rsrc = krope + static_cast<size_t>(tb + r_row) * kMlaRope + r_ch * 8;
        unsigned char* cdst = st + c_row * kCRow + c_ch * 16;
        unsigned char* rdst = rt + r_row * kRRow + r_ch * 16;
        if (tb + kMlaTile <= t1) {
#pragma unroll
            for (uint32_t j = 0; j < kMlaTile / 2; ++j) cp16(cdst + j * 2 * kCRow, csrc + j * 2 * kMlaLatent);
#pragma unroll
            for (uint32_t j = 0; j < kMlaTile / 16; ++j) cp16(rdst + j * 16 * kRRow, rsrc + j * 16 * kMlaRope);
        } else {
            for (uint32_t j = 0; j < kMlaTile / 2; ++j) {
                const bool ok = tb + c_row + 2 * j < t1;
                cp16_zfill(cdst + j * 2 * kCRow, ok ? csrc + j * 2 * kMlaLatent : ckv, ok ? 16u : 0u);
            }
            for (uint32_t j = 0; j < kMlaTile / 16; ++j) {
                const bool ok = tb + r_row + 16 * j < t1;
                cp16_zfill(rdst + j * 16 * kRRow, ok ? rsrc + j * 16 * kMlaRope : krope, ok ? 16u : 0u);
            }
        }
    };
    // the first tile before the wait unless it holds the row being appended
    const uint32_t fresh = fresh_pos ? __ldg(fresh_pos + b) : 0xffffffffu;
    const bool early = fresh < t0 || fresh >= min(t1, t0 + kMlaTile);
    if (early) {
        issue_tile(0, 0);
        cp_commit();
    }
    pdl_wait();
    pdl_launch_dependents();
    if (!early) {
        issue_tile(0, 0);
        cp_commit();
    }

    // This warp's Q' (dims 144w .. 144w+143) as mma A fragments, bf16 hi and lo
    // (residue): for k-step kk the fragment holds Q'[g][16kk + 2t, +1],
    // Q'[g+8][...], Q'[g][16kk + 8 + 2t, +1], Q'[g+8][...]
    const uint32_t kk0 = warp * kKStepsPerWarp;
    uint32_t qh[kKStepsPerWarp][4], ql[kKStepsPerWarp][4];
    {
        const float* qb = qp + static_cast<size_t>(b) * kMlaHeads * kMlaK;
        float2 v[kKStepsPerWarp][4];
#pragma unroll
        for (uint32_t j = 0; j < kKStepsPerWarp; ++j) {
            const uint32_t c = (kk0 + j) * 16 + 2 * t;
            v[j][0] = __ldcg(reinterpret_cast<const float2*>(qb + g * kMlaK + c));
            v[j][1] = __ldcg(reinterpret_cast<const float2*>(qb + (g + 8) * kMlaK + c));
            v[j][2] = __ldcg(reinterpret_cast<const float2*>(qb + g * kMlaK + c + 8));
            v[j][3] = __ldcg(reinterpret_cast<const float2*>(qb + (g + 8) * kMlaK + c + 8));
        }
#pragma unroll
        for (uint32_t j = 0; j < kKStepsPerWarp; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t h = pack_bf16x2(v[j][r].x, v[j][r].y);
                qh[j][r] = h;
                ql[j][r] = pack_bf16x2(v[j][r].x - bf16_bits_to_f32(h & 0xffffu), v[j][r].y - bf16_bits_to_f32(h >> 16));
            }
    }

    // running state: heads g and g+8 (per lane), context columns of this warp
    float m_run[2] = {NEG_INF, NEG_INF}, l_run[2] = {0.f, 0.f};
    constexpr int kONt = kColsPerWarp / 8;  // 16 n-tiles of context columns
    float o[kONt][4];
#pragma unroll
    for (int n = 0; n < kONt; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    // ldmatrix lane addressing: A (16 x 16 block): lane -> row (lane & 15), col half (lane >> 4)
    const uint32_t a_row = lane & 15, a_col = (lane >> 4) * 8;
    // B (n8 x k16) from [n][k] rows: lane -> row (lane & 7) + 8 * ((lane >> 4) & 1) for x4 over 2 n-tiles,
    // k half ((lane >> 3) & 1)
    const uint32_t b_row = (lane & 7) + ((lane >> 4) << 3), b_k = ((lane >> 3) & 1) * 8;
    const uint32_t tok0 = warp * 8;  // first token of this warp's softmax columns

    for (uint32_t tile = 0; tile < ntiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < ntiles) issue_tile(tile + 1, buf ^ 1);
        cp_commit();
        cp_wait<1>();
        __syncthreads();  // tile `tile` landed
        const unsigned char* st = stage0 + buf * kStageBytes;
        const unsigned char* rt = st + kMlaTile * kCRow;

        // ---- partial scores over this warp's k-steps, all 32 tokens
        {
            float sh[kTokNt][4], sl[kTokNt][4];
#pragma unroll
            for (int n = 0; n < kTokNt; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) sh[n][i] = sl[n][i] = 0.f;
            uint32_t fb[2][2][4];  // [step parity][16-token block][4]
            auto load_b = [&](int f, uint32_t kk) {
                const uint32_t kc = kk * 16 + b_k;
                const bool lat = kk < kMlaLatent / 16;
                const unsigned char* bsrc =
                    lat ? st + b_row * kCRow + kc * 2 : rt + b_row * kRRow + (kc - kMlaLatent) * 2;
                const uint32_t bstep = lat ? 16 * kCRow : 16 * kRRow;
                ldsm_x4(fb[f][0], bsrc);
                ldsm_x4(fb[f][1], bsrc + bstep);
            };
            load_b(0, kk0);
#pragma unroll
            for (uint32_t j = 0; j < kKStepsPerWarp; ++j) {
                const int f = j & 1;
                if (j + 1 < kKStepsPerWarp) load_b(f ^ 1, kk0 + j + 1);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    mma16816(sh[2 * q], qh[j], fb[f][q][0], fb[f][q][1]);
                    mma16816(sh[2 * q + 1], qh[j], fb[f][q][2], fb[f][q][3]);
                }
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    mma16816(sl[2 * q], ql[j], fb[f][q][0], fb[f][q][1]);
                    mma16816(sl[2 * q + 1], ql[j], fb[f][q][2], fb[f][q][3]);
                }
            }
            float* sw = spart + warp * kMlaHeads * kSRow;
#pragma unroll
            for (int n = 0; n < kTokNt; ++n) {
                const uint32_t col = n * 8 + 2 * t;
                *reinterpret_cast<float2*>(sw + g * kSRow + col) = make_float2(sh[n][0] + sl[n][0], sh[n][1] + sl[n][1]);
                *reinterpret_cast<float2*>(sw + (g + 8) * kSRow + col) =
                    make_float2(sh[n][2] + sl[n][2], sh[n][3] + sl[n][3]);
            }
        }
        __syncthreads();  // every warp's partial scores written
        // s[i]: (head g | g+8) x (token tok0 + 2t | +1), the warps' partials summed in order
        float s[4];
        const uint32_t tbase = t0 + tile * kMlaTile + tok0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kMlaWarps; ++w) {
                const float2 v =
                    *reinterpret_cast<const float2*>(spart + (w * kMlaHeads + g + 8 * r) * kSRow + tok0 + 2 * t);
                acc.x += v.x;
                acc.y += v.y;
            }
            const uint32_t tok = tbase + 2 * t;
            s[2 * r] = tok < t1 ? acc.x : NEG_INF;
            s[2 * r + 1] = tok + 1 < t1 ? acc.y : NEG_INF;
        }
        // per-head maximum over the tile: warp's 8 tokens, then across warps
        float mx[2] = {fmaxf(s[0], s[1]), fmaxf(s[2], s[3])};
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
        {
            float lsum[2];
            uint32_t pw[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const float p0 = (m_new[r] == NEG_INF) ? 0.f : exp2f(s[2 * r] - m_new[r]);
                const float p1 = (m_new[r] == NEG_INF) ? 0.f : exp2f(s[2 * r + 1] - m_new[r]);
                pw[r] = pack_bf16x2(p0, p1);
                lsum[r] = bf16_bits_to_f32(pw[r] & 0xffffu) + bf16_bits_to_f32(pw[r] >> 16);
            }
            const uint32_t col = (tok0 + 2 * t) * 2;
            *reinterpret_cast<uint32_t*>(pbuf + g * kPRow + col) = pw[0];
            *reinterpret_cast<uint32_t*>(pbuf + (g + 8) * kPRow + col) = pw[1];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                lsum[r] += __shfl_xor_sync(kFull, lsum[r], 1);
                lsum[r] += __shfl_xor_sync(kFull, lsum[r], 2);
                l_run[r] = l_run[r] * alpha[r] + lsum[r];  // this warp's tokens only; summed over warps at the end
            }
        }
#pragma unroll
        for (int n = 0; n < kONt; ++n) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        __syncthreads();  // P complete
        // ---- O[:, 128w .. 128w+127] += P (16 x 32) C (32 x 128): four steps
        // (16 tokens x 64 columns each), fragments one step ahead
        {
            uint32_t pa[2][4], cb[2][4][4];
            auto load_pv = [&](int f, uint32_t step) {
                const uint32_t kk = step >> 1, hh = step & 1u;
                ldsm_x4(pa[f], pbuf + a_row * kPRow + (kk * 16 + a_col) * 2);
                // trans loads: rows = tokens kk*16 + (lane & 15), columns 8-wide blocks
                const unsigned char* crow = st + (kk * 16 + (lane & 15)) * kCRow;
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    ldsm_x4_t(cb[f][q], crow + (warp * kColsPerWarp + hh * 64 + q * 16 + (lane >> 4) * 8) * 2);
            };
            load_pv(0, 0);
#pragma unroll
            for (uint32_t step = 0; step < 2 * (kMlaTile / 16); ++step) {
                const int f = step & 1;
                if (step + 1 < 2 * (kMlaTile / 16)) load_pv(f ^ 1, step + 1);
                const int hh = step & 1;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int n = hh * 8 + 2 * q;
                    mma16816(o[n], pa[f], cb[f][q][0], cb[f][q][1]);
                    mma16816(o[n + 1], pa[f], cb[f][q][2], cb[f][q][3]);
                }
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
    for (int n = 0; n < kONt; ++n) {
        const uint32_t col = warp * kColsPerWarp + n * 8 + 2 * t;
        *reinterpret_cast<float2*>(out + g * kMlaPartialFloats + 2 + col) = make_float2(o[n][0], o[n][1]);
        *reinterpret_cast<float2*>(out + (g + 8) * kMlaPartialFloats + 2 + col) = make_float2(o[n][2], o[n][3]);
    }
}

// ---------------------------------------------------------------- 3. merge + output
// grid (heads, batch), 256 threads, one CTA per SM. W_UV[h] (128 KB) is copied
// into shared memory by cp.async before the dependency wait. The splits of
// (sequence b, head h) are merged as
// ctx[c] = sum_s 2^(m_s - M) O_s[c] / sum_s 2^(m_s - M) l_s into shared memory:
// thread c holds columns c and c + 256 of up to kOutChunk splits, loaded
// together with the split maxima and sums (one L2 round trip up to kOutChunk
// splits). Then warp w computes out rows d = w, w + 8, ... of W_UV[h] ctx, a
// lane covering latent columns 8 lane .. +7 and 256 + 8 lane .. +7.
constexpr uint32_t kOutThreads = 256;
constexpr uint32_t kOutMaxSplits = 1024;
constexpr uint32_t kOutChunk = 48;  // splits whose partials a thread holds in registers at once
constexpr size_t kOutSmem = size_t(kMlaV) * kMlaLatent * 2;  // W_UV[h]
template <typename OT>
__global__ void __launch_bounds__(kOutThreads, 1) mla_merge_out_kernel(const float* __restrict__ partial,
                                                                        uint32_t splits,
                                                                        const uint16_t* __restrict__ w_uv,
                                                                        OT* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char wuv_s[];  // [128 rows][512] bf16
    __shared__ float wsc[kOutMaxSplits];
    __shared__ float lsc[kOutMaxSplits];
    __shared__ __align__(16) float cs[kMlaLatent];
    __shared__ float red[kOutThreads / 32];
    const uint32_t h = blockIdx.x, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // W_UV[h] does not depend on the earlier kernels
    {
        const unsigned char* src = reinterpret_cast<const unsigned char*>(w_uv + static_cast<size_t>(h) * kMlaV * kMlaLatent);
#pragma unroll 4
        for (uint32_t i = threadIdx.x; i < kOutSmem / 16; i += kOutThreads) cp16(wuv_s + i * 16, src + i * 16);
        cp_commit();
    }
    pdl_wait();
    pdl_launch_dependents();
    const float* base = partial + static_cast<size_t>(b) * splits * kMlaHeads * kMlaPartialFloats +
                        h * kMlaPartialFloats;
    const size_t stride = static_cast<size_t>(kMlaHeads) * kMlaPartialFloats;
    const float NEG_INF = -__int_as_float(0x7f800000);
    // the first chunk of this thread's context partials (columns c and c + 256)
    const float* oc = base + 2 + threadIdx.x;
    float v[2][kOutChunk];
#pragma unroll
    for (uint32_t j = 0; j < kOutChunk; ++j) {
        v[0][j] = j < splits ? __ldcg(oc + j * stride) : 0.f;
        v[1][j] = j < splits ? __ldcg(oc + kOutThreads + j * stride) : 0.f;
    }
    float M = NEG_INF;
    for (uint32_t sp = threadIdx.x; sp < splits; sp += blockDim.x) {
        const float m = __ldcg(base + sp * stride), l = __ldcg(base + sp * stride + 1);
        wsc[sp] = m;
        lsc[sp] = l;
        M = fmaxf(M, m);
    }
    M = warp_max(M);
    if (lane == 0) red[warp] = M;
    __syncthreads();
    M = red[0];
#pragma unroll
    for (int w = 1; w < kOutThreads / 32; ++w) M = fmaxf(M, red[w]);
    float tot = 0.f;
    for (uint32_t sp = threadIdx.x; sp < splits; sp += blockDim.x) {
        const float m = wsc[sp];
        const float w = (m == NEG_INF) ? 0.f : exp2f(m - M);
        wsc[sp] = w;
        tot += w * lsc[sp];
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
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (uint32_t sp0 = 0; sp0 < splits; sp0 += kOutChunk) {
        if (sp0 > 0) {
#pragma unroll
            for (uint32_t j = 0; j < kOutChunk; ++j) {
                v[0][j] = sp0 + j < splits ? __ldcg(oc + (sp0 + j) * stride) : 0.f;
                v[1][j] = sp0 + j < splits ? __ldcg(oc + kOutThreads + (sp0 + j) * stride) : 0.f;
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < kOutChunk; ++j) {
            const float w = sp0 + j < splits ? wsc[sp0 + j] : 0.f;
            acc[0][j & 3] = fmaf(w, v[0][j], acc[0][j & 3]);
            acc[1][j & 3] = fmaf(w, v[1][j], acc[1][j & 3]);
        }
    }
    cs[threadIdx.x] = ((acc[0][0] + acc[0][1]) + (acc[0][2] + acc[0][3])) * inv;
    cs[threadIdx.x + kOutThreads] = ((acc[1][0] + acc[1][1]) + (acc[1][2] + acc[1][3])) * inv;
    cp_wait<0>();
    __syncthreads();  // ctx and W_UV[h] in shared memory
    // out rows: warp w takes d = w + 8 i; lane covers latent columns 8 lane .. +7
    // and 256 + 8 lane .. +7 (16-byte shared reads, conflict-free)
    float cv[16];
    {
        const float4* c0 = reinterpret_cast<const float4*>(cs + lane * 8);
        const float4* c1 = reinterpret_cast<const float4*>(cs + kOutThreads + lane * 8);
        const float4 a0 = c0[0], a1 = c0[1], b0 = c1[0], b1 = c1[1];
        cv[0] = a0.x, cv[1] = a0.y, cv[2] = a0.z, cv[3] = a0.w, cv[4] = a1.x, cv[5] = a1.y, cv[6] = a1.z, cv[7] = a1.w;
        cv[8] = b0.x, cv[9] = b0.y, cv[10] = b0.z, cv[11] = b0.w, cv[12] = b1.x, cv[13] = b1.y, cv[14] = b1.z,
        cv[15] = b1.w;
    }
    constexpr uint32_t kRowsPerWarp = kMlaV / (kOutThreads / 32);  // 16
#pragma unroll
    for (uint32_t i = 0; i < kRowsPerWarp; ++i) {
        const uint32_t d = warp + i * (kOutThreads / 32);
        const uint16_t* wr = reinterpret_cast<const uint16_t*>(wuv_s) + static_cast<size_t>(d) * kMlaLatent;
        const uint4 w0 = *reinterpret_cast<const uint4*>(wr + lane * 8);
        const uint4 w1 = *reinterpret_cast<const uint4*>(wr + kOutThreads + lane * 8);
        const uint32_t wq[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float a = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            a = fmaf(bf16_bits_to_f32(wq[q] & 0xffffu), cv[2 * q], a);
            a = fmaf(bf16_bits_to_f32(wq[q] >> 16), cv[2 * q + 1], a);
        }
        a = warp_sum(a);
        if (lane == 0) store_act(out, (static_cast<size_t>(b) * kMlaHeads + h) * kMlaV + d, a);
    }
}

// ---------------------------------------------------------------- launch
size_t mla_smem_bytes() { return kMlaSmem; }

bool mla_shape_supported(uint32_t heads, uint32_t rope, uint32_t latent, uint32_t v_dim) {
    return heads == kMlaHeads && rope == kMlaRope && latent == kMlaLatent && v_dim == kMlaV;
}

// Splits of the longest cache such that batch x splits CTAs fill at most one
// wave (kMlaCtasPerSm attention CTAs per SM from batch 4 up; below that one
// per SM, since the merge reads every split's partial serially), each split
// at least two tiles; a split need not be a whole number of tiles (the last
// tile of a split is masked).
void mla_plan_splits(const MlaLaunch& a, int num_sms, uint32_t& split_tokens, uint32_t& splits) {
    uint32_t lmax = 1;
    for (uint32_t b = 0; b < a.batch; ++b) lmax = a.seqs.len[b] > lmax ? a.seqs.len[b] : lmax;
    const uint32_t per_sm = a.batch >= 4 ? kMlaCtasPerSm : 1u;
    uint32_t want = per_sm * static_cast<uint32_t>(num_sms) / (a.batch ? a.batch : 1);
    if (want < 1) want = 1;
    uint32_t st = (lmax + want - 1) / want;
    if (st < 2 * kMlaTile) st = 2 * kMlaTile;
    split_tokens = st;
    splits = (lmax + st - 1) / st;
}

uint32_t mla_max_splits(uint32_t max_batch, int num_sms) {
    return kMlaCtasPerSm * static_cast<uint32_t>(num_sms) / (max_batch ? max_batch : 1) + 1;
}

cudaError_t mla_decode_launch(const MlaLaunch& a, cudaStream_t s) {
    const float k = a.scale * 1.4426950408889634f;  // scores in base 2
    cudaError_t e;
    {
        const RopeAppendArgs ra = a.rope ? *a.rope : RopeAppendArgs{};
        if (a.rope) {  // f32 query (host-checked); append CTAs: ceil(batch / 16) more grid rows
            const dim3 grid(kMlaHeads, kMlaLatent / 64 + (a.batch + kMlaHeads - 1) / kMlaHeads);
            e = launch_pdl_kernel(mla_absorb_kernel<float, true>, grid, dim3(256), 0, s, static_cast<const float*>(a.q),
                                  a.batch, a.nope, a.w_uk, k, a.qp, ra);
        } else if (a.q_dtype == PBMOE_F32) {
            e = launch_pdl_kernel(mla_absorb_kernel<float>, dim3(kMlaHeads, kMlaLatent / 64), dim3(256), 0, s,
                                  static_cast<const float*>(a.q), a.batch, a.nope, a.w_uk, k, a.qp, ra);
        } else {
            e = launch_pdl_kernel(mla_absorb_kernel<uint16_t>, dim3(kMlaHeads, kMlaLatent / 64), dim3(256), 0, s,
                                  static_cast<const uint16_t*>(a.q), a.batch, a.nope, a.w_uk, k, a.qp, ra);
        }
        if (e != cudaSuccess) return e;
    }
    if ((e = cudaFuncSetAttribute(mla_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kMlaSmem))) != cudaSuccess)
        return e;
    const uint32_t* fresh = a.rope ? a.rope->positions : nullptr;
    if ((e = launch_pdl_kernel(mla_attn_kernel, dim3(a.splits, a.batch), dim3(kMlaThreads), kMlaSmem, s, a.qp,
                               a.seqs, a.split_tokens, a.splits, a.partial, fresh)) != cudaSuccess)
        return e;
    if (a.splits > kOutMaxSplits) return cudaErrorInvalidValue;
    const dim3 og(kMlaHeads, a.batch);
    if ((e = cudaFuncSetAttribute(mla_merge_out_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kOutSmem))) != cudaSuccess ||
        (e = cudaFuncSetAttribute(mla_merge_out_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(kOutSmem))) != cudaSuccess)
        return e;
    if (a.out_dtype == PBMOE_F32)
        return launch_pdl_kernel(mla_merge_out_kernel<float>, og, dim3(kOutThreads), kOutSmem, s, a.partial, a.splits, a.w_uv,
                                 static_cast<float*>(a.out));
    return launch_pdl_kernel(mla_merge_out_kernel<uint16_t>, og, dim3(kOutThreads), kOutSmem, s, a.partial, a.splits, a.w_uv,
                             static_cast<uint16_t*>(a.out));
}

}  // namespace pbmoe
