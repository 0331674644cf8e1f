// q4_gemm.cu — prefill Q4 GEMM on the 5th-generation tensor cores:
// Y[m, n] = sum_k X[m, k] * (q[n, k] * s[n, g(k)] + b[n, g(k)]) for a dense
// weight (config 2: X [2048 x 2048], W Q4 [5120 x 2048]) and, grouped, for
// per-expert weights with the routes bucketed by expert slot.
//
// Reference: the layer-major prefill path (qwen_layer_major_group_plan,
// metal/mod.rs:3197-3233; qwen_layer_major_gather, shaders.metal:1743-1754;
// q4_mmap_fma_matvec_batch_bf16_scale_bias, shaders.metal:973-1057), which
// re-streams every weight row for each pair of input rows with no matrix
// units.
//
// A persistent CTA per SM walks a static list of output tiles of 128 weight
// rows (the UMMA M dimension: one TMEM lane per row) x up to BN tokens (N), K
// advancing two 64-wide quantisation groups per step. Fourteen warps, each
// role on its own ring of buffers and mbarriers:
//
//   warp 0      loader (one thread): TMA loads of each step's nibbles (128
//               rows x 64 B, 64-byte swizzle) into a W ring, of the step's
//               fp16 token rows (two boxes of 64 k x BN rows, 128-byte
//               swizzle, the UMMA K-major layout) into a B ring, and bulk
//               copies of each tile's
//               scales and biases; all complete as transaction bytes on the
//               ring's mbarrier, so the loader never waits on its own copies.
//   warp 1      TMEM owner; lane 0 issues eight tcgen05.mma (K = 16 each, A
//               from TMEM, B from shared memory) per step when afull and bfull
//               complete, commits them to aempty / bempty and per tile to tfull.
//   warps 2-9   dequant, two warps per 32-row TMEM lane quarter, one per
//               group of the step: each thread takes its row's 64 weights of
//               that group, w = q*s + b to fp16 (one rounding), 32 packed
//               columns written straight into the step's A slot in TMEM
//               (tcgen05.st); lane 0 arrives on afull for the warp (mbarrier
//               arrivals are one per warp throughout). A never touches shared
//               memory, so no proxy fence is needed between the dequant and
//               the MMA.
//   warps 10-13 epilogue: tcgen05.ld of the finished accumulator (double-
//               buffered in TMEM, so tile t+1's MMAs overlap tile t's stores),
//               stores, arrive on tempty.
//
// Operands are fp16. bf16 weights would carry 2^-9 relative rounding per
// weight (up to ~0.9% max-relative error against the f32 reference on
// config-2 shapes); fp16 keeps 11 bits. bf16 activations convert to fp16
// exactly (x16_gather_kernel, which also gathers the grouped rows into
// grouped order); a magnitude >= 65536 or a non-finite value has no fp16
// image and latches PBMOE_DEV_ERR_F16_RANGE.
//
// Nibble unpack: byte t of a packed word holds k = 2t (low nibble) and
// 2t+1 (high nibble). prmt copies the byte into both halves, one lop3 keeps
// the low nibble in the low half and the high nibble (bits 4-7) in the high
// half and ORs in 1024.0 (low) / 64.0 (high): at those exponents the kept
// bits are worth exactly q, so one sub.f16x2 yields (q_2t, q_2t+1) exactly.
//
// Every wait is bounded: one that expires latches PBMOE_DEV_ERR_PIPE_TIMEOUT
// and raises a CTA-wide abort flag on which all roles stop; the MMA thread
// drains its issued MMAs and the loader its copies before TMEM is released.

#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "kernels.h"
#include "pipe.cuh"
#include "umma.cuh"

namespace pbmoe {

constexpr int kUmThreads = 448;  // loader, MMA, 8 dequant, 4 epilogue warps
constexpr uint32_t kDequantWarps = 8;
constexpr uint32_t kEpilogueWarps = 4;
constexpr uint32_t kUmRows = 128;
constexpr uint32_t kMagicPair = 0x54006400u;  // f16x2 (lo 1024.0, hi 64.0)
constexpr uint32_t kNoSlot = 0xffffffffu;

template <int BN_, int SB_, int SW_, bool kGathered_>
struct UmmaCfg {
    static constexpr int BN = BN_, SA = 3, SB = SB_, SW = SW_;
    static constexpr bool kGathered = kGathered_;
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 128, "UMMA N per accumulator");
    static constexpr uint32_t kBox = BN * 128;    // fp16 [BN tokens][64 k], 128B-swizzled (multiple of 1024)
    static constexpr uint32_t kB = 2 * kBox;      // one step: two k-boxes
    static constexpr uint32_t kW = kUmRows * 64;  // nibbles [128 rows][64 B] (two groups), 64B-swizzled
    static constexpr uint32_t kACols = 64;        // one step of A: 128 k as packed fp16 pairs
    static constexpr uint32_t kAccCols = 2 * BN;  // two accumulators, then SA A slots
    static constexpr uint32_t kTmemCols =
        (kAccCols + SA * kACols) <= 256 ? 256 : 512;
    static constexpr size_t sbuf_bytes(uint32_t groups) { return size_t(kUmRows) * groups * 4; }  // scales + biases
    static constexpr size_t smem(uint32_t groups, uint32_t table) {
        return 1024 + size_t(SB) * kB + size_t(SW) * kW + 2 * sbuf_bytes(groups) + size_t(table) * 4;
    }
};
using DenseCfg = UmmaCfg<128, 4, 6, false>;
using GroupedCfg = UmmaCfg<64, 6, 8, true>;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also stops when another role of the CTA has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                              uint32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait_hint(bar, parity, 20000u)) {
        if (*abort_flag) return false;
        if (global_ns() - t0 > kPipeWaitNs) {
            *abort_flag = 1u;
            if (status) atomicOr(status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Bounded wait for roles off the critical path (epilogue, loader): polls with
// a short sleep in between, so the waiting warp does not take issue slots
// from the dequant warp on its scheduler.
__device__ __forceinline__ bool wait_or_abort_lazy(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                   uint32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        __nanosleep(256);
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kPipeWaitNs) {
            *abort_flag = 1u;
            if (status) atomicOr(status, PBMOE_DEV_ERR_PIPE_TIMEOUT);
            return false;
        }
    }
}

// A wait decided by lane 0 and broadcast, so the warp stays converged for the
// warp-collective operations that follow.
template <bool kLazy>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                          uint32_t* status) {
    bool ok = false;
    if ((threadIdx.x & 31) == 0)
        ok = kLazy ? wait_or_abort_lazy(bar, parity, abort_flag, status) : wait_or_abort(bar, parity, abort_flag, status);
    return __shfl_sync(kFull, ok ? 1u : 0u, 0) != 0u;
}

// bf16 bits -> fp16 bits (round to nearest)
__device__ __forceinline__ uint32_t f16_of_bf16(uint32_t v16) {
    return __half_as_ushort(__float2half_rn(__uint_as_float(v16 << 16)));
}

// Four packed fp16 pairs (k = 8j .. 8j+7 in order) from packed word w of one row.
__device__ __forceinline__ void dequant_word_f16(uint32_t w, uint32_t s2, uint32_t b2, uint32_t* o) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t X = __byte_perm(w, 0u, 0x4040u + 0x0101u * t);  // (byte t, 0, byte t, 0)
        uint32_t m, q;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(m) : "r"(X), "r"(0x00F0000Fu), "r"(kMagicPair));  // (a & b) | c
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(m), "r"(kMagicPair));
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[t]) : "r"(q), "r"(s2), "r"(b2));
    }
}

// Kernel arguments. Dense: scales / biases of one matrix, the nibbles through
// the W tensor map (a single "expert"). Grouped: the expert table and the
// component offsets of one projection in a slot.
struct UmmaParams {
    const uint16_t* scales;
    const uint16_t* biases;
    const uint8_t* experts;
    uint64_t expert_bytes;
    uint64_t scales_offset, biases_offset;
    uint32_t N, K;  // per-matrix rows x cols
    uint32_t num_experts;
    uint32_t M;  // dense: token rows
    // grouped
    const uint32_t* slot_experts;
    const uint32_t* unique_count;
    uint32_t max_unique;
    const uint32_t* groups;
    uint32_t routes;
    uint32_t table_cap;  // grouped tile table capacity (entries)
    void* y;
    uint32_t* status;
};

// One output tile as every role sees it.
struct TileInfo {
    const uint16_t* scales;  // this tile's matrix
    const uint16_t* biases;
    uint32_t expert;  // W tensor-map coordinate
    uint32_t n0, rows_here;
    uint32_t ntok;   // 0: skip
    uint32_t first;  // first token row in the fp16 B matrix and the output
};

template <class Cfg>
__device__ __forceinline__ TileInfo tile_info(const UmmaParams& p, uint32_t t, uint32_t row_tiles,
                                              const uint32_t* table) {
    TileInfo ti;
    const uint32_t rt = t % row_tiles, jt = t / row_tiles;
    ti.n0 = rt * kUmRows;
    ti.rows_here = min(p.N - ti.n0, kUmRows);
    if constexpr (!Cfg::kGathered) {
        ti.scales = p.scales;
        ti.biases = p.biases;
        ti.expert = 0;
        ti.first = jt * Cfg::BN;
        ti.ntok = min(p.M - ti.first, static_cast<uint32_t>(Cfg::BN));
    } else {
        const uint32_t e = table[jt];  // (slot << 8) | token-tile, or kNoSlot
        ti.scales = ti.biases = nullptr;
        ti.expert = 0;
        if (e == kNoSlot) {
            ti.first = 0;
            ti.ntok = 0;
        } else {
            const uint32_t slot = e >> 8, tok0 = (e & 0xffu) * Cfg::BN;
            const uint32_t start = p.groups[2 * slot], cnt = p.groups[2 * slot + 1];
            ti.first = start + tok0;
            ti.ntok = min(cnt - tok0, static_cast<uint32_t>(Cfg::BN));
            ti.expert = p.slot_experts[slot];
            const uint8_t* base = p.experts + static_cast<size_t>(ti.expert) * p.expert_bytes;
            ti.scales = reinterpret_cast<const uint16_t*>(base + p.scales_offset);
            ti.biases = reinterpret_cast<const uint16_t*>(base + p.biases_offset);
        }
    }
    return ti;
}

template <class Cfg, typename YT>
__global__ void __launch_bounds__(kUmThreads, 1)
    q4_umma_kernel(const UmmaParams p, const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w) {
    constexpr int BN = Cfg::BN, SA = Cfg::SA, SB = Cfg::SB, SW = Cfg::SW;
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t wfull[SW], wfree[SW], sfull[2], sfree[2], afull[SA], aempty[SA], bfull[SB],
        bempty[SB], tfull[2], tempty[2], drain;
    __shared__ uint32_t tmem_base_sh, abort_sh, num_tiles_sh, warp_tot[kUmThreads / 32];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t G = p.K / 64;       // quantisation groups per row
    const uint32_t steps = G / 2;      // K steps of two groups
    unsigned char* bring = smem;                  // SB x B tiles
    unsigned char* wring = bring + SB * Cfg::kB;  // SW x [128][32] nibbles
    unsigned char* sbufs = wring + SW * Cfg::kW;  // 2 x [scales 128 x G | biases 128 x G] bf16
    uint32_t* table = reinterpret_cast<uint32_t*>(sbufs + 2 * Cfg::sbuf_bytes(G));
    volatile uint32_t* abort_flag = &abort_sh;
    uint32_t* status = p.status;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t row_tiles = (p.N + kUmRows - 1) / kUmRows;

    if (tid == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&wfree[i], kDequantWarps);  // one arrival per warp (lane 0 after __syncwarp)
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sfree[i], kDequantWarps);
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpilogueWarps);
        }
        for (int i = 0; i < SA; ++i) {
            mbar_init(&afull[i], kDequantWarps);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < SB; ++i) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        mbar_init(&drain, 1);
        abort_sh = 0;
        fence_mbar_init();
    }
    // tile list
    if constexpr (!Cfg::kGathered) {
        if (tid == 0) num_tiles_sh = row_tiles * ((p.M + BN - 1) / BN);
    } else {
        // token tiles over the groups in slot order: entry = (slot << 8) | k
        // for the k-th BN-route run of the slot
        const uint32_t unique = min(*p.unique_count, p.max_unique);
        uint32_t base = 0;
        for (uint32_t c0 = 0; c0 < unique; c0 += kUmThreads) {
            const uint32_t slot = c0 + tid;
            uint32_t tiles = 0;
            if (slot < unique) {
                const uint32_t start = p.groups[2 * slot], cnt = p.groups[2 * slot + 1];
                const uint32_t ex = p.slot_experts[slot];
                const bool valid = ex < p.num_experts && start + cnt <= p.routes && cnt <= 256u * BN;
                if (!valid && status) atomicOr(status, PBMOE_DEV_ERR_EXPERT_ID);
                tiles = valid ? (cnt + BN - 1) / BN : 0u;
            }
            uint32_t incl = tiles;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(kFull, incl, o);
                if (lane >= o) incl += v;
            }
            __syncthreads();
            if (lane == 31) warp_tot[warp] = incl;
            __syncthreads();
            uint32_t before = base, total = 0;
#pragma unroll
            for (int w = 0; w < kUmThreads / 32; ++w) {
                if (w < warp) before += warp_tot[w];
                total += warp_tot[w];
            }
            const uint32_t lo = before + incl - tiles;
            for (uint32_t k = 0; k < tiles; ++k)
                if (lo + k < p.table_cap) table[lo + k] = (slot << 8) | k;
            base += total;
        }
        if (tid == 0) num_tiles_sh = row_tiles * min(base, p.table_cap);
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_sh, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t num_tiles = num_tiles_sh;

    if (warp == 0) {
        // ------------------------------------------------------------ loader (lane 0)
        if (lane == 0) {
            uint32_t gs = 0, lt = 0;  // global step, local tile
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
                const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
                if (ti.ntok == 0) continue;
                const int sb = static_cast<int>(lt & 1);
                if (lt >= 2 && !wait_or_abort_lazy(&sfree[sb], ((lt >> 1) - 1) & 1, abort_flag, status)) {
                    ok = false;
                    break;
                }
                {  // the tile rows' scales and biases (contiguous: rows x G each)
                    unsigned char* sdst = sbufs + sb * Cfg::sbuf_bytes(G);
                    const uint32_t bytes = ti.rows_here * G * 2;
                    mbar_arrive_expect_tx(&sfull[sb], 2 * bytes);
                    bulk_load(sdst, ti.scales + static_cast<size_t>(ti.n0) * G, bytes, &sfull[sb]);
                    bulk_load(sdst + kUmRows * G * 2, ti.biases + static_cast<size_t>(ti.n0) * G, bytes, &sfull[sb]);
                }
                for (uint32_t i = 0; i < steps; ++i, ++gs) {
                    const int w = static_cast<int>(gs % SW), s = static_cast<int>(gs % SB);
                    if (gs >= static_cast<uint32_t>(SW) &&
                        !wait_or_abort_lazy(&wfree[w], ((gs / SW) - 1) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&wfull[w], Cfg::kW);
                    tma_load_3d(wring + w * Cfg::kW, &tm_w, static_cast<int32_t>(i * 64), static_cast<int32_t>(ti.n0),
                                static_cast<int32_t>(ti.expert), &wfull[w]);
                    if (gs >= static_cast<uint32_t>(SB) &&
                        !wait_or_abort_lazy(&bempty[s], ((gs / SB) - 1) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&bfull[s], Cfg::kB);
                    unsigned char* bdst = bring + s * Cfg::kB;
                    tma_load_2d(bdst, &tm_x, static_cast<int32_t>(i * 128), static_cast<int32_t>(ti.first), &bfull[s]);
                    tma_load_2d(bdst + Cfg::kBox, &tm_x, static_cast<int32_t>(i * 128 + 64),
                                static_cast<int32_t>(ti.first), &bfull[s]);
                }
                ++lt;
            }
            if (!ok) {
                // aborted: give the loads in flight time to land before the
                // CTA exits (each completes on its own; nothing waits on them)
                const uint64_t t0 = global_ns();
                while (global_ns() - t0 < 100000ull) __nanosleep(1000);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issue
        if (lane == 0) {
            uint32_t gs = 0, lt = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
                const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
                if (ti.ntok == 0) continue;
                const int acc = static_cast<int>(lt & 1);
                if (lt >= 2 && !wait_or_abort_lazy(&tempty[acc], ((lt >> 1) - 1) & 1, abort_flag, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t idesc = idesc_f16_f32(kUmRows, (ti.ntok + 15u) & ~15u);
                const uint32_t d = tmem + acc * BN;
                for (uint32_t i = 0; i < steps; ++i, ++gs) {
                    const int sa = static_cast<int>(gs % SA), s = static_cast<int>(gs % SB);
                    if (!wait_or_abort(&afull[sa], (gs / SA) & 1, abort_flag, status) ||
                        !wait_or_abort(&bfull[s], (gs / SB) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = tmem + Cfg::kAccCols + sa * Cfg::kACols, b0 = smem_u32(bring + s * Cfg::kB);
#pragma unroll
                    for (uint32_t kk = 0; kk < 8; ++kk)
                        umma_f16_ts(d, a + kk * 8, sw128_kmajor_desc(b0 + (kk >> 2) * Cfg::kBox + (kk & 3) * 32),
                                    idesc, (i | kk) != 0u);
                    umma_commit(&aempty[sa]);
                    umma_commit(&bempty[s]);
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                ++lt;
            }
            if (!ok) {
                // aborted: wait (bounded) for the MMAs in flight before TMEM is released
                umma_commit(&drain);
                const uint64_t t0 = global_ns();
                while (!mbar_try_wait_hint(&drain, 0, 20000u) && global_ns() - t0 < kPipeWaitNs) {
                }
            }
        }
        __syncwarp();
    } else if (warp < 10) {
        // ------------------------------------------------------------ dequant into TMEM
        const uint32_t q = warp & 3, r = 32u * q + lane;  // weight row = TMEM lane
        const uint32_t h = static_cast<uint32_t>(warp - 2) >> 2;  // group of the step (0, 1)
        // 64-byte swizzle of the nibble rows: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)
        const uint32_t wc0 = ((2 * h) ^ ((r >> 1) & 3)) << 4, wc1 = ((2 * h + 1) ^ ((r >> 1) & 3)) << 4;
        const uint32_t a_lane = tmem + ((32u * q) << 16) + Cfg::kAccCols + 32 * h;
        uint32_t gs = 0, lt = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
            if (ti.ntok == 0) continue;
            const int sbuf = static_cast<int>(lt & 1);
            if (!warp_wait<false>(&sfull[sbuf], (lt >> 1) & 1, abort_flag, status)) {
                ok = false;
                break;
            }
            // rows beyond the matrix (ragged N) dequantise with scale and bias 0
            const bool rok = r < ti.rows_here;
            const uint16_t* srow = reinterpret_cast<const uint16_t*>(sbufs + sbuf * Cfg::sbuf_bytes(G)) + r * G;
            const uint16_t* brow = srow + kUmRows * G;
            uint4 sq = make_uint4(0, 0, 0, 0), bq = sq;
            for (uint32_t i = 0; i < steps; ++i, ++gs) {
                if ((i & 3) == 0 && rok) {  // groups 2i .. 2i+7
                    sq = *reinterpret_cast<const uint4*>(srow + 2 * i);
                    bq = *reinterpret_cast<const uint4*>(brow + 2 * i);
                }
                const int w = static_cast<int>(gs % SW), sa = static_cast<int>(gs % SA);
                if (!warp_wait<false>(&wfull[w], (gs / SW) & 1, abort_flag, status) ||
                    (gs >= static_cast<uint32_t>(SA) &&
                     !warp_wait<false>(&aempty[sa], ((gs / SA) - 1) & 1, abort_flag, status))) {
                    ok = false;
                    break;
                }
                // group 2i + h: half h of word i & 3 of the eight cached groups
                const uint32_t sw = (i & 2) ? ((i & 1) ? sq.w : sq.z) : ((i & 1) ? sq.y : sq.x);
                const uint32_t bw = (i & 2) ? ((i & 1) ? bq.w : bq.z) : ((i & 1) ? bq.y : bq.x);
                const uint32_t s16 = f16_of_bf16(h ? (sw >> 16) : (sw & 0xffffu));
                const uint32_t b16 = f16_of_bf16(h ? (bw >> 16) : (bw & 0xffffu));
                const uint32_t s2 = s16 * 0x10001u, b2 = b16 * 0x10001u;
                const unsigned char* wr = wring + w * Cfg::kW + r * 64;
                const uint4 w0 = *reinterpret_cast<const uint4*>(wr + wc0);
                const uint4 w1 = *reinterpret_cast<const uint4*>(wr + wc1);
                __syncwarp();
                if (lane == 0) mbar_arrive(&wfree[w]);  // the warp's nibbles are in registers
                const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                uint32_t v[32];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) dequant_word_f16(words[jj], s2, b2, v + 4 * jj);
                tc_fence_after();  // after the aempty wait: the MMA reading this slot is done
                tmem_st32_wait(a_lane + sa * Cfg::kACols, v);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[sa]);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&sfree[sbuf]);
            ++lt;
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const uint32_t q = warp & 3, r = 32u * q + lane;
        YT* y = static_cast<YT*>(p.y);
        uint32_t lt = 0;
        for (uint32_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
            if (ti.ntok == 0) continue;
            const int acc = static_cast<int>(lt & 1);
            if (!warp_wait<true>(&tfull[acc], (lt >> 1) & 1, abort_flag, status)) break;
            tc_fence_after();
            const uint32_t taddr = tmem + (acc * BN) + ((32u * q) << 16);
            const bool rok = r < ti.rows_here;
            const uint32_t nmma = (ti.ntok + 15u) & ~15u;
            for (uint32_t c0 = 0; c0 < nmma; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(taddr + c0, v);
                if (rok) {
#pragma unroll
                    for (uint32_t j = 0; j < 32; ++j)
                        if (c0 + j < ti.ntok)
                            store_act(y + static_cast<size_t>(ti.first + c0 + j) * p.N + ti.n0, r,
                                      __uint_as_float(v[j]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            ++lt;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// fp16 rows for the tensor cores: out[j] = x[rows ? rows[j] : j] (bf16 or fp16
// in, K elements per row), eight values per thread step. A source row >= x_rows
// latches PBMOE_DEV_ERR_EXPERT_ID (written as zeros); a bf16 value of magnitude
// >= 65536 or non-finite latches PBMOE_DEV_ERR_F16_RANGE.
__global__ void __launch_bounds__(256) x16_gather_kernel(const uint4* __restrict__ x, int x_is_f16,
                                                         const uint32_t* __restrict__ rows, uint32_t nrows,
                                                         uint32_t x_rows, uint32_t K, uint4* __restrict__ out,
                                                         uint32_t* status) {
    const uint32_t per_row = K / 8;
    const size_t n8 = size_t(nrows) * per_row;
    uint32_t mx = 0;
    bool bad = false;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n8; i += size_t(gridDim.x) * blockDim.x) {
        const uint32_t j = static_cast<uint32_t>(i / per_row), c = static_cast<uint32_t>(i % per_row);
        const uint32_t src = rows ? __ldg(rows + j) : j;
        if (src >= x_rows) {
            bad = true;
            out[i] = make_uint4(0, 0, 0, 0);
            continue;
        }
        const uint4 v = __ldg(x + size_t(src) * per_row + c);
        if (x_is_f16) {
            out[i] = v;
            continue;
        }
        mx = __vmaxu2(mx, __vmaxu2(__vmaxu2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu),
                                   __vmaxu2(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu)));
        uint32_t o[4];
        const uint32_t in[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            asm("cvt.rn.f16x2.f32 %0, %1, %2;"
                : "=r"(o[k])
                : "f"(__uint_as_float(in[k] & 0xffff0000u)), "f"(__uint_as_float(in[k] << 16)));
        out[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (status) {
        if ((mx & 0xffffu) >= 0x4780u || (mx >> 16) >= 0x4780u) atomicOr(status, PBMOE_DEV_ERR_F16_RANGE);
        if (bad) atomicOr(status, PBMOE_DEV_ERR_EXPERT_ID);
    }
}

// ---------------------------------------------------------------- host side
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// fp16 token matrix [rows x K], box 64 k x box_rows rows, 128-byte swizzle.
cudaError_t make_x_map(CUtensorMap* m, const void* x16, uint32_t rows, uint32_t K, uint32_t box_rows) {
    EncodeTiledFn f = encode_fn();
    if (!f) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x16), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? cudaSuccess
               : cudaErrorInvalidValue;
}

// Nibble matrices [experts][N rows][K/2 bytes] (experts `stride` bytes apart),
// box 64 bytes (two groups) x 128 rows x 1, 64-byte swizzle.
cudaError_t make_w_map(CUtensorMap* m, const void* packed, uint32_t N, uint32_t K, uint32_t experts,
                       uint64_t stride) {
    EncodeTiledFn f = encode_fn();
    if (!f) return cudaErrorNotSupported;
    const cuuint64_t dims[3] = {K / 2, N, experts};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K / 2), experts > 1 ? stride : uint64_t(K / 2) * N};
    const cuuint32_t box[3] = {64, kUmRows, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return f(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(packed), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? cudaSuccess
               : cudaErrorInvalidValue;
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0, v = 0;
        n = (cudaGetDevice(&dev) == cudaSuccess &&
             cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
                ? v
                : 148;
    }
    return n;
}

template <class Cfg, typename YT>
cudaError_t launch_umma(const UmmaParams& p, const CUtensorMap& tx, const CUtensorMap& tw, uint32_t tiles,
                        size_t smem, cudaStream_t s) {
    auto k = q4_umma_kernel<Cfg, YT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const uint32_t grid = std::max<uint32_t>(1u, std::min<uint32_t>(tiles, static_cast<uint32_t>(num_sms())));
    k<<<grid, kUmThreads, smem, s>>>(p, tx, tw);
    return cudaGetLastError();
}

}  // namespace

bool q4_gemm_supported(uint32_t N, uint32_t K, uint32_t group) {
    return group == 64 && K % 512 == 0 && N > 0 && DenseCfg::smem(K / 64, 0) <= 227 * 1024;
}

uint32_t q4_grouped_tile_bound(uint32_t routes, uint32_t max_unique) {
    // sum over slots of ceil(count / BN) <= routes / BN + slots
    return (routes + GroupedCfg::BN - 1) / GroupedCfg::BN + max_unique;
}

bool q4_grouped_supported(uint32_t N, uint32_t K, uint32_t group, uint32_t routes, uint32_t max_unique) {
    return q4_gemm_supported(N, K, group) &&
           GroupedCfg::smem(K / 64, q4_grouped_tile_bound(routes, max_unique)) <= 227 * 1024;
}

cudaError_t x16_gather_launch(const void* x, bool x_is_f16, const uint32_t* rows, uint32_t nrows, uint32_t x_rows,
                              uint32_t K, void* out, uint32_t* status, cudaStream_t s) {
    const size_t n8 = size_t(nrows) * (K / 8);
    if (n8 == 0) return cudaSuccess;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((n8 + 255) / 256, 148 * 8));
    x16_gather_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(x), x_is_f16 ? 1 : 0, rows, nrows, x_rows, K,
                                           static_cast<uint4*>(out), status);
    return cudaGetLastError();
}

cudaError_t q4_gemm_launch(const Q4GemmArgs& a, cudaStream_t s) {
    UmmaParams p{};
    p.scales = a.scales;
    p.biases = a.biases;
    p.N = a.rows;
    p.K = a.cols;
    p.num_experts = 1;
    p.M = a.m;
    p.y = a.y;
    p.status = a.status;
    CUtensorMap tx, tw;
    cudaError_t e;
    if ((e = make_x_map(&tx, a.x16, a.m, a.cols, DenseCfg::BN)) != cudaSuccess) return e;
    if ((e = make_w_map(&tw, a.packed, a.rows, a.cols, 1, 0)) != cudaSuccess) return e;
    const uint32_t tiles = ((a.rows + kUmRows - 1) / kUmRows) * ((a.m + DenseCfg::BN - 1) / DenseCfg::BN);
    const size_t smem = DenseCfg::smem(a.cols / 64, 0);
    return a.y_dtype == PBMOE_F32 ? launch_umma<DenseCfg, float>(p, tx, tw, tiles, smem, s)
                                  : launch_umma<DenseCfg, uint16_t>(p, tx, tw, tiles, smem, s);
}

cudaError_t q4_gemm_grouped_launch(const Q4GroupedArgs& a, cudaStream_t s) {
    UmmaParams p{};
    p.experts = a.experts;
    p.expert_bytes = a.expert_bytes;
    p.scales_offset = a.scales_offset;
    p.biases_offset = a.biases_offset;
    p.N = a.rows;
    p.K = a.cols;
    p.num_experts = a.num_experts;
    p.slot_experts = a.slot_experts;
    p.unique_count = a.unique_count;
    p.max_unique = a.max_unique;
    p.groups = a.groups;
    p.routes = a.routes;
    p.table_cap = q4_grouped_tile_bound(a.routes, a.max_unique);
    p.y = a.y;
    p.status = a.status;
    CUtensorMap tx, tw;
    cudaError_t e;
    if ((e = make_x_map(&tx, a.xg16, a.routes, a.cols, GroupedCfg::BN)) != cudaSuccess) return e;
    if ((e = make_w_map(&tw, a.experts + a.packed_offset, a.rows, a.cols, a.num_experts, a.expert_bytes)) !=
        cudaSuccess)
        return e;
    const uint32_t tiles = ((a.rows + kUmRows - 1) / kUmRows) * p.table_cap;
    const size_t smem = GroupedCfg::smem(a.cols / 64, p.table_cap);
    return a.y_dtype == PBMOE_F32 ? launch_umma<GroupedCfg, float>(p, tx, tw, tiles, smem, s)
                                  : launch_umma<GroupedCfg, uint16_t>(p, tx, tw, tiles, smem, s);
}

}  // namespace pbmoe
