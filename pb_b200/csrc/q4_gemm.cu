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
// Here a persistent CTA per SM walks a static list of output tiles of 128
// weight rows (the UMMA M dimension: one TMEM lane per row) x up to BN tokens
// (N), K advancing one 64-wide quantisation group per step. Ten warps, each
// role on its own ring of shared-memory buffers and mbarriers, so that no role
// waits on another's latency:
//
//   warp 0      loader: cp.async of each step's nibbles (128 rows x 32 B) into
//               a deep W ring and of each tile's scales and biases (double-
//               buffered); completion arrives asynchronously on wfull / sfull
//               through cp.async.mbarrier.arrive.noinc, so it never waits on
//               its own copies.
//   warp 1      TMEM owner; lane 0 issues four tcgen05.mma (K = 16 each) per
//               step when afull completes and commits them to aempty / bempty
//               (frees the A and B stages) and, per tile, to tfull.
//   warps 2-5   one weight row per thread: dequantise w = q*s + b to fp16 (one
//               rounding) into the swizzled A tile; and, P steps ahead, copy
//               the tokens' fp16 rows (gathered by row index) into the
//               128B-swizzled K-major B ring. Each thread waits for its own
//               B copies of the step (cp.async.wait_group P), fences its A
//               stores and those copies to the async proxy the tensor core
//               reads through (fence.proxy.async) and arrives on afull.
//   warps 6-9   epilogue: tcgen05.ld of the finished accumulator (double-
//               buffered in TMEM, so tile t+1's MMAs overlap tile t's stores),
//               stores, arrive on tempty.
//
// Operands are fp16. bf16 weights would carry 2^-9 relative rounding per
// weight (up to ~0.9% max-relative error against the f32 reference on
// config-2 shapes); fp16 keeps 11 bits. bf16 activations convert to fp16
// exactly (x16_convert_kernel); a magnitude >= 65536 or a non-finite value
// has no fp16 image and latches PBMOE_DEV_ERR_F16_RANGE.
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

#include <algorithm>

#include "kernels.h"
#include "pipe.cuh"
#include "umma.cuh"

namespace pbmoe {

constexpr int kUmThreads = 320;
constexpr uint32_t kUmRows = 128;
constexpr uint32_t kMagicPair = 0x54006400u;  // f16x2 (lo 1024.0, hi 64.0)
constexpr uint32_t kNoSlot = 0xffffffffu;

template <int BN_, int SA_, int SB_, int SW_, bool kGathered_>
struct UmmaCfg {
    static constexpr int BN = BN_, SA = SA_, SB = SB_, SW = SW_;
    static constexpr int P = SB - 2;  // B copies run P steps ahead of the dequant step
    static constexpr bool kGathered = kGathered_;
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 128, "UMMA N per accumulator");
    static_assert(SA >= 2 && SB >= 3, "rings");
    static constexpr uint32_t kA = kUmRows * 128;  // fp16 [128 rows][64 k], swizzled
    static constexpr uint32_t kB = BN * 128;       // fp16 [BN tokens][64 k], swizzled (multiple of 1024)
    static constexpr uint32_t kW = kUmRows * 32;   // nibbles [128 rows][32 B]
    static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
    static constexpr int kBRows = BN / 16;         // token rows each dequant thread copies per step
    static constexpr size_t sbuf_bytes(uint32_t groups) { return size_t(kUmRows) * groups * 4; }  // scales + biases
    static constexpr size_t smem(uint32_t groups, uint32_t table) {
        return 1024 + size_t(SA) * kA + size_t(SB) * kB + size_t(SW) * kW + 2 * sbuf_bytes(groups) +
               size_t(table) * 4;
    }
};
using DenseCfg = UmmaCfg<128, 3, 6, 8, false>;
using GroupedCfg = UmmaCfg<64, 3, 8, 12, true>;

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

__device__ __forceinline__ bool warp_wait_lazy(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                               uint32_t* status) {
    bool ok = false;
    if ((threadIdx.x & 31) == 0) ok = wait_or_abort_lazy(bar, parity, abort_flag, status);
    return __shfl_sync(kFull, ok ? 1u : 0u, 0) != 0u;
}

// wait_or_abort decided by lane 0 and broadcast, so the warp stays converged
// for the warp-collective operations that follow.
__device__ __forceinline__ bool warp_wait_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                   uint32_t* status) {
    bool ok = false;
    if ((threadIdx.x & 31) == 0) ok = wait_or_abort(bar, parity, abort_flag, status);
    return __shfl_sync(kFull, ok ? 1u : 0u, 0) != 0u;
}

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes)
                 : "memory");
}

// bf16 bits -> fp16 bits (round to nearest)
__device__ __forceinline__ uint32_t f16_of_bf16(uint32_t v16) {
    return __half_as_ushort(__float2half_rn(__uint_as_float(v16 << 16)));
}

// Eight fp16 weights (k = 8j .. 8j+7) from packed word w of one row.
__device__ __forceinline__ uint4 dequant_word_f16(uint32_t w, uint32_t s2, uint32_t b2) {
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t X = __byte_perm(w, 0u, 0x4040u + 0x0101u * t);  // (byte t, 0, byte t, 0)
        uint32_t m, q;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(m) : "r"(X), "r"(0x00F0000Fu), "r"(kMagicPair));  // (a & b) | c
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(m), "r"(kMagicPair));
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[t]) : "r"(q), "r"(s2), "r"(b2));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Kernel arguments. Dense: packed / scales / biases of one matrix. Grouped:
// the expert table and the component offsets of one projection in a slot.
struct UmmaParams {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* biases;
    const uint8_t* experts;
    uint64_t expert_bytes;
    uint64_t packed_offset, scales_offset, biases_offset;
    uint32_t N, K;                 // per-matrix rows x cols
    uint32_t num_experts;
    const uint16_t* x16;  // fp16 activations [x_rows x K]
    uint32_t x_rows;
    uint32_t M;  // dense: token rows
    // grouped
    const uint32_t* slot_experts;
    const uint32_t* unique_count;
    uint32_t max_unique;
    const uint32_t* groups;
    const uint32_t* source_rows;
    uint32_t routes;
    uint32_t table_cap;  // grouped tile table capacity (entries)
    void* y;
    uint32_t* status;
};

// One output tile as every role sees it.
struct TileInfo {
    const uint8_t* packed;  // this tile's matrix
    const uint16_t* scales;
    const uint16_t* biases;
    uint32_t n0, rows_here;
    uint32_t ntok;   // 0: skip
    uint32_t first;  // dense: first token row; grouped: first grouped row
};

template <class Cfg>
__device__ __forceinline__ TileInfo tile_info(const UmmaParams& p, uint32_t t, uint32_t row_tiles,
                                              const uint32_t* table) {
    TileInfo ti;
    const uint32_t rt = t % row_tiles, jt = t / row_tiles;
    ti.n0 = rt * kUmRows;
    ti.rows_here = min(p.N - ti.n0, kUmRows);
    if constexpr (!Cfg::kGathered) {
        ti.packed = p.packed;
        ti.scales = p.scales;
        ti.biases = p.biases;
        ti.first = jt * Cfg::BN;
        ti.ntok = min(p.M - ti.first, static_cast<uint32_t>(Cfg::BN));
    } else {
        const uint32_t e = table[jt];  // (slot << 8) | token-tile, or kNoSlot
        ti.packed = nullptr;
        ti.scales = ti.biases = nullptr;
        if (e == kNoSlot) {
            ti.first = 0;
            ti.ntok = 0;
        } else {
            const uint32_t slot = e >> 8, tok0 = (e & 0xffu) * Cfg::BN;
            const uint32_t start = p.groups[2 * slot], cnt = p.groups[2 * slot + 1];
            ti.first = start + tok0;
            ti.ntok = min(cnt - tok0, static_cast<uint32_t>(Cfg::BN));
            const uint8_t* base = p.experts + static_cast<size_t>(p.slot_experts[slot]) * p.expert_bytes;
            ti.packed = base + p.packed_offset;
            ti.scales = reinterpret_cast<const uint16_t*>(base + p.scales_offset);
            ti.biases = reinterpret_cast<const uint16_t*>(base + p.biases_offset);
        }
    }
    return ti;
}

template <class Cfg, typename YT>
__global__ void __launch_bounds__(kUmThreads, 1) q4_umma_kernel(const UmmaParams p) {
    constexpr int BN = Cfg::BN, SA = Cfg::SA, SB = Cfg::SB, SW = Cfg::SW, P = Cfg::P;
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t wfull[SW], wfree[SW], sfull[2], sfree[2], afull[SA], aempty[SA], bempty[SB],
        tfull[2], tempty[2], drain;
    __shared__ uint32_t tmem_base_sh, abort_sh, num_tiles_sh, warp_tot[kUmThreads / 32];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t G = p.K / 64;
    unsigned char* aring = smem;                      // SA x A tiles
    unsigned char* bring = aring + SA * Cfg::kA;      // SB x B tiles
    unsigned char* wring = bring + SB * Cfg::kB;      // SW x [128][32] nibbles
    unsigned char* sbufs = wring + SW * Cfg::kW;      // 2 x [scales 128 x G | biases 128 x G] bf16
    uint32_t* table = reinterpret_cast<uint32_t*>(sbufs + 2 * Cfg::sbuf_bytes(G));
    volatile uint32_t* abort_flag = &abort_sh;
    uint32_t* status = p.status;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t row_tiles = (p.N + kUmRows - 1) / kUmRows;

    if (tid == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(&wfull[i], 32);  // one cp.async.mbarrier.arrive.noinc per loader lane
            mbar_init(&wfree[i], 128);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sfull[i], 32);
            mbar_init(&sfree[i], 128);
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 128);
        }
        for (int i = 0; i < SA; ++i) {
            mbar_init(&afull[i], 128);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < SB; ++i) mbar_init(&bempty[i], 1);
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
        // ------------------------------------------------------------ loader: nibbles, scales
        const size_t prow = p.K / 2;
        uint32_t gs = 0, lt = 0;  // global step, local tile
        bool ok = true;
        for (uint32_t t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
            if (ti.ntok == 0) continue;
            const int sb = static_cast<int>(lt & 1);
            if (lt >= 2 && !warp_wait_lazy(&sfree[sb], ((lt >> 1) - 1) & 1, abort_flag, status)) {
                ok = false;
                break;
            }
            {  // the tile rows' scales and biases (contiguous: rows x G each)
                unsigned char* sdst = sbufs + sb * Cfg::sbuf_bytes(G);
                const uint32_t chunks = kUmRows * G / 8, avail = ti.rows_here * G;
                for (uint32_t q = lane; q < chunks; q += 32) {
                    const bool in = q * 8 < avail;
                    const size_t off = static_cast<size_t>(ti.n0) * G + (in ? q * 8 : 0);
                    cp_async16_zfill(sdst + q * 16, ti.scales + off, in ? 16u : 0u);
                    cp_async16_zfill(sdst + kUmRows * G * 2 + q * 16, ti.biases + off, in ? 16u : 0u);
                }
                cp_async_arrive(&sfull[sb]);
            }
            for (uint32_t i = 0; i < G; ++i, ++gs) {
                const int w = static_cast<int>(gs % SW);
                if (gs >= static_cast<uint32_t>(SW) &&
                    !warp_wait_lazy(&wfree[w], ((gs / SW) - 1) & 1, abort_flag, status)) {
                    ok = false;
                    break;
                }
                unsigned char* wdst = wring + w * Cfg::kW;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {  // 128 rows x 2 chunks of nibbles
                    const uint32_t q = jj * 32 + lane, r = q >> 1, cc = q & 1;
                    const bool in = r < ti.rows_here;
                    const uint8_t* src =
                        ti.packed + (static_cast<size_t>(ti.n0 + (in ? r : 0)) * prow + i * 32 + cc * 16);
                    cp_async16_zfill(wdst + r * 32 + ((cc ^ ((r >> 2) & 1)) << 4), src, in ? 16u : 0u);
                }
                cp_async_arrive(&wfull[w]);
            }
            ++lt;
        }
        cp_async_wait_all();  // no copy outlives the CTA
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
                for (uint32_t i = 0; i < G; ++i, ++gs) {
                    const int sa = static_cast<int>(gs % SA), sbi = static_cast<int>(gs % SB);
                    if (!wait_or_abort(&afull[sa], (gs / SA) & 1, abort_flag, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(aring + sa * Cfg::kA), b0 = smem_u32(bring + sbi * Cfg::kB);
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; ++kk)
                        umma_f16(d, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), idesc,
                                 (i | kk) != 0u);
                    umma_commit(&aempty[sa]);
                    umma_commit(&bempty[sbi]);
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
    } else if (warp < 6) {
        // ------------------------------------------------------------ dequant + token rows
        const uint32_t dq = static_cast<uint32_t>(tid - 64);  // 0..127
        const uint32_t r = 32u * (warp & 3) + lane;          // weight row of this thread
        const uint32_t wsw = ((r >> 2) & 1) << 4;
        const uint32_t bc = dq & 7, bj = dq >> 3;  // B copies: chunk bc of token rows bj + 16u
        // B cursor: runs P steps ahead over the same tile sequence
        uint32_t bt = blockIdx.x, bi = 0, bgs = 0;
        TileInfo bti{};
        uint32_t brows[Cfg::kBRows];
        auto b_seek = [&]() {  // first tile with tokens at or after bt
            for (; bt < num_tiles; bt += gridDim.x) {
                bti = tile_info<Cfg>(p, bt, row_tiles, table);
                if (bti.ntok) break;
            }
            if (bt >= num_tiles) return;
#pragma unroll
            for (int u = 0; u < Cfg::kBRows; ++u) {
                const uint32_t j = bj + 16u * u;
                uint32_t row = 0;
                if (j < bti.ntok) {
                    if constexpr (Cfg::kGathered) {
                        row = __ldg(p.source_rows + bti.first + j);
                        if (row >= p.x_rows) {
                            if (status) atomicOr(status, PBMOE_DEV_ERR_EXPERT_ID);
                            row = 0;
                        }
                    } else {
                        row = bti.first + j;
                    }
                }
                brows[u] = row;
            }
        };
        bool ok = true;
        auto b_issue = [&]() {  // token rows of global step bgs, then advance; always one commit group
            if (ok && bt < num_tiles) {
                const int slot = static_cast<int>(bgs % SB);
                if (bgs >= static_cast<uint32_t>(SB) &&
                    !warp_wait_or_abort(&bempty[slot], ((bgs / SB) - 1) & 1, abort_flag, status)) {
                    ok = false;
                } else {
                    unsigned char* bdst = bring + slot * Cfg::kB;
#pragma unroll
                    for (int u = 0; u < Cfg::kBRows; ++u) {
                        const uint32_t j = bj + 16u * u;
                        if (j < bti.ntok)
                            cp_async16(bdst + sw128_offset(j, bc),
                                       p.x16 + static_cast<size_t>(brows[u]) * p.K + bi * 64 + bc * 8);
                    }
                    ++bgs;
                    if (++bi == G) {
                        bi = 0;
                        bt += gridDim.x;
                        b_seek();
                    }
                }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        b_seek();
        for (int k = 0; k < P; ++k) b_issue();

        uint32_t gs = 0, lt = 0;
        for (uint32_t t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
            if (ti.ntok == 0) continue;
            const int sbuf = static_cast<int>(lt & 1);
            if (!warp_wait_or_abort(&sfull[sbuf], (lt >> 1) & 1, abort_flag, status)) {
                ok = false;
                break;
            }
            const uint16_t* srow = reinterpret_cast<const uint16_t*>(sbufs + sbuf * Cfg::sbuf_bytes(G)) + r * G;
            const uint16_t* brow = srow + kUmRows * G;
            uint4 sq = make_uint4(0, 0, 0, 0), bq = sq;
            for (uint32_t i = 0; i < G; ++i, ++gs) {
                b_issue();  // step gs + P
                asm volatile("cp.async.wait_group %0;" ::"n"(P) : "memory");  // this thread's rows of step gs
                if ((i & 7) == 0) {
                    sq = *reinterpret_cast<const uint4*>(srow + i);
                    bq = *reinterpret_cast<const uint4*>(brow + i);
                }
                const int w = static_cast<int>(gs % SW), sa = static_cast<int>(gs % SA);
                if (!ok || !warp_wait_or_abort(&wfull[w], (gs / SW) & 1, abort_flag, status) ||
                    (gs >= static_cast<uint32_t>(SA) &&
                     !warp_wait_or_abort(&aempty[sa], ((gs / SA) - 1) & 1, abort_flag, status))) {
                    ok = false;
                    break;
                }
                // this step's scale and bias: half (i & 1) of word (i & 7) / 2
                const uint32_t sw = (i & 4) ? ((i & 2) ? sq.w : sq.z) : ((i & 2) ? sq.y : sq.x);
                const uint32_t bw = (i & 4) ? ((i & 2) ? bq.w : bq.z) : ((i & 2) ? bq.y : bq.x);
                const uint32_t s16 = f16_of_bf16((i & 1) ? (sw >> 16) : (sw & 0xffffu));
                const uint32_t b16 = f16_of_bf16((i & 1) ? (bw >> 16) : (bw & 0xffffu));
                const uint32_t s2 = s16 * 0x10001u, b2 = b16 * 0x10001u;
                const unsigned char* wr = wring + w * Cfg::kW + r * 32;
                const uint4 w0 = *reinterpret_cast<const uint4*>(wr + wsw);
                const uint4 w1 = *reinterpret_cast<const uint4*>(wr + (16 ^ wsw));
                mbar_arrive(&wfree[w]);  // nibbles are in registers
                unsigned char* arow = aring + sa * Cfg::kA;
                const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (uint32_t jj = 0; jj < 8; ++jj)
                    *reinterpret_cast<uint4*>(arow + sw128_offset(r, jj)) = dequant_word_f16(words[jj], s2, b2);
                fence_proxy_async_smem();  // A stores and the landed token rows, for the tensor core
                mbar_arrive(&afull[sa]);
            }
            if (!ok) break;
            mbar_arrive(&sfree[sbuf]);
            ++lt;
        }
        cp_async_wait_all();  // no copy outlives the CTA
    } else {
        // ------------------------------------------------------------ epilogue
        const uint32_t q = warp & 3, r = 32u * q + lane;
        YT* y = static_cast<YT*>(p.y);
        uint32_t lt = 0;
        for (uint32_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const TileInfo ti = tile_info<Cfg>(p, t, row_tiles, table);
            if (ti.ntok == 0) continue;
            const int acc = static_cast<int>(lt & 1);
            if (!warp_wait_lazy(&tfull[acc], (lt >> 1) & 1, abort_flag, status)) break;
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
            mbar_arrive(&tempty[acc]);
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

// bf16 -> fp16, eight values per thread step; latches PBMOE_DEV_ERR_F16_RANGE
// for a magnitude >= 65536 or a non-finite value.
__global__ void __launch_bounds__(256) x16_convert_kernel(const uint4* __restrict__ x, uint4* __restrict__ x16,
                                                          size_t n8, uint32_t* status) {
    uint32_t mx = 0;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n8; i += size_t(gridDim.x) * blockDim.x) {
        const uint4 v = __ldg(x + i);
        mx = __vmaxu2(mx, __vmaxu2(__vmaxu2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu),
                                   __vmaxu2(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu)));
        uint32_t o[4];
        const uint32_t in[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            asm("cvt.rn.f16x2.f32 %0, %1, %2;"
                : "=r"(o[k])
                : "f"(__uint_as_float(in[k] & 0xffff0000u)), "f"(__uint_as_float(in[k] << 16)));
        x16[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (((mx & 0xffffu) >= 0x4780u || (mx >> 16) >= 0x4780u) && status) atomicOr(status, PBMOE_DEV_ERR_F16_RANGE);
}

static int g_num_sms = 0;

static int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) ==
                                                      cudaSuccess)
            g_num_sms = n;
        else
            g_num_sms = 148;
    }
    return g_num_sms;
}

bool q4_gemm_supported(uint32_t N, uint32_t K, uint32_t group) {
    return group == 64 && K % 512 == 0 && N > 0 && DenseCfg::smem(K / 64, 0) <= 227 * 1024;
}

bool q4_grouped_supported(uint32_t N, uint32_t K, uint32_t group, uint32_t routes, uint32_t max_unique) {
    return q4_gemm_supported(N, K, group) &&
           GroupedCfg::smem(K / 64, q4_grouped_tile_bound(routes, max_unique)) <= 227 * 1024;
}

template <class Cfg, typename YT>
static cudaError_t launch_umma(const UmmaParams& p, uint32_t tiles, size_t smem, cudaStream_t s) {
    auto k = q4_umma_kernel<Cfg, YT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const uint32_t grid = std::max<uint32_t>(1u, std::min<uint32_t>(tiles, static_cast<uint32_t>(num_sms())));
    k<<<grid, kUmThreads, smem, s>>>(p);
    return cudaGetLastError();
}

cudaError_t x16_convert_launch(const void* x, void* x16, size_t elems, uint32_t* status, cudaStream_t s) {
    const size_t n8 = elems / 8;
    if (n8 == 0) return cudaSuccess;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((n8 + 255) / 256, 148 * 8));
    x16_convert_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(x), static_cast<uint4*>(x16), n8, status);
    return cudaGetLastError();
}

cudaError_t q4_gemm_launch(const Q4GemmArgs& a, cudaStream_t s) {
    UmmaParams p{};
    p.packed = a.packed;
    p.scales = a.scales;
    p.biases = a.biases;
    p.N = a.rows;
    p.K = a.cols;
    p.num_experts = 1;
    p.x16 = static_cast<const uint16_t*>(a.x16);
    p.x_rows = a.m;
    p.M = a.m;
    p.y = a.y;
    p.status = a.status;
    const uint32_t tiles = ((a.rows + kUmRows - 1) / kUmRows) * ((a.m + DenseCfg::BN - 1) / DenseCfg::BN);
    const size_t smem = DenseCfg::smem(a.cols / 64, 0);
    return a.y_dtype == PBMOE_F32 ? launch_umma<DenseCfg, float>(p, tiles, smem, s)
                                  : launch_umma<DenseCfg, uint16_t>(p, tiles, smem, s);
}

uint32_t q4_grouped_tile_bound(uint32_t routes, uint32_t max_unique) {
    // sum over slots of ceil(count / BN) <= routes / BN + slots
    return (routes + GroupedCfg::BN - 1) / GroupedCfg::BN + max_unique;
}

cudaError_t q4_gemm_grouped_launch(const Q4GroupedArgs& a, cudaStream_t s) {
    UmmaParams p{};
    p.experts = a.experts;
    p.expert_bytes = a.expert_bytes;
    p.packed_offset = a.packed_offset;
    p.scales_offset = a.scales_offset;
    p.biases_offset = a.biases_offset;
    p.N = a.rows;
    p.K = a.cols;
    p.num_experts = a.num_experts;
    p.x16 = static_cast<const uint16_t*>(a.x16);
    p.x_rows = a.x_rows;
    p.slot_experts = a.slot_experts;
    p.unique_count = a.unique_count;
    p.max_unique = a.max_unique;
    p.groups = a.groups;
    p.source_rows = a.source_rows;
    p.routes = a.routes;
    p.table_cap = q4_grouped_tile_bound(a.routes, a.max_unique);
    p.y = a.y;
    p.status = a.status;
    const uint32_t tiles = ((a.rows + kUmRows - 1) / kUmRows) * p.table_cap;
    const size_t smem = GroupedCfg::smem(a.cols / 64, p.table_cap);
    return a.y_dtype == PBMOE_F32 ? launch_umma<GroupedCfg, float>(p, tiles, smem, s)
                                  : launch_umma<GroupedCfg, uint16_t>(p, tiles, smem, s);
}

}  // namespace pbmoe
