// head.cu — the vocab head of a decode step: logits = W x (bf16 W [V x H],
// f32 accumulate) for up to 32 tokens, then each token's top-k candidates in
// the order of the reference's topk_vocab (shaders.metal:1796-1831), run on
// the resident LM-head projection by MetalResidentTopKBuilder
// (metal/mod.rs:2661-2800) for sample_from_hidden (runtime/generation.rs:
// 2200-2227).
//
// Kernel 1, head_gemv_kernel: the weight stream (622 MB at V 151936, H 2048)
// is the roofline; every weight byte is read once. Weights are the stationary
// operand of mma.sync m16n8k16 (16 vocabulary rows x 8 tokens x 16 columns):
// each lane loads 32 contiguous bytes of its row per 64-column step (four
// lanes cover one 128-byte line), and the 16 columns of each mma are a fixed
// permutation of the step's columns, applied identically to the activations.
// f32 activations are split into bf16 hi + lo halves in shared memory (two
// mma per fragment), so the products keep ~16 significant bits of x and
// exactly the bf16 weight; bf16 activations are exact as one half. The CTA's grid row is one half of H (blockIdx.y):
// the two halves add into zeroed logits with f32 atomics, and a sum of two
// terms onto zero is the same in either order, so logits are deterministic.
//
// Kernel 2, head_select_kernel: per (token, slice of 2048 logits) an exact
// top-k by radix selection of the k-th largest value key, then the selected
// entries sorted by (value desc, index asc): topk_vocab's order, where a
// non-finite logit counts as -inf, a disallowed token is never chosen, and
// slots beyond the allowed tokens are (0, -inf). Kernel 3, head_merge_kernel,
// merges the slices' sorted lists (and the lists of vocabulary shards held by
// other ranks): lists are concatenated in index order, so equal keys keep
// list order, which is index order.

#include "kernels.h"
#include "q4_mma.cuh"
#include "routing.cuh"

namespace pbmoe {

constexpr int kHeadWarps = 16;
constexpr int kHeadThreads = kHeadWarps * 32;
constexpr int kHeadDepth = 4;               // 64-column steps in flight per lane
constexpr uint32_t kHeadPadBytes = 16;      // token rows 16 bytes apart mod 128: conflict-free 16-byte reads
constexpr uint32_t kHeadMaxTokens = 32;
constexpr uint32_t kHeadMaxSelect = 256;   // largest k

__host__ __device__ inline uint32_t head_row_bytes(uint32_t H) { return H + kHeadPadBytes; }  // H/2 bf16

template <int NT, typename XT>
__global__ void __launch_bounds__(kHeadThreads, 1)
head_gemv_kernel(const uint16_t* __restrict__ W, uint32_t V, uint32_t H, const XT* __restrict__ x, uint32_t T,
                 float* __restrict__ logits) {
    // bf16 activations are exact in bf16: their lo half is zero and skipped
    constexpr bool kLo = sizeof(XT) == 4;
    extern __shared__ __align__(16) uint8_t hsm[];
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t Hh = H / 2;
    const uint32_t k0 = blockIdx.y * Hh;  // this CTA's half of the columns
    const uint32_t rb = head_row_bytes(H);
    uint8_t* xhi = hsm;
    uint8_t* xlo = hsm + static_cast<size_t>(NT) * 8 * rb;
    // x -> bf16 hi + lo (lo = bf16(x - hi), exact difference), two columns per thread
    const uint32_t pairs = Hh / 2;
    for (uint32_t i = threadIdx.x; i < NT * 8 * pairs; i += blockDim.x) {
        const uint32_t tok = i / pairs, c = (i - tok * pairs) * 2;
        float v0 = 0.f, v1 = 0.f;
        if (tok < T) {
            v0 = load_act<XT>(x, static_cast<size_t>(tok) * H + k0 + c);
            v1 = load_act<XT>(x, static_cast<size_t>(tok) * H + k0 + c + 1);
        }
        const uint16_t h0 = f32_to_bf16_bits(v0), h1 = f32_to_bf16_bits(v1);
        const uint16_t l0 = f32_to_bf16_bits(v0 - bf16_bits_to_f32(h0));
        const uint16_t l1 = f32_to_bf16_bits(v1 - bf16_bits_to_f32(h1));
        *reinterpret_cast<uint32_t*>(xhi + tok * rb + c * 2) = h0 | (static_cast<uint32_t>(h1) << 16);
        if constexpr (kLo) *reinterpret_cast<uint32_t*>(xlo + tok * rb + c * 2) = l0 | (static_cast<uint32_t>(l1) << 16);
    }
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, tq = lane & 3;
    const uint32_t nblk = (V + 15) / 16;
    const uint32_t steps = Hh / 64;  // a multiple of kHeadDepth (host check)
    for (uint32_t blk = blockIdx.x * kHeadWarps + warp; blk < nblk; blk += gridDim.x * kHeadWarps) {
        const uint32_t ra = blk * 16 + g, rbw = ra + 8;
        // rows past V read row V-1 (in bounds); their results are dropped
        const uint16_t* pa = W + static_cast<size_t>(min(ra, V - 1)) * H + k0 + 16 * tq;
        const uint16_t* pb = W + static_cast<size_t>(min(rbw, V - 1)) * H + k0 + 16 * tq;
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
        uint4 ring[kHeadDepth][4];
#pragma unroll
        for (int d = 0; d < kHeadDepth; ++d) {
            ring[d][0] = ld_stream_u4(pa + d * 64);
            ring[d][1] = ld_stream_u4(pa + d * 64 + 8);
            ring[d][2] = ld_stream_u4(pb + d * 64);
            ring[d][3] = ld_stream_u4(pb + d * 64 + 8);
        }
        for (uint32_t s0 = 0; s0 < steps; s0 += kHeadDepth) {
#pragma unroll
            for (int d = 0; d < kHeadDepth; ++d) {
                const uint32_t s = s0 + d;
                const uint32_t wa[8] = {ring[d][0].x, ring[d][0].y, ring[d][0].z, ring[d][0].w,
                                        ring[d][1].x, ring[d][1].y, ring[d][1].z, ring[d][1].w};
                const uint32_t wb[8] = {ring[d][2].x, ring[d][2].y, ring[d][2].z, ring[d][2].w,
                                        ring[d][3].x, ring[d][3].y, ring[d][3].z, ring[d][3].w};
                if (s + kHeadDepth < steps) {
                    const uint32_t off = (s + kHeadDepth) * 64;
                    ring[d][0] = ld_stream_u4(pa + off);
                    ring[d][1] = ld_stream_u4(pa + off + 8);
                    ring[d][2] = ld_stream_u4(pb + off);
                    ring[d][3] = ld_stream_u4(pb + off + 8);
                }
                const uint32_t cbyte = (s * 64 + 16 * tq) * 2;
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    const uint32_t tok = n * 8 + g;
                    const uint4 h0 = *reinterpret_cast<const uint4*>(xhi + tok * rb + cbyte);
                    const uint4 h1 = *reinterpret_cast<const uint4*>(xhi + tok * rb + cbyte + 16);
                    const uint32_t xh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                    uint32_t xl[8] = {};
                    if constexpr (kLo) {
                        const uint4 l0 = *reinterpret_cast<const uint4*>(xlo + tok * rb + cbyte);
                        const uint4 l1 = *reinterpret_cast<const uint4*>(xlo + tok * rb + cbyte + 16);
                        xl[0] = l0.x, xl[1] = l0.y, xl[2] = l0.z, xl[3] = l0.w;
                        xl[4] = l1.x, xl[5] = l1.y, xl[6] = l1.z, xl[7] = l1.w;
                    }
                    // mma `sub`: logical k 2tq+j <-> column 16tq+4sub+j, 2tq+8+j <-> 16tq+4sub+2+j
#pragma unroll
                    for (int sub = 0; sub < 4; ++sub) {
                        mma_bf16_16816(acc[n], wa[2 * sub], wb[2 * sub], wa[2 * sub + 1], wb[2 * sub + 1],
                                       xh[2 * sub], xh[2 * sub + 1]);
                        if constexpr (kLo)
                            mma_bf16_16816(acc[n], wa[2 * sub], wb[2 * sub], wa[2 * sub + 1], wb[2 * sub + 1],
                                           xl[2 * sub], xl[2 * sub + 1]);
                    }
                }
            }
        }
        // acc[n]: (row g, tokens 8n+2tq, +1), (row g+8, same tokens)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const uint32_t t0 = n * 8 + 2 * tq, t1 = t0 + 1;
            if (ra < V) {
                if (t0 < T) atomicAdd(logits + static_cast<size_t>(t0) * V + ra, acc[n][0]);
                if (t1 < T) atomicAdd(logits + static_cast<size_t>(t1) * V + ra, acc[n][1]);
            }
            if (rbw < V) {
                if (t0 < T) atomicAdd(logits + static_cast<size_t>(t0) * V + rbw, acc[n][2]);
                if (t1 < T) atomicAdd(logits + static_cast<size_t>(t1) * V + rbw, acc[n][3]);
            }
        }
    }
}

// ---------------------------------------------------------------- selection
constexpr int kSelThreads = 256;
constexpr uint32_t kSelSlice = 2048;      // logits per CTA of the first pass
constexpr uint32_t kMergeMax = 24576;     // candidates per token in a merge (lists x k)
constexpr uint32_t kMergeSort = 512;      // candidates at or above the bound sorted directly

// Candidate key: 0 = no candidate (a disallowed token, or a slot past the
// allowed tokens), else the order key of the value (non-finite as -inf) + 1.
__device__ __forceinline__ uint32_t head_value_key(float v) {
    if (!isfinite(v)) v = -__int_as_float(0x7f800000);
    return float_order_key(v) + 1u;
}

// CTA (t, y) selects the top `k` of slice y of token t's logits (ids =
// id_base + position, keys from the values and the allowed-token bitmask) by
// (key desc, position asc) and writes them sorted as the slice's list;
// positions past the slice get (key 0, id 0, -inf). Keys live in shared
// memory (kSelSlice u32), then the selected entries.
__global__ void __launch_bounds__(kSelThreads)
head_select_kernel(const float* __restrict__ logits, size_t logits_stride, uint32_t id_base,
                   const uint32_t* __restrict__ allowed, uint32_t n, uint32_t k, uint32_t* __restrict__ out_key,
                   uint32_t* __restrict__ out_id, float* __restrict__ out_val, size_t out_stride) {
    __shared__ uint32_t keys[kSelSlice];
    __shared__ uint32_t hist[256];
    __shared__ unsigned long long sel[kHeadMaxSelect];  // (key << 32) | ~position, sorted descending
    __shared__ uint32_t scan_tmp[32];
    __shared__ uint32_t s_prefix, s_rem, s_gt, s_eq;
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t t = blockIdx.x;
    const uint32_t base = blockIdx.y * kSelSlice;  // first position of this CTA's slice
    if (base >= n) return;
    const uint32_t m = min(kSelSlice, n - base);
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
        const uint32_t id = id_base + base + i;
        const bool ok = !allowed || ((allowed[id >> 5] >> (id & 31)) & 1u);
        keys[i] = ok ? head_value_key(logits[t * logits_stride + base + i]) : 0u;
    }
    const uint32_t want = min(k, m);
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_rem = want;
    }
    __syncthreads();
    // radix selection of the want-th largest key, 8 bits at a time
    uint32_t pmask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
            const uint32_t key = keys[i];
            if ((key & pmask) == prefix) {
                const uint32_t digit = (key >> shift) & 255u;
                // aggregate equal digits of the warp into one shared atomic
                const uint32_t active = __activemask();
                const uint32_t peers = __match_any_sync(active, digit);
                if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
            }
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // lane l holds bins 255-8l .. 248-8l (descending)
            const int lane = threadIdx.x;
            uint32_t c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = hist[255 - 8 * lane - j];
                tot += c[j];
            }
            uint32_t incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(kFull, incl, o);
                if (lane >= o) incl += v;
            }
            const uint32_t rem = s_rem;
            const uint32_t excl = incl - tot;
            const bool here = excl < rem && rem <= incl;  // exactly one lane
            if (here) {
                uint32_t above = excl;
                int j = 0;
                while (above + c[j] < rem) {
                    above += c[j];
                    ++j;
                }
                s_prefix = prefix | (static_cast<uint32_t>(255 - 8 * lane - j) << shift);
                s_rem = rem - above;
                s_eq = c[j];  // after the last pass: the keys equal to the threshold
            }
        }
        pmask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t thr = s_prefix;      // the want-th largest key
    const uint32_t need_eq = s_rem;     // entries equal to thr to take, lowest positions first
    const uint32_t n_gt = want - need_eq;
    if (threadIdx.x == 0) s_gt = 0;
    __syncthreads();
    // entries above the threshold, and the equal ones too when all of them
    // are taken (any order; sorted below)
    const bool all_eq = s_eq == need_eq;
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
        const uint32_t key = keys[i];
        if (key > thr || (all_eq && key == thr)) {
            const uint32_t slot = atomicAdd(&s_gt, 1u);
            sel[slot] = (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(~(base + i));
        }
    }
    // otherwise the need_eq lowest positions among the equal ones (each
    // thread scans a contiguous range, ranks from a block scan)
    if (!all_eq) {
        const uint32_t per = (m + blockDim.x - 1) / blockDim.x;
        const uint32_t lo = threadIdx.x * per, hi = min(lo + per, m);
        uint32_t cnt = 0;
        for (uint32_t i = lo; i < hi; ++i) cnt += keys[i] == thr ? 1u : 0u;
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        uint32_t incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) scan_tmp[w] = incl;
        __syncthreads();
        if (w == 0) {
            const uint32_t nw = blockDim.x / 32;
            uint32_t v = static_cast<uint32_t>(lane) < nw ? scan_tmp[lane] : 0u;
            uint32_t inc2 = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t u = __shfl_up_sync(kFull, inc2, o);
                if (lane >= o) inc2 += u;
            }
            if (static_cast<uint32_t>(lane) < nw) scan_tmp[lane] = inc2 - v;  // exclusive
        }
        __syncthreads();
        uint32_t rank = scan_tmp[w] + incl - cnt;
        for (uint32_t i = lo; i < hi && rank < need_eq; ++i) {
            if (keys[i] == thr) {
                sel[n_gt + rank] = (static_cast<unsigned long long>(thr) << 32) | static_cast<uint32_t>(~(base + i));
                ++rank;
            }
        }
    }
    // bitonic sort of the want entries (padded with zeros, which sort last)
    uint32_t P = 1;
    while (P < want) P <<= 1;
    __syncthreads();
    for (uint32_t i = want + threadIdx.x; i < P; i += blockDim.x) sel[i] = 0ull;
    __syncthreads();
    for (uint32_t size = 2; size <= P; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = threadIdx.x; i < P / 2; i += blockDim.x) {
                const uint32_t a = 2 * i - (i & (stride - 1));  // pair (a, a + stride)
                const uint32_t b = a + stride;
                const bool desc = (a & size) == 0;  // descending runs first
                const unsigned long long x = sel[a], y = sel[b];
                if ((x < y) == desc) {
                    sel[a] = y;
                    sel[b] = x;
                }
            }
            __syncthreads();
        }
    }
    // write the slice's list: (key, id, value); empty slots (0, 0, -inf)
    const size_t o = static_cast<size_t>(t) * out_stride + static_cast<size_t>(blockIdx.y) * k;
    for (uint32_t r = threadIdx.x; r < k; r += blockDim.x) {
        uint32_t key = 0, id = 0;
        float val = -__int_as_float(0x7f800000);
        if (r < want) {
            const unsigned long long e = sel[r];
            key = static_cast<uint32_t>(e >> 32);
            const uint32_t p = ~static_cast<uint32_t>(e);
            if (key) {
                id = id_base + p;
                const float v = logits[t * logits_stride + p];
                val = isfinite(v) ? v : val;
            }
        }
        out_key[o + r] = key;
        out_id[o + r] = id;
        out_val[o + r] = val;
    }
}

// Merge of sorted candidate lists: entry r of list l of token t sits at
// t * tok_stride + l * list_stride + r; every list is sorted by (key desc,
// id asc) and the lists cover increasing id ranges, so (key, position l*k+r)
// orders entries exactly as (key desc, id asc). The k-th largest of any
// subset of the union is a lower bound of the union's k-th; the subset taken
// is the first ceil(k / lists) entries of every list (>= k entries, <= k +
// lists), sorted once. Only entries at or above that bound can be selected
// (typically little more than k): they are gathered and sorted directly.
// When more than kMergeSort entries are at or above it, an entry's rank in
// the union is counted instead: r plus, per other list, a binary search for
// the entries ordering before it; ranks below k are written in place.
__global__ void __launch_bounds__(kSelThreads)
head_merge_kernel(const uint32_t* __restrict__ in_key, const uint32_t* __restrict__ in_id,
                  const float* __restrict__ in_val, size_t tok_stride, size_t list_stride, uint32_t lists,
                  uint32_t k, uint32_t* __restrict__ out_key, uint32_t* __restrict__ out_id,
                  float* __restrict__ out_val) {
    extern __shared__ unsigned long long comp[];  // [lists x k]: (key << 32) | ~position
    __shared__ unsigned long long cand[kMergeSort];  // the bound's subset, then the entries at or above it
    __shared__ unsigned long long s_bound;
    __shared__ uint32_t s_cnt;
    pdl_wait();
    pdl_launch_dependents();
    const uint32_t t = blockIdx.x, n = lists * k;
    for (uint32_t p = threadIdx.x; p < n; p += blockDim.x) {
        const uint32_t l = p / k, r = p - l * k;
        const uint32_t key = in_key[t * tok_stride + l * list_stride + r];
        comp[p] = (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(~p);
    }
    if (threadIdx.x == 0) s_cnt = 0;
    // the bound: k-th largest of the first m entries of every list
    const uint32_t m = (k + lists - 1) / lists;
    const uint32_t sub = m * lists;  // <= k + lists - 1 <= kMergeSort (host check)
    auto bitonic_desc = [&](uint32_t cnt) {  // sorts cand[0, cnt) descending; pads with 0
        uint32_t P = 1;
        while (P < cnt) P <<= 1;
        for (uint32_t i = cnt + threadIdx.x; i < P; i += blockDim.x) cand[i] = 0ull;
        __syncthreads();
        for (uint32_t size = 2; size <= P; size <<= 1) {
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                for (uint32_t i = threadIdx.x; i < P / 2; i += blockDim.x) {
                    const uint32_t a = 2 * i - (i & (stride - 1));
                    const uint32_t b = a + stride;
                    const bool desc = (a & size) == 0;
                    const unsigned long long x = cand[a], y = cand[b];
                    if ((x < y) == desc) {
                        cand[a] = y;
                        cand[b] = x;
                    }
                }
                __syncthreads();
            }
        }
    };
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < sub; i += blockDim.x) cand[i] = comp[(i / m) * k + i % m];
    __syncthreads();
    bitonic_desc(sub);
    if (threadIdx.x == 0) s_bound = cand[k - 1];
    __syncthreads();
    const unsigned long long bound = s_bound;
    for (uint32_t p = threadIdx.x; p < n; p += blockDim.x) {
        const unsigned long long c = comp[p];
        if (c >= bound) {
            const uint32_t slot = atomicAdd(&s_cnt, 1u);
            if (slot < kMergeSort) cand[slot] = c;
        }
    }
    __syncthreads();
    const uint32_t cnt = s_cnt;
    auto emit = [&](uint32_t rank, unsigned long long c) {
        const uint32_t p = ~static_cast<uint32_t>(c);
        const uint32_t l = p / k, r = p - l * k;
        const size_t q = t * tok_stride + l * list_stride + r;
        const size_t o = static_cast<size_t>(t) * k + rank;
        const uint32_t key = static_cast<uint32_t>(c >> 32);
        out_key[o] = key;
        out_id[o] = key ? in_id[q] : 0u;
        out_val[o] = key ? in_val[q] : -__int_as_float(0x7f800000);
    };
    if (cnt <= kMergeSort) {
        bitonic_desc(cnt);
        for (uint32_t r = threadIdx.x; r < k; r += blockDim.x) emit(r, cand[r]);
        return;
    }
    for (uint32_t p = threadIdx.x; p < n; p += blockDim.x) {
        const unsigned long long c = comp[p];
        if (c < bound) continue;
        const uint32_t l = p / k;
        uint32_t rank = p - l * k;
        for (uint32_t o = 0; o < lists && rank < k; ++o) {
            if (o == l) continue;
            const unsigned long long* lo = comp + static_cast<size_t>(o) * k;
            uint32_t a = 0, b = k;  // first index of list o whose comp < c
            while (a < b) {
                const uint32_t mid = (a + b) >> 1;
                if (lo[mid] > c) a = mid + 1;
                else b = mid;
            }
            rank += a;
        }
        if (rank < k) emit(rank, c);
    }
}

// ---------------------------------------------------------------- host side
uint32_t head_slices(uint32_t vocab) { return (vocab + kSelSlice - 1) / kSelSlice; }

static int head_tiles(uint32_t tokens) { return tokens <= 8 ? 1 : (tokens <= 16 ? 2 : 4); }
static size_t head_smem(uint32_t hidden, uint32_t tokens, bool lo) {
    return (lo ? 2ull : 1ull) * head_tiles(tokens) * 8 * head_row_bytes(hidden);  // x hi (+ lo)
}

bool head_supported(uint32_t vocab, uint32_t hidden, uint32_t tokens, uint32_t top_k) {
    const uint32_t steps = hidden / 2 / 64;
    return vocab > 0 && hidden > 0 && hidden % (2 * 64 * kHeadDepth) == 0 && steps % kHeadDepth == 0 &&
           tokens > 0 && tokens <= kHeadMaxTokens && top_k > 0 && top_k <= kHeadMaxSelect &&
           head_slices(vocab) * top_k <= kMergeMax && head_slices(vocab) + top_k - 1 <= kMergeSort &&
           head_smem(hidden, tokens, true) <= 227ull * 1024;
}

template <int NT, typename XT>
static cudaError_t head_gemv_t(const HeadArgs& a, cudaStream_t s) {
    auto fn = head_gemv_kernel<NT, XT>;
    const size_t smem = head_smem(a.hidden, a.tokens, sizeof(XT) == 4);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    // one CTA per SM, half of them per column half
    const uint32_t nblk = (a.vocab + 15) / 16;
    uint32_t per_half = static_cast<uint32_t>(sms > 1 ? sms / 2 : 1);
    const uint32_t need = (nblk + kHeadWarps - 1) / kHeadWarps;
    if (per_half > need) per_half = need;
    return launch_pdl_kernel(fn, dim3(per_half, 2), dim3(kHeadThreads), smem, s, a.weight, a.vocab, a.hidden,
                             static_cast<const XT*>(a.x), a.tokens, a.logits);
}

template <typename XT>
static cudaError_t head_gemv(const HeadArgs& a, cudaStream_t s) {
    if (a.tokens <= 8) return head_gemv_t<1, XT>(a, s);
    if (a.tokens <= 16) return head_gemv_t<2, XT>(a, s);
    return head_gemv_t<4, XT>(a, s);
}

cudaError_t head_topk_launch(const HeadArgs& a, cudaStream_t s) {
    if (!head_supported(a.vocab, a.hidden, a.tokens, a.top_k)) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(a.logits, 0, static_cast<size_t>(a.tokens) * a.vocab * sizeof(float), s);
    if (e != cudaSuccess) return e;
    e = a.x_dtype == PBMOE_BF16 ? head_gemv<uint16_t>(a, s) : head_gemv<float>(a, s);
    if (e != cudaSuccess) return e;
    const uint32_t S = head_slices(a.vocab);
    if ((e = launch_pdl_kernel(head_select_kernel, dim3(a.tokens, S), dim3(kSelThreads), 0, s, a.logits,
                               static_cast<size_t>(a.vocab), a.id_base, a.allowed, a.vocab, a.top_k, a.cand_key,
                               a.cand_id, a.cand_val, static_cast<size_t>(S) * a.top_k)) != cudaSuccess)
        return e;
    return head_merge_launch(a.cand_key, a.cand_id, a.cand_val, a.tokens, S, static_cast<size_t>(S) * a.top_k,
                             a.top_k, a.top_k, a.out_key, a.out_id, a.out_val, s);
}

cudaError_t head_merge_launch(const uint32_t* in_key, const uint32_t* in_id, const float* in_val, uint32_t tokens,
                              uint32_t lists, size_t tok_stride, size_t list_stride, uint32_t top_k,
                              uint32_t* out_key, uint32_t* out_id, float* out_val, cudaStream_t s) {
    if (tokens == 0 || lists == 0 || top_k == 0 || top_k > kHeadMaxSelect || lists * top_k > kMergeMax ||
        top_k + lists - 1 > kMergeSort)
        return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(lists) * top_k * sizeof(unsigned long long);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(head_merge_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_pdl_kernel(head_merge_kernel, dim3(tokens), dim3(kSelThreads), smem, s, in_key, in_id, in_val,
                             tok_stride, list_stride, lists, top_k, out_key, out_id, out_val);
}

}  // namespace pbmoe
