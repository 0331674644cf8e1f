// kernels.h — host-visible launch interfaces between the C-ABI layer
// (capi.cu) and the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "pbmoe_cuda.h"

namespace pbmoe {

// Device workspace of one MoE layer launch (carved out of one allocation by
// capi.cu, sized for the reserved maximum token count). Route index r is
// t*K + k for routed routes and T*K + t for token t's shared-expert route.
struct MoeWs {
    uint32_t* status;        // device status word (PBMOE_DEV_ERR_*)
    uint32_t* ticket;        // [2] router-kernel counters (CTAs with logits written, CTAs done
                             // routing), kept at 0 between launches
    float* logits;           // [T x E]
    float* shared_logit;     // [T]
    uint32_t* route_ids;     // [T x K]
    float* route_w;          // [T x K]
    uint32_t* num_groups;    // [1]
    uint32_t* group_expert;  // [gmax]  expert id, E = shared expert
    uint32_t* group_start;   // [gmax]  first grouped position
    uint32_t* group_count;   // [gmax]
    uint32_t* group_routes;  // [T*K + T] route index per grouped position
    uint32_t* group_tokens;  // [T*K + T] token index per grouped position
    float* h;                // [(T*K + T) x I] SwiGLU activations per route
    float* y;                // [(T*K + T) x H] expert outputs per route
    uint8_t* h_perm;         // [(T*K + T) x hperm_stride] SwiGLU activations as bf16 hi/lo pair
                             // slots + per-8 partial sums (input layout of the pipelined down kernel)
    uint16_t* xn;            // [T x H] bf16 RMSNorm(x) * w when the layer normalises its own input
};

// Bytes per route of MoeWs::h_perm for intermediate size I: hi slots, lo
// slots (I/8 x 16 B each) and I/8 f32 partial sums, rounded to 16.
__host__ __device__ inline size_t hperm_stride(uint32_t I) {
    return ((size_t(I / 8) * 16 * 2 + size_t(I / 8) * 4) + 15) / 16 * 16;
}

// Expert slot geometry as the kernels use it.
struct MoeLayoutDev {
    uint64_t off[9];
    uint64_t expert_bytes;
    uint32_t hidden;
    uint32_t inter;
    uint32_t group;
    uint32_t cpg_shift_h;  // log2(group/32) for rows of length hidden
    uint32_t cpg_shift_i;  // same for rows of length inter
    uint32_t mxfp4;        // slots are FIXED_MXFP4 (E2M1 + E8M0 per 32 columns), not affine Q4
};

// Expert-parallel combine: every rank's exchange buffer ([2 parity][world]
// [max_tokens][H] f32 partial outputs, then [world][max_tokens][pieces] u32
// epoch flags, then this rank's u32 epoch counter), addressed through peer pointers
// (this rank's own at index rank). The counter lives on the device and is
// advanced once per layer by the router kernel, so captured CUDA graphs
// replay with fresh epochs.
constexpr uint32_t kMaxEpRanks = 8;
// A token's row is combined in up to this many column pieces (one CTA each,
// one thread-block cluster per token), each with its own exchange flag.
constexpr uint32_t kCombinePieces = 8;
struct EpPeers {
    float* recv[kMaxEpRanks];
    uint32_t* flags[kMaxEpRanks];
    uint32_t* epoch;  // this rank's counter
    uint32_t rank, world, max_tokens;
    uint64_t timeout_ns;
};
__host__ __device__ inline size_t ep_recv_floats(uint32_t world, uint32_t max_tokens, uint32_t H) {
    return size_t(2) * world * max_tokens * H;
}
__host__ __device__ inline size_t ep_flags_offset(uint32_t world, uint32_t max_tokens, uint32_t H) {
    return ep_recv_floats(world, max_tokens, H) * 4;
}
__host__ __device__ inline size_t ep_epoch_offset(uint32_t world, uint32_t max_tokens, uint32_t H) {
    return (ep_flags_offset(world, max_tokens, H) + size_t(world) * max_tokens * kCombinePieces * 4 + 15) / 16 * 16;
}
__host__ __device__ inline size_t ep_buffer_bytes(uint32_t world, uint32_t max_tokens, uint32_t H) {
    return ep_epoch_offset(world, max_tokens, H) + 16;
}

struct MoeLaunch {
    MoeWs ws;
    MoeLayoutDev layout;
    uint32_t tokens, num_experts, top_k, normalization;
    float routed_scale, eps;
    const void* x;
    pbmoe_dtype x_dtype;
    const void* residual;
    void* out;
    pbmoe_dtype out_dtype;
    const float* next_norm_w;
    void* next_normed;
    const uint16_t* router_w;
    const uint16_t* shared_gate;
    // when set, x is the un-normalised hidden state: the router kernel writes
    // ws.xn = bf16(RMSNorm(x) * in_norm_w) (epsilon in_eps), and routing and
    // the experts run on it (the post-attention norm of CMD2)
    const float* in_norm_w;
    float in_eps;
    // f32 [E] router correction bias: sigmoid/noaux routing (NULL: softmax)
    const float* router_bias;
    const uint8_t* experts;
    const uint8_t* shared_slot;
    bool pdl;  // launch the router kernel with programmatic dependent launch
    void* const* phase_events;  // NULL, or 5 cudaEvent_t recorded around the kernels
    // expert parallelism: this rank runs experts [expert_lo, expert_lo +
    // expert_count) (0 = all), `experts` holding exactly those slots; with
    // `ep` set the combine sums the partials of every rank over peer memory
    uint32_t expert_lo, expert_count;
    const EpPeers* ep;
};

// Per-launch bytes of each workspace array, in MoeWs order (host arithmetic).
struct MoeWsSizes {
    size_t bytes[16];
    size_t total;
};
MoeWsSizes moe_ws_sizes(uint32_t max_tokens, uint32_t E, uint32_t K, uint32_t H, uint32_t I);
MoeWs moe_ws_carve(void* base, uint32_t* status, uint32_t max_tokens, uint32_t E, uint32_t K, uint32_t H,
                   uint32_t I);

// Layout and config checks shared by every MoE layer entry point: a PBMOE_*
// status, the failure's text in msg (len bytes).
int moe_check_layout(const pbmoe_expert_layout& L, char* msg, size_t len);
int moe_check_config(const pbmoe_moe_config* c, char* msg, size_t len);

cudaError_t moe_layer_launch(const MoeLaunch& a, cudaStream_t s);
// cudaLaunchKernelExC, with programmatic dependent launch when `pdl`.
cudaError_t moe_launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args, bool pdl);
// CUDA-core expert kernels for FIXED_MXFP4 slots (moe_mxfp4.cu).
cudaError_t moe_up_mxfp4_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl);
cudaError_t moe_down_mxfp4_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl);
// Tensor-core expert kernels (group-64 layouts, moe_mma.cu).
bool moe_mma_supported(const MoeLayoutDev& L);
cudaError_t moe_up_mma_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl);
cudaError_t moe_down_mma_launch(const MoeLaunch& a, uint32_t gmax, cudaStream_t s, bool pdl);
// Persistent, cp.async-pipelined expert kernels (moe_pipe.cu) for decode
// batches of at most 32 tokens (bf16 inputs above 8) on moe_mma_supported layouts.
bool moe_pipe_supported(const MoeLaunch& a);
cudaError_t moe_up_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl);
cudaError_t moe_down_pipe_launch(const MoeLaunch& a, cudaStream_t s, bool pdl);
size_t moe_router_smem(uint32_t T, uint32_t H, uint32_t E, uint32_t K);
// Dynamic shared memory the router kernel may use (the 227 KB per-CTA limit
// less its static shared memory, rounded down).
constexpr size_t kRouterSmemLimit = 224 * 1024;
cudaError_t route_topk_launch(const float* logits, uint32_t T, uint32_t E, uint32_t K, uint32_t normalization,
                              float routed_scale, uint32_t* ids, float* w, uint32_t* status, cudaStream_t s,
                              const float* bias = nullptr);

struct Q4MatvecArgs {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* biases;
    uint32_t rows, cols, group;
    const void* x;
    pbmoe_dtype x_dtype;
    void* y;
    pbmoe_dtype y_dtype;
    uint32_t batch;
    // fusions (pbmoe_q4_matvec_fused); zero = off
    const float* norm_w;  // x -> RMSNorm(x) * norm_w (epsilon eps) before the products; f32 x
    float eps;
    const void* residual;  // y = W x + residual ([batch x rows] in y_dtype)
    // a second matrix [rows2 x cols] (same group) on the same x, output y2
    const uint8_t* packed2;
    const uint16_t* scales2;
    const uint16_t* biases2;
    uint32_t rows2;
    void* y2;
    // or a set of up to kQ4MaxMats matrices [rows_i x cols] (same group) on the
    // same x, one launch (pbmoe_q4_matvec_batch); replaces packed/packed2
    uint32_t set_count;
    const struct Q4MatSpec* set;
};
// One matrix of a multi-matrix launch.
struct Q4MatSpec {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* biases;
    uint32_t rows;
    void* y;
};
constexpr uint32_t kQ4MaxMats = 16;
// Returns cudaErrorNotSupported when the shape needs more shared memory than
// a CTA has.
cudaError_t q4_matvec_launch(const Q4MatvecArgs& a, cudaStream_t s);

// ---------------------------------------------------------------- MLA decode (mla.cu)
constexpr uint32_t kMlaMaxBatch = 32;
constexpr uint32_t kMlaCtasPerSm = 2;  // attention CTAs resident per SM (the split plan fills them)

// Per-sequence latent caches, passed by value to the attention kernel.
struct MlaSeqs {
    const uint16_t* c_kv[kMlaMaxBatch];    // bf16 [len x latent]
    const uint16_t* k_rope[kMlaMaxBatch];  // bf16 [len x rope]
    uint32_t len[kMlaMaxBatch];
};

struct MlaLaunch {
    uint32_t batch, nope;
    float scale;
    const void* q;  // [batch x 16 x (nope + 64)], rope part rotated
    pbmoe_dtype q_dtype;
    MlaSeqs seqs;
    const uint16_t* w_uk;  // bf16 [16 x nope x 512]
    const uint16_t* w_uv;  // bf16 [16 x 128 x 512]
    void* out;             // [batch x 16 x 128]
    pbmoe_dtype out_dtype;
    // workspace
    float* qp;       // [batch x 16 x 576] scaled absorbed queries
    float* partial;  // [batch x splits x 16 x 514] per-split (max, sum, O)
    float* ctx;      // [batch x 16 x 512]
    uint32_t split_tokens, splits;
    const struct RopeAppendArgs* rope;  // non-null: the RoPE + cache append done by the absorb launch (f32 q)
};

bool mla_shape_supported(uint32_t heads, uint32_t rope, uint32_t latent, uint32_t v_dim);
size_t mla_smem_bytes();
void mla_plan_splits(const MlaLaunch& a, int num_sms, uint32_t& split_tokens, uint32_t& splits);
uint32_t mla_max_splits(uint32_t max_batch, int num_sms);
cudaError_t mla_decode_launch(const MlaLaunch& a, cudaStream_t s);

// ---------------------------------------------------------------- prefill Q4 GEMM (q4_gemm.cu)
struct Q4GemmArgs {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* biases;
    uint32_t rows, cols, group;  // W [rows x cols] (N x K)
    const void* x16;             // fp16 [m x cols]
    uint32_t m;
    void* y;  // [m x rows]
    pbmoe_dtype y_dtype;
    uint32_t* status;
};
bool q4_gemm_supported(uint32_t N, uint32_t K, uint32_t group);
cudaError_t q4_gemm_launch(const Q4GemmArgs& a, cudaStream_t s);
// fp16 rows for the tensor cores: out[j] = x[rows ? rows[j] : j] for j < nrows
// (K elements per row, bf16 converted or fp16 copied); latches
// PBMOE_DEV_ERR_F16_RANGE / PBMOE_DEV_ERR_EXPERT_ID.
cudaError_t x16_gather_launch(const void* x, bool x_is_f16, const uint32_t* rows, uint32_t nrows, uint32_t x_rows,
                              uint32_t K, void* out, uint32_t* status, cudaStream_t s);

// One projection of every expert (gate, up or down) against routes grouped by
// slot: y[j] = xg16[j] . W_{slot_experts[slot of j]}^T, xg16 the fp16 token
// rows already gathered into grouped order.
struct Q4GroupedArgs {
    const uint8_t* experts;
    uint64_t expert_bytes;
    uint64_t packed_offset, scales_offset, biases_offset;
    uint32_t rows, cols, num_experts;
    const uint32_t* slot_experts;  // [max_unique] expert id of each slot
    const uint32_t* unique_count;  // device scalar
    uint32_t max_unique;
    const uint32_t* groups;  // [unique x 2] (start, count)
    uint32_t routes;
    const void* xg16;  // fp16 [routes x cols], grouped order
    void* y;           // [routes x rows]
    pbmoe_dtype y_dtype;
    uint32_t* status;
};
uint32_t q4_grouped_tile_bound(uint32_t routes, uint32_t max_unique);
bool q4_grouped_supported(uint32_t N, uint32_t K, uint32_t group, uint32_t routes, uint32_t max_unique);
cudaError_t q4_gemm_grouped_launch(const Q4GroupedArgs& a, cudaStream_t s);

// ---------------------------------------------------------------- prefill group plan (prefill_plan.cu)
constexpr uint32_t kPlanMaxExperts = 1024;
struct PrefillPlanArgs {
    const uint32_t* route_ids;  // [rows x top_k]
    uint32_t rows, top_k, num_experts;
    uint32_t* slot_experts;    // [num_experts]: selected ids, ascending
    uint32_t* unique_count;    // device scalar
    uint32_t* route_slots;     // [routes] or null
    uint32_t* source_rows;     // [routes]
    uint32_t* output_indices;  // [routes]
    uint32_t* groups;          // [num_experts x 2]
    uint32_t* status;
};
size_t prefill_plan_smem(uint32_t num_experts);
cudaError_t prefill_plan_launch(const PrefillPlanArgs& a, cudaStream_t s);

// ---------------------------------------------------------------- decode-step glue (step.cu)
struct NormArgs {
    const void* x;
    pbmoe_dtype x_dtype;
    const void* residual;
    void* sum_out;
    pbmoe_dtype sum_dtype;
    const float* weight;
    float epsilon;
    void* out;
    pbmoe_dtype out_dtype;
    uint32_t rows, width, x_stride, residual_stride, sum_stride, out_stride;
};
cudaError_t rms_norm_launch(const NormArgs& a, cudaStream_t s);

struct RopeAppendArgs {
    uint32_t batch, heads, nope, rope, latent;
    float* query;               // [batch x heads x (nope + rope)]
    const float* kv;            // [batch x (latent + rope)]
    const float* latent_norm_w;  // [latent]: the latent part is normalised here (NULL: already normed)
    float eps;
    const uint32_t* positions;  // [batch]
    uint16_t* const* c_kv;      // [batch] cache rows [cache_len x latent]
    uint16_t* const* k_rope;    // [batch] cache rows [cache_len x rope]
    uint32_t cache_len;
    const float2* table;  // [max_positions x rope/2] (cos, sin)
    uint32_t max_positions;
    uint32_t* status;
};
bool rope_append_supported(uint32_t heads, uint32_t rope);
cudaError_t mla_rope_append_launch(const RopeAppendArgs& a, cudaStream_t s);

// ---------------------------------------------------------------- MXFP4 matvec (mxfp4.cu)
struct Mxfp4Args {
    const uint8_t* packed;  // [rows x cols/2] E2M1 nibbles, low nibble = even column
    const uint8_t* scales;  // [rows x cols/32] E8M0
    uint32_t rows, cols, group, batch;
    const void* x;  // [batch x cols]
    pbmoe_dtype x_dtype;
    void* y;  // [batch x rows]
    pbmoe_dtype y_dtype;
    uint32_t* status;
};
bool mxfp4_supported(uint32_t rows, uint32_t cols, uint32_t group, uint32_t batch);
cudaError_t mxfp4_matvec_launch(const Mxfp4Args& a, cudaStream_t s);

// ---------------------------------------------------------------- expert store (expert_store.cu)
// Validated FIXED_Q4_EXPERT_LAYER_V1 slots of experts [expert_begin,
// expert_begin + expert_count) copied to device memory on `stream`
// (synchronised before return); a PBMOE_* status, message in error_buf.
int expert_layer_upload(const char* root, uint32_t layer, const pbmoe_expert_layout* layout, uint32_t expert_begin,
                        uint32_t expert_count, void* device_dst, size_t dst_bytes, cudaStream_t stream,
                        char* error_buf, size_t error_len);

// ---------------------------------------------------------------- vocab head (head.cu)
// logits[t][v] = W[v] . x[t] for the rows [0, vocab) of a (possibly sharded)
// head whose row 0 is global token id `id_base`, then each token's top_k
// candidates (key, id, value) in topk_vocab order. Candidate lists of several
// shards are merged by head_merge_launch.
struct HeadArgs {
    const uint16_t* weight;  // bf16 [vocab x hidden]
    uint32_t vocab, hidden, id_base;
    const void* x;  // [tokens x hidden]
    pbmoe_dtype x_dtype;
    uint32_t tokens, top_k;
    const uint32_t* allowed;  // bitmask over global ids, or null
    float* logits;            // [tokens x vocab] workspace (zeroed here)
    uint32_t* cand_key;       // [tokens x slices x top_k] workspace
    uint32_t* cand_id;
    float* cand_val;
    uint32_t* out_key;  // [tokens x top_k]
    uint32_t* out_id;
    float* out_val;
};
uint32_t head_slices(uint32_t vocab);
bool head_supported(uint32_t vocab, uint32_t hidden, uint32_t tokens, uint32_t top_k);
cudaError_t head_topk_launch(const HeadArgs& a, cudaStream_t s);
// merge `lists` candidate lists of top_k per token (entry r of list l for
// token t at t * tok_stride + l * list_stride + r; lists in id order) into
// the final [tokens x top_k]
cudaError_t head_merge_launch(const uint32_t* in_key, const uint32_t* in_id, const float* in_val, uint32_t tokens,
                              uint32_t lists, size_t tok_stride, size_t list_stride, uint32_t top_k,
                              uint32_t* out_key, uint32_t* out_id, float* out_val, cudaStream_t s);

}  // namespace pbmoe
