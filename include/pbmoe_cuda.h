/*
 * pbmoe_cuda.h — C ABI of the B200 (sm_100a) FlashMoE hot path.
 *
 * This is the drop-in boundary that replaces the Metal execution backend of
 * Jc2k/pb's FlashMoE runtime (src/inference/flashmoe/metal/, driven through
 * MetalExecutionFacade, runtime/mod.rs:648-1416). The runtime's host code keeps
 * its model/scheduler API and calls these entry points instead of encoding
 * Metal command buffers, binding them from Rust with an `extern "C"` block
 * and linking the library from its build script.
 *
 * Conventions
 *  - Plain C: pointers, sizes, enums. No CUDA or torch types; a stream is a
 *    `void*` holding a cudaStream_t (NULL = the legacy default stream).
 *  - Every data pointer is a DEVICE pointer unless the comment says host.
 *  - Every call validates its geometry on the host before launching and
 *    returns a pbmoe_status; the text of the last failure is kept per context
 *    (pbmoe_last_error). Nothing falls back to a CPU path: an unsupported shape
 *    is PBMOE_ERR_UNSUPPORTED, mirroring the reference's
 *    `bail!("FlashMoe unsupported ...")` (docs/flashmoe-architecture-parity-plan.md:22-29).
 *  - Calls are stream-ordered and asynchronous. Errors detected by a kernel
 *    (invalid routing weights, bounded-wait timeouts) are latched in a device
 *    status word that pbmoe_device_status() reads back.
 *  - A context is not thread-safe; use one per engine, as the reference keeps
 *    one FlashMoeEngine per request (`&mut self`).
 *
 * Quantised weight format (shared by every entry point)
 *  - Q4 nibbles, row-major, ceil(cols/2) bytes per row; column c is the low
 *    nibble of byte c/2 when c is even, the high nibble when odd
 *    (math.rs:903-904; equivalently 8 nibbles per little-endian u32,
 *    shaders.metal:58-65).
 *  - Scales and biases: bf16 bits, [rows x ceil(cols/group_size)] row-major
 *    (experts/mod.rs:917-934).
 *  - w = q * scale + bias (math.rs:949).
 */
#ifndef PBMOE_CUDA_H
#define PBMOE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PBMOE_ABI_VERSION 2

#if defined(__GNUC__)
#define PBMOE_API __attribute__((visibility("default")))
#else
#define PBMOE_API
#endif

typedef enum pbmoe_status {
    PBMOE_OK = 0,
    PBMOE_ERR_INVALID_ARGUMENT = -1, /* bad pointer / size / geometry             */
    PBMOE_ERR_UNSUPPORTED = -2,      /* valid in the reference, not built here     */
    PBMOE_ERR_CUDA = -3,             /* a CUDA runtime call failed                 */
    PBMOE_ERR_TIMEOUT = -4,          /* a bounded device or host wait expired      */
    PBMOE_ERR_PEER = -5,             /* an expert-parallel peer failed / is absent */
    PBMOE_ERR_NO_WORKSPACE = -6,     /* pbmoe_reserve was not called or too small  */
    PBMOE_ERR_DEVICE_STATUS = -7     /* a kernel latched an error word             */
} pbmoe_status;

/* Device status bits latched by kernels (pbmoe_device_status). */
#define PBMOE_DEV_ERR_ROUTE_WEIGHTS 0x1u /* selected probabilities not positive-finite */
#define PBMOE_DEV_ERR_EXPERT_ID 0x2u     /* route expert id out of range               */
#define PBMOE_DEV_ERR_PEER_TIMEOUT 0x4u  /* expert-parallel combine wait expired       */
#define PBMOE_DEV_ERR_PIPE_TIMEOUT 0x8u  /* an asynchronous copy wait expired          */
#define PBMOE_DEV_ERR_F16_RANGE 0x10u    /* prefill GEMM input |x| >= 65536 or non-finite */
#define PBMOE_DEV_ERR_POSITION 0x20u     /* decode position past the cache or RoPE table  */
#define PBMOE_DEV_ERR_MXFP4_SCALE 0x40u  /* an E8M0 scale byte 255 (not finite)           */

typedef enum pbmoe_dtype {
    PBMOE_F32 = 0,
    PBMOE_BF16 = 1,
    PBMOE_F16 = 2 /* prefill GEMM activations only */
} pbmoe_dtype;

typedef struct pbmoe_ctx pbmoe_ctx;

/* One Q4 affine matrix [rows x cols]. Replaces Q4MatvecPayload
 * (experts/slots.rs:1172-1199) once its bytes are resident on the device. */
typedef struct pbmoe_q4_tensor {
    const void* packed;      /* rows * ceil(cols/2) bytes                      */
    const uint16_t* scales;  /* rows * ceil(cols/group_size) bf16              */
    const uint16_t* biases;  /* rows * ceil(cols/group_size) bf16              */
    uint32_t rows;
    uint32_t cols;
    uint32_t group_size;
} pbmoe_q4_tensor;

/* How an expert slot's weights are encoded (FixedQ4ExpertEncoding,
 * experts/slots.rs:3-45). */
typedef enum pbmoe_expert_encoding {
    /* AffineBf16: 4-bit q per weight, bf16 scale and bias per group_size
     * columns, w = q * scale + bias (FIXED_Q4_EXPERT_LAYER_V1) */
    PBMOE_EXPERT_AFFINE_Q4 = 0,
    /* MlxMxfp4: E2M1 nibbles, one E8M0 scale byte per 32 columns, no biases
     * (FIXED_MXFP4_EXPERT_LAYER_V1); group_size must be 32 */
    PBMOE_EXPERT_MXFP4 = 1
} pbmoe_expert_encoding;

/* Whole-expert slot layout. Replaces QwenMoeQ4ExpertLayout
 * (model_family.rs:839-1010): nine components in the order gate{W,S,B},
 * up{W,S,B}, down{W,S,B}; gate/up are [intermediate x hidden], down is
 * [hidden x intermediate]. MXFP4 slots have zero-sized bias components. */
typedef struct pbmoe_expert_layout {
    uint64_t component_offsets[9];
    uint64_t expert_bytes; /* slot stride in the expert table */
    uint32_t hidden;
    uint32_t intermediate;
    uint32_t group_size;
    uint32_t encoding;     /* pbmoe_expert_encoding; zero-initialised = affine Q4 */
} pbmoe_expert_layout;

/* Routing weight normalisation (QwenMoeRoutingWeightNormalization,
 * model_family.rs:111-115; applied in scheduler/expert_access.rs:80-133). */
typedef enum pbmoe_route_norm {
    PBMOE_ROUTE_RENORMALIZE_SELECTED = 0,
    PBMOE_ROUTE_DEEPSEEK_RENORMALIZE_WITH_FLOOR = 1
} pbmoe_route_norm;

/* Shapes and policy of one MoE FFN layer (QwenModelConfig fields,
 * model_family.rs:180-470). */
typedef struct pbmoe_moe_config {
    pbmoe_expert_layout layout;
    uint32_t num_experts;        /* experts per layer (E)                    */
    uint32_t top_k;              /* routed experts per token (K), 1..32       */
    uint32_t normalization;      /* pbmoe_route_norm                          */
    float routed_scaling_factor; /* multiplies the normalised weights (1.0)   */
    float norm_epsilon;          /* next-layer RMSNorm epsilon (1e-6)         */
} pbmoe_moe_config;

/* Device-resident weights of one MoE layer. */
typedef struct pbmoe_moe_weights {
    const uint16_t* router_weight;      /* bf16 [E x hidden]                          */
    const uint8_t* experts;             /* E slots, layout.expert_bytes apart          */
    const uint8_t* shared_expert;       /* one slot in the same layout, or NULL        */
    const uint16_t* shared_expert_gate; /* bf16 [hidden] sigmoid gate, or NULL (= 1.0)  */
    /* f32 [hidden] weight of the norm ahead of the router, or NULL. When given,
     * x is the un-normalised hidden state (the residual sum after attention) and
     * the layer routes and runs its experts on bf16(RMSNorm(x) * weight), with
     * config.norm_epsilon: the post-attention norm the reference encodes ahead
     * of the router (CMD2, metal/mod.rs:2864-3012; rms_norm_reduced,
     * shaders.metal:1176-1213), fused into the router kernel. 16-byte aligned. */
    const float* input_norm_weight;
    /* f32 [E] router correction bias, or NULL. When given, the layer routes as
     * GLM/DeepSeek noaux models do (routing_sigmoid_noaux_top_k, math.rs:
     * 788-819; QwenMoeRoutingPlacement::CpuSigmoidNoAuxTopK): experts are
     * selected on sigmoid(logit) + bias with routing_top_k_iter's slot order,
     * and a selected expert's weight is its raw sigmoid(logit), then the
     * config's normalisation and routed_scaling_factor. NULL = softmax top-k.
     * 16-byte aligned. */
    const float* router_correction_bias;
} pbmoe_moe_weights;

/* Optional outputs of pbmoe_moe_layer for inspection and parity checks. Any
 * member may be NULL. */
typedef struct pbmoe_moe_debug {
    float* router_logits;   /* f32 [tokens x E]                        */
    uint32_t* route_ids;    /* u32 [tokens x K], replacement-slot order */
    float* route_weights;   /* f32 [tokens x K], normalised and scaled  */
    float* shared_logit;    /* f32 [tokens]                             */
    /* Host array of 5 cudaEvent_t (as void*), or NULL. When given, event 0 is
     * recorded before the router kernel and event i after kernel i (router,
     * expert gate/up, expert down, combine), the CUDA counterpart of the
     * reference's per-phase timing buckets (FlashMoeTimingBuckets,
     * types.rs:600-640). Recording serialises the four kernels. */
    void* const* phase_events;
    /* bf16 [tokens x hidden]: the normalised layer input when
     * weights->input_norm_weight is given (what the router and experts read). */
    uint16_t* normed_input;
} pbmoe_moe_debug;

/* ---------------------------------------------------------------- context */

/* Create a context on CUDA device `device`. Allocates nothing on the device
 * beyond a status word; call pbmoe_reserve before pbmoe_moe_layer. */
PBMOE_API int pbmoe_init(int device, pbmoe_ctx** out);
PBMOE_API int pbmoe_destroy(pbmoe_ctx* ctx);
/* Text of the last failure on this context (empty when none). Valid until the
 * next call on the context. */
PBMOE_API const char* pbmoe_last_error(const pbmoe_ctx* ctx);
PBMOE_API int pbmoe_abi_version(void);

/* Size the context's device workspace for MoE layers of up to `max_tokens`
 * tokens with this config. Allocation happens here, never on the hot path
 * (the reference recycles pooled Metal buffers, metal/mod.rs:3270-3330). */
PBMOE_API int pbmoe_reserve(pbmoe_ctx* ctx, uint32_t max_tokens, const pbmoe_moe_config* config);
/* Workspace bytes pbmoe_reserve would allocate (host-only arithmetic). */
PBMOE_API size_t pbmoe_moe_workspace_bytes(uint32_t max_tokens, const pbmoe_moe_config* config);

/* Read (and clear when `clear` != 0) the device status word after
 * synchronising `stream`. *out receives PBMOE_DEV_ERR_* bits. */
PBMOE_API int pbmoe_device_status(pbmoe_ctx* ctx, void* stream, uint32_t* out, int clear);

/* Bounded wait for everything queued on `stream` (the CMD3 submission's
 * wait(), metal/mod.rs:3041-3127): PBMOE_OK once the stream is idle,
 * PBMOE_ERR_TIMEOUT if it is still busy after timeout_ms (the work is not
 * cancelled; the call may be repeated), PBMOE_ERR_CUDA if queued work failed.
 * timeout_ms 0 only polls. */
PBMOE_API int pbmoe_sync(pbmoe_ctx* ctx, void* stream, uint32_t timeout_ms);

/* Fill *out with the reference's fixed whole-expert layout
 * (QwenMoeQ4ExpertLayout::fixed_bf16, model_family.rs:954-1010). Host-only. */
PBMOE_API int pbmoe_fixed_q4_layout(uint32_t hidden, uint32_t intermediate, uint32_t group_size,
                          pbmoe_expert_layout* out);

/* The fixed MXFP4 whole-expert layout (QwenMoeQ4ExpertLayout::fixed_mxfp4,
 * model_family.rs:846-952): per projection the E2M1 nibbles then one E8M0
 * byte per group, the bias components zero-sized; encoding
 * PBMOE_EXPERT_MXFP4. The MoE layer runs such slots with group_size 32, the
 * only group the reference builds them with (experts/slots.rs:67-80).
 * Host-only. */
PBMOE_API int pbmoe_fixed_mxfp4_layout(uint32_t hidden, uint32_t intermediate, uint32_t group_size,
                                       pbmoe_expert_layout* out);

/* ---------------------------------------------------------------- kernels */

/* y[b, r] = sum_c (q[r,c] * scale + bias) * x[b, c] for b < batch.
 * x: [batch x cols] in x_dtype; y: [batch x rows] in y_dtype; fp32 accumulate.
 * Replaces q4_fma_matvec_bf16_scale_bias (shaders.metal:164-199, encoded by
 * MetalScheduledCmd3Builder::encode_q4_matvec, metal/mod.rs:4871-4916) and the
 * batched resident form (MetalExecutionFacade::resident_mmap_matvec_batch,
 * runtime/mod.rs:1184). */
PBMOE_API int pbmoe_q4_matvec(pbmoe_ctx* ctx, const pbmoe_q4_tensor* w, const void* x, pbmoe_dtype x_dtype,
                    void* y, pbmoe_dtype y_dtype, uint32_t batch, void* stream);

/* Fused decode projections of one layer, one launch:
 *   y[0][b] = W0 . n(x[b])  (+ residual[b])     and, when w[1] != NULL,
 *   y[1][b] = W1 . n(x[b])
 * where n(x) = x, or RMSNorm(x) * input_norm_weight (1/sqrt(mean(x^2) +
 * epsilon)) when input_norm_weight is given. It folds the separate dispatches
 * of the reference's MLA input projection chain and attention output
 * (execute_glm_mla_input_projection_chain, metal/qwen_execution.rs:289-480,
 * and mla_attention_output_values, runtime/mod.rs:2779-2940) into one kernel
 * each: q_a and kv_a read the same normed hidden state (two matrices); q_b
 * reads RMSNorm(q_a) (rms_norm_reduced, shaders.metal:1176-1213, as its
 * prologue); o_proj adds the residual stream (its epilogue). Both matrices
 * share cols and group_size. input_norm_weight (f32 [cols], 16-byte aligned)
 * needs f32 x; residual ([batch x w[0].rows] in y_dtype) needs w[1] == NULL.
 * The per-element fallback of pbmoe_q4_matvec has no fused forms: shapes that
 * need it are PBMOE_ERR_UNSUPPORTED here. */
typedef struct pbmoe_q4_fused_args {
    const pbmoe_q4_tensor* w[2]; /* w[0] required, w[1] optional */
    void* y[2];                  /* y[i]: [batch x w[i]->rows] in y_dtype */
    const void* x;               /* [batch x cols] in x_dtype */
    pbmoe_dtype x_dtype;
    pbmoe_dtype y_dtype;
    uint32_t batch;
    const float* input_norm_weight;
    float epsilon;
    const void* residual;
} pbmoe_q4_fused_args;
PBMOE_API int pbmoe_q4_matvec_fused(pbmoe_ctx* ctx, const pbmoe_q4_fused_args* args, void* stream);

/* A batch of resident projections on one input: y[i] = W_i x for the
 * `count` matrices of `weights` (all with the same cols and group_size; rows
 * may differ), y[i] [batch x weights[i].rows] in y_dtype. Replaces
 * resident_mmap_matvec_batch (runtime/mod.rs:1184), which encodes every
 * projection of the batch over the same input buffer: here up to 16 matrices
 * share one launch (more run as further launches of 16), so the projections
 * stream their weights back to back instead of paying a launch each. Needs
 * the fast or tensor-core path (cols a multiple of 32, group a power of two
 * >= 32, 16-byte aligned rows and x): other shapes are PBMOE_ERR_UNSUPPORTED
 * (use pbmoe_q4_matvec per matrix). Results equal pbmoe_q4_matvec's on each
 * matrix. */
PBMOE_API int pbmoe_q4_matvec_batch(pbmoe_ctx* ctx, const pbmoe_q4_tensor* weights, uint32_t count, const void* x,
                                    pbmoe_dtype x_dtype, void* const* y, pbmoe_dtype y_dtype, uint32_t batch,
                                    void* stream);

/* Routing on given logits: logits f32 [tokens x E] -> route_ids u32 [tokens x K]
 * (replacement-slot order of routing_top_k_iter, math.rs:746-765) and
 * route_weights f32 [tokens x K] (routing_softmax_top_k, math.rs:771-783, then
 * the config's normalisation x routed_scaling_factor,
 * scheduler/expert_access.rs:80-133). Replaces the CPU RoutingSoftmaxTopK stage
 * (capabilities.rs:21-31) that follows the router read-back
 * (metal/qwen_execution.rs:1036-1050). */
PBMOE_API int pbmoe_route_topk(pbmoe_ctx* ctx, const float* logits, uint32_t tokens, uint32_t num_experts,
                     uint32_t top_k, uint32_t normalization, float routed_scaling_factor,
                     uint32_t* route_ids, float* route_weights, void* stream);

/* Sigmoid/noaux routing on given logits (routing_sigmoid_noaux_top_k,
 * math.rs:788-819, the CpuSigmoidNoAuxTopK stage, capabilities.rs:96): per
 * token, experts selected on sigmoid(logit) + correction_bias[e] (f32 [E],
 * device) in routing_top_k_iter's slot order; route_weights = the selected
 * experts' raw sigmoid(logit), then `normalization` x routed_scaling_factor
 * (scheduler/expert_access.rs:80-133). The sigmoid is computed as the
 * reference's f32 arithmetic with a correctly rounded exp, so ids match it
 * bit for bit on identical logits. */
PBMOE_API int pbmoe_route_sigmoid_noaux(pbmoe_ctx* ctx, const float* logits, const float* correction_bias,
                                        uint32_t tokens, uint32_t num_experts, uint32_t top_k,
                                        uint32_t normalization, float routed_scaling_factor, uint32_t* route_ids,
                                        float* route_weights, void* stream);

/* One MoE FFN decode layer for `tokens` tokens (1..max_tokens of pbmoe_reserve):
 *   router logits -> top-k routing -> per-route SwiGLU expert on Q4 weights
 *   -> out = residual + sum_k w_k * expert_k(x) + sigmoid(shared_gate . x) * shared(x)
 * and, when next_norm_weight != NULL, next_normed = RMSNorm(out) * weight.
 * x: [tokens x hidden] in x_dtype; residual (nullable), out and next_normed in
 * out_dtype. Replaces MetalExecutionFacade::submit_scheduled_expert_command
 * (runtime/mod.rs:922-961 -> MetalScheduledCmd3Builder::encode_and_submit,
 * metal/mod.rs:4289-4470) together with the router projection and CPU top-k
 * that precede it (runtime/mod.rs:1065, math.rs:771). */
PBMOE_API int pbmoe_moe_layer(pbmoe_ctx* ctx, const pbmoe_moe_config* config, const pbmoe_moe_weights* weights,
                    const void* x, pbmoe_dtype x_dtype, const void* residual, void* out,
                    pbmoe_dtype out_dtype, uint32_t tokens, const float* next_norm_weight,
                    void* next_normed, const pbmoe_moe_debug* debug, void* stream);

/* pbmoe_moe_layer without any device allocation. No counterpart in the
 * reference: it exists for hosts that cannot call cudaMalloc at run time (an
 * engine whose own arena owns all device memory, code running under CUDA
 * graph capture, loops that must not risk the synchronisation an allocation
 * can cause) and therefore cannot create a pbmoe_ctx either.
 *
 * Same arithmetic, arguments and checks as pbmoe_moe_layer, with no context.
 * Its scratch is a fixed PBMOE_STATIC_SCRATCH_BYTES device array inside the
 * library, present on every GPU where the library's kernels are loaded until
 * the process exits; a call fits when 256 + pbmoe_moe_workspace_bytes(tokens,
 * config) <= PBMOE_STATIC_SCRATCH_BYTES (at most 29 tokens at hidden 2048 /
 * 512 experts / top-10 / intermediate 512), larger calls return
 * PBMOE_ERR_UNSUPPORTED. It launches exactly pbmoe_moe_layer's kernels (one
 * launch for up to 32 tokens, which is every call that fits). The array's
 * device address is looked up on the first call on each device (the calling
 * thread's current device): make that first call before any stream capture.
 * All calls share the array: calls that may
 * overlap on the GPU race and must be serialised by the caller.
 * device_status (nullable, device u32) receives PBMOE_DEV_ERR_* bits; when it
 * is NULL the bits land in the shared array, which the next call clears, so
 * errors detected on the device are not observable. The message of a failed
 * call goes to error_buf (nullable). */
#define PBMOE_STATIC_SCRATCH_BYTES (4u << 20)
PBMOE_API int pbmoe_moe_layer_static(const pbmoe_moe_config* config, const pbmoe_moe_weights* weights,
                                     const void* x, pbmoe_dtype x_dtype, const void* residual, void* out,
                                     pbmoe_dtype out_dtype, uint32_t tokens, const float* next_norm_weight,
                                     void* next_normed, uint32_t* device_status, char* error_buf,
                                     size_t error_len, void* stream);

/* ---------------------------------------------------------------- MLA decode */

/* Shapes of MLA absorbed decode attention (MlaAttentionLayout,
 * weights/mod.rs:651-664). The tensor-core kernels take heads 16, rope 64,
 * latent 512, v 128 and nope <= 128; other shapes are PBMOE_ERR_UNSUPPORTED. */
typedef struct pbmoe_mla_config {
    uint32_t heads;
    uint32_t nope_dim;
    uint32_t rope_dim;
    uint32_t latent_dim; /* kv_lora_rank */
    uint32_t v_dim;
    float softmax_scale; /* 0 = 1/sqrt(nope_dim + rope_dim) (weights/store.rs:1262) */
} pbmoe_mla_config;

/* One decode step of `batch` sequences, each attending over its own latent
 * cache (KvCache::mla_records, state/kv_cache.rs:414-450). */
typedef struct pbmoe_mla_args {
    uint32_t batch;                 /* 1..32                                             */
    const uint32_t* seq_lens;       /* HOST array [batch]: cache length of each sequence */
    const void* query;              /* [batch x heads x (nope + rope)] in query_dtype;
                                       the rope part already rotated                     */
    pbmoe_dtype query_dtype;
    const uint16_t* const* c_kv;    /* HOST array [batch] of device pointers:
                                       bf16 [seq_len x latent], 16-byte aligned          */
    const uint16_t* const* k_rope;  /* HOST array [batch] of device pointers:
                                       bf16 [seq_len x rope], rotated at write,
                                       16-byte aligned                                   */
    const uint16_t* w_uk;           /* bf16 [heads x nope x latent] (absorbed into q),
                                       16-byte aligned                                   */
    const uint16_t* w_uv;           /* bf16 [heads x v x latent], 16-byte aligned        */
    void* out;                      /* [batch x heads x v] in out_dtype                  */
    pbmoe_dtype out_dtype;
} pbmoe_mla_args;

/* Size the context's MLA workspace for batches of up to `max_batch`
 * sequences (any cache length). Allocation happens here, never in
 * pbmoe_mla_decode. */
PBMOE_API int pbmoe_mla_reserve(pbmoe_ctx* ctx, const pbmoe_mla_config* config, uint32_t max_batch);

/* out[b, h, :] = W_UV[h] . sum_t softmax_t(s_t) c_kv_b[t] with
 * s_t = ((W_UK[h]^T q_nope[b, h]) . c_kv_b[t] + q_rope[b, h] . k_rope_b[t]) * scale.
 * Replaces MetalExecutionFacade::resident_glm_mla_absorbed_attention /
 * resident_glm_mla_fused_attention (runtime/mod.rs:1327-1403, Metal kernels
 * glm_mla_absorbed_scores / glm_mla_softmax / glm_mla_context,
 * shaders.metal:1603-1682) and the CPU mla_absorbed_attention
 * (weights/store.rs:1179-1327) with bf16 W_UK / W_UV. */
PBMOE_API int pbmoe_mla_decode(pbmoe_ctx* ctx, const pbmoe_mla_config* config, const pbmoe_mla_args* args,
                               void* stream);

/* ---------------------------------------------------------------- prefill */

/* Size the context's prefill workspace: fp16 token rows for the tensor-core
 * GEMMs, max_rows x max_cols (pbmoe_q4_gemm with bf16 x: m rows;
 * pbmoe_q4_gemm_grouped: routes rows, the gathered rows in grouped order).
 * Allocation happens here, never in the GEMM calls; a dense GEMM on fp16 x
 * needs no workspace. */
PBMOE_API int pbmoe_prefill_reserve(pbmoe_ctx* ctx, uint32_t max_rows, uint32_t max_cols);

/* Y[m, r] = sum_c X[m, c] * (q[r,c] * scale + bias) for a dense Q4 weight:
 * X [m x cols] bf16 or fp16 (rows 16-byte aligned), Y [m x rows] in y_dtype
 * (f32 or bf16), fp32 accumulation on the tensor cores (tcgen05). Operands are
 * fp16: each weight is dequantised once (q * s + b, one fp16 rounding) and a
 * bf16 x converts exactly into the context's workspace (pbmoe_prefill_reserve);
 * an x entry of magnitude >= 65536 or non-finite latches
 * PBMOE_DEV_ERR_F16_RANGE (pbmoe_device_status).
 * Replaces the batched prefill matvec q4_mmap_fma_matvec_batch_bf16_scale_bias
 * (shaders.metal:973-1057, q4_mmap_fma_row_bf16_pair :768-866) as encoded by
 * encode_layer_major_q4_matrix_from_buffer (metal/mod.rs:4201-4275) for one
 * matrix. Needs group_size 64 and cols a multiple of 512 (whole 16-byte runs
 * of eight group scales per row) up to 3072 (the per-tile scale buffers stay
 * in shared memory); packed, scales, biases, x and y 16-byte aligned. */
PBMOE_API int pbmoe_q4_gemm(pbmoe_ctx* ctx, const pbmoe_q4_tensor* w, const void* x, pbmoe_dtype x_dtype,
                            void* y, pbmoe_dtype y_dtype, uint32_t m, void* stream);

/* Layer-major grouping of a prefill chunk's routes, on the device.
 * route_ids: device u32 [rows x top_k] (each row's routed experts).
 * Outputs (device): slot_experts [num_experts] = the selected experts in
 * ascending id order (slot s = s-th selected expert), *unique_count = their
 * number, route_slots [routes] (nullable) = the slot of each route,
 * source_rows [routes] / output_indices [routes] / groups [num_experts x 2]
 * as qwen_layer_major_group_plan (metal/mod.rs:3197-3233) returns them, slot
 * order from ScheduledLayerMajorExperts (scheduler/mod.rs:720-765). An expert
 * id >= num_experts latches PBMOE_DEV_ERR_EXPERT_ID and sets *unique_count
 * to 0. num_experts <= 1024. */
PBMOE_API int pbmoe_prefill_group_plan(pbmoe_ctx* ctx, const uint32_t* route_ids, uint32_t rows, uint32_t top_k,
                                       uint32_t num_experts, uint32_t* slot_experts, uint32_t* unique_count,
                                       uint32_t* route_slots, uint32_t* source_rows, uint32_t* output_indices,
                                       uint32_t* groups, void* stream);

/* One projection (gate, up or down) of every expert in an expert table. */
typedef struct pbmoe_q4_expert_matrix {
    const uint8_t* experts; /* slot table, expert_bytes apart (16-byte aligned) */
    uint64_t expert_bytes;
    uint64_t packed_offset; /* component offsets of this projection in a slot    */
    uint64_t scales_offset;
    uint64_t biases_offset;
    uint32_t num_experts;
    uint32_t rows, cols, group_size; /* per-expert matrix [rows x cols]         */
} pbmoe_q4_expert_matrix;

/* Grouped GEMM of the layer-major prefill: for every slot s with group
 * (start, count) and every j < count,
 *   y[start + j, :] = W_{slot_experts[s]} . x[source_rows[start + j], :].
 * The row gather of qwen_layer_major_gather (shaders.metal:1743-1754) is
 * fused with the fp16 conversion; y stays in grouped order like the
 * reference's per-group matrix outputs (encode_and_execute_layer_major,
 * metal/mod.rs:3334-3600). Plan arrays are device memory, as written by
 * pbmoe_prefill_group_plan; max_unique bounds *unique_count (the grid is
 * sized from routes and max_unique, so no read-back is needed). x [x_rows x
 * cols] bf16 or fp16, gathered into grouped order in the prefill workspace
 * (routes x cols fp16, pbmoe_prefill_reserve); a source row >= x_rows latches
 * PBMOE_DEV_ERR_EXPERT_ID. y [routes x rows] in y_dtype. */
PBMOE_API int pbmoe_q4_gemm_grouped(pbmoe_ctx* ctx, const pbmoe_q4_expert_matrix* w, const uint32_t* slot_experts,
                                    const uint32_t* unique_count, const uint32_t* groups,
                                    const uint32_t* source_rows, uint32_t routes, uint32_t max_unique,
                                    const void* x, pbmoe_dtype x_dtype, uint32_t x_rows, void* y,
                                    pbmoe_dtype y_dtype, void* stream);

/* ---------------------------------------------------------------- expert parallelism */

/* The reference runs on one device (no expert parallelism); this extends its
 * decode layer (encode_expert_phase, metal/mod.rs:4289-4470, and the combine
 * combine_expert_phase, shaders.metal:1723-1741) to experts sharded over
 * `world` GPUs of one node. Activations, router and shared expert are
 * replicated, so dispatch is local: every rank routes every token
 * (deterministically, identically) and runs the routes of its own experts;
 * the combine sums the ranks' partial outputs over NVLink peer memory in a
 * one-shot exchange (no multicast, bounded waits). */

/* Rank r of `world` owns experts [floor(r*E/world), floor((r+1)*E/world)).
 * Host-only. */
PBMOE_API int pbmoe_ep_expert_range(uint32_t num_experts, uint32_t rank, uint32_t world, uint32_t* begin,
                                    uint32_t* count);

#define PBMOE_EP_HANDLE_BYTES 64

/* Allocate this rank's exchange buffer (receive slots of every rank's partial
 * outputs for up to max_tokens tokens of `hidden` values, double-buffered,
 * plus epoch flags), zeroed. world <= 8. */
PBMOE_API int pbmoe_ep_reserve(pbmoe_ctx* ctx, uint32_t rank, uint32_t world, uint32_t max_tokens, uint32_t hidden);
/* The exchange buffer's CUDA IPC handle (PBMOE_EP_HANDLE_BYTES bytes) for the
 * other ranks' processes. */
PBMOE_API int pbmoe_ep_ipc_handle(pbmoe_ctx* ctx, void* handle);
/* Map every rank's exchange buffer: `handles` holds world handles in rank
 * order (this rank's own entry is ignored). */
PBMOE_API int pbmoe_ep_open_peers(pbmoe_ctx* ctx, const void* handles);
/* Same, for ranks driven from one process: device pointers of every rank's
 * exchange buffer in rank order (peer access already enabled by the caller;
 * NULL entries are left unmapped). */
PBMOE_API int pbmoe_ep_set_peers(pbmoe_ctx* ctx, void* const* buffers);
/* This rank's exchange buffer (device pointer), for pbmoe_ep_set_peers. */
PBMOE_API void* pbmoe_ep_buffer(pbmoe_ctx* ctx);

typedef struct pbmoe_ep_shard {
    uint32_t expert_begin; /* first expert id this rank owns                  */
    uint32_t expert_count; /* experts owned (weights->experts holds exactly   */
                           /* these slots, expert_begin first)                */
    uint32_t timeout_us;   /* bound of the wait for peers (0 = 2 s)           */
} pbmoe_ep_shard;

/* One MoE decode layer, expert-parallel. Every rank calls it with the same
 * inputs in the same order. weights->experts is this rank's shard;
 * weights->shared_expert (and its gate) is given on exactly one rank. Output
 * (and next_normed) is the full layer, identical on every rank. A peer that
 * does not arrive within the timeout latches PBMOE_DEV_ERR_PEER_TIMEOUT
 * (pbmoe_device_status) and its partial counts as zero. debug (nullable) is
 * pbmoe_moe_layer's: router logits, every token's route ids and weights (the
 * same on every rank), the normalised input; phase_events is not taken here. */
PBMOE_API int pbmoe_ep_moe_layer(pbmoe_ctx* ctx, const pbmoe_moe_config* config, const pbmoe_moe_weights* weights,
                                 const pbmoe_ep_shard* shard, const void* x, pbmoe_dtype x_dtype, const void* residual,
                                 void* out, pbmoe_dtype out_dtype, uint32_t tokens, const float* next_norm_weight,
                                 void* next_normed, const pbmoe_moe_debug* debug, void* stream);

/* The MoE decode layer on HOST rows, as the reference's facade takes them
 * (submit_scheduled_expert_command, runtime/mod.rs:922-961: normed and
 * residual as host slices; the submission's wait, metal/mod.rs:3041-3127,
 * hands back the host output): x and residual are copied into device rows
 * owned by the context (sized by pbmoe_reserve), the layer runs, and out is
 * copied back, all ordered on `stream` (synchronise it before reading out;
 * pinned host memory makes the copies asynchronous). Page-locked residual
 * and out buffers the device can address (cudaHostAlloc, cudaHostRegister;
 * 16-byte aligned) are not copied: the layer's last kernel reads the
 * residual and writes out in place. No next-layer norm. */
PBMOE_API int pbmoe_moe_layer_host(pbmoe_ctx* ctx, const pbmoe_moe_config* config, const pbmoe_moe_weights* weights,
                                   const void* x, pbmoe_dtype x_dtype, const void* residual, void* out,
                                   pbmoe_dtype out_dtype, uint32_t tokens, void* stream);

/* ---------------------------------------------------------------- vocab head
 * The LM head of sample_from_hidden (runtime/generation.rs:2200-2227):
 * lm_head_raw_top_candidates_with_metal(_masked) (weights/store.rs:1622-1680)
 * -> MetalResidentTopKBuilder::execute_with_allowed_tokens / encode_and_read
 * (metal/mod.rs:2661-2800), i.e. the resident bf16 projection
 * (dense_mmap_fma_matvec_bf16, shaders.metal:1059-1075) and topk_vocab
 * (shaders.metal:1796-1831), for up to 32 tokens per call.
 *
 * A head may be one vocabulary shard: rows [0, vocab) of `weight` are the
 * global token ids [id_base, id_base + vocab). */
typedef struct pbmoe_head {
    const uint16_t* weight; /* bf16 [vocab x hidden], device */
    uint32_t vocab;
    uint32_t hidden; /* a multiple of 512 */
    uint32_t id_base;
} pbmoe_head;

/* Workspace for pbmoe_head_topk: logits and per-slice candidate lists for
 * up to max_tokens tokens (<= 32), vocab rows and top_k <= max_top_k (<= 256). */
PBMOE_API int pbmoe_head_reserve(pbmoe_ctx* ctx, uint32_t max_tokens, uint32_t vocab, uint32_t max_top_k);

/* Per token t: logits = weight . x[t] (f32 accumulate), then the top_k
 * candidates in topk_vocab order: value descending, the lower token id first
 * among equal values, non-finite logits as -inf, tokens whose bit in
 * `allowed` (device bitmask over global ids, or NULL for all) is clear never
 * chosen, and slots past the allowed tokens (0, -inf). The reference first
 * clamps top_k to the vocabulary (execute_with_allowed_tokens); here top_k is
 * the row length of the outputs, slots past vocab being (0, -inf).
 * out_ids/out_values [tokens x top_k] device. out_keys (optional, [tokens x
 * top_k] u32) receives the candidates' ordering keys for pbmoe_head_merge;
 * out_logits (optional, [tokens x vocab] f32) receives the logits. */
PBMOE_API int pbmoe_head_topk(pbmoe_ctx* ctx, const pbmoe_head* head, const void* x, pbmoe_dtype x_dtype,
                              uint32_t tokens, uint32_t top_k, const uint32_t* allowed, uint32_t* out_ids,
                              float* out_values, uint32_t* out_keys, float* out_logits, void* stream);

/* Merge the candidate lists of `lists` vocabulary shards (keys/ids/values as
 * [lists][tokens][top_k], shards in id order, e.g. gathered from every rank)
 * into each token's final top_k (out_ids/out_values [tokens x top_k]). */
PBMOE_API int pbmoe_head_merge(pbmoe_ctx* ctx, const uint32_t* keys, const uint32_t* ids, const float* values,
                               uint32_t lists, uint32_t tokens, uint32_t top_k, uint32_t* out_ids,
                               float* out_values, void* stream);

/* ---------------------------------------------------------------- MXFP4
 * An MXFP4 matrix [rows x cols]: E2M1 nibbles row-major (low nibble = even
 * column; magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6, bit 3 the sign) and one E8M0
 * scale byte per 32 columns (2^(e-127); e = 0 is 2^-127), the GLM-5.2 expert
 * format (FIXED_MXFP4_EXPERT_LAYER_V1, experts/mod.rs:49). */
typedef struct pbmoe_mxfp4_tensor {
    const void* packed;    /* [rows x cols/2], 16-byte aligned rows */
    const uint8_t* scales; /* [rows x cols/group]                   */
    uint32_t rows, cols;   /* cols a multiple of 32                 */
    uint32_t group_size;   /* 32                                    */
} pbmoe_mxfp4_tensor;

/* y[t] = W x[t] for `batch` tokens (x bf16 or f32 [batch x cols], y [batch x
 * rows]), f32 accumulate: mxfp4_fma_matvec_e8m0 (shaders.metal:200-298) /
 * mxfp4_fma_matvec_with_group_size (experts/slots.rs:1239-1287). A scale
 * byte 255, where the reference bails, latches PBMOE_DEV_ERR_MXFP4_SCALE. */
PBMOE_API int pbmoe_mxfp4_matvec(pbmoe_ctx* ctx, const pbmoe_mxfp4_tensor* w, const void* x, pbmoe_dtype x_dtype,
                                 void* y, pbmoe_dtype y_dtype, uint32_t batch, void* stream);

/* ---------------------------------------------------------------- expert store
 * The fixed-Q4 expert layer store a pb expert cache holds
 * (FIXED_Q4_EXPERT_LAYER_V1, experts/mod.rs:44-50): root/layer_NN.json
 * (ExpertLayerPackMetadata, experts/mod.rs:306-454) and root/layer_NN.bin,
 * expert e's slot at e * expert_size (experts/store.rs:1154-1158) in the
 * QwenMoeQ4ExpertLayout byte image (model_family.rs:954-1010). The metadata is
 * validated as ExpertLayerPackMetadata::validate does (experts/mod.rs:372-429)
 * and every requested expert's records against `layout`; slot bytes are used
 * as stored. A FIXED_MXFP4_EXPERT_LAYER_V1 layer (experts/mod.rs:49) is read
 * as stored too, with a layout from pbmoe_fixed_mxfp4_layout; its records are
 * not checked, as the reference resolves it from the pack-level metadata
 * alone. A PBQ4EXPERT_LAYER_V1/V2 layer (a variable-length pack per slot:
 * experts/mod.rs:546-653) is read as the fixed-Q4 images the reference's
 * upgrade writes (experts/slots.rs:984-1113; f32 scales rounded to bf16).
 * This replaces the per-token pread of expert slots
 * (scheduler/mod.rs:662, :808) with one load into the HBM-resident table that
 * pbmoe_moe_weights.experts points at.
 *
 * pbmoe_expert_layer_read: into host memory (no device, no context);
 * the message of a failure goes to error_buf. */
PBMOE_API int pbmoe_expert_layer_read(const char* root, uint32_t layer, const pbmoe_expert_layout* layout,
                                      uint32_t expert_begin, uint32_t expert_count, void* host_dst,
                                      size_t dst_bytes, char* error_buf, size_t error_len);
/* pbmoe_expert_layer_load: into device memory (dst_bytes >= expert_count *
 * layout->expert_bytes), staged through pinned host buffers on `stream`;
 * returns once the copies are complete. For expert parallelism a rank loads
 * its own range (pbmoe_ep_expert_range). */
PBMOE_API int pbmoe_expert_layer_load(pbmoe_ctx* ctx, const char* root, uint32_t layer,
                                      const pbmoe_expert_layout* layout, uint32_t expert_begin,
                                      uint32_t expert_count, void* device_dst, size_t dst_bytes, void* stream);

/* ---------------------------------------------------------------- decode-step glue
 * Row RMSNorm, optionally fused with the residual add: s = x (+ residual);
 * sum_out (optional) receives s; out = s * 1/sqrt(mean(s^2) + epsilon) *
 * weight. Covers rms_norm_reduced (shaders.metal:1176-1213) on q_a and on the
 * latent part of kv_a in the MLA input projection chain
 * (metal/qwen_execution.rs:405-437; row stride 576, width 512 there) and the
 * residual add + post-attention norm ahead of the router (CMD2,
 * metal/mod.rs:2864-3012). Strides are in elements; out may alias x. */
typedef struct pbmoe_norm_args {
    const void* x;
    pbmoe_dtype x_dtype; /* f32 or bf16; residual has the same dtype */
    const void* residual;
    void* sum_out;
    pbmoe_dtype sum_dtype;
    const float* weight; /* [width] or NULL (no weight) */
    float epsilon;
    void* out;
    pbmoe_dtype out_dtype;
    uint32_t rows, width;
    uint32_t x_stride, residual_stride, sum_stride, out_stride;
} pbmoe_norm_args;
PBMOE_API int pbmoe_rms_norm(pbmoe_ctx* ctx, const pbmoe_norm_args* args, void* stream);

/* Cos/sin table of apply_rotary_interleaved_to_split_half (math.rs:822-846)
 * for positions [0, max_positions): f64 angles position * theta^(-2p/rope),
 * cast to f32, as the reference builds them (runtime/mod.rs:2825-2836). */
PBMOE_API int pbmoe_rope_reserve(pbmoe_ctx* ctx, uint32_t max_positions, uint32_t rope_dim, double theta);

/* For each of `batch` tokens: RoPE (interleaved pairs -> split halves) on the
 * rope part of every head of `query` (f32 [batch x heads x (nope + rope)], in
 * place) and on the rope part of `kv` (f32 [batch x (latent + rope)]), then
 * the latent row (bf16) and the rotated key row (bf16) written at the token's
 * position of its cache (KvCache::record_mla_kv, state/kv_cache.rs:414-450;
 * the rotation call sites are runtime/mod.rs:2896-2913). With
 * latent_norm_weight (f32 [latent]) the latent part is the kv_a output before
 * its norm, and the row written is RMSNorm(latent) * weight (epsilon): the
 * chain's second rms_norm_reduced (metal/qwen_execution.rs:405-437) fused
 * here; NULL = the latent part is already normed. positions: DEVICE u32
 * [batch]; c_kv / k_rope: DEVICE arrays [batch] of bf16 cache pointers
 * ([cache_len x latent], [cache_len x rope]). A position >= cache_len or
 * outside the RoPE table latches PBMOE_DEV_ERR_POSITION and writes nothing for
 * that token. */
PBMOE_API int pbmoe_mla_rope_append(pbmoe_ctx* ctx, const pbmoe_mla_config* config, uint32_t batch, float* query,
                                    const float* kv, const float* latent_norm_weight, float epsilon,
                                    const uint32_t* positions, uint16_t* const* c_kv, uint16_t* const* k_rope,
                                    uint32_t cache_len, void* stream);

/* pbmoe_mla_rope_append followed by pbmoe_mla_decode on the same tokens, in
 * one launch fewer: the RoPE rotation and the cache append run inside the
 * decode's first kernel (the query absorb), so a decode step's chain
 * (runtime/mod.rs:2896-2913 then resident_glm_mla_absorbed_attention,
 * runtime/mod.rs:1327-1403) loses one dependent launch. Same results as the
 * two calls: args->query (f32 only) is rotated in place, the latent and key
 * rows are written at each token's position (kv, latent_norm_weight,
 * epsilon, positions, c_kv_rows, k_rope_rows, cache_len as in
 * pbmoe_mla_rope_append; c_kv_rows / k_rope_rows are its DEVICE arrays of
 * cache row pointers, args->c_kv / args->k_rope the HOST arrays of the same
 * caches), then the attention reads every sequence's args->seq_lens rows,
 * the appended one included. A sequence's attended rows other than its own
 * appended row must not be rows another sequence of the call appends (the
 * attention may read them while the append runs). */
PBMOE_API int pbmoe_mla_append_decode(pbmoe_ctx* ctx, const pbmoe_mla_config* config, const pbmoe_mla_args* args,
                                      const float* kv, const float* latent_norm_weight, float epsilon,
                                      const uint32_t* positions, uint16_t* const* c_kv_rows,
                                      uint16_t* const* k_rope_rows, uint32_t cache_len, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* PBMOE_CUDA_H */
