// capi.cu — the extern "C" boundary (include/pbmoe_cuda.h): context, argument
// validation, workspace ownership and launches. Every entry point validates
// geometry on the host first and never falls back to a CPU path.

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <chrono>
#include <string>
#include <thread>
#include <vector>

#include "kernels.h"
#include "q4_rows.cuh"

struct pbmoe_ctx {
    int device = 0;
    uint32_t* status = nullptr;  // device status word
    void* ws_base = nullptr;     // MoE workspace
    size_t ws_bytes = 0;
    uint32_t ws_tokens = 0, ws_E = 0, ws_K = 0, ws_H = 0, ws_I = 0;
    void* mla_base = nullptr;  // MLA decode workspace
    size_t mla_bytes = 0;
    uint32_t mla_batch = 0;
    void* x16_base = nullptr;  // prefill fp16 activation image
    size_t x16_elems = 0;
    void* io_base = nullptr;  // device rows of pbmoe_moe_layer_host: x, residual, out
    size_t io_bytes = 0;
    void* ep_base = nullptr;  // expert-parallel exchange buffer
    size_t ep_bytes = 0;
    uint32_t ep_rank = 0, ep_world = 0, ep_max_tokens = 0, ep_hidden = 0;
    void* ep_peer[pbmoe::kMaxEpRanks] = {};
    bool ep_peer_ipc[pbmoe::kMaxEpRanks] = {};  // mapped through CUDA IPC (closed at destroy)
    float2* rope_table = nullptr;  // [rope_positions x rope_dim/2] (cos, sin)
    uint32_t rope_positions = 0, rope_dim = 0;
    void* head_base = nullptr;  // vocab head: logits, slice candidates, key scratch
    size_t head_bytes = 0;
    uint32_t head_tokens = 0, head_vocab = 0, head_k = 0;
    int num_sms = 0;
    std::string last_error;
};

namespace {

int fail(pbmoe_ctx* ctx, int code, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return code;
}

int cuda_fail(pbmoe_ctx* ctx, cudaError_t e, const char* what) {
    return fail(ctx, PBMOE_ERR_CUDA, "FlashMoe CUDA %s failed: %s", what, cudaGetErrorString(e));
}

// Make `ctx->device` current for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool aligned(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared checks (pbmoe::moe_check_config) with the message into the context.
int check_moe_config(pbmoe_ctx* ctx, const pbmoe_moe_config* c) {
    char msg[512];
    const int rc = pbmoe::moe_check_config(c, msg, sizeof msg);
    return rc == PBMOE_OK ? rc : fail(ctx, rc, "%s", msg);
}

}  // namespace

namespace pbmoe {

namespace {
int say(char* msg, size_t len, int code, const char* fmt, ...) {
    if (msg && len) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(msg, len, fmt, ap);
        va_end(ap);
    }
    return code;
}
}  // namespace

int moe_check_layout(const pbmoe_expert_layout& L, char* msg, size_t len) {
    const uint32_t H = L.hidden, I = L.intermediate, G = L.group_size;
    if (H == 0 || I == 0 || G == 0) return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT, "expert layout has a zero dimension");
    if (L.encoding == PBMOE_EXPERT_MXFP4) {
        // E2M1 nibbles [rows x cols/2] (16-byte groups of 32 columns), one E8M0 byte per group, no biases
        if (G != 32 || H % 32 != 0 || I % 32 != 0 || H > 16384 || I > 16384)
            return say(msg, len, PBMOE_ERR_UNSUPPORTED,
                       "FlashMoe unsupported MXFP4 expert geometry on CUDA: needs group_size 32 and hidden, "
                       "intermediate multiples of 32 up to 16384 (got hidden=%u intermediate=%u group=%u)",
                       H, I, G);
        const uint64_t gw = uint64_t(I) * H / 2, gs = uint64_t(I) * (H / 32);
        const uint64_t dw = uint64_t(H) * I / 2, ds = uint64_t(H) * (I / 32);
        const uint64_t sizes[9] = {gw, gs, 0, gw, gs, 0, dw, ds, 0};
        for (int i = 0; i < 9; ++i) {
            const uint64_t o = L.component_offsets[i];
            if (o > L.expert_bytes || sizes[i] > L.expert_bytes - o)
                return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT,
                           "expert component %d [%llu, +%llu) exceeds slot bytes %llu", i, (unsigned long long)o,
                           (unsigned long long)sizes[i], (unsigned long long)L.expert_bytes);
            if (i % 3 == 0 && o % 16 != 0)
                return say(msg, len, PBMOE_ERR_UNSUPPORTED, "expert component %d offset %llu is not 16-byte aligned",
                           i, (unsigned long long)o);
        }
        if (L.expert_bytes % 16 != 0)
            return say(msg, len, PBMOE_ERR_UNSUPPORTED, "expert slot stride %llu is not a multiple of 16",
                       (unsigned long long)L.expert_bytes);
        return PBMOE_OK;
    }
    if (L.encoding != PBMOE_EXPERT_AFFINE_Q4)
        return say(msg, len, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported expert encoding %u", L.encoding);
    if (H % G != 0 || I % G != 0)
        return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT,
                   "fixed-Q4 expert dimensions hidden=%u intermediate=%u must be divisible by group_size=%u", H, I, G);
    const bool pow2 = G >= 32 && (G & (G - 1)) == 0;
    if (!pow2 || H % 32 != 0 || I % 32 != 0 || H > 16384 || I > 16384)
        return say(msg, len, PBMOE_ERR_UNSUPPORTED,
                   "FlashMoe unsupported expert geometry on CUDA: needs group_size a power of two >= 32 and "
                   "hidden, intermediate multiples of 32 up to 16384 (got hidden=%u intermediate=%u group=%u)",
                   H, I, G);
    const uint64_t gate_w = uint64_t(I) * H / 2, gate_sb = uint64_t(I) * (H / G) * 2;
    const uint64_t down_w = uint64_t(H) * I / 2, down_sb = uint64_t(H) * (I / G) * 2;
    const uint64_t sizes[9] = {gate_w, gate_sb, gate_sb, gate_w, gate_sb, gate_sb, down_w, down_sb, down_sb};
    for (int i = 0; i < 9; ++i) {
        const uint64_t o = L.component_offsets[i];
        if (o > L.expert_bytes || sizes[i] > L.expert_bytes - o)
            return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT, "expert component %d [%llu, +%llu) exceeds slot bytes %llu",
                       i, (unsigned long long)o, (unsigned long long)sizes[i], (unsigned long long)L.expert_bytes);
        const uint64_t need = (i % 3 == 0) ? 16 : 2;
        if (o % need != 0)
            return say(msg, len, PBMOE_ERR_UNSUPPORTED, "expert component %d offset %llu is not %llu-byte aligned", i,
                       (unsigned long long)o, (unsigned long long)need);
    }
    if (L.expert_bytes % 16 != 0)
        return say(msg, len, PBMOE_ERR_UNSUPPORTED, "expert slot stride %llu is not a multiple of 16",
                   (unsigned long long)L.expert_bytes);
    return PBMOE_OK;
}

int moe_check_config(const pbmoe_moe_config* c, char* msg, size_t len) {
    if (!c) return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT, "null MoE config");
    int rc = moe_check_layout(c->layout, msg, len);
    if (rc) return rc;
    if (c->num_experts == 0 || c->num_experts > 4096)
        return say(msg, len, PBMOE_ERR_UNSUPPORTED, "num_experts %u outside 1..4096", c->num_experts);
    if (c->top_k == 0 || c->top_k > 32 || c->top_k > c->num_experts)
        return say(msg, len, PBMOE_ERR_UNSUPPORTED, "top_k %u outside 1..min(32, num_experts)", c->top_k);
    if (c->normalization > PBMOE_ROUTE_DEEPSEEK_RENORMALIZE_WITH_FLOOR)
        return say(msg, len, PBMOE_ERR_UNSUPPORTED,
                   "FlashMoe unsupported routing weights: normalisation %u is not implemented on CUDA",
                   c->normalization);
    if (!(c->routed_scaling_factor > 0.f) || !std::isfinite(c->routed_scaling_factor))
        return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT, "routed expert scale must be positive and finite");
    if (!(c->norm_epsilon >= 0.f) || !std::isfinite(c->norm_epsilon))
        return say(msg, len, PBMOE_ERR_INVALID_ARGUMENT, "norm epsilon must be finite and >= 0");
    return PBMOE_OK;
}

MoeWsSizes moe_ws_sizes(uint32_t T, uint32_t E, uint32_t K, uint32_t H, uint32_t I) {
    MoeWsSizes s{};
    const size_t R = size_t(T) * K + T;
    const size_t gmax = size_t(T) * K + T;  // routed groups of at most 8 routes + the shared expert's
    size_t* b = s.bytes;
    b[0] = 0;                    // status lives in the context
    b[1] = 8;                    // ticket[2]
    b[2] = size_t(T) * E * 4;    // logits
    b[3] = size_t(T) * 4;        // shared_logit
    b[4] = size_t(T) * K * 4;    // route_ids
    b[5] = size_t(T) * K * 4;    // route_w
    b[6] = 4;                    // num_groups
    b[7] = gmax * 4;             // group_expert
    b[8] = gmax * 4;             // group_start
    b[9] = gmax * 4;             // group_count
    b[10] = R * 4;               // group_routes
    b[11] = R * 4;               // group_tokens
    b[12] = R * I * 4;           // h
    b[13] = R * H * 4;           // y
    b[14] = R * hperm_stride(I); // h_perm
    b[15] = size_t(T) * H * 2;   // xn
    s.total = 0;
    for (int i = 0; i < 16; ++i) s.total += align_up(b[i], 256);
    return s;
}

MoeWs moe_ws_carve(void* base, uint32_t* status, uint32_t T, uint32_t E, uint32_t K, uint32_t H, uint32_t I) {
    MoeWsSizes s = moe_ws_sizes(T, E, K, H, I);
    char* p = static_cast<char*>(base);
    void* ptr[16];
    for (int i = 0; i < 16; ++i) {
        ptr[i] = p;
        p += align_up(s.bytes[i], 256);
    }
    MoeWs w;
    w.status = status;
    w.ticket = static_cast<uint32_t*>(ptr[1]);
    w.logits = static_cast<float*>(ptr[2]);
    w.shared_logit = static_cast<float*>(ptr[3]);
    w.route_ids = static_cast<uint32_t*>(ptr[4]);
    w.route_w = static_cast<float*>(ptr[5]);
    w.num_groups = static_cast<uint32_t*>(ptr[6]);
    w.group_expert = static_cast<uint32_t*>(ptr[7]);
    w.group_start = static_cast<uint32_t*>(ptr[8]);
    w.group_count = static_cast<uint32_t*>(ptr[9]);
    w.group_routes = static_cast<uint32_t*>(ptr[10]);
    w.group_tokens = static_cast<uint32_t*>(ptr[11]);
    w.h = static_cast<float*>(ptr[12]);
    w.y = static_cast<float*>(ptr[13]);
    w.h_perm = static_cast<uint8_t*>(ptr[14]);
    w.xn = static_cast<uint16_t*>(ptr[15]);
    return w;
}

}  // namespace pbmoe

using namespace pbmoe;

extern "C" {

int pbmoe_abi_version(void) { return PBMOE_ABI_VERSION; }

const char* pbmoe_last_error(const pbmoe_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

int pbmoe_init(int device, pbmoe_ctx** out) {
    if (!out) return PBMOE_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return PBMOE_ERR_CUDA;
    auto* ctx = new pbmoe_ctx();
    ctx->device = device;
    DeviceGuard g(device);
    if (!g.ok) {
        delete ctx;
        return PBMOE_ERR_CUDA;
    }
    if (cudaMalloc(&ctx->status, sizeof(uint32_t)) != cudaSuccess) {
        delete ctx;
        return PBMOE_ERR_CUDA;
    }
    if (cudaMemset(ctx->status, 0, sizeof(uint32_t)) != cudaSuccess) {
        cudaFree(ctx->status);
        delete ctx;
        return PBMOE_ERR_CUDA;
    }
    *out = ctx;
    return PBMOE_OK;
}

int pbmoe_destroy(pbmoe_ctx* ctx) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    {
        DeviceGuard g(ctx->device);
        if (ctx->ws_base) cudaFree(ctx->ws_base);
        if (ctx->io_base) cudaFree(ctx->io_base);
        if (ctx->mla_base) cudaFree(ctx->mla_base);
        if (ctx->x16_base) cudaFree(ctx->x16_base);
        if (ctx->head_base) cudaFree(ctx->head_base);
        if (ctx->rope_table) cudaFree(ctx->rope_table);
        for (uint32_t r = 0; r < pbmoe::kMaxEpRanks; ++r)
            if (ctx->ep_peer_ipc[r]) cudaIpcCloseMemHandle(ctx->ep_peer[r]);
        if (ctx->ep_base) cudaFree(ctx->ep_base);
        if (ctx->status) cudaFree(ctx->status);
    }
    delete ctx;
    return PBMOE_OK;
}

int pbmoe_fixed_q4_layout(uint32_t hidden, uint32_t intermediate, uint32_t group, pbmoe_expert_layout* out) {
    if (!out || hidden == 0 || intermediate == 0 || group == 0 || hidden % group || intermediate % group)
        return PBMOE_ERR_INVALID_ARGUMENT;
    const uint64_t gw = uint64_t(intermediate) * hidden / 2, gsb = uint64_t(intermediate) * (hidden / group) * 2;
    const uint64_t dw = uint64_t(hidden) * intermediate / 2, dsb = uint64_t(hidden) * (intermediate / group) * 2;
    const uint64_t sizes[9] = {gw, gsb, gsb, gw, gsb, gsb, dw, dsb, dsb};
    uint64_t off = 0;
    for (int i = 0; i < 9; ++i) {
        out->component_offsets[i] = off;
        off += sizes[i];
    }
    out->expert_bytes = off;
    out->hidden = hidden;
    out->intermediate = intermediate;
    out->group_size = group;
    out->encoding = PBMOE_EXPERT_AFFINE_Q4;
    return PBMOE_OK;
}

int pbmoe_fixed_mxfp4_layout(uint32_t hidden, uint32_t intermediate, uint32_t group, pbmoe_expert_layout* out) {
    if (!out || hidden == 0 || intermediate == 0 || group == 0 || hidden % group || intermediate % group ||
        (uint64_t(hidden) * intermediate) % 2)
        return PBMOE_ERR_INVALID_ARGUMENT;
    const uint64_t gw = uint64_t(intermediate) * hidden / 2, gs = uint64_t(intermediate) * (hidden / group);
    const uint64_t dw = uint64_t(hidden) * intermediate / 2, ds = uint64_t(hidden) * (intermediate / group);
    const uint64_t sizes[9] = {gw, gs, 0, gw, gs, 0, dw, ds, 0};  // biases: none
    uint64_t off = 0;
    for (int i = 0; i < 9; ++i) {
        out->component_offsets[i] = off;
        off += sizes[i];
    }
    out->expert_bytes = off;
    out->hidden = hidden;
    out->intermediate = intermediate;
    out->group_size = group;
    out->encoding = PBMOE_EXPERT_MXFP4;
    return PBMOE_OK;
}

size_t pbmoe_moe_workspace_bytes(uint32_t max_tokens, const pbmoe_moe_config* c) {
    if (!c || max_tokens == 0) return 0;
    return moe_ws_sizes(max_tokens, c->num_experts, c->top_k, c->layout.hidden, c->layout.intermediate).total;
}

int pbmoe_reserve(pbmoe_ctx* ctx, uint32_t max_tokens, const pbmoe_moe_config* c) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    int rc = check_moe_config(ctx, c);
    if (rc) return rc;
    if (max_tokens == 0 || max_tokens > 4096)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "max_tokens %u outside 1..4096", max_tokens);
    const uint32_t E = c->num_experts, K = c->top_k, H = c->layout.hidden, I = c->layout.intermediate;
    if (moe_router_smem(max_tokens, H, E, K) > kRouterSmemLimit)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "router staging for %u tokens exceeds shared memory", max_tokens);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    const size_t need = moe_ws_sizes(max_tokens, E, K, H, I).total;
    const size_t io_need = 3ull * max_tokens * H * sizeof(float);
    if (ctx->ws_base && ctx->ws_bytes >= need && ctx->ws_E == E && ctx->ws_K == K && ctx->ws_H == H &&
        ctx->ws_I == I && ctx->ws_tokens >= max_tokens && ctx->io_bytes >= io_need)
        return PBMOE_OK;
    if (ctx->ws_base || ctx->io_base) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before workspace resize");
        if (ctx->ws_base) cudaFree(ctx->ws_base);
        if (ctx->io_base) cudaFree(ctx->io_base);
        ctx->ws_base = ctx->io_base = nullptr;
        ctx->ws_bytes = ctx->io_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->io_base, io_need);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "host-call staging allocation");
    ctx->io_bytes = io_need;
    e = cudaMalloc(&ctx->ws_base, need);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "workspace allocation");
    e = cudaMemset(ctx->ws_base, 0, need);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "workspace clear");
    ctx->ws_bytes = need;
    ctx->ws_tokens = max_tokens;
    ctx->ws_E = E;
    ctx->ws_K = K;
    ctx->ws_H = H;
    ctx->ws_I = I;
    return PBMOE_OK;
}

int pbmoe_sync(pbmoe_ctx* ctx, void* stream, uint32_t timeout_ms) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return PBMOE_OK;
        if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "stream wait");
        if (std::chrono::steady_clock::now() >= deadline)
            return fail(ctx, PBMOE_ERR_TIMEOUT, "stream still busy after %u ms", timeout_ms);
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int pbmoe_device_status(pbmoe_ctx* ctx, void* stream, uint32_t* out, int clear) {
    if (!ctx || !out) return PBMOE_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(out, ctx->status, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "status read-back");
    if (clear) {
        e = cudaMemsetAsync(ctx->status, 0, sizeof(uint32_t), s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "status clear");
    }
    return PBMOE_OK;
}

int pbmoe_q4_matvec(pbmoe_ctx* ctx, const pbmoe_q4_tensor* w, const void* x, pbmoe_dtype x_dtype, void* y,
                    pbmoe_dtype y_dtype, uint32_t batch, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!w || !w->packed || !w->scales || !w->biases || !x || !y)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec: null pointer");
    if (w->group_size == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "group_size must be positive");
    if (w->rows == 0 || w->cols == 0 || batch == 0) return PBMOE_OK;
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16) || (y_dtype != PBMOE_F32 && y_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (!aligned(x, x_dtype == PBMOE_F32 ? 4 : 2) || !aligned(y, y_dtype == PBMOE_F32 ? 4 : 2) ||
        !aligned(w->scales, 2) || !aligned(w->biases, 2))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec: misaligned pointer");
    DeviceGuard g(ctx->device);
    Q4MatvecArgs a{static_cast<const uint8_t*>(w->packed), w->scales, w->biases, w->rows, w->cols, w->group_size,
                   x, x_dtype, y, y_dtype, batch};
    cudaError_t e = q4_matvec_launch(a, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorNotSupported)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported q4 matvec: cols=%u needs too much shared memory",
                    w->cols);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "q4 matvec launch");
    return PBMOE_OK;
}

int pbmoe_q4_matvec_fused(pbmoe_ctx* ctx, const pbmoe_q4_fused_args* f, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!f || !f->w[0] || !f->x || !f->y[0] || (f->w[1] && !f->y[1]))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: null pointer");
    for (int i = 0; i < 2; ++i) {
        const pbmoe_q4_tensor* w = f->w[i];
        if (!w) continue;
        if (!w->packed || !w->scales || !w->biases)
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: null weight pointer");
        if (w->group_size == 0 || w->rows == 0)
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: empty matrix or zero group");
        if (!aligned(w->scales, 2) || !aligned(w->biases, 2))
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: misaligned scales / biases");
    }
    const pbmoe_q4_tensor* w0 = f->w[0];
    const pbmoe_q4_tensor* w1 = f->w[1];
    if (w1 && (w1->cols != w0->cols || w1->group_size != w0->group_size))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: the two matrices differ in cols or group");
    if ((f->x_dtype != PBMOE_F32 && f->x_dtype != PBMOE_BF16) || (f->y_dtype != PBMOE_F32 && f->y_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (f->input_norm_weight && (f->x_dtype != PBMOE_F32 || !aligned(f->input_norm_weight, 16) ||
                                 !(f->epsilon >= 0.f) || !std::isfinite(f->epsilon)))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT,
                    "q4 fused matvec: the input norm needs f32 x, a 16-byte aligned weight and a finite epsilon");
    if (f->residual && w1)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: a residual goes with one matrix only");
    const size_t ys = f->y_dtype == PBMOE_F32 ? 4 : 2;
    if (!aligned(f->x, f->x_dtype == PBMOE_F32 ? 4 : 2) || !aligned(f->y[0], ys) || (w1 && !aligned(f->y[1], ys)) ||
        (f->residual && !aligned(f->residual, ys)))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 fused matvec: misaligned x / y / residual");
    if (f->batch == 0 || w0->cols == 0) return PBMOE_OK;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    Q4MatvecArgs a{static_cast<const uint8_t*>(w0->packed), w0->scales, w0->biases, w0->rows, w0->cols, w0->group_size,
                   f->x, f->x_dtype, f->y[0], f->y_dtype, f->batch};
    a.norm_w = f->input_norm_weight;
    a.eps = f->epsilon;
    a.residual = f->residual;
    if (w1) {
        a.packed2 = static_cast<const uint8_t*>(w1->packed);
        a.scales2 = w1->scales;
        a.biases2 = w1->biases;
        a.rows2 = w1->rows;
        a.y2 = f->y[1];
    }
    cudaError_t e = q4_matvec_launch(a, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorNotSupported)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported fused q4 matvec: cols=%u group=%u needs the fast path (cols a multiple of 32, "
                    "group a power of two >= 32, 16-byte aligned rows and x)", w0->cols, w0->group_size);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "q4 fused matvec launch");
    return PBMOE_OK;
}

int pbmoe_q4_matvec_batch(pbmoe_ctx* ctx, const pbmoe_q4_tensor* w, uint32_t count, const void* x,
                          pbmoe_dtype x_dtype, void* const* y, pbmoe_dtype y_dtype, uint32_t batch, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (count == 0 || batch == 0) return PBMOE_OK;
    if (!w || !x || !y) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec batch: null pointer");
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16) || (y_dtype != PBMOE_F32 && y_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    const size_t ys = y_dtype == PBMOE_F32 ? 4 : 2;
    if (!aligned(x, x_dtype == PBMOE_F32 ? 4 : 2))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec batch: misaligned x");
    const uint32_t cols = w[0].cols, group = w[0].group_size;
    if (cols == 0 || group == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec batch: empty matrix or zero group");
    for (uint32_t i = 0; i < count; ++i) {
        if (!w[i].packed || !w[i].scales || !w[i].biases || !y[i])
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec batch: null pointer in matrix %u", i);
        if (w[i].cols != cols || w[i].group_size != group)
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT,
                        "q4 matvec batch: matrix %u has cols %u group %u, matrix 0 has cols %u group %u", i, w[i].cols,
                        w[i].group_size, cols, group);
        if (w[i].rows == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec batch: matrix %u has no rows", i);
        if (!aligned(w[i].scales, 2) || !aligned(w[i].biases, 2) || !aligned(y[i], ys))
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 matvec batch: misaligned pointer in matrix %u", i);
    }
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    for (uint32_t i0 = 0; i0 < count; i0 += pbmoe::kQ4MaxMats) {
        const uint32_t n = std::min(count - i0, pbmoe::kQ4MaxMats);
        pbmoe::Q4MatSpec set[pbmoe::kQ4MaxMats];
        for (uint32_t i = 0; i < n; ++i)
            set[i] = {static_cast<const uint8_t*>(w[i0 + i].packed), w[i0 + i].scales, w[i0 + i].biases, w[i0 + i].rows,
                      y[i0 + i]};
        Q4MatvecArgs a{set[0].packed, set[0].scales, set[0].biases, set[0].rows, cols, group, x, x_dtype,
                       set[0].y, y_dtype, batch};
        a.set_count = n;
        a.set = set;
        cudaError_t e = q4_matvec_launch(a, static_cast<cudaStream_t>(stream));
        if (e == cudaErrorNotSupported)
            return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                        "FlashMoe unsupported q4 matvec batch: cols=%u group=%u needs the fast path (cols a multiple "
                        "of 32, group a power of two >= 32, 16-byte aligned rows and x)", cols, group);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "q4 matvec batch launch");
    }
    return PBMOE_OK;
}

int pbmoe_route_topk(pbmoe_ctx* ctx, const float* logits, uint32_t tokens, uint32_t E, uint32_t K,
                     uint32_t normalization, float routed_scale, uint32_t* ids, float* weights, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!logits || !ids || !weights) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "route top-k: null pointer");
    if (E == 0 || K == 0 || K > 32 || K > E)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "route top-k: K=%u over E=%u outside 1..min(32, E)", K, E);
    if (normalization > PBMOE_ROUTE_DEEPSEEK_RENORMALIZE_WITH_FLOOR)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported routing weights: normalisation %u is not implemented on CUDA", normalization);
    if (!(routed_scale > 0.f) || !std::isfinite(routed_scale))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "routed expert scale must be positive and finite");
    if (tokens == 0) return PBMOE_OK;
    DeviceGuard g(ctx->device);
    cudaError_t e = route_topk_launch(logits, tokens, E, K, normalization, routed_scale, ids, weights, ctx->status,
                                      static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "route top-k launch");
    return PBMOE_OK;
}

int pbmoe_route_sigmoid_noaux(pbmoe_ctx* ctx, const float* logits, const float* bias, uint32_t tokens, uint32_t E,
                              uint32_t K, uint32_t normalization, float routed_scale, uint32_t* ids, float* weights,
                              void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!logits || !bias || !ids || !weights)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "sigmoid/noaux routing: null pointer");
    if (E == 0 || K == 0 || K > 32 || K > E)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "sigmoid/noaux routing: K=%u over E=%u outside 1..min(32, E)", K, E);
    if (normalization > PBMOE_ROUTE_DEEPSEEK_RENORMALIZE_WITH_FLOOR)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported routing weights: normalisation %u is not implemented on CUDA", normalization);
    if (!(routed_scale > 0.f) || !std::isfinite(routed_scale))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "routed expert scale must be positive and finite");
    if (tokens == 0) return PBMOE_OK;
    DeviceGuard g(ctx->device);
    cudaError_t e = route_topk_launch(logits, tokens, E, K, normalization, routed_scale, ids, weights, ctx->status,
                                      static_cast<cudaStream_t>(stream), bias);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "sigmoid/noaux routing launch");
    return PBMOE_OK;
}

namespace {
// One decode layer; with `ep` set, the experts of [e_lo, e_lo + e_count) only
// and the expert-parallel combine.
int moe_layer_impl(pbmoe_ctx* ctx, const pbmoe_moe_config* c, const pbmoe_moe_weights* w, const void* x,
                   pbmoe_dtype x_dtype, const void* residual, void* out, pbmoe_dtype out_dtype, uint32_t tokens,
                   const float* next_norm_weight, void* next_normed, const pbmoe_moe_debug* debug, void* stream,
                   uint32_t e_lo, uint32_t e_count, const pbmoe::EpPeers* ep) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    int rc = check_moe_config(ctx, c);
    if (rc) return rc;
    if (!w || !w->router_weight || !w->experts || !x || !out)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "moe layer: null pointer");
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16) || (out_dtype != PBMOE_F32 && out_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if ((next_norm_weight == nullptr) != (next_normed == nullptr))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "next_norm_weight and next_normed must be given together");
    if (w->shared_expert_gate && !w->shared_expert)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "shared expert gate given without a shared expert");
    if (!aligned(x, 16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "moe layer: x must be 16-byte aligned (rows are read as 16-byte vectors)");
    if (!aligned(w->experts, 16) || (w->shared_expert && !aligned(w->shared_expert, 16)) ||
        !aligned(w->router_weight, 16) || (w->shared_expert_gate && !aligned(w->shared_expert_gate, 16)) ||
        (w->input_norm_weight && !aligned(w->input_norm_weight, 16)) ||
        (w->router_correction_bias && !aligned(w->router_correction_bias, 16)))
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "expert table, shared expert, router and input-norm weights must be 16-byte aligned");
    if (tokens == 0) return PBMOE_OK;
    const uint32_t E = c->num_experts, K = c->top_k, H = c->layout.hidden, I = c->layout.intermediate;
    if (!ctx->ws_base || tokens > ctx->ws_tokens || ctx->ws_E != E || ctx->ws_K != K || ctx->ws_H != H ||
        ctx->ws_I != I)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE,
                    "moe layer: workspace reserved for tokens<=%u E=%u K=%u H=%u I=%u, call needs tokens=%u E=%u K=%u "
                    "H=%u I=%u (call pbmoe_reserve)",
                    ctx->ws_tokens, ctx->ws_E, ctx->ws_K, ctx->ws_H, ctx->ws_I, tokens, E, K, H, I);
    DeviceGuard g(ctx->device);
    MoeLaunch a{};
    a.ws = moe_ws_carve(ctx->ws_base, ctx->status, ctx->ws_tokens, E, K, H, I);
    const pbmoe_expert_layout& L = c->layout;
    for (int i = 0; i < 9; ++i) a.layout.off[i] = L.component_offsets[i];
    a.layout.expert_bytes = L.expert_bytes;
    a.layout.hidden = H;
    a.layout.inter = I;
    a.layout.group = L.group_size;
    a.layout.cpg_shift_h = ilog2_u32(L.group_size / 32);
    a.layout.cpg_shift_i = ilog2_u32(L.group_size / 32);
    a.layout.mxfp4 = L.encoding == PBMOE_EXPERT_MXFP4;
    a.tokens = tokens;
    a.num_experts = E;
    a.top_k = K;
    a.normalization = c->normalization;
    a.routed_scale = c->routed_scaling_factor;
    a.eps = c->norm_epsilon;
    a.x = x;
    a.x_dtype = x_dtype;
    a.residual = residual;
    a.out = out;
    a.out_dtype = out_dtype;
    a.next_norm_w = next_norm_weight;
    a.next_normed = next_normed;
    a.router_w = w->router_weight;
    a.shared_gate = w->shared_expert_gate;
    a.experts = w->experts;
    a.shared_slot = w->shared_expert;
    a.in_norm_w = w->input_norm_weight;
    a.in_eps = c->norm_epsilon;
    a.router_bias = w->router_correction_bias;
    a.pdl = true;
    a.phase_events = debug ? debug->phase_events : nullptr;
    a.expert_lo = e_lo;
    a.expert_count = e_count;
    a.ep = ep;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Batches above 32 tokens run as consecutive chunks of 32 through the
    // pipelined expert kernels when those take the layout (chunks of 8 when
    // only the 8-token form does): every token's routing, combine and norm
    // are its own, so the chunks compute exactly what one launch computes for
    // those tokens. (Not with phase events, which time one launch, nor with
    // expert parallelism, whose exchange buffers hold one launch's tokens.)
    uint32_t chunk = tokens;
    if (tokens > 8 && !ep && !a.phase_events) {
        MoeLaunch probe = a;
        if (a.in_norm_w) probe.x_dtype = PBMOE_BF16;  // the experts read the normalised bf16 rows
        probe.tokens = tokens < 32 ? tokens : 32;
        if (pbmoe::moe_pipe_supported(probe)) {
            chunk = 32;
        } else {
            probe.tokens = 8;
            if (pbmoe::moe_pipe_supported(probe)) chunk = 8;
        }
    }
    const size_t xs = x_dtype == PBMOE_BF16 ? 2 : 4, os = out_dtype == PBMOE_BF16 ? 2 : 4;
    for (uint32_t c0 = 0; c0 < tokens; c0 += chunk) {
        MoeLaunch b = a;
        b.tokens = tokens - c0 < chunk ? tokens - c0 : chunk;
        b.x = static_cast<const char*>(x) + size_t(c0) * H * xs;
        b.residual = residual ? static_cast<const char*>(residual) + size_t(c0) * H * os : nullptr;
        b.out = static_cast<char*>(out) + size_t(c0) * H * os;
        b.next_normed = next_normed ? static_cast<char*>(next_normed) + size_t(c0) * H * os : nullptr;
        cudaError_t e = moe_layer_launch(b, s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "moe layer launch");
        if (debug) {
            const size_t n = b.tokens;
            auto at = [](void* p, size_t off) { return static_cast<char*>(p) + off; };
            if (debug->router_logits)
                e = cudaMemcpyAsync(at(debug->router_logits, c0 * E * 4), a.ws.logits, n * E * 4,
                                    cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && debug->route_ids)
                e = cudaMemcpyAsync(at(debug->route_ids, c0 * K * 4), a.ws.route_ids, n * K * 4,
                                    cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && debug->route_weights)
                e = cudaMemcpyAsync(at(debug->route_weights, c0 * K * 4), a.ws.route_w, n * K * 4,
                                    cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && debug->shared_logit)
                e = cudaMemcpyAsync(at(debug->shared_logit, c0 * 4), a.ws.shared_logit, n * 4,
                                    cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && debug->normed_input && a.in_norm_w)
                e = cudaMemcpyAsync(at(debug->normed_input, c0 * H * 2), a.ws.xn, n * H * 2,
                                    cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "moe debug copy");
        }
    }
    return PBMOE_OK;
}
}  // namespace

int pbmoe_moe_layer(pbmoe_ctx* ctx, const pbmoe_moe_config* c, const pbmoe_moe_weights* w, const void* x,
                    pbmoe_dtype x_dtype, const void* residual, void* out, pbmoe_dtype out_dtype, uint32_t tokens,
                    const float* next_norm_weight, void* next_normed, const pbmoe_moe_debug* debug, void* stream) {
    return moe_layer_impl(ctx, c, w, x, x_dtype, residual, out, out_dtype, tokens, next_norm_weight, next_normed,
                          debug, stream, 0, 0, nullptr);
}

int pbmoe_moe_layer_host(pbmoe_ctx* ctx, const pbmoe_moe_config* c, const pbmoe_moe_weights* w, const void* x,
                         pbmoe_dtype x_dtype, const void* residual, void* out, pbmoe_dtype out_dtype, uint32_t tokens,
                         void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!c || !x || !out) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "moe layer (host rows): null pointer");
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16) || (out_dtype != PBMOE_F32 && out_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (tokens == 0) return PBMOE_OK;
    const uint32_t H = c->layout.hidden;
    if (!ctx->io_base || tokens > ctx->ws_tokens || H != ctx->ws_H)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "moe layer (host rows): %u tokens of hidden %u need pbmoe_reserve",
                    tokens, H);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    const size_t xs = x_dtype == PBMOE_BF16 ? 2 : 4, os = out_dtype == PBMOE_BF16 ? 2 : 4;
    const size_t slot = size_t(ctx->ws_tokens) * H * sizeof(float);
    char* dx = static_cast<char*>(ctx->io_base);
    char* dres = dx + slot;
    char* dout = dres + slot;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Page-locked host rows that the device can address (cudaHostAlloc /
    // cudaHostRegister memory) are used in place by the one kernel that
    // touches each of them once per element: the combine kernel reads the
    // residual (before its dependency wait) and stores the output. x is read
    // by every router and expert CTA, so it is always copied in.
    auto device_view = [](const void* p) -> void* {
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        if (at.type != cudaMemoryTypeHost || !at.devicePointer) return nullptr;
        return reinterpret_cast<uintptr_t>(at.devicePointer) % 16 == 0 ? at.devicePointer : nullptr;
    };
    const void* res_in_place = residual ? device_view(residual) : nullptr;
    void* out_in_place = device_view(out);
    cudaError_t e = cudaMemcpyAsync(dx, x, size_t(tokens) * H * xs, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && residual && !res_in_place)
        e = cudaMemcpyAsync(dres, residual, size_t(tokens) * H * os, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "moe layer (host rows) input copy");
    const void* res_dev = residual ? (res_in_place ? res_in_place : dres) : nullptr;
    void* out_dev = out_in_place ? out_in_place : dout;
    const int rc = moe_layer_impl(ctx, c, w, dx, x_dtype, res_dev, out_dev, out_dtype, tokens, nullptr, nullptr,
                                  nullptr, stream, 0, 0, nullptr);
    if (rc != PBMOE_OK) return rc;
    if (!out_in_place) {
        e = cudaMemcpyAsync(out, dout, size_t(tokens) * H * os, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "moe layer (host rows) output copy");
    }
    return PBMOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- MLA decode
namespace {

struct MlaWsSizes {
    size_t qp, partial, ctx, total;
};

MlaWsSizes mla_ws_sizes(uint32_t max_batch, int num_sms) {
    MlaWsSizes w{};
    w.qp = align_up(size_t(max_batch) * 16 * 576 * 4, 256);
    // batch x splits <= kMlaCtasPerSm * num_sms + batch (pbmoe::mla_plan_splits)
    w.partial = align_up((size_t(pbmoe::kMlaCtasPerSm) * num_sms + 2 * max_batch) * 16 * 514 * 4, 256);
    w.ctx = align_up(size_t(max_batch) * 16 * 512 * 4, 256);
    w.total = w.qp + w.partial + w.ctx;
    return w;
}

int check_mla_config(pbmoe_ctx* ctx, const pbmoe_mla_config* c) {
    if (!c) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: null config");
    if (c->heads == 0 || c->nope_dim == 0 || c->rope_dim == 0 || c->latent_dim == 0 || c->v_dim == 0)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: zero dimension");
    if (!pbmoe::mla_shape_supported(c->heads, c->rope_dim, c->latent_dim, c->v_dim) || c->nope_dim > 128)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported MLA shape on CUDA: heads=%u nope=%u rope=%u latent=%u v=%u (built for "
                    "heads 16, rope 64, latent 512, v 128, nope <= 128)",
                    c->heads, c->nope_dim, c->rope_dim, c->latent_dim, c->v_dim);
    if (!(c->softmax_scale >= 0.f) || !std::isfinite(c->softmax_scale))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: softmax_scale must be finite and >= 0");
    return PBMOE_OK;
}

int sm_count(pbmoe_ctx* ctx) {
    if (ctx->num_sms <= 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, ctx->device) != cudaSuccess || n <= 0) n = 148;
        ctx->num_sms = n;
    }
    return ctx->num_sms;
}

}  // namespace

int pbmoe_mla_reserve(pbmoe_ctx* ctx, const pbmoe_mla_config* c, uint32_t max_batch) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    int rc = check_mla_config(ctx, c);
    if (rc) return rc;
    if (max_batch == 0 || max_batch > pbmoe::kMlaMaxBatch)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: max_batch %u outside 1..%u", max_batch,
                    pbmoe::kMlaMaxBatch);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    const size_t need = mla_ws_sizes(max_batch, sm_count(ctx)).total;
    if (ctx->mla_base && ctx->mla_bytes >= need && ctx->mla_batch >= max_batch) return PBMOE_OK;
    if (ctx->mla_base) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before MLA workspace resize");
        cudaFree(ctx->mla_base);
        ctx->mla_base = nullptr;
        ctx->mla_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->mla_base, need);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "MLA workspace allocation");
    ctx->mla_bytes = need;
    ctx->mla_batch = max_batch;
    return PBMOE_OK;
}

namespace {
int mla_decode_impl(pbmoe_ctx* ctx, const pbmoe_mla_config* c, const pbmoe_mla_args* a,
                    const pbmoe::RopeAppendArgs* rope, void* stream);
}  // namespace

int pbmoe_mla_decode(pbmoe_ctx* ctx, const pbmoe_mla_config* c, const pbmoe_mla_args* a, void* stream) {
    return mla_decode_impl(ctx, c, a, nullptr, stream);
}

int pbmoe_mla_append_decode(pbmoe_ctx* ctx, const pbmoe_mla_config* c, const pbmoe_mla_args* a, const float* kv,
                            const float* latent_norm_weight, float epsilon, const uint32_t* positions,
                            uint16_t* const* c_kv_rows, uint16_t* const* k_rope_rows, uint32_t cache_len,
                            void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!c || !a || !kv || !positions || !c_kv_rows || !k_rope_rows)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla append + decode: null pointer");
    if (a->query_dtype != PBMOE_F32)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla append + decode: the query must be f32 (rotated in place)");
    if (latent_norm_weight && (!(epsilon >= 0.f) || !std::isfinite(epsilon)))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla append + decode: norm epsilon must be finite and >= 0");
    if (!ctx->rope_table || ctx->rope_dim != c->rope_dim)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "mla append + decode: rope dim %u needs pbmoe_rope_reserve",
                    c->rope_dim);
    if (!pbmoe::rope_append_supported(c->heads, c->rope_dim) || c->latent_dim == 0 ||
        c->latent_dim > 4 * 256 || cache_len == 0)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported MLA RoPE append: %u heads x rope %u, latent %u",
                    c->heads, c->rope_dim, c->latent_dim);
    pbmoe::RopeAppendArgs r{};
    r.batch = a->batch;
    r.heads = c->heads;
    r.nope = c->nope_dim;
    r.rope = c->rope_dim;
    r.latent = c->latent_dim;
    r.query = static_cast<float*>(const_cast<void*>(a->query));
    r.kv = kv;
    r.latent_norm_w = latent_norm_weight;
    r.eps = epsilon;
    r.positions = positions;
    r.c_kv = c_kv_rows;
    r.k_rope = k_rope_rows;
    r.cache_len = cache_len;
    r.table = ctx->rope_table;
    r.max_positions = ctx->rope_positions;
    r.status = ctx->status;
    return mla_decode_impl(ctx, c, a, &r, stream);
}

namespace {
int mla_decode_impl(pbmoe_ctx* ctx, const pbmoe_mla_config* c, const pbmoe_mla_args* a,
                    const pbmoe::RopeAppendArgs* rope, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    int rc = check_mla_config(ctx, c);
    if (rc) return rc;
    if (!a || !a->seq_lens || !a->query || !a->c_kv || !a->k_rope || !a->w_uk || !a->w_uv || !a->out)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: null pointer");
    if (a->batch == 0 || a->batch > pbmoe::kMlaMaxBatch)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: batch %u outside 1..%u", a->batch, pbmoe::kMlaMaxBatch);
    if ((a->query_dtype != PBMOE_F32 && a->query_dtype != PBMOE_BF16) ||
        (a->out_dtype != PBMOE_F32 && a->out_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: unknown dtype");
    if (!ctx->mla_base || ctx->mla_batch < a->batch)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "mla: workspace reserved for batch<=%u, call needs %u "
                    "(call pbmoe_mla_reserve)", ctx->mla_batch, a->batch);
    if (!aligned(a->query, a->query_dtype == PBMOE_F32 ? 4 : 2) ||
        !aligned(a->out, a->out_dtype == PBMOE_F32 ? 4 : 2) || !aligned(a->w_uk, 16) || !aligned(a->w_uv, 16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: misaligned query / out / W_UK / W_UV");
    pbmoe::MlaLaunch L{};
    L.batch = a->batch;
    L.nope = c->nope_dim;
    L.scale = c->softmax_scale > 0.f ? c->softmax_scale
                                     : 1.0f / std::sqrt(static_cast<float>(c->nope_dim + c->rope_dim));
    L.q = a->query;
    L.q_dtype = a->query_dtype;
    for (uint32_t b = 0; b < a->batch; ++b) {
        if (a->seq_lens[b] == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: sequence %u is empty", b);
        if (!a->c_kv[b] || !a->k_rope[b])
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: null cache pointer for sequence %u", b);
        if (!aligned(a->c_kv[b], 16) || !aligned(a->k_rope[b], 16))
            return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla: cache of sequence %u not 16-byte aligned", b);
        L.seqs.c_kv[b] = a->c_kv[b];
        L.seqs.k_rope[b] = a->k_rope[b];
        L.seqs.len[b] = a->seq_lens[b];
    }
    L.w_uk = a->w_uk;
    L.w_uv = a->w_uv;
    L.out = a->out;
    L.out_dtype = a->out_dtype;
    const MlaWsSizes w = mla_ws_sizes(ctx->mla_batch, sm_count(ctx));
    char* base = static_cast<char*>(ctx->mla_base);
    L.qp = reinterpret_cast<float*>(base);
    L.partial = reinterpret_cast<float*>(base + w.qp);
    L.ctx = reinterpret_cast<float*>(base + w.qp + w.partial);
    L.rope = rope;
    pbmoe::mla_plan_splits(L, sm_count(ctx), L.split_tokens, L.splits);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    cudaError_t e = pbmoe::mla_decode_launch(L, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "MLA decode launch");
    return PBMOE_OK;
}
}  // namespace

int pbmoe_prefill_reserve(pbmoe_ctx* ctx, uint32_t max_rows, uint32_t max_cols) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (max_rows == 0 || max_cols == 0 || max_cols % 64)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "prefill reserve: %u x %u (cols must be a positive multiple of 64)",
                    max_rows, max_cols);
    const size_t need = size_t(max_rows) * max_cols;
    if (ctx->x16_base && ctx->x16_elems >= need) return PBMOE_OK;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    if (ctx->x16_base) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before prefill workspace resize");
        cudaFree(ctx->x16_base);
        ctx->x16_base = nullptr;
        ctx->x16_elems = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->x16_base, need * 2);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "prefill workspace allocation");
    ctx->x16_elems = need;
    return PBMOE_OK;
}

namespace {
// fp16 token rows for the tensor-core GEMMs: x itself (fp16, no gather), or
// x[rows[j]] converted / gathered into the context workspace (queued on
// `stream` ahead of the GEMM).
int prefill_rows(pbmoe_ctx* ctx, const void* x, pbmoe_dtype x_dtype, const uint32_t* rows, uint32_t nrows,
                 uint32_t x_rows, uint32_t K, cudaStream_t stream, const void** out) {
    if (x_dtype != PBMOE_BF16 && x_dtype != PBMOE_F16)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported prefill GEMM activations: dtype %d "
                    "(bf16 or fp16)", static_cast<int>(x_dtype));
    if (x_dtype == PBMOE_F16 && !rows) {
        *out = x;
        return PBMOE_OK;
    }
    const size_t elems = size_t(nrows) * K;
    if (!ctx->x16_base || ctx->x16_elems < elems)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "prefill GEMM: %u activation rows of %u need "
                    "pbmoe_prefill_reserve (workspace holds %zu elements)", nrows, K, ctx->x16_elems);
    cudaError_t e = pbmoe::x16_gather_launch(x, x_dtype == PBMOE_F16, rows, nrows, x_rows, K, ctx->x16_base,
                                             ctx->status, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "activation fp16 gather launch");
    *out = ctx->x16_base;
    return PBMOE_OK;
}
}  // namespace

int pbmoe_q4_gemm(pbmoe_ctx* ctx, const pbmoe_q4_tensor* w, const void* x, pbmoe_dtype x_dtype, void* y,
                  pbmoe_dtype y_dtype, uint32_t m, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!w || !w->packed || !w->scales || !w->biases || !x || !y)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 gemm: null pointer");
    if (w->group_size == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "group_size must be positive");
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16 && x_dtype != PBMOE_F16) ||
        (y_dtype != PBMOE_F32 && y_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (w->rows == 0 || w->cols == 0 || m == 0) return PBMOE_OK;
    if (x_dtype == PBMOE_F32 || !pbmoe::q4_gemm_supported(w->rows, w->cols, w->group_size))
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported q4 gemm: needs bf16 or fp16 x, group_size 64 and cols a multiple of 512 "
                    "(got x dtype %d, group %u, cols %u)", static_cast<int>(x_dtype), w->group_size, w->cols);
    if (!aligned(w->packed, 16) || !aligned(w->scales, 16) || !aligned(w->biases, 16) || !aligned(x, 16) ||
        !aligned(y, 16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 gemm: packed, scales, biases, x and y must be 16-byte aligned");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const void* x16 = nullptr;
    int rc = prefill_rows(ctx, x, x_dtype, nullptr, m, m, w->cols, s, &x16);
    if (rc) return rc;
    pbmoe::Q4GemmArgs a{static_cast<const uint8_t*>(w->packed), w->scales, w->biases, w->rows, w->cols,
                        w->group_size, x16, m, y, y_dtype, ctx->status};
    cudaError_t e = pbmoe::q4_gemm_launch(a, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "q4 gemm launch");
    return PBMOE_OK;
}

int pbmoe_prefill_group_plan(pbmoe_ctx* ctx, const uint32_t* route_ids, uint32_t rows, uint32_t top_k,
                             uint32_t num_experts, uint32_t* slot_experts, uint32_t* unique_count,
                             uint32_t* route_slots, uint32_t* source_rows, uint32_t* output_indices,
                             uint32_t* groups, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!route_ids || !slot_experts || !unique_count || !source_rows || !output_indices || !groups)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "prefill group plan: null pointer");
    // the reference rejects an empty plan (metal/mod.rs:3202-3204)
    if (rows == 0 || top_k == 0 || num_experts == 0)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT,
                    "Qwen layer-major group plan has invalid geometry routes=%u unique=%u active=%u", rows * top_k,
                    num_experts, top_k);
    if (num_experts > pbmoe::kPlanMaxExperts)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported prefill plan: %u experts (max %u)",
                    num_experts, pbmoe::kPlanMaxExperts);
    if (static_cast<uint64_t>(rows) * top_k > 0xffffffffull)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "prefill group plan: route count overflows u32");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    pbmoe::PrefillPlanArgs a{route_ids,   rows,        top_k,          num_experts, slot_experts, unique_count,
                             route_slots, source_rows, output_indices, groups,      ctx->status};
    cudaError_t e = pbmoe::prefill_plan_launch(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "prefill group plan launch");
    return PBMOE_OK;
}

int pbmoe_q4_gemm_grouped(pbmoe_ctx* ctx, const pbmoe_q4_expert_matrix* w, const uint32_t* slot_experts,
                          const uint32_t* unique_count, const uint32_t* groups, const uint32_t* source_rows,
                          uint32_t routes, uint32_t max_unique, const void* x, pbmoe_dtype x_dtype, uint32_t x_rows,
                          void* y, pbmoe_dtype y_dtype, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!w || !w->experts || !slot_experts || !unique_count || !groups || !source_rows || !x || !y)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 grouped gemm: null pointer");
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16 && x_dtype != PBMOE_F16) ||
        (y_dtype != PBMOE_F32 && y_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (w->group_size == 0 || w->rows == 0 || w->cols == 0 || w->num_experts == 0)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 grouped gemm: zero dimension");
    if (routes == 0 || max_unique == 0) return PBMOE_OK;
    if (x_rows == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 grouped gemm: x has no rows");
    if (x_dtype == PBMOE_F32 || !pbmoe::q4_grouped_supported(w->rows, w->cols, w->group_size, routes, max_unique))
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported q4 grouped gemm: needs bf16 or fp16 x, group_size 64, cols a multiple "
                    "of 512 and a tile table that fits in shared memory (got x dtype %d, group %u, cols %u, "
                    "%u routes over %u slots)", static_cast<int>(x_dtype), w->group_size, w->cols, routes, max_unique);
    const uint64_t wbytes = uint64_t(w->rows) * w->cols / 2, sbytes = uint64_t(w->rows) * (w->cols / 64) * 2;
    if (w->packed_offset + wbytes > w->expert_bytes || w->scales_offset + sbytes > w->expert_bytes ||
        w->biases_offset + sbytes > w->expert_bytes)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "q4 grouped gemm: projection does not fit in an expert slot");
    if (!aligned(w->experts, 16) || w->expert_bytes % 16 || w->packed_offset % 16 || w->scales_offset % 16 ||
        w->biases_offset % 16 || !aligned(x, 16) || !aligned(y, 16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT,
                    "q4 grouped gemm: expert table, slot stride, component offsets, x and y must be 16-byte aligned");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const void* xg16 = nullptr;
    int rc = prefill_rows(ctx, x, x_dtype, source_rows, routes, x_rows, w->cols, s, &xg16);
    if (rc) return rc;
    pbmoe::Q4GroupedArgs a{};
    a.experts = w->experts;
    a.expert_bytes = w->expert_bytes;
    a.packed_offset = w->packed_offset;
    a.scales_offset = w->scales_offset;
    a.biases_offset = w->biases_offset;
    a.rows = w->rows;
    a.cols = w->cols;
    a.num_experts = w->num_experts;
    a.slot_experts = slot_experts;
    a.unique_count = unique_count;
    a.max_unique = max_unique;
    a.groups = groups;
    a.routes = routes;
    a.xg16 = xg16;
    a.y = y;
    a.y_dtype = y_dtype;
    a.status = ctx->status;
    cudaError_t e = pbmoe::q4_gemm_grouped_launch(a, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "q4 grouped gemm launch");
    return PBMOE_OK;
}

// ---------------------------------------------------------------- expert parallelism
int pbmoe_ep_expert_range(uint32_t E, uint32_t rank, uint32_t world, uint32_t* begin, uint32_t* count) {
    if (!begin || !count || world == 0 || rank >= world || E < world) return PBMOE_ERR_INVALID_ARGUMENT;
    const uint64_t b = uint64_t(rank) * E / world, e = uint64_t(rank + 1) * E / world;
    *begin = static_cast<uint32_t>(b);
    *count = static_cast<uint32_t>(e - b);
    return PBMOE_OK;
}

namespace {
void ep_unmap(pbmoe_ctx* ctx) {
    for (uint32_t r = 0; r < pbmoe::kMaxEpRanks; ++r) {
        if (ctx->ep_peer_ipc[r]) cudaIpcCloseMemHandle(ctx->ep_peer[r]);
        ctx->ep_peer_ipc[r] = false;
        ctx->ep_peer[r] = nullptr;
    }
}
}  // namespace

int pbmoe_ep_reserve(pbmoe_ctx* ctx, uint32_t rank, uint32_t world, uint32_t max_tokens, uint32_t hidden) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (world == 0 || world > pbmoe::kMaxEpRanks || rank >= world)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "expert parallelism: rank %u of world %u (world 1..%u)", rank, world,
                    pbmoe::kMaxEpRanks);
    if (max_tokens == 0 || hidden == 0 || hidden % 8)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "expert parallelism: max_tokens %u, hidden %u", max_tokens, hidden);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    const size_t need = pbmoe::ep_buffer_bytes(world, max_tokens, hidden);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before exchange-buffer setup");
    ep_unmap(ctx);
    if (ctx->ep_base && ctx->ep_bytes != need) {
        cudaFree(ctx->ep_base);
        ctx->ep_base = nullptr;
    }
    if (!ctx->ep_base && (e = cudaMalloc(&ctx->ep_base, need)) != cudaSuccess)
        return cuda_fail(ctx, e, "exchange buffer allocation");
    if ((e = cudaMemset(ctx->ep_base, 0, need)) != cudaSuccess) return cuda_fail(ctx, e, "exchange buffer clear");
    ctx->ep_bytes = need;
    ctx->ep_rank = rank;
    ctx->ep_world = world;
    ctx->ep_max_tokens = max_tokens;
    ctx->ep_hidden = hidden;
    ctx->ep_peer[rank] = ctx->ep_base;
    return PBMOE_OK;
}

void* pbmoe_ep_buffer(pbmoe_ctx* ctx) { return ctx ? ctx->ep_base : nullptr; }

int pbmoe_ep_ipc_handle(pbmoe_ctx* ctx, void* handle) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!handle) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "ep ipc handle: null output");
    if (!ctx->ep_base) return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "ep ipc handle: call pbmoe_ep_reserve first");
    static_assert(sizeof(cudaIpcMemHandle_t) == PBMOE_EP_HANDLE_BYTES, "IPC handle size");
    DeviceGuard g(ctx->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, ctx->ep_base);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "exchange buffer IPC handle");
    std::memcpy(handle, &h, sizeof h);
    return PBMOE_OK;
}

int pbmoe_ep_open_peers(pbmoe_ctx* ctx, const void* handles) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!handles) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "ep open peers: null handles");
    if (!ctx->ep_base) return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "ep open peers: call pbmoe_ep_reserve first");
    DeviceGuard g(ctx->device);
    ep_unmap(ctx);
    ctx->ep_peer[ctx->ep_rank] = ctx->ep_base;
    for (uint32_t r = 0; r < ctx->ep_world; ++r) {
        if (r == ctx->ep_rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(handles) + size_t(r) * PBMOE_EP_HANDLE_BYTES, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            ep_unmap(ctx);
            ctx->ep_peer[ctx->ep_rank] = ctx->ep_base;
            return fail(ctx, PBMOE_ERR_PEER, "ep open peers: mapping rank %u failed: %s", r, cudaGetErrorString(e));
        }
        ctx->ep_peer[r] = p;
        ctx->ep_peer_ipc[r] = true;
    }
    return PBMOE_OK;
}

int pbmoe_ep_set_peers(pbmoe_ctx* ctx, void* const* buffers) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!buffers) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "ep set peers: null buffers");
    if (!ctx->ep_base) return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "ep set peers: call pbmoe_ep_reserve first");
    ep_unmap(ctx);
    for (uint32_t r = 0; r < ctx->ep_world; ++r) ctx->ep_peer[r] = r == ctx->ep_rank ? ctx->ep_base : buffers[r];
    return PBMOE_OK;
}

int pbmoe_ep_moe_layer(pbmoe_ctx* ctx, const pbmoe_moe_config* c, const pbmoe_moe_weights* w,
                       const pbmoe_ep_shard* shard, const void* x, pbmoe_dtype x_dtype, const void* residual, void* out,
                       pbmoe_dtype out_dtype, uint32_t tokens, const float* next_norm_weight, void* next_normed,
                       const pbmoe_moe_debug* debug, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    int rc = check_moe_config(ctx, c);
    if (rc) return rc;
    if (!shard) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "ep moe layer: null shard");
    if (shard->expert_count == 0 || uint64_t(shard->expert_begin) + shard->expert_count > c->num_experts)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "ep moe layer: experts [%u, %u) outside 0..%u", shard->expert_begin,
                    shard->expert_begin + shard->expert_count, c->num_experts);
    if (!ctx->ep_base)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "ep moe layer: call pbmoe_ep_reserve first");
    if (tokens > ctx->ep_max_tokens || c->layout.hidden != ctx->ep_hidden)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "ep moe layer: exchange buffer reserved for tokens<=%u hidden=%u, "
                    "call needs tokens=%u hidden=%u", ctx->ep_max_tokens, ctx->ep_hidden, tokens, c->layout.hidden);
    for (uint32_t r = 0; r < ctx->ep_world; ++r)
        if (!ctx->ep_peer[r])
            return fail(ctx, PBMOE_ERR_PEER, "ep moe layer: rank %u's exchange buffer is not mapped "
                        "(pbmoe_ep_open_peers / pbmoe_ep_set_peers)", r);
    if (tokens == 0) return PBMOE_OK;
    pbmoe::EpPeers ep{};
    const size_t flags_off = pbmoe::ep_flags_offset(ctx->ep_world, ctx->ep_max_tokens, ctx->ep_hidden);
    for (uint32_t r = 0; r < ctx->ep_world; ++r) {
        ep.recv[r] = static_cast<float*>(ctx->ep_peer[r]);
        ep.flags[r] = reinterpret_cast<uint32_t*>(static_cast<char*>(ctx->ep_peer[r]) + flags_off);
    }
    ep.epoch = reinterpret_cast<uint32_t*>(static_cast<char*>(ctx->ep_base) +
                                           pbmoe::ep_epoch_offset(ctx->ep_world, ctx->ep_max_tokens, ctx->ep_hidden));
    ep.rank = ctx->ep_rank;
    ep.world = ctx->ep_world;
    ep.max_tokens = ctx->ep_max_tokens;
    ep.timeout_ns = shard->timeout_us ? uint64_t(shard->timeout_us) * 1000ull : 2000000000ull;
    if (debug && debug->phase_events)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "ep moe layer: phase events are not taken here");
    return moe_layer_impl(ctx, c, w, x, x_dtype, residual, out, out_dtype, tokens, next_norm_weight, next_normed,
                          debug, stream, shard->expert_begin, shard->expert_count, &ep);
}

// ---------------------------------------------------------------- vocab head
namespace {
struct HeadWs {
    float* logits;
    uint32_t *cand_key, *cand_id;
    float* cand_val;
    uint32_t* key_scratch;
};
size_t head_ws_bytes(uint32_t T, uint32_t V, uint32_t K, HeadWs* carve, void* base) {
    const size_t S = pbmoe::head_slices(V);
    const size_t sizes[5] = {size_t(T) * V * 4, size_t(T) * S * K * 4, size_t(T) * S * K * 4, size_t(T) * S * K * 4,
                             size_t(T) * K * 4};
    size_t off = 0;
    void* ptr[5];
    for (int i = 0; i < 5; ++i) {
        ptr[i] = base ? static_cast<char*>(base) + off : nullptr;
        off += (sizes[i] + 255) / 256 * 256;
    }
    if (carve) {
        carve->logits = static_cast<float*>(ptr[0]);
        carve->cand_key = static_cast<uint32_t*>(ptr[1]);
        carve->cand_id = static_cast<uint32_t*>(ptr[2]);
        carve->cand_val = static_cast<float*>(ptr[3]);
        carve->key_scratch = static_cast<uint32_t*>(ptr[4]);
    }
    return off;
}
}  // namespace

int pbmoe_head_reserve(pbmoe_ctx* ctx, uint32_t max_tokens, uint32_t vocab, uint32_t max_top_k) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (max_tokens == 0 || max_tokens > 32 || vocab == 0 || max_top_k == 0 || max_top_k > 256)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "head reserve: tokens %u (1..32), vocab %u, top_k %u (1..256)",
                    max_tokens, vocab, max_top_k);
    if (pbmoe::head_slices(vocab) * max_top_k > 24576)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported head top-k: %u slices x top_k %u exceed 24576",
                    pbmoe::head_slices(vocab), max_top_k);
    if (ctx->head_base && ctx->head_tokens >= max_tokens && ctx->head_vocab >= vocab && ctx->head_k >= max_top_k)
        return PBMOE_OK;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    if (ctx->head_base) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before head workspace resize");
        cudaFree(ctx->head_base);
        ctx->head_base = nullptr;
    }
    const size_t bytes = head_ws_bytes(max_tokens, vocab, max_top_k, nullptr, nullptr);
    cudaError_t e = cudaMalloc(&ctx->head_base, bytes);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "head workspace allocation");
    ctx->head_bytes = bytes;
    ctx->head_tokens = max_tokens;
    ctx->head_vocab = vocab;
    ctx->head_k = max_top_k;
    return PBMOE_OK;
}

int pbmoe_head_topk(pbmoe_ctx* ctx, const pbmoe_head* head, const void* x, pbmoe_dtype x_dtype, uint32_t tokens,
                    uint32_t top_k, const uint32_t* allowed, uint32_t* out_ids, float* out_values, uint32_t* out_keys,
                    float* out_logits, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!head || !head->weight || !x || !out_ids || !out_values)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "head top-k: null pointer");
    if (x_dtype != PBMOE_BF16 && x_dtype != PBMOE_F32)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "head top-k: x must be bf16 or f32");
    if (tokens == 0) return PBMOE_OK;
    if (top_k == 0) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "head top-k: top_k must be positive");
    if (!pbmoe::head_supported(head->vocab, head->hidden, tokens, top_k))
        return fail(ctx, PBMOE_ERR_UNSUPPORTED,
                    "FlashMoe unsupported head top-k: vocab %u, hidden %u (a multiple of 512), tokens %u (<= 32), "
                    "top_k %u (<= 256, slices of 2048 x top_k <= 24576)", head->vocab, head->hidden, tokens, top_k);
    if (!ctx->head_base || ctx->head_tokens < tokens || ctx->head_vocab < head->vocab || ctx->head_k < top_k)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "head top-k: %u tokens x vocab %u x top_k %u need pbmoe_head_reserve",
                    tokens, head->vocab, top_k);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    HeadWs w;
    head_ws_bytes(tokens, head->vocab, top_k, &w, ctx->head_base);
    pbmoe::HeadArgs a{};
    a.weight = head->weight;
    a.vocab = head->vocab;
    a.hidden = head->hidden;
    a.id_base = head->id_base;
    a.x = x;
    a.x_dtype = x_dtype;
    a.tokens = tokens;
    a.top_k = top_k;
    a.allowed = allowed;
    a.logits = w.logits;
    a.cand_key = w.cand_key;
    a.cand_id = w.cand_id;
    a.cand_val = w.cand_val;
    a.out_key = out_keys ? out_keys : w.key_scratch;
    a.out_id = out_ids;
    a.out_val = out_values;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = pbmoe::head_topk_launch(a, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "head top-k launch");
    if (out_logits) {
        e = cudaMemcpyAsync(out_logits, w.logits, size_t(tokens) * head->vocab * 4, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "head logits copy");
    }
    return PBMOE_OK;
}

int pbmoe_head_merge(pbmoe_ctx* ctx, const uint32_t* keys, const uint32_t* ids, const float* values, uint32_t lists,
                     uint32_t tokens, uint32_t top_k, uint32_t* out_ids, float* out_values, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!keys || !ids || !values || !out_ids || !out_values)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "head merge: null pointer");
    if (tokens == 0) return PBMOE_OK;
    if (lists == 0 || top_k == 0 || top_k > 256 || size_t(lists) * top_k > 24576 || lists + top_k - 1 > 512)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported head merge: %u lists x top_k %u", lists, top_k);
    if (!ctx->head_base || ctx->head_tokens < tokens || ctx->head_k < top_k)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "head merge: %u tokens x top_k %u need pbmoe_head_reserve", tokens,
                    top_k);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    HeadWs w;
    head_ws_bytes(ctx->head_tokens, ctx->head_vocab, ctx->head_k, &w, ctx->head_base);
    // [lists][tokens][top_k]: token stride top_k, list stride tokens x top_k
    cudaError_t e = pbmoe::head_merge_launch(keys, ids, values, tokens, lists, top_k, size_t(tokens) * top_k, top_k,
                                             w.key_scratch, out_ids, out_values, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "head merge launch");
    return PBMOE_OK;
}

// ---------------------------------------------------------------- decode-step glue
int pbmoe_rms_norm(pbmoe_ctx* ctx, const pbmoe_norm_args* a, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!a || !a->x || !a->out) return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "rms norm: null pointer");
    auto known = [](pbmoe_dtype t) { return t == PBMOE_F32 || t == PBMOE_BF16; };
    if (!known(a->x_dtype) || !known(a->out_dtype) || (a->sum_out && !known(a->sum_dtype)))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "rms norm: dtypes must be f32 or bf16");
    if (a->rows == 0) return PBMOE_OK;
    if (a->width == 0 || a->x_stride < a->width || a->out_stride < a->width ||
        (a->residual && a->residual_stride < a->width) || (a->sum_out && a->sum_stride < a->width) ||
        !(a->epsilon >= 0.0f))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "rms norm: width %u with strides x %u out %u", a->width,
                    a->x_stride, a->out_stride);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    pbmoe::NormArgs n{a->x,      a->x_dtype, a->residual, a->sum_out,   a->sum_dtype,       a->weight,
                      a->epsilon, a->out,    a->out_dtype, a->rows,     a->width,           a->x_stride,
                      a->residual_stride,    a->sum_stride, a->out_stride};
    cudaError_t e = pbmoe::rms_norm_launch(n, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rms norm launch");
    return PBMOE_OK;
}

int pbmoe_rope_reserve(pbmoe_ctx* ctx, uint32_t max_positions, uint32_t rope_dim, double theta) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (max_positions == 0 || rope_dim == 0 || rope_dim % 2 || !(theta > 0.0))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "rope reserve: %u positions, rope dim %u (even), theta %g",
                    max_positions, rope_dim, theta);
    const uint32_t half = rope_dim / 2;
    std::vector<float2> table(size_t(max_positions) * half);
    for (uint32_t pair = 0; pair < half; ++pair) {
        const double frequency = std::pow(theta, -static_cast<double>(2 * pair) / static_cast<double>(rope_dim));
        for (uint32_t pos = 0; pos < max_positions; ++pos) {
            const double angle = static_cast<double>(pos) * frequency;
            table[size_t(pos) * half + pair] = make_float2(static_cast<float>(std::cos(angle)),
                                                           static_cast<float>(std::sin(angle)));
        }
    }
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    if (ctx->rope_table) {
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before rope table resize");
        cudaFree(ctx->rope_table);
        ctx->rope_table = nullptr;
    }
    cudaError_t e = cudaMalloc(&ctx->rope_table, table.size() * sizeof(float2));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rope table allocation");
    e = cudaMemcpy(ctx->rope_table, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rope table upload");
    ctx->rope_positions = max_positions;
    ctx->rope_dim = rope_dim;
    return PBMOE_OK;
}

int pbmoe_mla_rope_append(pbmoe_ctx* ctx, const pbmoe_mla_config* cfg, uint32_t batch, float* query, const float* kv,
                          const float* latent_norm_weight, float epsilon, const uint32_t* positions,
                          uint16_t* const* c_kv, uint16_t* const* k_rope, uint32_t cache_len, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!cfg || !query || !kv || !positions || !c_kv || !k_rope)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla rope append: null pointer");
    if (latent_norm_weight && (!(epsilon >= 0.f) || !std::isfinite(epsilon)))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mla rope append: norm epsilon must be finite and >= 0");
    if (batch == 0) return PBMOE_OK;
    if (!ctx->rope_table || ctx->rope_dim != cfg->rope_dim)
        return fail(ctx, PBMOE_ERR_NO_WORKSPACE, "mla rope append: rope dim %u needs pbmoe_rope_reserve",
                    cfg->rope_dim);
    if (!pbmoe::rope_append_supported(cfg->heads, cfg->rope_dim) || cfg->latent_dim == 0 ||
        cfg->latent_dim > 1024 || cache_len == 0)
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported MLA RoPE append: %u heads x rope %u, latent %u",
                    cfg->heads, cfg->rope_dim, cfg->latent_dim);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    pbmoe::RopeAppendArgs a{};
    a.batch = batch;
    a.heads = cfg->heads;
    a.nope = cfg->nope_dim;
    a.rope = cfg->rope_dim;
    a.latent = cfg->latent_dim;
    a.query = query;
    a.kv = kv;
    a.latent_norm_w = latent_norm_weight;
    a.eps = epsilon;
    a.positions = positions;
    a.c_kv = c_kv;
    a.k_rope = k_rope;
    a.cache_len = cache_len;
    a.table = ctx->rope_table;
    a.max_positions = ctx->rope_positions;
    a.status = ctx->status;
    cudaError_t e = pbmoe::mla_rope_append_launch(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "mla rope append launch");
    return PBMOE_OK;
}

// ---------------------------------------------------------------- expert store
int pbmoe_expert_layer_load(pbmoe_ctx* ctx, const char* root, uint32_t layer, const pbmoe_expert_layout* layout,
                            uint32_t expert_begin, uint32_t expert_count, void* device_dst, size_t dst_bytes,
                            void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    char msg[512] = {0};
    const int rc = pbmoe::expert_layer_upload(root, layer, layout, expert_begin, expert_count, device_dst, dst_bytes,
                                              static_cast<cudaStream_t>(stream), msg, sizeof msg);
    if (rc != PBMOE_OK) return fail(ctx, rc, "%s", msg);
    return PBMOE_OK;
}

// ---------------------------------------------------------------- MXFP4
int pbmoe_mxfp4_matvec(pbmoe_ctx* ctx, const pbmoe_mxfp4_tensor* w, const void* x, pbmoe_dtype x_dtype, void* y,
                       pbmoe_dtype y_dtype, uint32_t batch, void* stream) {
    if (!ctx) return PBMOE_ERR_INVALID_ARGUMENT;
    if (!w || !w->packed || !w->scales || !x || !y)
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mxfp4 matvec: null pointer");
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16) || (y_dtype != PBMOE_F32 && y_dtype != PBMOE_BF16))
        return fail(ctx, PBMOE_ERR_INVALID_ARGUMENT, "mxfp4 matvec: dtypes must be f32 or bf16");
    if (batch == 0 || w->rows == 0) return PBMOE_OK;
    if (!pbmoe::mxfp4_supported(w->rows, w->cols, w->group_size, batch) || !aligned(w->packed, 16))
        return fail(ctx, PBMOE_ERR_UNSUPPORTED, "FlashMoe unsupported MXFP4 matvec: %u x %u, group %u (needs group 32, "
                    "cols a multiple of 32, 16-byte aligned rows)", w->rows, w->cols, w->group_size);
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(ctx, PBMOE_ERR_CUDA, "cannot select device %d", ctx->device);
    pbmoe::Mxfp4Args a{static_cast<const uint8_t*>(w->packed), w->scales, w->rows, w->cols, w->group_size, batch,
                       x, x_dtype, y, y_dtype, ctx->status};
    cudaError_t e = pbmoe::mxfp4_matvec_launch(a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "mxfp4 matvec launch");
    return PBMOE_OK;
}
