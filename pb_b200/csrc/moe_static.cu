// moe_static.cu — pbmoe_moe_layer_static: the MoE FFN decode layer for callers
// that may not allocate device memory.
//
// Some hosts cannot call cudaMalloc once they are running: an engine whose
// device memory is handed out by its own fixed arena or pool (so a foreign
// allocation would break its accounting or fail outright when the pool owns
// the whole GPU), code that runs while a CUDA graph is being captured (where
// allocation calls are not allowed), or a latency-critical loop that must not
// take the implicit device synchronisation cudaMalloc/cudaFree can cause.
// Such callers also cannot use pbmoe_init, which allocates the context's
// status word, so this entry point needs no context at all.
//
// Its scratch (the same workspace pbmoe_moe_layer carves out of
// pbmoe_reserve's allocation) lives in g_moe_static_scratch below, a
// file-scope __device__ array of kStaticScratchBytes. The CUDA runtime creates
// it with the module, so every GPU on which this library's kernels are loaded
// holds those bytes until the process exits. Calls that need more workspace
// than that are rejected.
//
// Host code must not pass &g_moe_static_scratch to a kernel: on the host that
// name is only a stand-in for the device symbol (a kernel given it would fault,
// or silently touch host memory where the GPU can reach it). The device
// address is looked up once per device with cudaGetSymbolAddress, with that
// device current, by the first call made on the device; make that first call
// before any stream capture begins.
//
// Every call shares the one array and leaves its contents behind for the next
// call. The kernels fully rewrite what they read except the router kernel's
// arrival counter and the status word, which this entry point zeroes on the
// stream before launching. Calls whose kernels may overlap on the GPU (other
// streams, other host threads) race on the array and must be serialised by the
// caller.

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "kernels.h"
#include "q4_rows.cuh"

namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // PBMOE_STATIC_SCRATCH_BYTES
constexpr size_t kStatusBytes = 256;                      // status word, then the workspace
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_moe_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

int report(char* buf, size_t len, int code, const char* fmt, ...) {
    if (buf && len) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, len, fmt, ap);
        va_end(ap);
    }
    return code;
}

// Device address of the scratch array on the current device (resolved once).
cudaError_t scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_addr[device] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_moe_static_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return cudaSuccess;
}

}  // namespace

using namespace pbmoe;

extern "C" PBMOE_API int pbmoe_moe_layer_static(const pbmoe_moe_config* c, const pbmoe_moe_weights* w,
                                                const void* x, pbmoe_dtype x_dtype, const void* residual,
                                                void* out, pbmoe_dtype out_dtype, uint32_t tokens,
                                                const float* next_norm_weight, void* next_normed,
                                                uint32_t* device_status, char* error_buf, size_t error_len,
                                                void* stream) {
    if (error_buf && error_len) error_buf[0] = '\0';
    if (!c || !w || !w->router_weight || !w->experts || !x || !out)
        return report(error_buf, error_len, PBMOE_ERR_INVALID_ARGUMENT, "moe layer (static): null pointer");
    const pbmoe_expert_layout& L = c->layout;
    const uint32_t H = L.hidden, I = L.intermediate, G = L.group_size, E = c->num_experts, K = c->top_k;
    {  // the same layout and config checks as pbmoe_moe_layer
        char msg[512];
        const int rc = moe_check_config(c, msg, sizeof msg);
        if (rc != PBMOE_OK) return report(error_buf, error_len, rc, "%s", msg);
    }
    if ((x_dtype != PBMOE_F32 && x_dtype != PBMOE_BF16) || (out_dtype != PBMOE_F32 && out_dtype != PBMOE_BF16))
        return report(error_buf, error_len, PBMOE_ERR_INVALID_ARGUMENT, "unknown dtype");
    if ((next_norm_weight == nullptr) != (next_normed == nullptr) || (w->shared_expert_gate && !w->shared_expert))
        return report(error_buf, error_len, PBMOE_ERR_INVALID_ARGUMENT, "inconsistent optional arguments");
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w->experts) % 16 ||
        reinterpret_cast<uintptr_t>(w->router_weight) % 16 ||
        (w->shared_expert && reinterpret_cast<uintptr_t>(w->shared_expert) % 16) ||
        (w->shared_expert_gate && reinterpret_cast<uintptr_t>(w->shared_expert_gate) % 16) ||
        (w->input_norm_weight && reinterpret_cast<uintptr_t>(w->input_norm_weight) % 16) ||
        (w->router_correction_bias && reinterpret_cast<uintptr_t>(w->router_correction_bias) % 16))
        return report(error_buf, error_len, PBMOE_ERR_INVALID_ARGUMENT,
                      "moe layer (static): x, experts, router and shared weights must be 16-byte aligned");
    if (tokens == 0) return PBMOE_OK;
    const size_t need = kStatusBytes + moe_ws_sizes(tokens, E, K, H, I).total;
    if (need > kStaticScratchBytes)
        return report(error_buf, error_len, PBMOE_ERR_UNSUPPORTED,
                      "moe layer (static): %u tokens need %zu scratch bytes, more than the fixed %zu-byte array "
                      "(use pbmoe_moe_layer with pbmoe_reserve)",
                      tokens, need, kStaticScratchBytes);
    if (moe_router_smem(tokens, H, E, K) > kRouterSmemLimit)
        return report(error_buf, error_len, PBMOE_ERR_UNSUPPORTED, "router staging exceeds shared memory");

    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess || device < 0 || device >= kMaxDevices)
        return report(error_buf, error_len, PBMOE_ERR_CUDA, "no usable current CUDA device");
    void* base = nullptr;
    e = scratch_address(device, &base);
    if (e != cudaSuccess)
        return report(error_buf, error_len, PBMOE_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s",
                      cudaGetErrorString(e));

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t* status = device_status ? device_status : static_cast<uint32_t*>(base);
    MoeLaunch a{};
    a.ws = moe_ws_carve(static_cast<char*>(base) + kStatusBytes, status, tokens, E, K, H, I);
    // state that must start at zero: the router's arrival counter (and the
    // status word when it lives in the array)
    e = cudaMemsetAsync(a.ws.ticket, 0, 2 * sizeof(uint32_t), s);
    if (e == cudaSuccess && !device_status) e = cudaMemsetAsync(base, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess)
        return report(error_buf, error_len, PBMOE_ERR_CUDA, "scratch clear failed: %s", cudaGetErrorString(e));
    for (int i = 0; i < 9; ++i) a.layout.off[i] = L.component_offsets[i];
    a.layout.expert_bytes = L.expert_bytes;
    a.layout.hidden = H;
    a.layout.inter = I;
    a.layout.group = G;
    a.layout.cpg_shift_h = ilog2_u32(G / 32);
    a.layout.cpg_shift_i = ilog2_u32(G / 32);
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
    a.pdl = false;  // the memset above must complete before the router kernel reads the counter
    a.phase_events = nullptr;
    e = moe_layer_launch(a, s);
    if (e != cudaSuccess)
        return report(error_buf, error_len, PBMOE_ERR_CUDA, "moe layer (static) launch failed: %s",
                      cudaGetErrorString(e));
    return PBMOE_OK;
}
