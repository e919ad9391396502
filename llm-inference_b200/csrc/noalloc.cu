// Batched split-KV attention with its scratch in a fixed device array instead of a caller buffer.
//
// Some callers cannot allocate device memory on the decode path: a host runtime that owns every
// cudaMalloc up front (a fixed memory pool sized at start-up), a plugin called from inside
// another framework's allocator-controlled region, or code that runs where an allocation would
// synchronize the device or could fail part-way through serving. q3_attention_batched needs a
// scratch buffer (scores, softmax statistics, per-chunk partial outputs); this entry point takes
// that scratch from `g_attn_scratch`, a file-scope device array that every GPU loading the
// library holds until the process exits, and runs exactly the same kernels.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace q3 {

int check_device();
int attention_check(int n_heads, int n_kv_heads, int head_dim, int max_seq, int n_rows);
int score_ld(int max_seq);
size_t attention_scratch_layout(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq, AttnSplit *sp,
                                float **scores, void *base);
int attention(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *scores, int ld,
              const int *pos, int n_rows, long long q_stride, KvLayout kv, int n_heads, int n_kv_heads,
              int head_dim, int max_seq, float scale, const AttnSplit *split, cudaStream_t s);

namespace {

// The scratch itself. Host code must not pass this name to a kernel: on the host it only stands
// for the symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_attn_scratch[Q3_ATTENTION_STATIC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void *g_addr[MAX_DEVICES] = {};
void *g_ctx[MAX_DEVICES] = {};  // the context g_addr[dev] was looked up in

// The current context (CUcontext) through the driver entry point, so the library needs no -lcuda.
void *current_context() {
    typedef int (*GetCurrent)(void **);
    static GetCurrent fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        fn = reinterpret_cast<GetCurrent>(p);
    }
    void *ctx = nullptr;
    return fn(&ctx) == 0 ? ctx : nullptr;
}

// Device address of g_attn_scratch on the current device, looked up once per device and context:
// the first call on a device (and the first after a cudaDeviceReset, which replaces the context and
// reloads the module at a possibly different address) does the lookup. The lookup can load the
// module, so that first call should come before any stream capture.
int scratch_address(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (dev < 0 || dev >= MAX_DEVICES) return Q3_ERR_DEVICE;
    void *ctx = current_context();
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev] || ctx == nullptr || ctx != g_ctx[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p) return record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
        g_addr[dev] = p;
        g_ctx[dev] = current_context();  // the lookup made the device's context current if none was
    }
    *out = g_addr[dev];
    return Q3_OK;
}

}  // namespace
}  // namespace q3

using namespace q3;

extern "C" int q3_attention_batched_static(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *key_cache,
                                           const q3_bf16 *value_cache, long long cache_seq_stride,
                                           long long cache_pos_stride, long long cache_head_stride,
                                           const int *d_pos, int batch, int n_heads, int n_kv_heads, int head_dim,
                                           int max_seq, float scale, void *stream) {
    int st = check_device();
    if (st != Q3_OK) return st;
    st = attention_check(n_heads, n_kv_heads, head_dim, max_seq, batch);
    if (st != Q3_OK) return st;
    const size_t need = attention_scratch_layout(batch, n_heads, n_kv_heads, head_dim, max_seq, nullptr, nullptr,
                                                 nullptr);
    if (need > (size_t)Q3_ATTENTION_STATIC_SCRATCH_BYTES) return Q3_ERR_SCRATCH_LIMIT;
    void *scratch = nullptr;
    st = scratch_address(&scratch);
    if (st != Q3_OK) return st;
    // Every scratch value the kernels use is written earlier in the same call (the bulk copies
    // also read a few padding bytes next to those values, which no kernel uses), so what a
    // previous call left in the array needs no clearing.
    AttnSplit sp;
    float *scores = nullptr;
    attention_scratch_layout(batch, n_heads, n_kv_heads, head_dim, max_seq, &sp, &scores, scratch);
    const KvLayout kv = {cache_seq_stride, cache_pos_stride, cache_head_stride};
    return attention(reinterpret_cast<bf16 *>(out), reinterpret_cast<const bf16 *>(q),
                     reinterpret_cast<const bf16 *>(key_cache), reinterpret_cast<const bf16 *>(value_cache), scores,
                     score_ld(max_seq), d_pos, batch, (long long)n_heads * head_dim, kv, n_heads, n_kv_heads,
                     head_dim, max_seq, scale, &sp, reinterpret_cast<cudaStream_t>(stream));
}
