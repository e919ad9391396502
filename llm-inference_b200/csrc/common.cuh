// Shared device helpers for the sm_100a decode kernels: bf16 types, error reporting,
// mbarrier / bulk-copy / programmatic-dependent-launch PTX wrappers and a launch helper.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/qwen3_b200.h"

typedef __nv_bfloat16 bf16;

namespace q3 {

// ------------------------------------------------------------------ errors
//
// Every translation unit has its own device error word (internal linkage). A kernel whose
// bounded wait gives up ORs a code into it and returns; q3_device_error() collects the
// words of all units. Codes are bit flags so several failures stay visible.
enum DeviceError : unsigned {
    DEV_ERR_WAIT_TIMEOUT = 1u << 0,   // an mbarrier wait passed its time limit
    DEV_ERR_TOKEN_RANGE = 1u << 1,    // a token id outside [0, vocab) reached a gather
    DEV_ERR_POS_RANGE = 1u << 2,      // a position outside [0, max_seq) reached a kernel
    DEV_ERR_TMEM = 1u << 3,           // tensor-memory allocation gave back a bad address
};

// Give up an mbarrier wait after this long (the kernels' waits normally end in microseconds).
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

// ------------------------------------------------------------------ small helpers

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16(v)); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The dynamic shared-memory base rounded up to a multiple of A bytes (the swizzled TMA tiles
// want 1024). The offset is added to the shared array's own pointer, so the compiler still
// knows that every pointer derived from the result is in shared memory and emits shared loads.
// Rounding through an integer cast would lose that, and every access would become a generic
// load, which the hardware must resolve at run time.
template <int A>
__device__ __forceinline__ unsigned char *align_shared(unsigned char *base) {
    return base + ((A - (smem_u32(base) & (A - 1))) & (A - 1));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ programmatic dependent launch
//
// A kernel launched with programmatic stream serialization may start while its predecessor
// still runs. Every kernel here touches activations only after pdl_wait(), which returns once
// the predecessor grid has completed and its writes are visible; loads of constant weights
// may be issued before it. pdl_trigger() lets the successor be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ mbarriers

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later async-proxy
// (bulk copy / TMA / tensor core) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false, after setting
// DEV_ERR_WAIT_TIMEOUT in *err, if that takes longer than WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t start = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - start > WAIT_LIMIT_NS) {
            atomicOr(err, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------------------ bulk copies (no tensor map)

// Global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same with an L2 eviction-priority hint (policy from createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void *dst_smem, const void *src, uint32_t bytes,
                                              uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
        "%2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ------------------------------------------------------------------ bf16x8 helpers

struct alignas(16) bf16x8 {
    __nv_bfloat162 h[4];
};

__device__ __forceinline__ bf16x8 lds128(const void *p) { return *reinterpret_cast<const bf16x8 *>(p); }

__device__ __forceinline__ bf16x8 ldg128(const void *p) {
    uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
    return *reinterpret_cast<bf16x8 *>(&u);
}

// sum = fma(w[e], x[e], sum) for e = 0..7, in element order: the per-chunk order of the
// reference's warp_dot (src/kernels.cu:92-99), where nvcc fuses `sum += a * b`.
__device__ __forceinline__ float dot8(const bf16x8 &w, const bf16x8 &x, float sum) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float2 a = __bfloat1622float2(w.h[k]);
        float2 b = __bfloat1622float2(x.h[k]);
        sum = __fmaf_rn(a.x, b.x, sum);
        sum = __fmaf_rn(a.y, b.y, sum);
    }
    return sum;
}

// ------------------------------------------------------------------ launch helper

// Launches with programmatic stream serialization (and an optional cluster shape).
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   int cluster_x, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    int n = 0;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
    if (cluster_x > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = cluster_x;
        attrs[n].val.clusterDim.y = 1;
        attrs[n].val.clusterDim.z = 1;
        n++;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Element strides of a KV cache: sequence b, position t, kv head h start at
// cache + b*seq + t*pos + h*head. The reference's per-layer cache is [max_seq][n_kv*head_dim]
// (pos = n_kv*head_dim, head = head_dim); the engine's is head-major, [n_kv][max_seq][head_dim]
// per sequence (pos = head_dim, head = max_seq*head_dim), so each head's positions are
// contiguous in memory.
struct KvLayout {
    long long seq, pos, head;
};

// Batch-1 decode step as one persistent kernel (decode_stream.cu): per-layer weight pointers
// and the step's buffers, filled by the engine.
struct MkLayer {
    const bf16 *attn_norm, *wq, *wk, *wv, *q_norm, *k_norm, *wo, *mlp_norm, *w_gate, *w_up, *w_down;
};

constexpr int DS_STAGE_BYTES = 40960;  // one stage of the weight ring: whole rows, 8 of 5 KB, 2 of 19 KB
constexpr int DS_MAX_STAGES = 8;

struct DsParams {
    const MkLayer *layers;  // device array [n_layers]
    const bf16 *embed, *final_norm, *lm_head;
    int n_layers, H, I, n_heads, n_kv, vocab;  // head_dim is 128
    float eps, theta, scale;
    bf16 *x, *q, *k, *v, *attn_out, *act, *logits;
    bf16 *key_cache, *value_cache;  // layer l at + l * layer_stride; [n_kv][max_seq][128]
    long long layer_stride;
    int max_seq;
    float *scores;   // [n_heads][ld]
    int ld;
    float *cmax;     // [n_kv][chunks][n_heads / n_kv] chunk maxima
    float *csum;     // [n_kv][n_heads / n_kv * 128] softmax sum chains
    float *partial;  // [n_kv][chunks][n_heads / n_kv][128] P.V partial sums
    float *amax_val;  // [grid]
    int *amax_idx;
    unsigned *sync;  // barrier counters and the error word (decode_stream_sync_words), zero at rest
    int *next_token, *pos, *out_token, *history, *step;
    int history_cap;
    int stages;      // weight-ring depth (decode_stream_plan)
    int chunks;      // attention CTAs per kv head (decode_stream_plan)
};

int decode_stream_plan(DsParams &p);  // grid (one CTA per SM), or 0 if the shapes do not fit
int decode_stream_launch(const DsParams &p, int grid, cudaStream_t s);
int decode_stream_sync_words(int n_kv);

// Scratch of the split-KV attention (attention.cu): softmax statistics and per-chunk partial
// outputs (the counters are unused).
struct AttnSplit {
    float *stats;
    float *partial;
    int *count_a, *count_b;
    int chunk_b, max_chunks;
};

int num_sms();               // SM count of the current device (cached per device)
// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device (cached, so
// repeated launches make no runtime call; safe during stream capture).
cudaError_t allow_smem(const void *kernel, size_t bytes);
int record_cuda_error(cudaError_t e);  // remembers e for q3_last_cuda_error(); returns Q3_ERR_CUDA or Q3_OK

}  // namespace q3

#define Q3_TRY_LAUNCH(expr)                                   \
    do {                                                      \
        cudaError_t e_ = (expr);                              \
        if (e_ != cudaSuccess) return q3::record_cuda_error(e_); \
    } while (0)
