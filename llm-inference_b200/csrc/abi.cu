// The C ABI of libqwen3_b200.so (include/qwen3_b200.h): argument checks, device checks and
// dispatch to the kernels. Launchers never allocate or synchronize.
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace q3 {

// kernels (gemv.cu, decode_kernels.cu, attention.cu)
int gemv_plain(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t s);
int gemv_residual(bf16 *x, const bf16 *w, const bf16 *in, int rows, int cols, bf16 *tap, cudaStream_t s);
int gemv_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x,
             int q_rows, int kv_rows, int cols, cudaStream_t s);
int gemv_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                 bf16 *gate_tap, bf16 *up_tap, cudaStream_t s);
int embedding(bf16 *out, const bf16 *table, const int *tokens, int n_rows, int hidden, int vocab,
              cudaStream_t s);
int rmsnorm(bf16 *out, const bf16 *in, const bf16 *weight, int rows, int dim, float eps, cudaStream_t s);
int qk_norm_rope(bf16 *q, bf16 *k, const bf16 *v, const bf16 *q_norm_w, const bf16 *k_norm_w,
                 bf16 *key_cache, bf16 *value_cache, const int *pos, int n_rows, long long q_stride,
                 long long kv_stride, KvLayout kv, int n_heads, int n_kv_heads, int head_dim,
                 int max_seq, float eps, float theta, bf16 *q_tap, bf16 *k_tap, cudaStream_t s);
int argmax_rows(const bf16 *x, int n, int n_rows, long long row_stride, int *out, int *next_token,
                int *pos, int *history, int *step, int history_cap, cudaStream_t s);
int sample(int *out, const bf16 *x, int n, float inv_temp, float u, cudaStream_t s);
int attention(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *scores, int ld,
              const int *pos, int n_rows, long long q_stride, KvLayout kv, int n_heads, int n_kv_heads,
              int head_dim, int max_seq, float scale, const AttnSplit *split, cudaStream_t s);
unsigned take_error_gemv();
unsigned take_error_decode();
unsigned take_error_attention();
unsigned take_error_tc();
unsigned take_error_stream();
unsigned take_error_attn_fused();
unsigned take_error_selftest();

namespace {
constexpr int MAX_DEVICES = 64;
thread_local int t_last_cuda_error = 0;
std::mutex g_mu;
int g_sms[MAX_DEVICES];
int g_arch_ok[MAX_DEVICES];  // 0 unknown, 1 sm_100, -1 other

struct SmemEntry {
    const void *kernel;
    int device;
    size_t bytes;
};
SmemEntry g_smem[256];
int g_n_smem = 0;

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d < 0 || d >= MAX_DEVICES ? 0 : d;
}
}  // namespace

int record_cuda_error(cudaError_t e) {
    if (e == cudaSuccess) return Q3_OK;
    t_last_cuda_error = (int)e;
    cudaGetLastError();  // a failed call leaves a non-sticky error pending: clear it for other users
    return Q3_ERR_CUDA;
}

int num_sms() {
    const int d = current_device();
    if (g_sms[d] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
        g_sms[d] = n > 0 ? n : 148;
    }
    return g_sms[d];
}

cudaError_t allow_smem(const void *kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    const int d = current_device();
    std::lock_guard<std::mutex> lock(g_mu);
    for (int i = 0; i < g_n_smem; i++)
        if (g_smem[i].kernel == kernel && g_smem[i].device == d) {
            if (g_smem[i].bytes >= bytes) return cudaSuccess;
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
            if (e == cudaSuccess) g_smem[i].bytes = bytes;
            return e;
        }
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess && g_n_smem < 256) g_smem[g_n_smem++] = {kernel, d, bytes};
    return e;
}

// The kernels use sm_100a instructions (tcgen05, bulk copies with L2 hints, clusters).
int check_device() {
    const int d = current_device();
    if (g_arch_ok[d] == 0) {
        int major = 0, minor = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) != cudaSuccess)
            return record_cuda_error(cudaGetLastError());
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d);
        g_arch_ok[d] = (major == 10 && minor == 0) ? 1 : -1;
    }
    return g_arch_ok[d] == 1 ? Q3_OK : Q3_ERR_DEVICE;
}

}  // namespace q3

using q3::check_device;

#define B(p) reinterpret_cast<bf16 *>(p)
#define CB(p) reinterpret_cast<const bf16 *>(p)
#define S(p) reinterpret_cast<cudaStream_t>(p)
#define DEVICE_OR_RETURN()             \
    do {                               \
        int st_ = check_device();      \
        if (st_ != Q3_OK) return st_;  \
    } while (0)

extern "C" {

const char *q3_status_string(int status) {
    switch (status) {
        case Q3_OK: return "ok";
        case Q3_ERR_SHAPE: return "a size violates a precondition";
        case Q3_ERR_ALIGN: return "a pointer is not 16-byte aligned";
        case Q3_ERR_CUDA: return "a CUDA call failed";
        case Q3_ERR_DEVICE: return "the current device is not sm_100 (B200)";
        case Q3_ERR_ARG: return "a null pointer or an invalid option";
        case Q3_ERR_SCRATCH_LIMIT: return "the shape needs more scratch than the static scratch array holds";
        default: return "unknown status";
    }
}

int q3_last_cuda_error(void) { return q3::t_last_cuda_error; }

int q3_device_error(void *stream, unsigned *flags) {
    if (!flags) return Q3_ERR_ARG;
    cudaError_t e = cudaStreamSynchronize(S(stream));
    if (e != cudaSuccess) return q3::record_cuda_error(e);
    *flags = q3::take_error_gemv() | q3::take_error_decode() | q3::take_error_attention() | q3::take_error_tc() |
             q3::take_error_stream() | q3::take_error_attn_fused() | q3::take_error_selftest();
    return Q3_OK;
}

int q3_embedding_forward(q3_bf16 *out, const q3_bf16 *table, const int *d_token, int hidden, void *stream) {
    DEVICE_OR_RETURN();
    return q3::embedding(B(out), CB(table), d_token, 1, hidden, 0, S(stream));
}

int q3_rmsnorm_forward(q3_bf16 *out, const q3_bf16 *in, const q3_bf16 *weight, int rows, int dim, float eps,
                       void *stream) {
    DEVICE_OR_RETURN();
    return q3::rmsnorm(B(out), CB(in), CB(weight), rows, dim, eps, S(stream));
}

int q3_gemv_forward(q3_bf16 *out, const q3_bf16 *w, const q3_bf16 *x, int rows, int cols, void *stream) {
    DEVICE_OR_RETURN();
    return q3::gemv_plain(B(out), CB(w), CB(x), rows, cols, S(stream));
}

int q3_gemv_residual_forward(q3_bf16 *x, const q3_bf16 *w, const q3_bf16 *in, int rows, int cols,
                             q3_bf16 *tap, void *stream) {
    DEVICE_OR_RETURN();
    return q3::gemv_residual(B(x), CB(w), CB(in), rows, cols, B(tap), S(stream));
}

int q3_qkv_forward(q3_bf16 *q, q3_bf16 *k, q3_bf16 *v, const q3_bf16 *wq, const q3_bf16 *wk,
                   const q3_bf16 *wv, const q3_bf16 *x, int q_rows, int kv_rows, int cols, void *stream) {
    DEVICE_OR_RETURN();
    return q3::gemv_qkv(B(q), B(k), B(v), CB(wq), CB(wk), CB(wv), CB(x), q_rows, kv_rows, cols, S(stream));
}

int q3_gate_up_forward(q3_bf16 *act, const q3_bf16 *w_gate, const q3_bf16 *w_up, const q3_bf16 *x,
                       int rows, int cols, q3_bf16 *gate_tap, q3_bf16 *up_tap, void *stream) {
    DEVICE_OR_RETURN();
    return q3::gemv_gate_up(B(act), CB(w_gate), CB(w_up), CB(x), rows, cols, B(gate_tap), B(up_tap),
                            S(stream));
}

int q3_qk_norm_rope_forward(q3_bf16 *q, q3_bf16 *k, const q3_bf16 *v, const q3_bf16 *q_norm_w,
                            const q3_bf16 *k_norm_w, q3_bf16 *key_cache, q3_bf16 *value_cache,
                            const int *d_pos, int n_heads, int n_kv_heads, int head_dim, float eps,
                            float theta, q3_bf16 *q_tap, q3_bf16 *k_tap, void *stream) {
    DEVICE_OR_RETURN();
    const long long qd = (long long)n_heads * head_dim, kvd = (long long)n_kv_heads * head_dim;
    const q3::KvLayout kv = {0, kvd, head_dim};  // the reference's [max_seq][n_kv * head_dim] cache
    return q3::qk_norm_rope(B(q), B(k), CB(v), CB(q_norm_w), CB(k_norm_w), B(key_cache), B(value_cache),
                            d_pos, 1, qd, kvd, kv, n_heads, n_kv_heads, head_dim, 0, eps, theta, B(q_tap),
                            B(k_tap), S(stream));
}

int q3_attention_forward(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *key_cache,
                         const q3_bf16 *value_cache, float *att, int n_heads, int n_kv_heads, int head_dim,
                         const int *d_pos, int max_seq, float scale, void *stream) {
    DEVICE_OR_RETURN();
    const q3::KvLayout kv = {0, (long long)n_kv_heads * head_dim, head_dim};
    return q3::attention(B(out), CB(q), CB(key_cache), CB(value_cache), att, max_seq, d_pos, 1,
                         (long long)n_heads * head_dim, kv, n_heads, n_kv_heads, head_dim, max_seq, scale,
                         nullptr, S(stream));
}

int q3_argmax_forward(int *out, const q3_bf16 *x, int n, void *stream) {
    DEVICE_OR_RETURN();
    return q3::argmax_rows(CB(x), n, 1, 0, out, nullptr, nullptr, nullptr, nullptr, 0, S(stream));
}

int q3_sample_forward(int *out, const q3_bf16 *x, int n, float inv_temp, float u, void *stream) {
    DEVICE_OR_RETURN();
    return q3::sample(out, CB(x), n, inv_temp, u, S(stream));
}

}  // extern "C"
