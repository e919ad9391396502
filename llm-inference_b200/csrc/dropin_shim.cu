// The reference's C++ launcher names, exported by libqwen3_b200.so so that the reference host
// code (src/forward.cu, src/main.cu) links against this library instead of src/kernels.cu.
//
// The ten declarations below are the interface of src/kernels.cuh:7-26 -- same names, same
// parameter types, hence the same mangled symbols. Each forwards to the q3_ C entry point and
// keeps the reference's error behaviour: a message on stderr and exit(EXIT_FAILURE) on a bad
// shape (src/kernels.cu:147-152, :392-396) or a failed launch (src/common.cuh:11-22).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>

#include "../../include/qwen3_b200.h"

typedef __nv_bfloat16 bf16;

namespace {
void check(const char *name, int status) {
    if (status == Q3_OK) return;
    if (status == Q3_ERR_CUDA)
        fprintf(stderr, "CUDA error in %s: %s\n", name, cudaGetErrorString((cudaError_t)q3_last_cuda_error()));
    else
        fprintf(stderr, "%s: %s\n", name, q3_status_string(status));
    exit(EXIT_FAILURE);
}
q3_bf16 *P(bf16 *p) { return reinterpret_cast<q3_bf16 *>(p); }
const q3_bf16 *P(const bf16 *p) { return reinterpret_cast<const q3_bf16 *>(p); }
}  // namespace

void embedding_forward(bf16 *out, const bf16 *table, const int *d_token, int hidden, cudaStream_t stream) {
    check("embedding", q3_embedding_forward(P(out), P(table), d_token, hidden, stream));
}

void rmsnorm_forward(bf16 *out, const bf16 *in, const bf16 *weight, int rows, int dim, float eps,
                     cudaStream_t stream) {
    check("rmsnorm", q3_rmsnorm_forward(P(out), P(in), P(weight), rows, dim, eps, stream));
}

void gemv_forward(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t stream) {
    check("gemv", q3_gemv_forward(P(out), P(w), P(x), rows, cols, stream));
}

void gemv_residual_forward(bf16 *x, const bf16 *w, const bf16 *in, int rows, int cols, bf16 *tap,
                           cudaStream_t stream) {
    check("gemv_residual", q3_gemv_residual_forward(P(x), P(w), P(in), rows, cols, P(tap), stream));
}

void qkv_forward(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x,
                 int q_rows, int kv_rows, int cols, cudaStream_t stream) {
    check("qkv", q3_qkv_forward(P(q), P(k), P(v), P(wq), P(wk), P(wv), P(x), q_rows, kv_rows, cols, stream));
}

void gate_up_forward(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                     bf16 *gate_tap, bf16 *up_tap, cudaStream_t stream) {
    check("gate_up", q3_gate_up_forward(P(act), P(w_gate), P(w_up), P(x), rows, cols, P(gate_tap),
                                        P(up_tap), stream));
}

void qk_norm_rope_forward(bf16 *q, bf16 *k, const bf16 *v, const bf16 *q_norm_w, const bf16 *k_norm_w,
                          bf16 *key_cache, bf16 *value_cache, const int *d_pos, int n_heads, int n_kv_heads,
                          int head_dim, float eps, float theta, bf16 *q_tap, bf16 *k_tap, cudaStream_t stream) {
    check("qk_norm_rope", q3_qk_norm_rope_forward(P(q), P(k), P(v), P(q_norm_w), P(k_norm_w), P(key_cache),
                                                  P(value_cache), d_pos, n_heads, n_kv_heads, head_dim, eps,
                                                  theta, P(q_tap), P(k_tap), stream));
}

void attention_forward(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *att,
                       int n_heads, int n_kv_heads, int head_dim, const int *d_pos, int max_seq, float scale,
                       cudaStream_t stream) {
    check("attention", q3_attention_forward(P(out), P(q), P(key_cache), P(value_cache), att, n_heads,
                                            n_kv_heads, head_dim, d_pos, max_seq, scale, stream));
}

void argmax_forward(int *out, const bf16 *x, int n, cudaStream_t stream) {
    check("argmax", q3_argmax_forward(out, P(x), n, stream));
}

void sample_forward(int *out, const bf16 *x, int n, float inv_temp, float u, cudaStream_t stream) {
    check("sample", q3_sample_forward(out, P(x), n, inv_temp, u, stream));
}
