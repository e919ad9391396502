// TEST INFRASTRUCTURE ONLY: extern "C" entry points over the reference's own kernel launchers.
//
// oracle/Makefile compiles this file together with the reference's src/kernels.cu (read in
// place from the mounted reference tree, never copied) into oracle/_ref/libqwen3_ref.so for
// sm_100a. The GPU parity tests load that library through ctypes and use the reference
// kernels as the exact oracle for the sm_100a kernels of llm-inference_b200. Nothing in the
// product links it.
//
// Each wrapper forwards to the launcher of the same name declared in src/kernels.cuh:7-26
// and returns the CUDA error of the launch (the reference launchers exit() on bad shapes).
#include "kernels.cuh"

extern "C" {

int ref_embedding_forward(bf16 *out, const bf16 *table, const int *d_token, int hidden,
                          void *stream) {
    embedding_forward(out, table, d_token, hidden, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_rmsnorm_forward(bf16 *out, const bf16 *in, const bf16 *weight, int rows, int dim,
                        float eps, void *stream) {
    rmsnorm_forward(out, in, weight, rows, dim, eps, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_gemv_forward(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, void *stream) {
    gemv_forward(out, w, x, rows, cols, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_gemv_residual_forward(bf16 *x, const bf16 *w, const bf16 *in, int rows, int cols,
                              bf16 *tap, void *stream) {
    gemv_residual_forward(x, w, in, rows, cols, tap, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_qkv_forward(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv,
                    const bf16 *x, int q_rows, int kv_rows, int cols, void *stream) {
    qkv_forward(q, k, v, wq, wk, wv, x, q_rows, kv_rows, cols, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_gate_up_forward(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x,
                        int rows, int cols, bf16 *gate_tap, bf16 *up_tap, void *stream) {
    gate_up_forward(act, w_gate, w_up, x, rows, cols, gate_tap, up_tap, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_qk_norm_rope_forward(bf16 *q, bf16 *k, const bf16 *v, const bf16 *q_norm_w,
                             const bf16 *k_norm_w, bf16 *key_cache, bf16 *value_cache,
                             const int *d_pos, int n_heads, int n_kv_heads, int head_dim,
                             float eps, float theta, bf16 *q_tap, bf16 *k_tap, void *stream) {
    qk_norm_rope_forward(q, k, v, q_norm_w, k_norm_w, key_cache, value_cache, d_pos, n_heads,
                         n_kv_heads, head_dim, eps, theta, q_tap, k_tap, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_attention_forward(bf16 *out, const bf16 *q, const bf16 *key_cache,
                          const bf16 *value_cache, float *att, int n_heads, int n_kv_heads,
                          int head_dim, const int *d_pos, int max_seq, float scale,
                          void *stream) {
    attention_forward(out, q, key_cache, value_cache, att, n_heads, n_kv_heads, head_dim, d_pos,
                      max_seq, scale, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_argmax_forward(int *out, const bf16 *x, int n, void *stream) {
    argmax_forward(out, x, n, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

int ref_sample_forward(int *out, const bf16 *x, int n, float inv_temp, float u, void *stream) {
    sample_forward(out, x, n, inv_temp, u, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

}  // extern "C"
