// Batched C entry points: the reference launchers with a batch of independent decode sequences.
// Activations are [batch, dim] row-major; each sequence has its own token id, position and KV
// cache (sequence b's cache rows start at cache + b * cache_seq_stride). The reference has no
// batch dimension, so these have no counterpart there; per sequence they compute what the
// reference kernel computes for that sequence.
//
// Projections: batch 1 runs the bit-exact batch-1 kernels (gemv.cu); batch >= 2 runs the
// tcgen05 tensor-core GEMM (gemm_tc.cu), whose fp32 sums follow the tensor core's order.
#include "common.cuh"

namespace q3 {

int check_device();
int gemv_plain(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t s);
int gemv_residual(bf16 *x, const bf16 *w, const bf16 *in, int rows, int cols, bf16 *tap, cudaStream_t s);
int gemv_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x,
             int q_rows, int kv_rows, int cols, cudaStream_t s);
int gemv_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                 bf16 *gate_tap, bf16 *up_tap, cudaStream_t s);
int tc_gemv(bf16 *out, const bf16 *w, const bf16 *x, int batch, int rows, int cols, cudaStream_t s);
int tc_gemv_residual(bf16 *x, const bf16 *w, const bf16 *in, int batch, int rows, int cols, bf16 *tap,
                     cudaStream_t s);
int tc_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x, int batch,
           int q_rows, int kv_rows, int cols, cudaStream_t s);
int tc_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int batch, int rows, int cols,
               bf16 *gate_tap, bf16 *up_tap, cudaStream_t s);
int embedding(bf16 *out, const bf16 *table, const int *tokens, int n_rows, int hidden, int vocab,
              cudaStream_t s);
int qk_norm_rope(bf16 *q, bf16 *k, const bf16 *v, const bf16 *q_norm_w, const bf16 *k_norm_w,
                 bf16 *key_cache, bf16 *value_cache, const int *pos, int n_rows, long long q_stride,
                 long long kv_stride, KvLayout kv, int n_heads, int n_kv_heads, int head_dim,
                 int max_seq, float eps, float theta, bf16 *q_tap, bf16 *k_tap, cudaStream_t s);
int argmax_rows(const bf16 *x, int n, int n_rows, long long row_stride, int *out, int *next_token,
                int *pos, int *history, int *step, int history_cap, cudaStream_t s);
int attention(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *scores, int ld,
              const int *pos, int n_rows, long long q_stride, KvLayout kv, int n_heads, int n_kv_heads,
              int head_dim, int max_seq, float scale, const AttnSplit *split, cudaStream_t s);
int attention_check(int n_heads, int n_kv_heads, int head_dim, int max_seq, int n_rows);
int fused_chunks(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq);
int attention_fused(bf16 *out, const bf16 *q, const bf16 *k, const bf16 *v, const bf16 *q_norm_w,
                    const bf16 *k_norm_w, bf16 *key_cache, bf16 *value_cache, KvLayout kv, const int *pos, int batch,
                    long long q_stride, long long kv_stride, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                    float eps, float theta, float scale, int chunks, cudaStream_t s);

// ---------------------------------------------------------------- batched projections

int proj(bf16 *out, const bf16 *w, const bf16 *x, int batch, int rows, int cols, cudaStream_t s) {
    if (batch < 0) return Q3_ERR_SHAPE;
    if (batch == 0) return Q3_OK;
    if (batch == 1) return gemv_plain(out, w, x, rows, cols, s);
    for (int b0 = 0; b0 < batch; b0 += 256) {  // the MMA's N is at most 256
        const int nb = batch - b0 < 256 ? batch - b0 : 256;
        int st = tc_gemv(out + (size_t)b0 * rows, w, x + (size_t)b0 * cols, nb, rows, cols, s);
        if (st != Q3_OK) return st;
    }
    return Q3_OK;
}

int proj_residual(bf16 *x, const bf16 *w, const bf16 *in, int batch, int rows, int cols, bf16 *tap,
                  cudaStream_t s) {
    if (batch < 0) return Q3_ERR_SHAPE;
    if (batch == 0) return Q3_OK;
    if (batch == 1) return gemv_residual(x, w, in, rows, cols, tap, s);
    for (int b0 = 0; b0 < batch; b0 += 256) {
        const int nb = batch - b0 < 256 ? batch - b0 : 256;
        int st = tc_gemv_residual(x + (size_t)b0 * rows, w, in + (size_t)b0 * cols, nb, rows, cols,
                                  tap ? tap + (size_t)b0 * rows : nullptr, s);
        if (st != Q3_OK) return st;
    }
    return Q3_OK;
}

int proj_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x,
             int batch, int q_rows, int kv_rows, int cols, cudaStream_t s) {
    if (batch < 0) return Q3_ERR_SHAPE;
    if (batch == 0) return Q3_OK;
    if (batch == 1) return gemv_qkv(q, k, v, wq, wk, wv, x, q_rows, kv_rows, cols, s);
    for (int b0 = 0; b0 < batch; b0 += 256) {
        const int nb = batch - b0 < 256 ? batch - b0 : 256;
        int st = tc_qkv(q + (size_t)b0 * q_rows, k + (size_t)b0 * kv_rows, v + (size_t)b0 * kv_rows, wq, wk, wv,
                        x + (size_t)b0 * cols, nb, q_rows, kv_rows, cols, s);
        if (st != Q3_OK) return st;
    }
    return Q3_OK;
}

int proj_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int batch, int rows, int cols,
                 bf16 *gate_tap, bf16 *up_tap, cudaStream_t s) {
    if (batch < 0) return Q3_ERR_SHAPE;
    if (batch == 0) return Q3_OK;
    if (batch == 1) return gemv_gate_up(act, w_gate, w_up, x, rows, cols, gate_tap, up_tap, s);
    for (int b0 = 0; b0 < batch; b0 += 256) {
        const int nb = batch - b0 < 256 ? batch - b0 : 256;
        const size_t o = (size_t)b0 * rows;
        int st = tc_gate_up(act + o, w_gate, w_up, x + (size_t)b0 * cols, nb, rows, cols,
                            gate_tap ? gate_tap + o : nullptr, up_tap ? up_tap + o : nullptr, s);
        if (st != Q3_OK) return st;
    }
    return Q3_OK;
}

// ---------------------------------------------------------------- attention scratch

// Split-mode scratch layout: scores [B][H][ld] f32 (ld = max_seq rounded up to 4, so score rows
// stay 16-byte aligned) | stats [B][H][2] f32 | partial [B][H][max_chunks][hd] f32.
constexpr int ATTN_CHUNK = 512;

int score_ld(int max_seq) { return (max_seq + 3) / 4 * 4; }

size_t attention_scratch_layout(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq, AttnSplit *sp,
                                float **scores, void *base) {
    const int max_chunks = (max_seq + ATTN_CHUNK - 1) / ATTN_CHUNK;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += (bytes + 255) / 256 * 256;
        return o;
    };
    const size_t o_scores = take((size_t)batch * n_heads * score_ld(max_seq) * 4);
    const size_t o_stats = take((size_t)batch * n_heads * 2 * 4);
    const size_t o_part = take((size_t)batch * n_heads * max_chunks * head_dim * 4);
    if (base && sp && scores) {
        char *p = static_cast<char *>(base);
        *scores = reinterpret_cast<float *>(p + o_scores);
        sp->stats = reinterpret_cast<float *>(p + o_stats);
        sp->partial = reinterpret_cast<float *>(p + o_part);
        sp->count_a = nullptr;
        sp->count_b = nullptr;
        sp->chunk_b = ATTN_CHUNK;
        sp->max_chunks = max_chunks;
    }
    return off;
}

}  // namespace q3

using namespace q3;
#define B(p) reinterpret_cast<bf16 *>(p)
#define CB(p) reinterpret_cast<const bf16 *>(p)
#define S(p) reinterpret_cast<cudaStream_t>(p)
#define DEVICE_OR_RETURN()             \
    do {                               \
        int st_ = check_device();      \
        if (st_ != Q3_OK) return st_;  \
    } while (0)

extern "C" {

int q3_embedding_batched(q3_bf16 *out, const q3_bf16 *table, const int *d_tokens, int batch, int hidden,
                         int vocab, void *stream) {
    DEVICE_OR_RETURN();
    if (vocab <= 0) return Q3_ERR_SHAPE;
    return embedding(B(out), CB(table), d_tokens, batch, hidden, vocab, S(stream));
}

int q3_gemv_batched(q3_bf16 *out, const q3_bf16 *w, const q3_bf16 *x, int batch, int rows, int cols,
                    void *stream) {
    DEVICE_OR_RETURN();
    return proj(B(out), CB(w), CB(x), batch, rows, cols, S(stream));
}

int q3_gemv_residual_batched(q3_bf16 *x, const q3_bf16 *w, const q3_bf16 *in, int batch, int rows, int cols,
                             q3_bf16 *tap, void *stream) {
    DEVICE_OR_RETURN();
    return proj_residual(B(x), CB(w), CB(in), batch, rows, cols, B(tap), S(stream));
}

int q3_qkv_batched(q3_bf16 *q, q3_bf16 *k, q3_bf16 *v, const q3_bf16 *wq, const q3_bf16 *wk, const q3_bf16 *wv,
                   const q3_bf16 *x, int batch, int q_rows, int kv_rows, int cols, void *stream) {
    DEVICE_OR_RETURN();
    return proj_qkv(B(q), B(k), B(v), CB(wq), CB(wk), CB(wv), CB(x), batch, q_rows, kv_rows, cols, S(stream));
}

int q3_gate_up_batched(q3_bf16 *act, const q3_bf16 *w_gate, const q3_bf16 *w_up, const q3_bf16 *x, int batch,
                       int rows, int cols, q3_bf16 *gate_tap, q3_bf16 *up_tap, void *stream) {
    DEVICE_OR_RETURN();
    return proj_gate_up(B(act), CB(w_gate), CB(w_up), CB(x), batch, rows, cols, B(gate_tap), B(up_tap),
                        S(stream));
}

int q3_qk_norm_rope_batched(q3_bf16 *q, q3_bf16 *k, const q3_bf16 *v, const q3_bf16 *q_norm_w,
                            const q3_bf16 *k_norm_w, q3_bf16 *key_cache, q3_bf16 *value_cache,
                            long long cache_seq_stride, long long cache_pos_stride, long long cache_head_stride,
                            const int *d_pos, int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                            float eps, float theta, q3_bf16 *q_tap, q3_bf16 *k_tap, void *stream) {
    DEVICE_OR_RETURN();
    if (max_seq <= 0 || cache_pos_stride <= 0) return Q3_ERR_SHAPE;
    const KvLayout kv = {cache_seq_stride, cache_pos_stride, cache_head_stride};
    return qk_norm_rope(B(q), B(k), CB(v), CB(q_norm_w), CB(k_norm_w), B(key_cache), B(value_cache), d_pos, batch,
                        (long long)n_heads * head_dim, (long long)n_kv_heads * head_dim, kv, n_heads, n_kv_heads,
                        head_dim, max_seq, eps, theta, B(q_tap), B(k_tap), S(stream));
}

size_t q3_attention_scratch_bytes(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq) {
    if (attention_check(n_heads, n_kv_heads, head_dim, max_seq, batch) != Q3_OK) return 0;
    return attention_scratch_layout(batch, n_heads, n_kv_heads, head_dim, max_seq, nullptr, nullptr, nullptr);
}

int q3_attention_batched(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *key_cache, const q3_bf16 *value_cache,
                         long long cache_seq_stride, long long cache_pos_stride, long long cache_head_stride,
                         void *scratch, const int *d_pos, int batch, int n_heads, int n_kv_heads, int head_dim,
                         int max_seq, float scale, void *stream) {
    DEVICE_OR_RETURN();
    if (!scratch) return Q3_ERR_ARG;
    int st = attention_check(n_heads, n_kv_heads, head_dim, max_seq, batch);
    if (st != Q3_OK) return st;
    AttnSplit sp;
    float *scores = nullptr;
    attention_scratch_layout(batch, n_heads, n_kv_heads, head_dim, max_seq, &sp, &scores, scratch);
    const KvLayout kv = {cache_seq_stride, cache_pos_stride, cache_head_stride};
    return attention(B(out), CB(q), CB(key_cache), CB(value_cache), scores, score_ld(max_seq), d_pos, batch,
                     (long long)n_heads * head_dim, kv, n_heads, n_kv_heads, head_dim, max_seq, scale, &sp,
                     S(stream));
}

int q3_rope_attention_chunks(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq) {
    if (check_device() != Q3_OK) return 0;
    return fused_chunks(batch, n_heads, n_kv_heads, head_dim, max_seq);
}

int q3_rope_attention_batched(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *k, const q3_bf16 *v,
                              const q3_bf16 *q_norm_w, const q3_bf16 *k_norm_w, q3_bf16 *key_cache,
                              q3_bf16 *value_cache, long long cache_seq_stride, long long cache_pos_stride,
                              long long cache_head_stride, const int *d_pos, int batch, int n_heads, int n_kv_heads,
                              int head_dim, int max_seq, float eps, float theta, float scale, int chunks,
                              void *stream) {
    DEVICE_OR_RETURN();
    const KvLayout kv = {cache_seq_stride, cache_pos_stride, cache_head_stride};
    return attention_fused(B(out), CB(q), CB(k), CB(v), CB(q_norm_w), CB(k_norm_w), B(key_cache), B(value_cache), kv,
                           d_pos, batch, (long long)n_heads * head_dim, (long long)n_kv_heads * head_dim, n_heads,
                           n_kv_heads, head_dim, max_seq, eps, theta, scale, chunks, S(stream));
}

int q3_argmax_batched(int *out, const q3_bf16 *x, int batch, int n, void *stream) {
    DEVICE_OR_RETURN();
    return argmax_rows(CB(x), n, batch, n, out, nullptr, nullptr, nullptr, nullptr, 0, S(stream));
}

}  // extern "C"
