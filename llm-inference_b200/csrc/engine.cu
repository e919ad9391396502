// Batched greedy decode engine: the reference's forward pass (src/forward.cu) for B independent
// sequences on one GPU, with every buffer on the device and one CUDA graph per decode step.
//
// RunState (src/forward.cuh:6-25) becomes batched: activations [B, dim], one KV cache per layer
// and sequence, stored head-major -- [n_layers][B][n_kv_heads][max_seq][head_dim] -- so that the
// positions of one (sequence, kv head) are contiguous and attention streams them in long runs
// (the reference keeps one layer's heads interleaved per position, [max_seq][n_kv*head_dim]);
// per-sequence token ids and positions live in device memory.
// The launch order of one step is forward_kernels (src/forward.cu:118-193) followed by the
// greedy argmax (:229-236), which here also feeds the next step on the device: it writes
// next_token[b], advances pos[b] and appends the token to a history buffer, so a captured step
// replays back to back with no host round trip. The reference protocol -- host token and
// position in, one step, host token out -- is q3_engine_forward + q3_engine_sample_argmax.
//
// Projections: batch 1 uses the bit-exact batch-1 kernels, batch >= 2 the tcgen05 GEMM.
// Attention: split-KV by default; Q3_ENGINE_EXACT_ATTENTION selects the bit-exact single-chunk
// kernels (slower at long context).
#include <stdlib.h>
#include <string.h>

#include <vector>

#include <algorithm>
#include <climits>

#include "common.cuh"

namespace q3 {
int check_device();
int proj(bf16 *out, const bf16 *w, const bf16 *x, int batch, int rows, int cols, cudaStream_t s);
int proj_residual(bf16 *x, const bf16 *w, const bf16 *in, int batch, int rows, int cols, bf16 *tap,
                  cudaStream_t s);
int proj_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x,
             int batch, int q_rows, int kv_rows, int cols, cudaStream_t s);
int proj_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int batch, int rows, int cols,
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
int attention(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *scores, int ld,
              const int *pos, int n_rows, long long q_stride, KvLayout kv, int n_heads, int n_kv_heads,
              int head_dim, int max_seq, float scale, const AttnSplit *split, cudaStream_t s);
int attention_check(int n_heads, int n_kv_heads, int head_dim, int max_seq, int n_rows);
int score_ld(int max_seq);
size_t attention_scratch_layout(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq, AttnSplit *sp,
                                float **scores, void *base);
int gemv_plain_n(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t s, const bf16 *norm_w,
                 float eps);
int gemv_qkv_n(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x, int q_rows,
               int kv_rows, int cols, cudaStream_t s, const bf16 *norm_w, float eps);
int gemv_gate_up_n(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                   bf16 *gate_tap, bf16 *up_tap, cudaStream_t s, const bf16 *norm_w, float eps);
int fused_chunks(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq);
int attention_fused(bf16 *out, const bf16 *q, const bf16 *k, const bf16 *v, const bf16 *q_norm_w,
                    const bf16 *k_norm_w, bf16 *key_cache, bf16 *value_cache, KvLayout kv, const int *pos, int batch,
                    long long q_stride, long long kv_stride, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                    float eps, float theta, float scale, int chunks, cudaStream_t s);
int fill_normal(bf16 *dst, long long n, unsigned long long seed, float mean, float std, cudaStream_t s);
int fill_normal_blocks(bf16 *dst, long long n_blocks, long long block_len, long long block_stride,
                       unsigned long long seed, float mean, float std, cudaStream_t s);
}  // namespace q3

using namespace q3;

struct q3_engine {
    q3_config cfg;
    std::vector<q3_layer_weights> layers;
    const bf16 *embed, *final_norm, *lm_head;
    int B, max_seq, history_cap, flags;
    cudaStream_t stream;
    // activations
    bf16 *x, *xb, *q, *k, *v, *attn_out, *hb, *logits;
    bf16 *key_cache, *value_cache;
    void *attn_scratch;
    float *scores;
    AttnSplit split;
    // small batches: RoPE and attention in one launch (attn_fused.cu), this many chunks per head
    int fused_chunks = 0;
    // ... up to this position of the longest sequence; from it on a step runs the split-KV
    // kernels, captured as a second graph (INT_MAX: the fused launch throughout)
    int split_from = INT_MAX;
    long long pos_hint = 0;   // the largest position the next step attends up to (host's count)
    bool split_now = false;   // enqueue the split-KV kernels even where the fused launch applies
    // decode-loop state
    int *next_token, *pos, *out_token, *history, *step;
    int *pf_token, *pf_pos;  // prefill: one chunk's token ids and positions
    // Q3_ENGINE_MEGAKERNEL: the whole step as one persistent kernel with a streamed weight ring
    // (decode_stream.cu, batch 1)
    bool mk = false;
    DsParams mkp = {};
    int mk_grid = 0;
    int *host_io;  // pinned: [2B] for token/position uploads, [B] for downloads
    cudaGraphExec_t graph = nullptr;
    int graph_kernels = 0;  // kernel nodes of the captured step
    cudaGraphExec_t graph_split = nullptr;  // the step with split-KV attention, when split_from < max_seq
    int graph_split_kernels = 0;
    cudaStream_t own_stream;  // created when the caller passes the legacy default stream
    std::vector<void *> allocations;
};

namespace {

int alloc(q3_engine *e, void **p, size_t bytes) {
    cudaError_t err = cudaMalloc(p, bytes);
    if (err != cudaSuccess) return record_cuda_error(err);
    e->allocations.push_back(*p);
    return Q3_OK;
}

// positions per fused-attention CTA from which a step runs the split-KV kernels instead
constexpr int FUSED_SPLIT_PER_CTA = 600;

#define TRY(expr)                     \
    do {                              \
        int st_ = (expr);             \
        if (st_ != Q3_OK) return st_; \
    } while (0)

// The decoder layers for `rows` rows of activations. Row b reads its token id and position from
// tok[b] / pos[b]; its KV rows go to the cache of sequence (cache_seq + b), or, when
// shared_cache, every row's to the cache of sequence cache_seq (one prompt's chunk at
// consecutive positions: row b attends positions 0..pos[b] of that cache, so the chunk is causal).
int enqueue_layers(q3_engine *e, int rows, const int *tok, const int *pos, int cache_seq, bool shared_cache) {
    const q3_config &c = e->cfg;
    const int B = e->B, H = c.hidden_size, I = c.intermediate_size;
    const int qd = c.n_heads * c.head_dim, kvd = c.n_kv_heads * c.head_dim;
    const long long seq_stride = (long long)e->max_seq * kvd;  // one (layer, sequence): n_kv heads x max_seq rows
    const KvLayout kv = {shared_cache ? 0 : seq_stride, c.head_dim, (long long)e->max_seq * c.head_dim};
    const float scale = (float)(1.0 / sqrt((double)c.head_dim));
    cudaStream_t s = e->stream;
    const bool exact_attn = (e->flags & Q3_ENGINE_EXACT_ATTENTION) != 0;
    // rows of a prompt share one cache and read each other's new rows: not in one fused launch
    const bool fused = e->fused_chunks > 0 && !shared_cache && !e->split_now;
    // one row: the batch-1 projections that read a normed input normalize it themselves
    const bool norm_in_gemv = rows == 1 && H <= 8192;
    const float eps = c.rms_norm_eps;

    TRY(embedding(e->x, e->embed, tok, rows, H, c.vocab_size, s));
    for (int l = 0; l < c.n_layers; l++) {
        const q3_layer_weights &w = e->layers[l];
        bf16 *kc = e->key_cache + ((size_t)l * B + cache_seq) * seq_stride;
        bf16 *vc = e->value_cache + ((size_t)l * B + cache_seq) * seq_stride;
        if (norm_in_gemv) {
            TRY(gemv_qkv_n(e->q, e->k, e->v, (const bf16 *)w.wq, (const bf16 *)w.wk, (const bf16 *)w.wv, e->x, qd, kvd,
                           H, s, (const bf16 *)w.attn_norm, eps));
        } else {
            TRY(rmsnorm(e->xb, e->x, (const bf16 *)w.attn_norm, rows, H, eps, s));
            TRY(proj_qkv(e->q, e->k, e->v, (const bf16 *)w.wq, (const bf16 *)w.wk, (const bf16 *)w.wv, e->xb, rows,
                         qd, kvd, H, s));
        }
        if (fused) {
            TRY(attention_fused(e->attn_out, e->q, e->k, e->v, (const bf16 *)w.q_norm, (const bf16 *)w.k_norm, kc, vc,
                                kv, pos, rows, qd, kvd, c.n_heads, c.n_kv_heads, c.head_dim, e->max_seq, eps,
                                c.rope_theta, scale, e->fused_chunks, s));
        } else {
            TRY(qk_norm_rope(e->q, e->k, e->v, (const bf16 *)w.q_norm, (const bf16 *)w.k_norm, kc, vc, pos, rows,
                             qd, kvd, kv, c.n_heads, c.n_kv_heads, c.head_dim, e->max_seq, eps, c.rope_theta,
                             nullptr, nullptr, s));
            TRY(attention(e->attn_out, e->q, kc, vc, e->scores, score_ld(e->max_seq), pos, rows, qd, kv, c.n_heads,
                          c.n_kv_heads, c.head_dim, e->max_seq, scale, exact_attn ? nullptr : &e->split, s));
        }
        TRY(proj_residual(e->x, (const bf16 *)w.wo, e->attn_out, rows, H, qd, nullptr, s));
        if (norm_in_gemv) {
            TRY(gemv_gate_up_n(e->hb, (const bf16 *)w.w_gate, (const bf16 *)w.w_up, e->x, I, H, nullptr, nullptr, s,
                               (const bf16 *)w.mlp_norm, eps));
        } else {
            TRY(rmsnorm(e->xb, e->x, (const bf16 *)w.mlp_norm, rows, H, eps, s));
            TRY(proj_gate_up(e->hb, (const bf16 *)w.w_gate, (const bf16 *)w.w_up, e->xb, rows, I, H, nullptr, nullptr,
                             s));
        }
        TRY(proj_residual(e->x, (const bf16 *)w.w_down, e->hb, rows, H, I, nullptr, s));
    }
    if (norm_in_gemv) {
        TRY(gemv_plain_n(e->logits, e->lm_head, e->x, c.vocab_size, H, s, e->final_norm, eps));
    } else {
        TRY(rmsnorm(e->xb, e->x, e->final_norm, rows, H, eps, s));
        TRY(proj(e->logits, e->lm_head, e->xb, rows, c.vocab_size, H, s));
    }
    return Q3_OK;
}

int enqueue_step(q3_engine *e) {
    if (e->mk) return decode_stream_launch(e->mkp, e->mk_grid, e->stream);
    const q3_config &c = e->cfg;
    const int B = e->B;
    cudaStream_t s = e->stream;
    TRY(enqueue_layers(e, B, e->next_token, e->pos, 0, false));
    TRY(argmax_rows(e->logits, c.vocab_size, B, c.vocab_size, e->out_token, e->next_token, e->pos, e->history,
                    e->step, e->history_cap, s));
    return Q3_OK;
}

// Captures one decode step (split: the split-KV attention kernels throughout) into *out.
int capture_step(q3_engine *e, bool split, cudaGraphExec_t *out, int *kernels_out) {
    cudaGraph_t g;
    int r = record_cuda_error(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    if (r != Q3_OK) return r;
    e->split_now = split;
    const int st = enqueue_step(e);
    e->split_now = false;
    r = record_cuda_error(cudaStreamEndCapture(e->stream, &g));
    if (st != Q3_OK) {
        if (r == Q3_OK) cudaGraphDestroy(g);
        return st;
    }
    if (r != Q3_OK) return r;
    size_t n_nodes = 0;
    cudaGraphGetNodes(g, nullptr, &n_nodes);
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    int kernels = 0;
    if (n_nodes && cudaGraphGetNodes(g, nodes.data(), &n_nodes) == cudaSuccess)
        for (auto nd : nodes) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
        }
    *kernels_out = kernels;
    r = record_cuda_error(cudaGraphInstantiate(out, g, 0));
    cudaGraphDestroy(g);
    return r;
}

void release(q3_engine *e) {
    if (e->graph) cudaGraphExecDestroy(e->graph);
    if (e->graph_split) cudaGraphExecDestroy(e->graph_split);
    if (e->own_stream) cudaStreamDestroy(e->own_stream);
    for (void *p : e->allocations) cudaFree(p);
    if (e->host_io) cudaFreeHost(e->host_io);
    delete e;
}

}  // namespace

extern "C" {

size_t q3_weight_bytes_per_step(const q3_config *c) {
    if (!c) return 0;
    const size_t hidden = c->hidden_size, hd = c->head_dim, q = (size_t)c->n_heads * hd,
                 kv = (size_t)c->n_kv_heads * hd, inter = c->intermediate_size;
    size_t layer = hidden + q * hidden + 2 * kv * hidden + 2 * hd + hidden * q + hidden + 3 * inter * hidden;
    size_t elems = layer * c->n_layers + hidden + (size_t)c->vocab_size * hidden + hidden;
    return elems * 2;
}

size_t q3_kv_bytes_per_position(const q3_config *c) {
    if (!c) return 0;
    return 2 * (size_t)c->n_layers * c->n_kv_heads * c->head_dim * 2;
}

int q3_engine_create(const q3_config *cfg, const q3_weights *w, int batch, int max_seq, int history_cap, int flags,
                     void *stream, q3_engine **out) {
    if (!cfg || !w || !out || !w->layers || !w->embed || !w->final_norm || !w->lm_head) return Q3_ERR_ARG;
    *out = nullptr;
    int st = check_device();
    if (st != Q3_OK) return st;
    const q3_config &c = *cfg;
    if (batch <= 0 || max_seq <= 0 || history_cap < 0 || c.n_layers <= 0 || c.hidden_size <= 0 ||
        c.intermediate_size <= 0 || c.vocab_size <= 0 || c.hidden_size % 8 || c.intermediate_size % 8)
        return Q3_ERR_SHAPE;
    st = attention_check(c.n_heads, c.n_kv_heads, c.head_dim, max_seq, batch);
    if (st != Q3_OK) return st;
    const bool mk = (flags & Q3_ENGINE_MEGAKERNEL) != 0;
    if (mk && (batch != 1 || c.head_dim != 128)) return Q3_ERR_SHAPE;
    q3_engine *e = new q3_engine();
    e->cfg = c;
    e->layers.assign(w->layers, w->layers + c.n_layers);
    e->embed = (const bf16 *)w->embed;
    e->final_norm = (const bf16 *)w->final_norm;
    e->lm_head = (const bf16 *)w->lm_head;
    e->B = batch;
    e->max_seq = max_seq;
    e->history_cap = history_cap;
    e->flags = flags;
    e->stream = (cudaStream_t)stream;
    if (e->stream == nullptr) {  // stream capture is not possible on the legacy default stream
        cudaError_t err = cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking);
        if (err != cudaSuccess) {
            release(e);
            return record_cuda_error(err);
        }
        e->stream = e->own_stream;
    }
    const size_t B = batch, H = c.hidden_size, I = c.intermediate_size, qd = (size_t)c.n_heads * c.head_dim,
                 kvd = (size_t)c.n_kv_heads * c.head_dim;
    const size_t cache = (size_t)c.n_layers * B * max_seq * kvd * 2;
    int r = Q3_OK;
    auto A = [&](void **p, size_t bytes) {
        if (r == Q3_OK) r = alloc(e, p, bytes > 0 ? bytes : 16);
    };
    A((void **)&e->x, B * H * 2);
    A((void **)&e->xb, B * H * 2);
    A((void **)&e->q, B * qd * 2);
    A((void **)&e->k, B * kvd * 2);
    A((void **)&e->v, B * kvd * 2);
    A((void **)&e->attn_out, B * qd * 2);
    A((void **)&e->hb, B * I * 2);
    A((void **)&e->logits, B * (size_t)c.vocab_size * 2);
    A((void **)&e->key_cache, cache);
    A((void **)&e->value_cache, cache);
    const size_t scratch = attention_scratch_layout(batch, c.n_heads, c.n_kv_heads, c.head_dim, max_seq, nullptr,
                                                    nullptr, nullptr);
    A(&e->attn_scratch, scratch);
    A((void **)&e->next_token, B * 4);
    A((void **)&e->pos, B * 4);
    A((void **)&e->out_token, B * 4);
    A((void **)&e->history, (size_t)(history_cap > 0 ? history_cap : 1) * B * 4);
    A((void **)&e->step, 16);
    A((void **)&e->pf_token, B * 4);
    A((void **)&e->pf_pos, B * 4);
    if (!mk && !(flags & (Q3_ENGINE_EXACT_ATTENTION | Q3_ENGINE_SPLIT_ATTENTION)))
        e->fused_chunks = fused_chunks(batch, c.n_heads, c.n_kv_heads, c.head_dim, max_seq);
    // From about 600 positions per cluster CTA on, the split-KV kernels, which spread every row
    // over all SMs, are the faster path; below it the single fused launch is. Measured on B200,
    // tok/s fused against split: Qwen3-4B batch 1 (10-CTA clusters) at position 256 454 / 375,
    // 4096 364 / 344, 6144 336 / 335, 8192 306 / 328; Qwen3-1.7B at position 2048, 8 sequences
    // (2-CTA clusters, 1024 per CTA) 3544 / 3698, 4 sequences (4-CTA, 512 per CTA) 2088 / 2027.
    // Both steps are captured and q3_engine_step picks one by the host's count of positions.
    if (e->fused_chunks > 0) e->split_from = FUSED_SPLIT_PER_CTA * e->fused_chunks;
    if (mk) {
        e->mk = true;
        DsParams &p = e->mkp;
        p.n_layers = c.n_layers;
        p.H = c.hidden_size;
        p.I = c.intermediate_size;
        p.n_heads = c.n_heads;
        p.n_kv = c.n_kv_heads;
        p.vocab = c.vocab_size;
        e->mk_grid = decode_stream_plan(p);
        if (e->mk_grid <= 0 && r == Q3_OK) r = Q3_ERR_SHAPE;
        const size_t nrep = (size_t)c.n_heads / c.n_kv_heads, groups = (size_t)c.n_kv_heads * std::max(p.chunks, 1);
        A((void **)&p.cmax, groups * nrep * 4);
        A((void **)&p.csum, (size_t)c.n_kv_heads * nrep * 128 * 4);
        A((void **)&p.partial, groups * nrep * 128 * 4);
        A((void **)&p.amax_val, (size_t)std::max(e->mk_grid, 1) * 4);
        A((void **)&p.amax_idx, (size_t)std::max(e->mk_grid, 1) * 4);
        A((void **)&p.sync, (size_t)decode_stream_sync_words(c.n_kv_heads) * 4);
        A((void **)&p.layers, (size_t)c.n_layers * sizeof(MkLayer));
    }
    if (r == Q3_OK) r = record_cuda_error(cudaMallocHost((void **)&e->host_io, 3 * B * sizeof(int)));
    if (r != Q3_OK) {
        release(e);
        return r;
    }
    attention_scratch_layout(batch, c.n_heads, c.n_kv_heads, c.head_dim, max_seq, &e->split, &e->scores,
                             e->attn_scratch);
    cudaStream_t s = e->stream;
    r = record_cuda_error(cudaMemsetAsync(e->attn_scratch, 0, scratch, s));
    if (r == Q3_OK) r = record_cuda_error(cudaMemsetAsync(e->key_cache, 0, cache, s));
    if (r == Q3_OK) r = record_cuda_error(cudaMemsetAsync(e->value_cache, 0, cache, s));
    if (r == Q3_OK) r = record_cuda_error(cudaMemsetAsync(e->next_token, 0, B * 4, s));
    if (r == Q3_OK) r = record_cuda_error(cudaMemsetAsync(e->pos, 0, B * 4, s));
    if (r == Q3_OK) r = record_cuda_error(cudaMemsetAsync(e->step, 0, 16, s));
    if (mk && r == Q3_OK) {
        std::vector<MkLayer> lw(c.n_layers);
        for (int l = 0; l < c.n_layers; l++) {
            const q3_layer_weights &w_ = e->layers[l];
            lw[l] = {(const bf16 *)w_.attn_norm, (const bf16 *)w_.wq, (const bf16 *)w_.wk, (const bf16 *)w_.wv,
                     (const bf16 *)w_.q_norm, (const bf16 *)w_.k_norm, (const bf16 *)w_.wo, (const bf16 *)w_.mlp_norm,
                     (const bf16 *)w_.w_gate, (const bf16 *)w_.w_up, (const bf16 *)w_.w_down};
        }
        r = record_cuda_error(cudaMemcpyAsync((void *)e->mkp.layers, lw.data(), lw.size() * sizeof(MkLayer),
                                              cudaMemcpyHostToDevice, s));
        if (r == Q3_OK)
            r = record_cuda_error(
                cudaMemsetAsync(e->mkp.sync, 0, (size_t)decode_stream_sync_words(c.n_kv_heads) * 4, s));
        if (r == Q3_OK) r = record_cuda_error(cudaStreamSynchronize(s));  // `lw` leaves scope
        DsParams &p = e->mkp;
        p.embed = e->embed;
        p.final_norm = e->final_norm;
        p.lm_head = e->lm_head;
        p.eps = c.rms_norm_eps;
        p.theta = c.rope_theta;
        p.scale = (float)(1.0 / sqrt((double)c.head_dim));
        p.x = e->x;
        p.q = e->q;
        p.k = e->k;
        p.v = e->v;
        p.attn_out = e->attn_out;
        p.act = e->hb;
        p.logits = e->logits;
        p.key_cache = e->key_cache;
        p.value_cache = e->value_cache;
        p.layer_stride = (long long)max_seq * kvd;
        p.max_seq = max_seq;
        p.scores = e->scores;
        p.ld = score_ld(max_seq);
        p.next_token = e->next_token;
        p.pos = e->pos;
        p.out_token = e->out_token;
        p.history = history_cap > 0 ? e->history : nullptr;
        p.step = e->step;
        p.history_cap = history_cap;
    }
    if (r == Q3_OK) r = record_cuda_error(cudaStreamSynchronize(s));
    if (r != Q3_OK) {
        release(e);
        return r;
    }
    *out = e;
    return Q3_OK;
}

int q3_engine_destroy(q3_engine *e) {
    if (!e) return Q3_ERR_ARG;
    cudaStreamSynchronize(e->stream);
    release(e);
    return Q3_OK;
}

int q3_engine_capture(q3_engine *e) {
    if (!e) return Q3_ERR_ARG;
    if (e->mk) {  // a step is already one launch
        e->graph_kernels = 1;
        return Q3_OK;
    }
    for (cudaGraphExec_t *g : {&e->graph, &e->graph_split})
        if (*g) {
            cudaGraphExecDestroy(*g);
            *g = nullptr;
        }
    TRY(capture_step(e, false, &e->graph, &e->graph_kernels));
    if (e->split_from < e->max_seq) TRY(capture_step(e, true, &e->graph_split, &e->graph_split_kernels));
    return Q3_OK;
}

int q3_engine_step(q3_engine *e, int n_steps) {
    if (!e || n_steps < 0) return Q3_ERR_ARG;
    for (int i = 0; i < n_steps; i++) {
        const bool split = e->pos_hint >= e->split_from;
        cudaGraphExec_t g = split && e->graph_split ? e->graph_split : e->graph;
        if (g) {
            int r = record_cuda_error(cudaGraphLaunch(g, e->stream));
            if (r != Q3_OK) return r;
        } else {
            e->split_now = split;
            const int r = enqueue_step(e);
            e->split_now = false;
            if (r != Q3_OK) return r;
        }
        e->pos_hint++;  // every row's position advances by one (argmax_rows)
    }
    return Q3_OK;
}

int q3_engine_set_state(q3_engine *e, const int *tokens, const int *positions) {
    if (!e || !tokens || !positions) return Q3_ERR_ARG;
    for (int b = 0; b < e->B; b++) {
        if (tokens[b] < 0 || tokens[b] >= e->cfg.vocab_size || positions[b] < 0 || positions[b] >= e->max_seq)
            return Q3_ERR_SHAPE;
    }
    int *io = e->host_io;
    int r = record_cuda_error(cudaStreamSynchronize(e->stream));  // the pinned staging buffer is reused
    if (r != Q3_OK) return r;
    memcpy(io, tokens, e->B * sizeof(int));
    memcpy(io + e->B, positions, e->B * sizeof(int));
    e->pos_hint = *std::max_element(positions, positions + e->B);
    r = record_cuda_error(cudaMemcpyAsync(e->next_token, io, e->B * sizeof(int), cudaMemcpyHostToDevice, e->stream));
    if (r == Q3_OK)
        r = record_cuda_error(cudaMemcpyAsync(e->pos, io + e->B, e->B * sizeof(int), cudaMemcpyHostToDevice, e->stream));
    return r;
}

int q3_engine_forward(q3_engine *e, const int *tokens, const int *positions) {
    int r = q3_engine_set_state(e, tokens, positions);
    return r == Q3_OK ? q3_engine_step(e, 1) : r;
}

int q3_engine_prefill(q3_engine *e, int seq, const int *tokens, int n_tokens, int start_pos) {
    if (!e || !tokens) return Q3_ERR_ARG;
    if (seq < 0 || seq >= e->B || n_tokens <= 0 || start_pos < 0 || (long long)start_pos + n_tokens > e->max_seq)
        return Q3_ERR_SHAPE;
    for (int i = 0; i < n_tokens; i++)
        if (tokens[i] < 0 || tokens[i] >= e->cfg.vocab_size) return Q3_ERR_SHAPE;
    const int V = e->cfg.vocab_size;
    int *io = e->host_io;
    int rows = 0;
    for (int c0 = 0; c0 < n_tokens; c0 += e->B) {
        rows = std::min(e->B, n_tokens - c0);
        int r = record_cuda_error(cudaStreamSynchronize(e->stream));  // the pinned staging buffer is reused
        if (r != Q3_OK) return r;
        for (int i = 0; i < rows; i++) {
            io[i] = tokens[c0 + i];
            io[e->B + i] = start_pos + c0 + i;
        }
        r = record_cuda_error(cudaMemcpyAsync(e->pf_token, io, rows * sizeof(int), cudaMemcpyHostToDevice, e->stream));
        if (r == Q3_OK)
            r = record_cuda_error(cudaMemcpyAsync(e->pf_pos, io + e->B, rows * sizeof(int), cudaMemcpyHostToDevice,
                                                  e->stream));
        if (r != Q3_OK) return r;
        TRY(enqueue_layers(e, rows, e->pf_token, e->pf_pos, seq, true));
    }
    // the prompt's last token: its logits give the sequence's next token; its position follows
    TRY(argmax_rows(e->logits + (size_t)(rows - 1) * V, V, 1, V, e->out_token + seq, e->next_token + seq, nullptr,
                    nullptr, nullptr, 0, e->stream));
    int r = record_cuda_error(cudaStreamSynchronize(e->stream));
    if (r != Q3_OK) return r;
    io[2 * e->B] = start_pos + n_tokens;
    e->pos_hint = std::max(e->pos_hint, (long long)start_pos + n_tokens);
    r = record_cuda_error(cudaMemcpyAsync(e->pos + seq, io + 2 * e->B, sizeof(int), cudaMemcpyHostToDevice, e->stream));
    if (r == Q3_OK) r = record_cuda_error(cudaStreamSynchronize(e->stream));
    return r;
}

int q3_engine_sample_argmax(q3_engine *e, int *tokens_out) {
    if (!e || !tokens_out) return Q3_ERR_ARG;
    int *io = e->host_io + 2 * e->B;
    int r = record_cuda_error(cudaMemcpyAsync(io, e->out_token, e->B * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    if (r == Q3_OK) r = record_cuda_error(cudaStreamSynchronize(e->stream));
    if (r == Q3_OK) memcpy(tokens_out, io, e->B * sizeof(int));
    return r;
}

int q3_engine_fill_kv_normal(q3_engine *e, int n_positions, unsigned long long seed) {
    if (!e || n_positions < 0 || n_positions > e->max_seq) return Q3_ERR_ARG;
    const q3_config &c = e->cfg;
    // One block per (layer, sequence, kv head): its first n_positions rows of the head-major cache.
    const long long n_blocks = (long long)c.n_layers * e->B * c.n_kv_heads;
    const long long head_rows = (long long)e->max_seq * c.head_dim;
    const long long n = (long long)n_positions * c.head_dim;
    const unsigned long long sk = seed * 1000003ull;
    TRY(fill_normal_blocks(e->key_cache, n_blocks, n, head_rows, sk, 0.0f, 1.0f, e->stream));
    TRY(fill_normal_blocks(e->value_cache, n_blocks, n, head_rows, sk + (unsigned long long)n_blocks, 0.0f, 1.0f,
                           e->stream));
    return Q3_OK;
}

int q3_engine_info(const q3_engine *e, q3_engine_buffers *out) {
    if (!e || !out) return Q3_ERR_ARG;
    out->x = (q3_bf16 *)e->x;
    out->logits = (q3_bf16 *)e->logits;
    out->key_cache = (q3_bf16 *)e->key_cache;
    out->value_cache = (q3_bf16 *)e->value_cache;
    out->next_token = e->next_token;
    out->pos = e->pos;
    out->out_token = e->out_token;
    out->history = e->history;
    out->step = e->step;
    out->batch = e->B;
    out->max_seq = e->max_seq;
    out->history_cap = e->history_cap;
    const bool split = e->pos_hint >= e->split_from && e->graph_split;
    out->launches_per_step = split ? e->graph_split_kernels : e->graph_kernels;
    out->split_from = e->split_from < e->max_seq ? e->split_from : -1;
    return Q3_OK;
}

int q3_fill_normal_bf16(q3_bf16 *dst, long long n, unsigned long long seed, float mean, float std, void *stream) {
    int st = check_device();
    if (st != Q3_OK) return st;
    return fill_normal((bf16 *)dst, n, seed, mean, std, (cudaStream_t)stream);
}

}  // extern "C"
