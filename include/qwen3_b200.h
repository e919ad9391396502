/*
 * qwen3_b200.h -- C ABI of libqwen3_b200.so, the sm_100a (B200) decode kernels for Qwen3.
 *
 * The library is a drop-in for the kernels of William-Lamer/llm-inference. Its first ten
 * entry points take exactly the parameters of the reference launchers in src/kernels.cuh:7-26
 * (same order, same meaning, same units); each one's comment names the launcher it replaces.
 * The differences are only those a C ABI needs:
 *
 *   - extern "C" linkage and an int status instead of void (Q3_OK = 0). Where the reference
 *     prints a message and calls exit() (bad shapes, src/kernels.cu:147-152, :392-396; launch
 *     errors, src/common.cuh:11-22) these return Q3_ERR_SHAPE or Q3_ERR_CUDA and change nothing.
 *     csrc/dropin_shim.cu turns the codes back into the reference's print-and-exit behaviour
 *     under the reference's C++ names, so the reference host code links unchanged.
 *   - bf16 pointers are q3_bf16 (the 16 raw bits, layout-compatible with __nv_bfloat16).
 *   - cudaStream_t is passed as void * (0 = the legacy default stream).
 *
 * Ownership and graph rules are the reference's (src/forward.cu:196-227): every pointer is
 * caller-owned device memory, launchers allocate nothing and never synchronize, positions and
 * token ids are read from device memory inside the kernels, so a launch sequence captured in
 * a CUDA graph stays valid for every position. All kernels are launched with programmatic
 * stream serialization: each may start while the previous kernel on the stream finishes,
 * prefetching weights, and waits for it before touching activations.
 *
 * Preconditions, as in the reference: matrix column counts are multiples of 8 and matrix,
 * vector and cache pointers are 16-byte aligned (the reference's uint4 loads need the same,
 * src/kernels.cu:146-152); head_dim is a multiple of 32 up to 1024; n_heads is a multiple of
 * n_kv_heads.
 */
#ifndef QWEN3_B200_H
#define QWEN3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t q3_bf16;

enum q3_status {
    Q3_OK = 0,
    Q3_ERR_SHAPE = 1,    /* a size violates a precondition (the reference would exit) */
    Q3_ERR_ALIGN = 2,    /* a pointer is not 16-byte aligned */
    Q3_ERR_CUDA = 3,     /* a CUDA call failed; q3_last_cuda_error() gives the cudaError_t */
    Q3_ERR_DEVICE = 4,   /* the current device is not sm_100 (B200) */
    Q3_ERR_ARG = 5,      /* a null pointer or an invalid option */
    Q3_ERR_SCRATCH_LIMIT = 6, /* the shape needs more scratch than Q3_ATTENTION_STATIC_SCRATCH_BYTES */
};

/* Text for a q3_status value. */
const char *q3_status_string(int status);

/* The cudaError_t behind the most recent Q3_ERR_CUDA on this thread. */
int q3_last_cuda_error(void);

/* Reads and clears the device error flags that bounded waits and range checks inside the
 * kernels set (bit 0: a wait timed out, bit 1: token id out of range, bit 2: position out of
 * range). Synchronizes `stream` first. Returns a q3_status; the flags go to *flags. */
int q3_device_error(void *stream, unsigned *flags);

/* Self-test of the bounded waits the kernels use (no counterpart in the reference): launches one
 * wait on an mbarrier phase that nothing completes. The wait gives up after its time limit (about
 * two seconds), sets device flag bit 0 and returns; *done (device int) becomes 2. The context stays
 * usable. Used by the failure-detection test; never part of a decode step. */
int q3_selftest_wait_timeout(int *done, void *stream);

/* ---------------------------------------------------------------------------------------
 * Drop-in launchers (batch 1). Each replaces the launcher of the same name without the
 * q3_ prefix in src/kernels.cuh, with identical parameters.
 * ------------------------------------------------------------------------------------- */

/* src/kernels.cuh:7-8 embedding_forward: out[i] = table[*d_token * hidden + i]. */
int q3_embedding_forward(q3_bf16 *out, const q3_bf16 *table, const int *d_token, int hidden,
                         void *stream);

/* src/kernels.cuh:9-10 rmsnorm_forward: per row y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w). */
int q3_rmsnorm_forward(q3_bf16 *out, const q3_bf16 *in, const q3_bf16 *weight, int rows, int dim,
                       float eps, void *stream);

/* src/kernels.cuh:11 gemv_forward: out[r] = bf16(w[r] . x), w is [rows, cols] row-major. */
int q3_gemv_forward(q3_bf16 *out, const q3_bf16 *w, const q3_bf16 *x, int rows, int cols,
                    void *stream);

/* src/kernels.cuh:12-13 gemv_residual_forward: y = bf16(w[r] . in); tap[r] = y if tap;
 * x[r] = bf16(x[r] + y). */
int q3_gemv_residual_forward(q3_bf16 *x, const q3_bf16 *w, const q3_bf16 *in, int rows, int cols,
                             q3_bf16 *tap, void *stream);

/* src/kernels.cuh:14-15 qkv_forward: q = wq . x, k = wk . x, v = wv . x. */
int q3_qkv_forward(q3_bf16 *q, q3_bf16 *k, q3_bf16 *v, const q3_bf16 *wq, const q3_bf16 *wk,
                   const q3_bf16 *wv, const q3_bf16 *x, int q_rows, int kv_rows, int cols,
                   void *stream);

/* src/kernels.cuh:16-17 gate_up_forward: act[r] = bf16(bf16(silu(g)) * u) with
 * g = bf16(w_gate[r] . x), u = bf16(w_up[r] . x); gate_tap/up_tap receive g and u if non-null. */
int q3_gate_up_forward(q3_bf16 *act, const q3_bf16 *w_gate, const q3_bf16 *w_up,
                       const q3_bf16 *x, int rows, int cols, q3_bf16 *gate_tap, q3_bf16 *up_tap,
                       void *stream);

/* src/kernels.cuh:18-21 qk_norm_rope_forward: per-head RMSNorm of q and k, neox RoPE at
 * position *d_pos, in place; k and v are written to key_cache/value_cache row *d_pos (one
 * layer's [max_seq, n_kv_heads * head_dim] caches). q_tap/k_tap receive the normed heads. */
int q3_qk_norm_rope_forward(q3_bf16 *q, q3_bf16 *k, const q3_bf16 *v, const q3_bf16 *q_norm_w,
                            const q3_bf16 *k_norm_w, q3_bf16 *key_cache, q3_bf16 *value_cache,
                            const int *d_pos, int n_heads, int n_kv_heads, int head_dim, float eps,
                            float theta, q3_bf16 *q_tap, q3_bf16 *k_tap, void *stream);

/* src/kernels.cuh:22-24 attention_forward: GQA decode attention of q over cache positions
 * 0..*d_pos with the reference's rounding points; att is caller scratch [n_heads, max_seq]. */
int q3_attention_forward(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *key_cache,
                         const q3_bf16 *value_cache, float *att, int n_heads, int n_kv_heads,
                         int head_dim, const int *d_pos, int max_seq, float scale, void *stream);

/* src/kernels.cuh:25 argmax_forward: *out = index of the largest of x[0..n), lowest index on
 * ties, NaN never chosen. */
int q3_argmax_forward(int *out, const q3_bf16 *x, int n, void *stream);

/* src/kernels.cuh:26 sample_forward: inverse-CDF sample from softmax(x * inv_temp) with the
 * host uniform u in [0, 1); *out = -1 if no token is found. */
int q3_sample_forward(int *out, const q3_bf16 *x, int n, float inv_temp, float u, void *stream);

/* ---------------------------------------------------------------------------------------
 * Batched launchers: `batch` independent decode sequences. The reference has no batch
 * dimension; per sequence each computes what the reference launcher computes for it.
 * Activations are [batch, dim] row-major. A KV cache is addressed by three element strides:
 * the row of sequence b, position t, kv head h starts at
 * cache + b*cache_seq_stride + t*cache_pos_stride + h*cache_head_stride. The reference's layout
 * (one layer's [max_seq][n_kv_heads * head_dim]) is pos = n_kv_heads*head_dim, head = head_dim;
 * head-major caches ([n_kv_heads][max_seq][head_dim] per sequence: pos = head_dim,
 * head = max_seq*head_dim) keep each head's positions contiguous, which attention reads in
 * longer runs. Token ids and positions are per sequence in device memory. Projections with batch 1 run the bit-exact batch-1 kernels; batch >= 2 runs
 * the tcgen05 tensor-core GEMM (fp32 sums in the tensor core's order).
 * ------------------------------------------------------------------------------------- */

/* out[b] = table[d_tokens[b]]; an id outside [0, vocab) writes zeros and sets device error
 * bit 1 instead of reading outside the table. */
int q3_embedding_batched(q3_bf16 *out, const q3_bf16 *table, const int *d_tokens, int batch, int hidden,
                         int vocab, void *stream);

/* out[b][r] = bf16(w[r] . x[b]) */
int q3_gemv_batched(q3_bf16 *out, const q3_bf16 *w, const q3_bf16 *x, int batch, int rows, int cols,
                    void *stream);

/* x[b][r] = bf16(x[b][r] + bf16(w[r] . in[b])) */
int q3_gemv_residual_batched(q3_bf16 *x, const q3_bf16 *w, const q3_bf16 *in, int batch, int rows, int cols,
                             q3_bf16 *tap, void *stream);

int q3_qkv_batched(q3_bf16 *q, q3_bf16 *k, q3_bf16 *v, const q3_bf16 *wq, const q3_bf16 *wk, const q3_bf16 *wv,
                   const q3_bf16 *x, int batch, int q_rows, int kv_rows, int cols, void *stream);

int q3_gate_up_batched(q3_bf16 *act, const q3_bf16 *w_gate, const q3_bf16 *w_up, const q3_bf16 *x, int batch,
                       int rows, int cols, q3_bf16 *gate_tap, q3_bf16 *up_tap, void *stream);

/* qk_norm_rope_forward per sequence at position d_pos[b]; positions outside [0, max_seq) set
 * device error bit 2 and skip that sequence. */
int q3_qk_norm_rope_batched(q3_bf16 *q, q3_bf16 *k, const q3_bf16 *v, const q3_bf16 *q_norm_w,
                            const q3_bf16 *k_norm_w, q3_bf16 *key_cache, q3_bf16 *value_cache,
                            long long cache_seq_stride, long long cache_pos_stride, long long cache_head_stride,
                            const int *d_pos, int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                            float eps, float theta, q3_bf16 *q_tap, q3_bf16 *k_tap, void *stream);

/* Bytes of scratch q3_attention_batched needs (0 for unsupported shapes: head_dim above 256 or
 * a group size n_heads / n_kv_heads other than 1, 2, 4 or 8). */
size_t q3_attention_scratch_bytes(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq);

/* Split-KV attention per sequence over positions 0..d_pos[b], with the reference's rounding
 * points for scores and probabilities; `scratch` (size from q3_attention_scratch_bytes) needs no
 * initialization. Calls sharing a scratch buffer must not overlap on the GPU. */
int q3_attention_batched(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *key_cache, const q3_bf16 *value_cache,
                         long long cache_seq_stride, long long cache_pos_stride, long long cache_head_stride,
                         void *scratch, const int *d_pos, int batch, int n_heads, int n_kv_heads, int head_dim,
                         int max_seq, float scale, void *stream);

/* Size of the device array that q3_attention_batched_static uses as its scratch (32 MiB; every
 * GPU that loads this library holds it until the process exits). Enough, for example, for 32
 * sequences x 32 query heads x 4352 positions at head_dim 128. */
#define Q3_ATTENTION_STATIC_SCRATCH_BYTES (32u << 20)

/* q3_attention_batched without a scratch argument, for callers that cannot allocate device
 * memory while they run: a host runtime that reserves all of its GPU memory in one pool at
 * start-up, a plugin living inside another framework's memory manager, or a serving loop where
 * an allocation could block or fail mid-request. It allocates nothing: the scratch is a fixed
 * array in the library (Q3_ATTENTION_STATIC_SCRATCH_BYTES per device), and it runs the same
 * kernels as q3_attention_batched, so the results are the same. This entry point has no
 * counterpart in the reference.
 *   - Shapes whose scratch (q3_attention_scratch_bytes) exceeds the array return
 *     Q3_ERR_SCRATCH_LIMIT and launch nothing.
 *   - The first call on a device looks up the array's device address (once per device, with
 *     that device current); make that first call before any stream capture. The address is kept
 *     per device and CUDA context: after a cudaDeviceReset the next call looks it up again, so
 *     that call too should come before any capture.
 *   - Every call on a device shares the one array. Calls that overlap on the GPU (other
 *     streams, other host threads) race on it; serialize them. Nothing in the array needs
 *     clearing between calls: each call writes every scratch value before using it. */
int q3_attention_batched_static(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *key_cache,
                                const q3_bf16 *value_cache, long long cache_seq_stride, long long cache_pos_stride,
                                long long cache_head_stride, const int *d_pos, int batch, int n_heads,
                                int n_kv_heads, int head_dim, int max_seq, float scale, void *stream);

/* qk_norm_rope followed by attention (src/kernels.cu:301-403 then :439-497) for a few sequences
 * in one launch: q, k and v are the raw projections (unchanged by the call; the roped rows are
 * not written back), the new key and value rows go to row d_pos[b] of the caches (strides as
 * above), and out receives the attention output. Each (sequence, kv head)'s positions are cut
 * into `chunks` contiguous ranges, the CTAs of one thread-block cluster, which exchange the
 * softmax statistics and their partial outputs through distributed shared memory; it needs no
 * scratch memory. Probabilities are the reference's bit for bit, and only the fp32 order of the
 * P.V sum differs (chunk partials added in chunk order; chunks = 1 gives the reference's output
 * bit for bit).
 *   - q3_rope_attention_chunks gives the chunk count for `batch` sequences of up to max_seq
 *     positions on the current device (2 to 16: the largest whose clusters all fit at once),
 *     or 0 when the kernel does not apply: head_dim other than 64 or 128,
 *     n_heads / n_kv_heads other than 1, 2, 4 or 8, or too many sequences.
 *   - chunks is 1 to 16; Q3_ERR_SHAPE if one cluster of that size (with its chunk's scores in
 *     shared memory) does not fit on the device. With batch > 1 the sequences must have separate
 *     caches (cache_seq_stride > 0).
 * No counterpart in the reference (it launches the two kernels one after the other). */
int q3_rope_attention_chunks(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq);
int q3_rope_attention_batched(q3_bf16 *out, const q3_bf16 *q, const q3_bf16 *k, const q3_bf16 *v,
                              const q3_bf16 *q_norm_w, const q3_bf16 *k_norm_w, q3_bf16 *key_cache,
                              q3_bf16 *value_cache, long long cache_seq_stride, long long cache_pos_stride,
                              long long cache_head_stride, const int *d_pos, int batch, int n_heads, int n_kv_heads,
                              int head_dim, int max_seq, float eps, float theta, float scale, int chunks,
                              void *stream);

/* out[b] = argmax of x[b][0..n) with argmax_forward's tie and NaN rules. */
int q3_argmax_batched(int *out, const q3_bf16 *x, int batch, int n, void *stream);

/* dst[i] = bf16(mean + std * N(0,1)), a counter-based generator seeded by `seed` (synthetic
 * weights and KV caches for benchmarks). */
int q3_fill_normal_bf16(q3_bf16 *dst, long long n, unsigned long long seed, float mean, float std, void *stream);

/* ---------------------------------------------------------------------------------------
 * Decode engine: the reference's forward pass (src/forward.cu:118-236) for `batch`
 * sequences with all state on the device and one CUDA graph per decode step.
 * ------------------------------------------------------------------------------------- */

/* The model shape, as src/model.cuh:10-24 (Config) reads it from config.json. */
typedef struct q3_config {
    int hidden_size;
    int intermediate_size;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int vocab_size;
    float rms_norm_eps;
    float rope_theta;
} q3_config;

/* Device pointers of one layer, fields as src/model.cuh:26-39 (LayerWeights); matrices are
 * [out, in] row-major. */
typedef struct q3_layer_weights {
    const q3_bf16 *attn_norm, *wq, *wk, *wv, *q_norm, *k_norm, *wo, *mlp_norm, *w_gate, *w_up, *w_down;
} q3_layer_weights;

/* src/model.cuh:47-59 (Weights): `layers` is a host array of n_layers entries; lm_head equals
 * embed for tied embeddings. The engine keeps the pointers, not copies of the weights. */
typedef struct q3_weights {
    const q3_bf16 *embed;
    const q3_layer_weights *layers;
    const q3_bf16 *final_norm;
    const q3_bf16 *lm_head;
} q3_weights;

typedef struct q3_engine q3_engine;

/* Device buffers of an engine, for inspection. */
typedef struct q3_engine_buffers {
    q3_bf16 *x;            /* [batch, hidden] residual stream after the last step */
    q3_bf16 *logits;       /* [batch, vocab] */
    q3_bf16 *key_cache;    /* [n_layers][batch][n_kv_heads][max_seq][head_dim] (head-major) */
    q3_bf16 *value_cache;
    int *next_token;       /* [batch] read by the next step's embedding */
    int *pos;              /* [batch] position the next step writes and attends up to */
    int *out_token;        /* [batch] argmax of the last step */
    int *history;          /* [history_cap][batch] tokens of steps 0, 1, ... */
    int *step;             /* steps run since creation */
    int batch, max_seq, history_cap;
    int launches_per_step; /* kernel launches in the captured step the next q3_engine_step runs
                              (0 before q3_engine_capture) */
    int split_from;        /* with the fused RoPE + attention launch (small batches): the position
                              of the longest sequence from which a step runs the split-KV kernels
                              instead, captured as a second graph; -1 when one path serves every
                              position */
} q3_engine_buffers;

enum {
    Q3_ENGINE_EXACT_ATTENTION = 1, /* bit-exact single-chunk attention instead of split-KV */
    /* batch 1 only: each step is one cooperative kernel whose CTAs pass through the step's phases
     * (norms, projections, RoPE, attention, LM head, argmax) separated by grid barriers, instead
     * of ~290 kernels; per-row arithmetic as in the other path, P.V summed in 128-position parts */
    Q3_ENGINE_MEGAKERNEL = 2,
    /* keep the separate RoPE kernel and the four-kernel split-KV attention even for batches where
     * q3_rope_attention_batched's single launch applies (it is the default there) */
    Q3_ENGINE_SPLIT_ATTENTION = 4
};

/* src/forward.cu:83-114 weight_bytes_per_step and kv_bytes_per_position. */
size_t q3_weight_bytes_per_step(const q3_config *cfg);
size_t q3_kv_bytes_per_position(const q3_config *cfg);

/* Allocates the run state for `batch` sequences of up to `max_seq` positions (caches zeroed,
 * tokens and positions 0) on the current device; work goes to `stream`, or to a stream the
 * engine creates when `stream` is 0 (the legacy default stream cannot be captured). */
int q3_engine_create(const q3_config *cfg, const q3_weights *weights, int batch, int max_seq, int history_cap,
                     int flags, void *stream, q3_engine **out);
int q3_engine_destroy(q3_engine *e);

/* Captures one decode step into a CUDA graph (src/forward.cu:196-204); q3_engine_step then
 * replays it. Without a capture, steps launch their kernels one by one. */
int q3_engine_capture(q3_engine *e);

/* Runs n decode steps back to back on the device: each embeds next_token[b], runs the layers at
 * pos[b], and its argmax writes next_token[b], out_token[b] and history, then advances pos[b]. */
int q3_engine_step(q3_engine *e, int n_steps);

/* Copies host token ids and positions ([batch] each) to the device (src/forward.cu:218-220). */
int q3_engine_set_state(q3_engine *e, const int *tokens, const int *positions);

/* The reference's per-token protocol: forward = set_state + one step (src/forward.cu:206-227);
 * sample_argmax copies the step's tokens to the host and waits for them (:229-236). */
int q3_engine_forward(q3_engine *e, const int *tokens, const int *positions);
int q3_engine_sample_argmax(q3_engine *e, int *tokens_out);

/* Prefill (the reference feeds a prompt one token per forward, src/main.cu:122-124): runs the
 * n_tokens host token ids of sequence `seq` at positions start_pos .. start_pos + n_tokens - 1
 * through the layers, up to `batch` tokens per pass. The rows of a pass share the sequence's
 * cache and attend causally (row i sees positions up to its own). Their K and V rows are written
 * to the cache. next_token[seq] / out_token[seq] become the argmax of the last token's logits and
 * pos[seq] becomes start_pos + n_tokens, so decode steps continue from there. Other sequences'
 * caches and state are left as they were; the logits buffer is overwritten. Waits for its work. */
int q3_engine_prefill(q3_engine *e, int seq, const int *tokens, int n_tokens, int start_pos);

/* Fills cache positions [0, n_positions) of every layer and sequence with bf16 N(0,1). */
int q3_engine_fill_kv_normal(q3_engine *e, int n_positions, unsigned long long seed);

int q3_engine_info(const q3_engine *e, q3_engine_buffers *out);

#ifdef __cplusplus
}
#endif

#endif /* QWEN3_B200_H */
