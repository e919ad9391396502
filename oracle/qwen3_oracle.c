/*
 * CPU restatement of the reference decode kernels -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity checker for the sm_100a kernels in llm-inference_b200/csrc.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it,
 * and only to check results. The product path never calls it.
 *
 * Each function restates the arithmetic of one kernel of the reference engine
 * (William-Lamer/llm-inference, src/kernels.cu) in plain C, in the same order:
 * the same per-thread partial sums, the same warp-shuffle trees, the same serial
 * sums of warp partials and the same bf16 rounding points. Where nvcc contracts
 * `a += b * c` into one fused multiply-add, this file calls fmaf(); it is built
 * with -ffp-contract=off so that nothing else is fused.
 *
 * Differences from the GPU, which are the only sources of mismatch:
 *   - rsqrtf: CUDA's is a hardware approximation; here it is 1/sqrtf.
 *   - expf, powf, cosf, sinf come from the host libm, not from CUDA's libdevice.
 * Both change fp32 results in the last bit or two, which moves a bf16 result by at
 * most one unit in rare cases. The tests state that tolerance beside each check.
 *
 * Parity pins: tests/golden/ref_kernels.npz holds outputs of the reference kernels
 * themselves (compiled for sm_100a and run on a B200 by tests/golden/make_ref_kernel_golden.py),
 * and tests/golden/hf_tiny/ holds the reference's Hugging Face harness dumps
 * (tests/golden/make_hf_golden.py). tests/test_oracle_golden.py checks this file against both.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef uint16_t bf16_t;

static inline float bf2f(bf16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* round to nearest even, NaN -> canonical 0x7fff (cvt.rn.bf16.f32 behaviour) */
static inline bf16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (bf16_t)(u >> 16);
}

static inline float round_bf16(float v) { return bf2f(f2bf(v)); }

float oracle_bf16_to_float(bf16_t h) { return bf2f(h); }
bf16_t oracle_float_to_bf16(float f) { return f2bf(f); }

/* __shfl_xor_sync butterfly over one warp: every lane ends with the same sum. */
static float warp_xor_sum(float *lanes) {
    float tmp[32];
    for (int off = 16; off > 0; off >>= 1) {
        for (int l = 0; l < 32; l++) tmp[l] = lanes[l] + lanes[l ^ off];
        memcpy(lanes, tmp, sizeof(tmp));
    }
    return lanes[0];
}

/* __shfl_down_sync tree over one warp; the result is lane 0's value.
 * A lane whose source is past lane 31 keeps its own value (only lane 0 is used). */
static float warp_down_sum(float *lanes) {
    float tmp[32];
    for (int off = 16; off > 0; off >>= 1) {
        for (int l = 0; l < 32; l++) tmp[l] = lanes[l] + (l + off < 32 ? lanes[l + off] : lanes[l]);
        memcpy(lanes, tmp, sizeof(tmp));
    }
    return lanes[0];
}

/* src/kernels.cu:7-23 embedding_kernel */
void oracle_embedding(bf16_t *out, const bf16_t *table, int token, int hidden) {
    memcpy(out, table + (size_t)token * hidden, (size_t)hidden * sizeof(bf16_t));
}

/* src/kernels.cu:25-71 rmsnorm_kernel, launched with 256 threads per row (:68). */
void oracle_rmsnorm(bf16_t *out, const bf16_t *in, const bf16_t *weight, int rows, int dim,
                    float eps) {
    enum { BLOCK = 256 };
    for (int row = 0; row < rows; row++) {
        const bf16_t *x = in + (size_t)row * dim;
        bf16_t *y = out + (size_t)row * dim;
        float part[BLOCK];
        for (int t = 0; t < BLOCK; t++) {
            float s = 0.0f;
            for (int i = t; i < dim; i += BLOCK) {
                float v = bf2f(x[i]);
                s = fmaf(v, v, s);
            }
            part[t] = s;
        }
        float total = 0.0f;
        for (int w = 0; w < BLOCK / 32; w++) total += warp_xor_sum(part + 32 * w);
        float inv_rms = 1.0f / sqrtf(total / dim + eps);
        for (int i = 0; i < dim; i++) {
            float v = bf2f(x[i]);
            float normed = round_bf16(v * inv_rms);
            y[i] = f2bf(normed * bf2f(weight[i]));
        }
    }
}

/* src/kernels.cu:79-106 warp_dot: lane l sums 16-byte chunks l, l+32, ... with one FMA per
 * element, then a __shfl_down_sync tree. */
static float warp_dot(const bf16_t *w, const bf16_t *x, int cols) {
    int n_vec = cols / 8;
    float lanes[32];
    for (int l = 0; l < 32; l++) {
        float s = 0.0f;
        for (int i = l; i < n_vec; i += 32) {
            const bf16_t *wc = w + 8 * i;
            const bf16_t *xc = x + 8 * i;
            for (int e = 0; e < 8; e++) s = fmaf(bf2f(wc[e]), bf2f(xc[e]), s);
        }
        lanes[l] = s;
    }
    return warp_down_sum(lanes);
}

/* src/kernels.cu:159-182 gemv_kernel */
void oracle_gemv(bf16_t *out, const bf16_t *w, const bf16_t *x, int rows, int cols) {
    for (int r = 0; r < rows; r++) out[r] = f2bf(warp_dot(w + (size_t)r * cols, x, cols));
}

/* src/kernels.cu:185-212 gemv_residual_kernel: x[r] = bf16(x[r] + bf16(W[r].in)) */
void oracle_gemv_residual(bf16_t *x, const bf16_t *w, const bf16_t *in, int rows, int cols,
                          bf16_t *tap) {
    for (int r = 0; r < rows; r++) {
        bf16_t y = f2bf(warp_dot(w + (size_t)r * cols, in, cols));
        if (tap) tap[r] = y;
        x[r] = f2bf(bf2f(x[r]) + bf2f(y));
    }
}

/* src/kernels.cu:215-257 qkv_kernel */
void oracle_qkv(bf16_t *q, bf16_t *k, bf16_t *v, const bf16_t *wq, const bf16_t *wk,
                const bf16_t *wv, const bf16_t *x, int q_rows, int kv_rows, int cols) {
    oracle_gemv(q, wq, x, q_rows, cols);
    oracle_gemv(k, wk, x, kv_rows, cols);
    oracle_gemv(v, wv, x, kv_rows, cols);
}

/* src/kernels.cu:260-298 gate_up_kernel; warp_dot2 (:109-144) has the same per-row order
 * as warp_dot. act = bf16(round_bf16(g / (1 + expf(-g))) * u) with g, u rounded to bf16. */
void oracle_gate_up(bf16_t *act, const bf16_t *w_gate, const bf16_t *w_up, const bf16_t *x,
                    int rows, int cols, bf16_t *gate_tap, bf16_t *up_tap) {
    for (int r = 0; r < rows; r++) {
        bf16_t gate = f2bf(warp_dot(w_gate + (size_t)r * cols, x, cols));
        bf16_t up = f2bf(warp_dot(w_up + (size_t)r * cols, x, cols));
        if (gate_tap) {
            gate_tap[r] = gate;
            up_tap[r] = up;
        }
        float g = bf2f(gate);
        float u = bf2f(up);
        float silu = round_bf16(g / (1.0f + expf(-g)));
        act[r] = f2bf(silu * u);
    }
}

/* src/kernels.cu:301-403 qk_norm_rope_kernel: one block of head_dim threads per q or k head.
 * key_cache / value_cache are one layer's [max_seq, kv_dim] caches. */
void oracle_qk_norm_rope(bf16_t *q, bf16_t *k, const bf16_t *v, const bf16_t *q_norm_w,
                         const bf16_t *k_norm_w, bf16_t *key_cache, bf16_t *value_cache, int pos,
                         int n_heads, int n_kv_heads, int head_dim, float eps, float theta,
                         bf16_t *q_tap, bf16_t *k_tap) {
    int kv_dim = n_kv_heads * head_dim;
    int half = head_dim / 2;
    float *lanes = (float *)malloc(sizeof(float) * head_dim);
    bf16_t *normed = (bf16_t *)malloc(sizeof(bf16_t) * head_dim);
    for (int blk = 0; blk < n_heads + n_kv_heads; blk++) {
        int is_key = blk >= n_heads;
        int head = is_key ? blk - n_heads : blk;
        bf16_t *x = is_key ? k + head * head_dim : q + head * head_dim;
        const bf16_t *nw = is_key ? k_norm_w : q_norm_w;
        bf16_t *tap = is_key ? k_tap : q_tap;
        for (int i = 0; i < head_dim; i++) {
            float xi = bf2f(x[i]);
            lanes[i] = xi * xi;
        }
        float total = 0.0f;
        for (int w = 0; w < head_dim / 32; w++) total += warp_xor_sum(lanes + 32 * w);
        float inv_rms = 1.0f / sqrtf(total / head_dim + eps);
        for (int i = 0; i < head_dim; i++) {
            float nv = round_bf16(bf2f(x[i]) * inv_rms);
            normed[i] = f2bf(nv * bf2f(nw[i]));
            if (tap) tap[head * head_dim + i] = normed[i];
        }
        size_t slot = (size_t)pos * kv_dim + (size_t)head * head_dim;
        for (int j = 0; j < half; j++) {
            float inv_freq = 1.0f / powf(theta, (float)(2 * j) / head_dim);
            float angle = pos * inv_freq;
            float c = round_bf16(cosf(angle));
            float s = round_bf16(sinf(angle));
            float a = bf2f(normed[j]);
            float b = bf2f(normed[j + half]);
            float a_cos = round_bf16(a * c);
            float b_sin = round_bf16(b * s);
            float b_cos = round_bf16(b * c);
            float a_sin = round_bf16(a * s);
            bf16_t out_a = f2bf(a_cos - b_sin);
            bf16_t out_b = f2bf(b_cos + a_sin);
            x[j] = out_a;
            x[j + half] = out_b;
            if (is_key) {
                key_cache[slot + j] = out_a;
                key_cache[slot + j + half] = out_b;
            }
        }
        if (is_key)
            for (int i = 0; i < head_dim; i++) value_cache[slot + i] = v[head * head_dim + i];
    }
    free(lanes);
    free(normed);
}

/* The scores step of src/kernels.cu:450-461 alone: scores[h][t] = round_bf16(round_bf16(dot) * scale)
 * with dot the serial fused multiply-add chain over head_dim, for t = 0..pos, into out[h * (pos + 1) + t]. */
void oracle_scores(float *out, const bf16_t *q, const bf16_t *key_cache, int n_heads, int n_kv_heads, int head_dim,
                   int pos, float scale) {
    int n_rep = n_heads / n_kv_heads;
    int kv_dim = n_kv_heads * head_dim;
    for (int h = 0; h < n_heads; h++) {
        const bf16_t *qh = q + (size_t)h * head_dim;
        for (int t = 0; t <= pos; t++) {
            const bf16_t *kt = key_cache + (size_t)t * kv_dim + (size_t)(h / n_rep) * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot = fmaf(bf2f(qh[d]), bf2f(kt[d]), dot);
            out[(size_t)h * (pos + 1) + t] = round_bf16(round_bf16(dot) * scale);
        }
    }
}

/* src/kernels.cu:439-497 attention_kernel, 128 threads per q head (:492).
 * block_sum (:406-420): xor tree per warp, then a serial sum of the warp partials. */
void oracle_attention(bf16_t *out, const bf16_t *q, const bf16_t *key_cache,
                      const bf16_t *value_cache, int n_heads, int n_kv_heads, int head_dim,
                      int pos, float scale) {
    enum { BLOCK = 128 };
    int n_rep = n_heads / n_kv_heads;
    int kv_dim = n_kv_heads * head_dim;

    for (int h = 0; h < n_heads; h++) {
        int kv_head = h / n_rep;
        const bf16_t *qh = q + (size_t)h * head_dim;
        float *scores = (float *)malloc(sizeof(float) * (pos + 1));
        for (int t = 0; t <= pos; t++) {
            const bf16_t *kt = key_cache + (size_t)t * kv_dim + (size_t)kv_head * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; d++) dot = fmaf(bf2f(qh[d]), bf2f(kt[d]), dot);
            scores[t] = round_bf16(round_bf16(dot) * scale);
        }
        float max_score = -INFINITY;
        for (int t = 0; t <= pos; t++) max_score = fmaxf(max_score, scores[t]);
        float part[BLOCK];
        for (int j = 0; j < BLOCK; j++) {
            float s = 0.0f;
            for (int t = j; t <= pos; t += BLOCK) s += expf(scores[t] - max_score);
            part[j] = s;
        }
        float sum_exp = 0.0f;
        for (int w = 0; w < BLOCK / 32; w++) sum_exp += warp_xor_sum(part + 32 * w);
        for (int t = 0; t <= pos; t++) scores[t] = round_bf16(expf(scores[t] - max_score) / sum_exp);
        for (int d = 0; d < head_dim; d++) {
            float acc = 0.0f;
            for (int t = 0; t <= pos; t++) {
                const bf16_t *vt = value_cache + (size_t)t * kv_dim + (size_t)kv_head * head_dim;
                acc = fmaf(scores[t], bf2f(vt[d]), acc);
            }
            out[(size_t)h * head_dim + d] = f2bf(acc);
        }
        free(scores);
    }
}

/* src/kernels.cu:500-544 argmax: larger value wins, ties go to the lowest index, NaN never
 * wins. The combine is associative, so a sequential scan gives the kernel's answer. */
int oracle_argmax(const bf16_t *x, int n) {
    float best_val = -INFINITY;
    int best_idx = 2147483647;
    for (int i = 0; i < n; i++) {
        float v = bf2f(x[i]);
        if (v > best_val || (v == best_val && i < best_idx)) {
            best_val = v;
            best_idx = i;
        }
    }
    return best_idx;
}

/* src/kernels.cu:546-602 sample_kernel with 1024 threads: per-thread chunk sums of
 * expf((x - max) * inv_temp), a serial total, then an inverse-CDF walk over the chunks. */
int oracle_sample(const bf16_t *x, int n, float inv_temp, float u) {
    enum { BLOCK = 1024 };
    float max_val = -INFINITY;
    for (int i = 0; i < n; i++) max_val = fmaxf(max_val, bf2f(x[i]));
    int chunk = (n + BLOCK - 1) / BLOCK;
    float *sums = (float *)malloc(sizeof(float) * BLOCK);
    for (int t = 0; t < BLOCK; t++) {
        int start = t * chunk;
        int end = start + chunk < n ? start + chunk : n;
        float s = 0.0f;
        for (int i = start; i < end; i++) s += expf((bf2f(x[i]) - max_val) * inv_temp);
        sums[t] = s;
    }
    float total = 0.0f;
    for (int t = 0; t < BLOCK; t++) total += sums[t];
    float target = u * total;
    float cdf = 0.0f;
    int t = 0;
    while (t < BLOCK - 1 && cdf + sums[t] <= target) {
        cdf += sums[t];
        t++;
    }
    int chosen = -1;
    int cs = t * chunk;
    int ce = cs + chunk < n ? cs + chunk : n;
    float s = 0.0f;
    for (int i = cs; i < ce; i++) {
        s += expf((bf2f(x[i]) - max_val) * inv_temp);
        if (cdf + s > target) {
            chosen = i;
            break;
        }
    }
    free(sums);
    return chosen;
}
