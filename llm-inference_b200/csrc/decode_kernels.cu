// Embedding gather, RMSNorm, QK-norm + RoPE + KV-cache write, argmax and sampling for sm_100a.
//
// Every kernel reproduces the arithmetic of the reference kernel it replaces
// (src/kernels.cu:7-71, :301-403, :500-602): the same per-thread partial sums, shuffle trees,
// serial sums of warp partials and bf16 rounding points, so the results are bit-identical.
// What changes is the parallel shape around that arithmetic: a batch dimension (grid.y, with
// per-sequence strides, token ids and positions read from device memory), vector loads,
// programmatic dependent launch, and an argmax spread over a cluster of CTAs that combine
// their partial results through distributed shared memory.
#include <cooperative_groups.h>
#include <limits.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ------------------------------------------------------------------ embedding
// out[b, i] = table[tokens[b] * hidden + i]   (src/kernels.cu:7-23, with a batch of tokens)
// vocab > 0 enables a range check: an out-of-range id writes zeros and raises
// DEV_ERR_TOKEN_RANGE instead of reading outside the table.
template <bool VEC>
__global__ void embedding_kernel(bf16 *out, const bf16 *table, const int *tokens, int hidden,
                                 int vocab) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.y;
    const int token = tokens[b];
    const bool bad = vocab > 0 && (token < 0 || token >= vocab);
    if (bad && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&g_dev_error, DEV_ERR_TOKEN_RANGE);
    bf16 *dst = out + (size_t)b * hidden;
    const bf16 *src = table + (size_t)(bad ? 0 : token) * hidden;
    if (VEC) {
        const int n = hidden / 8;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
            uint4 v = bad ? make_uint4(0, 0, 0, 0) : reinterpret_cast<const uint4 *>(src)[i];
            reinterpret_cast<uint4 *>(dst)[i] = v;
        }
    } else {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
            dst[i] = bad ? __float2bfloat16(0.0f) : src[i];
    }
}

// ------------------------------------------------------------------ rmsnorm
// src/kernels.cu:25-71, one 256-thread block per row, same reduction order. Rows of up to
// RMS_CACHE * 256 elements stay in registers between the two passes, and the weight, which no
// kernel writes, is loaded before the wait on the previous kernel.
constexpr int RMS_CACHE = 16;

__global__ void __launch_bounds__(256) rmsnorm_kernel(bf16 *out, const bf16 *in, const bf16 *weight,
                                                      int dim, float eps) {
    pdl_trigger();
    const bool cached = dim <= RMS_CACHE * 256;
    float wv[RMS_CACHE], xv[RMS_CACHE];
    if (cached) {
#pragma unroll
        for (int j = 0; j < RMS_CACHE; j++) {
            const int i = threadIdx.x + j * 256;
            wv[j] = i < dim ? __bfloat162float(weight[i]) : 0.0f;
        }
    }
    pdl_wait();
    const bf16 *x = in + (size_t)blockIdx.x * dim;
    bf16 *y = out + (size_t)blockIdx.x * dim;
    float sum = 0.0f;
    if (cached) {
#pragma unroll
        for (int j = 0; j < RMS_CACHE; j++) {
            const int i = threadIdx.x + j * 256;
            xv[j] = i < dim ? __bfloat162float(x[i]) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < RMS_CACHE; j++)
            if (threadIdx.x + j * 256 < dim) sum = __fmaf_rn(xv[j], xv[j], sum);
    } else {
        for (int i = threadIdx.x; i < dim; i += 256) {
            const float v = __bfloat162float(x[i]);
            sum = __fmaf_rn(v, v, sum);
        }
    }
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    __shared__ float warp_sums[8];
    if (threadIdx.x % 32 == 0) warp_sums[threadIdx.x / 32] = sum;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) total += warp_sums[w];
    const float inv_rms = rsqrtf(total / dim + eps);
    if (cached) {
#pragma unroll
        for (int j = 0; j < RMS_CACHE; j++) {
            const int i = threadIdx.x + j * 256;
            if (i < dim) y[i] = __float2bfloat16(round_bf16(xv[j] * inv_rms) * wv[j]);
        }
    } else {
        for (int i = threadIdx.x; i < dim; i += 256) {
            const float v = __bfloat162float(x[i]);
            const bf16 normed = __float2bfloat16(v * inv_rms);
            y[i] = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(weight[i]));
        }
    }
}

// ------------------------------------------------------------------ qk_norm_rope
// The per-head RMSNorm, RoPE and cache write of src/kernels.cu:301-403, one WARP per (sequence,
// q or k head) instead of one head_dim-thread block: the reference's block of head_dim threads is
// head_dim / 32 warps, and lane l here holds the elements l, l + 32, ... of the head -- element
// l + 32*j is the reference's warp j, lane l. So the same arithmetic runs without a block barrier
// or shared-memory exchange:
//   - the sum of squares: per element x*x, one xor-shuffle tree per reference warp j (all lanes
//     end with the bit-identical warp total), the totals added in j order from 0 -- the
//     reference's warp_sums loop;
//   - rsqrtf(total / head_dim + eps), then bf16(bf16(x * inv_rms) * w) per element;
//   - RoPE pairs element t with t + head_dim/2. For head_dim a multiple of 64 both sit in the same
//     lane (slots j and j + head_dim/64), so each lane rotates its own pairs in registers; other
//     head widths exchange the normed head through the warp's slice of shared memory.
// The rotation angle depends on the position and the pair only, so a CTA -- one sequence's block
// of eight heads -- computes the rounded cos / sin of each pair once, before its warps start
// (the reference computes them per head; the values are the same). Each product keeps the
// reference's rounding: c and s rounded to bf16, each product rounded, then the difference and
// the sum. q/k/v strides are in elements between consecutive sequences; the cache row of sequence
// b, position t, kv head h starts at key_cache + b*kv.seq + t*kv.pos + h*kv.head.
struct RopeArgs {
    bf16 *q, *k;
    const bf16 *v;
    const bf16 *q_norm_w, *k_norm_w;
    bf16 *key_cache, *value_cache;
    const int *pos;
    bf16 *q_tap, *k_tap;
    long long q_stride, kv_stride;
    KvLayout kv;
    int n_heads, n_kv_heads, head_dim;
    int max_seq;  // > 0: positions are range-checked
    float eps, theta;
};

constexpr int ROPE_WARPS = 8;  // heads per CTA
constexpr int ROPE_EPL = 32;   // elements per lane at the largest head_dim (1024)

// EPL: elements per lane (head_dim / 32) when fixed at compile time -- then a pair's two
// elements are registers j and j + EPL/2 of one lane -- or 0 for any head_dim, whose pairs meet
// in shared memory. Grid: (head blocks of ROPE_WARPS, sequences).
template <int EPL>
__global__ void __launch_bounds__(ROPE_WARPS * 32) qk_norm_rope_kernel(const __grid_constant__ RopeArgs a) {
    constexpr int NE = EPL > 0 ? EPL : ROPE_EPL;
    constexpr bool REG_PAIRS = EPL > 0 && EPL % 2 == 0;
    __shared__ float cs_s[512], sn_s[512];  // rounded cos / sin of each pair at this position
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x % 32, wib = threadIdx.x / 32;
    const int b = blockIdx.y;
    const int D = EPL > 0 ? 32 * EPL : a.head_dim, epl = D / 32, half = D / 2;
    const int pos = a.pos[b];
    if (a.max_seq > 0 && (pos < 0 || pos >= a.max_seq)) {  // uniform over the CTA
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&g_dev_error, DEV_ERR_POS_RANGE);
        return;
    }
    for (int t = threadIdx.x; t < half; t += ROPE_WARPS * 32) {  // src/kernels.cu:359-365
        const float inv_freq = 1.0f / powf(a.theta, (float)(2 * t) / D);
        const float angle = pos * inv_freq;
        cs_s[t] = round_bf16(cosf(angle));
        sn_s[t] = round_bf16(sinf(angle));
    }
    __syncthreads();
    int head = blockIdx.x * ROPE_WARPS + wib;
    if (head >= a.n_heads + a.n_kv_heads) return;
    const bool is_key = head >= a.n_heads;
    bf16 *x;
    const bf16 *norm_w;
    bf16 *tap;
    if (is_key) {
        head -= a.n_heads;
        x = a.k + b * a.kv_stride + head * D;
        norm_w = a.k_norm_w;
        tap = a.k_tap ? a.k_tap + b * a.kv_stride + head * D : nullptr;
    } else {
        x = a.q + b * a.q_stride + head * D;
        norm_w = a.q_norm_w;
        tap = a.q_tap ? a.q_tap + b * a.q_stride + head * D : nullptr;
    }

    float xv[NE];
#pragma unroll
    for (int j = 0; j < NE; j++)
        if (j < epl) xv[j] = __bfloat162float(x[lane + 32 * j]);
    float total = 0.0f;
#pragma unroll
    for (int j = 0; j < NE; j++) {
        if (j < epl) {
            // separate multiply and adds, as the reference's `sum = xi * xi; sum += shfl(...)`
            // (no contraction into a fused multiply-add)
            float sum = __fmul_rn(xv[j], xv[j]);
            for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
            total = __fadd_rn(total, sum);
        }
    }
    const float inv_rms = rsqrtf(total / D + a.eps);
    float y[NE];
#pragma unroll
    for (int j = 0; j < NE; j++) {
        if (j < epl) {
            const int t = lane + 32 * j;
            const bf16 normed = __float2bfloat16(xv[j] * inv_rms);
            const bf16 yb = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(norm_w[t]));
            if (tap != nullptr) tap[t] = yb;
            y[j] = __bfloat162float(yb);
        }
    }
    bf16 *stage = nullptr;
    if constexpr (!REG_PAIRS) {
        __shared__ bf16 stage_s[ROPE_WARPS][1024];
        stage = stage_s[wib];
#pragma unroll
        for (int j = 0; j < NE; j++)
            if (j < epl) stage[lane + 32 * j] = __float2bfloat16(y[j]);
        __syncwarp();
    }

    const size_t slot = (size_t)b * a.kv.seq + (size_t)pos * a.kv.pos + (size_t)head * a.kv.head;
#pragma unroll
    for (int j = 0; j < NE; j++) {
        const int t = lane + 32 * j;  // the pair's first element
        if (j < epl && t < half) {
            const float c = cs_s[t], sn = sn_s[t];
            float av, bv;
            if constexpr (REG_PAIRS) {
                av = y[j];
                bv = y[(j + EPL / 2) % NE];  // j < EPL / 2 here
            } else {
                av = __bfloat162float(stage[t]);
                bv = __bfloat162float(stage[t + half]);
            }
            const float a_cos = round_bf16(av * c);
            const float b_sin = round_bf16(bv * sn);
            const float b_cos = round_bf16(bv * c);
            const float a_sin = round_bf16(av * sn);
            const bf16 out_a = __float2bfloat16(a_cos - b_sin);
            const bf16 out_b = __float2bfloat16(b_cos + a_sin);
            x[t] = out_a;
            x[t + half] = out_b;
            if (is_key) {
                a.key_cache[slot + t] = out_a;
                a.key_cache[slot + t + half] = out_b;
            }
        }
    }
    if (is_key) {
        const bf16 *vh = a.v + b * a.kv_stride + head * D;
#pragma unroll
        for (int j = 0; j < NE; j++)
            if (j < epl) a.value_cache[slot + lane + 32 * j] = vh[lane + 32 * j];
    }
}

// ------------------------------------------------------------------ argmax
// src/kernels.cu:500-544. The combine keeps the larger value and, on ties, the lower index;
// NaN never wins. That combine is associative and commutative, so any split gives the same
// answer. Here a cluster of ARGMAX_CTAS CTAs covers one row; each CTA reduces its slice, and
// CTA rank 0 gathers the partial results from the others' shared memory.
constexpr int ARGMAX_CTAS = 8;
constexpr int ARGMAX_THREADS = 512;

__device__ __forceinline__ void argmax_pair(float &val, int &idx, float v2, int i2) {
    if (v2 > val || (v2 == val && i2 < idx)) {
        val = v2;
        idx = i2;
    }
}

struct ArgmaxOut {
    int *out;          // out[b]
    int *next_token;   // optional: next_token[b] = out[b] (decode loop)
    int *pos;          // optional: pos[b] += 1 (decode loop)
    int *history;      // optional: history[*step * n_rows + b] = token while *step < history_cap
    int *step;         // optional: step counter, incremented once per launch
    int history_cap;   // rows of `history`
};

template <bool VEC>
__global__ void __launch_bounds__(ARGMAX_THREADS) argmax_kernel(const bf16 *x, int n, long long row_stride,
                                                                ArgmaxOut o) {
    pdl_trigger();
    pdl_wait();
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int row = blockIdx.x / ARGMAX_CTAS;
    const bf16 *xr = x + row * row_stride;

    // CTA slice in units of 8 elements
    const int n8 = (n + 7) / 8;
    const int c0 = (int)((long long)n8 * rank / ARGMAX_CTAS);
    const int c1 = (int)((long long)n8 * (rank + 1) / ARGMAX_CTAS);
    float best_val = -INFINITY;
    int best_idx = INT_MAX;
    for (int c = c0 + threadIdx.x; c < c1; c += ARGMAX_THREADS) {
        const int base = c * 8;
        if (VEC && base + 8 <= n) {
            const bf16x8 v = ldg128(xr + base);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float2 f = __bfloat1622float2(v.h[k]);
                argmax_pair(best_val, best_idx, f.x, base + 2 * k);
                argmax_pair(best_val, best_idx, f.y, base + 2 * k + 1);
            }
        } else {
            for (int e = base; e < min(base + 8, n); e++)
                argmax_pair(best_val, best_idx, __bfloat162float(xr[e]), e);
        }
    }
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_val, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_idx, off);
        argmax_pair(best_val, best_idx, ov, oi);
    }
    __shared__ float warp_vals[ARGMAX_THREADS / 32];
    __shared__ int warp_idxs[ARGMAX_THREADS / 32];
    __shared__ float cta_val;
    __shared__ int cta_idx;
    if (threadIdx.x % 32 == 0) {
        warp_vals[threadIdx.x / 32] = best_val;
        warp_idxs[threadIdx.x / 32] = best_idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 0; w < ARGMAX_THREADS / 32; w++) argmax_pair(best_val, best_idx, warp_vals[w], warp_idxs[w]);
        cta_val = best_val;
        cta_idx = best_idx;
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
        for (int r = 1; r < ARGMAX_CTAS; r++) {
            const float v = *cluster.map_shared_rank(&cta_val, r);
            const int i = *cluster.map_shared_rank(&cta_idx, r);
            argmax_pair(best_val, best_idx, v, i);
        }
        o.out[row] = best_idx;
        if (o.next_token) o.next_token[row] = best_idx;
        if (o.history && *o.step >= 0 && *o.step < o.history_cap)
            o.history[(size_t)(*o.step) * (gridDim.x / ARGMAX_CTAS) + row] = best_idx;
        if (o.pos) o.pos[row] += 1;
    }
    cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

// Advances the decode-loop step counter after the argmax of a step has used it.
__global__ void step_advance_kernel(int *step) {
    pdl_trigger();
    pdl_wait();
    *step += 1;
}

// ------------------------------------------------------------------ sample
// src/kernels.cu:546-602, same block size (1024), chunking and summation order.
__global__ void __launch_bounds__(1024) sample_kernel(int *out, const bf16 *x, int n, float inv_temp,
                                                      float u) {
    pdl_trigger();
    pdl_wait();
    __shared__ float chunk_sums[1024];
    __shared__ float partials[32];
    float local_max = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) local_max = fmaxf(local_max, __bfloat162float(x[i]));
    for (int off = 16; off > 0; off >>= 1) local_max = fmaxf(local_max, __shfl_xor_sync(0xffffffffu, local_max, off));
    if (threadIdx.x % 32 == 0) partials[threadIdx.x / 32] = local_max;
    __syncthreads();
    float max_val = -INFINITY;
    for (int w = 0; w < 32; w++) max_val = fmaxf(max_val, partials[w]);

    const int chunk = (n + blockDim.x - 1) / blockDim.x;
    const int start = threadIdx.x * chunk;
    const int end = min(start + chunk, n);
    float sum = 0.0f;
    for (int i = start; i < end; i++) sum += expf((__bfloat162float(x[i]) - max_val) * inv_temp);
    chunk_sums[threadIdx.x] = sum;
    __syncthreads();
    if (threadIdx.x != 0) return;
    float total = 0.0f;
    for (int t = 0; t < (int)blockDim.x; t++) total += chunk_sums[t];
    const float target = u * total;
    float cdf = 0.0f;
    int t = 0;
    while (t < (int)blockDim.x - 1 && cdf + chunk_sums[t] <= target) {
        cdf += chunk_sums[t];
        t++;
    }
    int chosen = -1;
    const int cs = t * chunk;
    const int ce = min(cs + chunk, n);
    float s = 0.0f;
    for (int i = cs; i < ce; i++) {
        s += expf((__bfloat162float(x[i]) - max_val) * inv_temp);
        if (cdf + s > target) {
            chosen = i;
            break;
        }
    }
    *out = chosen;
}

// ------------------------------------------------------------------ synthetic fill
// dst[i] = bf16(mean + std * z), z ~ N(0, 1) from a counter-based hash of (seed, i) and the
// Box-Muller transform; used to pre-fill KV caches and weights of synthetic benchmarks.
__device__ __forceinline__ uint32_t mix32(uint64_t x) {
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdull;
    x ^= x >> 33;
    x *= 0xc4ceb9fe1a85ec53ull;
    x ^= x >> 33;
    return (uint32_t)x;
}

// Block j (of n_blocks, block_len values each, starting block_stride elements apart) holds the
// stream of seed + j: element i is Box-Muller over two hashed 24-bit uniforms of counter
// (seed + j) * golden + i, so a block's values do not depend on the launch shape.
__global__ void fill_normal_kernel(bf16 *dst, long long n_blocks, long long block_len, long long block_stride,
                                   unsigned long long seed, float mean, float std) {
    const long long n = n_blocks * block_len;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long j = idx / block_len, i = idx - j * block_len;
        const uint64_t c = (seed + (uint64_t)j) * 0x9e3779b97f4a7c15ull + (uint64_t)i;
        const float u1 = ((mix32(2 * c) >> 8) + 1) * (1.0f / 16777217.0f);  // (0, 1]
        const float u2 = (mix32(2 * c + 1) >> 8) * (1.0f / 16777216.0f);
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        dst[j * block_stride + i] = __float2bfloat16(mean + std * z);
    }
}

}  // namespace

int fill_normal_blocks(bf16 *dst, long long n_blocks, long long block_len, long long block_stride,
                       unsigned long long seed, float mean, float std, cudaStream_t s) {
    if (!dst || n_blocks < 0 || block_len < 0 || (n_blocks > 1 && block_stride < block_len)) return Q3_ERR_ARG;
    const long long n = n_blocks * block_len;
    if (n == 0) return Q3_OK;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    fill_normal_kernel<<<blocks, 256, 0, s>>>(dst, n_blocks, block_len, block_stride, seed, mean, std);
    return record_cuda_error(cudaGetLastError());
}

int fill_normal(bf16 *dst, long long n, unsigned long long seed, float mean, float std, cudaStream_t s) {
    return fill_normal_blocks(dst, 1, n, n, seed, mean, std, s);
}

unsigned take_error_decode() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

int embedding(bf16 *out, const bf16 *table, const int *tokens, int n_rows, int hidden, int vocab,
              cudaStream_t s) {
    if (!out || !table || !tokens) return Q3_ERR_ARG;
    if (hidden < 0 || n_rows < 0) return Q3_ERR_SHAPE;
    if (hidden == 0 || n_rows == 0) return Q3_OK;
    const bool vec = hidden % 8 == 0 && aligned16(out) && aligned16(table);
    const int per_row = vec ? hidden / 8 : hidden;
    const int blocks = std::min((per_row + 255) / 256, 64);
    dim3 grid(blocks, n_rows);
    if (vec) Q3_TRY_LAUNCH(launch(embedding_kernel<true>, grid, dim3(256), 0, s, 1, out, table, tokens, hidden, vocab));
    else Q3_TRY_LAUNCH(launch(embedding_kernel<false>, grid, dim3(256), 0, s, 1, out, table, tokens, hidden, vocab));
    return Q3_OK;
}

int rmsnorm(bf16 *out, const bf16 *in, const bf16 *weight, int rows, int dim, float eps, cudaStream_t s) {
    if (!out || !in || !weight) return Q3_ERR_ARG;
    if (rows < 0 || dim <= 0) return Q3_ERR_SHAPE;
    if (rows == 0) return Q3_OK;
    if (rows > 65535 * 1024) return Q3_ERR_SHAPE;
    Q3_TRY_LAUNCH(launch(rmsnorm_kernel, dim3(rows), dim3(256), 0, s, 1, out, in, weight, dim, eps));
    return Q3_OK;
}

int qk_norm_rope(bf16 *q, bf16 *k, const bf16 *v, const bf16 *q_norm_w, const bf16 *k_norm_w,
                 bf16 *key_cache, bf16 *value_cache, const int *pos, int n_rows, long long q_stride,
                 long long kv_stride, KvLayout kv, int n_heads, int n_kv_heads, int head_dim,
                 int max_seq, float eps, float theta, bf16 *q_tap, bf16 *k_tap, cudaStream_t s) {
    if (!q || !k || !v || !q_norm_w || !k_norm_w || !key_cache || !value_cache || !pos) return Q3_ERR_ARG;
    if (head_dim % 32 != 0 || head_dim <= 0 || head_dim > 1024) return Q3_ERR_SHAPE;
    if (n_heads < 0 || n_kv_heads < 0 || n_rows < 0) return Q3_ERR_SHAPE;
    if (n_rows == 0 || n_heads + n_kv_heads == 0) return Q3_OK;
    RopeArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.q_norm_w = q_norm_w;
    a.k_norm_w = k_norm_w;
    a.key_cache = key_cache;
    a.value_cache = value_cache;
    a.pos = pos;
    a.q_tap = q_tap;
    a.k_tap = k_tap;
    a.q_stride = q_stride;
    a.kv_stride = kv_stride;
    a.kv = kv;
    a.n_heads = n_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.max_seq = max_seq;
    a.eps = eps;
    a.theta = theta;
    if (n_rows > 65535) return Q3_ERR_SHAPE;  // grid.y
    const dim3 grid((unsigned)((n_heads + n_kv_heads + ROPE_WARPS - 1) / ROPE_WARPS), (unsigned)n_rows),
        block(ROPE_WARPS * 32);
    switch (head_dim) {
        case 64: Q3_TRY_LAUNCH(launch(qk_norm_rope_kernel<2>, grid, block, 0, s, 1, a)); break;
        case 128: Q3_TRY_LAUNCH(launch(qk_norm_rope_kernel<4>, grid, block, 0, s, 1, a)); break;
        case 256: Q3_TRY_LAUNCH(launch(qk_norm_rope_kernel<8>, grid, block, 0, s, 1, a)); break;
        default: Q3_TRY_LAUNCH(launch(qk_norm_rope_kernel<0>, grid, block, 0, s, 1, a)); break;
    }
    return Q3_OK;
}

int argmax_rows(const bf16 *x, int n, int n_rows, long long row_stride, int *out, int *next_token,
                int *pos, int *history, int *step, int history_cap, cudaStream_t s) {
    if (!x || !out) return Q3_ERR_ARG;
    if (n < 0 || n_rows <= 0) return n_rows == 0 ? Q3_OK : Q3_ERR_SHAPE;
    if (history && !step) return Q3_ERR_ARG;
    ArgmaxOut o = {out, next_token, pos, history, step, history_cap};
    const bool vec = aligned16(x) && (row_stride % 8 == 0 || n_rows == 1);
    dim3 grid(ARGMAX_CTAS * n_rows);
    if (vec) Q3_TRY_LAUNCH(launch(argmax_kernel<true>, grid, dim3(ARGMAX_THREADS), 0, s, ARGMAX_CTAS, x, n, row_stride, o));
    else Q3_TRY_LAUNCH(launch(argmax_kernel<false>, grid, dim3(ARGMAX_THREADS), 0, s, ARGMAX_CTAS, x, n, row_stride, o));
    if (step) Q3_TRY_LAUNCH(launch(step_advance_kernel, dim3(1), dim3(1), 0, s, 1, step));
    return Q3_OK;
}

int sample(int *out, const bf16 *x, int n, float inv_temp, float u, cudaStream_t s) {
    if (!out || !x) return Q3_ERR_ARG;
    if (n < 0) return Q3_ERR_SHAPE;
    Q3_TRY_LAUNCH(launch(sample_kernel, dim3(1), dim3(1024), 0, s, 1, out, x, n, inv_temp, u));
    return Q3_OK;
}

}  // namespace q3
