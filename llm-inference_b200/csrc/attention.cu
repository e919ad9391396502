// GQA decode attention for sm_100a with the reference's rounding points (src/kernels.cu:439-497).
//
// The reference runs one 128-thread block per query head and does everything serially inside
// it. Here the work is split into two kernels over persistent grids:
//
//   scores  (work item = sequence b, kv head, 128 positions): the K rows of the item are staged
//           in shared memory with cp.async (padded rows, conflict-free), each thread owns one
//           position and computes the dot products of all query heads of the kv group with it,
//           serially over head_dim as the reference does, so each K row is read once per group.
//           s = round_bf16(round_bf16(dot) * scale) goes to the scores buffer [b][head][pos].
//           With split work (below), the last CTA of each (b, kv head) also computes the softmax
//           statistics of its heads.
//   pv      (work item = sequence b, kv head, a chunk of positions): probabilities
//           p = round_bf16(expf(s - max) / sum) as in the reference, then thread d accumulates
//           p[t] * v[t][d] over the chunk's positions in order with fused multiply-adds, the V
//           rows staged through a cp.async ring.
//
// The softmax statistics use the reference's exact order: 128 slots, slot j summing positions
// j, j+128, ... serially, then an xor tree per warp and a serial sum of the four warp totals.
//
// Exact mode (one chunk per (b, kv head), used by the drop-in attention_forward): the P.V sum is
// the reference's single serial chain, so the output is bit-identical; the statistics are
// computed by each pv CTA itself. Split mode (the decode engine): chunks of a few hundred
// positions give more parallelism; their fp32 partial sums are added in chunk order by the last
// CTA of each (b, kv head), which changes only fp32 rounding inside the sum.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int A_THREADS = 128;   // scores: one thread per position, 128 positions per item
constexpr int B_THREADS = 128;   // pv: threads over head_dim; 128 slots for the statistics
constexpr int VT = 64;           // pv: positions per staged V tile
constexpr int V_STAGES = 3;
constexpr int MAX_B = 1024;      // sequences per launch (prefix table in shared memory)

struct AttnArgs {
    const bf16 *q;        // sequence b: q + b*q_stride, heads concatenated
    const bf16 *kc, *vc;  // sequence b: kc + b*cache_stride, rows [max_seq][kv_dim]
    bf16 *out;            // like q
    float *scores;        // [B][n_heads][max_seq]
    float *stats;         // split mode: [B][n_heads][2] (max, sum of exp)
    float *partial;       // split mode: [B][n_heads][max_chunks][head_dim]
    int *count_a;         // split mode: [B][n_kv], zero between launches
    int *count_b;         // split mode: [B][n_kv], zero between launches
    const int *pos;       // [B]
    long long q_stride, cache_stride;
    int B, n_heads, n_kv, head_dim, kv_dim, max_seq;
    int chunk_b;          // positions per pv item (split mode); ignored in exact mode
    int max_chunks;       // split mode: capacity of `partial` along the chunk axis
    float scale;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Item table: items of sequence b occupy [prefix[b], prefix[b+1]); n_chunks(b) per kv head.
__device__ int build_prefix(const AttnArgs &a, int chunk, int *prefix) {
    if (threadIdx.x == 0) {
        int total = 0;
        for (int b = 0; b < a.B; b++) {
            prefix[b] = total;
            int p = a.pos[b];
            if (p < 0 || p >= a.max_seq) {
                atomicOr(&g_dev_error, DEV_ERR_POS_RANGE);
                p = -1;  // no work for this sequence
            }
            total += a.n_kv * ((p + chunk) / chunk);
        }
        prefix[a.B] = total;
    }
    __syncthreads();
    return prefix[a.B];
}

__device__ __forceinline__ void find_item(const AttnArgs &a, const int *prefix, int chunk, int item,
                                          int &b, int &kvh, int &c, int &nc, int &pos) {
    b = 0;
    while (prefix[b + 1] <= item) b++;
    pos = a.pos[b];
    nc = (pos + chunk) / chunk;
    const int r = item - prefix[b];
    kvh = r / nc;
    c = r - kvh * nc;
}

// Softmax statistics of the NREP heads of (b, kvh) over positions 0..pos, in the reference's
// order (block_max / block_sum of src/kernels.cu:406-436 over 128 threads). Needs 128 threads.
template <int NREP>
__device__ void softmax_stats(const AttnArgs &a, int b, int kvh, int pos, float *m_out, float *s_out,
                              float (*red)[NREP]) {
    const int tid = threadIdx.x;
    const int lane = tid % 32, warp = tid / 32;
    const float *sc = a.scores + ((size_t)b * a.n_heads + (size_t)kvh * NREP) * a.max_seq;
    float mx[NREP];
#pragma unroll
    for (int h = 0; h < NREP; h++) mx[h] = -INFINITY;
    for (int t = tid; t <= pos; t += 128)
#pragma unroll
        for (int h = 0; h < NREP; h++) mx[h] = fmaxf(mx[h], __ldcg(sc + (size_t)h * a.max_seq + t));
#pragma unroll
    for (int h = 0; h < NREP; h++)
        for (int off = 16; off > 0; off >>= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
    if (lane == 0)
#pragma unroll
        for (int h = 0; h < NREP; h++) red[warp][h] = mx[h];
    __syncthreads();
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        float r = -INFINITY;
        for (int w = 0; w < 4; w++) r = fmaxf(r, red[w][h]);
        mx[h] = r;
    }
    __syncthreads();
    float sm[NREP];
#pragma unroll
    for (int h = 0; h < NREP; h++) sm[h] = 0.0f;
    for (int t = tid; t <= pos; t += 128)
#pragma unroll
        for (int h = 0; h < NREP; h++) sm[h] += expf(__ldcg(sc + (size_t)h * a.max_seq + t) - mx[h]);
#pragma unroll
    for (int h = 0; h < NREP; h++)
        for (int off = 16; off > 0; off >>= 1) sm[h] += __shfl_xor_sync(0xffffffffu, sm[h], off);
    if (lane == 0)
#pragma unroll
        for (int h = 0; h < NREP; h++) red[warp][h] = sm[h];
    __syncthreads();
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        float total = 0.0f;
        for (int w = 0; w < 4; w++) total += red[w][h];
        m_out[h] = mx[h];
        s_out[h] = total;
    }
    __syncthreads();
}

// ------------------------------------------------------------------ scores
template <int NREP>
__global__ void __launch_bounds__(A_THREADS) attn_scores_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int hd = a.head_dim;
    const int row_elems = hd + 8;  // padded K row: consecutive rows shift by 16 bytes
    bf16 *ktile[2] = {reinterpret_cast<bf16 *>(smem), reinterpret_cast<bf16 *>(smem) + A_THREADS * row_elems};
    float *q_s = reinterpret_cast<float *>(smem + 2 * A_THREADS * row_elems * 2);  // [NREP][hd]
    int *prefix = reinterpret_cast<int *>(q_s + NREP * hd);
    __shared__ float red[4][NREP];
    __shared__ int is_last;

    pdl_trigger();
    pdl_wait();
    const int total = build_prefix(a, A_THREADS, prefix);
    const int tid = threadIdx.x;
    const int cpr = hd / 8;  // 16-byte chunks per K row

    auto issue = [&](int item, int buf) {
        int b, kvh, c, nc, pos;
        find_item(a, prefix, A_THREADS, item, b, kvh, c, nc, pos);
        const int t0 = c * A_THREADS;
        const int rows = min(A_THREADS, pos + 1 - t0);
        const bf16 *src = a.kc + (size_t)b * a.cache_stride + (size_t)t0 * a.kv_dim + (size_t)kvh * hd;
        for (int j = tid; j < rows * cpr; j += A_THREADS) {
            const int r = j / cpr, ch = j - r * cpr;
            cp_async16(ktile[buf] + r * row_elems + ch * 8, src + (size_t)r * a.kv_dim + ch * 8);
        }
        cp_async_commit();
    };

    int item = blockIdx.x;
    if (item < total) issue(item, 0);
    int buf = 0;
    for (; item < total; item += gridDim.x, buf ^= 1) {
        int b, kvh, c, nc, pos;
        find_item(a, prefix, A_THREADS, item, b, kvh, c, nc, pos);
        const int next = item + gridDim.x;
        if (next < total) {
            issue(next, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        // q of the group's heads as fp32
        const bf16 *qg = a.q + (size_t)b * a.q_stride + (size_t)kvh * NREP * hd;
        for (int j = tid; j < NREP * hd; j += A_THREADS) q_s[j] = __bfloat162float(qg[j]);
        __syncthreads();

        const int t = c * A_THREADS + tid;
        if (t <= pos) {
            float acc[NREP];
#pragma unroll
            for (int h = 0; h < NREP; h++) acc[h] = 0.0f;
            const bf16 *krow = ktile[buf] + tid * row_elems;
            for (int ch = 0; ch < cpr; ch++) {
                const bf16x8 kv = lds128(krow + ch * 8);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f = __bfloat1622float2(kv.h[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int h = 0; h < NREP; h++) {
                    const float4 q0 = *reinterpret_cast<const float4 *>(q_s + h * hd + ch * 8);
                    const float4 q1 = *reinterpret_cast<const float4 *>(q_s + h * hd + ch * 8 + 4);
                    acc[h] = __fmaf_rn(q0.x, kf[0], acc[h]);
                    acc[h] = __fmaf_rn(q0.y, kf[1], acc[h]);
                    acc[h] = __fmaf_rn(q0.z, kf[2], acc[h]);
                    acc[h] = __fmaf_rn(q0.w, kf[3], acc[h]);
                    acc[h] = __fmaf_rn(q1.x, kf[4], acc[h]);
                    acc[h] = __fmaf_rn(q1.y, kf[5], acc[h]);
                    acc[h] = __fmaf_rn(q1.z, kf[6], acc[h]);
                    acc[h] = __fmaf_rn(q1.w, kf[7], acc[h]);
                }
            }
            float *sc = a.scores + ((size_t)b * a.n_heads + (size_t)kvh * NREP) * a.max_seq + t;
#pragma unroll
            for (int h = 0; h < NREP; h++) sc[(size_t)h * a.max_seq] = round_bf16(round_bf16(acc[h]) * a.scale);
        }

        if (a.count_a != nullptr) {
            // split mode: the last CTA of (b, kvh) computes the softmax statistics
            __threadfence();
            __syncthreads();
            if (tid == 0) {
                const int done = atomicAdd(a.count_a + b * a.n_kv + kvh, 1);
                is_last = done == nc - 1;
            }
            __syncthreads();
            if (is_last) {
                __threadfence();
                float m[NREP], s[NREP];
                softmax_stats<NREP>(a, b, kvh, pos, m, s, red);
                if (tid < NREP) {
                    float *st = a.stats + ((size_t)b * a.n_heads + kvh * NREP + tid) * 2;
                    st[0] = m[tid];
                    st[1] = s[tid];
                }
                if (tid == 0) a.count_a[b * a.n_kv + kvh] = 0;
            }
        }
        __syncthreads();  // ktile[buf] and q_s are reused by the next item
    }
}

// ------------------------------------------------------------------ pv
template <int NREP, int DPT>
__global__ void __launch_bounds__(B_THREADS) attn_pv_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int hd = a.head_dim;
    bf16 *vtile = reinterpret_cast<bf16 *>(smem);                       // [V_STAGES][VT][hd]
    float *p_s = reinterpret_cast<float *>(vtile + V_STAGES * VT * hd);  // [V_STAGES][NREP][VT]
    int *prefix = reinterpret_cast<int *>(p_s + V_STAGES * NREP * VT);
    __shared__ float red[4][NREP];
    __shared__ float m_s[NREP], s_s[NREP];
    __shared__ int is_last;

    pdl_trigger();
    pdl_wait();
    const bool split = a.count_b != nullptr;
    const int chunk = split ? a.chunk_b : a.max_seq;
    const int total = build_prefix(a, chunk, prefix);
    const int tid = threadIdx.x;
    const int cpr = hd / 8;

    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        int b, kvh, c, nc, pos;
        find_item(a, prefix, chunk, item, b, kvh, c, nc, pos);
        const int t0 = c * chunk;
        const int t1 = min(t0 + chunk, pos + 1);
        const int n_tiles = (t1 - t0 + VT - 1) / VT;
        const float *sc = a.scores + ((size_t)b * a.n_heads + (size_t)kvh * NREP) * a.max_seq;
        const bf16 *vsrc = a.vc + (size_t)b * a.cache_stride + (size_t)kvh * hd;

        auto issue = [&](int tile) {
            const int st = tile % V_STAGES;
            const int tt0 = t0 + tile * VT;
            const int rows = min(VT, t1 - tt0);
            bf16 *dst = vtile + st * VT * hd;
            for (int j = tid; j < rows * cpr; j += B_THREADS) {
                const int r = j / cpr, ch = j - r * cpr;
                cp_async16(dst + r * hd + ch * 8, vsrc + (size_t)(tt0 + r) * a.kv_dim + ch * 8);
            }
            cp_async_commit();
        };
        // V loads do not depend on the statistics: start the ring first
        for (int tile = 0; tile < V_STAGES - 1; tile++) {
            if (tile < n_tiles) issue(tile);
            else cp_async_commit();
        }

        if (split) {
            if (tid < NREP) {
                const float *st = a.stats + ((size_t)b * a.n_heads + kvh * NREP + tid) * 2;
                m_s[tid] = __ldcg(st);
                s_s[tid] = __ldcg(st + 1);
            }
            __syncthreads();
        } else {
            float m[NREP], s[NREP];
            softmax_stats<NREP>(a, b, kvh, pos, m, s, red);
            if (tid < NREP) {
                m_s[tid] = m[tid];
                s_s[tid] = s[tid];
            }
            __syncthreads();
        }

        float acc[NREP][DPT];
#pragma unroll
        for (int h = 0; h < NREP; h++)
#pragma unroll
            for (int k = 0; k < DPT; k++) acc[h][k] = 0.0f;

        for (int tile = 0; tile < n_tiles; tile++) {
            const int st = tile % V_STAGES;
            const int tt0 = t0 + tile * VT;
            const int rows = min(VT, t1 - tt0);
            // probabilities of this tile
            float *pt = p_s + st * NREP * VT;
            for (int j = tid; j < NREP * VT; j += B_THREADS) {
                const int h = j / VT, r = j - h * VT;
                if (r < rows) {
                    const float sv = __ldcg(sc + (size_t)h * a.max_seq + tt0 + r);
                    pt[h * VT + r] = round_bf16(expf(sv - m_s[h]) / s_s[h]);
                }
            }
            if (tile + V_STAGES - 1 < n_tiles) issue(tile + V_STAGES - 1);
            else cp_async_commit();
            cp_async_wait<V_STAGES - 1>();
            __syncthreads();
            const bf16 *vt = vtile + st * VT * hd;
#pragma unroll
            for (int k = 0; k < DPT; k++) {
                const int d = tid + k * B_THREADS;
                if (d < hd) {
                    for (int r = 0; r < rows; r++) {
                        const float v = __bfloat162float(vt[r * hd + d]);
#pragma unroll
                        for (int h = 0; h < NREP; h++) acc[h][k] = __fmaf_rn(pt[h * VT + r], v, acc[h][k]);
                    }
                }
            }
            __syncthreads();  // the stage is refilled V_STAGES - 1 tiles later
        }
        cp_async_wait<0>();

        const size_t out_base = (size_t)b * a.q_stride + (size_t)kvh * NREP * hd;
        if (!split || nc == 1) {
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DPT; k++) {
                    const int d = tid + k * B_THREADS;
                    if (d < hd) a.out[out_base + (size_t)h * hd + d] = __float2bfloat16(acc[h][k]);
                }
            if (split && tid == 0) a.count_b[b * a.n_kv + kvh] = 0;  // single chunk: nothing to combine
        } else {
            float *part = a.partial + ((size_t)b * a.n_heads + kvh * NREP) * a.max_chunks * hd;
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DPT; k++) {
                    const int d = tid + k * B_THREADS;
                    if (d < hd) part[((size_t)h * a.max_chunks + c) * hd + d] = acc[h][k];
                }
            __threadfence();
            __syncthreads();
            if (tid == 0) is_last = atomicAdd(a.count_b + b * a.n_kv + kvh, 1) == nc - 1;
            __syncthreads();
            if (is_last) {
                __threadfence();
#pragma unroll
                for (int h = 0; h < NREP; h++)
#pragma unroll
                    for (int k = 0; k < DPT; k++) {
                        const int d = tid + k * B_THREADS;
                        if (d < hd) {
                            float o = 0.0f;
                            for (int cc = 0; cc < nc; cc++) o += __ldcg(part + ((size_t)h * a.max_chunks + cc) * hd + d);
                            a.out[out_base + (size_t)h * hd + d] = __float2bfloat16(o);
                        }
                    }
                if (tid == 0) a.count_b[b * a.n_kv + kvh] = 0;
            }
        }
        __syncthreads();
    }
}

template <int NREP>
int launch_nrep(const AttnArgs &a, int dpt, cudaStream_t s) {
    const int nsm = num_sms();
    const size_t a_smem = (size_t)2 * A_THREADS * (a.head_dim + 8) * 2 + (size_t)NREP * a.head_dim * 4 +
                          (size_t)(a.B + 1) * 4;
    const size_t b_smem = (size_t)V_STAGES * VT * a.head_dim * 2 + (size_t)V_STAGES * NREP * VT * 4 +
                          (size_t)(a.B + 1) * 4;
    Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_scores_kernel<NREP>), a_smem));
    // grids: enough CTAs to cover the largest number of items, at most a few per SM
    const long long max_items_a = (long long)a.B * a.n_kv * ((a.max_seq + A_THREADS - 1) / A_THREADS);
    const int grid_a = (int)std::min<long long>(max_items_a, 4LL * nsm);
    Q3_TRY_LAUNCH(launch(attn_scores_kernel<NREP>, dim3(grid_a), dim3(A_THREADS), a_smem, s, 1, a));
    const bool split = a.count_b != nullptr;
    const long long chunk = split ? a.chunk_b : a.max_seq;
    const long long max_items_b = (long long)a.B * a.n_kv * ((a.max_seq + chunk - 1) / chunk);
    const int grid_b = (int)std::min<long long>(max_items_b, 4LL * nsm);
    if (dpt == 1) {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_kernel<NREP, 1>), b_smem));
        Q3_TRY_LAUNCH(launch(attn_pv_kernel<NREP, 1>, dim3(grid_b), dim3(B_THREADS), b_smem, s, 1, a));
    } else {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_kernel<NREP, 2>), b_smem));
        Q3_TRY_LAUNCH(launch(attn_pv_kernel<NREP, 2>, dim3(grid_b), dim3(B_THREADS), b_smem, s, 1, a));
    }
    return Q3_OK;
}

}  // namespace

unsigned take_error_attention() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

// Shapes the attention kernels accept.
int attention_check(int n_heads, int n_kv_heads, int head_dim, int max_seq, int n_rows) {
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0) return Q3_ERR_SHAPE;
    const int nrep = n_heads / n_kv_heads;
    if (nrep != 1 && nrep != 2 && nrep != 4 && nrep != 8) return Q3_ERR_SHAPE;
    if (head_dim % 32 != 0 || head_dim <= 0 || head_dim > 256) return Q3_ERR_SHAPE;
    if (max_seq <= 0 || n_rows <= 0 || n_rows > MAX_B) return Q3_ERR_SHAPE;
    return Q3_OK;
}

// Attention over n_rows sequences. Exact mode when split == nullptr; otherwise `split` holds the
// split-mode scratch (stats, partial, count_a, count_b, chunk_b, max_chunks).

int attention(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *scores,
              const int *pos, int n_rows, long long q_stride, long long cache_stride, int n_heads,
              int n_kv_heads, int head_dim, int max_seq, float scale, const AttnSplit *split,
              cudaStream_t s) {
    if (!out || !q || !key_cache || !value_cache || !scores || !pos) return Q3_ERR_ARG;
    int st = attention_check(n_heads, n_kv_heads, head_dim, max_seq, n_rows);
    if (st != Q3_OK) return st;
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(key_cache) || !al(value_cache) || (cache_stride * 2) % 16 != 0) return Q3_ERR_ALIGN;
    AttnArgs a = {};
    a.q = q;
    a.kc = key_cache;
    a.vc = value_cache;
    a.out = out;
    a.scores = scores;
    a.pos = pos;
    a.q_stride = q_stride;
    a.cache_stride = cache_stride;
    a.B = n_rows;
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.head_dim = head_dim;
    a.kv_dim = n_kv_heads * head_dim;
    a.max_seq = max_seq;
    a.scale = scale;
    if (split) {
        if (!split->stats || !split->partial || !split->count_a || !split->count_b) return Q3_ERR_ARG;
        if (split->chunk_b <= 0 || (long long)split->chunk_b * split->max_chunks < max_seq) return Q3_ERR_SHAPE;
        a.stats = split->stats;
        a.partial = split->partial;
        a.count_a = split->count_a;
        a.count_b = split->count_b;
        a.chunk_b = split->chunk_b;
        a.max_chunks = split->max_chunks;
    }
    const int dpt = head_dim <= 128 ? 1 : 2;
    switch (n_heads / n_kv_heads) {
        case 1: return launch_nrep<1>(a, dpt, s);
        case 2: return launch_nrep<2>(a, dpt, s);
        case 4: return launch_nrep<4>(a, dpt, s);
        default: return launch_nrep<8>(a, dpt, s);
    }
}

}  // namespace q3
