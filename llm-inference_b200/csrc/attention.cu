// GQA decode attention for sm_100a with the reference's rounding points (src/kernels.cu:439-497).
//
// The reference runs one 128-thread block per query head and does everything serially inside
// it. Here the work is split over persistent grids, each CTA taking a contiguous, balanced range
// of work items, with every global read staged through shared memory by cp.async so that no
// loop waits on a global round trip per iteration:
//
//   scores  item = (sequence b, kv head, 256 positions). The item's K rows are staged in shared
//           memory (padded rows, conflict-free) through a 2-deep ring; each thread owns one
//           position and computes the dot products of all query heads of the kv group with it,
//           serially over head_dim as the reference does, so each K row is read once per group.
//           s = round_bf16(round_bf16(dot) * scale) goes to the scores buffer [b][head][pos].
//   stats   one CTA per (b, kv head): the softmax max and sum of each head in the reference's
//           exact order -- 128 slots, slot j summing positions j, j+128, ... serially, an xor
//           tree per warp, a serial sum of the four warp totals (block_max / block_sum,
//           src/kernels.cu:406-436) -- over scores staged in shared memory.
//   pv      item = (b, kv head, a chunk of positions). Probabilities
//           p = round_bf16(expf(s - max) / sum) as in the reference (:472-474) from staged score
//           tiles, then thread d accumulates p[t] * v[t][d] over the chunk in position order with
//           fused multiply-adds (:478-485), V rows staged through a cp.async ring.
//   combine sums the chunks' fp32 partial outputs in chunk order and rounds to bf16.
//
// Exact mode (the drop-in attention_forward): one pv chunk spans all positions, so P.V is the
// reference's single serial chain, and the pv CTA computes its statistics itself; the output is
// bit-identical. Split mode (the batched engine): chunks of 512 positions for parallelism; their
// partial sums are added in chunk order, which changes only fp32 rounding inside the sum.
//
// Split mode streams the K tiles by TMA into a deep shared-memory ring (attn_scores_exact_kernel)
// and keeps the reference's serial dot products, so its scores -- and so its probabilities --
// are the reference's bit for bit; P.V runs on the tensor cores (attn_pv_tc_kernel), where the
// products p * v are exact and only the fp32 order of the sums differs.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "tc_common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int THREADS = 128;     // stats / pv: 128 slots, threads over head_dim
constexpr int SC_THREADS = 256;  // scores: one thread per position
constexpr int SC_CHUNK = 256;    // positions per scores item (128 for head_dim > 128)
constexpr int K_STAGES = 2;
constexpr int VT = 64;           // positions per staged V tile
constexpr int V_STAGES = 3;
constexpr int MAX_B = 1024;      // sequences per launch (prefix table in shared memory)

struct AttnArgs {
    const bf16 *q;        // sequence b: q + b*q_stride, heads concatenated
    const bf16 *kc, *vc;  // row (b, t, kv head h) at kc + b*kv.seq + t*kv.pos + h*kv.head
    bf16 *out;            // like q
    float *scores;        // [B][n_heads][ld]
    float *stats;         // split mode: [B][n_heads][2] (max, sum of exp)
    float *partial;       // split mode: [B][n_heads][max_chunks][head_dim]
    const int *pos;       // [B]
    long long q_stride;
    KvLayout kv;
    int ld;               // row stride of scores (>= max_seq)
    int B, n_heads, n_kv, head_dim, kv_dim, max_seq;
    int chunk_b;          // positions per pv item
    int sc_chunk;         // positions per scores item
    int max_chunks;       // split mode: capacity of `partial` along the chunk axis
    float scale;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Positions of sequence b, or 0 (no work) for an out-of-range position, which is flagged.
__device__ __forceinline__ int seq_len(const AttnArgs &a, int b) {
    const int p = a.pos[b];
    if (p < 0 || p >= a.max_seq) return 0;
    return p + 1;
}

// Item table in shared memory (PREFIX_INTS(B) ints): items of sequence b occupy
// [prefix[b], prefix[b+1]), and prefix[B + 1 + b] holds its length, so that walking the items
// reads no global memory. The positions are loaded by all threads at once.
#define PREFIX_INTS(B) (2 * (B) + 1)
__device__ int build_prefix(const AttnArgs &a, int chunk, int *prefix) {
    int *lens = prefix + a.B + 1;
    for (int b = threadIdx.x; b < a.B; b += blockDim.x) {
        const int n = seq_len(a, b);
        lens[b] = n;
        if (n == 0 && blockIdx.x == 0) atomicOr(&g_dev_error, DEV_ERR_POS_RANGE);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int total = 0;
        for (int b = 0; b < a.B; b++) {
            prefix[b] = total;
            total += a.n_kv * ((lens[b] + chunk - 1) / chunk);
        }
        prefix[a.B] = total;
    }
    __syncthreads();
    return prefix[a.B];
}

struct Item {
    int b, kvh, c, nc, len;
};

// build_prefix over groups of G consecutive rows (the rows of one prompt, sharing a cache): a
// group's length is its longest row's. G == 1 is build_prefix.
__device__ int build_prefix_rows(const AttnArgs &a, int chunk, int *prefix, int G) {
    const int Bg = (a.B + G - 1) / G;
    int *lens = prefix + Bg + 1;
    for (int g = threadIdx.x; g < Bg; g += blockDim.x) {
        int n = 0;
        for (int i = 0; i < G && g * G + i < a.B; i++) {
            const int l = seq_len(a, g * G + i);
            if (l == 0 && blockIdx.x == 0) atomicOr(&g_dev_error, DEV_ERR_POS_RANGE);
            n = max(n, l);
        }
        lens[g] = n;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int total = 0;
        for (int g = 0; g < Bg; g++) {
            prefix[g] = total;
            total += a.n_kv * ((lens[g] + chunk - 1) / chunk);
        }
        prefix[Bg] = total;
    }
    __syncthreads();
    return prefix[Bg];
}

__device__ __forceinline__ Item find_item(const AttnArgs &a, const int *prefix, int chunk, int item) {
    Item it;
    int b = 0;
    while (prefix[b + 1] <= item) b++;
    it.b = b;
    it.len = prefix[a.B + 1 + b];
    it.nc = (it.len + chunk - 1) / chunk;
    const int r = item - prefix[b];
    it.kvh = r / it.nc;
    it.c = r - it.kvh * it.nc;
    return it;
}

// Sequence whose items contain `item` (prefix[B] > item): the largest b with prefix[b] <= item,
// which skips sequences without items.
__device__ __forceinline__ int first_seq(const int *prefix, int B, int item) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (prefix[mid] <= item) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// find_item for increasing items: `b` is the caller's cursor (start it at first_seq).
__device__ __forceinline__ Item item_at(const AttnArgs &a, const int *prefix, int chunk, int item, int &b) {
    while (prefix[b + 1] <= item) b++;
    Item it;
    it.b = b;
    it.len = prefix[a.B + 1 + b];
    it.nc = (it.len + chunk - 1) / chunk;
    const int r = item - prefix[b];
    it.kvh = r / it.nc;
    it.c = r - it.kvh * it.nc;
    return it;
}

// The CTA's items [i0, i0 + n) as a table in shared memory, filled by all threads at once:
// (b | kvh << 16, c | nc << 16) per item. The split kernels' producer is one thread issuing a copy
// every few hundred cycles next to warps that keep its scheduler busy; computing each item there
// (a search over the sequences, a division) made it fall behind, the table makes an item one
// shared-memory load. `cap` is the table's size; a CTA with more items, or items whose fields do
// not fit 16 bits, computes them with item_at instead (fill_items returns false).
__device__ bool fill_items(const AttnArgs &a, const int *prefix, int chunk, int i0, int n, int2 *tab, int cap) {
    const bool fits = n <= cap && (a.max_seq + chunk - 1) / chunk < 65536 && a.B <= 65536 && a.n_kv <= 65536;
    if (fits)
        for (int k = threadIdx.x; k < n; k += blockDim.x) {
            int b = first_seq(prefix, a.B, i0 + k);
            const Item it = item_at(a, prefix, chunk, i0 + k, b);
            tab[k] = make_int2(it.b | (it.kvh << 16), it.c | (it.nc << 16));
        }
    __syncthreads();
    return fits;
}

// Item i0 + k: from the table when it holds the CTA's items, else computed (`cur` is the caller's
// sequence cursor for item_at, and k must increase from call to call).
__device__ __forceinline__ Item item_k(const AttnArgs &a, const int *prefix, int chunk, const int2 *tab, bool tabbed,
                                       int i0, int k, int &cur) {
    if (!tabbed) return item_at(a, prefix, chunk, i0 + k, cur);
    const int2 v = tab[k];
    Item it;
    it.b = (int)((unsigned)v.x & 0xffffu);
    it.kvh = (int)((unsigned)v.x >> 16);
    it.c = (int)((unsigned)v.y & 0xffffu);
    it.nc = (int)((unsigned)v.y >> 16);
    it.len = prefix[a.B + 1 + it.b];
    return it;
}

// Offset (in ints) of the item table after a PREFIX_INTS(B) prefix table: 8-byte aligned.
#define ITEM_TAB_OFF(B) ((PREFIX_INTS(B) + 1) / 2 * 2)
constexpr int ITEM_TAB_MAX = 1024;
constexpr size_t SMEM_CTA_MAX = 232448;  // dynamic shared memory a CTA may opt in to on sm_100

// Copies n scores (floats) from global to shared memory as cp.async groups' members.
__device__ __forceinline__ void stage_scores(float *dst, const float *src, int n) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        const int n4 = n / 4;
        for (int i = threadIdx.x; i < n4; i += THREADS) cp_async16(dst + 4 * i, src + 4 * i);
        for (int i = 4 * n4 + threadIdx.x; i < n; i += THREADS) cp_async4(dst + i, src + i);
    } else {
        for (int i = threadIdx.x; i < n; i += THREADS) cp_async4(dst + i, src + i);
    }
}

// Softmax statistics of the NREP heads of (b, kvh) over positions [0, len) in the reference's
// order, scores staged through `buf` (cap floats) slice by slice. Needs 128 threads.
template <int NREP>
__device__ void softmax_stats(const AttnArgs &a, int b, int kvh, int len, float *buf, int cap, float *m_out,
                              float *s_out) {
    __shared__ float red[4][NREP];
    const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const float *sc = a.scores + ((size_t)b * a.n_heads + (size_t)kvh * NREP) * a.ld;
    const int slice = max(THREADS, (cap / NREP) / THREADS * THREADS);  // a multiple of 128 positions
    const bool resident = len <= slice;  // one slice holds every score: stage it once
    float mx[NREP], sm[NREP];
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        mx[h] = -INFINITY;
        sm[h] = 0.0f;
    }
    for (int pass = 0; pass < 2; pass++) {
        for (int t0 = 0; t0 < len; t0 += slice) {
            const int n = min(slice, len - t0);
            if (pass == 0 || !resident) {
                __syncthreads();  // the previous slice has been read
#pragma unroll
                for (int h = 0; h < NREP; h++) stage_scores(buf + h * slice, sc + (size_t)h * a.ld + t0, n);
                cp_async_commit();
                cp_async_wait<0>();
                __syncthreads();
            }
            for (int t = tid; t < n; t += THREADS)
#pragma unroll
                for (int h = 0; h < NREP; h++) {
                    const float v = buf[h * slice + t];
                    if (pass == 0) mx[h] = fmaxf(mx[h], v);
                    else sm[h] += expf(v - mx[h]);
                }
        }
        // block_max / block_sum: xor tree per warp, then the warp totals in warp order
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            float v = pass == 0 ? mx[h] : sm[h];
            for (int off = 16; off > 0; off >>= 1) {
                const float o = __shfl_xor_sync(0xffffffffu, v, off);
                v = pass == 0 ? fmaxf(v, o) : v + o;
            }
            if (lane == 0) red[warp][h] = v;
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            float r = pass == 0 ? -INFINITY : 0.0f;
            for (int w = 0; w < 4; w++) r = pass == 0 ? fmaxf(r, red[w][h]) : r + red[w][h];
            if (pass == 0) mx[h] = r;
            else sm[h] = r;
        }
        __syncthreads();
    }
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        m_out[h] = mx[h];
        s_out[h] = sm[h];
    }
}

// ------------------------------------------------------------------ scores
template <int NREP>
__global__ void __launch_bounds__(SC_THREADS) attn_scores_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int hd = a.head_dim;
    const int row_elems = hd + 8;  // padded K row: consecutive rows shift by 16 bytes
    const int tile_elems = a.sc_chunk * row_elems;
    bf16 *ktiles = reinterpret_cast<bf16 *>(smem);
    float *q_s = reinterpret_cast<float *>(smem + (size_t)K_STAGES * tile_elems * 2);  // [NREP][hd]
    int *prefix = reinterpret_cast<int *>(q_s + NREP * hd);

    pdl_trigger();
    pdl_wait();
    const int total = build_prefix(a, a.sc_chunk, prefix);
    const int tid = threadIdx.x;
    const int cpr = hd / 8;  // 16-byte chunks per K row
    const int i0 = (int)((long long)total * blockIdx.x / gridDim.x);
    const int i1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);

    auto issue = [&](int item, int stage) {
        const Item it = find_item(a, prefix, a.sc_chunk, item);
        const int t0 = it.c * a.sc_chunk;
        const int rows = min(a.sc_chunk, it.len - t0);
        const bf16 *src = a.kc + (size_t)it.b * a.kv.seq + (size_t)t0 * a.kv.pos + (size_t)it.kvh * a.kv.head;
        bf16 *dst = ktiles + (size_t)stage * tile_elems;
        for (int j = tid; j < rows * cpr; j += SC_THREADS) {
            const int r = j / cpr, ch = j - r * cpr;
            cp_async16(dst + r * row_elems + ch * 8, src + (size_t)r * a.kv.pos + ch * 8);
        }
    };

    // prologue: K_STAGES - 1 items in flight
    for (int s = 0; s < K_STAGES - 1; s++) {
        if (i0 + s < i1) issue(i0 + s, s);
        cp_async_commit();
    }
    int cur_b = -1, cur_kvh = -1;
    for (int item = i0; item < i1; item++) {
        const int k = item - i0;
        if (item + K_STAGES - 1 < i1) issue(item + K_STAGES - 1, (k + K_STAGES - 1) % K_STAGES);
        cp_async_commit();
        const Item it = find_item(a, prefix, a.sc_chunk, item);
        if (it.b != cur_b || it.kvh != cur_kvh) {  // q of the group's heads, as fp32
            __syncthreads();
            const bf16 *qg = a.q + (size_t)it.b * a.q_stride + (size_t)it.kvh * NREP * hd;
            for (int j = tid; j < NREP * hd; j += SC_THREADS) q_s[j] = __bfloat162float(qg[j]);
            cur_b = it.b;
            cur_kvh = it.kvh;
        }
        cp_async_wait<K_STAGES - 1>();
        __syncthreads();

        const int t = it.c * a.sc_chunk + tid;
        if (tid < a.sc_chunk && t < it.len) {
            float acc[NREP];
#pragma unroll
            for (int h = 0; h < NREP; h++) acc[h] = 0.0f;
            const bf16 *krow = ktiles + (size_t)(k % K_STAGES) * tile_elems + tid * row_elems;
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
            float *sc = a.scores + ((size_t)it.b * a.n_heads + (size_t)it.kvh * NREP) * a.ld + t;
#pragma unroll
            for (int h = 0; h < NREP; h++) sc[(size_t)h * a.ld] = round_bf16(round_bf16(acc[h]) * a.scale);
        }
        __syncthreads();  // this stage is refilled K_STAGES - 1 items later
    }
    cp_async_wait<0>();
}

// ------------------------------------------------------------------ stats (split mode)
// Softmax statistics of every query head of (sequence, kv head) in the reference's order
// (src/kernels.cu:406-436): for each head, 128 slots, slot s taking positions s, s + 128, ... in
// order, then an xor tree per warp and the four warp totals in warp order; first the max, then
// the sum of expf(score - max).
//
// One thread per (head, slot): 128 * NREP threads, so that the exp / add chain of each slot is
// spread over NREP times more warps than one 128-thread block would give it. A thread keeps its
// first STATS_REG scores in registers between the two passes; longer rows re-read the rest (from
// L2: the scores kernel wrote them just before).
constexpr int STATS_REG = 32;

template <int NREP>
__global__ void __launch_bounds__(128 * NREP) attn_stats_kernel(const __grid_constant__ AttnArgs a) {
    __shared__ float red[NREP][4];
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x / a.n_kv, kvh = blockIdx.x % a.n_kv;
    const int len = seq_len(a, b);
    if (len == 0) return;
    const int h = threadIdx.x / 128, slot = threadIdx.x % 128, lane = slot % 32, w = slot / 32;
    const float *sc = a.scores + ((size_t)b * a.n_heads + (size_t)kvh * NREP + h) * a.ld;
    float v[STATS_REG];
#pragma unroll
    for (int k = 0; k < STATS_REG; k++) {
        const int t = slot + 128 * k;
        v[k] = t < len ? __ldcg(sc + t) : -INFINITY;  // -inf leaves the max unchanged
    }
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < STATS_REG; k++) mx = fmaxf(mx, v[k]);
    for (int t = slot + 128 * STATS_REG; t < len; t += 128) mx = fmaxf(mx, __ldcg(sc + t));
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[h][w] = mx;
    __syncthreads();
    mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; i++) mx = fmaxf(mx, red[h][i]);
    __syncthreads();  // red is reused for the sums
    float sm = 0.0f;
#pragma unroll
    for (int k = 0; k < STATS_REG; k++)
        if (slot + 128 * k < len) sm += expf(v[k] - mx);
    for (int t = slot + 128 * STATS_REG; t < len; t += 128) sm += expf(__ldcg(sc + t) - mx);
    for (int off = 16; off > 0; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
    if (lane == 0) red[h][w] = sm;
    __syncthreads();
    if (slot == 0) {
        float r = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) r += red[h][i];
        float *st = a.stats + ((size_t)b * a.n_heads + kvh * NREP + h) * 2;
        st[0] = mx;
        st[1] = r;
    }
}

// Few (sequence, kv head) groups (batch 1 and 2 at 8 kv heads): the same statistics with one
// 128-thread CTA per (sequence, query head), so that B * n_heads SMs share the reads. The CTA
// first copies the head's scores into shared memory (every 16-byte piece in flight at once: one
// round trip to L2), then thread s runs slot s's chain from there, its loads and expf calls
// independent of the chain's additions and so issued ahead of them. Same values in the same
// order as attn_stats_kernel: the max is order-free, and each slot still adds its positions s,
// s + 128, ... serially before the xor tree and the four warp totals in order.
__global__ void __launch_bounds__(128) attn_stats_row_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) float row[];  // this head's len scores
    __shared__ float red[4];
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x / a.n_heads, hq = blockIdx.x % a.n_heads;
    const int len = seq_len(a, b);
    if (len == 0) return;
    const int slot = threadIdx.x, lane = slot % 32, w = slot / 32;
    const float *sc = a.scores + ((size_t)b * a.n_heads + hq) * a.ld;
    if ((reinterpret_cast<uintptr_t>(sc) & 15) == 0) {
        const int n4 = len / 4;
        for (int i = slot; i < n4; i += 128) cp_async16(row + 4 * i, sc + 4 * i);
        for (int i = 4 * n4 + slot; i < len; i += 128) cp_async4(row + i, sc + i);
    } else {
        for (int i = slot; i < len; i += 128) cp_async4(row + i, sc + i);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float mx = -INFINITY;
#pragma unroll 8
    for (int t = slot; t < len; t += 128) mx = fmaxf(mx, row[t]);
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[w] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();  // red is reused for the sums
    float sm = 0.0f;
#pragma unroll 8
    for (int t = slot; t < len; t += 128) sm += expf(row[t] - mx);
    for (int off = 16; off > 0; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
    if (lane == 0) red[w] = sm;
    __syncthreads();
    if (slot == 0) {
        float r = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) r += red[i];
        float *st = a.stats + ((size_t)b * a.n_heads + hq) * 2;
        st[0] = mx;
        st[1] = r;
    }
}
constexpr size_t STATS_ROW_SMEM_MAX = 200 * 1024;

// ------------------------------------------------------------------ pv
template <int NREP, int DPT>
__global__ void __launch_bounds__(THREADS) attn_pv_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int hd = a.head_dim;
    bf16 *vtile = reinterpret_cast<bf16 *>(smem);                          // [V_STAGES][VT][hd]
    float *s_tile = reinterpret_cast<float *>(vtile + V_STAGES * VT * hd);  // [V_STAGES][NREP][VT]
    float *p_tile = s_tile + V_STAGES * NREP * VT;                          // [NREP][VT]
    int *prefix = reinterpret_cast<int *>(p_tile + NREP * VT);
    __shared__ float m_s[NREP], s_s[NREP];

    pdl_trigger();
    pdl_wait();
    const bool split = a.stats != nullptr;
    const int chunk = a.chunk_b;
    const int total = build_prefix(a, chunk, prefix);
    const int tid = threadIdx.x;
    const int cpr = hd / 8;
    const int i0 = (int)((long long)total * blockIdx.x / gridDim.x);
    const int i1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);

    for (int item = i0; item < i1; item++) {
        const Item it = find_item(a, prefix, chunk, item);
        const int t0 = it.c * chunk;
        const int t1 = min(t0 + chunk, it.len);
        const int n_tiles = (t1 - t0 + VT - 1) / VT;
        const float *sc = a.scores + ((size_t)it.b * a.n_heads + (size_t)it.kvh * NREP) * a.ld;
        const bf16 *vsrc = a.vc + (size_t)it.b * a.kv.seq + (size_t)it.kvh * a.kv.head;

        auto issue = [&](int tile) {
            const int st = tile % V_STAGES;
            const int tt0 = t0 + tile * VT;
            const int rows = min(VT, t1 - tt0);
            bf16 *dst = vtile + st * VT * hd;
            for (int j = tid; j < rows * cpr; j += THREADS) {
                const int r = j / cpr, ch = j - r * cpr;
                cp_async16(dst + r * hd + ch * 8, vsrc + (size_t)(tt0 + r) * a.kv.pos + ch * 8);
            }
#pragma unroll
            for (int h = 0; h < NREP; h++) stage_scores(s_tile + (st * NREP + h) * VT, sc + (size_t)h * a.ld + tt0, rows);
        };

        if (split) {
            if (tid < NREP) {
                const float *st = a.stats + ((size_t)it.b * a.n_heads + it.kvh * NREP + tid) * 2;
                m_s[tid] = __ldcg(st);
                s_s[tid] = __ldcg(st + 1);
            }
        } else {
            // exact mode: this CTA is the only one of (b, kvh); the V ring memory stages the scores
            float m[NREP], s[NREP];
            const int cap = (V_STAGES * VT * hd * 2) / 4;
            softmax_stats<NREP>(a, it.b, it.kvh, it.len, reinterpret_cast<float *>(vtile), cap, m, s);
            if (tid < NREP) {
                m_s[tid] = m[tid];
                s_s[tid] = s[tid];
            }
        }
        __syncthreads();
        for (int tile = 0; tile < V_STAGES - 1; tile++) {
            if (tile < n_tiles) issue(tile);
            cp_async_commit();
        }

        float acc[NREP][DPT];
#pragma unroll
        for (int h = 0; h < NREP; h++)
#pragma unroll
            for (int k = 0; k < DPT; k++) acc[h][k] = 0.0f;

        for (int tile = 0; tile < n_tiles; tile++) {
            const int st = tile % V_STAGES;
            const int rows = min(VT, t1 - (t0 + tile * VT));
            if (tile + V_STAGES - 1 < n_tiles) issue(tile + V_STAGES - 1);
            cp_async_commit();
            cp_async_wait<V_STAGES - 1>();
            __syncthreads();
            // probabilities of this tile (src/kernels.cu:472-474)
            const float *stile = s_tile + st * NREP * VT;
            for (int j = tid; j < NREP * VT; j += THREADS) {
                const int h = j / VT, r = j - h * VT;
                if (r < rows) p_tile[j] = round_bf16(expf(stile[j] - m_s[h]) / s_s[h]);
            }
            __syncthreads();
            const bf16 *vt = vtile + st * VT * hd;
#pragma unroll
            for (int k = 0; k < DPT; k++) {
                const int d = tid + k * THREADS;
                if (d < hd) {
#pragma unroll 8
                    for (int r = 0; r < rows; r++) {
                        const float v = __bfloat162float(vt[r * hd + d]);
#pragma unroll
                        for (int h = 0; h < NREP; h++) acc[h][k] = __fmaf_rn(p_tile[h * VT + r], v, acc[h][k]);
                    }
                }
            }
            __syncthreads();  // the stage and p_tile are rewritten next
        }
        cp_async_wait<0>();

        const size_t out_base = (size_t)it.b * a.q_stride + (size_t)it.kvh * NREP * hd;
        if (it.nc == 1) {
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DPT; k++) {
                    const int d = tid + k * THREADS;
                    if (d < hd) a.out[out_base + (size_t)h * hd + d] = __float2bfloat16(acc[h][k]);
                }
        } else {
            float *part = a.partial + ((size_t)it.b * a.n_heads + it.kvh * NREP) * a.max_chunks * hd;
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DPT; k++) {
                    const int d = tid + k * THREADS;
                    if (d < hd) part[((size_t)h * a.max_chunks + it.c) * hd + d] = acc[h][k];
                }
        }
    }
}

// ------------------------------------------------------------------ scores, TMA-fed (split mode)
// The reference's score arithmetic, bit for bit, at streaming speed. One item = (b, kv head, 128
// positions). A producer thread loads the item's K tile by TMA as head_dim / 64 boxes of
// [128 positions][64 dims] (128-byte swizzle), one box per ring stage, into a ring of SX_STAGES
// boxes, never waiting for anything but a free stage, so the cache streams while the dot products
// run. G groups of two consumer warps take the CTA's items in turn; in a group, thread r owns
// the positions r and r + 64 of the tile. For each box it copies its two rows' 128-byte pieces
// into registers and frees the stage at once -- the ring then holds almost only copies in
// flight, which is what keeps HBM busy -- and then computes, for each of its two rows and every
// query head of the kv group, the reference's dot product: one fp32 chain per (row, head), dims
// in order, one fused multiply-add each (src/kernels.cu:455-460, where nvcc fuses
// `dot += q * k`), then s = round_bf16(round_bf16(dot) * scale). Each step is one
// mixed-precision fma of the bf16 q and k into the fp32 chain (fma_bb): no conversions, and bit
// for bit the fp32 fma of the converted operands. The group's query heads sit in shared memory as
// bf16 [dim][head], so one vector load gives two dims' values for every head and serves both
// rows. The swizzle puts the 16-byte chunk c of row r at chunk c ^ (r % 8): a warp's
// 32 threads reading the same logical chunk of 32 consecutive rows need only the four wavefronts
// of their 512 bytes.
constexpr int SX_TILE = 128;
constexpr int SX_BOX = SX_TILE * 128;  // one 64-dim box: 16 KB
constexpr int SX_STAGES = 12;
constexpr int SX_GWARPS = 2;  // warps per group: 64 threads, two rows each
// Consumer groups per CTA, by boxes per item (head_dim / 64). A group waits on the ring stages of
// its own items only, with the parity of the lap it expects; that is sound only if the stage's
// previous box also belonged to this group (a box of another group may not have landed yet, and a
// wait two phases ahead of the barrier passes at once). With items dealt round-robin that holds
// when SX_STAGES is a multiple of groups x boxes per item: 6 groups for one box an item (head_dim
// 64), 3 for two (head_dim 128: each group then has two items in flight while it computes; with
// six groups it had one, and the Qwen3-4B B = 32 decode step took 6.41 ms instead of 6.32),
// 4 for three (head_dim 192), 3 for four (head_dim 256).
constexpr int sx_groups(int halves) { return halves == 1 ? 6 : halves == 3 ? 4 : 3; }
static_assert(SX_STAGES % (sx_groups(1) * 1) == 0 && SX_STAGES % (sx_groups(2) * 2) == 0 &&
                  SX_STAGES % (sx_groups(3) * 3) == 0 && SX_STAGES % (sx_groups(4) * 4) == 0,
              "a ring stage must come back to the group that used it last");
constexpr int sx_threads(int groups) { return 32 + groups * SX_GWARPS * 32; }  // producer warp + the groups

struct ScoreXPlan {
    int halves;           // head_dim / 64: boxes per item
    int k_rows_per_seq;   // rows of the K map per sequence (kv.seq / kv.pos)
    int k_rows_per_head;  // head-major caches: rows per kv head (kv.head / kv.pos), else 0
    int k_cols_per_head;  // heads within a row: columns per kv head (kv.head), else 0
    int tab_cap;          // items the shared-memory item table holds
};

__device__ __forceinline__ void group_sync(int group) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "n"(SX_GWARPS * 32) : "memory");
}

// True in every thread of the group if `v` is true in any (a barrier of the group).
__device__ __forceinline__ bool group_any(int group, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(1 + group), "n"(SX_GWARPS * 32)
        : "memory");
    return r != 0;
}

// q words of two consecutive dims d, d + 1 for the NREP heads, bf16 [dim][head]: with NREP >= 2
// word i of dim d holds heads 2i, 2i + 1 and dim d + 1's words follow; with one head the word
// holds dim d in its low half and d + 1 in its high half. One shared-memory vector load.
template <int NREP>
struct QPair {
    uint32_t w[NREP == 1 ? 1 : NREP];
};
template <int NREP>
__device__ __forceinline__ QPair<NREP> load_q2(const bf16 *p) {
    QPair<NREP> q;
    if constexpr (NREP == 8) {
        const uint4 u0 = *reinterpret_cast<const uint4 *>(p), u1 = *reinterpret_cast<const uint4 *>(p + 8);
        q.w[0] = u0.x, q.w[1] = u0.y, q.w[2] = u0.z, q.w[3] = u0.w;
        q.w[4] = u1.x, q.w[5] = u1.y, q.w[6] = u1.z, q.w[7] = u1.w;
    } else if constexpr (NREP == 4) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        q.w[0] = u.x, q.w[1] = u.y, q.w[2] = u.z, q.w[3] = u.w;
    } else if constexpr (NREP == 2) {
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        q.w[0] = u.x, q.w[1] = u.y;
    } else {
        q.w[0] = *reinterpret_cast<const uint32_t *>(p);
    }
    return q;
}

// acc = fma(q, k, acc) with q and k the low or high bf16 halves of q2 and k2. sm_100's
// mixed-precision fma takes the bf16 operands as they are: their product is exact in fp32 (8 + 8
// significant bits) and the one rounding of q * k + acc is that of fmaf(float(q), float(k), acc),
// so the chain is the reference's bit for bit with no operand converted first.
__device__ __forceinline__ void fma_bb(float &acc, uint32_t q2, bool qhi, uint32_t k2, bool khi) {
#define Q3_FMA_BB(QR, KR)                                                                  \
    asm("{\n\t.reg .b16 ql, qh, kl, kh;\n\tmov.b32 {ql, qh}, %1;\n\tmov.b32 {kl, kh}, %2;\n\t" \
        "fma.rn.f32.bf16 %0, " QR ", " KR ", %0;\n\t}"                                       \
        : "+f"(acc)                                                                        \
        : "r"(q2), "r"(k2))
    if (qhi) {
        if (khi) Q3_FMA_BB("qh", "kh");
        else Q3_FMA_BB("qh", "kl");
    } else {
        if (khi) Q3_FMA_BB("ql", "kh");
        else Q3_FMA_BB("ql", "kl");
    }
#undef Q3_FMA_BB
}

// Dim d (0 or 1) of the pair for every head of one row; k is the row's word holding both dims.
template <int NREP>
__device__ __forceinline__ void fma_heads_bb(float (&acc)[NREP], const QPair<NREP> &q, int d, uint32_t kw) {
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        if constexpr (NREP == 1) fma_bb(acc[h], q.w[0], d == 1, kw, d == 1);
        else fma_bb(acc[h], q.w[d * (NREP / 2) + h / 2], (h & 1) == 1, kw, d == 1);
    }
}

template <int NREP, int G>
__global__ void __launch_bounds__(sx_threads(G), 1)
    attn_scores_exact_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ AttnArgs a,
                             const __grid_constant__ ScoreXPlan pl) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = align_shared<1024>(smem_raw);
    const int hd = a.head_dim;
    bf16 *q_all = reinterpret_cast<bf16 *>(smem + (size_t)SX_STAGES * SX_BOX);  // [G][hd][NREP]
    uint64_t *full = reinterpret_cast<uint64_t *>(q_all + G * NREP * hd);
    uint64_t *empty = full + SX_STAGES;
    int *prefix = reinterpret_cast<int *>(empty + SX_STAGES);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int i = 0; i < SX_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], SX_GWARPS);  // the warps of the group that reads the box
        }
        fence_barrier_init();
        prefetch_tmap(&tmK);
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();  // positions, queries and the newest cache rows come from the previous kernels
    const int total = build_prefix(a, SX_TILE, prefix);
    const int i0 = (int)((long long)total * blockIdx.x / gridDim.x);
    const int i1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
    const int n = i1 - i0;
    int2 *tab = reinterpret_cast<int2 *>(prefix + ITEM_TAB_OFF(a.B));
    const bool tabbed = fill_items(a, prefix, SX_TILE, i0, n, tab, pl.tab_cap);
    int cur = n > 0 ? first_seq(prefix, a.B, i0) : 0;  // this thread's sequence cursor

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer: box j of the ring is box j % halves of item j / halves
            const uint64_t stream_pol = policy_evict_first();  // K rows are read once per step
            const int nbox = n * pl.halves;
            int j = 0;
            for (; j < nbox; j++) {
                const int st = j % SX_STAGES;
                if (j >= SX_STAGES && !mbar_wait(&empty[st], ((j / SX_STAGES) - 1) & 1, &g_dev_error)) break;
                const int h = j % pl.halves;
                const Item it = item_k(a, prefix, SX_TILE, tab, tabbed, i0, j / pl.halves, cur);
                mbar_arrive_expect_tx(&full[st], (uint32_t)SX_BOX);
                const int krow = it.b * pl.k_rows_per_seq + it.kvh * pl.k_rows_per_head + it.c * SX_TILE;
                tma_load_2d_stream(smem + (size_t)st * SX_BOX, &tmK, it.kvh * pl.k_cols_per_head + h * TMA_BK, krow,
                                   &full[st], stream_pol);
            }
            // copies still in flight land before the CTA exits (bounded waits)
            for (int i = max(0, j - SX_STAGES); i < j; i++)
                mbar_wait(&full[i % SX_STAGES], (i / SX_STAGES) & 1, &g_dev_error);
        }
        return;
    }
    // ---------------- consumers: group g takes items g, g + G, ...
    const int group = (warp - 1) / SX_GWARPS;
    const int gt = threadIdx.x - 32 - group * SX_GWARPS * 32;  // 0..63
    bf16 *q_s = q_all + group * NREP * hd;                      // [hd][NREP]
    int qb = -1, qk = -1;
    const int sw = gt & 7;  // rows gt and gt + 64 share the swizzle phase
    bool failed = false;
    for (int k = group; k < n && !failed; k += G) {
        const Item it = item_k(a, prefix, SX_TILE, tab, tabbed, i0, k, cur);
        if (it.b != qb || it.kvh != qk) {  // the group's query heads, bf16, dims outermost
            group_sync(group);             // nobody still reads the previous ones
            const bf16 *qg = a.q + (size_t)it.b * a.q_stride + (size_t)it.kvh * NREP * hd;
            for (int j = gt; j < NREP * hd; j += SX_GWARPS * 32) q_s[(j % hd) * NREP + j / hd] = qg[j];
            group_sync(group);
            qb = it.b;
            qk = it.kvh;
        }
        const int ta = it.c * SX_TILE + gt, tb = ta + 64;
        float acc_a[NREP], acc_b[NREP];
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            acc_a[h] = 0.0f;
            acc_b[h] = 0.0f;
        }
        for (int half = 0; half < pl.halves; half++) {
            const int j = k * pl.halves + half;  // ring box
            const int st = j % SX_STAGES;
            const bool ok = mbar_wait(&full[st], (j / SX_STAGES) & 1, &g_dev_error);
            // a timed-out wait ends the group's loop in all of its threads together (the group
            // barriers above need all of them)
            failed = group_any(group, !ok);
            bf16x8 ka[8], kb[8];
            if (ok) {
                const unsigned char *rowa = smem + (size_t)st * SX_BOX + gt * 128;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    ka[c] = lds128(rowa + ((c ^ sw) << 4));
                    kb[c] = lds128(rowa + 64 * 128 + ((c ^ sw) << 4));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);  // the rows are in registers: the box is free
            if (failed) break;
            const bf16 *qd = q_s + half * 64 * NREP;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint4 wa = *reinterpret_cast<const uint4 *>(&ka[c]);
                const uint4 wb = *reinterpret_cast<const uint4 *>(&kb[c]);
                const uint32_t pa[4] = {wa.x, wa.y, wa.z, wa.w}, pb[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const QPair<NREP> q = load_q2<NREP>(qd + (c * 8 + e) * NREP);
                    fma_heads_bb<NREP>(acc_a, q, 0, pa[e / 2]);
                    fma_heads_bb<NREP>(acc_b, q, 0, pb[e / 2]);
                    fma_heads_bb<NREP>(acc_a, q, 1, pa[e / 2]);
                    fma_heads_bb<NREP>(acc_b, q, 1, pb[e / 2]);
                }
            }
        }
        if (failed) break;
        float *sc = a.scores + ((size_t)it.b * a.n_heads + (size_t)it.kvh * NREP) * a.ld;
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            if (ta < it.len) sc[(size_t)h * a.ld + ta] = round_bf16(round_bf16(acc_a[h]) * a.scale);
            if (tb < it.len) sc[(size_t)h * a.ld + tb] = round_bf16(round_bf16(acc_b[h]) * a.scale);
        }
    }
}

// ------------------------------------------------------------------ pv on tcgen05 (split mode)
// One item = (b, kv head, chunk of positions); per 128-position tile the MMA computes
// D[head_dim x 16] += V_tile^T[head_dim x 128] . P^T[128 x 16] into a TMEM accumulator.
//   A = V tile, loaded by TMA as two 64-dim halves of [128 positions][64 dims] (128-byte swizzle):
//       MN-major (dims contiguous), LBO = 16 KB between the halves, SBO = 1 KB per 8 positions.
//   B = P, [16 rows][128 positions] bf16 written by the p warps in the K-major 128-byte swizzle
//       layout: row h holds p = round_bf16(expf(s - max) / sum) of query head h of the group
//       (src/kernels.cu:472-474), rows NREP..15 are zero, as are positions past the sequence.
// p and v are bf16 and the accumulator fp32, so every product is exact; only the order of the
// fp32 additions differs from a serial chain. V rows past the end of the sequence are zeroed in
// shared memory before the MMA (the cache there may hold anything, and 0 * NaN is NaN).
constexpr int PV_TILE = 128;
#ifndef Q3_PV_STAGES
#define Q3_PV_STAGES 4
#endif
constexpr int PV_STAGES = Q3_PV_STAGES;
constexpr int PV_ACC = 2;
#ifndef Q3_PV_GROUPS
#define Q3_PV_GROUPS 2
#endif
// p-warp groups: group g computes the probabilities of query heads h with h % PV_GROUPS == g.
// One warp per scheduler leaves the exp / divide / round chain of every tile without latency
// hiding; more groups shorten the chain each warp runs per tile.
constexpr int PV_GROUPS = Q3_PV_GROUPS;
constexpr int PV_P_THREADS = 128 * PV_GROUPS;
constexpr int PV_THREADS = 64 + PV_P_THREADS;  // producer warp, MMA warp, p warps
constexpr int PV_V_BYTES = PV_TILE * 128;      // one 64-dim half of a V tile
constexpr int PV_P_OFF = 2 * PV_V_BYTES;       // P: 2 swizzle atoms of 16 rows x 128 B
constexpr int PV_S_OFF = PV_P_OFF + 2 * 16 * 128;
constexpr int PV_T_OFF = PV_S_OFF + 16 * PV_TILE * 4;       // scores of the 16 P rows
constexpr int PV_STAGE_BYTES = PV_T_OFF + 1024;             // their (max, sum) pairs, 64 B per row

struct PvTcPlan {
    int k_rows_per_seq, k_rows_per_head, k_cols_per_head;
    uint32_t idesc;
    int tab_cap;  // items the shared-memory item table holds
    int rows;     // rows per item: 16 / NREP when the rows share one cache (a prompt), else 1
};

template <int NREP, int GR>
__global__ void __launch_bounds__(PV_THREADS, 1)
    attn_pv_tc_kernel(const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnArgs a,
                      const __grid_constant__ PvTcPlan pl) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = align_shared<1024>(smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)PV_STAGES * PV_STAGE_BYTES);
    uint64_t *pfull = full + PV_STAGES;
    uint64_t *empty = pfull + PV_STAGES;
    uint64_t *acc_full = empty + PV_STAGES;
    uint64_t *acc_empty = acc_full + PV_ACC;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + PV_ACC);
    int *prefix = reinterpret_cast<int *>(tmem_slot + 4);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int chunk = a.chunk_b;  // a multiple of PV_TILE

    if (threadIdx.x == 0) {
        for (int i = 0; i < PV_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&pfull[i], PV_P_THREADS);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < PV_ACC; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], PV_P_THREADS);
        }
        fence_barrier_init();
        prefetch_tmap(&tmV);
    }
    if (warp >= 2) {  // zero the padding rows (past rows x NREP) of every stage's P once
        const int t = threadIdx.x - 64;
        for (int j = t; j < PV_STAGES * 2 * 16 * 8; j += PV_P_THREADS) {  // 16-byte units
            const int st = j / 256, r = j % 256, atom = r / 128, row = (r % 128) / 8, c = r % 8;
            if (row >= GR * NREP)
                *reinterpret_cast<uint4 *>(smem + (size_t)st * PV_STAGE_BYTES + PV_P_OFF + atom * 2048 + row * 128 + c * 16) =
                    make_uint4(0, 0, 0, 0);
        }
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(32)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();
    pdl_wait();  // positions, scores and statistics come from the previous kernels
    // An item is (row group g, kv head, chunk): G rows r = g*G + i share the item's V tiles, and
    // the MMA's N = 16 columns are their NREP heads each (G = 16 / NREP rows of one prompt, whose
    // rows read one cache; one row otherwise). `ag` describes the groups to the item helpers.
    constexpr int G = GR;
    AttnArgs ag = a;
    ag.B = (a.B + G - 1) / G;
    const int total = build_prefix_rows(a, chunk, prefix, G);
    const int i0 = (int)((long long)total * blockIdx.x / gridDim.x);
    const int i1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
    int2 *tab = reinterpret_cast<int2 *>(prefix + ITEM_TAB_OFF(a.B));
    const bool tabbed = fill_items(ag, prefix, chunk, i0, i1 - i0, tab, pl.tab_cap);
    int cur = i1 > i0 ? first_seq(prefix, ag.B, i0) : 0;

    if (warp == 0 && lane == 0) {
        // ---------------- producer: V tile halves by TMA, the group's scores by bulk copy
        const uint64_t stream_pol = policy_evict_first();  // V rows are read once per step
        int k = 0;
        bool ok = true;
        const uint32_t stat_slot = 1024u / (uint32_t)G;  // bytes of the stats area per row
        for (int item = i0; item < i1 && ok; item++) {
            const Item it = item_k(ag, prefix, chunk, tab, tabbed, i0, item - i0, cur);
            const int t0 = it.c * chunk, t1 = min(t0 + chunk, it.len);
            const int r0 = it.b * G, nr = min(G, a.B - r0);  // the item's rows
            const int row0 = it.b * pl.k_rows_per_seq + it.kvh * pl.k_rows_per_head;
            // each row's statistics, from the 16-byte boundary below them (the stats region is
            // padded to 256 bytes, so the rounded-up copy stays inside it)
            uint32_t tbytes_all = 0;
            for (int i = 0; i < nr; i++) {
                const float *stp = a.stats + ((size_t)(r0 + i) * a.n_heads + (size_t)it.kvh * NREP) * 2;
                const uintptr_t st_al = reinterpret_cast<uintptr_t>(stp) & ~uintptr_t(15);
                tbytes_all += (uint32_t)((reinterpret_cast<uintptr_t>(stp) - st_al + NREP * 8 + 15) & ~15u);
            }
            for (int tt = t0; tt < t1; tt += PV_TILE, k++) {
                const int st = k % PV_STAGES;
                if (k >= PV_STAGES && !mbar_wait(&empty[st], ((k / PV_STAGES) - 1) & 1, &g_dev_error)) {
                    ok = false;
                    break;
                }
                const int rows = min(PV_TILE, t1 - tt);
                const uint32_t sbytes = (uint32_t)((rows + 3) / 4) * 16;  // within ld: ld is a multiple of 4
                unsigned char *base = smem + (size_t)st * PV_STAGE_BYTES;
                const bool first = tt == t0;
                mbar_arrive_expect_tx(&full[st], 2 * PV_V_BYTES + (uint32_t)(nr * NREP) * sbytes + (first ? tbytes_all : 0));
                if (first)
                    for (int i = 0; i < nr; i++) {
                        const float *stp = a.stats + ((size_t)(r0 + i) * a.n_heads + (size_t)it.kvh * NREP) * 2;
                        const uintptr_t st_al = reinterpret_cast<uintptr_t>(stp) & ~uintptr_t(15);
                        const uint32_t tb = (uint32_t)((reinterpret_cast<uintptr_t>(stp) - st_al + NREP * 8 + 15) & ~15u);
                        bulk_g2s(base + PV_T_OFF + i * stat_slot, reinterpret_cast<const void *>(st_al), tb, &full[st]);
                    }
                tma_load_2d_stream(base, &tmV, it.kvh * pl.k_cols_per_head, row0 + tt, &full[st], stream_pol);
                tma_load_2d_stream(base + PV_V_BYTES, &tmV, it.kvh * pl.k_cols_per_head + TMA_BK, row0 + tt, &full[st], stream_pol);
                for (int i = 0; i < nr; i++) {
                    const float *sc = a.scores + ((size_t)(r0 + i) * a.n_heads + (size_t)it.kvh * NREP) * a.ld;
#pragma unroll
                    for (int h = 0; h < NREP; h++)
                        bulk_g2s(base + PV_S_OFF + (i * NREP + h) * PV_TILE * 4, sc + (size_t)h * a.ld + tt, sbytes,
                                 &full[st]);
                }
            }
        }
        // drain: every issued copy lands before the CTA exits
        for (int j = max(0, k - PV_STAGES); j < k; j++) mbar_wait(&full[j % PV_STAGES], (j / PV_STAGES) & 1, &g_dev_error);
        // tail: the MMA frees each stage with tcgen05.commit, whose arrive on `empty` is performed
        // asynchronously when the MMAs finish -- possibly after the accumulator's own commit, which
        // is all the epilogue waits for. Wait for the last uses' arrives too, so that none lands in
        // the shared memory of the next CTA on this SM.
        for (int j = max(0, k - PV_STAGES); j < k; j++) mbar_wait(&empty[j % PV_STAGES], (j / PV_STAGES) & 1, &g_dev_error);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer
        int k = 0, n_items = 0;
        bool ok = true;
        for (int item = i0; item < i1 && ok; item++, n_items++) {
            const Item it = item_k(ag, prefix, chunk, tab, tabbed, i0, item - i0, cur);
            const int t0 = it.c * chunk, t1 = min(t0 + chunk, it.len);
            const int buf = n_items % PV_ACC;
            if (n_items >= PV_ACC && !mbar_wait(&acc_empty[buf], ((n_items / PV_ACC) - 1) & 1, &g_dev_error)) break;
            const uint32_t d_tmem = tmem_base + buf * 16;
            for (int tt = t0; tt < t1; tt += PV_TILE, k++) {
                const int st = k % PV_STAGES;
                if (!mbar_wait(&full[st], (k / PV_STAGES) & 1, &g_dev_error) ||
                    !mbar_wait(&pfull[st], (k / PV_STAGES) & 1, &g_dev_error)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t vb = smem_u32(smem + (size_t)st * PV_STAGE_BYTES);
                const uint32_t pb = vb + PV_P_OFF;
#pragma unroll
                for (int kk = 0; kk < PV_TILE / 16; kk++) {
                    const uint64_t ad = smem_desc_sw128(vb + kk * 16 * 128, PV_V_BYTES, 1024);
                    const uint64_t bd = smem_desc_sw128(pb + (kk / 4) * 2048 + (kk % 4) * 32, 16, 1024);
                    mma_bf16(d_tmem, ad, bd, pl.idesc, (tt > t0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&empty[st]);
            }
            if (ok) mma_commit(&acc_full[buf]);
        }
    } else if (warp >= 2) {
        // ---------------- p warps: one position per thread and group; then the item's epilogue
        const int t = (threadIdx.x - 64) % 128, grp = (threadIdx.x - 64) / 128;
        const int quarter = warp % 4;
        const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
        const int d = quarter * 32 + lane;  // accumulator row = head dim
        // The epilogue of an item runs after the first tile of the next one has been handed to
        // the MMA, so that waiting for the accumulator overlaps the next item's work.
        Item pend = {};
        int pend_n = -1;
        // P rows n = i * NREP + h: row r0 + i of the item, query head h of the kv group
        constexpr int NP = G * NREP;
        const uint32_t stat_slot = 1024u / (uint32_t)G;
        auto epilogue = [&](const Item &it, int n_item) -> bool {
            const int buf = n_item % PV_ACC;
            // warp-uniform exit: tcgen05.ld below is warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (n_item / PV_ACC) & 1, &g_dev_error))) return false;
            tc_fence_after();
            float acc[16];
            tmem_ld8(lane_addr + buf * 16, acc);
            if (NP > 8) tmem_ld8(lane_addr + buf * 16 + 8, acc + 8);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&acc_empty[buf]);
            if (d < a.head_dim) {
                const int r0 = it.b * G;
#pragma unroll
                for (int n = 0; n < NP; n++) {
                    if (n % PV_GROUPS != grp) continue;
                    const int r = r0 + n / NREP, h = n % NREP;
                    if (r >= a.B) continue;
                    // this row's own chunk count: rows of a group end at different positions
                    const int nc = G == 1 ? it.nc : (seq_len(a, r) + chunk - 1) / chunk;
                    if (it.c >= nc) continue;
                    if (nc == 1) {
                        a.out[(size_t)r * a.q_stride + ((size_t)it.kvh * NREP + h) * a.head_dim + d] = __float2bfloat16(acc[n]);
                    } else {
                        float *part = a.partial + ((size_t)r * a.n_heads + it.kvh * NREP + h) * a.max_chunks * a.head_dim;
                        part[(size_t)it.c * a.head_dim + d] = acc[n];
                    }
                }
            }
            return true;
        };
        int k = 0, n_items = 0;
        bool ok = true;
        for (int item = i0; item < i1 && ok; item++, n_items++) {
            const Item it = item_k(ag, prefix, chunk, tab, tabbed, i0, item - i0, cur);
            const int t0 = it.c * chunk, t1 = min(t0 + chunk, it.len);
            const int r0 = it.b * G;
            float m[NP], sum[NP];
            int len[NP];  // each P row's sequence length: its positions past it get p = 0
#pragma unroll
            for (int n = 0; n < NP; n++) len[n] = G == 1 ? it.len : r0 + n / NREP < a.B ? seq_len(a, r0 + n / NREP) : 0;
            for (int tt = t0; tt < t1; tt += PV_TILE, k++) {
                const int st = k % PV_STAGES;
                if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (k / PV_STAGES) & 1, &g_dev_error))) {
                    ok = false;  // the whole warp leaves: the epilogue's tcgen05.ld is warp-collective
                    break;
                }
                unsigned char *base = smem + (size_t)st * PV_STAGE_BYTES;
                if (tt == t0) {  // the statistics came with the item's first tile
#pragma unroll
                    for (int n = 0; n < NP; n++) {
                        if (len[n] == 0) continue;
                        const int i = n / NREP, h = n % NREP;
                        const uintptr_t src = reinterpret_cast<uintptr_t>(
                            a.stats + ((size_t)(r0 + i) * a.n_heads + (size_t)it.kvh * NREP) * 2);
                        const float *stp = reinterpret_cast<const float *>(base + PV_T_OFF + i * stat_slot + (src & 15));
                        m[n] = stp[2 * h];
                        sum[n] = stp[2 * h + 1];
                    }
                }
                const int rows = min(PV_TILE, t1 - tt);
                const float *s_st = reinterpret_cast<const float *>(base + PV_S_OFF);
                unsigned char *prow = base + PV_P_OFF + (t / 64) * 2048 + (t % 8) * 2;
                const int c16 = (t % 64) / 8;
#pragma unroll
                for (int n = 0; n < NP; n++) {
                    if (n % PV_GROUPS != grp) continue;
                    const float p = tt + t < len[n] ? round_bf16(expf(s_st[n * PV_TILE + t] - m[n]) / sum[n]) : 0.0f;
                    *reinterpret_cast<bf16 *>(prow + n * 128 + ((c16 ^ (n & 7)) << 4)) = __float2bfloat16(p);
                }
                if (t >= rows) {  // V rows past the sequence: zero both halves of row t, split over the groups
                    for (int half = grp; half < 2; half += PV_GROUPS) {
                        uint4 *v = reinterpret_cast<uint4 *>(base + half * PV_V_BYTES + t * 128);
#pragma unroll
                        for (int c = 0; c < 8; c++) v[c] = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_proxy_async();
                mbar_arrive(&pfull[st]);
                if (pend_n >= 0) {
                    if (!epilogue(pend, pend_n)) ok = false;
                    pend_n = -1;
                    if (!ok) break;
                }
            }
            pend = it;
            pend_n = n_items;
        }
        if (ok && pend_n >= 0) epilogue(pend, pend_n);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(32) : "memory");
    }
}

// ------------------------------------------------------------------ pv, vectorized (split mode)
// Thread t covers dims 2*(t % P), 2*(t % P) + 1 (P = head_dim / 2 threads per group) for the
// positions of group t / P: group g takes the g-th of G = 128 / P contiguous slices of every V
// tile. The G partial sums are added in group order at the end of the item.
template <int NREP>
__global__ void __launch_bounds__(THREADS) attn_pv_vec_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int hd = a.head_dim;
    const int P = hd / 2, G = THREADS / P;
    bf16 *vtile = reinterpret_cast<bf16 *>(smem);                          // [V_STAGES][VT][hd]
    float *s_tile = reinterpret_cast<float *>(vtile + V_STAGES * VT * hd);  // [V_STAGES][NREP][VT]
    float *p_tile = s_tile + V_STAGES * NREP * VT;                          // [VT][NREP]
    float *red = p_tile + VT * NREP;                                        // [G][NREP][hd]
    int *prefix = reinterpret_cast<int *>(red + G * NREP * hd);
    __shared__ float m_s[NREP], s_s[NREP];

    pdl_trigger();
    pdl_wait();
    const int chunk = a.chunk_b;
    const int total = build_prefix(a, chunk, prefix);
    const int tid = threadIdx.x;
    const int cpr = hd / 8;
    const int pair = tid % P, grp = tid / P;
    const int i0 = (int)((long long)total * blockIdx.x / gridDim.x);
    const int i1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
    const int sub = VT / G;  // positions of a tile per group

    for (int item = i0; item < i1; item++) {
        const Item it = find_item(a, prefix, chunk, item);
        const int t0 = it.c * chunk;
        const int t1 = min(t0 + chunk, it.len);
        const int n_tiles = (t1 - t0 + VT - 1) / VT;
        const float *sc = a.scores + ((size_t)it.b * a.n_heads + (size_t)it.kvh * NREP) * a.ld;
        const bf16 *vsrc = a.vc + (size_t)it.b * a.kv.seq + (size_t)it.kvh * a.kv.head;
        auto issue = [&](int tile) {
            const int st = tile % V_STAGES;
            const int tt0 = t0 + tile * VT;
            const int rows = min(VT, t1 - tt0);
            bf16 *dst = vtile + st * VT * hd;
            for (int j = tid; j < rows * cpr; j += THREADS) {
                const int r = j / cpr, ch = j - r * cpr;
                cp_async16(dst + r * hd + ch * 8, vsrc + (size_t)(tt0 + r) * a.kv.pos + ch * 8);
            }
#pragma unroll
            for (int h = 0; h < NREP; h++) stage_scores(s_tile + (st * NREP + h) * VT, sc + (size_t)h * a.ld + tt0, rows);
        };
        if (tid < NREP) {
            const float *st = a.stats + ((size_t)it.b * a.n_heads + it.kvh * NREP + tid) * 2;
            m_s[tid] = __ldcg(st);
            s_s[tid] = __ldcg(st + 1);
        }
        __syncthreads();
        for (int tile = 0; tile < V_STAGES - 1; tile++) {
            if (tile < n_tiles) issue(tile);
            cp_async_commit();
        }
        float acc[NREP][2];
#pragma unroll
        for (int h = 0; h < NREP; h++) acc[h][0] = acc[h][1] = 0.0f;
        for (int tile = 0; tile < n_tiles; tile++) {
            const int st = tile % V_STAGES;
            const int rows = min(VT, t1 - (t0 + tile * VT));
            if (tile + V_STAGES - 1 < n_tiles) issue(tile + V_STAGES - 1);
            cp_async_commit();
            cp_async_wait<V_STAGES - 1>();
            __syncthreads();
            const float *stile = s_tile + st * NREP * VT;
            for (int j = tid; j < NREP * VT; j += THREADS) {
                const int h = j / VT, r = j - h * VT;
                if (r < rows) p_tile[r * NREP + h] = round_bf16(expf(stile[j] - m_s[h]) / s_s[h]);
            }
            __syncthreads();
            const bf16 *vt = vtile + st * VT * hd + 2 * pair;
            const int r0 = grp * sub, r1 = min(r0 + sub, rows);
#pragma unroll 4
            for (int r = r0; r < r1; r++) {
                const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(vt + r * hd));
                float pv[NREP];
                if (NREP == 4) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(p_tile + r * 4);
                    pv[0] = p4.x; pv[1] = p4.y; pv[2] = p4.z; pv[3] = p4.w;
                } else {
#pragma unroll
                    for (int h = 0; h < NREP; h++) pv[h] = p_tile[r * NREP + h];
                }
#pragma unroll
                for (int h = 0; h < NREP; h++) {
                    acc[h][0] = __fmaf_rn(pv[h], v.x, acc[h][0]);
                    acc[h][1] = __fmaf_rn(pv[h], v.y, acc[h][1]);
                }
            }
            __syncthreads();
        }
        cp_async_wait<0>();
        // groups' partial sums, added in group order
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            red[(grp * NREP + h) * hd + 2 * pair] = acc[h][0];
            red[(grp * NREP + h) * hd + 2 * pair + 1] = acc[h][1];
        }
        __syncthreads();
        const size_t out_base = (size_t)it.b * a.q_stride + (size_t)it.kvh * NREP * hd;
        float *part = a.partial + ((size_t)it.b * a.n_heads + it.kvh * NREP) * a.max_chunks * hd;
        for (int j = tid; j < NREP * hd; j += THREADS) {
            const int h = j / hd, d = j - h * hd;
            float o = 0.0f;
            for (int g = 0; g < G; g++) o += red[(g * NREP + h) * hd + d];
            if (it.nc == 1) a.out[out_base + (size_t)h * hd + d] = __float2bfloat16(o);
            else part[((size_t)h * a.max_chunks + it.c) * hd + d] = o;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ combine (split mode)
__global__ void __launch_bounds__(256) attn_combine_kernel(const __grid_constant__ AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.y, h = blockIdx.x;
    const int len = seq_len(a, b);
    const int nc = (len + a.chunk_b - 1) / a.chunk_b;
    if (nc <= 1) return;  // the pv kernel wrote the output directly
    const float *part = a.partial + ((size_t)b * a.n_heads + h) * a.max_chunks * a.head_dim;
    for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) {
        float o = 0.0f;
        int c = 0;
        for (; c + 4 <= nc; c += 4) {  // four loads in flight, added in chunk order
            const float p0 = __ldcg(part + (size_t)(c + 0) * a.head_dim + d);
            const float p1 = __ldcg(part + (size_t)(c + 1) * a.head_dim + d);
            const float p2 = __ldcg(part + (size_t)(c + 2) * a.head_dim + d);
            const float p3 = __ldcg(part + (size_t)(c + 3) * a.head_dim + d);
            o += p0;
            o += p1;
            o += p2;
            o += p3;
        }
        for (; c < nc; c++) o += __ldcg(part + (size_t)c * a.head_dim + d);
        a.out[(size_t)b * a.q_stride + (size_t)h * a.head_dim + d] = __float2bfloat16(o);
    }
}

// Rows of the [rows, kv.pos] view of a K or V cache that the TMA maps cover: every sequence's
// rows, or, when all rows share one cache (sequence stride 0: the rows of one prompt), that
// cache's rows (n_kv heads of max_seq positions head-major, or max_seq positions).
long long cache_map_rows(const AttnArgs &a) {
    if (a.kv.seq > 0) return (long long)a.B * (a.kv.seq / a.kv.pos);
    return a.kv.head >= a.kv.pos ? (long long)a.n_kv * (a.kv.head / a.kv.pos) : (long long)a.max_seq;
}

template <int NREP, int G>
int launch_scores_exact_g(const CUtensorMap &mk, const AttnArgs &a, const ScoreXPlan &pl, int grid, size_t smem,
                          cudaStream_t s) {
    Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_scores_exact_kernel<NREP, G>), smem));
    Q3_TRY_LAUNCH(launch(attn_scores_exact_kernel<NREP, G>, dim3(grid), dim3(sx_threads(G)), smem, s, 1, mk, a, pl));
    return Q3_OK;
}

template <int NREP>
int launch_scores_exact(const AttnArgs &a, cudaStream_t s) {
    ScoreXPlan pl;
    pl.halves = a.head_dim / TMA_BK;
    pl.k_rows_per_seq = (int)(a.kv.seq / a.kv.pos);
    pl.k_rows_per_head = a.kv.head >= a.kv.pos ? (int)(a.kv.head / a.kv.pos) : 0;
    pl.k_cols_per_head = a.kv.head >= a.kv.pos ? 0 : (int)a.kv.head;
    CUtensorMap mk;
    if (!make_map_strided(&mk, a.kc, cache_map_rows(a), a.kv.pos, a.kv.pos, SX_TILE)) return Q3_ERR_ARG;
    const int G = sx_groups(pl.halves);
    if (pl.halves < 1 || pl.halves > 4 || SX_STAGES % (G * pl.halves) != 0) return Q3_ERR_SHAPE;
    const size_t base = 1024 + (size_t)SX_STAGES * SX_BOX + (size_t)G * NREP * a.head_dim * 2 +
                        2 * SX_STAGES * 8 + (size_t)ITEM_TAB_OFF(a.B) * 4;
    pl.tab_cap = base < SMEM_CTA_MAX ? (int)std::min<size_t>(ITEM_TAB_MAX, (SMEM_CTA_MAX - base) / 8) : 0;
    const size_t smem = base + (size_t)pl.tab_cap * 8;
    const long long max_items = (long long)a.B * a.n_kv * ((a.max_seq + SX_TILE - 1) / SX_TILE);
    const int grid = (int)std::min<long long>(max_items, num_sms());
    switch (G) {
        case 6: return launch_scores_exact_g<NREP, 6>(mk, a, pl, grid, smem, s);
        case 4: return launch_scores_exact_g<NREP, 4>(mk, a, pl, grid, smem, s);
        default: return launch_scores_exact_g<NREP, 3>(mk, a, pl, grid, smem, s);
    }
}

// One block of 128 * NREP threads per (sequence, kv head).
// Fewer (sequence, kv head) groups than SMs: one CTA per (sequence, query head) instead.
template <int NREP>
int launch_stats(const AttnArgs &a, cudaStream_t s) {
    const size_t row_smem = (size_t)a.max_seq * 4;
    if (a.B * a.n_kv < num_sms() && row_smem <= STATS_ROW_SMEM_MAX) {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_stats_row_kernel), row_smem));
        Q3_TRY_LAUNCH(launch(attn_stats_row_kernel, dim3(a.B * a.n_heads), dim3(128), row_smem, s, 1, a));
        return Q3_OK;
    }
    Q3_TRY_LAUNCH(launch(attn_stats_kernel<NREP>, dim3(a.B * a.n_kv), dim3(128 * NREP), 0, s, 1, a));
    return Q3_OK;
}

template <int NREP>
int launch_pv_tc(const AttnArgs &a, cudaStream_t s) {
    PvTcPlan pl;
    pl.k_rows_per_seq = (int)(a.kv.seq / a.kv.pos);
    pl.k_rows_per_head = a.kv.head >= a.kv.pos ? (int)(a.kv.head / a.kv.pos) : 0;
    pl.k_cols_per_head = a.kv.head >= a.kv.pos ? 0 : (int)a.kv.head;
    // kind::f16: fp32 accumulate, bf16 A (MN-major) and B (K-major), N = 16, M = 128
    pl.idesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | ((uint32_t)(16 >> 3) << 17) |
               ((uint32_t)(128 >> 4) << 24);
    // rows that share one cache (sequence stride 0: a prompt's rows at consecutive positions) go
    // 16 / NREP to an item, so that one V tile in shared memory serves all of them
    pl.rows = a.kv.seq == 0 && a.B > 1 ? 16 / NREP : 1;
    CUtensorMap mv;
    if (!make_map_strided(&mv, a.vc, cache_map_rows(a), a.kv.pos, a.kv.pos, PV_TILE)) return Q3_ERR_ARG;
    const size_t base = 1024 + (size_t)PV_STAGES * PV_STAGE_BYTES + 256 + (size_t)ITEM_TAB_OFF(a.B) * 4;
    pl.tab_cap = base < SMEM_CTA_MAX ? (int)std::min<size_t>(ITEM_TAB_MAX, (SMEM_CTA_MAX - base) / 8) : 0;
    const size_t smem = base + (size_t)pl.tab_cap * 8;
    const long long max_items =
        (long long)((a.B + pl.rows - 1) / pl.rows) * a.n_kv * ((a.max_seq + a.chunk_b - 1) / a.chunk_b);
    const int grid = (int)std::min<long long>(max_items, num_sms());
    if (pl.rows == 1) {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_tc_kernel<NREP, 1>), smem));
        Q3_TRY_LAUNCH(launch(attn_pv_tc_kernel<NREP, 1>, dim3(grid), dim3(PV_THREADS), smem, s, 1, mv, a, pl));
    } else {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_tc_kernel<NREP, 16 / NREP>), smem));
        Q3_TRY_LAUNCH(launch(attn_pv_tc_kernel<NREP, 16 / NREP>, dim3(grid), dim3(PV_THREADS), smem, s, 1, mv, a, pl));
    }
    return Q3_OK;
}

// The TMA-fed scores need whole 64-dim halves and contiguous per-sequence caches in kv_dim rows;
// the vectorized pv needs an even head_dim that splits 128 threads into groups.
bool split_fast_path(const AttnArgs &a) {
    const KvLayout &kv = a.kv;
    const bool heads_in_row = kv.head < kv.pos;  // reference layout
    return a.head_dim % TMA_BK == 0 && a.head_dim <= 256 && kv.pos > 0 && kv.seq % kv.pos == 0 &&
           (heads_in_row ? kv.head % 8 == 0 : kv.head % kv.pos == 0) && kv.pos % 8 == 0 &&
           128 % (a.head_dim / 2) == 0 &&
           (kv.seq / kv.pos) * (long long)a.B < (1LL << 31);
}

template <int NREP>
int launch_nrep(const AttnArgs &a, int dpt, cudaStream_t s) {
    const int nsm = num_sms();
    const bool split = a.stats != nullptr;
    const size_t prefix_bytes = (size_t)PREFIX_INTS(a.B) * 4;
    if (split && split_fast_path(a)) {
        int st = launch_scores_exact<NREP>(a, s);
        if (st != Q3_OK) return st;
        st = launch_stats<NREP>(a, s);
        if (st != Q3_OK) return st;
        if (a.head_dim == 128 && a.chunk_b % PV_TILE == 0) {  // P.V on the tensor cores
            st = launch_pv_tc<NREP>(a, s);
            if (st != Q3_OK) return st;
            Q3_TRY_LAUNCH(launch(attn_combine_kernel, dim3(a.n_heads, a.B), dim3(128), 0, s, 1, a));
            return Q3_OK;
        }
        const int G = THREADS / (a.head_dim / 2);
        const size_t pv_smem = (size_t)V_STAGES * VT * a.head_dim * 2 + (size_t)V_STAGES * NREP * VT * 4 +
                               (size_t)VT * NREP * 4 + (size_t)G * NREP * a.head_dim * 4 + prefix_bytes;
        const long long max_pv = (long long)a.B * a.n_kv * ((a.max_seq + a.chunk_b - 1) / a.chunk_b);
        const int per_sm_pv = std::max(1, (int)((200 * 1024) / pv_smem));
        const int grid_pv = (int)std::min<long long>(max_pv, (long long)nsm * per_sm_pv);
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_vec_kernel<NREP>), pv_smem));
        Q3_TRY_LAUNCH(launch(attn_pv_vec_kernel<NREP>, dim3(grid_pv), dim3(THREADS), pv_smem, s, 1, a));
        Q3_TRY_LAUNCH(launch(attn_combine_kernel, dim3(a.n_heads, a.B), dim3(128), 0, s, 1, a));
        return Q3_OK;
    }
    // scores
    const size_t sc_smem = (size_t)K_STAGES * a.sc_chunk * (a.head_dim + 8) * 2 + (size_t)NREP * a.head_dim * 4 + prefix_bytes;
    Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_scores_kernel<NREP>), sc_smem));
    const long long max_sc = (long long)a.B * a.n_kv * ((a.max_seq + a.sc_chunk - 1) / a.sc_chunk);
    const int per_sm = std::max(1, (int)((200 * 1024) / sc_smem));
    const int grid_sc = (int)std::min<long long>(max_sc, (long long)nsm * per_sm);
    Q3_TRY_LAUNCH(launch(attn_scores_kernel<NREP>, dim3(grid_sc), dim3(SC_THREADS), sc_smem, s, 1, a));
    // stats
    if (split) {
        const int st = launch_stats<NREP>(a, s);
        if (st != Q3_OK) return st;
    }
    // pv
    const size_t pv_smem = (size_t)V_STAGES * VT * a.head_dim * 2 + (size_t)V_STAGES * NREP * VT * 4 +
                           (size_t)NREP * VT * 4 + prefix_bytes;
    const long long max_pv = (long long)a.B * a.n_kv * ((a.max_seq + a.chunk_b - 1) / a.chunk_b);
    const int per_sm_pv = std::max(1, (int)((200 * 1024) / pv_smem));
    const int grid_pv = (int)std::min<long long>(max_pv, (long long)nsm * per_sm_pv);
    if (dpt == 1) {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_kernel<NREP, 1>), pv_smem));
        Q3_TRY_LAUNCH(launch(attn_pv_kernel<NREP, 1>, dim3(grid_pv), dim3(THREADS), pv_smem, s, 1, a));
    } else {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(attn_pv_kernel<NREP, 2>), pv_smem));
        Q3_TRY_LAUNCH(launch(attn_pv_kernel<NREP, 2>, dim3(grid_pv), dim3(THREADS), pv_smem, s, 1, a));
    }
    // combine
    if (split) Q3_TRY_LAUNCH(launch(attn_combine_kernel, dim3(a.n_heads, a.B), dim3(128), 0, s, 1, a));
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

// Attention over n_rows sequences. `scores` has rows of `ld` floats per (sequence, head). Exact
// mode when split == nullptr; otherwise `split` holds the split-mode scratch (stats, partial,
// chunk_b, max_chunks; the counters are unused).
int attention(bf16 *out, const bf16 *q, const bf16 *key_cache, const bf16 *value_cache, float *scores, int ld,
              const int *pos, int n_rows, long long q_stride, KvLayout kv, int n_heads, int n_kv_heads,
              int head_dim, int max_seq, float scale, const AttnSplit *split, cudaStream_t s) {
    if (!out || !q || !key_cache || !value_cache || !scores || !pos) return Q3_ERR_ARG;
    int st = attention_check(n_heads, n_kv_heads, head_dim, max_seq, n_rows);
    if (st != Q3_OK) return st;
    if (ld < max_seq || kv.pos <= 0 || kv.seq < 0 || kv.head < 0) return Q3_ERR_SHAPE;
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!al(key_cache) || !al(value_cache) || kv.seq % 8 || kv.pos % 8 || kv.head % 8) return Q3_ERR_ALIGN;
    AttnArgs a = {};
    a.q = q;
    a.kc = key_cache;
    a.vc = value_cache;
    a.out = out;
    a.scores = scores;
    a.ld = ld;
    a.pos = pos;
    a.q_stride = q_stride;
    a.kv = kv;
    a.B = n_rows;
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.head_dim = head_dim;
    a.kv_dim = n_kv_heads * head_dim;
    a.max_seq = max_seq;
    a.scale = scale;
    a.chunk_b = max_seq;  // exact mode: one chunk spans every position
    a.sc_chunk = head_dim <= 128 ? SC_CHUNK : SC_CHUNK / 2;  // K ring within shared memory
    if (split) {
        if (!split->stats || !split->partial) return Q3_ERR_ARG;
        if (split->chunk_b <= 0 || (long long)split->chunk_b * split->max_chunks < max_seq) return Q3_ERR_SHAPE;
        a.stats = split->stats;
        a.partial = split->partial;
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
