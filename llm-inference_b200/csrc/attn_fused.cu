// Decode attention for a few sequences, with the query/key RMSNorm, RoPE and the KV-cache write of
// the new position folded into the same launch: src/kernels.cu:301-403 (qk_norm_rope) followed by
// :439-497 (attention), for batch sizes where the split-KV path (attention.cu) has too few work
// items per kernel to keep 148 SMs busy and its four launches cost more than their bytes.
//
// Grid: one thread-block cluster per (sequence b, kv head), one CTA of the cluster per chunk of
// the positions 0..pos[b] (C chunks of ceil(len / C) positions). The CTAs of a cluster exchange
// what the softmax needs through distributed shared memory (DSMEM) and meet at hardware cluster
// barriers; nothing goes through global memory except the cache rows and the output. Every CTA
//   1. stages its chunk's K and V rows in tiles of 128 positions with TMA (K in 64-column boxes
//      with the 128-byte swizzle, so that one thread per position reads its row without bank
//      conflicts; V unswizzled), issued before the RMSNorm so that they stream meanwhile;
//   2. recomputes the group's query heads and key head from the raw projections: per-head RMSNorm
//      in the reference's order (xor tree per warp, warp sums in order), bf16 rounding, RoPE with
//      bf16 cos/sin and the reference's per-product rounding. The CTA holding position pos[b]
//      writes the new key and value rows to the caches and uses them from shared memory (the
//      cache row of pos[b] is never read in this launch);
//   3. computes the scores of its chunk exactly as the reference does -- one thread per position,
//      a serial fused multiply-add chain over head_dim, round(round(dot) * scale) -- into its
//      shared memory, with the chunk's maximum per head;
//   4. (cluster barrier) takes the maximum over the chunk maxima, read from the other CTAs'
//      shared memory (exact: max does not depend on order), and replaces its scores by
//      e = expf(s - max);
//   5. (cluster barrier) sums e over all positions in the reference's order -- 128 slots, slot j
//      taking positions j, j + 128, ... serially, an xor tree per warp, the four warp totals in
//      order -- so that p = round_bf16(e / sum) is the reference's probability bit for bit. The
//      NREP * 128 (head, slot) chains are shared out over the cluster's CTAs, one thread each,
//      reading each position's e from the CTA that holds it; (cluster barrier) every CTA then
//      gathers the chain sums and finishes the tree itself;
//   6. accumulates p * v over its chunk in position order (one fused multiply-add chain per
//      output element) into its shared memory;
//   7. (cluster barrier) adds the C chunk partials of its slice of the outputs in chunk order and
//      writes them as bf16; a last cluster barrier keeps every CTA's shared memory alive until the
//      others have read it.
// With one chunk the result is the reference's single chain, bit for bit; with C chunks only the
// fp32 order of the P.V sum differs (C partial chains added in order).
#include <math.h>

#include <algorithm>
#include <mutex>

#include <cooperative_groups.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int FA_THREADS = 256;
constexpr int FA_TILE = 128;  // positions per staged K / V tile
constexpr int FA_STAGES = 2;
constexpr int FA_MAX_CLUSTER = 16;  // chunks per (sequence, kv head): CTAs of one cluster

struct FusedArgs {
    const bf16 *q, *k, *v;            // raw projections: sequence b at q + b*q_stride, k/v + b*kv_stride
    const bf16 *q_norm_w, *k_norm_w;  // [head_dim]
    bf16 *kc, *vc;                    // row (b, t, kv head h) at kc + b*kv.seq + t*kv.pos + h*kv.head
    bf16 *out;                        // like q
    const int *pos;                   // [B]
    KvLayout kv;
    long long q_stride, kv_stride;
    int n_heads, n_kv, max_seq, C;
    int cap;                          // positions of the longest chunk, rounded up to 4
    // the tensor maps view a cache as [rows, kv.pos] rows: (b, kv head h, position t) is row
    // b*rows_per_seq + h*rows_per_head + t, columns from h*cols_per_head
    int rows_per_seq, rows_per_head, cols_per_head;
    float eps, theta, scale;
};

template <int NREP, int HD>
__global__ void __launch_bounds__(FA_THREADS, 1)
    attn_fused_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ FusedArgs a) {
    constexpr int HALVES = HD / 64;             // 64-column (128-byte) swizzled boxes per K row
    constexpr int KTILE_BYTES = FA_TILE * HD * 2;
    constexpr int VTILE_BYTES = FA_TILE * HD * 2;
    constexpr int CPR = HD / 8;                 // 16-byte chunks per row
    constexpr int HG = FA_THREADS / FA_TILE;    // head groups in the scores and sum phases (2)
    constexpr int HPT = (NREP + HG - 1) / HG;   // heads per thread there
    constexpr int PV_HG = FA_THREADS / HD;      // head groups in the P.V phase
    constexpr int PV_HPT = (NREP + PV_HG - 1) / PV_HG;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base: the K boxes use the 128-byte swizzle
    unsigned char *smem = align_shared<1024>(smem_raw);
    unsigned char *ks = smem;                                                   // [FA_STAGES][HALVES][FA_TILE][64], swizzled
    bf16 *vs = reinterpret_cast<bf16 *>(smem + FA_STAGES * KTILE_BYTES);       // [FA_STAGES][FA_TILE][HD]
    float *qf = reinterpret_cast<float *>(smem + FA_STAGES * (KTILE_BYTES + VTILE_BYTES));  // [NREP][HD] roped queries
    float *part = qf + NREP * HD;                                             // [NREP][HD] this chunk's P.V
    float *cmx = part + NREP * HD;                                            // [16] this chunk's maxima
    bf16 *yh = reinterpret_cast<bf16 *>(cmx + 16);                            // [NREP + 1][HD] normed heads
    bf16 *knew = yh + (NREP + 1) * HD;                                        // [HD] key row of position pos
    bf16 *vnew = knew + HD;                                                   // [HD] value row of position pos
    uint64_t *bars = reinterpret_cast<uint64_t *>(vnew + HD);                 // kfull[2], vfull[2]
    float *ex = reinterpret_cast<float *>(bars + 2 * FA_STAGES);             // [NREP][cap] scores, then e
    float *pr = ex + NREP * a.cap;                                            // [NREP][cap] probabilities
    __shared__ float red[NREP + 1][HD / 32];
    __shared__ float wred[NREP][FA_TILE / 32];
    __shared__ float cm_s[FA_MAX_CLUSTER * NREP];
    __shared__ float gmax_s[NREP], gsum_s[NREP];
    __shared__ float chs[NREP * FA_TILE];  // sums of the chains this CTA computes (per_cta <= NREP * 128)
    // RoPE: each pair's inverse frequency, then its rounded cos and sin at this position. The
    // reference computes them per head (src/kernels.cu:359-365); the NREP + 1 heads of the group
    // share one computation here (the values are the same), the frequencies before the
    // programmatic-dependency wait.
    constexpr int HALF = HD / 2;
    __shared__ float rope_f[HALF], rope_c[HALF], rope_s[HALF];

    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid % 32;
    const int C = a.C, c = (int)cluster.block_rank();  // the cluster's CTAs are consecutive blocks
    const int g = blockIdx.x / C;
    const int b = g / a.n_kv, kvh = g % a.n_kv;

    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 2 * FA_STAGES; i++) mbar_init(&bars[i], 1);
        fence_barrier_init();
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    for (int j = tid; j < HALF; j += FA_THREADS) rope_f[j] = 1.0f / powf(a.theta, (float)(2 * j) / HD);
    __syncthreads();
    pdl_trigger();  // no CTA here waits for another grid's CTAs: successors may be scheduled early
    pdl_wait();

    // the raw projections and the position, loaded together
    const bf16 *qg = a.q + (size_t)b * a.q_stride + (size_t)kvh * NREP * HD;
    const bf16 *kg = a.k + (size_t)b * a.kv_stride + (size_t)kvh * HD;
    constexpr int NE = (NREP + 1) * HD;
    constexpr int EPT = (NE + FA_THREADS - 1) / FA_THREADS;
    float xv[EPT];
#pragma unroll
    for (int j = 0; j < EPT; j++) {
        const int e = tid + j * FA_THREADS;
        xv[j] = e < NE ? __bfloat162float(e < NREP * HD ? qg[e] : kg[e - NREP * HD]) : 0.0f;
    }
    const int p = a.pos[b];
    if (p < 0 || p >= a.max_seq) {  // every CTA of the cluster leaves here, before any cluster barrier
        if (c == 0 && tid == 0) atomicOr(&g_dev_error, DEV_ERR_POS_RANGE);
        return;
    }
    const int len = p + 1;
    for (int j = tid; j < HALF; j += FA_THREADS) {  // ordered before the RoPE by the norm's barriers
        const float angle = p * rope_f[j];
        rope_c[j] = round_bf16(cosf(angle));
        rope_s[j] = round_bf16(sinf(angle));
    }
    const int CH = (len + C - 1) / C;  // positions per chunk (<= cap)
    const int t0 = min(len, c * CH), t1 = min(len, t0 + CH);
    const int n_own = t1 - t0;
    const int n_tiles = (n_own + FA_TILE - 1) / FA_TILE;
    const bool mine_p = c == (len - 1) / CH;  // this CTA's chunk holds position p
    if (mine_p)
        for (int i = tid; i < HD; i += FA_THREADS) vnew[i] = a.v[(size_t)b * a.kv_stride + (size_t)kvh * HD + i];
    // rows of this (sequence, kv head) in the maps' [rows, cols] view of a cache
    const int row0 = b * a.rows_per_seq + kvh * a.rows_per_head;
    const int col0 = kvh * a.cols_per_head;
    const uint64_t pol = policy_evict_first();  // cache rows are read once per step

    // Tile i: FA_TILE rows from position t0 + i * FA_TILE (rows past the chunk are loaded and not
    // used; position p is not taken from the cache). One thread issues.
    auto issue = [&](bool is_v, int i) {
        const int st = i % FA_STAGES;
        const int y = row0 + t0 + i * FA_TILE;
        if (!is_v) {
            mbar_arrive_expect_tx(&bars[st], KTILE_BYTES);
#pragma unroll
            for (int h = 0; h < HALVES; h++)
                tma_load_2d_stream(ks + st * KTILE_BYTES + h * FA_TILE * 128, &tmK, col0 + h * 64, y, &bars[st], pol);
        } else {
            mbar_arrive_expect_tx(&bars[FA_STAGES + st], VTILE_BYTES);
            tma_load_2d_stream(reinterpret_cast<unsigned char *>(vs) + st * VTILE_BYTES, &tmV, col0, y,
                               &bars[FA_STAGES + st], pol);
        }
    };
    auto wait_tile = [&](bool is_v, int i) {
        return mbar_wait(&bars[(is_v ? FA_STAGES : 0) + i % FA_STAGES], (i / FA_STAGES) & 1, &g_dev_error);
    };
    if (tid == 0) {
        for (int i = 0; i < min(FA_STAGES, n_tiles); i++) issue(false, i);
        for (int i = 0; i < min(FA_STAGES, n_tiles); i++) issue(true, i);
    }

    // ---- 2. RMSNorm of the group's NREP query heads and its key head (src/kernels.cu:301-347)
#pragma unroll
    for (int j = 0; j < EPT; j++) {
        const int e = tid + j * FA_THREADS;
        if (e < NE) {  // uniform across a warp: NE and FA_THREADS are multiples of 32
            float sq = xv[j] * xv[j];
            for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
            if (lane == 0) red[e / HD][(e % HD) / 32] = sq;
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < EPT; j++) {
        const int e = tid + j * FA_THREADS;
        if (e < NE) {
            const int hh = e / HD, i = e % HD;
            float total = 0.0f;
#pragma unroll
            for (int w = 0; w < HD / 32; w++) total += red[hh][w];
            const float inv_rms = rsqrtf(total / HD + a.eps);
            const bf16 normed = __float2bfloat16(xv[j] * inv_rms);
            const bf16 *nw = hh < NREP ? a.q_norm_w : a.k_norm_w;
            yh[e] = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(nw[i]));
        }
    }
    __syncthreads();
    // RoPE at position p (src/kernels.cu:349-390): pairs (j, j + HD/2)
    for (int e = tid; e < (NREP + 1) * HALF; e += FA_THREADS) {
        const int hh = e / HALF, j = e % HALF;
        const float cs = rope_c[j], sn = rope_s[j];
        const float av = __bfloat162float(yh[hh * HD + j]);
        const float bv = __bfloat162float(yh[hh * HD + j + HALF]);
        const bf16 out_a = __float2bfloat16(round_bf16(av * cs) - round_bf16(bv * sn));
        const bf16 out_b = __float2bfloat16(round_bf16(bv * cs) + round_bf16(av * sn));
        if (hh < NREP) {
            qf[hh * HD + j] = __bfloat162float(out_a);
            qf[hh * HD + j + HALF] = __bfloat162float(out_b);
        } else {
            knew[j] = out_a;
            knew[j + HALF] = out_b;
        }
    }
    __syncthreads();
    if (mine_p) {  // the new cache rows (src/kernels.cu:383-390)
        const size_t slot = (size_t)b * a.kv.seq + (size_t)p * a.kv.pos + (size_t)kvh * a.kv.head;
        for (int i = tid; i < HD; i += FA_THREADS) {
            a.kc[slot + i] = knew[i];
            a.vc[slot + i] = vnew[i];
        }
    }

    // ---- 3. scores of this chunk (src/kernels.cu:456-465): thread (r, head group hgp)
    const int r = tid % FA_TILE, hgp = tid / FA_TILE;
    float cm[HPT];
#pragma unroll
    for (int k = 0; k < HPT; k++) cm[k] = -INFINITY;
    bool ok = true;  // uniform over the block
    for (int i = 0; i < n_tiles; i++) {
        if (!__syncthreads_and(wait_tile(false, i))) ok = false;
        const int t = t0 + i * FA_TILE + r;
        if (ok && t < t1) {
            const bool newest = t == p;
            const unsigned char *kt = ks + (i % FA_STAGES) * KTILE_BYTES + r * 128;
            float acc[HPT];
#pragma unroll
            for (int k = 0; k < HPT; k++) acc[k] = 0.0f;
#pragma unroll
            for (int ch = 0; ch < CPR; ch++) {
                // 128-byte swizzle: chunk ch of row r sits at chunk (ch % 8) ^ (r % 8) of its box row
                const bf16x8 kv8 = newest ? lds128(knew + ch * 8)
                                          : lds128(kt + (ch / 8) * FA_TILE * 128 + (((ch % 8) ^ (r % 8)) << 4));
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f = __bfloat1622float2(kv8.h[e]);
#pragma unroll
                    for (int k = 0; k < HPT; k++) {
                        const int h = hgp + HG * k;
                        if (h < NREP) {
                            const float *qh = qf + h * HD + ch * 8 + 2 * e;
                            acc[k] = __fmaf_rn(qh[0], f.x, acc[k]);
                            acc[k] = __fmaf_rn(qh[1], f.y, acc[k]);
                        }
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < HPT; k++) {
                const int h = hgp + HG * k;
                if (h < NREP) {
                    const float sc = round_bf16(round_bf16(acc[k]) * a.scale);
                    ex[h * a.cap + (t - t0)] = sc;
                    cm[k] = fmaxf(cm[k], sc);
                }
            }
        }
        __syncthreads();  // stage i % FA_STAGES is free
        if (tid == 0 && i + FA_STAGES < n_tiles) issue(false, i + FA_STAGES);
    }
    // chunk maxima per head: xor tree per warp (all lanes of a warp share hgp), then the warps of hgp
#pragma unroll
    for (int k = 0; k < HPT; k++) {
        const int h = hgp + HG * k;
        float m = cm[k];
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (h < NREP && lane == 0) wred[h][r / 32] = m;
    }
    __syncthreads();
    if (tid < NREP) {
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < FA_TILE / 32; w++) m = fmaxf(m, wred[tid][w]);
        cmx[tid] = m;
    }

    // ---- 4. the maximum over the chunks (src/kernels.cu:467-468, block_max :422-436): exact in any
    // order; then e = expf(s - max) for this chunk, in place
    cluster.sync();
    if (tid < C * NREP) cm_s[tid] = *cluster.map_shared_rank(cmx + tid % NREP, tid / NREP);
    __syncthreads();
    if (tid < NREP) {
        float m = -INFINITY;
        for (int cc = 0; cc < C; cc++) m = fmaxf(m, cm_s[cc * NREP + tid]);
        gmax_s[tid] = m;
    }
    __syncthreads();
    for (int e = tid; e < NREP * n_own; e += FA_THREADS) {
        const int h = e / n_own, i = e - h * n_own;
        ex[h * a.cap + i] = expf(ex[h * a.cap + i] - gmax_s[h]);
    }

    // ---- 5. the sum of e in the reference's order (src/kernels.cu:469-470, block_sum :406-420).
    // Each (head, slot) chain -- slot j adding positions j, j + 128, ... serially -- is computed by
    // one thread of one CTA of the cluster (chain i by CTA i / per_cta), which reads each position's
    // e from the CTA holding it, SB values in flight at once; after a cluster barrier every CTA
    // gathers the 128 chain sums of each head and runs the xor tree and the warp totals in order.
    cluster.sync();
    {
        // tpc lanes of one warp share a chain: lane q loads its elements m = q, q + tpc, ...
        // (position slot + 128 m), all of a batch in flight at once, and the chain is folded in
        // order m = 0, 1, 2, ... through shuffles
        constexpr int SB = 8;
        const int n_chains = NREP * FA_TILE;
        const int per_cta = (n_chains + C - 1) / C;
        int tpc = 1;
        while (tpc < 32 && 2 * tpc * per_cta <= FA_THREADS) tpc *= 2;
        const int cpi = FA_THREADS / tpc;           // chains per pass of the block
        const int m_max = (len + FA_TILE - 1) / FA_TILE;  // elements of the longest chain (slot 0)
        const int q = lane % tpc, lane0 = lane - q;
        for (int i0 = 0; i0 < per_cta; i0 += cpi) {
            const int i = i0 + tid / tpc;
            const int chain = c * per_cta + i;
            const bool valid = i < per_cta && chain < n_chains;
            const int h = valid ? chain / FA_TILE : 0, slot = valid ? chain % FA_TILE : 0;
            const int m_end = valid && slot < len ? (len - 1 - slot) / FA_TILE + 1 : 0;  // this chain's elements
            float sum = 0.0f;
            for (int mb = 0; mb < m_max; mb += SB * tpc) {  // uniform over the block
                float vals[SB];
#pragma unroll
                for (int j = 0; j < SB; j++) {
                    const int m = mb + j * tpc + q;
                    float x = 0.0f;
                    if (m < m_end) {
                        const int t = slot + m * FA_TILE, owner = t / CH;
                        x = cluster.map_shared_rank(ex, owner)[h * a.cap + (t - owner * CH)];
                    }
                    vals[j] = x;
                }
#pragma unroll
                for (int j = 0; j < SB; j++)
                    for (int r = 0; r < tpc; r++) {
                        const float x = __shfl_sync(0xffffffffu, vals[j], lane0 + r);
                        if (mb + j * tpc + r < m_end) sum += x;
                    }
            }
            if (valid && q == 0) chs[i] = sum;
        }
    }
    cluster.sync();
    {
        const int slot = tid % FA_TILE;
        const int per_cta = (NREP * FA_TILE + C - 1) / C;
#pragma unroll
        for (int k = 0; k < HPT; k++) {
            const int h = hgp + HG * k;
            const int chain = (h < NREP ? h : 0) * FA_TILE + slot;
            float x = h < NREP ? *cluster.map_shared_rank(chs + chain % per_cta, chain / per_cta) : 0.0f;
            for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
            if (h < NREP && lane == 0) wred[h][slot / 32] = x;
        }
        __syncthreads();
        if (tid < NREP) {
            float x = 0.0f;
#pragma unroll
            for (int w = 0; w < FA_TILE / 32; w++) x += wred[tid][w];
            gsum_s[tid] = x;
        }
        __syncthreads();
        // probabilities of this chunk (src/kernels.cu:472-474)
        for (int e = tid; e < NREP * n_own; e += FA_THREADS) {
            const int h = e / n_own, i = e - h * n_own;
            pr[h * a.cap + i] = round_bf16(ex[h * a.cap + i] / gsum_s[h]);
        }
        __syncthreads();
    }

    // ---- 6. P.V over this chunk (src/kernels.cu:476-485), thread (d, head group)
    const int d = tid % HD, phg = tid / HD;
    float acc[PV_HPT];
#pragma unroll
    for (int k = 0; k < PV_HPT; k++) acc[k] = 0.0f;
    for (int i = 0; i < n_tiles; i++) {
        if (!__syncthreads_and(wait_tile(true, i))) ok = false;
        const int r0 = t0 + i * FA_TILE;
        const int rows = min(FA_TILE, t1 - r0);
        const float *pt = pr + (r0 - t0);  // head h's probabilities of this tile at pt[h * cap + rr]
        if (ok) {
            const bf16 *vt = vs + (i % FA_STAGES) * (VTILE_BYTES / 2);
            const int rows_c = (r0 + rows == len) ? rows - 1 : rows;  // rows from the cache
#pragma unroll 4
            for (int rr = 0; rr < rows_c; rr++) {
                const float vv = __bfloat162float(vt[rr * HD + d]);
#pragma unroll
                for (int k = 0; k < PV_HPT; k++) {
                    const int h = phg + PV_HG * k;
                    if (h < NREP) acc[k] = __fmaf_rn(pt[h * a.cap + rr], vv, acc[k]);
                }
            }
            if (rows_c < rows) {  // position p
                const float vv = __bfloat162float(vnew[d]);
#pragma unroll
                for (int k = 0; k < PV_HPT; k++) {
                    const int h = phg + PV_HG * k;
                    if (h < NREP) acc[k] = __fmaf_rn(pt[h * a.cap + rows_c], vv, acc[k]);
                }
            }
        }
        __syncthreads();  // the stage is refilled next
        if (tid == 0 && i + FA_STAGES < n_tiles) issue(true, i + FA_STAGES);
    }
#pragma unroll
    for (int k = 0; k < PV_HPT; k++) {
        const int h = phg + PV_HG * k;
        if (h < NREP) part[h * HD + d] = ok ? acc[k] : __int_as_float(0x7fc00000);  // NaN marks a failed wait
    }

    // ---- 7. this CTA's slice of the outputs: the chunks' partials added in chunk order
    cluster.sync();
    {
        constexpr int E = NREP * HD;
        const int per = (E + C - 1) / C;
        bf16 *og = a.out + (size_t)b * a.q_stride + (size_t)kvh * NREP * HD;
        for (int e = c * per + tid; e < min(E, (c + 1) * per); e += FA_THREADS) {
            float vals[FA_MAX_CLUSTER];  // every chunk's value in flight at once, then added in order
#pragma unroll
            for (int cc = 0; cc < FA_MAX_CLUSTER; cc++) vals[cc] = cc < C ? *cluster.map_shared_rank(part + e, cc) : 0.0f;
            float o = 0.0f;
#pragma unroll
            for (int cc = 0; cc < FA_MAX_CLUSTER; cc++)
                if (cc < C) o += vals[cc];
            og[e] = __float2bfloat16(o);
        }
    }
    cluster.sync();  // the other CTAs have read this one's shared memory
}

// Dynamic shared memory: alignment slack, K ring (swizzled boxes), V ring, queries, the chunk's P.V
// partial, chunk maxima, normed heads, new K/V rows, mbarriers, and the chunk's e and p values
// (cap positions per head each).
size_t fused_smem_bytes(int nrep, int hd, int cap) {
    return 1024 + (size_t)FA_STAGES * FA_TILE * hd * 2 * 2 + 2 * (size_t)nrep * hd * 4 + 64 +
           (size_t)(nrep + 1) * hd * 2 + 2 * (size_t)hd * 2 + 2 * FA_STAGES * 8 + 2 * (size_t)nrep * cap * 4;
}

int chunk_cap(int max_seq, int chunks) { return ((max_seq + chunks - 1) / chunks + 3) / 4 * 4; }

template <int NREP, int HD>
const void *fused_kernel() {
    return reinterpret_cast<const void *>(attn_fused_kernel<NREP, HD>);
}

const void *fused_kernel_for(int nrep, int hd) {
    if (hd == 128) {
        switch (nrep) {
            case 1: return fused_kernel<1, 128>();
            case 2: return fused_kernel<2, 128>();
            case 4: return fused_kernel<4, 128>();
            case 8: return fused_kernel<8, 128>();
        }
    } else if (hd == 64) {
        switch (nrep) {
            case 1: return fused_kernel<1, 64>();
            case 2: return fused_kernel<2, 64>();
            case 4: return fused_kernel<4, 64>();
            case 8: return fused_kernel<8, 64>();
        }
    }
    return nullptr;
}

// Clusters of C CTAs (with `smem` bytes of dynamic shared memory each) that the current device
// holds at once, or 0 when one does not fit. The answer is kept per device, kernel and shape.
int fused_clusters(const void *k, int C, size_t smem) {
    struct Entry {
        const void *k;
        int dev, C;
        size_t smem;
        int n;
    };
    static Entry cache[64];
    static int n_cache = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    for (int i = 0; i < n_cache; i++)
        if (cache[i].k == k && cache[i].dev == dev && cache[i].C == C && cache[i].smem == smem) return cache[i].n;
    int n = 0;
    if (smem <= 227 * 1024 && allow_smem(k, smem) == cudaSuccess &&
        (C <= 8 || cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess)) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(C);
        cfg.blockDim = dim3(FA_THREADS);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = C;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    if (n_cache < 64) cache[n_cache++] = {k, dev, C, smem, n};
    return n;
}

template <int NREP, int HD>
cudaError_t launch_fused(const CUtensorMap &mk, const CUtensorMap &mv, const FusedArgs &a, int groups, size_t smem,
                         cudaStream_t s) {
    return launch(attn_fused_kernel<NREP, HD>, dim3(groups * a.C), dim3(FA_THREADS), smem, s, a.C, mk, mv, a);
}

}  // namespace

unsigned take_error_attn_fused() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

// Chunks (CTAs per cluster) per (sequence, kv head) for `batch` sequences of up to max_seq
// positions: the largest size up to 16 whose clusters all fit on the device at once, or 0 when the
// fused kernel does not apply (head_dim other than 64 / 128, group size other than 1, 2, 4, 8, or
// too many sequences for clusters of two: the split-KV path is the better fit there).
int fused_chunks(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq) {
    if (batch <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || max_seq <= 0) return 0;
    const int nrep = n_heads / n_kv_heads;
    const void *k = fused_kernel_for(nrep, head_dim);
    if (!k) return 0;
    const long long groups = (long long)batch * n_kv_heads;
    for (int C = FA_MAX_CLUSTER; C >= 2; C--)
        if (fused_clusters(k, C, fused_smem_bytes(nrep, head_dim, chunk_cap(max_seq, C))) >= groups) return C;
    return 0;
}

int attention_fused(bf16 *out, const bf16 *q, const bf16 *k, const bf16 *v, const bf16 *q_norm_w,
                    const bf16 *k_norm_w, bf16 *key_cache, bf16 *value_cache, KvLayout kv, const int *pos, int batch,
                    long long q_stride, long long kv_stride, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                    float eps, float theta, float scale, int chunks, cudaStream_t s) {
    if (!out || !q || !k || !v || !q_norm_w || !k_norm_w || !key_cache || !value_cache || !pos) return Q3_ERR_ARG;
    if (batch <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || max_seq <= 0) return Q3_ERR_SHAPE;
    const int nrep = n_heads / n_kv_heads;
    const void *kern = fused_kernel_for(nrep, head_dim);
    if (!kern) return Q3_ERR_SHAPE;
    if (chunks < 1 || chunks > FA_MAX_CLUSTER) return Q3_ERR_SHAPE;
    const int cap = chunk_cap(max_seq, chunks);
    const size_t smem = fused_smem_bytes(nrep, head_dim, cap);
    // one cluster must fit on the device (its chunks' scores in shared memory included)
    if (fused_clusters(kern, chunks, smem) < 1) return Q3_ERR_SHAPE;
    if ((long long)batch * n_kv_heads * chunks >= (1ll << 31)) return Q3_ERR_SHAPE;
    if (kv.pos <= 0 || kv.seq < 0 || kv.head < 0 || q_stride < (long long)n_heads * head_dim ||
        kv_stride < (long long)n_kv_heads * head_dim)
        return Q3_ERR_SHAPE;
    // rows of one sequence must not overlap those of another: each launch writes one row per
    // sequence that other sequences' CTAs would otherwise read
    if (batch > 1 && kv.seq == 0) return Q3_ERR_SHAPE;
    auto al = [](const void *p_) { return (reinterpret_cast<uintptr_t>(p_) & 15) == 0; };
    if (!al(key_cache) || !al(value_cache) || kv.seq % 8 || kv.pos % 8 || kv.head % 8) return Q3_ERR_ALIGN;
    // the caches as [rows, kv.pos] matrices for the tensor maps: a sequence's rows, and a head's
    // rows (head-major) or columns (position-major), must be whole rows of that view
    if (kv.seq % kv.pos) return Q3_ERR_SHAPE;
    const bool head_rows = kv.head >= kv.pos;
    if (head_rows ? kv.head % kv.pos != 0 : (long long)(n_kv_heads - 1) * kv.head + head_dim > kv.pos)
        return Q3_ERR_SHAPE;
    long long map_rows;
    if (kv.seq > 0) map_rows = (long long)batch * (kv.seq / kv.pos);
    else map_rows = head_rows ? (long long)n_kv_heads * (kv.head / kv.pos) : max_seq;
    if (map_rows >= (1ll << 31)) return Q3_ERR_SHAPE;
    FusedArgs a = {};
    a.q = q;
    a.k = k;
    a.v = v;
    a.q_norm_w = q_norm_w;
    a.k_norm_w = k_norm_w;
    a.kc = key_cache;
    a.vc = value_cache;
    a.out = out;
    a.pos = pos;
    a.kv = kv;
    a.q_stride = q_stride;
    a.kv_stride = kv_stride;
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.max_seq = max_seq;
    a.C = chunks;
    a.cap = cap;
    a.rows_per_seq = (int)(kv.seq / kv.pos);
    a.rows_per_head = head_rows ? (int)(kv.head / kv.pos) : 0;
    a.cols_per_head = head_rows ? 0 : (int)kv.head;
    a.eps = eps;
    a.theta = theta;
    a.scale = scale;
    CUtensorMap mk, mv;
    if (!make_map_strided(&mk, key_cache, map_rows, kv.pos, kv.pos, FA_TILE) ||
        !make_map_plain(&mv, value_cache, map_rows, kv.pos, kv.pos, FA_TILE, head_dim))
        return Q3_ERR_ARG;
    const int groups = batch * n_kv_heads;
    cudaError_t e;
    if (head_dim == 128) {
        switch (nrep) {
            case 1: e = launch_fused<1, 128>(mk, mv, a, groups, smem, s); break;
            case 2: e = launch_fused<2, 128>(mk, mv, a, groups, smem, s); break;
            case 4: e = launch_fused<4, 128>(mk, mv, a, groups, smem, s); break;
            default: e = launch_fused<8, 128>(mk, mv, a, groups, smem, s); break;
        }
    } else {
        switch (nrep) {
            case 1: e = launch_fused<1, 64>(mk, mv, a, groups, smem, s); break;
            case 2: e = launch_fused<2, 64>(mk, mv, a, groups, smem, s); break;
            case 4: e = launch_fused<4, 64>(mk, mv, a, groups, smem, s); break;
            default: e = launch_fused<8, 64>(mk, mv, a, groups, smem, s); break;
        }
    }
    Q3_TRY_LAUNCH(e);
    return Q3_OK;
}

}  // namespace q3
