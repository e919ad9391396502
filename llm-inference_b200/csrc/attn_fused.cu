// Decode attention for a few sequences, with the query/key RMSNorm, RoPE and the KV-cache write of
// the new position folded into the same launch: src/kernels.cu:301-403 (qk_norm_rope) followed by
// :439-497 (attention), for batch sizes where the split-KV path (attention.cu) has too few work
// items per kernel to keep 148 SMs busy and its four launches cost more than their bytes.
//
// Grid: one CTA per (sequence b, kv head, chunk c of the positions 0..pos[b]); the C chunks of a
// (sequence, kv head) group are contiguous position ranges of near-equal length. Every CTA
//   1. stages its chunk's K and V rows in tiles of 128 positions with TMA (K in 64-column boxes
//      with the 128-byte swizzle, so that one thread per position reads its row without bank
//      conflicts; V unswizzled), issued before the RMSNorm so that they stream meanwhile;
//   2. recomputes the group's query heads and key head from the raw projections: per-head RMSNorm
//      in the reference's order (xor tree per warp, warp sums in order), bf16 rounding, RoPE with
//      bf16 cos/sin and the reference's per-product rounding. The CTA of the last chunk writes the
//      new key and value rows to the caches; position pos[b] itself is never read from the cache
//      in this launch, every CTA holds its own copy of it;
//   3. computes the scores of its chunk exactly as the reference does -- one thread per position,
//      a serial fused multiply-add chain over head_dim, round(round(dot) * scale) -- writes them
//      out, keeps its own in shared memory and publishes the chunk's maximum per head;
//   4. meets the other CTAs of its group at a barrier (a counter and a generation word in global
//      memory; the wait is bounded by %globaltimer and sets DEV_ERR_WAIT_TIMEOUT when it gives up);
//   5. takes the maximum over the chunk maxima (exact: max does not depend on order) and sums
//      expf(s - max) over all positions in the reference's order (128 slots, slot j taking
//      positions j, j + 128, ... serially, an xor tree per warp, the four warp totals in order),
//      so that p = round_bf16(expf(s - max) / sum) is the reference's probability bit for bit;
//   6. accumulates p * v over its chunk in position order (one fused multiply-add chain per
//      output element) and stores the fp32 partial; the last CTA of the group to finish adds
//      the C partials in chunk order and writes the bf16 output.
// With one chunk the result is the reference's single chain, bit for bit; with C chunks only the
// fp32 order of the P.V sum differs (C partial chains added in order).
//
// Co-residency: the barrier needs every CTA of a group resident at once. The grid never exceeds
// the SMs times the CTAs that fit on one, the wait starts only after griddepcontrol.wait (every
// earlier kernel has finished and left the SMs), and the successor kernel is allowed to launch
// (griddepcontrol.launch_dependents) only after the barrier, so it cannot take the SMs of a CTA of
// this grid that is still waiting to be scheduled.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "tc_common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int FA_THREADS = 256;
constexpr int FA_TILE = 128;  // positions per staged K / V tile
constexpr int FA_STAGES = 2;
constexpr int FA_MAX_CHUNKS = 32;

struct FusedArgs {
    const bf16 *q, *k, *v;            // raw projections: sequence b at q + b*q_stride, k/v + b*kv_stride
    const bf16 *q_norm_w, *k_norm_w;  // [head_dim]
    bf16 *kc, *vc;                    // row (b, t, kv head h) at kc + b*kv.seq + t*kv.pos + h*kv.head
    bf16 *out;                        // like q
    const int *pos;                   // [B]
    float *scores;                    // [B][n_heads][ld]
    float *cmax;                      // [groups][C][NREP] chunk maxima
    float *partial;                   // [groups][C][NREP][head_dim]
    unsigned *ctr;                    // [groups][4]: arrivals, generation, finished chunks (zero at rest)
    KvLayout kv;
    long long q_stride, kv_stride;
    int ld, n_heads, n_kv, max_seq, C;
    int cap;                          // positions of the longest chunk, rounded up to 4
    // the tensor maps view a cache as [rows, kv.pos] rows: (b, kv head h, position t) is row
    // b*rows_per_seq + h*rows_per_head + t, columns from h*cols_per_head
    int rows_per_seq, rows_per_head, cols_per_head;
    float eps, theta, scale;
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void red_add_release(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Barrier of the C CTAs of one group, called by one thread of each after a __syncthreads (the
// release of the arrival covers the stores the CTA's threads made before it). Returns false after
// a timeout.
__device__ bool group_barrier(unsigned *ctr, unsigned n) {
    const unsigned my = ld_acquire(ctr + 1);
    if (atom_add_acq_rel(ctr, 1u) == n - 1) {
        atomicExch(ctr, 0u);  // ordered before the release below
        red_add_release(ctr + 1, 1u);
        return true;
    }
    const uint64_t t0 = globaltimer();
    while (ld_acquire(ctr + 1) == my) {
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(&g_dev_error, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

template <int NREP, int HD>
__global__ void __launch_bounds__(FA_THREADS, 1)
    attn_fused_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ FusedArgs a) {
    constexpr int HALVES = HD / 64;             // 64-column (128-byte) swizzled boxes per K row
    constexpr int KTILE_BYTES = FA_TILE * HD * 2;
    constexpr int VTILE_BYTES = FA_TILE * HD * 2;
    constexpr int CPR = HD / 8;                 // 16-byte chunks per row
    constexpr int HG = FA_THREADS / FA_TILE;    // head groups in the scores phase (2)
    constexpr int HPT = (NREP + HG - 1) / HG;   // heads per thread there
    constexpr int PV_HG = FA_THREADS / HD;      // head groups in the P.V phase
    constexpr int PV_HPT = (NREP + PV_HG - 1) / PV_HG;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base: the K boxes use the 128-byte swizzle
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *ks = smem;                                                   // [FA_STAGES][HALVES][FA_TILE][64], swizzled
    bf16 *vs = reinterpret_cast<bf16 *>(smem + FA_STAGES * KTILE_BYTES);       // [FA_STAGES][FA_TILE][HD]
    float *qf = reinterpret_cast<float *>(smem + FA_STAGES * (KTILE_BYTES + VTILE_BYTES));  // [NREP][HD] roped queries
    bf16 *yh = reinterpret_cast<bf16 *>(qf + NREP * HD);                      // [NREP + 1][HD] normed heads
    bf16 *knew = yh + (NREP + 1) * HD;                                        // [HD] key row of position pos
    bf16 *vnew = knew + HD;                                                   // [HD] value row of position pos
    uint64_t *bars = reinterpret_cast<uint64_t *>(vnew + HD);                 // kfull[2], vfull[2]
    float *pown = reinterpret_cast<float *>(bars + 2 * FA_STAGES);           // [NREP][cap] own scores, then p
    __shared__ float red[NREP + 1][HD / 32];
    __shared__ float wred[NREP][FA_TILE / 32];
    __shared__ float cm_s[FA_MAX_CHUNKS * NREP];
    __shared__ float gmax_s[NREP], gsum_s[NREP];
    __shared__ int flag_s;

    const int tid = threadIdx.x, lane = tid % 32;
    const int g = blockIdx.x / a.C, c = blockIdx.x % a.C;
    const int b = g / a.n_kv, kvh = g % a.n_kv;

    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 2 * FA_STAGES; i++) mbar_init(&bars[i], 1);
        fence_barrier_init();
        flag_s = 0;
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    __syncthreads();
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
    const bool last = c == a.C - 1;  // its chunk ends at position p
    if (last)
        for (int i = tid; i < HD; i += FA_THREADS) vnew[i] = a.v[(size_t)b * a.kv_stride + (size_t)kvh * HD + i];
    if (p < 0 || p >= a.max_seq) {  // every CTA of the group leaves here: no barrier is entered
        if (c == 0 && tid == 0) atomicOr(&g_dev_error, DEV_ERR_POS_RANGE);
        return;
    }
    const int len = p + 1;
    const int t0 = (int)((long long)len * c / a.C), t1 = (int)((long long)len * (c + 1) / a.C);
    const int n_tiles = (t1 - t0 + FA_TILE - 1) / FA_TILE;
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
    constexpr int HALF = HD / 2;
    for (int e = tid; e < (NREP + 1) * HALF; e += FA_THREADS) {
        const int hh = e / HALF, j = e % HALF;
        const float inv_freq = 1.0f / powf(a.theta, (float)(2 * j) / HD);
        const float angle = p * inv_freq;
        const float cs = round_bf16(cosf(angle));
        const float sn = round_bf16(sinf(angle));
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
    if (last) {  // the new cache rows (src/kernels.cu:383-390)
        const size_t slot = (size_t)b * a.kv.seq + (size_t)p * a.kv.pos + (size_t)kvh * a.kv.head;
        for (int i = tid; i < HD; i += FA_THREADS) {
            a.kc[slot + i] = knew[i];
            a.vc[slot + i] = vnew[i];
        }
    }

    // ---- 3. scores of this chunk (src/kernels.cu:456-465): thread (r, head group hgp)
    float *sc_g = a.scores + ((size_t)b * a.n_heads + (size_t)kvh * NREP) * a.ld;
    const int r = tid % FA_TILE, hgp = tid / FA_TILE;
    float cm[HPT];
#pragma unroll
    for (int k = 0; k < HPT; k++) cm[k] = -INFINITY;
    bool ok = true;  // uniform over the block
    for (int i = 0; i < n_tiles; i++) {
        if (!__syncthreads_and(wait_tile(false, i))) ok = false;
        const int t = t0 + i * FA_TILE + r;
        if (ok && t < t1) {
            const bool mine = last && t == p;
            const unsigned char *kt = ks + (i % FA_STAGES) * KTILE_BYTES + r * 128;
            float acc[HPT];
#pragma unroll
            for (int k = 0; k < HPT; k++) acc[k] = 0.0f;
#pragma unroll
            for (int ch = 0; ch < CPR; ch++) {
                // 128-byte swizzle: chunk ch of row r sits at chunk (ch % 8) ^ (r % 8) of its box row
                const bf16x8 kv8 = mine ? lds128(knew + ch * 8)
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
                    sc_g[(size_t)h * a.ld + t] = sc;
                    pown[h * a.cap + (t - t0)] = sc;
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
        a.cmax[((size_t)g * a.C + c) * NREP + tid] = m;
    }

    // ---- 4. group barrier
    __syncthreads();
    if (tid == 0 && !group_barrier(a.ctr + 4 * (size_t)g, (unsigned)a.C)) flag_s = 1;
    __syncthreads();
    pdl_trigger();
    if (flag_s) ok = false;

    // ---- 5. softmax statistics (src/kernels.cu:467-470 with block_max / block_sum, :406-436).
    // The maximum over the chunk maxima is the maximum over all positions (exact in any order);
    // the sum of expf(s - max) runs in the reference's order over all positions' scores, SB per
    // head and thread in flight at once (from L2: the group's CTAs wrote them just before).
    const int slot = tid % FA_TILE;  // FA_TILE == 128 slots
    constexpr int SB = HPT <= 2 ? 32 : 16;
    float v[HPT][SB];
    const float *shk[HPT];
#pragma unroll
    for (int k = 0; k < HPT; k++) shk[k] = sc_g + (size_t)(hgp + HG * k < NREP ? hgp + HG * k : 0) * a.ld;
    auto load_batch = [&](int t) {
#pragma unroll
        for (int k = 0; k < HPT; k++)
#pragma unroll
            for (int j = 0; j < SB; j++)
                v[k][j] = (ok && hgp + HG * k < NREP && t + j * 128 < len) ? __ldcg(shk[k] + t + j * 128) : 0.0f;
    };
    load_batch(slot);
    if (ok && tid < a.C * NREP) cm_s[tid] = __ldcg(a.cmax + (size_t)g * a.C * NREP + tid);
    __syncthreads();
    if (tid < NREP) {
        float m = -INFINITY;
        for (int cc = 0; cc < a.C; cc++) m = fmaxf(m, cm_s[cc * NREP + tid]);
        gmax_s[tid] = m;
    }
    __syncthreads();
    {
        float sm[HPT], mk[HPT];
#pragma unroll
        for (int k = 0; k < HPT; k++) {
            sm[k] = 0.0f;
            mk[k] = hgp + HG * k < NREP ? gmax_s[hgp + HG * k] : 0.0f;
        }
        for (int t = slot; t < len; t += SB * 128) {
            if (t > slot) load_batch(t);
#pragma unroll
            for (int k = 0; k < HPT; k++)
#pragma unroll
                for (int j = 0; j < SB; j++)
                    if (hgp + HG * k < NREP && t + j * 128 < len) sm[k] += expf(v[k][j] - mk[k]);
        }
#pragma unroll
        for (int k = 0; k < HPT; k++) {
            const int h = hgp + HG * k;
            float x = sm[k];
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
        // probabilities of this chunk (src/kernels.cu:472-474), in place of its scores
        const int nown = t1 - t0;
        if (ok)
            for (int e = tid; e < NREP * nown; e += FA_THREADS) {
                const int h = e / nown, i = e - h * nown;
                float *ps = pown + h * a.cap + i;
                *ps = round_bf16(expf(*ps - gmax_s[h]) / gsum_s[h]);
            }
        __syncthreads();
    }

    // ---- 6. P.V over this chunk (src/kernels.cu:472-485), thread (d, head group)
    const int d = tid % HD, phg = tid / HD;
    float acc[PV_HPT];
#pragma unroll
    for (int k = 0; k < PV_HPT; k++) acc[k] = 0.0f;
    for (int i = 0; i < n_tiles; i++) {
        if (!__syncthreads_and(wait_tile(true, i))) ok = false;
        const int r0 = t0 + i * FA_TILE;
        const int rows = min(FA_TILE, t1 - r0);
        const float *pt = pown + (r0 - t0);  // head h's probabilities of this tile at pt[h * cap + rr]
        if (ok) {
            const bf16 *vt = vs + (i % FA_STAGES) * (VTILE_BYTES / 2);
            const int rows_c = (last && r0 + rows == len) ? rows - 1 : rows;  // rows from the cache
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
    if (!ok) return;  // every tile issued has been waited for above

    float *part = a.partial + ((size_t)g * a.C + c) * NREP * HD;
#pragma unroll
    for (int k = 0; k < PV_HPT; k++) {
        const int h = phg + PV_HG * k;
        if (h < NREP) part[h * HD + d] = acc[k];
    }
    __syncthreads();
    if (tid == 0) flag_s = atom_add_acq_rel(a.ctr + 4 * (size_t)g + 2, 1u) == (unsigned)a.C - 1 ? 2 : 0;
    __syncthreads();
    if (flag_s != 2) return;
    // the last CTA of the group: add the chunks' partials in chunk order
    bf16 *og = a.out + (size_t)b * a.q_stride + (size_t)kvh * NREP * HD;
    const float *pg = a.partial + (size_t)g * a.C * NREP * HD;
    for (int e = tid; e < NREP * HD; e += FA_THREADS) {
        float vals[FA_MAX_CHUNKS];  // every chunk's load in flight at once, then added in chunk order
#pragma unroll
        for (int cc = 0; cc < FA_MAX_CHUNKS; cc++) vals[cc] = cc < a.C ? __ldcg(pg + (size_t)cc * NREP * HD + e) : 0.0f;
        float o = 0.0f;
#pragma unroll
        for (int cc = 0; cc < FA_MAX_CHUNKS; cc++)
            if (cc < a.C) o += vals[cc];
        og[e] = __float2bfloat16(o);
    }
    if (tid == 0) atomicExch(a.ctr + 4 * (size_t)g + 2, 0u);
}

// Dynamic shared memory: alignment slack, K ring (swizzled boxes), V ring, queries, normed heads,
// new K/V rows, mbarriers, and the chunk's own scores (cap positions per head).
size_t fused_smem_bytes(int nrep, int hd, int cap) {
    return 1024 + (size_t)FA_STAGES * FA_TILE * hd * 2 * 2 + (size_t)nrep * hd * 4 + (size_t)(nrep + 1) * hd * 2 +
           2 * (size_t)hd * 2 + 2 * FA_STAGES * 8 + (size_t)nrep * cap * 4;
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

// CTAs of the fused kernel that fit on one SM with `smem` bytes of dynamic shared memory, or 0
// (the last answer is kept per device and shape).
int fused_per_sm(int nrep, int hd, size_t smem) {
    struct Entry {
        size_t smem;
        int n;
    };
    static Entry cache[64][2][4] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const void *k = fused_kernel_for(nrep, hd);
    if (!k || dev < 0 || dev >= 64) return 0;
    if (smem > 227 * 1024) return 0;
    const int hi = hd == 128 ? 1 : 0, ni = nrep == 1 ? 0 : nrep == 2 ? 1 : nrep == 4 ? 2 : 3;
    Entry &v = cache[dev][hi][ni];
    if (v.smem != smem || v.n == 0) {
        int n = 0;
        if (allow_smem(k, smem) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, FA_THREADS, smem) != cudaSuccess)
            n = 0;
        cudaGetLastError();
        v = {smem, n > 0 ? n : -1};
    }
    return v.n > 0 ? v.n : 0;
}

template <int NREP, int HD>
cudaError_t launch_fused(const CUtensorMap &mk, const CUtensorMap &mv, const FusedArgs &a, int groups, size_t smem,
                         cudaStream_t s) {
    cudaError_t e = allow_smem(reinterpret_cast<const void *>(attn_fused_kernel<NREP, HD>), smem);
    if (e != cudaSuccess) return e;
    return launch(attn_fused_kernel<NREP, HD>, dim3(groups * a.C), dim3(FA_THREADS), smem, s, 1, mk, mv, a);
}

}  // namespace

unsigned take_error_attn_fused() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

// Chunks per (sequence, kv head) group for `batch` sequences of up to max_seq positions, or 0 when
// the fused kernel does not apply (head_dim other than 64 / 128, group size other than 1, 2, 4, 8,
// fewer than two chunks per group in one wave of resident CTAs -- the split-KV path is the
// better fit there -- or a chunk too long for shared memory).
int fused_chunks(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq) {
    if (batch <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || max_seq <= 0) return 0;
    const int nrep = n_heads / n_kv_heads;
    if (!fused_kernel_for(nrep, head_dim)) return 0;
    const long long groups = (long long)batch * n_kv_heads;
    // the most CTAs per SM that still fit once the chunk's own scores are counted
    for (int per_sm = fused_per_sm(nrep, head_dim, fused_smem_bytes(nrep, head_dim, 0)); per_sm >= 1; per_sm--) {
        const long long resident = (long long)num_sms() * per_sm;
        if (2 * groups > resident) continue;
        const int C = (int)std::min<long long>(FA_MAX_CHUNKS, resident / groups);
        if (fused_per_sm(nrep, head_dim, fused_smem_bytes(nrep, head_dim, chunk_cap(max_seq, C))) >= per_sm) return C;
    }
    return 0;
}

// Scratch of the fused kernel: scores [B][n_heads][ld] | chunk maxima | partials | counters
// (each region 256-byte aligned). The counters must be zero before the first launch; every launch
// leaves them at zero.
size_t fused_scratch_layout(int batch, int n_heads, int n_kv_heads, int head_dim, int max_seq, int chunks,
                            void *base, float **scores, float **cmax, float **partial, unsigned **ctr) {
    const int ld = (max_seq + 3) / 4 * 4;
    const size_t groups = (size_t)batch * n_kv_heads, nrep = (size_t)(n_heads / n_kv_heads);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) / 256 * 256;
        return o;
    };
    const size_t o_sc = take((size_t)batch * n_heads * ld * 4);
    const size_t o_cm = take(groups * chunks * nrep * 4);
    const size_t o_pa = take(groups * chunks * nrep * head_dim * 4);
    const size_t o_ct = take(groups * 4 * 4);
    if (base) {
        unsigned char *p = static_cast<unsigned char *>(base);
        *scores = reinterpret_cast<float *>(p + o_sc);
        *cmax = reinterpret_cast<float *>(p + o_cm);
        *partial = reinterpret_cast<float *>(p + o_pa);
        *ctr = reinterpret_cast<unsigned *>(p + o_ct);
    }
    return off;
}

int attention_fused(bf16 *out, const bf16 *q, const bf16 *k, const bf16 *v, const bf16 *q_norm_w,
                    const bf16 *k_norm_w, bf16 *key_cache, bf16 *value_cache, KvLayout kv, const int *pos, int batch,
                    long long q_stride, long long kv_stride, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                    float eps, float theta, float scale, int chunks, void *scratch, cudaStream_t s) {
    if (!out || !q || !k || !v || !q_norm_w || !k_norm_w || !key_cache || !value_cache || !pos || !scratch)
        return Q3_ERR_ARG;
    if (batch <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads != 0 || max_seq <= 0) return Q3_ERR_SHAPE;
    const int nrep = n_heads / n_kv_heads;
    if (!fused_kernel_for(nrep, head_dim)) return Q3_ERR_SHAPE;
    if (chunks < 1 || chunks > FA_MAX_CHUNKS) return Q3_ERR_SHAPE;
    const int cap = chunk_cap(max_seq, chunks);
    const size_t smem = fused_smem_bytes(nrep, head_dim, cap);
    const int per_sm = fused_per_sm(nrep, head_dim, smem);
    // the group barrier needs the whole grid resident at once (and the chunk's scores must fit)
    if (per_sm <= 0 || (long long)batch * n_kv_heads * chunks > (long long)num_sms() * per_sm) return Q3_ERR_SHAPE;
    if (kv.pos <= 0 || kv.seq < 0 || kv.head < 0 || q_stride < (long long)n_heads * head_dim ||
        kv_stride < (long long)n_kv_heads * head_dim)
        return Q3_ERR_SHAPE;
    // rows of one sequence must not overlap those of another: each launch writes one row per
    // sequence that other sequences' CTAs would otherwise read
    if (batch > 1 && kv.seq == 0) return Q3_ERR_SHAPE;
    auto al = [](const void *p_) { return (reinterpret_cast<uintptr_t>(p_) & 15) == 0; };
    if (!al(key_cache) || !al(value_cache) || kv.seq % 8 || kv.pos % 8 || kv.head % 8) return Q3_ERR_ALIGN;
    if (!al(scratch)) return Q3_ERR_ALIGN;
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
    fused_scratch_layout(batch, n_heads, n_kv_heads, head_dim, max_seq, chunks, scratch, &a.scores, &a.cmax,
                         &a.partial, &a.ctr);
    a.kv = kv;
    a.q_stride = q_stride;
    a.kv_stride = kv_stride;
    a.ld = (max_seq + 3) / 4 * 4;
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.max_seq = max_seq;
    a.C = chunks;
    a.cap = cap;
    a.rows_per_seq = (int)(kv.seq / kv.pos);
    a.rows_per_head = head_rows ? (int)(kv.head / kv.pos) : 0;
    a.cols_per_head = head_rows ? 0 : (int)kv.head;
    CUtensorMap mk, mv;
    if (!make_map_strided(&mk, key_cache, map_rows, kv.pos, kv.pos, FA_TILE) ||
        !make_map_plain(&mv, value_cache, map_rows, kv.pos, kv.pos, FA_TILE, head_dim))
        return Q3_ERR_ARG;
    a.eps = eps;
    a.theta = theta;
    a.scale = scale;
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
