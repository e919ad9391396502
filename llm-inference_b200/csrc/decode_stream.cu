// Batch-1 decode step as one persistent kernel whose weight stream never waits (sm_100a).
//
// At batch 1 a token reads every weight once (8 GB for Qwen3-4B), so the step is bound by HBM
// bandwidth -- if HBM never idles. Between the kernels of a per-op graph it does: each kernel
// boundary, each dependency (x before q/k/v, attention before o_proj, ...) drains the memory
// pipeline. Here one cooperative launch runs the whole token with one CTA per SM, and the
// weights stop depending on anything:
//
//   - Warp 8 of every CTA (one elected thread) is the PRODUCER. It walks the token's phases in
//     order -- per layer qkv, o_proj, gate_up, down, then the LM head -- and for each phase copies
//     this CTA's contiguous slice of weight rows into a ring of shared-memory stages with
//     cp.async.bulk (the rows are contiguous in memory, so a stage is one to three bulk copies).
//     It waits only for a free stage, never for an activation. A second cursor runs DS_PREFETCH
//     stages ahead and issues L2 prefetches of the same rows (and, entering a layer, of this
//     CTA's chunk of the K and V caches), so while the consumers sit at a barrier or in
//     attention, HBM keeps streaming the next phases into L2 beyond what the ring holds.
//   - Warps 0-7 are the CONSUMERS (256 threads, the reference's rmsnorm block). Each phase they
//     build the input vector in shared memory (rmsnorm of the residual stream, or the attention
//     output, or the SwiGLU activations), then take the phase's rows from the ring: row i of the
//     CTA's slice goes to warp i % 8, so rows that fill one stage are worked by several warps
//     and long rows (down_proj) by warps on consecutive stages at once.
//   - The per-row arithmetic is the reference's (src/kernels.cu): lane l accumulates the 16-byte
//     chunks l, l+32, ... of the row with one fused multiply-add per element in order, the
//     __shfl_down tree, bf16 rounding at the reference's points (:79-298); rmsnorm with 256
//     threads in the reference's order (:25-71); the per-head q/k RMSNorm and RoPE (:301-403);
//     scores with the serial dot, softmax max and sum in the reference's 128-slot order,
//     probabilities round_bf16(expf(s - max) / sum) (:439-497). Only P.V sums in another fp32
//     order: the positions are cut into chunks whose partial sums are added in chunk order.
//   - Attention: the CTAs are split into one group per kv head (C = grid / n_kv CTAs each), each
//     CTA one chunk of the positions. RoPE is recomputed by every CTA of a group from the raw
//     projections; the CTA holding the newest position writes its K and V rows. Two group
//     barriers (chunk maxima, then the 128-slot sum chains) and a last-arriver combine replace
//     grid-wide steps.
//   - Grid barriers separate the phases that need a complete vector: after qkv, attention,
//     o_proj, gate_up and down. The LM head keeps a running argmax per warp; the last CTA to
//     finish reduces the CTAs' candidates, writes the token, advances the position and resets
//     the barrier counters for the next launch.
//
// Every wait is bounded (WAIT_LIMIT_NS): a timed-out wait sets the shared error word, after
// which every CTA leaves at its next wait; the producer stops issuing copies and waits for
// those in flight before the CTA exits. Every exit decision of the consumers is made uniform
// over the CTA's 256 consumer threads (their barriers need all of them).
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int DS_CWARPS = 8;
constexpr int DS_CTHREADS = DS_CWARPS * 32;   // consumers
constexpr int DS_THREADS = DS_CTHREADS + 32;  // + the producer warp
constexpr int DS_HD = 128;
constexpr int DS_XRES = 64;                   // residual rows a CTA may own per phase
constexpr int DS_PT = 64;                     // positions per staged probability tile
constexpr int DS_LINE = 32;                   // sync words: one counter per 128-byte line
constexpr int DS_PREFETCH = 8;                // stages the L2 prefetch runs ahead of the copies (320 KB)
constexpr int DS_NORM_REG = 32;               // x values a thread keeps in the rmsnorm (dim <= 8192)

enum : int { PH_QKV = 0, PH_OPROJ = 1, PH_GATEUP = 2, PH_DOWN = 3, PH_LMHEAD = 4 };

// sync word indices (times DS_LINE)
constexpr int SW_GRID = 0, SW_ERR = 1, SW_DONE = 2, SW_GROUPS = 3;  // then g1[n_kv], g2[n_kv], g3[n_kv]

__device__ __forceinline__ float ldcg_f(const float *p) { return __ldcg(p); }
__device__ __forceinline__ float ldcg_bf(const bf16 *p) {
    return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short *>(p))));
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acquire() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(DS_CTHREADS) : "memory"); }

// A consumer barrier that also returns, in every consumer thread, whether `v` held in all of them.
__device__ __forceinline__ bool cbar_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(DS_CTHREADS)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// One phase's rows for this CTA: units [u0, u1) of R, `ub` bytes per unit, `per` units per stage.
struct Phase {
    int kind, R, ub, per, u0, u1, stages;
};

// Balanced contiguous split of R units over G CTAs; the CTAs rot, rot+1, ... (mod G) take the
// rem = R % G extra units, and rot advances by rem every phase, so over a token every CTA
// streams about the same number of bytes.
__device__ __forceinline__ void split_units(int R, int G, int b, int rot, int &u0, int &u1) {
    const int base = R / G, rem = R % G;
    auto extra_before = [&](int x) {  // CTAs < x holding an extra unit
        if (rot + rem <= G) return min(max(x - rot, 0), rem);
        return min(x, rot + rem - G) + min(max(x - rot, 0), G - rot);
    };
    const bool mine = ((b - rot + G) % G) < rem;
    u0 = b * base + extra_before(b);
    u1 = u0 + base + (mine ? 1 : 0);
}

__device__ __forceinline__ Phase make_phase(const DsParams &a, int kind, int rot) {
    Phase p;
    p.kind = kind;
    const int qd = a.n_heads * DS_HD, kvd = a.n_kv * DS_HD;
    switch (kind) {
        case PH_QKV: p.R = qd + 2 * kvd; p.ub = 2 * a.H; break;
        case PH_OPROJ: p.R = a.H; p.ub = 2 * qd; break;
        case PH_GATEUP: p.R = a.I; p.ub = 4 * a.H; break;  // a gate row and an up row
        case PH_DOWN: p.R = a.H; p.ub = 2 * a.I; break;
        default: p.R = a.vocab; p.ub = 2 * a.H; break;
    }
    p.per = DS_STAGE_BYTES / p.ub;
    split_units(p.R, gridDim.x, blockIdx.x, rot, p.u0, p.u1);
    p.stages = (p.u1 - p.u0 + p.per - 1) / p.per;
    return p;
}

__device__ __forceinline__ int next_rot(const Phase &p, int rot) { return (rot + p.R % (int)gridDim.x) % (int)gridDim.x; }

// The producer's walk over the token's ring stages: layer l, phase kind, stage s of the phase.
struct Cursor {
    int l, kind, s, rot;
    Phase ph;
    bool done;
};

__device__ __forceinline__ void cursor_phase(Cursor &c, const DsParams &a) {
    c.ph = make_phase(a, c.kind, c.rot);
    c.rot = next_rot(c.ph, c.rot);
    c.s = 0;
}

// Moves to the next stage (skipping phases in which this CTA has no rows).
__device__ __forceinline__ void cursor_next(Cursor &c, const DsParams &a) {
    c.s++;
    while (!c.done && c.s >= c.ph.stages) {
        if (c.kind == PH_LMHEAD) {
            c.done = true;
            break;
        }
        if (c.kind == PH_DOWN) {
            c.l++;
            c.kind = c.l < a.n_layers ? PH_QKV : PH_LMHEAD;
        } else {
            c.kind++;
        }
        cursor_phase(c, a);
    }
}

__device__ __forceinline__ void cursor_init(Cursor &c, const DsParams &a) {
    c.l = 0;
    c.kind = PH_QKV;
    c.rot = 0;
    c.done = false;
    cursor_phase(c, a);
    c.s = -1;
    cursor_next(c, a);
}

// The global source ranges of the cursor's stage: fn(byte offset in the stage, source, bytes).
template <typename F>
__device__ __forceinline__ void stage_segments(const Cursor &c, const DsParams &a, F fn) {
    const Phase &ph = c.ph;
    const MkLayer *w = a.layers + min(c.l, a.n_layers - 1);
    const int qd = a.n_heads * DS_HD, kvd = a.n_kv * DS_HD;
    const int ra = ph.u0 + c.s * ph.per, rb = min(ra + ph.per, ph.u1), n = rb - ra;
    if (c.kind == PH_QKV) {  // rows of wq, wk, wv as one concatenated matrix
        const int ends[3] = {qd, qd + kvd, qd + 2 * kvd};
        const bf16 *mats[3] = {w->wq, w->wk, w->wv};
        int start = 0;
        for (int m = 0; m < 3; m++) {
            const int lo = max(ra, start), hi = min(rb, ends[m]);
            if (lo < hi) fn((lo - ra) * ph.ub, mats[m] + (size_t)(lo - start) * a.H, (uint32_t)((hi - lo) * ph.ub));
            start = ends[m];
        }
    } else if (c.kind == PH_GATEUP) {  // gate rows, then up rows at per * 2H
        const uint32_t half = (uint32_t)(n * 2 * a.H);
        fn(0, w->w_gate + (size_t)ra * a.H, half);
        fn(ph.per * 2 * a.H, w->w_up + (size_t)ra * a.H, half);
    } else {
        const bf16 *m = c.kind == PH_OPROJ ? w->wo : c.kind == PH_DOWN ? w->w_down : a.lm_head;
        fn(0, m + (size_t)ra * (ph.ub / 2), (uint32_t)(n * ph.ub));
    }
}

// ------------------------------------------------------------------ barriers

// Barrier among the consumer threads of the CTAs counting on `ctr`: every CTA adds 1 (a release:
// the CTA's writes before the consumer barrier are visible to whoever acquires the count), then
// waits for `target` arrivals, polling with relaxed loads and acquiring once at the end. Returns
// false once any CTA has recorded an error (or this wait timed out).
__device__ bool count_barrier(unsigned *sync, unsigned *ctr, unsigned target, int *flag_s) {
    cbar();
    if (threadIdx.x == 0) {
        red_release_add(ctr, 1u);
        int ok = 1;
        if ((int)(ld_relaxed(ctr) - target) < 0) {
            const uint64_t t0 = globaltimer();
            while ((int)(ld_relaxed(ctr) - target) < 0) {
                if (ld_relaxed(sync + SW_ERR * DS_LINE)) {
                    ok = 0;
                    break;
                }
                if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                    atomicOr(sync + SW_ERR * DS_LINE, 1u);
                    atomicOr(&g_dev_error, DEV_ERR_WAIT_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        fence_acquire();
        *flag_s = ok;
    }
    cbar();
    return *(volatile int *)flag_s != 0;
}

// mbarrier wait that also gives up once the error word is set (another CTA failed).
__device__ bool ring_wait(uint64_t *bar, uint32_t parity, unsigned *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (ld_relaxed(err)) return false;
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(err, 1u);
            atomicOr(&g_dev_error, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------------------ consumer pieces

// y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w) into shared memory: src/kernels.cu:25-71 with its
// 256 threads -- thread t sums x[t], x[t + 256], ... with fused multiply-adds, an xor tree per
// warp, the eight warp sums in order. x is global memory written in this kernel (read from L2,
// once: each thread keeps its values in registers for the scaling).
__device__ void block_rmsnorm(const bf16 *x, const bf16 *w, bf16 *out, int dim, float eps, float *red) {
    const int tid = threadIdx.x;
    float xv[DS_NORM_REG];
#pragma unroll
    for (int j = 0; j < DS_NORM_REG; j++) {  // all loads first: one round trip to L2
        const int i = tid + j * DS_CTHREADS;
        xv[j] = i < dim ? ldcg_bf(x + i) : 0.0f;
    }
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < DS_NORM_REG; j++)
        if (tid + j * DS_CTHREADS < dim) sum = __fmaf_rn(xv[j], xv[j], sum);
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (tid % 32 == 0) red[tid / 32] = sum;
    cbar();
    float total = 0.0f;
#pragma unroll
    for (int wi = 0; wi < DS_CWARPS; wi++) total += red[wi];
    const float inv_rms = rsqrtf(total / dim + eps);
#pragma unroll
    for (int j = 0; j < DS_NORM_REG; j++) {
        const int i = tid + j * DS_CTHREADS;
        if (i < dim) {
            const bf16 normed = __float2bfloat16(xv[j] * inv_rms);
            out[i] = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(w[i]));
        }
    }
    cbar();
}

// A vector written in this kernel (global, L2) into shared memory, 16 bytes per load.
__device__ void load_vec(const bf16 *src, bf16 *dst, int n) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int i = threadIdx.x; i < n / 8; i += DS_CTHREADS) d[i] = __ldcg(s + i);
    cbar();
}

// Dot products of one or two weight rows in shared memory with the input vector in shared
// memory, in the reference warp_dot order; valid in lane 0.
template <int NR>
__device__ __forceinline__ void rows_dot(const unsigned char *w0, const unsigned char *w1, const bf16 *xv, int n_vec,
                                         int lane, float *acc) {
    float a0 = 0.0f, a1 = 0.0f;
    int i = lane;
    for (; i + 96 < n_vec; i += 128) {  // four chunks of each row in flight
        bf16x8 wa[4], wb[4], xc[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            wa[u] = lds128(w0 + 16 * (i + 32 * u));
            if (NR == 2) wb[u] = lds128(w1 + 16 * (i + 32 * u));
            xc[u] = lds128(xv + 8 * (i + 32 * u));
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            a0 = dot8(wa[u], xc[u], a0);
            if (NR == 2) a1 = dot8(wb[u], xc[u], a1);
        }
    }
    for (; i < n_vec; i += 32) {
        const bf16x8 xc = lds128(xv + 8 * i);
        a0 = dot8(lds128(w0 + 16 * i), xc, a0);
        if (NR == 2) a1 = dot8(lds128(w1 + 16 * i), xc, a1);
    }
    for (int off = 16; off > 0; off >>= 1) {
        a0 += __shfl_down_sync(0xffffffffu, a0, off);
        if (NR == 2) a1 += __shfl_down_sync(0xffffffffu, a1, off);
    }
    acc[0] = a0;
    if (NR == 2) acc[1] = a1;
}

struct Smem {
    unsigned char *ring;
    bf16 *xvec;      // the phase's input vector; during attention, this CTA's chunk scores
    uint64_t *full, *empty;
    float *red;      // [32]
    float *xres;     // [DS_XRES]
    float *qf;       // [NREP][128] roped queries
    float *knew;     // [128] roped key row of the newest position
    float *vnew;     // [128] value row of the newest position
    bf16 *hs;        // [2][128] normed heads (RoPE staging)
    float *m_s, *s_s;  // [NREP] softmax max and sum
    float *ptile;    // [NREP][DS_PT] probabilities
    float *pvh;      // [NREP][128] the second half's P.V partial
    float *bv;       // [8] argmax candidates per warp
    int *bi;
    int *flag;       // [4]
};

// argmax order: larger value wins, lower index on ties, NaN never wins (src/kernels.cu:500-544)
__device__ __forceinline__ void amax_take(float &best, int &bi, float v, int i) {
    if (v > best || (v == best && i < bi)) {
        best = v;
        bi = i;
    }
}

}  // namespace

// ------------------------------------------------------------------ the kernel

template <int NREP>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_stream_kernel(const __grid_constant__ DsParams a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int qd = a.n_heads * DS_HD, kvd = a.n_kv * DS_HD;
    const int xv_elems = max(max(a.H, qd), a.I);
    Smem sm;
    {
        unsigned char *p = smem_raw;
        sm.ring = p;
        p += (size_t)a.stages * DS_STAGE_BYTES;
        sm.xvec = reinterpret_cast<bf16 *>(p);
        p += ((size_t)xv_elems * 2 + 127) / 128 * 128;
        sm.full = reinterpret_cast<uint64_t *>(p);
        sm.empty = sm.full + DS_MAX_STAGES;
        p += 2 * DS_MAX_STAGES * 8;
        sm.red = reinterpret_cast<float *>(p);
        sm.xres = sm.red + 32;
        sm.qf = sm.xres + DS_XRES;
        sm.knew = sm.qf + NREP * DS_HD;
        sm.vnew = sm.knew + DS_HD;
        sm.m_s = sm.vnew + DS_HD;
        sm.s_s = sm.m_s + 8;
        sm.ptile = sm.s_s + 8;
        sm.pvh = sm.ptile + NREP * DS_PT;
        sm.bv = sm.pvh + NREP * DS_HD;
        sm.bi = reinterpret_cast<int *>(sm.bv + 8);
        sm.flag = sm.bi + 8;
        sm.hs = reinterpret_cast<bf16 *>(sm.flag + 4);
    }
    const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const int G = gridDim.x;
    unsigned *err = a.sync + SW_ERR * DS_LINE;

    if (tid == 0) {
        for (int i = 0; i < a.stages; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], DS_CWARPS);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const int token = __ldcg(a.next_token);
    const int pos = __ldcg(a.pos);
    const bool valid = token >= 0 && token < a.vocab && pos >= 0 && pos < a.max_seq;
    if (!valid) {  // every CTA reads the same values and leaves here, before any barrier
        if (blockIdx.x == 0 && tid == 0)
            atomicOr(&g_dev_error, token < 0 || token >= a.vocab ? DEV_ERR_TOKEN_RANGE : DEV_ERR_POS_RANGE);
        return;
    }
    const int len = pos + 1;
    const int C = a.chunks;
    const bool attn_cta = (int)blockIdx.x < a.n_kv * C;
    const int h = blockIdx.x / C, c = blockIdx.x % C;  // attention group (kv head) and chunk
    const int L = (len + C - 1) / C;
    const int t0 = min(c * L, len), t1 = min(t0 + L, len);
    const size_t head_stride = (size_t)a.max_seq * DS_HD;

    if (warp == DS_CWARPS) {
        // ============================ producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();  // weights are read once per token
            Cursor cp, pf;
            cursor_init(cp, a);
            cursor_init(pf, a);
            auto prefetch_stage = [&]() {
                if (pf.done) return;
                if (attn_cta && pf.kind == PH_QKV && pf.s == 0 && t1 > t0) {
                    const size_t off = (size_t)pf.l * a.layer_stride + (size_t)h * head_stride + (size_t)t0 * DS_HD;
                    prefetch_l2(a.key_cache + off, (uint32_t)((t1 - t0) * DS_HD * 2));
                    prefetch_l2(a.value_cache + off, (uint32_t)((t1 - t0) * DS_HD * 2));
                }
                stage_segments(pf, a, [&](int, const bf16 *src, uint32_t bytes) { prefetch_l2(src, bytes); });
                cursor_next(pf, a);
            };
            for (int k = 0; k < DS_PREFETCH; k++) prefetch_stage();
            uint32_t it = 0;
            for (; !cp.done; it++) {
                const int slot = it % a.stages;
                if (it >= (uint32_t)a.stages && !ring_wait(&sm.empty[slot], ((it / a.stages) - 1) & 1, err)) break;
                unsigned char *dst = sm.ring + (size_t)slot * DS_STAGE_BYTES;
                uint64_t *bar = &sm.full[slot];
                const int ra = cp.ph.u0 + cp.s * cp.ph.per, n = min(cp.ph.per, cp.ph.u1 - ra);
                mbar_arrive_expect_tx(bar, (uint32_t)(n * cp.ph.ub));
                stage_segments(cp, a, [&](int off, const bf16 *src, uint32_t bytes) {
                    bulk_g2s_hint(dst + off, src, bytes, bar, pol);
                });
                cursor_next(cp, a);
                prefetch_stage();
            }
            // copies still in flight land before the CTA exits
            const uint32_t first = it > (uint32_t)a.stages ? it - a.stages : 0;
            for (uint32_t j = first; j < it; j++) mbar_wait(&sm.full[j % a.stages], (j / a.stages) & 1, &g_dev_error);
        }
        return;
    }

    // ============================ consumers
    uint32_t it = 0;  // ring stage counter, in step with the producer's
    int rot = 0;
    unsigned nbar = 0;  // grid barriers passed
    bool ok = true;
    float best = -INFINITY;  // LM head: this warp's running argmax
    int bidx = 0x7fffffff;

    // the embedding row into the residual stream (src/kernels.cu:7-23); ordered before its first
    // reader (o_proj of layer 0) by the barrier after qkv
    const bf16 *emb = a.embed + (size_t)token * a.H;
    for (int i = blockIdx.x * DS_CTHREADS + tid; i < a.H; i += G * DS_CTHREADS) a.x[i] = emb[i];

    // One GEMV phase over the ring; `epi(unit, acc)` writes a row's result (lane 0). Returns, in
    // every consumer thread, whether all of its waits succeeded.
    auto run_phase = [&](const Phase &ph, auto epi) {
        const int n_vec = (ph.kind == PH_GATEUP ? ph.ub / 2 : ph.ub) / 16;
        bool good = true;
        for (int s = 0; s < ph.stages && good; s++, it++) {
            const int slot = it % a.stages;
            if (!ring_wait(&sm.full[slot], (it / a.stages) & 1, err)) {
                good = false;
                break;
            }
            const unsigned char *stage = sm.ring + (size_t)slot * DS_STAGE_BYTES;
            const int ra = ph.u0 + s * ph.per, n = min(ph.per, ph.u1 - ra);
            // unit j of the stage is unit s * per + j of the CTA's slice: warp (s * per + j) % 8
            for (int j = (warp - (s * ph.per) % DS_CWARPS + DS_CWARPS) % DS_CWARPS; j < n; j += DS_CWARPS) {
                float acc[2];
                if (ph.kind == PH_GATEUP)
                    rows_dot<2>(stage + (size_t)j * (ph.ub / 2), stage + (size_t)(ph.per + j) * (ph.ub / 2), sm.xvec,
                                n_vec, lane, acc);
                else
                    rows_dot<1>(stage + (size_t)j * ph.ub, nullptr, sm.xvec, n_vec, lane, acc);
                if (lane == 0) epi(ra + j, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[slot]);
        }
        return cbar_all(good);
    };

    for (int l = 0; l < a.n_layers && ok; l++) {
        const MkLayer w = a.layers[l];
        bf16 *kc = a.key_cache + (size_t)l * a.layer_stride;
        bf16 *vc = a.value_cache + (size_t)l * a.layer_stride;

        // ---- attention norm + q, k, v (src/kernels.cu:215-257); layer 0 normalizes the table row
        block_rmsnorm(l == 0 ? emb : a.x, w.attn_norm, sm.xvec, a.H, a.eps, sm.red);
        {
            const Phase ph = make_phase(a, PH_QKV, rot);
            rot = next_rot(ph, rot);
            ok = run_phase(ph, [&](int r, const float *acc) {
                const bf16 y = __float2bfloat16(acc[0]);
                if (r < qd) a.q[r] = y;
                else if (r < qd + kvd) a.k[r - qd] = y;
                else a.v[r - qd - kvd] = y;
            });
        }
        if (!ok || !count_barrier(a.sync, a.sync + SW_GRID * DS_LINE, ++nbar * G, sm.flag)) {
            ok = false;
            break;
        }

        // ---- attention of this CTA's (kv head, chunk)
        if (attn_cta) {
            const unsigned gtarget = (unsigned)(C * (l + 1));
            unsigned *g1 = a.sync + (SW_GROUPS + h) * DS_LINE;
            unsigned *g2 = a.sync + (SW_GROUPS + a.n_kv + h) * DS_LINE;
            unsigned *g3 = a.sync + (SW_GROUPS + 2 * a.n_kv + h) * DS_LINE;
            // q/k RMSNorm and RoPE of the group's heads (src/kernels.cu:301-403), two heads a round
            {
                const int sub = tid / DS_HD, i = tid % DS_HD;
                for (int r0 = 0; r0 < NREP + 1; r0 += 2) {
                    const int hi = r0 + sub;
                    const bool act = hi < NREP + 1;
                    const bool is_key = hi == NREP;
                    const bf16 *src = is_key ? a.k + h * DS_HD : a.q + (size_t)(h * NREP + (act ? hi : 0)) * DS_HD;
                    const float xi = act ? ldcg_bf(src + i) : 0.0f;
                    float sum = xi * xi;
                    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                    if (lane == 0) sm.red[warp] = sum;
                    cbar();
                    float total = 0.0f;
                    for (int wi = 0; wi < DS_HD / 32; wi++) total += sm.red[sub * (DS_HD / 32) + wi];
                    const float inv_rms = rsqrtf(total / DS_HD + a.eps);
                    const bf16 normed = __float2bfloat16(xi * inv_rms);
                    const bf16 *nw = is_key ? w.k_norm : w.q_norm;
                    sm.hs[sub * DS_HD + i] = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(nw[i]));
                    cbar();
                    const int half = DS_HD / 2;
                    if (act && i < half) {
                        const float inv_freq = 1.0f / powf(a.theta, (float)(2 * i) / DS_HD);
                        const float angle = pos * inv_freq;
                        const float cs = round_bf16(cosf(angle));
                        const float sn = round_bf16(sinf(angle));
                        const float av = __bfloat162float(sm.hs[sub * DS_HD + i]);
                        const float bv = __bfloat162float(sm.hs[sub * DS_HD + i + half]);
                        const float oa = round_bf16(round_bf16(av * cs) - round_bf16(bv * sn));
                        const float ob = round_bf16(round_bf16(bv * cs) + round_bf16(av * sn));
                        float *dst = is_key ? sm.knew : sm.qf + hi * DS_HD;
                        dst[i] = oa;
                        dst[i + half] = ob;
                    }
                    cbar();
                }
                if (tid < DS_HD) sm.vnew[tid] = ldcg_bf(a.v + h * DS_HD + tid);
                cbar();
                if (t0 <= pos && pos < t1 && tid < DS_HD) {  // the newest position's cache rows
                    kc[(size_t)h * head_stride + (size_t)pos * DS_HD + tid] = __float2bfloat16(sm.knew[tid]);
                    vc[(size_t)h * head_stride + (size_t)pos * DS_HD + tid] = __float2bfloat16(sm.vnew[tid]);
                }
            }
            // scores of the chunk: one position per thread, the serial dot over head_dim. They go to
            // global memory (the sum chains of the whole group read them) and, when they fit, also
            // to shared memory over the input vector (idle during attention) for this CTA's P.V.
            float *sc_s = reinterpret_cast<float *>(sm.xvec);
            const bool sc_local = (size_t)NREP * L * 4 <= (size_t)xv_elems * 2;
            float lmax[NREP];
#pragma unroll
            for (int j = 0; j < NREP; j++) lmax[j] = -INFINITY;
            for (int t = t0 + tid; t < t1; t += DS_CTHREADS) {
                float acc[NREP];
#pragma unroll
                for (int j = 0; j < NREP; j++) acc[j] = 0.0f;
                const bf16 *krow = kc + (size_t)h * head_stride + (size_t)t * DS_HD;
                for (int c8 = 0; c8 < DS_HD / 8; c8 += 4) {
                    float kf[32];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        if (t == pos) {
#pragma unroll
                            for (int e = 0; e < 8; e++) kf[u * 8 + e] = sm.knew[(c8 + u) * 8 + e];
                        } else {
                            const bf16x8 kv = ldg128(krow + (c8 + u) * 8);
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const float2 f = __bfloat1622float2(kv.h[e]);
                                kf[u * 8 + 2 * e] = f.x;
                                kf[u * 8 + 2 * e + 1] = f.y;
                            }
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 32; e++)
#pragma unroll
                        for (int j = 0; j < NREP; j++) acc[j] = __fmaf_rn(sm.qf[j * DS_HD + c8 * 8 + e], kf[e], acc[j]);
                }
#pragma unroll
                for (int j = 0; j < NREP; j++) {
                    const float sc = round_bf16(round_bf16(acc[j]) * a.scale);
                    a.scores[(size_t)(h * NREP + j) * a.ld + t] = sc;
                    if (sc_local) sc_s[j * L + (t - t0)] = sc;
                    lmax[j] = fmaxf(lmax[j], sc);
                }
            }
            // chunk maxima (order does not matter for a max)
#pragma unroll
            for (int j = 0; j < NREP; j++) {
                float v = lmax[j];
                for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
                lmax[j] = v;
            }
            if (lane == 0)
#pragma unroll
                for (int j = 0; j < NREP; j++) sm.pvh[warp * NREP + j] = lmax[j];
            cbar();
            if (tid < NREP) {
                float v = -INFINITY;
                for (int wi = 0; wi < DS_CWARPS; wi++) v = fmaxf(v, sm.pvh[wi * NREP + tid]);
                a.cmax[((size_t)h * C + c) * NREP + tid] = v;
            }
            if (!count_barrier(a.sync, g1, gtarget, sm.flag)) {
                ok = false;
                break;
            }
            // the group's maxima, then the 128-slot sum chains: chain q = c + C * tid
            if (tid < NREP) {
                float v = -INFINITY;
                for (int cc = 0; cc < C; cc++) v = fmaxf(v, ldcg_f(a.cmax + ((size_t)h * C + cc) * NREP + tid));
                sm.m_s[tid] = v;
            }
            cbar();
            {
                const int q = c + C * tid;
                if (q < NREP * 128) {
                    const int j = q / 128, slot = q % 128;
                    const float m = sm.m_s[j];
                    const float *sc = a.scores + (size_t)(h * NREP + j) * a.ld;
                    float sacc = 0.0f;
                    int t = slot;
                    for (; t + 3 * 128 < len; t += 4 * 128) {  // four loads in flight, summed in order
                        const float v0 = ldcg_f(sc + t), v1 = ldcg_f(sc + t + 128), v2 = ldcg_f(sc + t + 256),
                                    v3 = ldcg_f(sc + t + 384);
                        sacc += expf(v0 - m);
                        sacc += expf(v1 - m);
                        sacc += expf(v2 - m);
                        sacc += expf(v3 - m);
                    }
                    for (; t < len; t += 128) sacc += expf(ldcg_f(sc + t) - m);
                    a.csum[(size_t)h * NREP * 128 + q] = sacc;
                }
            }
            if (!count_barrier(a.sync, g2, gtarget, sm.flag)) {
                ok = false;
                break;
            }
            // block_sum of each head: xor tree over each warp's 32 slots, the four totals in order
            if (warp < NREP) {
                float total = 0.0f;
                for (int p4 = 0; p4 < 4; p4++) {
                    float v = ldcg_f(a.csum + (size_t)h * NREP * 128 + warp * 128 + p4 * 32 + lane);
                    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                    total += v;
                }
                if (lane == 0) sm.s_s[warp] = total;
            }
            cbar();
            // P.V of the chunk: thread (half, d) sums the first or second 32 positions of each tile
            {
                const int hf = tid / DS_HD, d = tid % DS_HD;
                float acc[NREP];
#pragma unroll
                for (int j = 0; j < NREP; j++) acc[j] = 0.0f;
                const bf16 *vcol = vc + (size_t)h * head_stride + d;
                for (int tt = t0; tt < t1; tt += DS_PT) {
                    const int n = min(DS_PT, t1 - tt);
                    for (int idx = tid; idx < NREP * DS_PT; idx += DS_CTHREADS) {
                        const int j = idx / DS_PT, tl = idx % DS_PT;
                        if (tl < n) {
                            const float sc = sc_local ? sc_s[j * L + (tt + tl - t0)]
                                                      : ldcg_f(a.scores + (size_t)(h * NREP + j) * a.ld + tt + tl);
                            sm.ptile[idx] = round_bf16(expf(sc - sm.m_s[j]) / sm.s_s[j]);
                        } else {
                            sm.ptile[idx] = 0.0f;
                        }
                    }
                    cbar();
                    const int ta = hf * (DS_PT / 2), tb = min(ta + DS_PT / 2, n);
                    int tl = ta;
                    for (; tl + 8 <= tb; tl += 8) {
                        float vv[8];
#pragma unroll
                        for (int u = 0; u < 8; u++) {
                            const int t = tt + tl + u;
                            vv[u] = t == pos ? sm.vnew[d] : __bfloat162float(vcol[(size_t)t * DS_HD]);
                        }
#pragma unroll
                        for (int u = 0; u < 8; u++)
#pragma unroll
                            for (int j = 0; j < NREP; j++) acc[j] = __fmaf_rn(sm.ptile[j * DS_PT + tl + u], vv[u], acc[j]);
                    }
                    for (; tl < tb; tl++) {
                        const int t = tt + tl;
                        const float vv = t == pos ? sm.vnew[d] : __bfloat162float(vcol[(size_t)t * DS_HD]);
#pragma unroll
                        for (int j = 0; j < NREP; j++) acc[j] = __fmaf_rn(sm.ptile[j * DS_PT + tl], vv, acc[j]);
                    }
                    cbar();
                }
                if (hf == 1)
#pragma unroll
                    for (int j = 0; j < NREP; j++) sm.pvh[j * DS_HD + d] = acc[j];
                cbar();
                if (hf == 0)
#pragma unroll
                    for (int j = 0; j < NREP; j++)
                        a.partial[(((size_t)h * C + c) * NREP + j) * DS_HD + d] = acc[j] + sm.pvh[j * DS_HD + d];
            }
            // the group's last CTA adds the chunk partials in chunk order
            cbar();
            if (tid == 0) {
                __threadfence();
                sm.flag[1] = atomicAdd(g3, 1u) == gtarget - 1;
                __threadfence();
            }
            cbar();
            if (sm.flag[1]) {
                for (int o = tid; o < NREP * DS_HD; o += DS_CTHREADS) {
                    float sacc = 0.0f;
                    for (int cc = 0; cc < C; cc++) sacc += ldcg_f(a.partial + ((size_t)h * C + cc) * NREP * DS_HD + o);
                    a.attn_out[(size_t)h * NREP * DS_HD + o] = __float2bfloat16(sacc);
                }
            }
        }
        if (!count_barrier(a.sync, a.sync + SW_GRID * DS_LINE, ++nbar * G, sm.flag)) {
            ok = false;
            break;
        }

        // ---- o_proj + residual (src/kernels.cu:185-212)
        {
            const Phase ph = make_phase(a, PH_OPROJ, rot);
            rot = next_rot(ph, rot);
            for (int j = tid; j < ph.u1 - ph.u0; j += DS_CTHREADS) sm.xres[j] = ldcg_bf(a.x + ph.u0 + j);
            load_vec(a.attn_out, sm.xvec, qd);
            ok = run_phase(ph, [&](int r, const float *acc) {
                const bf16 y = __float2bfloat16(acc[0]);
                a.x[r] = __float2bfloat16(sm.xres[r - ph.u0] + __bfloat162float(y));
            });
        }
        if (!ok || !count_barrier(a.sync, a.sync + SW_GRID * DS_LINE, ++nbar * G, sm.flag)) {
            ok = false;
            break;
        }

        // ---- MLP norm + gate/up with SwiGLU (src/kernels.cu:260-298)
        block_rmsnorm(a.x, w.mlp_norm, sm.xvec, a.H, a.eps, sm.red);
        {
            const Phase ph = make_phase(a, PH_GATEUP, rot);
            rot = next_rot(ph, rot);
            ok = run_phase(ph, [&](int r, const float *acc) {
                const float gv = __bfloat162float(__float2bfloat16(acc[0]));
                const float uv = __bfloat162float(__float2bfloat16(acc[1]));
                a.act[r] = __float2bfloat16(round_bf16(gv / (1.0f + expf(-gv))) * uv);
            });
        }
        if (!ok || !count_barrier(a.sync, a.sync + SW_GRID * DS_LINE, ++nbar * G, sm.flag)) {
            ok = false;
            break;
        }

        // ---- down + residual
        {
            const Phase ph = make_phase(a, PH_DOWN, rot);
            rot = next_rot(ph, rot);
            for (int j = tid; j < ph.u1 - ph.u0; j += DS_CTHREADS) sm.xres[j] = ldcg_bf(a.x + ph.u0 + j);
            load_vec(a.act, sm.xvec, a.I);
            ok = run_phase(ph, [&](int r, const float *acc) {
                const bf16 y = __float2bfloat16(acc[0]);
                a.x[r] = __float2bfloat16(sm.xres[r - ph.u0] + __bfloat162float(y));
            });
        }
        if (!ok || !count_barrier(a.sync, a.sync + SW_GRID * DS_LINE, ++nbar * G, sm.flag)) {
            ok = false;
            break;
        }
    }

    // ---- final norm + LM head (src/forward.cu:188-191) with the argmax folded in
    if (ok) {  // uniform over the consumers (every exit from the layer loop is)
        block_rmsnorm(a.x, a.final_norm, sm.xvec, a.H, a.eps, sm.red);
        const Phase ph = make_phase(a, PH_LMHEAD, rot);
        ok = run_phase(ph, [&](int r, const float *acc) {
            const bf16 y = __float2bfloat16(acc[0]);
            a.logits[r] = y;
            amax_take(best, bidx, __bfloat162float(y), r);
        });
    }
    if (lane == 0) {
        sm.bv[warp] = best;
        sm.bi[warp] = bidx;
    }
    cbar();
    if (tid == 0) {
        float b = -INFINITY;
        int bi = 0x7fffffff;
        for (int wi = 0; wi < DS_CWARPS; wi++) amax_take(b, bi, sm.bv[wi], sm.bi[wi]);
        a.amax_val[blockIdx.x] = b;
        a.amax_idx[blockIdx.x] = bi;
        __threadfence();
        const bool last = atomicAdd(a.sync + SW_DONE * DS_LINE, 1u) == (unsigned)G - 1;
        if (last) {
            __threadfence();
            const bool failed = ld_relaxed(err) != 0;
            if (!failed) {
                float bb = -INFINITY;
                int bbi = 0x7fffffff;
                for (int cc = 0; cc < G; cc++) amax_take(bb, bbi, ldcg_f(a.amax_val + cc), __ldcg(a.amax_idx + cc));
                if (bbi == 0x7fffffff) bbi = 0;  // every logit NaN: the reference's initial index
                *a.out_token = bbi;
                *a.next_token = bbi;
                const int st = *a.step;
                if (a.history && st >= 0 && st < a.history_cap) a.history[st] = bbi;
                *a.step = st + 1;
                *a.pos = pos + 1;
            }
            // every CTA has passed its last wait: reset the counters for the next launch
            const int words = SW_GROUPS + 3 * a.n_kv;
            for (int i = 0; i < words; i++) a.sync[i * DS_LINE] = 0u;
            __threadfence();
        }
    }
}

namespace {

template <int NREP>
const void *kernel_ptr() {
    return reinterpret_cast<const void *>(decode_stream_kernel<NREP>);
}

const void *kernel_for(int nrep) {
    switch (nrep) {
        case 1: return kernel_ptr<1>();
        case 2: return kernel_ptr<2>();
        case 4: return kernel_ptr<4>();
        case 8: return kernel_ptr<8>();
        default: return nullptr;
    }
}

// Shared memory beyond the ring: the input vector, barriers and the attention/argmax scratch.
size_t fixed_smem(int H, int I, int n_heads, int n_kv) {
    const int nrep = n_kv > 0 ? n_heads / n_kv : 1;
    const size_t xv = ((size_t)std::max(std::max(H, n_heads * DS_HD), I) * 2 + 127) / 128 * 128;
    const size_t floats = 32 + DS_XRES + (size_t)nrep * DS_HD + 2 * DS_HD + 16 + (size_t)nrep * DS_PT +
                          (size_t)nrep * DS_HD + 8 + 8 + 4;
    return xv + 2 * DS_MAX_STAGES * 8 + floats * 4 + 2 * DS_HD * 2;
}

}  // namespace

// Plans a launch on the current device: fills p.stages and p.chunks and returns the grid (one CTA
// per SM), or 0 when the shapes do not fit this kernel.
int decode_stream_plan(DsParams &p) {
    const int nrep = p.n_kv > 0 ? p.n_heads / p.n_kv : 0;
    const void *k = kernel_for(nrep);
    if (!k || p.n_heads % p.n_kv) return 0;
    const int qd = p.n_heads * DS_HD;
    if (4 * p.H > DS_STAGE_BYTES || 2 * qd > DS_STAGE_BYTES || 2 * p.I > DS_STAGE_BYTES) return 0;
    if (p.H % 8 || p.I % 8 || p.H > DS_NORM_REG * DS_CTHREADS) return 0;
    int dev = 0, optin = 0, nsm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0;
    const size_t fixed = fixed_smem(p.H, p.I, p.n_heads, p.n_kv);
    if ((size_t)optin <= fixed) return 0;
    const int stages = (int)std::min<size_t>(DS_MAX_STAGES, ((size_t)optin - fixed) / DS_STAGE_BYTES);
    if (stages < 2) return 0;
    const size_t smem = fixed + (size_t)stages * DS_STAGE_BYTES;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, DS_THREADS, smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        return 0;
    }
    const int grid = nsm;
    if ((p.H + grid - 1) / grid + 1 > DS_XRES || p.n_kv > grid) return 0;
    if ((grid / p.n_kv) * DS_CTHREADS < nrep * 128) return 0;  // every softmax sum chain has a thread
    p.stages = stages;
    p.chunks = grid / p.n_kv;
    return grid;
}

int decode_stream_launch(const DsParams &p, int grid, cudaStream_t s) {
    const void *k = kernel_for(p.n_kv > 0 ? p.n_heads / p.n_kv : 0);
    if (!k || grid <= 0) return Q3_ERR_SHAPE;
    const size_t smem = fixed_smem(p.H, p.I, p.n_heads, p.n_kv) + (size_t)p.stages * DS_STAGE_BYTES;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the barriers need it
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    void *args[] = {const_cast<DsParams *>(&p)};
    return record_cuda_error(cudaLaunchKernelExC(&cfg, k, args));
}

int decode_stream_sync_words(int n_kv) { return (SW_GROUPS + 3 * n_kv) * DS_LINE; }

unsigned take_error_stream() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

}  // namespace q3
