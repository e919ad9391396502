// Batch-1 decode step in one persistent kernel (sm_100a).
//
// At batch 1 every kernel of the decode step moves little data, so the step's time is set by
// the ~290 kernel boundaries of a token: each pays its ramp (first loads), its drain and the
// dependency hand-off, even with programmatic dependent launch. Here one cooperative launch
// runs a whole token. Its CTAs (all resident: 2 per SM) pass through the step's phases and
// meet at grid barriers between them. A barrier is a counter and a generation word in global
// memory; its wait is bounded, and a timed-out wait sets a sticky error word that ends every
// other CTA's waits at once.
//
// The phases restate, per row, exactly the arithmetic of the batch-1 kernels (and so of the
// reference kernels, src/kernels.cu):
//   - rmsnorm as one 256-thread block in the reference's order (:25-71), computed by every CTA
//     for itself into shared memory;
//   - projections warp per row with the lane-strided fused multiply-add order and shuffle tree
//     (:79-144), gate and up as two such rows (:260-298), the residual add (:185-212);
//   - qk norm, RoPE and the KV write, one head per head_dim threads (:301-403);
//   - attention scores with the serial dot order, the softmax max and sum over 128 slots in the
//     reference's order, probabilities round_bf16(expf(s - max) / sum) (:406-497).
// Only P.V differs: its positions are split into chunks of 128 whose fp32 partial sums are
// added in position order, as in the engine's split-KV attention.
//
// Activations written by other CTAs within the kernel are read with ld.global.cg (L2), never
// from a possibly stale L1 line.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int MK_THREADS = 256;
constexpr int MK_WARPS = MK_THREADS / 32;
constexpr int MK_MIN_CTAS = 2;     // resident CTAs per SM the register budget allows
constexpr int MK_UR = 8;           // 16-byte chunks per lane in flight per row batch
constexpr int MK_TILE = 256;       // positions per scores / P.V item (one per thread)
constexpr int MK_MAX_HD = 128;
constexpr int MK_MAX_H = 8192;     // largest hidden size (normed x lives in shared memory)

__device__ __forceinline__ float ldcg_f(const float *p) { return __ldcg(p); }
__device__ __forceinline__ float ldcg_bf(const bf16 *p) {
    return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short *>(p))));
}
__device__ __forceinline__ bf16x8 ldcg128(const void *p) {
    uint4 u = __ldcg(reinterpret_cast<const uint4 *>(p));
    return *reinterpret_cast<bf16x8 *>(&u);
}
__device__ __forceinline__ uint4 ldg_stream(const void *p, uint64_t policy) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}

// Grid barrier. Returns false once any CTA has recorded an error (a timed-out wait here or a
// range error elsewhere): every CTA then leaves at its next barrier.
__device__ bool grid_sync(unsigned *bar) {
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned *gen = bar + 1;
        volatile unsigned *err = bar + 2;
        const unsigned my = *gen;
        __threadfence();
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            // poll the generation with acquire loads and a short back-off, so that the waiting
            // CTAs do not crowd the arrivals at the same L2 line
            const uint64_t t0 = globaltimer();
            unsigned g;
            while (true) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar + 1) : "memory");
                if (g != my || *err != 0) break;
                __nanosleep(64);
                if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                    atomicOr(bar + 2, 1u);
                    atomicOr(&g_dev_error, DEV_ERR_WAIT_TIMEOUT);
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
    return *(volatile unsigned *)(bar + 2) == 0;
}

// y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w) into shared memory: src/kernels.cu:25-71 with
// 256 threads, thread i summing x[i], x[i + 256], ... serially, an xor tree per warp, then the
// eight warp sums in order.
__device__ __noinline__ void block_rmsnorm(const bf16 *x, const bf16 *w, bf16 *out, int dim, float eps, float *warp_sums) {
    float sum = 0.0f;
    for (int i = threadIdx.x; i < dim; i += MK_THREADS) {
        const float v = ldcg_bf(x + i);
        sum = __fmaf_rn(v, v, sum);
    }
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (threadIdx.x % 32 == 0) warp_sums[threadIdx.x / 32] = sum;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int wi = 0; wi < MK_WARPS; wi++) total += warp_sums[wi];
    const float inv_rms = rsqrtf(total / dim + eps);
    for (int i = threadIdx.x; i < dim; i += MK_THREADS) {
        const bf16 normed = __float2bfloat16(ldcg_bf(x + i) * inv_rms);
        out[i] = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(w[i]));
    }
    __syncthreads();
}

// One row's dot product, the reference warp_dot order; the result is valid in lane 0. x is in
// shared memory (x_shared) or global memory written in this kernel.
template <int UR>
__device__ __noinline__ float warp_row_ur(const bf16 *wrow, const bf16 *x, bool x_shared, int n_vec, int lane,
                                          uint64_t policy) {
    const uint4 *wv = reinterpret_cast<const uint4 *>(wrow);
    float acc = 0.0f;
    for (int r0 = 0; 32 * r0 < n_vec; r0 += UR) {
        uint4 w[UR];
#pragma unroll
        for (int j = 0; j < UR; j++) {
            const int i = lane + 32 * (r0 + j);
            if (i < n_vec) w[j] = ldg_stream(wv + i, policy);
        }
#pragma unroll
        for (int j = 0; j < UR; j++) {
            const int i = lane + 32 * (r0 + j);
            if (i < n_vec) {
                const bf16x8 xc = x_shared ? lds128(x + i * 8) : ldcg128(x + i * 8);
                acc = dot8(*reinterpret_cast<const bf16x8 *>(&w[j]), xc, acc);
            }
        }
    }
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, off);
    return acc;
}

__device__ __forceinline__ float warp_row(const bf16 *wrow, const bf16 *x, bool x_shared, int n_vec, int lane,
                                          uint64_t policy) {
    return warp_row_ur<MK_UR>(wrow, x, x_shared, n_vec, lane, policy);
}

template <int NREP>
__global__ void __launch_bounds__(MK_THREADS, MK_MIN_CTAS) decode_b1_kernel(const __grid_constant__ MkParams a) {
    __shared__ __align__(16) bf16 xs[MK_MAX_H];                 // normed activations
    __shared__ __align__(16) float q_s[NREP * MK_MAX_HD];       // scores: the group's queries
    __shared__ __align__(16) float p_s[NREP * MK_TILE];         // P.V: the item's probabilities
    __shared__ float red[32];
    __shared__ bf16 head_s[MK_THREADS];
    __shared__ float m_s[NREP], sum_s[NREP];

    const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
    const int gw = blockIdx.x * MK_WARPS + warp, nw = gridDim.x * MK_WARPS;
    const uint64_t policy = policy_evict_first();
    const int H = a.H, hd = a.hd, qd = a.n_heads * hd, kvd = a.n_kv * hd;
    unsigned *bar = a.bar;

    const int token = __ldcg(a.next_token);
    const int pos = __ldcg(a.pos);
    if (token < 0 || token >= a.vocab || pos < 0 || pos >= a.max_seq) {
        if (blockIdx.x == 0 && tid == 0) {
            atomicOr(&g_dev_error, token < 0 || token >= a.vocab ? DEV_ERR_TOKEN_RANGE : DEV_ERR_POS_RANGE);
            atomicOr(bar + 2, 1u);
        }
        return;  // every CTA takes this branch: the same values are read by all
    }
    const int len = pos + 1;
    const int n_items = a.n_kv * ((len + MK_TILE - 1) / MK_TILE);

    // ---- embedding (src/kernels.cu:7-23)
    for (int i = blockIdx.x * MK_THREADS + tid; i < H; i += gridDim.x * MK_THREADS) a.x[i] = a.embed[(size_t)token * H + i];
    if (!grid_sync(bar)) return;

    for (int l = 0; l < a.n_layers; l++) {
        const MkLayer &w = a.layers[l];
        bf16 *kc = a.key_cache + (size_t)l * a.layer_stride;
        bf16 *vc = a.value_cache + (size_t)l * a.layer_stride;
        const size_t head_stride = (size_t)a.max_seq * hd;

        // ---- attention norm + q, k, v (src/kernels.cu:215-257)
        block_rmsnorm(a.x, w.attn_norm, xs, H, a.eps, red);
        for (int r = gw; r < qd + 2 * kvd; r += nw) {
            const bf16 *wr;
            bf16 *o;
            if (r < qd) {
                wr = w.wq + (size_t)r * H;
                o = a.q + r;
            } else if (r < qd + kvd) {
                wr = w.wk + (size_t)(r - qd) * H;
                o = a.k + (r - qd);
            } else {
                wr = w.wv + (size_t)(r - qd - kvd) * H;
                o = a.v + (r - qd - kvd);
            }
            const float y = warp_row(wr, xs, true, H / 8, lane, policy);
            if (lane == 0) *o = __float2bfloat16(y);
        }
        if (!grid_sync(bar)) return;

        // ---- qk norm, RoPE, KV write (src/kernels.cu:301-403): head_dim threads per head
        {
            const int hpc = MK_THREADS / hd;  // heads per CTA round
            const int sub = tid / hd, i = tid % hd, hw = hd / 32;
            for (int h0 = blockIdx.x * hpc; h0 < a.n_heads + a.n_kv; h0 += gridDim.x * hpc) {
                const int head_all = h0 + sub;
                const bool act = head_all < a.n_heads + a.n_kv;
                const bool is_key = head_all >= a.n_heads;
                const int head = is_key ? head_all - a.n_heads : head_all;
                bf16 *xh = act ? (is_key ? a.k + head * hd : a.q + head * hd) : nullptr;
                const bf16 *nw_ = is_key ? w.k_norm : w.q_norm;
                const float xi = act ? ldcg_bf(xh + i) : 0.0f;
                float sum = xi * xi;
                for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                if (lane == 0) red[warp] = sum;
                __syncthreads();
                float total = 0.0f;
                for (int wi = 0; wi < hw; wi++) total += red[sub * hw + wi];
                const float inv_rms = rsqrtf(total / hd + a.eps);
                const bf16 normed = __float2bfloat16(xi * inv_rms);
                head_s[tid] = __float2bfloat16(__bfloat162float(normed) * __bfloat162float(nw_[i]));
                __syncthreads();
                const int half = hd / 2;
                if (act && i < half) {
                    const float inv_freq = 1.0f / powf(a.theta, (float)(2 * i) / hd);
                    const float angle = pos * inv_freq;
                    const float c = round_bf16(cosf(angle));
                    const float s = round_bf16(sinf(angle));
                    const float av = __bfloat162float(head_s[sub * hd + i]);
                    const float bv = __bfloat162float(head_s[sub * hd + i + half]);
                    const bf16 out_a = __float2bfloat16(round_bf16(av * c) - round_bf16(bv * s));
                    const bf16 out_b = __float2bfloat16(round_bf16(bv * c) + round_bf16(av * s));
                    xh[i] = out_a;
                    xh[i + half] = out_b;
                    if (is_key) {
                        const size_t slot = (size_t)head * head_stride + (size_t)pos * hd;
                        kc[slot + i] = out_a;
                        kc[slot + i + half] = out_b;
                    }
                }
                if (act && is_key)
                    vc[(size_t)head * head_stride + (size_t)pos * hd + i] =
                        __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short *>(a.v + head * hd + i)));
                __syncthreads();
            }
        }
        if (!grid_sync(bar)) return;

        // ---- scores: one position per thread, the serial dot over head_dim
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            const int kvh = it % a.n_kv, tile = it / a.n_kv;
            for (int j = tid; j < NREP * hd; j += MK_THREADS) q_s[j] = ldcg_bf(a.q + (size_t)kvh * NREP * hd + j);
            __syncthreads();
            const int t = tile * MK_TILE + tid;
            if (t < len) {
                const bf16 *krow = kc + (size_t)kvh * head_stride + (size_t)t * hd;
                float acc[NREP];
#pragma unroll
                for (int h = 0; h < NREP; h++) acc[h] = 0.0f;
                for (int c0 = 0; c0 < hd / 8; c0 += 8) {  // eight 16-byte chunks of the row in flight
                    bf16x8 kv8[8];
#pragma unroll
                    for (int u = 0; u < 8; u++)
                        if (c0 + u < hd / 8) kv8[u] = ldcg128(krow + (c0 + u) * 8);
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        if (c0 + u >= hd / 8) continue;
                        const int ch = c0 + u;
                        float kf[8];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float2 f = __bfloat1622float2(kv8[u].h[e]);
                            kf[2 * e] = f.x;
                            kf[2 * e + 1] = f.y;
                        }
#pragma unroll
                        for (int h = 0; h < NREP; h++)
#pragma unroll
                            for (int e = 0; e < 8; e++) acc[h] = __fmaf_rn(q_s[h * hd + ch * 8 + e], kf[e], acc[h]);
                    }
                }
#pragma unroll
                for (int h = 0; h < NREP; h++)
                    a.scores[(size_t)(kvh * NREP + h) * a.ld + t] = round_bf16(round_bf16(acc[h]) * a.scale);
            }
            __syncthreads();
        }
        if (!grid_sync(bar)) return;

        // ---- softmax statistics: 128 threads per head, the reference's slot order
        for (int h0 = blockIdx.x * 2; h0 < a.n_heads; h0 += gridDim.x * 2) {
            const int sub = tid / 128, j = tid % 128, h = h0 + sub;
            const bool act = h < a.n_heads;
            const float *sc = a.scores + (size_t)(act ? h : 0) * a.ld;
            float mx = -INFINITY;
            if (act)
                for (int t = j; t < len; t += 128) mx = fmaxf(mx, ldcg_f(sc + t));
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            if (lane == 0) red[warp] = mx;
            __syncthreads();
            float m = -INFINITY;
            for (int wi = 0; wi < 4; wi++) m = fmaxf(m, red[sub * 4 + wi]);
            __syncthreads();
            float sm = 0.0f;
            if (act)
                for (int t = j; t < len; t += 128) sm += expf(ldcg_f(sc + t) - m);
            for (int off = 16; off > 0; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
            if (lane == 0) red[warp] = sm;
            __syncthreads();
            float s = 0.0f;
            for (int wi = 0; wi < 4; wi++) s += red[sub * 4 + wi];
            if (act && j == 0) {
                a.stats[2 * h] = m;
                a.stats[2 * h + 1] = s;
            }
            __syncthreads();
        }
        if (!grid_sync(bar)) return;

        // ---- P.V: item = (kv head, 256 positions); threads (half, dim) sum 128 positions each
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
            const int kvh = it % a.n_kv, tile = it / a.n_kv;
            const int t0 = tile * MK_TILE;
            if (tid < NREP) {
                m_s[tid] = ldcg_f(a.stats + 2 * (kvh * NREP + tid));
                sum_s[tid] = ldcg_f(a.stats + 2 * (kvh * NREP + tid) + 1);
            }
            __syncthreads();
            for (int j = tid; j < NREP * MK_TILE; j += MK_THREADS) {
                const int h = j / MK_TILE, t = j % MK_TILE;
                p_s[j] = t0 + t < len
                             ? round_bf16(expf(ldcg_f(a.scores + (size_t)(kvh * NREP + h) * a.ld + t0 + t) - m_s[h]) / sum_s[h])
                             : 0.0f;
            }
            __syncthreads();
            const int half = tid / hd, d = tid % hd;  // hd = 128: halves 0 and 1; hd = 64: four quarters
            const int parts = MK_THREADS / hd, span = MK_TILE / parts;
            const int ta = half * span, tb = min(ta + span, len - t0);
            float acc[NREP];
#pragma unroll
            for (int h = 0; h < NREP; h++) acc[h] = 0.0f;
            const bf16 *vcol = vc + (size_t)kvh * head_stride + (size_t)t0 * hd + d;
            int t = ta;
            for (; t + 8 <= tb; t += 8) {
                float vv[8];
#pragma unroll
                for (int u = 0; u < 8; u++) vv[u] = ldcg_bf(vcol + (size_t)(t + u) * hd);
#pragma unroll
                for (int u = 0; u < 8; u++)
#pragma unroll
                    for (int h = 0; h < NREP; h++) acc[h] = __fmaf_rn(p_s[h * MK_TILE + t + u], vv[u], acc[h]);
            }
            for (; t < tb; t++) {
                const float vv = ldcg_bf(vcol + (size_t)t * hd);
#pragma unroll
                for (int h = 0; h < NREP; h++) acc[h] = __fmaf_rn(p_s[h * MK_TILE + t], vv, acc[h]);
            }
            // partial number tile * parts + half: position order
#pragma unroll
            for (int h = 0; h < NREP; h++)
                a.partial[((size_t)(tile * parts + half) * a.n_heads + kvh * NREP + h) * hd + d] = acc[h];
            __syncthreads();
        }
        if (!grid_sync(bar)) return;

        // ---- combine the partial sums in position order
        {
            const int n_parts = ((len + MK_TILE - 1) / MK_TILE) * (MK_THREADS / hd);
            for (int o = blockIdx.x * MK_THREADS + tid; o < qd; o += gridDim.x * MK_THREADS) {
                float s = 0.0f;
                for (int pi = 0; pi < n_parts; pi++) s += ldcg_f(a.partial + (size_t)pi * qd + o);
                a.attn_out[o] = __float2bfloat16(s);
            }
        }
        if (!grid_sync(bar)) return;

        // ---- o_proj + residual (src/kernels.cu:185-212)
        for (int r = gw; r < H; r += nw) {
            const float y = warp_row(w.wo + (size_t)r * qd, a.attn_out, false, qd / 8, lane, policy);
            if (lane == 0) {
                const bf16 yb = __float2bfloat16(y);
                a.x[r] = __float2bfloat16(ldcg_bf(a.x + r) + __bfloat162float(yb));
            }
        }
        if (!grid_sync(bar)) return;

        // ---- MLP norm + gate/up with SwiGLU (src/kernels.cu:260-298)
        block_rmsnorm(a.x, w.mlp_norm, xs, H, a.eps, red);
        for (int r = gw; r < a.I; r += nw) {
            const float g = warp_row(w.w_gate + (size_t)r * H, xs, true, H / 8, lane, policy);
            const float u = warp_row(w.w_up + (size_t)r * H, xs, true, H / 8, lane, policy);
            if (lane == 0) {
                const float gv = __bfloat162float(__float2bfloat16(g));
                const float uv = __bfloat162float(__float2bfloat16(u));
                a.act[r] = __float2bfloat16(round_bf16(gv / (1.0f + expf(-gv))) * uv);
            }
        }
        if (!grid_sync(bar)) return;

        // ---- down + residual
        for (int r = gw; r < H; r += nw) {
            const float y = warp_row(w.w_down + (size_t)r * a.I, a.act, false, a.I / 8, lane, policy);
            if (lane == 0) {
                const bf16 yb = __float2bfloat16(y);
                a.x[r] = __float2bfloat16(ldcg_bf(a.x + r) + __bfloat162float(yb));
            }
        }
        if (!grid_sync(bar)) return;
    }

    // ---- final norm + LM head (src/forward.cu:188-191)
    block_rmsnorm(a.x, a.final_norm, xs, H, a.eps, red);
    for (int r = gw; r < a.vocab; r += nw) {
        const float y = warp_row(a.lm_head + (size_t)r * H, xs, true, H / 8, lane, policy);
        if (lane == 0) a.logits[r] = __float2bfloat16(y);
    }
    if (!grid_sync(bar)) return;

    // ---- argmax (src/kernels.cu:500-544): larger value, lower index on ties, NaN never wins
    {
        float best = -INFINITY;
        int bi = 0x7fffffff;
        const int per = (a.vocab + gridDim.x - 1) / gridDim.x;
        const int lo = blockIdx.x * per, hi = min(lo + per, a.vocab);
        for (int i = lo + tid; i < hi; i += MK_THREADS) {
            const float v = ldcg_bf(a.logits + i);
            if (v > best || (v == best && i < bi)) {
                best = v;
                bi = i;
            }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > best || (ov == best && oi < bi)) {
                best = ov;
                bi = oi;
            }
        }
        __shared__ float bv_s[MK_WARPS];
        __shared__ int bi_s[MK_WARPS];
        if (lane == 0) {
            bv_s[warp] = best;
            bi_s[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            for (int wi = 1; wi < MK_WARPS; wi++)
                if (bv_s[wi] > best || (bv_s[wi] == best && bi_s[wi] < bi)) {
                    best = bv_s[wi];
                    bi = bi_s[wi];
                }
            a.amax_val[blockIdx.x] = best;
            a.amax_idx[blockIdx.x] = bi;
        }
    }
    if (!grid_sync(bar)) return;
    if (blockIdx.x == 0 && tid == 0) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (unsigned c = 0; c < gridDim.x; c++) {
            const float v = ldcg_f(a.amax_val + c);
            const int i = __ldcg(a.amax_idx + c);
            if (v > best || (v == best && i < bi)) {
                best = v;
                bi = i;
            }
        }
        if (bi == 0x7fffffff) bi = 0;  // every logit NaN: the reference's initial index
        *a.out_token = bi;
        *a.next_token = bi;
        const int st = *a.step;
        if (a.history && st >= 0 && st < a.history_cap) a.history[st] = bi;
        *a.step = st + 1;
        *a.pos = pos + 1;
    }
}

}  // namespace

// Host side: the number of co-resident CTAs (the grid) for the group size, and the cooperative
// launch, which guarantees that all CTAs of the grid run at once.
int megakernel_grid(int nrep) {
    int n = 0;
    cudaError_t e;
    switch (nrep) {
        case 1: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_b1_kernel<1>, MK_THREADS, 0); break;
        case 2: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_b1_kernel<2>, MK_THREADS, 0); break;
        case 4: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_b1_kernel<4>, MK_THREADS, 0); break;
        case 8: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_b1_kernel<8>, MK_THREADS, 0); break;
        default: return 0;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n * num_sms();
}

template <int NREP>
int launch_mk(const MkParams &p, int grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return record_cuda_error(cudaLaunchKernelEx(&cfg, decode_b1_kernel<NREP>, p));
}

int megakernel_launch(const MkParams &p, int nrep, int grid, cudaStream_t s) {
    if (grid <= 0) return Q3_ERR_SHAPE;
    switch (nrep) {
        case 1: return launch_mk<1>(p, grid, s);
        case 2: return launch_mk<2>(p, grid, s);
        case 4: return launch_mk<4>(p, grid, s);
        case 8: return launch_mk<8>(p, grid, s);
        default: return Q3_ERR_SHAPE;
    }
}

unsigned take_error_megakernel() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

}  // namespace q3
