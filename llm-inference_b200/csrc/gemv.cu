// Batch-1 GEMV family for sm_100a: gemv (LM head), gemv_residual, qkv and gate_up.
//
// Arithmetic: bit-identical to the reference's warp-per-row kernels (src/kernels.cu:79-298).
// Each output row is computed by one warp; lane l accumulates the 16-byte chunks l, l+32,
// l+64, ... of the row in order with one fused multiply-add per element, then the warp
// reduces with the same __shfl_down_sync tree, and lane 0 rounds to bf16 at the reference's
// points. Splitting a row into column segments keeps that order because every segment but
// the last is a multiple of 32 chunks.
//
// Memory pipeline (what is new): persistent warps, each owning output rows w, w + W, ... (W =
// warps of the grid, sized to what is resident). The warps of a CTA take consecutive rows, so
// each SM streams contiguous slabs of the matrix: measured faster, chained in a decode
// step, than spreading every SM's rows over the whole matrix to even out the rows per SM. A warp loads up to GV_U 16-byte chunks per lane
// of its row at once (8 KB of one row per warp in flight) with streaming loads that bypass L1
// and are marked evict-first in L2, then runs the reference's FMA chain over them. The first
// batch of a warp's first row is loaded before the programmatic-dependency wait, because weights
// never depend on the previous kernel, and the next row's first batch is loaded before the
// current row's reduction and store.
//
// The input vector x is the previous launch's output. After the programmatic-dependency wait every
// CTA copies it into shared memory with cp.async, all of its 16-byte pieces in flight at once (one
// round trip to L2), and the dot products read it from there: read from global memory inside the
// dot loop, its loads serialized behind the register-bound weight batch, it cost the residual
// projections about half their time in a decode step (o_proj 7.7 us and down 15.9 us per layer
// after the wait at batch 1, against rooflines of 3.2 and 7.6). Vectors wider than GV_X_MAX_COLS
// stay in global memory.
//
// Fused RMSNorm (NORM): when the projection's input is rmsnorm(x) (qkv, gate_up and the LM head
// take the normed residual stream), every CTA recomputes the normed vector itself into shared
// memory, with the reference rmsnorm_kernel's arithmetic (src/kernels.cu:25-71: 256 threads,
// thread t summing x[t], x[t + 256], ... with fused multiply-adds, an xor tree per warp, the eight
// warp sums in order, then bf16(bf16(x * inv_rms) * w)), from the staged copy of x; the norm weight
// is staged before the programmatic-dependency wait. The separate rmsnorm launch and its
// dependency hop disappear; the extra reads (x and the weight, a few KB per CTA) come from L2.
#include <algorithm>

#include "common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

// Threads per CTA. The residual projections (o_proj, down) run 4-warp CTAs, measured faster than 8
// in the chained batch-1 step (the next kernel's CTAs take an SM's slots as soon as a few warps of
// the previous one are done); the others keep 8, where the in-kernel rmsnorm costs per CTA.
constexpr int GV_THREADS = 256;
constexpr int GV_THREADS_RESIDUAL = 128;
#ifndef Q3_GEMV_LONG_ROWS
#define Q3_GEMV_LONG_ROWS 1
#endif
// UR: chunk rounds (one 16-byte chunk per lane each) per batch and row; a unit's batch holds
// RPU * UR chunks per lane. The host picks the smallest UR in {8, 10, 12, 16} that covers a row in
// one batch, else 16 (8 for gate_up, whose batches hold two rows).

enum Epi : int { PLAIN = 0, RESIDUAL = 1, QKV = 2, GATE_UP = 3 };

struct GemvArgs {
    const bf16 *w0, *w1, *w2;  // PLAIN/RESIDUAL: w0; QKV: wq, wk, wv; GATE_UP: w_gate, w_up
    const bf16 *x;             // input vector [cols]
    bf16 *out0, *out1, *out2;  // PLAIN: out; RESIDUAL: residual x (read-modify-write); QKV: q, k, v; GATE_UP: act
    bf16 *tap0, *tap1;         // RESIDUAL: tap; GATE_UP: gate_tap, up_tap
    int rows0, rows1;          // QKV: q_rows, kv_rows
    int units;                 // output rows
    int cols;
    const bf16 *norm_w;        // NORM: rmsnorm weight [cols]; x is then the raw residual stream
    float eps;
};

constexpr int GV_NORM_MAX_COLS = 8192;   // NORM: the weight and x, then the normed x, in shared memory
constexpr int GV_X_MAX_COLS = 16384;     // x staged in shared memory up to this width

// How a kernel reads its input vector.
enum XMode : int { X_GLOBAL = 0, X_STAGED = 1, X_NORM = 2 };

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

template <int EPI>
__device__ __forceinline__ const bf16 *unit_row(const GemvArgs &a, int u, int r) {
    if (EPI == QKV) {
        if (u < a.rows0) return a.w0 + (size_t)u * a.cols;
        u -= a.rows0;
        if (u < a.rows1) return a.w1 + (size_t)u * a.cols;
        return a.w2 + (size_t)(u - a.rows1) * a.cols;
    }
    if (EPI == GATE_UP) return (r == 0 ? a.w0 : a.w1) + (size_t)u * a.cols;
    return a.w0 + (size_t)u * a.cols;
}

// 16-byte streaming load: no L1 allocation, evict-first in L2.
__device__ __forceinline__ uint4 ldg_stream(const void *p, uint64_t policy) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}

template <int EPI, int UR, int XMODE, int THREADS, int MINB>
__global__ void __launch_bounds__(THREADS, MINB) gemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr bool NORM = XMODE == X_NORM;
    constexpr int REF = 256;                      // the reference rmsnorm's block
    constexpr int NREF = REF / THREADS;           // reference threads each thread stands in for
    static_assert(REF % THREADS == 0, "the rmsnorm order needs a divisor of 256 threads");
    constexpr int RPU = EPI == GATE_UP ? 2 : 1;  // weight rows per output unit
    // X_STAGED: [cols] x; NORM: [cols] the norm weight, then the normed x, and [cols] x
    extern __shared__ __align__(16) bf16 xs[];
    __shared__ float warp_sums[REF / 32];
    const int lane = threadIdx.x % 32;
    const int nw = gridDim.x * (THREADS / 32);
    const int n_vec = a.cols / 8;
    const uint64_t policy = policy_evict_first();
    uint4 w[RPU][UR];
    // rounds r0 .. r0 + UR - 1 of unit u: chunk lane + 32 * round of each of its rows
    auto load_batch = [&](int u, int r0) {
#pragma unroll
        for (int r = 0; r < RPU; r++) {
            const uint4 *row = reinterpret_cast<const uint4 *>(unit_row<EPI>(a, u, r));
#pragma unroll
            for (int j = 0; j < UR; j++) {
                const int i = lane + 32 * (r0 + j);
                if (i < n_vec) w[r][j] = ldg_stream(row + i, policy);
            }
        }
    };

    int u = blockIdx.x * (THREADS / 32) + threadIdx.x / 32;
    pdl_trigger();
    if (u < a.units) load_batch(u, 0);
    if (NORM)
        for (int i = threadIdx.x; i < a.cols; i += THREADS) xs[i] = a.norm_w[i];
    pdl_wait();
    bf16 *xraw = NORM ? xs + a.cols : xs;  // the staged x
    if (XMODE != X_GLOBAL) {
        const uint4 *xg = reinterpret_cast<const uint4 *>(a.x);
        for (int i = threadIdx.x; i < n_vec; i += THREADS) cp_async16(reinterpret_cast<uint4 *>(xraw) + i, xg + i);
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
        __syncthreads();
    }
    if (NORM) {
        // reference thread r = threadIdx.x + k * THREADS sums x[r], x[r + 256], ... (accumulator k)
        float sum[NREF];
#pragma unroll
        for (int k = 0; k < NREF; k++) sum[k] = 0.0f;
#pragma unroll 8
        for (int i0 = 0; i0 < a.cols; i0 += REF)
#pragma unroll
            for (int k = 0; k < NREF; k++) {
                const int i = i0 + threadIdx.x + k * THREADS;
                if (i < a.cols) {
                    const float v = __bfloat162float(xraw[i]);
                    sum[k] = __fmaf_rn(v, v, sum[k]);
                }
            }
#pragma unroll
        for (int k = 0; k < NREF; k++) {  // reference warp threadIdx.x / 32 + k * THREADS / 32
            for (int off = 16; off > 0; off >>= 1) sum[k] += __shfl_xor_sync(0xffffffffu, sum[k], off);
            if (lane == 0) warp_sums[threadIdx.x / 32 + k * (THREADS / 32)] = sum[k];
        }
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w_ = 0; w_ < REF / 32; w_++) total += warp_sums[w_];
        const float inv_rms = rsqrtf(total / a.cols + a.eps);
        // bf16(bf16(x * inv_rms) * w), eight elements per thread and step (an element's value does not
        // depend on which thread computes it)
        for (int c = threadIdx.x; c < n_vec; c += THREADS) {
            const bf16x8 xr = lds128(xraw + 8 * c), wr = lds128(xs + 8 * c);
            bf16x8 o;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 xf = __bfloat1622float2(xr.h[e]), wf = __bfloat1622float2(wr.h[e]);
                const float n0 = round_bf16(xf.x * inv_rms), n1 = round_bf16(xf.y * inv_rms);
                o.h[e] = __floats2bfloat162_rn(n0 * wf.x, n1 * wf.y);
            }
            *reinterpret_cast<bf16x8 *>(xs + 8 * c) = o;
        }
        __syncthreads();
    }
    const uint4 *xv = reinterpret_cast<const uint4 *>(XMODE == X_GLOBAL ? a.x : xs);
    for (; u < a.units; u += nw) {
        float acc[RPU];
#pragma unroll
        for (int r = 0; r < RPU; r++) acc[r] = 0.0f;
        for (int r0 = 0; 32 * r0 < n_vec; r0 += UR) {
            if (r0 > 0) load_batch(u, r0);
#pragma unroll
            for (int j = 0; j < UR; j++) {
                const int i = lane + 32 * (r0 + j);
                if (i < n_vec) {
                    const bf16x8 xc = XMODE == X_GLOBAL ? ldg128(xv + i) : lds128(xv + i);
#pragma unroll
                    for (int r = 0; r < RPU; r++) acc[r] = dot8(*reinterpret_cast<const bf16x8 *>(&w[r][j]), xc, acc[r]);
                }
            }
        }
        if (u + nw < a.units) load_batch(u + nw, 0);  // in flight during the reduction and store
#pragma unroll
        for (int r = 0; r < RPU; r++)
            for (int off = 16; off > 0; off >>= 1) acc[r] += __shfl_down_sync(0xffffffffu, acc[r], off);
        if (lane != 0) continue;
        if (EPI == PLAIN) {
            a.out0[u] = __float2bfloat16(acc[0]);
        } else if (EPI == RESIDUAL) {
            const bf16 y = __float2bfloat16(acc[0]);
            if (a.tap0 != nullptr) a.tap0[u] = y;
            a.out0[u] = __float2bfloat16(__bfloat162float(a.out0[u]) + __bfloat162float(y));
        } else if (EPI == QKV) {
            const bf16 y = __float2bfloat16(acc[0]);
            if (u < a.rows0) a.out0[u] = y;
            else if (u < a.rows0 + a.rows1) a.out1[u - a.rows0] = y;
            else a.out2[u - a.rows0 - a.rows1] = y;
        } else {
            const bf16 gate = __float2bfloat16(acc[0]);
            const bf16 up = __float2bfloat16(acc[RPU - 1]);
            if (a.tap0 != nullptr) {
                a.tap0[u] = gate;
                a.tap1[u] = up;
            }
            const float gv = __bfloat162float(gate);
            const float uv = __bfloat162float(up);
            const float silu = round_bf16(gv / (1.0f + expf(-gv)));
            a.out0[u] = __float2bfloat16(silu * uv);
        }
    }
}

bool aligned16(const void *p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int EPI, int UR, int XMODE, int MINB = 1>
int launch_gemv_x(const GemvArgs &a, cudaStream_t stream) {
    constexpr int THREADS = EPI == RESIDUAL ? GV_THREADS_RESIDUAL : GV_THREADS;
    static int per_sm[64] = {};  // resident CTAs per SM, by device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return Q3_ERR_DEVICE;
    // occupancy counted at the largest staged vector, so one grid size fits every width
    const size_t smem = XMODE == X_NORM ? (size_t)a.cols * 4 : XMODE == X_STAGED ? (size_t)a.cols * 2 : 0;
    const size_t smem_plan = XMODE == X_NORM     ? (size_t)GV_NORM_MAX_COLS * 4
                             : XMODE == X_STAGED ? (size_t)GV_X_MAX_COLS * 2
                                                 : 0;
    if (per_sm[dev] == 0) {
        Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(gemv_kernel<EPI, UR, XMODE, THREADS, MINB>), smem_plan));
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_kernel<EPI, UR, XMODE, THREADS, MINB>, THREADS,
                                                          smem_plan) !=
                cudaSuccess ||
            n < 1)
            n = 1;
        cudaGetLastError();
        per_sm[dev] = n;
    }
    const long long want = (a.units + THREADS / 32 - 1) / (THREADS / 32);
    const int grid = (int)std::min<long long>(want, (long long)num_sms() * per_sm[dev]);
    Q3_TRY_LAUNCH(launch(gemv_kernel<EPI, UR, XMODE, THREADS, MINB>, dim3(grid), dim3(THREADS), smem, stream, 1, a));
    return Q3_OK;
}

template <int EPI, int UR, int MINB = 1>
int launch_gemv_ur(const GemvArgs &a, cudaStream_t stream) {
    if (a.norm_w) return launch_gemv_x<EPI, UR, X_NORM, MINB>(a, stream);
    if (a.cols <= GV_X_MAX_COLS) return launch_gemv_x<EPI, UR, X_STAGED, MINB>(a, stream);
    return launch_gemv_x<EPI, UR, X_GLOBAL, MINB>(a, stream);
}

template <int EPI>
int launch_gemv(GemvArgs a, cudaStream_t stream) {
    if (a.units <= 0 || a.cols <= 0) return a.units == 0 ? Q3_OK : Q3_ERR_SHAPE;
    if (a.cols % 8 != 0) return Q3_ERR_SHAPE;
    if (a.norm_w && (a.cols > GV_NORM_MAX_COLS || (reinterpret_cast<uintptr_t>(a.norm_w) & 15))) return Q3_ERR_SHAPE;
    const int rounds = (a.cols / 8 + 31) / 32;
    if (rounds <= 8) return launch_gemv_ur<EPI, 8>(a, stream);
    // 2560-wide rows (Qwen3-4B's hidden size) take 10 rounds: a batch of exactly 10 keeps gate_up at
    // 117 registers, two CTAs (16 warps) per SM instead of one, and qkv and the LM head at three
    if (rounds <= 10) return launch_gemv_ur<EPI, 10>(a, stream);
    if (rounds <= 12) return launch_gemv_ur<EPI, 12>(a, stream);
    if constexpr (EPI == RESIDUAL) {
        if (rounds <= 16) return launch_gemv_ur<EPI, 16, 5>(a, stream);
#if Q3_GEMV_LONG_ROWS
        // long rows (down_proj: 38 rounds): 20 chunks per lane in flight, two batches a row instead
        // of three; at most 102 registers keep 5 CTAs (20 warps) per SM, one row per warp
        if (rounds <= 40) return launch_gemv_ur<EPI, 20, 5>(a, stream);
#endif
    }
    if constexpr (EPI == GATE_UP) {
        return launch_gemv_ur<EPI, 8>(a, stream);  // two rows: 16 chunks a batch
    } else {
        return launch_gemv_ur<EPI, 16>(a, stream);
    }
}

}  // namespace

unsigned take_error_gemv() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

// The _n variants take an optional rmsnorm: with norm_w, the input is rmsnorm(x, norm_w, eps),
// computed in the kernel.
int gemv_plain_n(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t s, const bf16 *norm_w,
                 float eps) {
    if (!out || !w || !x) return Q3_ERR_ARG;
    if (!aligned16(w) || !aligned16(x)) return Q3_ERR_ALIGN;
    GemvArgs a = {};
    a.norm_w = norm_w;
    a.eps = eps;
    a.w0 = w;
    a.x = x;
    a.out0 = out;
    a.units = rows;
    a.cols = cols;
    return launch_gemv<PLAIN>(a, s);
}

int gemv_residual(bf16 *x, const bf16 *w, const bf16 *in, int rows, int cols, bf16 *tap,
                  cudaStream_t s) {
    if (!x || !w || !in) return Q3_ERR_ARG;
    if (!aligned16(w) || !aligned16(in)) return Q3_ERR_ALIGN;
    GemvArgs a = {};
    a.w0 = w;
    a.x = in;
    a.out0 = x;
    a.tap0 = tap;
    a.units = rows;
    a.cols = cols;
    return launch_gemv<RESIDUAL>(a, s);
}

int gemv_qkv_n(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv,
               const bf16 *x, int q_rows, int kv_rows, int cols, cudaStream_t s, const bf16 *norm_w, float eps) {
    if (!q || !k || !v || !wq || !wk || !wv || !x) return Q3_ERR_ARG;
    if (!aligned16(wq) || !aligned16(wk) || !aligned16(wv) || !aligned16(x)) return Q3_ERR_ALIGN;
    if (q_rows < 0 || kv_rows < 0) return Q3_ERR_SHAPE;
    GemvArgs a = {};
    a.norm_w = norm_w;
    a.eps = eps;
    a.w0 = wq;
    a.w1 = wk;
    a.w2 = wv;
    a.x = x;
    a.out0 = q;
    a.out1 = k;
    a.out2 = v;
    a.rows0 = q_rows;
    a.rows1 = kv_rows;
    a.units = q_rows + 2 * kv_rows;
    a.cols = cols;
    return launch_gemv<QKV>(a, s);
}

int gemv_gate_up_n(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                   bf16 *gate_tap, bf16 *up_tap, cudaStream_t s, const bf16 *norm_w, float eps) {
    if (!act || !w_gate || !w_up || !x) return Q3_ERR_ARG;
    if ((gate_tap == nullptr) != (up_tap == nullptr)) return Q3_ERR_ARG;
    if (!aligned16(w_gate) || !aligned16(w_up) || !aligned16(x)) return Q3_ERR_ALIGN;
    GemvArgs a = {};
    a.norm_w = norm_w;
    a.eps = eps;
    a.w0 = w_gate;
    a.w1 = w_up;
    a.x = x;
    a.out0 = act;
    a.tap0 = gate_tap;
    a.tap1 = up_tap;
    a.units = rows;
    a.cols = cols;
    return launch_gemv<GATE_UP>(a, s);
}

int gemv_plain(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t s) {
    return gemv_plain_n(out, w, x, rows, cols, s, nullptr, 0.0f);
}

int gemv_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x, int q_rows,
             int kv_rows, int cols, cudaStream_t s) {
    return gemv_qkv_n(q, k, v, wq, wk, wv, x, q_rows, kv_rows, cols, s, nullptr, 0.0f);
}

int gemv_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                 bf16 *gate_tap, bf16 *up_tap, cudaStream_t s) {
    return gemv_gate_up_n(act, w_gate, w_up, x, rows, cols, gate_tap, up_tap, s, nullptr, 0.0f);
}

}  // namespace q3
