// Batch-1 GEMV family for sm_100a: gemv (LM head), gemv_residual, qkv and gate_up.
//
// Arithmetic: bit-identical to the reference's warp-per-row kernels (src/kernels.cu:79-298).
// Each output row is computed by one warp; lane l accumulates the 16-byte chunks l, l+32,
// l+64, ... of the row in order with one fused multiply-add per element, then the warp
// reduces with the same __shfl_down_sync tree, and lane 0 rounds to bf16 at the reference's
// points. Splitting a row into column segments keeps that order because every segment but
// the last is a multiple of 32 chunks.
//
// Memory pipeline (what is new): a persistent grid of one CTA per SM owns a balanced,
// contiguous range of output rows. A producer warp streams the CTA's weight rows through a
// ring of shared-memory stages with cp.async.bulk (completion on mbarriers), evict-first in
// L2, and starts doing so before the programmatic-dependency wait, because weights never
// depend on the previous kernel; eight consumer warps read the stages. The stage ring keeps
// ~64 KB of weights in flight per SM.
#include <algorithm>

#include "common.cuh"

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int WARPS = 8;                  // consumer warps; one output row each per group
constexpr int THREADS = (WARPS + 1) * 32;  // + one producer warp
constexpr int STAGES = 4;
constexpr int STAGE_TARGET_BYTES = 16384;

enum Epi : int { PLAIN = 0, RESIDUAL = 1, QKV = 2, GATE_UP = 3 };

struct GemvArgs {
    const bf16 *w0, *w1, *w2;  // PLAIN/RESIDUAL: w0; QKV: wq, wk, wv; GATE_UP: w_gate, w_up
    const bf16 *x;             // input vector [cols]
    bf16 *out0, *out1, *out2;  // PLAIN: out; RESIDUAL: residual x (read-modify-write); QKV: q, k, v; GATE_UP: act
    bf16 *tap0, *tap1;         // RESIDUAL: tap; GATE_UP: gate_tap, up_tap
    int rows0, rows1;          // QKV: q_rows, kv_rows
    int units;                 // output rows
    int cols;
    int seg_cols;              // columns per stage segment (a multiple of 256, or cols)
    int n_seg;
    int x_bytes;               // shared bytes reserved for x (cols * 2 rounded up)
};

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

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int RPU = EPI == GATE_UP ? 2 : 1;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + STAGES;
    bf16 *x_s = reinterpret_cast<bf16 *>(smem + 128);
    unsigned char *stages = smem + 128 + a.x_bytes;
    const size_t row_stride = (size_t)a.seg_cols * 2;  // bytes per row slot in a stage
    const size_t stage_bytes = (size_t)WARPS * RPU * row_stride;

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int u0 = (int)(((long long)a.units * blockIdx.x) / gridDim.x);
    const int u1 = (int)(((long long)a.units * (blockIdx.x + 1)) / gridDim.x);
    const int nu = u1 - u0;
    const int n_groups = (nu + WARPS - 1) / WARPS;
    const int n_items = n_groups * a.n_seg;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], WARPS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == WARPS) {
        // ---------------- producer: weights only, so it may run ahead of pdl_wait()
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            int it = 0;
            for (; it < n_items; it++) {
                const int slot = it % STAGES;
                if (it >= STAGES && !mbar_wait(&empty[slot], ((it / STAGES) - 1) & 1, &g_dev_error))
                    break;
                const int g = it / a.n_seg;
                const int s = it - g * a.n_seg;
                const int c0 = s * a.seg_cols;
                const uint32_t row_bytes = (uint32_t)min(a.seg_cols, a.cols - c0) * 2;
                const int gu = min(WARPS, nu - g * WARPS);
                mbar_arrive_expect_tx(&full[slot], (uint32_t)(gu * RPU) * row_bytes);
                unsigned char *st = stages + slot * stage_bytes;
                for (int w = 0; w < gu; w++) {
                    const int u = u0 + g * WARPS + w;
#pragma unroll
                    for (int r = 0; r < RPU; r++)
                        bulk_g2s_hint(st + (w * RPU + r) * row_stride, unit_row<EPI>(a, u, r) + c0,
                                      row_bytes, &full[slot], policy);
                }
            }
            // Do not leave while copies issued into this CTA's shared memory may be in flight.
            for (int j = max(0, it - STAGES); j < it; j++)
                mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &g_dev_error);
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();
    {
        const int n8 = a.cols / 8;
        const uint4 *xg = reinterpret_cast<const uint4 *>(a.x);
        uint4 *xs = reinterpret_cast<uint4 *>(x_s);
        for (int i = threadIdx.x; i < n8; i += WARPS * 32) xs[i] = xg[i];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(WARPS * 32) : "memory");

    for (int g = 0; g < n_groups; g++) {
        const int u = u0 + g * WARPS + warp;
        const bool active = u < u1;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int s = 0; s < a.n_seg; s++) {
            const int it = g * a.n_seg + s;
            const int slot = it % STAGES;
            if (!mbar_wait(&full[slot], (it / STAGES) & 1, &g_dev_error)) return;
            if (active) {
                const int c0 = s * a.seg_cols;
                const int nchunk = min(a.seg_cols, a.cols - c0) / 8;
                const unsigned char *row0 = stages + slot * stage_bytes + (warp * RPU) * row_stride;
                const bf16 *xs = x_s + c0;
                for (int i = lane; i < nchunk; i += 32) {
                    const bf16x8 xv = lds128(xs + i * 8);
                    acc0 = dot8(lds128(row0 + i * 16), xv, acc0);
                    if (EPI == GATE_UP) acc1 = dot8(lds128(row0 + row_stride + i * 16), xv, acc1);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (!active) continue;
        for (int off = 16; off > 0; off >>= 1) {
            acc0 += __shfl_down_sync(0xffffffffu, acc0, off);
            if (EPI == GATE_UP) acc1 += __shfl_down_sync(0xffffffffu, acc1, off);
        }
        if (lane != 0) continue;
        if (EPI == PLAIN) {
            a.out0[u] = __float2bfloat16(acc0);
        } else if (EPI == RESIDUAL) {
            const bf16 y = __float2bfloat16(acc0);
            if (a.tap0 != nullptr) a.tap0[u] = y;
            a.out0[u] = __float2bfloat16(__bfloat162float(a.out0[u]) + __bfloat162float(y));
        } else if (EPI == QKV) {
            const bf16 y = __float2bfloat16(acc0);
            if (u < a.rows0) a.out0[u] = y;
            else if (u < a.rows0 + a.rows1) a.out1[u - a.rows0] = y;
            else a.out2[u - a.rows0 - a.rows1] = y;
        } else {
            const bf16 gate = __float2bfloat16(acc0);
            const bf16 up = __float2bfloat16(acc1);
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

template <int EPI>
int launch_gemv(GemvArgs a, cudaStream_t stream) {
    constexpr int RPU = EPI == GATE_UP ? 2 : 1;
    if (a.units <= 0 || a.cols <= 0) return a.units == 0 ? Q3_OK : Q3_ERR_SHAPE;
    if (a.cols % 8 != 0) return Q3_ERR_SHAPE;
    int seg = (STAGE_TARGET_BYTES / (WARPS * RPU * 2)) / 256 * 256;
    seg = std::max(seg, 256);
    a.seg_cols = a.cols <= seg ? a.cols : seg;
    a.n_seg = (a.cols + a.seg_cols - 1) / a.seg_cols;
    a.x_bytes = (a.cols * 2 + 127) / 128 * 128;
    const size_t smem = 128 + (size_t)a.x_bytes + (size_t)STAGES * WARPS * RPU * a.seg_cols * 2;
    if (smem > 227 * 1024) return Q3_ERR_SHAPE;
    Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(gemv_kernel<EPI>), smem));
    const int grid = std::min(num_sms(), a.units);
    Q3_TRY_LAUNCH(launch(gemv_kernel<EPI>, dim3(grid), dim3(THREADS), smem, stream, 1, a));
    return Q3_OK;
}

}  // namespace

unsigned take_error_gemv() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

int gemv_plain(bf16 *out, const bf16 *w, const bf16 *x, int rows, int cols, cudaStream_t s) {
    if (!out || !w || !x) return Q3_ERR_ARG;
    if (!aligned16(w) || !aligned16(x)) return Q3_ERR_ALIGN;
    GemvArgs a = {};
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

int gemv_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv,
             const bf16 *x, int q_rows, int kv_rows, int cols, cudaStream_t s) {
    if (!q || !k || !v || !wq || !wk || !wv || !x) return Q3_ERR_ARG;
    if (!aligned16(wq) || !aligned16(wk) || !aligned16(wv) || !aligned16(x)) return Q3_ERR_ALIGN;
    if (q_rows < 0 || kv_rows < 0) return Q3_ERR_SHAPE;
    GemvArgs a = {};
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

int gemv_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int rows, int cols,
                 bf16 *gate_tap, bf16 *up_tap, cudaStream_t s) {
    if (!act || !w_gate || !w_up || !x) return Q3_ERR_ARG;
    if ((gate_tap == nullptr) != (up_tap == nullptr)) return Q3_ERR_ARG;
    if (!aligned16(w_gate) || !aligned16(w_up) || !aligned16(x)) return Q3_ERR_ALIGN;
    GemvArgs a = {};
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

}  // namespace q3
