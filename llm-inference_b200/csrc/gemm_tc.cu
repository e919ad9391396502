// Batched decode projections on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// For B >= 2 decode sequences the projections of a layer are real contractions:
// out[b][m] = sum_k W[m][k] * X[b][k] with W the [M, K] row-major weight (the reference's
// layout, src/model.cuh:26-39) and X the [B, K] activations. Mapped "swap-AB": weight rows are
// the MMA's M = 128 side, the (padded) batch is the N side (16..256), K advances 64 columns
// per pipeline stage (one 128-byte swizzle row), 4 MMAs of K = 16 per stage.
//
//   warp 0, lane 0   TMA producer: weight tile [R rows x 64] and activation tile [Bp x 64]
//                    per stage into a ring of shared-memory stages (128-byte swizzle); the
//                    weight loads of the first stages are issued before the programmatic-
//                    dependency wait, the activation loads after it.
//   warp 1, lane 0   MMA issuer: tcgen05.mma kind::f16 (bf16 in, fp32 accumulate) into TMEM,
//                    tcgen05.commit releases each stage and, after the last K step, the
//                    accumulator.
//   warps 2..        epilogue, EPI_GROUPS groups of 4 warps: tcgen05.ld of the fp32 accumulator
//                    rows (one TMEM lane per output row; warp w reads lanes 32*(w%4)..+31, group
//                    g every EPI_GROUPS-th chunk of 8 columns from 8g), then the reference's bf16
//                    rounding points: plain, residual (src/kernels.cu:196-201), q/k/v, or
//                    SwiGLU (:277-286). The single accumulator is reused tile after tile; the
//                    producer keeps prefetching the next tile's stages meanwhile.
//
// Work: weight rows are cut into tiles of R <= 128 rows and K into S slices; a tile's S slices
// run on the S CTAs of one thread-block cluster. R and S are chosen so that tiles x S fill the
// SMs in one wave with as many weight bytes per pipeline stage as possible (o_proj and down,
// 2560 rows: S = 4). With S > 1, ranks 1..S-1 of the cluster write their fp32 partial tiles
// into a receive buffer in rank 0's shared memory (distributed shared memory stores, then a
// release arrive on rank 0's mbarrier) and exit; rank 0 adds them to its own accumulator in rank
// order and runs the epilogue. No cluster barrier sits at the end of the kernel: the only one is
// split into an arrive after set-up and a wait before the epilogue, which guarantees that rank
// 0's mbarrier is initialized before anyone arrives on it. With S = 1 a persistent grid
// walks the tiles. The gate and up projections share a tile (two accumulators side by
// side in TMEM).
//
// Arithmetic note: the fp32 sums run in the tensor core's order, not the reference's
// lane-strided order, so results can differ from the batch-1 kernels in the last bf16 bit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

#ifndef Q3_GEMM_EPI_GROUPS
#define Q3_GEMM_EPI_GROUPS 2
#endif
// Epilogue warp groups. Each group of four warps covers the 128 TMEM lanes once and takes every
// G-th chunk of 8 accumulator columns. One warp per scheduler runs the epilogue's dependent chain
// of conversions, divides and stores without any latency hiding; G groups split it G ways.
constexpr int EPI_GROUPS = Q3_GEMM_EPI_GROUPS;
constexpr int EPI_THREADS = 128 * EPI_GROUPS;
constexpr int TC_THREADS = 64 + EPI_THREADS;  // producer warp, MMA warp, epilogue warps
constexpr int BK = 64;            // K per stage: 64 bf16 = one 128-byte swizzle row
constexpr int TILE_M = 128;       // MMA M
constexpr int MAX_STAGES = 12;
#ifndef Q3_GEMM_KSUB
#define Q3_GEMM_KSUB 4
#endif
constexpr int KSUB = Q3_GEMM_KSUB;  // 64-column sub-tiles per stage: 512 contiguous bytes per weight row
#ifndef Q3_GEMM_SMEM_BUDGET_KB
#define Q3_GEMM_SMEM_BUDGET_KB 112  // leaves room for a co-resident successor kernel
#endif
constexpr size_t SMEM_BUDGET = (size_t)Q3_GEMM_SMEM_BUDGET_KB * 1024;
#ifndef Q3_GEMM_MAX_SPLIT
#define Q3_GEMM_MAX_SPLIT 8  // largest K split (cluster size) the planner considers
#endif
constexpr size_t SMEM_MAX = 220 * 1024;
constexpr int BAR_BYTES = 256;  // mbarriers and the TMEM slot after the stage ring
constexpr int RES_TMA_MAX_BP = 64;  // residual tiles loaded by TMA up to this padded batch

enum Epi : int { PLAIN = 0, RESIDUAL = 1, QKV = 2, GATE_UP = 3 };

struct TcArgs {
    bf16 *out0, *out1, *out2;      // PLAIN: out; RESIDUAL: x; QKV: q, k, v; GATE_UP: act
    bf16 *tap0, *tap1;             // RESIDUAL: tap; GATE_UP: gate, up
    int rows[3];                   // rows of each weight matrix (QKV: 3; else rows[0])
    int tile_start[4];             // first tile of each matrix in the tile list
    int n_tiles;
    int R;                         // rows per tile (TMA box rows)
    int K, nk;                     // columns and number of pipeline stages of ksub * BK columns
    int ksub;                      // 64-column sub-tiles per stage (adjacent: longer DRAM runs per row)
    int splits;                    // S: CTAs of a cluster sharing a tile along K
    int B, Bp;                     // batch rows and MMA N
    int stages;
    int stage_bytes;
    int a_tile_bytes;              // shared bytes of one weight tile: R rows rounded up to 8, x 128
    uint32_t idesc;
    uint32_t tmem_cols;
    int res_tma;                   // RESIDUAL: rank 0 loads its tile's residual x [Bp, R] by TMA
    int res_off;                   // shared-memory offset of that tile (from the aligned base)
};

// ---------------------------------------------------------------- kernel

// Cluster barrier in two halves (every thread of every CTA of the cluster executes each once).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }

// Arrive on the mbarrier at the same shared-memory offset in cluster CTA `rank`, with release
// semantics at cluster scope (this thread's earlier stores, remote ones included, are visible
// to a thread that observes the phase with an acquire wait).
__device__ __forceinline__ void mbar_arrive_remote(uint64_t *bar, unsigned rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(bar)), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

// mbar_wait with acquire semantics at cluster scope (for arrivals from other CTAs).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, unsigned *err) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t start = globaltimer();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (globaltimer() - start > WAIT_LIMIT_NS) {
            atomicOr(err, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tile_coords(const TcArgs &a, int t, int &mat, int &row0) {
    mat = 0;
    while (mat < 2 && t >= a.tile_start[mat + 1]) mat++;
    row0 = (t - a.tile_start[mat]) * a.R;
}

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmR, const __grid_constant__ TcArgs a) {
    constexpr int NA = EPI == GATE_UP ? 2 : 1;  // weight tiles per stage (gate and up)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    unsigned char *smem = align_shared<1024>(smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)a.stages * a.stage_bytes);
    uint64_t *empty = full + a.stages;
    uint64_t *acc_full = empty + a.stages;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *recv_full = acc_empty + 1;  // split-K, rank 0: the other ranks' partial tiles arrived
    uint64_t *res_full = recv_full + 1;   // the residual tile arrived
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(res_full + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int S = a.stages;

    // split-K: the S CTAs of a cluster share tile blockIdx.x / S, rank r takes K steps [k0, k1)
    const int S_split = a.splits;
    const int rank = S_split > 1 ? (int)cg::this_cluster().block_rank() : 0;
    const int tile_base = S_split > 1 ? (int)blockIdx.x / S_split : (int)blockIdx.x;
    const int tile_stride = S_split > 1 ? (int)gridDim.x / S_split : (int)gridDim.x;
    const int k0 = a.nk * rank / S_split, k1 = a.nk * (rank + 1) / S_split;
    const int nks = k1 - k0;
    const int my_tiles = a.n_tiles > tile_base ? (a.n_tiles - 1 - tile_base) / tile_stride + 1 : 0;
    const int total_steps = my_tiles * nks;
    const uint32_t a_bytes = (uint32_t)a.R * BK * 2;
    const uint32_t x_bytes = (uint32_t)a.Bp * BK * 2;
    const CUtensorMap *maps[3] = {&tmA0, &tmA1, &tmA2};
    const uint64_t stream_pol = policy_evict_first();  // weights are read once per step
    // stage layout: [A sub-tiles 0..ksub-1][A1 sub-tiles (gate_up)][X sub-tiles 0..ksub-1]
    auto stage_a = [&](int s, int i, int j) {
        return smem + (size_t)s * a.stage_bytes + (size_t)(i * a.ksub + j) * a.a_tile_bytes;
    };
    auto stage_x = [&](int s, int j) {
        return smem + (size_t)s * a.stage_bytes + (size_t)NA * a.ksub * a.a_tile_bytes + (size_t)j * x_bytes;
    };
    auto subs_of = [&](int ks) { return min(a.ksub, (a.K - ks * a.ksub * BK + BK - 1) / BK); };
    auto issue_weights = [&](int it) {
        const int s = it % S;
        const int t = tile_base + (it / nks) * tile_stride;
        const int ks = k0 + it % nks;
        const int nsub = subs_of(ks);
        int mat, row0;
        tile_coords(a, t, mat, row0);
        mbar_arrive_expect_tx(&full[s], nsub * (NA * a_bytes + x_bytes));
        for (int j = 0; j < nsub; j++) {
            const int col = (ks * a.ksub + j) * BK;
            if (EPI == GATE_UP) {
                tma_load_2d_stream(stage_a(s, 0, j), &tmA0, col, row0, &full[s], stream_pol);
                tma_load_2d_stream(stage_a(s, 1, j), &tmA1, col, row0, &full[s], stream_pol);
            } else {
                tma_load_2d_stream(stage_a(s, 0, j), maps[mat], col, row0, &full[s], stream_pol);
            }
        }
    };
    const int pre = min(S, total_steps);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, EPI_THREADS);
        if (a.splits > 1) mbar_init(recv_full, (a.splits - 1) * EPI_THREADS);
        mbar_init(res_full, 1);
        fence_barrier_init();
        prefetch_tmap(&tmA0);
        prefetch_tmap(&tmX);
        if (EPI == GATE_UP || EPI == QKV) prefetch_tmap(&tmA1);
        if (EPI == QKV) prefetch_tmap(&tmA2);
        if (EPI == RESIDUAL && a.res_tma) prefetch_tmap(&tmR);
        // the first stages' weights: they depend on no earlier kernel, and nothing below (TMEM
        // allocation, the block barrier, the dependency wait) has to come before them
        for (int it = 0; it < pre; it++) issue_weights(it);
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // split-K: rank 0's recv_full must be initialized before any rank arrives on it. Every
    // thread arrives here and waits just before the epilogue, long after.
    if (a.splits > 1) cluster_arrive_relaxed();
    pdl_trigger();

    bool ok = true;

    if (warp == 0 && lane == 0) {
        // ---------------- producer
        auto issue_x = [&](int it) {
            const int ks = k0 + it % nks;
            const int nsub = subs_of(ks);
            for (int j = 0; j < nsub; j++) tma_load_2d(stage_x(it % S, j), &tmX, (ks * a.ksub + j) * BK, 0, &full[it % S]);
        };
        pdl_wait();
        const bool res_load = EPI == RESIDUAL && a.res_tma && rank == 0 && my_tiles > 0;
        if (res_load) {  // x rows of this tile for every batch row: read by the epilogue
            int mat, row0;
            tile_coords(a, tile_base, mat, row0);
            mbar_arrive_expect_tx(res_full, (uint32_t)(a.R * a.Bp * 2));
            tma_load_2d(smem + a.res_off, &tmR, row0, 0, res_full);
        }
        for (int it = 0; it < pre; it++) issue_x(it);
        int it = pre;
        for (; it < total_steps; it++) {
            if (!mbar_wait(&empty[it % S], ((it / S) - 1) & 1, &g_dev_error)) {
                ok = false;
                break;
            }
            issue_weights(it);
            issue_x(it);
        }
        // leave no copy in flight into this CTA's shared memory
        for (int j = max(0, it - S); j < it; j++) mbar_wait(&full[j % S], (j / S) & 1, &g_dev_error);
        // nor an arrive: the MMA frees each stage with tcgen05.commit, whose arrive on `empty` is
        // performed asynchronously when the MMAs finish, possibly after the accumulator's commit that
        // the epilogue waits for. Wait for the last stages' arrives as well.
        for (int j = max(0, it - S); j < it; j++) mbar_wait(&empty[j % S], (j / S) & 1, &g_dev_error);
        if (res_load) mbar_wait(res_full, 0, &g_dev_error);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer
        int it = 0;
        for (int tl = 0; tl < my_tiles && ok; tl++) {
            if (tl > 0 && !mbar_wait(acc_empty, (tl - 1) & 1, &g_dev_error)) {
                ok = false;
                break;
            }
            tc_fence_after();
            for (int ks = 0; ks < nks; ks++, it++) {
                const int s = it % S;
                if (!mbar_wait(&full[s], (it / S) & 1, &g_dev_error)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int kglob = k0 + ks;
                const int nsub = min(a.ksub, (a.K - kglob * a.ksub * BK + BK - 1) / BK);
                const uint32_t sbase = smem_u32(smem + (size_t)s * a.stage_bytes);
                const uint32_t xbase = sbase + NA * a.ksub * a.a_tile_bytes;
                for (int j = 0; j < nsub; j++) {
                    const uint32_t xs = xbase + j * (uint32_t)(a.Bp * BK * 2);
#pragma unroll
                    for (int i = 0; i < NA; i++) {
                        const uint32_t as = sbase + (i * a.ksub + j) * a.a_tile_bytes;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++)
                            mma_bf16(tmem_base + i * a.Bp, smem_desc_sw128(as + kk * 32), smem_desc_sw128(xs + kk * 32),
                                     a.idesc, (ks > 0 || j > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
            }
            if (ok) mma_commit(acc_full);
        }
    }

    __syncwarp();
    if (S_split > 1) cluster_wait();
    if (S_split > 1 && rank > 0) {
        // ---------------- split-K, ranks 1..S-1: push the fp32 partial tile into rank 0's
        // receive buffer (distributed shared memory) and leave; nothing reads this CTA's memory.
        if (warp >= 2 && my_tiles > 0) {
            const int quarter = warp % 4, group = (warp - 2) / 4;
            const int row_local = quarter * 32 + lane;
            const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
            const int ldr = NA * a.Bp + 4;
            float *recv = reinterpret_cast<float *>(smem + (size_t)a.stages * a.stage_bytes + BAR_BYTES);
            float *dst = cg::this_cluster().map_shared_rank(recv, 0) + ((size_t)(rank - 1) * a.R + row_local) * ldr;
            const bool got = mbar_wait(acc_full, 0, &g_dev_error);
            tc_fence_after();
            // tcgen05.ld is warp-collective (.sync.aligned): every lane issues it; only the
            // stores are guarded
            const bool store = got && row_local < a.R;
            for (int c0 = 8 * group; c0 < NA * a.Bp; c0 += 8 * EPI_GROUPS) {
                float v[8];
                tmem_ld8(lane_addr + c0, v);
                tmem_wait_ld();
                if (store) {
                    reinterpret_cast<float4 *>(dst + c0)[0] = make_float4(v[0], v[1], v[2], v[3]);
                    reinterpret_cast<float4 *>(dst + c0)[1] = make_float4(v[4], v[5], v[6], v[7]);
                }
            }
            tc_fence_before();
            mbar_arrive_remote(recv_full, 0);  // release: the stores above are visible to rank 0
        }
    } else if (warp >= 2) {
    // ---------------- epilogue (warps 2.., one accumulator row per thread and group). With split-K this
    // is rank 0 of the cluster: its own partial (K steps of rank 0) plus the received partials
    // of ranks 1..S-1, added in rank order.
    pdl_wait();
    const int quarter = warp % 4, group = (warp - 2) / 4;
    const int row_local = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    const int ldr = NA * a.Bp + 4;
    const float *recv = reinterpret_cast<const float *>(smem + (size_t)a.stages * a.stage_bytes + BAR_BYTES) +
                        (size_t)row_local * ldr;
    for (int tl = 0; tl < my_tiles; tl++) {
        bool got = mbar_wait(acc_full, tl & 1, &g_dev_error);
        if (got && S_split > 1) got = mbar_wait_cluster(recv_full, 0, &g_dev_error);
        if (got && EPI == RESIDUAL && a.res_tma) got = mbar_wait(res_full, 0, &g_dev_error);
        // the warp leaves together, never splitting around the warp-collective tcgen05.ld below
        if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const int t = tile_base + tl * tile_stride;
        int mat, row0;
        tile_coords(a, t, mat, row0);
        const int m = row0 + row_local;
        const bool valid = row_local < a.R && m < a.rows[mat];
        bf16 *o = EPI == QKV ? (mat == 0 ? a.out0 : mat == 1 ? a.out1 : a.out2) : a.out0;
        const long long ostride = a.rows[mat];
        for (int c0 = 8 * group; c0 < a.Bp; c0 += 8 * EPI_GROUPS) {
            float acc[8], acc2[8];
            tmem_ld8(lane_addr + c0, acc);
            if (EPI == GATE_UP) tmem_ld8(lane_addr + a.Bp + c0, acc2);
            tmem_wait_ld();
            if (!valid) continue;
            for (int q = 1; q < S_split; q++) {
                const float *pq = recv + (size_t)(q - 1) * a.R * ldr;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    acc[j] += pq[c0 + j];
                    if (EPI == GATE_UP) acc2[j] += pq[a.Bp + c0 + j];
                }
            }
            float xr[8];
            if (EPI == RESIDUAL) {  // the residual tile in shared memory, else 8 loads issued together
                const bf16 *rt = reinterpret_cast<const bf16 *>(smem + a.res_off) + row_local;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int b = c0 + j;
                    xr[j] = a.res_tma ? __bfloat162float(rt[(size_t)b * a.R])
                                      : (b < a.B ? __bfloat162float(o[(size_t)b * ostride + m]) : 0.0f);
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int b = c0 + j;
                if (b >= a.B) break;
                const size_t idx = (size_t)b * ostride + m;
                if (EPI == PLAIN || EPI == QKV) {
                    o[idx] = __float2bfloat16(acc[j]);
                } else if (EPI == RESIDUAL) {
                    const bf16 y = __float2bfloat16(acc[j]);
                    if (a.tap0) a.tap0[idx] = y;
                    o[idx] = __float2bfloat16(xr[j] + __bfloat162float(y));
                } else {
                    const bf16 gate = __float2bfloat16(acc[j]);
                    const bf16 up = __float2bfloat16(acc2[j]);
                    if (a.tap0) {
                        a.tap0[idx] = gate;
                        a.tap1[idx] = up;
                    }
                    const float gv = __bfloat162float(gate), uv = __bfloat162float(up);
                    const float silu = round_bf16(gv / (1.0f + expf(-gv)));
                    o[idx] = __float2bfloat16(silu * uv);
                }
            }
        }
        tc_fence_before();
        mbar_arrive(acc_empty);
    }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(a.tmem_cols)
                     : "memory");
    }
}

// ---------------------------------------------------------------- host side

bool aligned16(const void *p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int EPI>
int launch_tc(TcArgs a, const bf16 *w0, const bf16 *w1, const bf16 *w2, const bf16 *x, cudaStream_t stream) {
    constexpr int NA = EPI == GATE_UP ? 2 : 1;
    if (a.B <= 0 || a.B > 256) return Q3_ERR_SHAPE;
    if (a.K <= 0 || a.K % 8 != 0) return Q3_ERR_SHAPE;
    const int n_mat = EPI == QKV ? 3 : 1;
    long long total_rows = 0;
    for (int i = 0; i < n_mat; i++) {
        if (a.rows[i] < 0) return Q3_ERR_SHAPE;
        total_rows += a.rows[i];
    }
    if (total_rows == 0) return Q3_OK;
    const int nsm = num_sms();
    a.Bp = std::max(16, (a.B + 15) / 16 * 16);
    const int k64 = (a.K + BK - 1) / BK;  // 64-column steps
    // wide stages for long contiguous weight runs, narrower when the activation tiles grow
    a.ksub = std::min(a.Bp <= 64 ? KSUB : a.Bp <= 128 ? 2 : 1, k64);
    a.nk = (k64 + a.ksub - 1) / a.ksub;
    auto tiles_for = [&](int R) {
        int n = 0;
        for (int i = 0; i < n_mat; i++) n += (a.rows[i] + R - 1) / R;
        return n;
    };
    // Residual x tile by TMA: its first column must sit on a 16-byte boundary, so R is a
    // multiple of 8 (as are the rows, for the row pitch); small batches only.
    const bool res_cand = EPI == RESIDUAL && a.Bp <= RES_TMA_MAX_BP && a.rows[0] % 8 == 0 &&
                          (reinterpret_cast<uintptr_t>(a.out0) & 15) == 0;
    const int r_step = res_cand ? 8 : 1;
    auto res_bytes = [&](int R_) { return res_cand ? (size_t)R_ * a.Bp * 2 : (size_t)0; };
    // Plan (R rows per tile, S K-slices): every cluster of S CTAs resident in one wave (checked
    // with the occupancy API, since clusters must fit inside one GPC), minimizing the work of the
    // busiest SM: K stages of its CTAs times their rows (rows below 64 count as 64).
    auto smem_for = [&](int R_, int S_, int *stages_out) {
        const int at = (R_ + 7) / 8 * 8 * BK * 2;
        const int sb = a.ksub * (NA * at + a.Bp * BK * 2);
        // split-K: rank 0 receives the other ranks' fp32 partial tiles after the barriers
        const size_t recv = S_ > 1 ? (size_t)(S_ - 1) * R_ * (NA * a.Bp + 4) * 4 : 0;
        const size_t room = SMEM_BUDGET - 1024 - BAR_BYTES - res_bytes(R_);
        int st = room > recv ? (int)std::min<size_t>(MAX_STAGES, (room - recv) / sb) : 0;
        st = std::max(st, 2);
        // the M = 128 MMA reads up to (128 - R) rows past a weight tile: slack beyond the last stage
        const int over = (TILE_M - (R_ + 7) / 8 * 8) * BK * 2 - a.ksub * a.Bp * BK * 2;
        if (stages_out) *stages_out = st;
        // the over-read may land in the receive buffer: it only feeds accumulator rows never read;
        // the residual tile follows, 128-byte aligned
        const size_t tail = ((size_t)st * sb + BAR_BYTES + std::max<size_t>((size_t)std::max(over, 0), recv) + 127) / 128 * 128;
        return (size_t)1024 + tail + res_bytes(R_);
    };
    auto resident = [&](int S_, size_t smem_) {
        int n = 0;
        if (smem_ > SMEM_MAX) return 0;
        if (allow_smem(reinterpret_cast<const void *>(tc_gemm_kernel<EPI>), smem_) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        if (S_ == 1) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, tc_gemm_kernel<EPI>, TC_THREADS, smem_) != cudaSuccess)
                n = 1;
            cudaGetLastError();
            return n * nsm;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S_ * nsm);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = smem_;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = S_;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<EPI>, &cfg) != cudaSuccess) n = 0;
        cudaGetLastError();
        return n;
    };
    int R = 0, S_best = 1;
    long long best = -1;
    bool cached = false;
    int dev = 0;
    cudaGetDevice(&dev);
    const long long key[7] = {EPI, a.rows[0], a.rows[1], a.rows[2], a.K, a.B, dev};
    static std::mutex plan_mu;
    static std::vector<std::pair<std::vector<long long>, std::pair<int, int>>> plans;
    {
        std::lock_guard<std::mutex> lock(plan_mu);
        for (auto &pl : plans)
            if (std::equal(pl.first.begin(), pl.first.end(), key)) {
                R = pl.second.first;
                S_best = pl.second.second;
                cached = true;
            }
    }
    for (int S = 1; !cached && S <= Q3_GEMM_MAX_SPLIT && S <= a.nk; S *= 2) {
        int slots = nsm / S, r = 0;
        for (int pass = 0; pass < 2; pass++) {
            r = std::max(8, (int)((total_rows + slots - 1) / std::max(slots, 1)));
            r = (r + r_step - 1) / r_step * r_step;
            while (r <= TILE_M && tiles_for(r) > slots) r += r_step;
            if (r > TILE_M) break;
            slots = std::min(slots, resident(S, smem_for(r, S, nullptr)));
            if (slots <= 0) {
                r = TILE_M + 1;
                break;
            }
        }
        if (r > TILE_M || tiles_for(r) > slots) continue;
        const long long ctas = (long long)tiles_for(r) * S;
        const long long per_sm = (ctas + nsm - 1) / nsm;
        const long long cost = per_sm * std::max(r, 64) * ((a.nk + S - 1) / S);
        if (best < 0 || cost < best) {
            best = cost;
            R = r;
            S_best = S;
        }
    }
    if (R == 0) {  // more rows than one wave holds: persistent CTAs over 128-row-or-less tiles
        const long long waves = (total_rows + (long long)nsm * TILE_M - 1) / ((long long)nsm * TILE_M);
        R = (int)std::min<long long>(TILE_M, (total_rows + nsm * waves - 1) / (nsm * waves));
        while (R < TILE_M && tiles_for(R) > nsm * waves) R++;
        S_best = 1;
    }
    {
        std::lock_guard<std::mutex> lock(plan_mu);
        bool known = false;
        for (auto &pl : plans) known = known || std::equal(pl.first.begin(), pl.first.end(), key);
        if (!known) plans.push_back({std::vector<long long>(key, key + 7), {R, S_best}});
    }
    a.R = R;
    a.splits = S_best;
    a.tile_start[0] = 0;
    for (int i = 0; i < 3; i++) a.tile_start[i + 1] = a.tile_start[i] + (i < n_mat ? (a.rows[i] + R - 1) / R : 0);
    a.n_tiles = a.tile_start[3];
    // A weight tile holds R rows (8-row swizzle atoms). The M = 128 MMA reads 128 rows from the
    // tile's start; rows past R land in the following shared memory (the next tile, the
    // activation tiles, or the slack reserved at the end) and produce accumulator rows that the
    // epilogue never reads.
    a.a_tile_bytes = (R + 7) / 8 * 8 * BK * 2;
    a.stage_bytes = a.ksub * (NA * a.a_tile_bytes + a.Bp * BK * 2);
    int stages = 2;
    const size_t smem = smem_for(R, a.splits, &stages);
    a.stages = stages;
    if (smem > SMEM_MAX) return Q3_ERR_SHAPE;
    // one tile per CTA (or cluster): the residual tile is loaded once, at the start
    const int grid_ctas = a.splits > 1 ? a.n_tiles * a.splits : std::min(nsm, a.n_tiles);
    a.res_tma = res_cand && R % 8 == 0 && a.n_tiles * a.splits <= grid_ctas ? 1 : 0;
    a.res_off = (int)(smem - 1024 - res_bytes(R));
    uint32_t cols = 32;
    while (cols < (uint32_t)(NA * a.Bp)) cols *= 2;
    a.tmem_cols = cols;
    // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, N = Bp, M = 128
    a.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.Bp >> 3) << 17) | ((uint32_t)(TILE_M >> 4) << 24);

    CUtensorMap m0, m1, m2, mx, mr;
    memset(&mr, 0, sizeof(mr));
    if (a.res_tma && !make_map_plain(&mr, a.out0, a.B, a.rows[0], a.rows[0], a.Bp, R)) return Q3_ERR_ARG;
    memset(&m1, 0, sizeof(m1));
    memset(&m2, 0, sizeof(m2));
    if (!make_map(&m0, w0, a.rows[0], a.K, R)) return Q3_ERR_ARG;
    if (EPI == GATE_UP && !make_map(&m1, w1, a.rows[0], a.K, R)) return Q3_ERR_ARG;
    if (EPI == QKV) {
        if (!make_map(&m1, w1, a.rows[1], a.K, R) || !make_map(&m2, w2, a.rows[2], a.K, R)) return Q3_ERR_ARG;
    }
    if (!make_map(&mx, x, a.B, a.K, a.Bp)) return Q3_ERR_ARG;

    Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(tc_gemm_kernel<EPI>), smem));
    const int grid = a.splits > 1 ? a.n_tiles * a.splits : std::min(nsm, a.n_tiles);
    Q3_TRY_LAUNCH(launch(tc_gemm_kernel<EPI>, dim3(grid), dim3(TC_THREADS), smem, stream, a.splits, m0, m1, m2, mx, mr, a));
    return Q3_OK;
}

}  // namespace

unsigned take_error_tc() {
    unsigned v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v)) != cudaSuccess) return 0;
    if (v) cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(zero));
    return v;
}

int tc_gemv(bf16 *out, const bf16 *w, const bf16 *x, int batch, int rows, int cols, cudaStream_t s) {
    if (!out || !w || !x) return Q3_ERR_ARG;
    if (!aligned16(w) || !aligned16(x)) return Q3_ERR_ALIGN;
    TcArgs a = {};
    a.out0 = out;
    a.rows[0] = rows;
    a.K = cols;
    a.B = batch;
    return launch_tc<PLAIN>(a, w, nullptr, nullptr, x, s);
}

int tc_gemv_residual(bf16 *x, const bf16 *w, const bf16 *in, int batch, int rows, int cols, bf16 *tap,
                     cudaStream_t s) {
    if (!x || !w || !in) return Q3_ERR_ARG;
    if (!aligned16(w) || !aligned16(in)) return Q3_ERR_ALIGN;
    TcArgs a = {};
    a.out0 = x;
    a.tap0 = tap;
    a.rows[0] = rows;
    a.K = cols;
    a.B = batch;
    return launch_tc<RESIDUAL>(a, w, nullptr, nullptr, in, s);
}

int tc_qkv(bf16 *q, bf16 *k, bf16 *v, const bf16 *wq, const bf16 *wk, const bf16 *wv, const bf16 *x, int batch,
           int q_rows, int kv_rows, int cols, cudaStream_t s) {
    if (!q || !k || !v || !wq || !wk || !wv || !x) return Q3_ERR_ARG;
    if (!aligned16(wq) || !aligned16(wk) || !aligned16(wv) || !aligned16(x)) return Q3_ERR_ALIGN;
    TcArgs a = {};
    a.out0 = q;
    a.out1 = k;
    a.out2 = v;
    a.rows[0] = q_rows;
    a.rows[1] = kv_rows;
    a.rows[2] = kv_rows;
    a.K = cols;
    a.B = batch;
    return launch_tc<QKV>(a, wq, wk, wv, x, s);
}

int tc_gate_up(bf16 *act, const bf16 *w_gate, const bf16 *w_up, const bf16 *x, int batch, int rows, int cols,
               bf16 *gate_tap, bf16 *up_tap, cudaStream_t s) {
    if (!act || !w_gate || !w_up || !x) return Q3_ERR_ARG;
    if ((gate_tap == nullptr) != (up_tap == nullptr)) return Q3_ERR_ARG;
    if (!aligned16(w_gate) || !aligned16(w_up) || !aligned16(x)) return Q3_ERR_ALIGN;
    TcArgs a = {};
    a.out0 = act;
    a.tap0 = gate_tap;
    a.tap1 = up_tap;
    a.rows[0] = rows;
    a.K = cols;
    a.B = batch;
    return launch_tc<GATE_UP>(a, w_gate, w_up, nullptr, x, s);
}

}  // namespace q3
