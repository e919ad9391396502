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
//   warps 2-5        epilogue: tcgen05.ld of the fp32 accumulator rows (one TMEM lane per
//                    output row; warp w reads lanes 32*(w%4)..+31), then the reference's bf16
//                    rounding points: plain, residual (src/kernels.cu:196-201), q/k/v, or
//                    SwiGLU (:277-286). The single accumulator is reused tile after tile; the
//                    producer keeps prefetching the next tile's stages meanwhile.
//
// Work: weight rows are cut into tiles of R <= 128 rows and K into S slices; a tile's S slices
// run on the S CTAs of one thread-block cluster. R and S are chosen so that tiles x S fill the
// SMs in one wave with as many weight bytes per pipeline stage as possible (o_proj and down,
// 2560 rows: S = 4). With S > 1 each CTA stages its fp32 partial tile in shared memory and,
// after a cluster barrier, reduces its share of the tile's rows over the S CTAs' partials
// (distributed shared memory, in rank order) before the epilogue. With S = 1 a persistent
// grid walks the tiles. The gate and up projections share a tile (two accumulators side by
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

#include "common.cuh"

namespace cg = cooperative_groups;

namespace q3 {
namespace {

__device__ unsigned g_dev_error;

constexpr int TC_THREADS = 192;  // producer warp, MMA warp, 4 epilogue warps
constexpr int EPI_THREADS = 128;
constexpr int BK = 64;            // K per stage: 64 bf16 = one 128-byte swizzle row
constexpr int TILE_M = 128;       // MMA M
constexpr int A_TILE_BYTES = TILE_M * BK * 2;  // 16 KB
constexpr int MAX_STAGES = 8;
constexpr size_t SMEM_BUDGET = 112 * 1024;  // leaves room for a co-resident successor kernel
constexpr size_t SMEM_MAX = 220 * 1024;

enum Epi : int { PLAIN = 0, RESIDUAL = 1, QKV = 2, GATE_UP = 3 };

struct TcArgs {
    bf16 *out0, *out1, *out2;      // PLAIN: out; RESIDUAL: x; QKV: q, k, v; GATE_UP: act
    bf16 *tap0, *tap1;             // RESIDUAL: tap; GATE_UP: gate, up
    int rows[3];                   // rows of each weight matrix (QKV: 3; else rows[0])
    int tile_start[4];             // first tile of each matrix in the tile list
    int n_tiles;
    int R;                         // rows per tile (TMA box rows)
    int K, nk;                     // columns and number of BK steps
    int splits;                    // S: CTAs of a cluster sharing a tile along K
    int B, Bp;                     // batch rows and MMA N
    int stages;
    int stage_bytes;
    uint32_t idesc;
    uint32_t tmem_cols;
};

// ---------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// K-major operand in the 128-byte swizzle layout: rows of 128 bytes, 8-row groups 1024 bytes
// apart (stride byte offset), leading byte offset 16 bytes, descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float *v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- kernel

__device__ __forceinline__ void tile_coords(const TcArgs &a, int t, int &mat, int &row0) {
    mat = 0;
    while (mat < 2 && t >= a.tile_start[mat + 1]) mat++;
    row0 = (t - a.tile_start[mat]) * a.R;
}

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ TcArgs a) {
    constexpr int NA = EPI == GATE_UP ? 2 : 1;  // weight tiles per stage (gate and up)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)a.stages * a.stage_bytes);
    uint64_t *empty = full + a.stages;
    uint64_t *acc_full = empty + a.stages;
    uint64_t *acc_empty = acc_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int S = a.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, EPI_THREADS);
        fence_barrier_init();
        prefetch_tmap(&tmA0);
        prefetch_tmap(&tmX);
        if (EPI == GATE_UP || EPI == QKV) prefetch_tmap(&tmA1);
        if (EPI == QKV) prefetch_tmap(&tmA2);
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
    pdl_trigger();

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
    bool ok = true;

    if (warp == 0 && lane == 0) {
        // ---------------- producer
        const CUtensorMap *maps[3] = {&tmA0, &tmA1, &tmA2};
        auto stage_a = [&](int s, int i) { return smem + (size_t)s * a.stage_bytes + (size_t)i * A_TILE_BYTES; };
        auto stage_x = [&](int s) { return smem + (size_t)s * a.stage_bytes + (size_t)NA * A_TILE_BYTES; };
        auto issue_weights = [&](int it) {
            const int s = it % S;
            const int t = tile_base + (it / nks) * tile_stride;
            const int ks = k0 + it % nks;
            int mat, row0;
            tile_coords(a, t, mat, row0);
            mbar_arrive_expect_tx(&full[s], NA * a_bytes + x_bytes);
            if (EPI == GATE_UP) {
                tma_load_2d(stage_a(s, 0), &tmA0, ks * BK, row0, &full[s]);
                tma_load_2d(stage_a(s, 1), &tmA1, ks * BK, row0, &full[s]);
            } else {
                tma_load_2d(stage_a(s, 0), maps[mat], ks * BK, row0, &full[s]);
            }
        };
        auto issue_x = [&](int it) { tma_load_2d(stage_x(it % S), &tmX, (k0 + it % nks) * BK, 0, &full[it % S]); };
        const int pre = min(S, total_steps);
        for (int it = 0; it < pre; it++) issue_weights(it);  // weights do not depend on the previous kernel
        pdl_wait();
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
                const uint32_t xs = smem_u32(smem + (size_t)s * a.stage_bytes + (size_t)NA * A_TILE_BYTES);
#pragma unroll
                for (int i = 0; i < NA; i++) {
                    const uint32_t as = smem_u32(smem + (size_t)s * a.stage_bytes + (size_t)i * A_TILE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        mma_bf16(tmem_base + i * a.Bp, smem_desc_sw128(as + kk * 32), smem_desc_sw128(xs + kk * 32),
                                 a.idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
            }
            if (ok) mma_commit(acc_full);
        }
    }

    __syncwarp();
    if (S_split > 1) {
        // ---------------- split-K epilogue: partial tile -> shared memory -> cluster reduction
        // (one tile per cluster; the pipeline ring is idle and is reused for the partial tile)
        const int ld = NA * a.Bp + 1;  // padded row: conflict-free column writes
        float *part = reinterpret_cast<float *>(smem);
        if (warp >= 2 && my_tiles > 0) {
            const int quarter = warp % 4;
            const int row_local = quarter * 32 + lane;
            const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
            if (!mbar_wait(acc_full, 0, &g_dev_error)) ok = false;
            tc_fence_after();
            for (int c0 = 0; c0 < NA * a.Bp; c0 += 8) {
                float acc[8];
                tmem_ld8(lane_addr + c0, acc);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; j++) part[row_local * ld + c0 + j] = acc[j];
            }
            tc_fence_before();
        }
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        if (my_tiles > 0) {
            pdl_wait();
            int mat, row0;
            tile_coords(a, tile_base, mat, row0);
            bf16 *o = EPI == QKV ? (mat == 0 ? a.out0 : mat == 1 ? a.out1 : a.out2) : a.out0;
            const long long ostride = a.rows[mat];
            const int r_lo = a.R * rank / S_split, r_hi = a.R * (rank + 1) / S_split;
            const int nr = r_hi - r_lo;
            const float *peer[8];
            for (int q = 0; q < S_split; q++) peer[q] = cluster.map_shared_rank(part, q);
            for (int i = threadIdx.x; i < nr * a.B; i += TC_THREADS) {
                const int b = i / nr, rl = r_lo + i % nr;  // consecutive threads: consecutive rows
                const int m = row0 + rl;
                if (m >= a.rows[mat]) continue;
                float acc = 0.0f, acc2 = 0.0f;
                for (int q = 0; q < S_split; q++) {
                    acc += peer[q][rl * ld + b];
                    if (EPI == GATE_UP) acc2 += peer[q][rl * ld + a.Bp + b];
                }
                const size_t idx = (size_t)b * ostride + m;
                if (EPI == PLAIN || EPI == QKV) {
                    o[idx] = __float2bfloat16(acc);
                } else if (EPI == RESIDUAL) {
                    const bf16 y = __float2bfloat16(acc);
                    if (a.tap0) a.tap0[idx] = y;
                    o[idx] = __float2bfloat16(__bfloat162float(o[idx]) + __bfloat162float(y));
                } else {
                    const bf16 gate = __float2bfloat16(acc), up = __float2bfloat16(acc2);
                    if (a.tap0) {
                        a.tap0[idx] = gate;
                        a.tap1[idx] = up;
                    }
                    const float gv = __bfloat162float(gate), uv = __bfloat162float(up);
                    o[idx] = __float2bfloat16(round_bf16(gv / (1.0f + expf(-gv))) * uv);
                }
            }
        }
        cluster.sync();  // every CTA's partial tile stays alive until all ranks have read it
    } else if (warp >= 2) {
    // ---------------- epilogue (warps 2-5, one accumulator row per thread)
    pdl_wait();
    const int quarter = warp % 4;
    const int row_local = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    for (int tl = 0; tl < my_tiles; tl++) {
        if (!mbar_wait(acc_full, tl & 1, &g_dev_error)) {
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
        for (int c0 = 0; c0 < a.Bp; c0 += 8) {
            float acc[8], acc2[8];
            tmem_ld8(lane_addr + c0, acc);
            if (EPI == GATE_UP) tmem_ld8(lane_addr + a.Bp + c0, acc2);
            tmem_wait_ld();
            if (!valid) continue;
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
                    o[idx] = __float2bfloat16(__bfloat162float(o[idx]) + __bfloat162float(y));
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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 map over a row-major [rows, cols] matrix with a [box_rows, 64] box, 128-byte swizzle.
bool make_map(CUtensorMap *map, const void *base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

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
    a.nk = (a.K + BK - 1) / BK;
    auto tiles_for = [&](int R) {
        int n = 0;
        for (int i = 0; i < n_mat; i++) n += (a.rows[i] + R - 1) / R;
        return n;
    };
    // Plan (R rows per tile, S K-slices): all tiles x S CTAs in one wave, minimizing the K steps
    // of one CTA weighted by its rows (rows below 64 count as 64: small tiles waste stages).
    int R = 0, S_best = 1;
    long long best = -1;
    for (int S = 1; S <= 8 && S <= a.nk; S++) {
        const int slots = nsm / S;
        int r = std::max(8, (int)((total_rows + slots - 1) / slots));
        while (r <= TILE_M && tiles_for(r) > slots) r++;
        if (r > TILE_M) continue;
        const long long cost = (long long)std::max(r, 64) * ((a.nk + S - 1) / S);
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
    a.R = R;
    a.splits = S_best;
    a.tile_start[0] = 0;
    for (int i = 0; i < 3; i++) a.tile_start[i + 1] = a.tile_start[i] + (i < n_mat ? (a.rows[i] + R - 1) / R : 0);
    a.n_tiles = a.tile_start[3];
    a.Bp = std::max(16, (a.B + 15) / 16 * 16);
    a.stage_bytes = NA * A_TILE_BYTES + a.Bp * BK * 2;
    a.stages = (int)std::min<size_t>(MAX_STAGES, (SMEM_BUDGET - 1024 - 256) / a.stage_bytes);
    if (a.stages < 2) a.stages = 2;
    if ((size_t)a.stages * a.stage_bytes + 1024 + 256 > SMEM_MAX) return Q3_ERR_SHAPE;
    uint32_t cols = 32;
    while (cols < (uint32_t)(NA * a.Bp)) cols *= 2;
    a.tmem_cols = cols;
    // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, N = Bp, M = 128
    a.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.Bp >> 3) << 17) | ((uint32_t)(TILE_M >> 4) << 24);

    CUtensorMap m0, m1, m2, mx;
    memset(&m1, 0, sizeof(m1));
    memset(&m2, 0, sizeof(m2));
    if (!make_map(&m0, w0, a.rows[0], a.K, R)) return Q3_ERR_ARG;
    if (EPI == GATE_UP && !make_map(&m1, w1, a.rows[0], a.K, R)) return Q3_ERR_ARG;
    if (EPI == QKV) {
        if (!make_map(&m1, w1, a.rows[1], a.K, R) || !make_map(&m2, w2, a.rows[2], a.K, R)) return Q3_ERR_ARG;
    }
    if (!make_map(&mx, x, a.B, a.K, a.Bp)) return Q3_ERR_ARG;

    // split-K reuses the ring for the fp32 partial tile [128][NA*Bp + 1]
    if (a.splits > 1 && (size_t)a.stages * a.stage_bytes < (size_t)TILE_M * (NA * a.Bp + 1) * 4) {
        a.stages = (int)(((size_t)TILE_M * (NA * a.Bp + 1) * 4 + a.stage_bytes - 1) / a.stage_bytes);
        if ((size_t)a.stages * a.stage_bytes + 1024 + 256 > SMEM_MAX) return Q3_ERR_SHAPE;
    }
    const size_t smem = 1024 + (size_t)a.stages * a.stage_bytes + (2 * a.stages + 2) * 8 + 16;
    Q3_TRY_LAUNCH(allow_smem(reinterpret_cast<const void *>(tc_gemm_kernel<EPI>), smem));
    const int grid = a.splits > 1 ? a.n_tiles * a.splits : std::min(nsm, a.n_tiles);
    Q3_TRY_LAUNCH(launch(tc_gemm_kernel<EPI>, dim3(grid), dim3(TC_THREADS), smem, stream, a.splits, m0, m1, m2, mx, a));
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
