// project_mma.cu — batched projections (prompt chunks) on the 5th-generation tensor cores.
//
// Replaces the reference's batched prefill projections (tampajohn/fpga-qwen engine/core.cpp:294,
// project() with more than one row: cblas_sgemm of the FP32 rows against the FP32 widening of
// the FP16 matrix; :387-394, :625-641 through project / project_group):
//     y[b][r] = sum_k x[b][k] * W[r][k]    FP16 W [rows][cols], FP32 x [batch][cols] and y.
// tcgen05.mma multiplies FP16 operands, so each input row is first split (split_rows_kernel):
// scaled by a power of two 2^e that brings its largest magnitude to [2^13, 2^14) (exact), then
// x_hi = fp16(x * 2^e) and x_lo = fp16(x * 2^e - x_hi), 22 bits of the row's significand in
// two FP16 halves. W x_hi and W x_lo accumulate in FP32 in two TMEM column ranges and the
// epilogue adds them and multiplies by 2^-e (exact). The products of FP16 weights with the 22-bit input are
// exact; the result lies within FP32 accumulation rounding of the exact product, as sgemm's
// does (its summation order is unpublished, so no sum order can be bit-identical to it).
//
// project_gemm_kernel: persistent, one CTA per SM; work units are 128-row x 128-batch output
// tiles (times the K splits), taken in an order where the units that share a weight tile run at
// the same time, so each weight byte comes from HBM once. Warp 0 runs a 4-stage TMA ring of
// 64-column K steps (W tile 16 KB, x_hi and x_lo tiles 16 KB each, 128-byte swizzle) across
// units; warp 1 issues the MMAs (M = 128 weight rows, N = 256: the unit's 128 batch rows of
// x_hi then of x_lo, K = 16 per instruction) into one of two 256-column TMEM accumulators;
// warps 2-5 (each its TMEM lane quarter: 32 weight rows) empty the other accumulator at the
// same time, so a unit's epilogue overlaps the next unit's K loop. Each epilogue warp stages
// 32 x 32 sub-tiles in shared memory and writes them with TMA stores (ragged row counts take
// plain coalesced stores). Launched as a programmatic dependent of the split kernel: set-up and
// the first weight tiles overlap it.
// Launches with fewer tiles than SMs (o_proj, down_proj: 1,024 rows) split K: the splits of a
// tile form one thread-block cluster, each leaves its scaled partial tile in its shared memory,
// and after a cluster barrier each CTA adds a share of the tile's batch rows over the peers'
// shared memory in split order (deterministic) and stores y. Rows past a matrix's end, batch rows past
// the chunk and K past cols read as zero (TMA out of bounds fill). Each K step moves 48 KB
// into shared memory for four 128 x 256 x 16 MMAs (512 tensor-pipe cycles). Every wait is
// bounded (globaltimer, 2 s); on expiry the kernel records an error code, drains what it
// issued and frees its TMEM.
#include <algorithm>

#include "qattn_common.cuh"
#include "sm100.cuh"

namespace qattn {
namespace {

using namespace sm100;

constexpr int GM = 128, GN = 128, GK = 64, GSTAGES = 4;
constexpr int EPI_WARP0 = 2, EPI_WARPS = 4, GTHREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr int SUB = 32;                                  // epilogue sub-tile: 32 rows x 32 batch rows
constexpr uint32_t W_TILE = GM * GK * 2;                 // 16 KB
constexpr uint32_t X_TILE = GN * GK * 2;                 // 16 KB
constexpr uint32_t STAGE_BYTES = W_TILE + 2 * X_TILE;    // 48 KB
constexpr uint32_t STAGING_BYTES = EPI_WARPS * 2 * SUB * SUB * 4;   // two 4 KB sub-tiles per warp
constexpr int GSMEM = GSTAGES * STAGE_BYTES + STAGING_BYTES + 1024 + 256;  // + alignment slack + barriers
static_assert(GSMEM <= 232448, "shared memory per CTA");

struct GemmMaps {
    CUtensorMap w[MAX_PROJECT_MATS];
    CUtensorMap xhi, xlo;
    CUtensorMap y[MAX_PROJECT_MATS];  // FP32 [batch][rows[m]], boxes of 32 rows x 32 batch rows
};

struct GemmArgs {
    int n_mats;
    int rows[MAX_PROJECT_MATS];
    int tile0[MAX_PROJECT_MATS + 1];  // first row tile of each matrix
    float* y[MAX_PROJECT_MATS];       // [batch][rows[m]]
    int cols, b0, nb;                 // this chunk: batch rows [b0, b0 + nb)
    const float* inv_scale;           // [nb]: 2^-e of each split row
    int ksplit;                       // K splits per tile, one cluster of ksplit CTAs per tile when > 1
    int tma_store;                    // 1: sub-tiles leave through shared memory and TMA stores
    int* error;
};

// One CTA per input row; the row stays in registers (PER elements per thread, cols <= 256 PER)
// between the max and the split. Rows whose largest magnitude is below 2^-112 take e = 126 (the
// largest exponent whose 2^-e is a normal float): they keep fewer than 22 bits.
template <int PER>
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int cols, __half* hi, __half* lo,
                                                        float* inv_scale) {
    __shared__ float red[8];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // the GEMM may start its set-up
    const float* xr = x + (size_t)blockIdx.x * cols;
    float v[PER];
    float m = 0.f;
    #pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int c = threadIdx.x + 256 * i;
        v[i] = c < cols ? __ldg(xr + c) : 0.f;
        m = fmaxf(m, fabsf(v[i]));
    }
    #pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
    #pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    int e = 0;
    if (m > 0.f && m <= 3.0e38f) {                       // finite, non-zero: bring the max to [2^13, 2^14)
        int ex;
        frexpf(m, &ex);                                   // m = f * 2^ex, f in [0.5, 1)
        e = min(14 - ex, 126);
    }
    const float s = ldexpf(1.f, e);
    __half* h = hi + (size_t)blockIdx.x * cols;
    __half* l = lo + (size_t)blockIdx.x * cols;
    #pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (c < cols) {
            const float t = v[i] * s;
            const __half th = __float2half_rn(t);
            h[c] = th;
            l[c] = __float2half_rn(t - __half2float(th));
        }
    }
    if (threadIdx.x == 0) inv_scale[blockIdx.x] = ldexpf(1.f, -e);
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Every thread of every CTA of the cluster arrives; shared-memory writes before it are visible
// to the peers' reads after it.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// No memory clobber: the loads may overlap one another and the global stores between them;
// volatile keeps them after the cluster barrier.
__device__ __forceinline__ float4 ld_peer4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// A work unit: matrix m, weight rows [r0, r0 + 128), batch rows [bt0, bt0 + 128) of the chunk,
// K steps [kt0, kt0 + kt_n) of split z. Units sharing a weight tile are consecutive, the splits
// of one output tile first (they form a cluster: split z is cluster rank z).
struct Unit {
    int m, r0, bt0, z, kt0, kt_n;
};
__device__ __forceinline__ Unit unit_of(const GemmArgs& a, int u, int n_bt, int kt_all) {
    Unit w;
    w.z = u % a.ksplit;
    const int rest = u / a.ksplit, by = rest % n_bt, t = rest / n_bt;
    w.m = 0;
    while (w.m + 1 < a.n_mats && t >= a.tile0[w.m + 1]) ++w.m;
    w.r0 = (t - a.tile0[w.m]) * GM;
    w.bt0 = by * GN;
    w.kt0 = (int)((long long)kt_all * w.z / a.ksplit);
    w.kt_n = (int)((long long)kt_all * (w.z + 1) / a.ksplit) - w.kt0;
    return w;
}

__global__ void __launch_bounds__(GTHREADS, 1) project_gemm_kernel(const __grid_constant__ GemmMaps maps,
                                                                  const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* staging = reinterpret_cast<float*>(smem + GSTAGES * STAGE_BYTES);   // [warp][2][SUB batch][SUB rows]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + GSTAGES * STAGE_BYTES + STAGING_BYTES);
    uint64_t* empty = full + GSTAGES;
    uint64_t* acc_full = empty + GSTAGES;                  // accumulator b holds a finished unit
    uint64_t* acc_empty = acc_full + 2;                    // the epilogue has read accumulator b
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    __shared__ int abort_flag, never_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_bt = (a.nb + GN - 1) / GN;
    const int units = a.tile0[a.n_mats] * n_bt * a.ksplit;
    const int kt_all = (a.cols + GK - 1) / GK;

    if (tid == 0) {
        abort_flag = 0;
        never_abort = 0;
        for (int s = 0; s < GSTAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], EPI_WARPS); }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 4 * GN); tmem_relinquish(); }   // two accumulators of 2 x 128 columns
    if (warp == 0 && lane == 0) {
        for (int m = 0; m < a.n_mats; ++m) prefetch_tmap(&maps.w[m]);
        prefetch_tmap(&maps.xhi);
        prefetch_tmap(&maps.xlo);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    volatile int* abortp = &abort_flag;
    auto fail = [&](int code) { *abortp = 1; atomicCAS(a.error, 0, code); };

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: K step g (counted across units) into stage g % GSTAGES ----
            // The first unit's first weight tiles are requested before waiting for the split
            // kernel (the weights do not depend on it); its x halves after.
            int pre = 0;
            if ((int)blockIdx.x < units) {
                const Unit w = unit_of(a, blockIdx.x, n_bt, kt_all);
                pre = min(GSTAGES, w.kt_n);
                for (int kt = 0; kt < pre; ++kt) {
                    mbar_arrive_expect_tx(&full[kt], STAGE_BYTES);
                    tma_load_3d(smem + kt * STAGE_BYTES, &maps.w[w.m], (w.kt0 + kt) * GK, w.r0, 0, &full[kt]);
                }
            }
            griddep_wait();
            uint32_t g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const Unit w = unit_of(a, u, n_bt, kt_all);
                for (int kt = 0; kt < w.kt_n; ++kt, ++g) {
                    const int s = g % GSTAGES;
                    uint8_t* st = smem + s * STAGE_BYTES;
                    const int kx = (w.kt0 + kt) * GK;
                    if ((int)g >= pre) {
                        if (g >= GSTAGES && !mbar_wait(&empty[s], ((g / GSTAGES) - 1) & 1, abortp)) {
                            fail(61);
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                        tma_load_3d(st, &maps.w[w.m], kx, w.r0, 0, &full[s]);
                    }
                    tma_load_3d(st + W_TILE, &maps.xhi, kx, w.bt0, 0, &full[s]);
                    tma_load_3d(st + W_TILE + X_TILE, &maps.xlo, kx, w.bt0, 0, &full[s]);
                }
            }
            if (!ok) {                                     // drain this thread's copies (bounded)
                const uint32_t issued = max(g, (uint32_t)pre);
                for (uint32_t it = issued > GSTAGES ? issued - GSTAGES : 0; it < issued; ++it)
                    mbar_wait(&full[it % GSTAGES], (it / GSTAGES) & 1, &never_abort, 500000000ull);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: [D_hi | D_lo] (+)= W [x_hi; x_lo]^T per 16-column K slice ----
        // The x_lo tile follows the x_hi tile in the stage, so one N = 256 MMA takes both as a
        // 256-row operand (128-row MMAs cannot be issued fast enough by one thread to keep the
        // tensor pipe busy; 256-row ones can). The whole warp runs the loop and the elected lane
        // issues (warp-converged issue, sm100.cuh); descriptors step by their low words.
        const uint32_t leader = elect_one();
        const uint32_t idesc = idesc_f16_f32(GM, 2 * GN, false);
        const uint32_t d_hi = (uint32_t)(sw128_desc(0, 16, 1024) >> 32);
        uint32_t g = 0;
        bool ok = true;
        int i = 0;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
            const Unit w = unit_of(a, u, n_bt, kt_all);
            const int b = i & 1;
            if (i >= 2 && !mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1, abortp)) { fail(64); break; }
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(b * 2 * GN);
            for (int kt = 0; kt < w.kt_n; ++kt, ++g) {
                const int s = g % GSTAGES;
                if (!mbar_wait(&full[s], (g / GSTAGES) & 1, abortp)) { fail(62); ok = false; break; }
                tc_fence_after();
                const uint32_t wl = (uint32_t)sw128_desc(smem_u32(smem + s * STAGE_BYTES), 16, 1024);
                const uint32_t xl = wl + (uint32_t)(W_TILE >> 4);
                static_assert(GK / 16 == 4, "four 16-column K slices per stage");
                mma_f16_ss_warp<0, 0>(acc, wl, xl, d_hi, idesc, kt > 0 ? 1u : 0u, leader);
                mma_f16_ss_warp<2, 2>(acc, wl, xl, d_hi, idesc, 1u, leader);   // +32 bytes per slice
                mma_f16_ss_warp<4, 4>(acc, wl, xl, d_hi, idesc, 1u, leader);
                mma_f16_ss_warp<6, 6>(acc, wl, xl, d_hi, idesc, 1u, leader);
                mma_commit_warp(&empty[s], leader);        // the stage is free once these MMAs complete
            }
            if (ok) mma_commit_warp(&acc_full[b], leader); // the unit's accumulator is final
        }
        mma_commit_warp(drain, leader);                    // every MMA issued has completed
        mbar_wait(drain, 0, &never_abort);
    } else {
        // ---- epilogue: warp holds weight rows r0 + 32 q + lane (its TMEM lane quarter q) ----
        const int q = warp & 3, ew = warp - EPI_WARP0;
        float* stage_w = staging + ew * 2 * SUB * SUB;
        griddep_wait();                                    // inv_scale is the split kernel's output
        uint32_t sub = 0;                                  // sub-tiles stored by this warp
        int i = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++i) {
            const Unit w = unit_of(a, u, n_bt, kt_all);
            const int b = i & 1;
            // the unit's 2^-e of batch row bt0 + 32 k + lane, loaded while the K loop runs
            float inv[GN / SUB];
            #pragma unroll
            for (int k = 0; k < GN / SUB; ++k) {
                const int bl = w.bt0 + SUB * k + lane;
                inv[k] = bl < a.nb ? a.inv_scale[bl] : 0.f;
            }
            if (!mbar_wait(&acc_full[b], (i >> 1) & 1, abortp)) { fail(63); break; }
            tc_fence_after();
            const int nb = a.nb, rows_m = a.rows[w.m], r = w.r0 + 32 * q + lane;
            const bool row_ok = r < rows_m;
            // plain-store path: y[b0 + b][r]
            const size_t pitch = rows_m;
            float* out = a.y[w.m] + (size_t)a.b0 * pitch + r;
            // split K: this split's tile [128 batch rows][128 weight rows] in shared memory (the
            // stage buffers: the unit's MMAs, the last readers, have completed)
            float* part = reinterpret_cast<float*>(smem);
            const uint32_t acc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * 2 * GN);
            #pragma unroll
            for (int k = 0; k < GN / SUB; ++k, ++sub) {
                const int c0 = k * SUB;
                uint32_t v[32], x[32];
                tmem_ld32(acc + c0, v);
                tmem_ld32(acc + GN + c0, x);
                const float my_inv = inv[k];                // broadcast below, one batch row per j
                tmem_wait_ld();
                if (c0 + SUB == GN) {                      // the accumulator is read: the MMA warp may reuse it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[b]);
                }
                if (a.ksplit > 1) {
                    #pragma unroll
                    for (int j = 0; j < SUB; ++j)
                        part[(c0 + j) * GM + 32 * q + lane] =
                            (__uint_as_float(v[j]) + __uint_as_float(x[j])) * __shfl_sync(0xffffffffu, my_inv, j);
                } else if (a.tma_store) {
                    float* sb = stage_w + (sub & 1) * SUB * SUB;
                    if (lane == 0 && sub >= 2) bulk_wait_read_1();   // this buffer's previous store has read it
                    __syncwarp();
                    #pragma unroll
                    for (int j = 0; j < SUB; ++j)
                        sb[j * SUB + lane] = (__uint_as_float(v[j]) + __uint_as_float(x[j])) * __shfl_sync(0xffffffffu, my_inv, j);
                    fence_proxy_async_smem();              // the sub-tile is visible to the TMA unit
                    __syncwarp();
                    if (lane == 0) {                       // rows and batch rows outside the extent are clipped
                        tma_store_3d(&maps.y[w.m], sb, w.r0 + 32 * q, a.b0 + w.bt0 + c0, 0);
                        bulk_commit();
                    }
                } else {
                    #pragma unroll
                    for (int j = 0; j < SUB; ++j) {
                        const float sc = __shfl_sync(0xffffffffu, my_inv, j);
                        const int bb = w.bt0 + c0 + j;
                        if (row_ok && bb < nb) out[(size_t)bb * pitch] = (__uint_as_float(v[j]) + __uint_as_float(x[j])) * sc;
                    }
                }
            }
        }
        if (lane == 0) bulk_wait_read_all();               // shared memory outlives this warp's stores
        __syncwarp();
    }
    if (a.ksplit > 1) {
        // one unit per CTA (the launch has one CTA per unit): sum the splits' tiles in split
        // order over the cluster's shared memory; this CTA takes batch rows [z per, (z + 1) per)
        __syncwarp();
        cluster_sync_all();
        const Unit w = unit_of(a, blockIdx.x, n_bt, kt_all);
        const uint32_t z = cluster_rank();
        const int per = (GN + a.ksplit - 1) / a.ksplit, bb0 = (int)z * per, bb1 = min(GN, bb0 + per);
        const int rows_m = a.rows[w.m];
        uint32_t peer[4];
        #pragma unroll
        for (int k = 0; k < 4; ++k) peer[k] = peer_addr(smem, (uint32_t)min(k, a.ksplit - 1));
        // four consecutive weight rows per thread and step, three steps' loads in flight
        const int n4 = (bb1 - bb0) * (GM / 4);
        float* ym = a.y[w.m];
        for (int e0 = tid; e0 < n4; e0 += 3 * GTHREADS) {
            float4 sum[3];
            #pragma unroll
            for (int h = 0; h < 3; ++h) {
                const int e = e0 + h * GTHREADS;
                if (e < n4) {
                    const uint32_t off = (uint32_t)((bb0 + e / (GM / 4)) * GM + 4 * (e % (GM / 4))) * 4u;
                    sum[h] = ld_peer4(peer[0] + off);
                    #pragma unroll
                    for (int k = 1; k < 4; ++k)
                        if (k < a.ksplit) {
                            const float4 t = ld_peer4(peer[k] + off);
                            sum[h].x += t.x; sum[h].y += t.y; sum[h].z += t.z; sum[h].w += t.w;
                        }
                }
            }
            #pragma unroll
            for (int h = 0; h < 3; ++h) {
                const int e = e0 + h * GTHREADS;
                if (e >= n4) continue;
                const int bg = w.bt0 + bb0 + e / (GM / 4), r = w.r0 + 4 * (e % (GM / 4));
                if (bg >= a.nb) continue;
                float* yr = ym + (size_t)(a.b0 + bg) * rows_m + r;
                if (a.tma_store) {                         // rows_m % 128 == 0, 16-byte aligned y
                    *reinterpret_cast<float4*>(yr) = sum[h];
                } else {
                    const float t[4] = {sum[h].x, sum[h].y, sum[h].z, sum[h].w};
                    #pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (r + i < rows_m) yr[i] = t[i];
                }
            }
        }
        cluster_sync_all();                                // no CTA leaves while a peer reads its tile
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 4 * GN);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&fn), cudaEnableDefault, &q) !=
            cudaSuccess)
            fn = nullptr;
    }
    return fn;
}

// FP32 output [d2][d1][d0] (innermost d0), boxes of 32 x 32 x 1, no swizzle.
bool encode_out(CUtensorMap* map, void* base, int d0, int d1, int d2) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)d0 * 4, (cuuint64_t)d0 * 4 * d1};
    cuuint32_t box[3] = {SUB, SUB, 1}, elem[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// FP16 matrix [rows][cols] (row stride cols): boxes of 64 columns x 128 rows, 128-byte swizzle,
// zero fill outside.
bool encode_rows(CUtensorMap* map, const void* base, int rows, int cols) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, 1};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)cols * 2 * rows};
    cuuint32_t box[3] = {GK, 128, 1}, elem[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t project_gemm_scratch_bytes() {
    return (size_t)GEMM_CHUNK_ROWS * GEMM_MAX_COLS * 2 * sizeof(__half) + GEMM_CHUNK_ROWS * sizeof(float) + 512;
}

int launch_project_gemm(const ProjectArgs& p, void* scratch, int* error, cudaStream_t s) {
    if (p.cols > GEMM_MAX_COLS || !scratch) return -1;
    static bool attr = false;
    static int sms = NUM_SMS_B200;
    if (!attr) {
        if (cudaFuncSetAttribute(project_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GSMEM) != cudaSuccess)
            return -2;
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        attr = true;
    }
    GemmMaps maps;
    GemmArgs a{};
    a.n_mats = p.n_mats;
    a.cols = p.cols;
    a.error = error;
    a.tile0[0] = 0;
    // TMA stores need 16-byte row pitches, aligned bases and tiles that end at their matrix's end
    bool tma_store = true;
    for (int m = 0; m < p.n_mats; ++m) {
        a.rows[m] = p.rows[m];
        a.y[m] = p.y[m];
        a.tile0[m + 1] = a.tile0[m] + (p.rows[m] + GM - 1) / GM;
        if (!encode_rows(&maps.w[m], p.w[m], p.rows[m], p.cols)) return -3;
        tma_store = tma_store && p.rows[m] % GM == 0 && reinterpret_cast<uintptr_t>(p.y[m]) % 16 == 0 &&
                    encode_out(&maps.y[m], p.y[m], p.rows[m], p.batch, 1);
    }
    for (int b0 = 0; b0 < p.batch; b0 += GEMM_CHUNK_ROWS) {
        const int nb = std::min(GEMM_CHUNK_ROWS, p.batch - b0);
        __half* hi = static_cast<__half*>(scratch);
        __half* lo = hi + (((size_t)nb * p.cols + 127) & ~size_t(127));
        float* inv = reinterpret_cast<float*>(lo + (((size_t)nb * p.cols + 127) & ~size_t(127)));
        if (!encode_rows(&maps.xhi, hi, nb, p.cols) || !encode_rows(&maps.xlo, lo, nb, p.cols)) return -3;
        const float* xc = p.x + (size_t)b0 * p.cols;
        if (p.cols <= 1024) split_rows_kernel<4><<<nb, 256, 0, s>>>(xc, p.cols, hi, lo, inv);
        else if (p.cols <= 2048) split_rows_kernel<8><<<nb, 256, 0, s>>>(xc, p.cols, hi, lo, inv);
        else if (p.cols <= 4096) split_rows_kernel<16><<<nb, 256, 0, s>>>(xc, p.cols, hi, lo, inv);
        else split_rows_kernel<32><<<nb, 256, 0, s>>>(xc, p.cols, hi, lo, inv);
        a.b0 = b0;
        a.nb = nb;
        a.inv_scale = inv;
        // Launches with fewer tiles than SMs split K (at least four K steps per split) so that
        // more SMs stream the matrix; then every CTA has one unit and each tile's splits form a
        // cluster that adds them. Otherwise persistent: one CTA per SM at most.
        const int tiles = a.tile0[p.n_mats] * ((nb + GN - 1) / GN), KT = (p.cols + GK - 1) / GK;
        a.ksplit = std::max(1, std::min({4, sms / std::max(1, tiles), KT / 4}));
        a.tma_store = tma_store ? 1 : 0;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)(a.ksplit > 1 ? tiles * a.ksplit : std::min(tiles, sms)));
        cfg.blockDim = dim3(GTHREADS);
        cfg.dynamicSmemBytes = GSMEM;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // overlaps the split kernel
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = (unsigned)a.ksplit;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = a.ksplit > 1 ? 2 : 1;
        if (cudaLaunchKernelEx(&cfg, project_gemm_kernel, maps, a) != cudaSuccess) return -4;
    }
    return 0;
}

}  // namespace qattn
