// project_mma.cu — batched projections (prompt chunks) on the 5th-generation tensor cores.
//
// Replaces the reference's batched prefill projections (tampajohn/fpga-qwen engine/core.cpp:294,
// project() with more than one row: cblas_sgemm of the FP32 rows against the FP32 widening of
// the FP16 matrix; :387-394, :625-641 through project / project_group):
//     y[b][r] = sum_k x[b][k] * W[r][k]    FP16 W [rows][cols], FP32 x [batch][cols] and y.
// tcgen05.mma multiplies FP16 operands, so each input row is first split (split_rows_kernel):
// scaled by a power of two 2^e that brings its largest magnitude to [2^13, 2^14) (exact), then
// x_hi = fp16(x * 2^e) and x_lo = fp16(x * 2^e - x_hi), 22 bits of the row's significand in
// two FP16 halves. Two MMAs per K step accumulate W x_hi + W x_lo in FP32 in TMEM and the
// epilogue multiplies by 2^-e (exact). The products of FP16 weights with the 22-bit input are
// exact; the result lies within FP32 accumulation rounding of the exact product, as sgemm's
// does (its summation order is unpublished, so no sum order can be bit-identical to it).
//
// project_gemm_kernel: one CTA per 128-row x 128-batch output tile, full K: a 4-stage TMA ring
// of 64-column K steps (W tile 16 KB, x_hi and x_lo tiles 16 KB each, 128-byte swizzle), one
// thread issuing the MMAs (M = 128 weight rows, N = 128 batch rows, K = 16 per instruction),
// the accumulator in 128 TMEM columns, and an epilogue of all four warps (each its TMEM lane
// quarter: 32 weight rows) that stores y with one coalesced 128-byte row segment per column.
// Launches with fewer tiles than SMs (o_proj, down_proj: 1,024 rows) split K over blockIdx.z
// and add the splits' partial sums in order in a second kernel. Rows past a matrix's end, batch
// rows past the chunk and K past cols read as zero (TMA out of bounds fill). Each K step moves
// 48 KB for 4.2 MFLOP of MMA (the split doubles both the input tiles and the MMAs), so the
// kernel is bound by the operand traffic through L2, not by the tensor pipe. Every wait is bounded (globaltimer, 2 s); on expiry the kernel records an error
// code, drains what it issued and frees its TMEM.
#include <algorithm>

#include "qattn_common.cuh"
#include "sm100.cuh"

namespace qattn {
namespace {

using namespace sm100;

constexpr int GM = 128, GN = 128, GK = 64, GSTAGES = 4, GTHREADS = 128;
constexpr uint32_t W_TILE = GM * GK * 2;                 // 16 KB
constexpr uint32_t X_TILE = GN * GK * 2;                 // 16 KB
constexpr uint32_t STAGE_BYTES = W_TILE + 2 * X_TILE;    // 48 KB
constexpr int GSMEM = GSTAGES * STAGE_BYTES + 1024 + 128;  // + alignment slack + barriers
static_assert(GSMEM <= 232448, "shared memory per CTA");

struct GemmMaps {
    CUtensorMap w[MAX_PROJECT_MATS];
    CUtensorMap xhi, xlo;
};

struct GemmArgs {
    int n_mats;
    int rows[MAX_PROJECT_MATS];
    int tile0[MAX_PROJECT_MATS + 1];  // first row tile of each matrix
    float* y[MAX_PROJECT_MATS];       // [batch][rows[m]]
    int cols, b0, nb;                 // this chunk: batch rows [b0, b0 + nb)
    const float* inv_scale;           // [nb]: 2^-e of each split row
    int ksplit;                       // K split over blockIdx.z (1: the tile writes y directly)
    int total_rows;                   // sum of rows: the row pitch of `partial`
    int row0_of[MAX_PROJECT_MATS];    // first row of each matrix in that concatenation
    float* partial;                   // ksplit > 1: [ksplit][nb][total_rows] tile sums, summed in order
    int* error;
};

__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int cols, __half* hi, __half* lo,
                                                        float* inv_scale) {
    __shared__ float red[8];
    const float* xr = x + (size_t)blockIdx.x * cols;
    float m = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(xr[c]));
    #pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    int e = 0;
    if (m > 0.f && m <= 3.0e38f) {                       // finite, non-zero: bring the max to [2^13, 2^14)
        int ex;
        frexpf(m, &ex);                                   // m = f * 2^ex, f in [0.5, 1)
        e = 14 - ex;
    }
    const float s = ldexpf(1.f, e);
    __half* h = hi + (size_t)blockIdx.x * cols;
    __half* l = lo + (size_t)blockIdx.x * cols;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float v = xr[c] * s;
        const __half vh = __float2half_rn(v);
        h[c] = vh;
        l[c] = __float2half_rn(v - __half2float(vh));
    }
    if (threadIdx.x == 0) inv_scale[blockIdx.x] = ldexpf(1.f, -e);
}

__global__ void __launch_bounds__(GTHREADS, 1) project_gemm_kernel(const __grid_constant__ GemmMaps maps,
                                                                  const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + GSTAGES * STAGE_BYTES);
    uint64_t* empty = full + GSTAGES;
    uint64_t* done = empty + GSTAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int abort_flag, never_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int m = 0;
    const int t = blockIdx.x;
    while (m + 1 < a.n_mats && t >= a.tile0[m + 1]) ++m;
    const int r0 = (t - a.tile0[m]) * GM;                  // first weight row of the tile
    const int bt0 = blockIdx.y * GN;                       // first batch row of the tile (in the chunk)
    const int KT_all = (a.cols + GK - 1) / GK;
    const int kt_begin = (int)((long long)KT_all * blockIdx.z / a.ksplit);
    const int KT = (int)((long long)KT_all * (blockIdx.z + 1) / a.ksplit) - kt_begin;   // this split's K steps

    if (tid == 0) {
        abort_flag = 0;
        never_abort = 0;
        for (int s = 0; s < GSTAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, GN); tmem_relinquish(); }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&maps.w[m]);
        prefetch_tmap(&maps.xhi);
        prefetch_tmap(&maps.xlo);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    volatile int* abortp = &abort_flag;
    auto fail = [&](int code) { *abortp = 1; atomicCAS(a.error, 0, code); };

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: K step kt into stage kt % GSTAGES ----
        int issued = 0;
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % GSTAGES;
            if (kt >= GSTAGES && !mbar_wait(&empty[s], ((kt / GSTAGES) - 1) & 1, abortp)) { fail(61); ok = false; break; }
            uint8_t* st = smem + s * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            const int kx = (kt_begin + kt) * GK;
            tma_load_3d(st, &maps.w[m], kx, r0, 0, &full[s]);
            tma_load_3d(st + W_TILE, &maps.xhi, kx, bt0, 0, &full[s]);
            tma_load_3d(st + W_TILE + X_TILE, &maps.xlo, kx, bt0, 0, &full[s]);
            ++issued;
        }
        if (!ok) {                                         // drain this thread's copies (bounded)
            for (int it = std::max(0, issued - GSTAGES); it < issued; ++it)
                mbar_wait(&full[it % GSTAGES], (it / GSTAGES) & 1, &never_abort, 500000000ull);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer: D (+)= W x_hi^T + W x_lo^T per 16-column K slice ----
        const uint32_t idesc = idesc_f16_f32(GM, GN, false);
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % GSTAGES;
            if (!mbar_wait(&full[s], (kt / GSTAGES) & 1, abortp)) { fail(62); break; }
            tc_fence_after();
            const uint32_t wb = smem_u32(smem + s * STAGE_BYTES), hb = wb + W_TILE, lb = hb + X_TILE;
            #pragma unroll
            for (int ks = 0; ks < GK / 16; ++ks) {
                mma_f16_ss(tmem, sw128_desc(wb + ks * 32, 16, 1024), sw128_desc(hb + ks * 32, 16, 1024), idesc,
                           (kt > 0 || ks > 0) ? 1u : 0u);
                mma_f16_ss(tmem, sw128_desc(wb + ks * 32, 16, 1024), sw128_desc(lb + ks * 32, 16, 1024), idesc, 1u);
            }
            mma_commit(&empty[s]);                         // the stage is free once these MMAs complete
        }
        mma_commit(done);                                  // every MMA issued: the accumulator is final
    }
    __syncwarp();

    // ---- epilogue: warp w holds weight rows r0 + 32 w + lane; 32 batch columns per TMEM load ----
    if (!mbar_wait(done, 0, &never_abort)) atomicCAS(a.error, 0, 63);
    tc_fence_after();
    const int r = r0 + warp * 32 + lane;
    const int rows_m = a.rows[m];
    float* y = a.y[m];
    // split K: this split's sum goes to partial[z][b][row offset of m + r]
    float* part = a.ksplit > 1 ? a.partial + (size_t)blockIdx.z * a.nb * a.total_rows : nullptr;
    #pragma unroll 1
    for (int c0 = 0; c0 < GN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
        tmem_wait_ld();
        if (r < rows_m) {
            #pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int b = bt0 + c0 + j;
                if (b < a.nb) {
                    const float val = __uint_as_float(v[j]) * a.inv_scale[b];
                    if (part) part[(size_t)b * a.total_rows + a.row0_of[m] + r] = val;
                    else y[(size_t)(a.b0 + b) * rows_m + r] = val;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, GN);
    }
}

// y of a split-K launch: the splits' sums added in split order (deterministic).
__global__ void __launch_bounds__(256) sum_splits_kernel(const GemmArgs a) {
    const size_t n = (size_t)a.nb * a.total_rows;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = a.partial[i];
        for (int z = 1; z < a.ksplit; ++z) v += a.partial[(size_t)z * n + i];
        const int b = (int)(i / a.total_rows), row = (int)(i - (size_t)b * a.total_rows);
        int m = 0;
        while (m + 1 < a.n_mats && row >= a.row0_of[m + 1]) ++m;
        a.y[m][(size_t)(a.b0 + b) * a.rows[m] + (row - a.row0_of[m])] = v;
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

// Split-K partial sums share the scratch: room for 4 splits of a 512 x 2048 output.
constexpr size_t PARTIAL_FLOATS_MAX = (size_t)4 * GEMM_CHUNK_ROWS * 2048;

size_t project_gemm_scratch_bytes() {
    return (size_t)GEMM_CHUNK_ROWS * GEMM_MAX_COLS * 2 * sizeof(__half) + GEMM_CHUNK_ROWS * sizeof(float) + 512 +
           PARTIAL_FLOATS_MAX * sizeof(float);
}

int launch_project_gemm(const ProjectArgs& p, void* scratch, int* error, cudaStream_t s) {
    if (p.cols > GEMM_MAX_COLS || !scratch) return -1;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(project_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GSMEM) != cudaSuccess)
            return -2;
        attr = true;
    }
    GemmMaps maps;
    GemmArgs a{};
    a.n_mats = p.n_mats;
    a.cols = p.cols;
    a.error = error;
    a.tile0[0] = 0;
    a.total_rows = 0;
    for (int m = 0; m < p.n_mats; ++m) {
        a.row0_of[m] = a.total_rows;
        a.total_rows += p.rows[m];
        a.rows[m] = p.rows[m];
        a.y[m] = p.y[m];
        a.tile0[m + 1] = a.tile0[m] + (p.rows[m] + GM - 1) / GM;
        if (!encode_rows(&maps.w[m], p.w[m], p.rows[m], p.cols)) return -3;
    }
    for (int b0 = 0; b0 < p.batch; b0 += GEMM_CHUNK_ROWS) {
        const int nb = std::min(GEMM_CHUNK_ROWS, p.batch - b0);
        __half* hi = static_cast<__half*>(scratch);
        __half* lo = hi + (((size_t)nb * p.cols + 127) & ~size_t(127));
        float* inv = reinterpret_cast<float*>(lo + (((size_t)nb * p.cols + 127) & ~size_t(127)));
        if (!encode_rows(&maps.xhi, hi, nb, p.cols) || !encode_rows(&maps.xlo, lo, nb, p.cols)) return -3;
        split_rows_kernel<<<nb, 256, 0, s>>>(p.x + (size_t)b0 * p.cols, p.cols, hi, lo, inv);
        a.b0 = b0;
        a.nb = nb;
        a.inv_scale = inv;
        // Launches with fewer tiles than SMs split K (at least four K steps per split) so that
        // more SMs stream the matrix; the partial sums are then added in split order.
        const int tiles = a.tile0[p.n_mats] * ((nb + GN - 1) / GN), KT = (p.cols + GK - 1) / GK;
        int sms = NUM_SMS_B200, dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        a.ksplit = std::max(1, std::min({4, sms / std::max(1, tiles), KT / 4}));
        a.partial = reinterpret_cast<float*>(
            reinterpret_cast<char*>(scratch) + (size_t)GEMM_CHUNK_ROWS * GEMM_MAX_COLS * 2 * sizeof(__half) +
            GEMM_CHUNK_ROWS * sizeof(float) + 512);
        if ((size_t)a.ksplit * nb * a.total_rows > PARTIAL_FLOATS_MAX) a.ksplit = 1;
        project_gemm_kernel<<<dim3(a.tile0[p.n_mats], (nb + GN - 1) / GN, a.ksplit), GTHREADS, GSMEM, s>>>(maps, a);
        if (a.ksplit > 1) {
            const size_t n = (size_t)nb * a.total_rows;
            sum_splits_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, (size_t)sms * 8), 256, 0, s>>>(a);
        }
    }
    return 0;
}

}  // namespace qattn
