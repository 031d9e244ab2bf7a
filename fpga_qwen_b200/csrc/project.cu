// project.cu — decode projections over FP16 matrices in the reference's eight-lane order.
//
// Replaces Model::Impl::project for one row (tampajohn/fpga-qwen engine/core.cpp:292-301:
// dot / dot4, :119-147), project_group (:302-320, q/k/v and gate/up sharing one input), the
// B2 verification forms (project_verify / project_group_verify, :321-349, dot_verify_pair /
// dot_verify_two_rows, :182-206) and the FP16-only vocabulary head (:705, :713):
//     y[b][r] = dot(x[b], W[r])   over an FP16 matrix W [rows][cols], FP32 x and y.
// The reference's dot keeps two 4-lane FP32 accumulators, a over channels j..j+3 and b over
// j+4..j+7, fused multiply-adds with j ascending by 8, then vaddvq(a + b), whose pairwise
// reduction is (s0 + s1) + (s2 + s3) with s_i = a_i + b_i. Every variant above keeps that
// sequence per output, so one kernel reproduces all of them bit for bit: two threads own one
// output row, thread 0 the four chains of a (channels j..j+3), thread 1 the four of b
// (channels j+4..j+7), each step one 8-byte load of four FP16 weights and two packed FP32x2
// fused multiply-adds (each lane rounded once, as vfmaq_f32); one shuffle then forms
// s_i = a_i + b_i and each row's (s0 + s1) + (s2 + s3).
//
// The work is HBM-bound (2 bytes of matrix per multiply-add). The kernel is persistent (one
// wave of CTAs): a CTA owns row tiles in turn and streams their columns through a cp.async
// ring of 128-column chunks that runs on from one tile to the next (16-byte copies with
// shift-only indexing; shared-memory rows padded by 16 bytes so a warp's 16 rows read without
// bank conflicts); each stage also carries the chunk's input columns, so the multiply-add
// chains read only shared memory. Several matrices that share one input (the reference's
// project_group) run as one launch over their concatenated row tiles.
#include <algorithm>

#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int PR_CHUNK = 128;                     // columns per ring stage
constexpr int PR_ROW_BYTES = PR_CHUNK * 2 + 16;   // padded: row r starts 4 banks after row r-1
constexpr int PR_BATCH = 2;                       // batch rows per pass over a tile
constexpr int PR_PIECES = PR_CHUNK * 2 / 16;      // 16-byte pieces per row segment of a full chunk
static_assert(PR_PIECES == 16, "shift-only copy indexing assumes 16 pieces per row segment");
// Tiles of ROWS rows, two threads per row. Large matrices (the vocabulary head) use 64-row
// tiles and a 4-stage ring; a launch with fewer 64-row tiles than half a wave uses 16-row tiles,
// four times as many CTAs, and an 8-stage ring that holds a whole 1024-column tile in flight,
// so that small per-layer matrices still spread over the GPU and wait for memory only once.
template <int ROWS> struct Shape {
    static constexpr int THREADS = 2 * ROWS;
    static constexpr int STAGES = ROWS >= 64 ? 4 : 8;
    static constexpr int W_BYTES = ROWS * PR_ROW_BYTES;
    static constexpr int STAGE_BYTES = W_BYTES + PR_BATCH * PR_CHUNK * 4;   // + the input columns of the chunk
    static constexpr int SMEM = STAGES * STAGE_BYTES;
};

// Position in a CTA's chunk sequence: column chunk k of pass `pass` (a pair of batch rows) of the
// CTA's tile number `it`, advanced without divisions.
struct Cursor {
    int k = 0, pass = 0, it = 0;
    __device__ __forceinline__ bool next(int nch, int passes) {     // true when a new tile starts
        if (++k < nch) return false;
        k = 0;
        if (++pass < passes) return false;
        pass = 0;
        ++it;
        return true;
    }
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r, ua = *reinterpret_cast<unsigned long long*>(&a), ub = *reinterpret_cast<unsigned long long*>(&b),
                          uc = *reinterpret_cast<unsigned long long*>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(ua), "l"(ub), "l"(uc));
    return *reinterpret_cast<float2*>(&r);
}

struct Tile { int m, r0, rows; const __half* w; };
template <int ROWS>
__device__ __forceinline__ Tile tile_at(const ProjectArgs& a, int t) {
    Tile ti;
    ti.m = 0;
    while (ti.m + 1 < a.n_mats && t >= a.tile0[ti.m + 1]) ++ti.m;
    ti.r0 = (t - a.tile0[ti.m]) * ROWS;
    ti.rows = min(ROWS, a.rows[ti.m] - ti.r0);
    ti.w = a.w[ti.m] + (size_t)ti.r0 * a.cols;
    return ti;
}

// Persistent: CTA c takes tiles c, c + grid, c + 2*grid, ...; every tile is `passes` passes
// (pairs of batch rows) of `nch` column chunks. The CTA's chunks form one sequence that the
// ring streams without draining between tiles, so HBM sees a continuous read per CTA.
template <int ROWS>
__global__ void __launch_bounds__(Shape<ROWS>::THREADS) project_kernel(const ProjectArgs a) {
    using S = Shape<ROWS>;
    extern __shared__ __align__(16) uint8_t ring[];
    const int tid = threadIdx.x, r = tid >> 1, hl = tid & 1;     // row of the tile, a (0) or b (1) lanes
    const int ntiles = a.tile0[a.n_mats];
    const int nch = (a.cols + PR_CHUNK - 1) / PR_CHUNK;
    const int passes = (a.batch + PR_BATCH - 1) / PR_BATCH;
    const int my_tiles = ((int)blockIdx.x < ntiles) ? (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int per_tile = passes * nch;
    const int total = my_tiles * per_tile;

    // chunk g of the sequence into ring stage g % STAGES: the tile's row segments and the
    // pass's input columns (16-byte copies), so the multiply-add chains read only shared memory.
    // The producer cursor runs STAGES - 1 chunks ahead of the consumers'.
    Cursor pc;
    Tile pt = tile_at<ROWS>(a, blockIdx.x);
    int g_load = 0;
    auto load = [&]() {
        if (g_load < total) {
            const int k = pc.k, b0 = pc.pass * PR_BATCH;
            const int cw = min(PR_CHUNK, a.cols - k * PR_CHUNK);     // columns in this chunk (multiple of 8)
            uint8_t* st = ring + (g_load % S::STAGES) * S::STAGE_BYTES;
            const __half* src = pt.w + (size_t)k * PR_CHUNK;
            if (cw == PR_CHUNK) {
                #pragma unroll
                for (int i = 0; i < ROWS * PR_PIECES / S::THREADS; ++i) {   // 8 pieces per thread
                    const int piece = tid + i * S::THREADS, rr = piece >> 4, p = piece & 15;
                    if (rr < pt.rows) cp_async16(st + rr * PR_ROW_BYTES + p * 16, src + (size_t)rr * a.cols + p * 8);
                }
            } else {
                const int per_row = cw / 8;                          // the ragged last chunk of a row
                for (int i = tid; i < pt.rows * per_row; i += S::THREADS) {
                    const int rr = i / per_row, p = i - rr * per_row;
                    cp_async16(st + rr * PR_ROW_BYTES + p * 16, src + (size_t)rr * a.cols + p * 8);
                }
            }
            const int xq = cw / 4;                                   // 16-byte pieces per input row
            const int nb = min(PR_BATCH, a.batch - b0);
            for (int i = tid; i < nb * PR_CHUNK / 4; i += S::THREADS) {
                const int bb = i >> 5, p = i & 31;                   // PR_CHUNK / 4 == 32 pieces per row
                if (p < xq)
                    cp_async16(st + S::W_BYTES + bb * PR_CHUNK * 4 + p * 16,
                               a.x + (size_t)(b0 + bb) * a.cols + (size_t)k * PR_CHUNK + p * 4);
            }
            ++g_load;
            if (pc.next(nch, passes) && g_load < total)
                pt = tile_at<ROWS>(a, (int)blockIdx.x + pc.it * (int)gridDim.x);
        }
        cp_commit();
    };

    #pragma unroll
    for (int s = 0; s < S::STAGES - 1; ++s) load();
    float2 acc[PR_BATCH][2];                         // this thread's four lane chains (two pairs) per batch row
    #pragma unroll
    for (int bb = 0; bb < PR_BATCH; ++bb) acc[bb][0] = acc[bb][1] = make_float2(0.f, 0.f);
    Cursor cc;
    Tile ti = tile_at<ROWS>(a, blockIdx.x);
    for (int g = 0; g < total; ++g) {
        cp_wait<S::STAGES - 2>();                        // chunk g has landed (this thread's copies)
        __syncthreads();                                 // ... everyone's; chunk g-1 fully read
        load();                                          // chunk g + STAGES - 1, into the stage chunk g-1 used
        const int k = cc.k, b0 = cc.pass * PR_BATCH, nb = min(PR_BATCH, a.batch - b0);
        const int cw = min(PR_CHUNK, a.cols - k * PR_CHUNK);
        const uint8_t* st = ring + (g % S::STAGES) * S::STAGE_BYTES;
        const uint8_t* row = st + r * PR_ROW_BYTES + hl * 8;
        const float* xs = reinterpret_cast<const float*>(st + S::W_BYTES) + hl * 4;
        #pragma unroll 4
        for (int jj = 0; jj < cw / 8; ++jj) {
            const uint2 wv = *reinterpret_cast<const uint2*>(row + jj * 16);      // 4 FP16 weights
            const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
            const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
            const float4 x0 = *reinterpret_cast<const float4*>(xs + jj * 8);
            acc[0][0] = ffma2(make_float2(x0.x, x0.y), w01, acc[0][0]);
            acc[0][1] = ffma2(make_float2(x0.z, x0.w), w23, acc[0][1]);
            if (nb == PR_BATCH) {
                const float4 x1 = *reinterpret_cast<const float4*>(xs + PR_CHUNK + jj * 8);
                acc[1][0] = ffma2(make_float2(x1.x, x1.y), w01, acc[1][0]);
                acc[1][1] = ffma2(make_float2(x1.z, x1.w), w23, acc[1][1]);
            }
        }
        if (k == nch - 1) {
            // s_i = a_i + b_i (the partner thread holds b), then (s0 + s1) + (s2 + s3)
            #pragma unroll
            for (int bb = 0; bb < PR_BATCH; ++bb) {
                float2 o0, o1;
                o0.x = __shfl_xor_sync(0xffffffffu, acc[bb][0].x, 1); o0.y = __shfl_xor_sync(0xffffffffu, acc[bb][0].y, 1);
                o1.x = __shfl_xor_sync(0xffffffffu, acc[bb][1].x, 1); o1.y = __shfl_xor_sync(0xffffffffu, acc[bb][1].y, 1);
                const float s0 = acc[bb][0].x + o0.x, s1 = acc[bb][0].y + o0.y;
                const float s2 = acc[bb][1].x + o1.x, s3 = acc[bb][1].y + o1.y;
                const float y = (s0 + s1) + (s2 + s3);
                if (bb < nb && hl == 0 && r < ti.rows) a.y[ti.m][(size_t)(b0 + bb) * a.rows[ti.m] + ti.r0 + r] = y;
                acc[bb][0] = acc[bb][1] = make_float2(0.f, 0.f);
            }
        }
        if (cc.next(nch, passes) && g + 1 < total) ti = tile_at<ROWS>(a, (int)blockIdx.x + cc.it * (int)gridDim.x);
    }
    cp_wait<0>();
}

// ---- small launches: every row of the launch resident in shared memory at once ----------------
// The per-layer matrices of one decode token (1,024 to 6,144 rows) are too small to keep a ring
// busy: the persistent kernel's few CTAs would wait for memory once per chunk. Here each of
// about one CTA per SM takes a slice of R consecutive rows (of the launch's concatenated
// matrices), issues copies of the whole slice at once in four column groups and runs the
// multiply-add chains over each group as it lands, so the launch costs about one memory latency
// plus its bytes at full bandwidth. The chains, their order and the final reduction are the
// persistent kernel's, so both give the same bits. Launched as a programmatic dependent: the
// weight copies (constant data) start while the previous kernel finishes; the input is read
// only after griddepcontrol.wait.
constexpr int PS_THREADS = 256;
constexpr int PS_GROUPS = 4;                       // column groups, one cp.async group each
constexpr int PS_MAX_ROWS = PS_THREADS / 2;        // at least two threads per row
constexpr int PS_MAX_SMEM = 200 * 1024;

__device__ __forceinline__ int ps_stride(int cols) { return cols * 2 + 16; }   // padded row, bytes

// TPR threads per row, each owning 8 / TPR of the dot's eight lanes (a0..a3 = channels j..j+3,
// b0..b3 = channels j+4..j+7 of every 8-channel step): every lane is still one chain of fused
// multiply-adds in ascending j, so the bits do not depend on TPR. Slices of few rows (o_proj,
// down_proj: about 7 rows per SM) use 8 threads per row, so that a CTA runs more than one
// warp of chains; TPR = 2 reproduces the persistent kernel's thread layout.
template <int TPR>
__global__ void __launch_bounds__(PS_THREADS) project_small_kernel(const ProjectArgs a, int rows_per_cta) {
    constexpr int LANES = 8 / TPR;                 // lanes (channels of each 8-channel step) per thread
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ const __half* rowptr[PS_MAX_ROWS];
    __shared__ float* outptr[PS_MAX_ROWS];
    __shared__ int outstride[PS_MAX_ROWS];
    const int tid = threadIdx.x, cols = a.cols, pieces = cols / 8, stride = ps_stride(cols);
    int total = 0;
    for (int m = 0; m < a.n_mats; ++m) total += a.rows[m];
    const int row0 = blockIdx.x * rows_per_cta, nrows = min(rows_per_cta, total - row0);
    const int xbytes = a.batch * cols * 4;
    uint8_t* wbase = sm + xbytes;
    if (tid < nrows) {                             // the matrix and output of each row of the slice
        int m = 0, r = row0 + tid;
        while (m + 1 < a.n_mats && r >= a.rows[m]) r -= a.rows[m++];
        rowptr[tid] = a.w[m] + (size_t)r * cols;
        outptr[tid] = a.y[m] + r;
        outstride[tid] = a.rows[m];
    }
    __syncthreads();
    #pragma unroll
    for (int g = 0; g < PS_GROUPS; ++g) {
        const int p0 = pieces * g / PS_GROUPS, np = pieces * (g + 1) / PS_GROUPS - p0;
        for (int i = tid; i < nrows * np; i += PS_THREADS) {
            const int r = i / np, p = p0 + (i - r * np);
            cp_async16(wbase + r * stride + p * 16, rowptr[r] + p * 8);
        }
        cp_commit();
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");        // the input is the previous kernel's
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (int i = tid; i < xbytes / 16; i += PS_THREADS)
        reinterpret_cast<float4*>(sm)[i] = __ldcg(reinterpret_cast<const float4*>(a.x) + i);

    // TPR threads per row; the warps that hold no row only join the barriers
    const int r = tid / TPR, q = tid % TPR;
    const bool active_warp = (tid & ~31) < TPR * nrows;
    const uint8_t* row = wbase + min(r, nrows - 1) * stride + q * LANES * 2;
    const float* xs = reinterpret_cast<const float*>(sm) + q * LANES;
    float acc[PR_BATCH][LANES];
    #pragma unroll
    for (int bb = 0; bb < PR_BATCH; ++bb)
        #pragma unroll
        for (int l = 0; l < LANES; ++l) acc[bb][l] = 0.f;
    #pragma unroll
    for (int g = 0; g < PS_GROUPS; ++g) {
        if (g == 0) cp_wait<PS_GROUPS - 1>();
        else if (g == 1) cp_wait<PS_GROUPS - 2>();
        else if (g == 2) cp_wait<PS_GROUPS - 3>();
        else cp_wait<0>();
        __syncthreads();
        if (!active_warp) continue;
        const int j0 = pieces * g / PS_GROUPS, j1 = pieces * (g + 1) / PS_GROUPS;
        #pragma unroll 4
        for (int jj = j0; jj < j1; ++jj) {
            float w[LANES], x0[LANES], x1[LANES];
            if constexpr (LANES == 4) {
                const uint2 wv = *reinterpret_cast<const uint2*>(row + jj * 16);
                const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
                const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
                w[0] = w01.x; w[1] = w01.y; w[2] = w23.x; w[3] = w23.y;
                const float4 v = *reinterpret_cast<const float4*>(xs + jj * 8);
                x0[0] = v.x; x0[1] = v.y; x0[2] = v.z; x0[3] = v.w;
            } else if constexpr (LANES == 2) {
                const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(row + jj * 16));
                w[0] = w01.x; w[1] = w01.y;
                const float2 v = *reinterpret_cast<const float2*>(xs + jj * 8);
                x0[0] = v.x; x0[1] = v.y;
            } else {
                w[0] = __half2float(*reinterpret_cast<const __half*>(row + jj * 16));
                x0[0] = xs[jj * 8];
            }
            #pragma unroll
            for (int l = 0; l < LANES; ++l) acc[0][l] = fmaf(x0[l], w[l], acc[0][l]);
            if (a.batch == PR_BATCH) {
                #pragma unroll
                for (int l = 0; l < LANES; ++l) x1[l] = xs[cols + jj * 8 + l];
                #pragma unroll
                for (int l = 0; l < LANES; ++l) acc[1][l] = fmaf(x1[l], w[l], acc[1][l]);
            }
        }
    }
    if (!active_warp) return;
    #pragma unroll
    for (int bb = 0; bb < PR_BATCH; ++bb) {
        // s_i = a_i + b_i, then (s0 + s1) + (s2 + s3), with the reference's association
        float y;
        if constexpr (TPR == 2) {                  // q = 0: a0..a3, q = 1: b0..b3
            float s[4];
            #pragma unroll
            for (int l = 0; l < 4; ++l) s[l] = acc[bb][l] + __shfl_xor_sync(0xffffffffu, acc[bb][l], 1);
            y = (s[0] + s[1]) + (s[2] + s[3]);
        } else if constexpr (TPR == 4) {           // q: lanes 2q, 2q+1 (q = 0, 1: a; 2, 3: b)
            const float s0 = acc[bb][0] + __shfl_xor_sync(0xffffffffu, acc[bb][0], 2);
            const float s1 = acc[bb][1] + __shfl_xor_sync(0xffffffffu, acc[bb][1], 2);
            const float h = s0 + s1;               // q = 0: s0 + s1, q = 1: s2 + s3
            y = h + __shfl_xor_sync(0xffffffffu, h, 1);
        } else {                                   // q: lane q (0..3: a_q, 4..7: b_(q-4))
            const float s = acc[bb][0] + __shfl_xor_sync(0xffffffffu, acc[bb][0], 4);
            const float h = s + __shfl_xor_sync(0xffffffffu, s, 1);     // q = 0: s0 + s1, q = 2: s2 + s3
            y = h + __shfl_xor_sync(0xffffffffu, h, 2);
        }
        if (bb < a.batch && q == 0 && r < nrows) outptr[r][(size_t)bb * outstride[r]] = y;
    }
}

// The small-launch plan: rows per CTA, threads per row and dynamic shared memory, or false when
// the launch belongs to the persistent kernel (a batch beyond one pass, or a slice too large).
bool small_plan(const ProjectArgs& a, int sms, int* rows_per_cta, int* tpr, int* grid, size_t* smem) {
    if (a.batch > PR_BATCH) return false;
    int total = 0;
    for (int m = 0; m < a.n_mats; ++m) total += a.rows[m];
    const int r = (total + sms - 1) / sms;
    if (r > PS_MAX_ROWS) return false;
    const size_t bytes = (size_t)a.batch * a.cols * 4 + (size_t)r * (a.cols * 2 + 16);
    if (bytes > PS_MAX_SMEM) return false;
    *rows_per_cta = r;
    *tpr = 8 * r <= PS_THREADS ? 8 : 4 * r <= PS_THREADS ? 4 : 2;
    *grid = (total + r - 1) / r;
    *smem = bytes;
    return true;
}

template <int ROWS>
int resident_ctas() {
    // one wave of persistent CTAs: as many as fit on every SM at once
    static int resident = 0;
    if (!resident) {
        int dev = 0, sms = NUM_SMS_B200, per_sm = 1;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaFuncSetAttribute(project_kernel<ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, Shape<ROWS>::SMEM);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, project_kernel<ROWS>, Shape<ROWS>::THREADS,
                                                          Shape<ROWS>::SMEM) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        resident = sms * per_sm;
    }
    return resident;
}

template <int ROWS>
void launch_rows(ProjectArgs a, cudaStream_t s) {
    a.tile0[0] = 0;
    for (int m = 0; m < a.n_mats; ++m) a.tile0[m + 1] = a.tile0[m] + (a.rows[m] + ROWS - 1) / ROWS;
    const int grid = std::min(a.tile0[a.n_mats], resident_ctas<ROWS>());
    project_kernel<ROWS><<<grid, Shape<ROWS>::THREADS, Shape<ROWS>::SMEM, s>>>(a);
}

}  // namespace

void launch_project(ProjectArgs a, cudaStream_t s) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        sms = NUM_SMS_B200;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaFuncSetAttribute(project_small_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, PS_MAX_SMEM);
        cudaFuncSetAttribute(project_small_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, PS_MAX_SMEM);
        cudaFuncSetAttribute(project_small_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, PS_MAX_SMEM);
    }
    int rows_per_cta = 0, tpr = 2, grid = 0;
    size_t smem = 0;
    if (small_plan(a, sms, &rows_per_cta, &tpr, &grid, &smem)) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(grid); cfg.blockDim = dim3(PS_THREADS); cfg.dynamicSmemBytes = smem; cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr; cfg.numAttrs = 1;
        if (tpr == 8) cudaLaunchKernelEx(&cfg, project_small_kernel<8>, a, rows_per_cta);
        else if (tpr == 4) cudaLaunchKernelEx(&cfg, project_small_kernel<4>, a, rows_per_cta);
        else cudaLaunchKernelEx(&cfg, project_small_kernel<2>, a, rows_per_cta);
        return;
    }
    int tiles64 = 0;
    for (int m = 0; m < a.n_mats; ++m) tiles64 += (a.rows[m] + 63) / 64;
    if (2 * tiles64 >= resident_ctas<64>()) launch_rows<64>(a, s);
    else launch_rows<16>(a, s);
}

}  // namespace qattn
