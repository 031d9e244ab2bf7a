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
// sequence per output, so one kernel reproduces all of them bit for bit: eight threads own
// one output row, thread c the lane chain of channels c, c+8, c+16, ... (chain c < 4 is a_c,
// chain c >= 4 is b_{c-4}); after the last column the eight chains combine with three
// shuffles in the reference's order.
//
// The work is HBM-bound (2 bytes of matrix per multiply-add): a CTA of 128 threads owns 16
// rows and streams their columns through a 4-stage cp.async ring of 256-column chunks
// (16-byte copies, whole 512-byte row segments per warp, padded shared-memory rows so the
// eight chains of four rows read without bank conflicts). The input row is read through the
// read-only cache into registers a chunk at a time. Several matrices that share one input
// (the reference's project_group) run as one launch over their concatenated row tiles.
#include <algorithm>

#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int PR_ROWS = 16;                       // rows per CTA
constexpr int PR_THREADS = PR_ROWS * 8;           // eight lane chains per row
constexpr int PR_CHUNK = 256;                     // columns per ring stage
constexpr int PR_STAGES = 4;
constexpr int PR_ROW_BYTES = PR_CHUNK * 2 + 16;   // padded: row r starts 4 banks after row r-1
constexpr int PR_STAGE_BYTES = PR_ROWS * PR_ROW_BYTES;
constexpr int PR_SMEM = PR_STAGES * PR_STAGE_BYTES;
constexpr int PR_BATCH = 2;                       // batch rows per pass over the matrix

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(PR_THREADS) project_kernel(const ProjectArgs a) {
    extern __shared__ __align__(16) uint8_t ring[];
    // this CTA's matrix and first row
    int m = 0;
    while (m + 1 < a.n_mats && (int)blockIdx.x >= a.tile0[m + 1]) ++m;
    const int r0 = ((int)blockIdx.x - a.tile0[m]) * PR_ROWS;
    const int rows_here = min(PR_ROWS, a.rows[m] - r0);
    const __half* W = a.w[m] + (size_t)r0 * a.cols;
    const int tid = threadIdx.x, r = tid >> 3, c = tid & 7;
    const int nch = (a.cols + PR_CHUNK - 1) / PR_CHUNK;

    // chunk k of the CTA's rows into ring stage k % PR_STAGES: each row segment is
    // (cols of the chunk) x 2 bytes, copied 16 bytes per thread-step
    auto load = [&](int k) {
        if (k < nch) {
            const int cw = min(PR_CHUNK, a.cols - k * PR_CHUNK);     // columns in this chunk (multiple of 8)
            const int per_row = cw / 8;                              // 16-byte pieces per row
            uint8_t* st = ring + (k % PR_STAGES) * PR_STAGE_BYTES;
            for (int i = tid; i < rows_here * per_row; i += PR_THREADS) {
                const int rr = i / per_row, p = i - rr * per_row;
                cp_async16(st + rr * PR_ROW_BYTES + p * 16, W + (size_t)rr * a.cols + (size_t)k * PR_CHUNK + p * 8);
            }
        }
        cp_commit();
    };

    for (int b0 = 0; b0 < a.batch; b0 += PR_BATCH) {
        const int nb = min(PR_BATCH, a.batch - b0);
        float acc[PR_BATCH] = {0.f, 0.f};
        if (b0 > 0) __syncthreads();                         // the previous pass has read the ring
        #pragma unroll
        for (int s = 0; s < PR_STAGES - 1; ++s) load(s);
        for (int k = 0; k < nch; ++k) {
            cp_wait<PR_STAGES - 2>();                        // chunk k has landed (this thread's copies)
            __syncthreads();                                 // ... everyone's; chunk k-1 fully read
            load(k + PR_STAGES - 1);                         // into the stage chunk k-1 used
            const int cw = min(PR_CHUNK, a.cols - k * PR_CHUNK);
            const uint8_t* row = ring + (k % PR_STAGES) * PR_STAGE_BYTES + r * PR_ROW_BYTES + c * 2;
            const float* xb = a.x + (size_t)b0 * a.cols + (size_t)k * PR_CHUNK + c;
            if (nb == PR_BATCH) {
                #pragma unroll 8
                for (int jj = 0; jj < cw / 8; ++jj) {
                    const float wv = __half2float(*reinterpret_cast<const __half*>(row + jj * 16));
                    acc[0] = fmaf(__ldg(xb + jj * 8), wv, acc[0]);
                    acc[1] = fmaf(__ldg(xb + a.cols + jj * 8), wv, acc[1]);
                }
            } else {
                #pragma unroll 8
                for (int jj = 0; jj < cw / 8; ++jj) {
                    const float wv = __half2float(*reinterpret_cast<const __half*>(row + jj * 16));
                    acc[0] = fmaf(__ldg(xb + jj * 8), wv, acc[0]);
                }
            }
        }
        cp_wait<0>();
        // (s0 + s1) + (s2 + s3), s_i = a_i + b_i: chain c and chain c + 4, then pairs
        #pragma unroll
        for (int bb = 0; bb < PR_BATCH; ++bb) {
            const float s = acc[bb] + __shfl_xor_sync(0xffffffffu, acc[bb], 4);
            const float t = s + __shfl_xor_sync(0xffffffffu, s, 1);
            const float y = t + __shfl_xor_sync(0xffffffffu, t, 2);
            if (bb < nb && c == 0 && r < rows_here) a.y[m][(size_t)(b0 + bb) * a.rows[m] + r0 + r] = y;
        }
    }
}

}  // namespace

void launch_project(ProjectArgs a, cudaStream_t s) {
    a.tile0[0] = 0;
    for (int m = 0; m < a.n_mats; ++m) a.tile0[m + 1] = a.tile0[m] + (a.rows[m] + PR_ROWS - 1) / PR_ROWS;
    project_kernel<<<a.tile0[a.n_mats], PR_THREADS, PR_SMEM, s>>>(a);
}

}  // namespace qattn
