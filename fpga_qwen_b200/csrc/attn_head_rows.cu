// attn_head_rows.cu — FP32 causal attention for the first rows of a sequence.
//
// Prefill rows at absolute position < 128 attend to at most 128 keys, and their attention
// is concentrated on few keys; there FP16 probabilities (tensor-core path) would exceed the
// 1e-3 output tolerance, so these rows are computed in FP32 on CUDA cores, with the
// reference's formula (engine/core.cpp:407-605 per output): s_t = q.K_t/sqrt(128), softmax
// over t <= position, out = Σ p_t V_t.
//
// One CTA per (layer, KV head) stages K (transposed) and V of the first nk <= 128 positions
// in shared memory as FP32, once. Each warp then takes groups of four consecutive positions
// with both GQA query heads: eight query rows share every shared-memory read.
//   scores   lane l owns keys l, l+32, l+64, l+96 (a 32-key chunk is skipped by the whole
//            warp when it lies above the group's last position); the eight rows' query
//            values for one channel come as two broadcast float4 reads of the warp's Q
//            buffer ([channel][row]), so one K read feeds 8 FMAs.
//   softmax  per row over the warp (shuffle max and sum), probabilities written to the same
//            warp buffer as [key][row].
//   output   lane l owns channels 4l..4l+3: per key one float4 of V and two broadcast float4
//            of probabilities feed 32 FMAs. Rows go where OutRows says (local layout, or the
//            full-head layout here and on the peers).
// Both products run as packed FP32 FMAs over row pairs (fma.rn.f32x2, each lane rounded once,
// as fmaf), which halves the FMA instructions issued.
#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int THREADS = 512;
constexpr int WARPS = THREADS / 32;
constexpr int MAXK = 128;
constexpr int POS_PER_GROUP = 4;
constexpr int QR = POS_PER_GROUP * GROUP;      // query rows per warp pass (row r: position r/2, head r%2)
static_assert(QR == 8, "the row buffers are read as two float4 per channel or key");
constexpr size_t SMEM_BYTES = ((size_t)D * MAXK + (size_t)MAXK * D + (size_t)WARPS * QR * MAXK) * sizeof(float);

// Packed FP32 FMA (one instruction, two lanes, each rounded once like fmaf).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r, ua = *reinterpret_cast<unsigned long long*>(&a), ub = *reinterpret_cast<unsigned long long*>(&b),
                          uc = *reinterpret_cast<unsigned long long*>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(ua), "l"(ub), "l"(uc));
    return *reinterpret_cast<float2*>(&r);
}

// Scores of the warp's eight rows against keys lane + 32j, j < NJ; rows 2i and 2i+1 share
// one packed FMA per key.
template <int NJ>
__device__ __forceinline__ void score_rows(const float* __restrict__ KT, const float* __restrict__ wq, int lane,
                                           float (&acc)[4][QR]) {
    float2 a2[NJ][QR / 2];
    #pragma unroll
    for (int j = 0; j < NJ; ++j)
        #pragma unroll
        for (int i = 0; i < QR / 2; ++i) a2[j][i] = make_float2(0.f, 0.f);
    #pragma unroll 4
    for (int c = 0; c < D; ++c) {
        const float4 qa = *reinterpret_cast<const float4*>(wq + c * QR);
        const float4 qb = *reinterpret_cast<const float4*>(wq + c * QR + 4);
        const float2 q2[QR / 2] = {make_float2(qa.x, qa.y), make_float2(qa.z, qa.w), make_float2(qb.x, qb.y),
                                   make_float2(qb.z, qb.w)};
        #pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const float k = KT[c * MAXK + lane + 32 * j];
            const float2 kk = make_float2(k, k);
            #pragma unroll
            for (int i = 0; i < QR / 2; ++i) a2[j][i] = ffma2(q2[i], kk, a2[j][i]);
        }
    }
    #pragma unroll
    for (int j = 0; j < NJ; ++j)
        #pragma unroll
        for (int i = 0; i < QR / 2; ++i) { acc[j][2 * i] = a2[j][i].x; acc[j][2 * i + 1] = a2[j][i].y; }
}

__global__ void __launch_bounds__(THREADS, 1) attn_head_rows_kernel(const RowsArgs a, const OutRows o) {
    extern __shared__ __align__(16) float smem[];
    float* KT = smem;                                   // [128 channels][MAXK keys]
    float* Vs = KT + D * MAXK;                          // [MAXK keys][128 channels]
    float* wbuf = Vs + MAXK * D;                        // per warp: Q [128][QR], then P [MAXK][QR]
    const int l = blockIdx.x / a.hkv, kh = blockIdx.x % a.hkv;
    const int layer = a.layer0 + l;
    const int rows = a.row_end;                         // rows [0, rows), positions pos0.. < 128
    const int nk = a.pos0 + rows;                       // keys needed (<= 128)
    const int nk32 = (nk + 31) & ~31;
    const __half* Kp = a.kv.plane(a.seq, layer, 0, kh);
    const __half* Vp = a.kv.plane(a.seq, layer, 1, kh);
    // K transposed: consecutive threads take consecutive keys of one 8-channel group, so
    // the transposed shared-memory writes are conflict-free; keys [nk, nk32) read as zero
    for (int i = threadIdx.x; i < nk32 * (D / 8); i += THREADS) {
        const int c8 = (i / nk32) * 8, t = i % nk32;
        uint4 ku = make_uint4(0u, 0u, 0u, 0u);
        if (t < nk) ku = *reinterpret_cast<const uint4*>(Kp + (size_t)t * D + c8);
        const __half* k8 = reinterpret_cast<const __half*>(&ku);
        #pragma unroll
        for (int e = 0; e < 8; ++e) KT[(c8 + e) * MAXK + t] = __half2float(k8[e]);
    }
    // V row-major: consecutive threads take consecutive 8-channel groups of one key
    for (int i = threadIdx.x; i < nk * (D / 8); i += THREADS) {
        const int t = i / (D / 8), c8 = (i % (D / 8)) * 8;
        const uint4 vu = *reinterpret_cast<const uint4*>(Vp + (size_t)t * D + c8);
        const __half* v8 = reinterpret_cast<const __half*>(&vu);
        float4* dst = reinterpret_cast<float4*>(Vs + t * D + c8);
        dst[0] = make_float4(__half2float(v8[0]), __half2float(v8[1]), __half2float(v8[2]), __half2float(v8[3]));
        dst[1] = make_float4(__half2float(v8[4]), __half2float(v8[5]), __half2float(v8[6]), __half2float(v8[7]));
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* wq = wbuf + warp * QR * MAXK;
    const float scale = 1.4426950408889634f * 0.08838834764831845f;   // log2(e)/sqrt(128)
    const int groups = (rows + POS_PER_GROUP - 1) / POS_PER_GROUP;
    for (int grp = warp; grp < groups; grp += WARPS) {
        const int b0 = grp * POS_PER_GROUP;
        const int last = min(b0 + POS_PER_GROUP, rows) - 1;           // last valid row of the group
        const int pmax = a.pos0 + last;
        // query rows -> wq[c][r]; rows past the end of the call are zero and never stored
        #pragma unroll
        for (int i = 0; i < D / 32; ++i) {
            const int c = lane + 32 * i;
            float q[QR];
            #pragma unroll
            for (int r = 0; r < QR; ++r) {
                const int b = b0 + (r >> 1);
                q[r] = b < rows ? __ldg(a.q + (((size_t)l * a.n + b) * a.hq + kh * GROUP + (r & 1)) * D + c) : 0.f;
            }
            *reinterpret_cast<float4*>(wq + c * QR) = make_float4(q[0], q[1], q[2], q[3]);
            *reinterpret_cast<float4*>(wq + c * QR + 4) = make_float4(q[4], q[5], q[6], q[7]);
        }
        __syncwarp();
        float acc[4][QR];
        const int nj = pmax / 32 + 1;                   // 32-key chunks at or below the last position
        switch (nj) {
            case 1: score_rows<1>(KT, wq, lane, acc); break;
            case 2: score_rows<2>(KT, wq, lane, acc); break;
            case 3: score_rows<3>(KT, wq, lane, acc); break;
            default: score_rows<4>(KT, wq, lane, acc); break;
        }
        // softmax per row: key t = lane + 32j is visible to row r iff t <= its position
        float inv[QR];
        #pragma unroll
        for (int r = 0; r < QR; ++r) {
            const int pos = a.pos0 + min(b0 + (r >> 1), last);
            float m = -INFINITY;
            #pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool ok = j < nj && lane + 32 * j <= pos;
                acc[j][r] = ok ? acc[j][r] * scale : -INFINITY;
                m = fmaxf(m, acc[j][r]);
            }
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            float s = 0.f;
            #pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[j][r] = j < nj ? exp2f(acc[j][r] - m) : 0.f;
                s += acc[j][r];
            }
            #pragma unroll
            for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            inv[r] = 1.f / s;
        }
        __syncwarp();                                   // every lane is done reading wq
        float* wp = wq;                                 // probabilities [key][row]
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j < nj) {
                const int t = lane + 32 * j;
                *reinterpret_cast<float4*>(wp + t * QR) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
                *reinterpret_cast<float4*>(wp + t * QR + 4) = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
            }
        }
        __syncwarp();
        // acc_o[i][ch]: channel 4*lane + ch of rows 2i (.x) and 2i+1 (.y)
        float2 acc_o[QR / 2][4];
        #pragma unroll
        for (int i = 0; i < QR / 2; ++i)
            #pragma unroll
            for (int ch = 0; ch < 4; ++ch) acc_o[i][ch] = make_float2(0.f, 0.f);
        #pragma unroll 2
        for (int t = 0; t <= pmax; ++t) {
            const float4 pa = *reinterpret_cast<const float4*>(wp + t * QR);
            const float4 pb = *reinterpret_cast<const float4*>(wp + t * QR + 4);
            const float2 p2[QR / 2] = {make_float2(pa.x, pa.y), make_float2(pa.z, pa.w), make_float2(pb.x, pb.y),
                                       make_float2(pb.z, pb.w)};
            const float4 v = *reinterpret_cast<const float4*>(Vs + t * D + lane * 4);
            const float2 vv[4] = {make_float2(v.x, v.x), make_float2(v.y, v.y), make_float2(v.z, v.z),
                                  make_float2(v.w, v.w)};
            #pragma unroll
            for (int i = 0; i < QR / 2; ++i)
                #pragma unroll
                for (int ch = 0; ch < 4; ++ch) acc_o[i][ch] = ffma2(p2[i], vv[ch], acc_o[i][ch]);
        }
        #pragma unroll
        for (int r = 0; r < QR; ++r) {
            const int b = b0 + (r >> 1);
            if (b < rows) {
                const size_t off = (((size_t)l * a.n + b) * o.heads + o.head0 + kh * GROUP + (r & 1)) * D;
                const float2* orow = acc_o[r >> 1];
                const float4 val = (r & 1) ? make_float4(orow[0].y * inv[r], orow[1].y * inv[r], orow[2].y * inv[r],
                                                         orow[3].y * inv[r])
                                           : make_float4(orow[0].x * inv[r], orow[1].x * inv[r], orow[2].x * inv[r],
                                                         orow[3].x * inv[r]);
                reinterpret_cast<float4*>(o.out + off)[lane] = val;
                #pragma unroll
                for (int p = 0; p < MAX_RANKS - 1; ++p)
                    if (p < o.n_peers) reinterpret_cast<float4*>(o.peers[p] + off)[lane] = val;
            }
        }
        __syncwarp();                                   // wq / wp reuse by the next group
    }
    if (o.n_peers) {                                    // rows stored to peers: visible system-wide at exit
        __syncthreads();
        if (threadIdx.x == 0) __threadfence_system();
    }
}

}  // namespace

void launch_attn_head_rows(const RowsArgs& a, const OutRows& o, cudaStream_t s) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_head_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
        attr = true;
    }
    attn_head_rows_kernel<<<a.n_layers * a.hkv, THREADS, SMEM_BYTES, s>>>(a, o);
}

}  // namespace qattn
