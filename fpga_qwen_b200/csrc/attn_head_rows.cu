// attn_head_rows.cu — FP32 causal attention for the first rows of a sequence.
//
// Prefill rows at absolute position < 128 attend to at most 128 keys, and their attention
// is concentrated on few keys; there FP16 probabilities (tensor-core path) would exceed the
// 1e-3 output tolerance, so these rows are computed in FP32 on CUDA cores, with the
// reference's formula (engine/core.cpp:407-605 per output): s_t = q.K_t/sqrt(128), softmax
// over t <= position, out = Σ p_t V_t.
//
// One CTA per (layer, KV head): it stages K (transposed, FP32) and V (FP32) of the first
// nk <= 128 positions in shared memory once, then each warp takes query vectors (row, GQA
// head) in turn: lane l scores keys l, l+32, l+64, l+96 against the query (broadcast from
// shared memory), the warp forms the softmax with shuffle reductions, and lane l
// accumulates output channels 4l..4l+3.
#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int THREADS = 256;
constexpr int MAXK = 128;
constexpr int KT_STRIDE = MAXK + 4;    // transposed K rows: [channel][key]

__global__ void __launch_bounds__(THREADS, 1) attn_head_rows_kernel(const RowsArgs a) {
    extern __shared__ __align__(16) float smem[];
    float* KT = smem;                                   // [128 channels][KT_STRIDE]
    float* Vs = KT + D * KT_STRIDE;                     // [MAXK][128]
    float* qbuf = Vs + MAXK * D;                        // [warps][128]
    float* pbuf = qbuf + (THREADS / 32) * D;            // [warps][MAXK]
    const int l = blockIdx.x / a.hkv, kh = blockIdx.x % a.hkv;
    const int layer = a.layer0 + l;
    const int rows = a.row_end;                         // rows [0, rows), positions pos0.. < 128
    const int nk = a.pos0 + rows;                       // keys needed (<= 128)
    const __half* Kp = a.kv.plane(a.seq, layer, 0, kh);
    const __half* Vp = a.kv.plane(a.seq, layer, 1, kh);
    // K transposed: consecutive threads take consecutive keys of one 8-channel group, so
    // the transposed shared-memory writes are conflict-free
    for (int i = threadIdx.x; i < nk * (D / 8); i += THREADS) {
        const int c8 = (i / nk) * 8, t = i % nk;
        const uint4 ku = *reinterpret_cast<const uint4*>(Kp + (size_t)t * D + c8);
        const __half* k8 = reinterpret_cast<const __half*>(&ku);
        #pragma unroll
        for (int e = 0; e < 8; ++e) KT[(c8 + e) * KT_STRIDE + t] = __half2float(k8[e]);
    }
    // V row-major: consecutive threads take consecutive 8-channel groups of one key
    for (int i = threadIdx.x; i < nk * (D / 8); i += THREADS) {
        const int t = i / (D / 8), c8 = (i % (D / 8)) * 8;
        const uint4 vu = *reinterpret_cast<const uint4*>(Vp + (size_t)t * D + c8);
        const __half* v8 = reinterpret_cast<const __half*>(&vu);
        #pragma unroll
        for (int e = 0; e < 8; ++e) Vs[t * D + c8 + e] = __half2float(v8[e]);
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* qw = qbuf + warp * D;
    float* pw = pbuf + warp * MAXK;
    const float scale = 1.4426950408889634f * 0.08838834764831845f;   // log2(e)/sqrt(128)
    for (int vec = warp; vec < rows * GROUP; vec += THREADS / 32) {
        const int b = vec / GROUP, g = vec % GROUP;
        const int pos = a.pos0 + b;
        const size_t row = ((size_t)l * a.n + b) * a.hq + (size_t)kh * GROUP + g;
        *reinterpret_cast<float4*>(qw + lane * 4) = __ldg(reinterpret_cast<const float4*>(a.q + row * D) + lane);
        __syncwarp();
        float s[MAXK / 32];
        #pragma unroll
        for (int i = 0; i < MAXK / 32; ++i) s[i] = 0.f;
        #pragma unroll 8
        for (int c = 0; c < D; ++c) {
            const float qc = qw[c];
            #pragma unroll
            for (int i = 0; i < MAXK / 32; ++i) s[i] = fmaf(qc, KT[c * KT_STRIDE + lane + 32 * i], s[i]);
        }
        float m = -INFINITY;
        #pragma unroll
        for (int i = 0; i < MAXK / 32; ++i) {
            s[i] = (lane + 32 * i <= pos) ? s[i] * scale : -INFINITY;
            m = fmaxf(m, s[i]);
        }
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float lsum = 0.f;
        #pragma unroll
        for (int i = 0; i < MAXK / 32; ++i) {
            const float p = exp2f(s[i] - m);
            pw[lane + 32 * i] = p;
            lsum += p;
        }
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
        __syncwarp();
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int t = 0; t <= pos; ++t) {
            const float p = pw[t];
            const float4 v = *reinterpret_cast<const float4*>(Vs + t * D + lane * 4);
            o.x = fmaf(p, v.x, o.x); o.y = fmaf(p, v.y, o.y); o.z = fmaf(p, v.z, o.z); o.w = fmaf(p, v.w, o.w);
        }
        const float inv = 1.f / lsum;
        reinterpret_cast<float4*>(a.out + row * D)[lane] = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
        __syncwarp();                                   // qw / pw reuse by the next vector
    }
}

}  // namespace

void launch_attn_head_rows(const RowsArgs& a, cudaStream_t s) {
    const size_t smem = ((size_t)D * KT_STRIDE + (size_t)MAXK * D + (THREADS / 32) * D + (THREADS / 32) * MAXK) *
                        sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_head_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    attn_head_rows_kernel<<<a.n_layers * a.hkv, THREADS, smem, s>>>(a);
}

}  // namespace qattn
