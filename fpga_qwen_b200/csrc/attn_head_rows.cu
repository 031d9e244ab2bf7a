// attn_head_rows.cu — FP32 causal attention for the first rows of a sequence.
//
// Prefill rows at absolute position < 128 attend to at most 128 keys, and their attention
// is concentrated on few keys; there FP16 probabilities (tensor-core path) would exceed the
// 1e-3 output tolerance, so these rows are computed in FP32 on CUDA cores, with the
// reference's formula (engine/core.cpp:407-605 per output): s_t = q.K_t/sqrt(128), softmax
// over t <= position, out = Σ p_t V_t.
//
// One CTA per (layer, KV head): it stages K (transposed, FP32) and V (FP32) of the first
// nk <= 128 positions in shared memory once, then each warp takes rows in turn, both GQA
// query heads at once: lane l scores keys 4l..4l+3 (one 16-byte read of the transposed K
// feeds 8 FMAs), the warp forms both softmaxes with shuffle reductions, and lane l
// accumulates output channels 4l..4l+3 of both heads.
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
    float* qbuf = Vs + MAXK * D;                        // [warps][GROUP][128]
    float* pbuf = qbuf + (THREADS / 32) * GROUP * D;    // [warps][GROUP][MAXK]
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
    float* qw = qbuf + warp * GROUP * D;                // both query heads of the row
    float* pw = pbuf + warp * GROUP * MAXK;
    const float scale = 1.4426950408889634f * 0.08838834764831845f;   // log2(e)/sqrt(128)
    // one warp per row, both GQA heads at once; lane l scores keys 4l..4l+3 and accumulates
    // output channels 4l..4l+3
    for (int b = warp; b < rows; b += THREADS / 32) {
        const int pos = a.pos0 + b;
        const size_t row0 = ((size_t)l * a.n + b) * a.hq + (size_t)kh * GROUP;
        #pragma unroll
        for (int g = 0; g < GROUP; ++g)
            *reinterpret_cast<float4*>(qw + g * D + lane * 4) =
                __ldg(reinterpret_cast<const float4*>(a.q + (row0 + g) * D) + lane);
        __syncwarp();
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
        #pragma unroll 2
        for (int c = 0; c < D; c += 4) {
            const float4 qa = *reinterpret_cast<const float4*>(qw + c);
            const float4 qb = *reinterpret_cast<const float4*>(qw + D + c);
            const float q0[4] = {qa.x, qa.y, qa.z, qa.w}, q1[4] = {qb.x, qb.y, qb.z, qb.w};
            #pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const float4 k = *reinterpret_cast<const float4*>(KT + (c + cc) * KT_STRIDE + lane * 4);
                s0[0] = fmaf(q0[cc], k.x, s0[0]); s0[1] = fmaf(q0[cc], k.y, s0[1]);
                s0[2] = fmaf(q0[cc], k.z, s0[2]); s0[3] = fmaf(q0[cc], k.w, s0[3]);
                s1[0] = fmaf(q1[cc], k.x, s1[0]); s1[1] = fmaf(q1[cc], k.y, s1[1]);
                s1[2] = fmaf(q1[cc], k.z, s1[2]); s1[3] = fmaf(q1[cc], k.w, s1[3]);
            }
        }
        float m0 = -INFINITY, m1 = -INFINITY;
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool ok = lane * 4 + i <= pos;
            s0[i] = ok ? s0[i] * scale : -INFINITY;
            s1[i] = ok ? s1[i] * scale : -INFINITY;
            m0 = fmaxf(m0, s0[i]); m1 = fmaxf(m1, s1[i]);
        }
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
            m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
        }
        float p0[4], p1[4], l0 = 0.f, l1 = 0.f;
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            p0[i] = exp2f(s0[i] - m0); p1[i] = exp2f(s1[i] - m1);
            l0 += p0[i]; l1 += p1[i];
        }
        *reinterpret_cast<float4*>(pw + lane * 4) = make_float4(p0[0], p0[1], p0[2], p0[3]);
        *reinterpret_cast<float4*>(pw + MAXK + lane * 4) = make_float4(p1[0], p1[1], p1[2], p1[3]);
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, off);
            l1 += __shfl_xor_sync(0xffffffffu, l1, off);
        }
        __syncwarp();
        float4 o0 = make_float4(0.f, 0.f, 0.f, 0.f), o1 = o0;
        for (int t = 0; t <= pos; ++t) {
            const float pa = pw[t], pb = pw[MAXK + t];
            const float4 v = *reinterpret_cast<const float4*>(Vs + t * D + lane * 4);
            o0.x = fmaf(pa, v.x, o0.x); o0.y = fmaf(pa, v.y, o0.y); o0.z = fmaf(pa, v.z, o0.z); o0.w = fmaf(pa, v.w, o0.w);
            o1.x = fmaf(pb, v.x, o1.x); o1.y = fmaf(pb, v.y, o1.y); o1.z = fmaf(pb, v.z, o1.z); o1.w = fmaf(pb, v.w, o1.w);
        }
        const float i0 = 1.f / l0, i1 = 1.f / l1;
        reinterpret_cast<float4*>(a.out + row0 * D)[lane] = make_float4(o0.x * i0, o0.y * i0, o0.z * i0, o0.w * i0);
        reinterpret_cast<float4*>(a.out + (row0 + 1) * D)[lane] = make_float4(o1.x * i1, o1.y * i1, o1.z * i1, o1.w * i1);
        __syncwarp();                                   // qw / pw reuse by the next row
    }
}

}  // namespace

void launch_attn_head_rows(const RowsArgs& a, cudaStream_t s) {
    const size_t smem = ((size_t)D * KT_STRIDE + (size_t)MAXK * D + (THREADS / 32) * GROUP * (D + MAXK)) *
                        sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_head_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    attn_head_rows_kernel<<<a.n_layers * a.hkv, THREADS, smem, s>>>(a);
}

}  // namespace qattn
