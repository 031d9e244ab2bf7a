// attn_rows.cu — split-context (flash-decoding) causal GQA attention on CUDA cores.
//
// Used for single-token decode (reference engine/core.cpp:606-624), the two-row B2 verify
// attention (:671-689), and the rows of a prefill whose absolute position is below one
// tensor-core tile, where FP32 accuracy is needed because attention is concentrated on a
// few keys. The math per output row is the reference's: s_t = q.K_t / sqrt(128),
// p_t = exp(s_t - max) / Σ exp(s_t - max), out = Σ p_t V_t — evaluated here in the
// base-2 domain with the query pre-scaled by log2(e)/sqrt(128), and in FP32 throughout.
//
// Work decomposition. One CTA = (layer, row, KV head, split). Both query heads of the GQA
// pair share every K and V load (the GPU analogue of the reference's head pairing,
// core.cpp:150-159). A half-warp owns one 256-byte key row per step, each lane holding
// 8 channels (16-byte vector loads); partial dot products meet by shuffle reduction.
// Scores of the split live in shared memory, so the split's max and sum are exact over
// its keys; the PV pass re-reads V once. With splits > 1, each CTA writes (m, l, acc) to
// a scratch record and the last CTA of the (layer, row, head) unit to finish — found
// with one atomic counter, no waiting — merges the records and writes the output.
#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int THREADS = 128;
constexpr int HALF_WARPS = THREADS / 16;   // 8 key rows in flight per step
constexpr int UNROLL = 4;                  // key rows per half-warp per step (transpose-reduce needs 4)
static_assert(UNROLL * GROUP == 8, "transpose-reduce is written for 8 values per lane");

__device__ __forceinline__ void unpack8(const uint4 u, float f[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    #pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
}

__global__ void __launch_bounds__(THREADS) attn_rows_kernel(const RowsArgs a) {
    extern __shared__ __align__(16) float smem[];
    float* scores = smem;                                   // [GROUP][keys_per_split]
    __shared__ float red[GROUP][THREADS / 32];
    __shared__ float stat[2 * GROUP];                       // m[GROUP], l[GROUP]
    __shared__ float accbuf[HALF_WARPS][GROUP][D];
    __shared__ int is_last;

    // blockIdx.x -> (unit, split); units ordered (layer, row desc, head) so long rows start first
    const int splits = a.splits;
    const int split = blockIdx.x % splits;
    const int unit = blockIdx.x / splits;
    const int kh = unit % a.hkv;
    const int lr = unit / a.hkv;
    const int rows = a.row_end - a.row_begin;
    const int l = lr / rows;
    const int b = a.row_end - 1 - (lr - l * rows);
    const int ctx_len = a.pos0 + b + 1;
    const int k0 = split * a.keys_per_split;
    const int k1 = min(ctx_len, k0 + a.keys_per_split);
    const int cnt = max(0, k1 - k0);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hw = tid >> 4, sl = tid & 15;
    const int layer = a.layer0 + l;
    const __half* Kp = a.kv.plane(a.seq, layer, 0, kh);
    const __half* Vp = a.kv.plane(a.seq, layer, 1, kh);
    const size_t qrow = ((size_t)l * a.n + b) * a.hq + (size_t)kh * GROUP;
    const float qscale = 1.4426950408889634f * 0.08838834764831845f;   // log2(e) / sqrt(128)

    float q[GROUP][8];
    #pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        const float4* src = reinterpret_cast<const float4*>(a.q + (qrow + g) * D + sl * 8);
        const float4 u = __ldg(src), v = __ldg(src + 1);
        q[g][0] = u.x * qscale; q[g][1] = u.y * qscale; q[g][2] = u.z * qscale; q[g][3] = u.w * qscale;
        q[g][4] = v.x * qscale; q[g][5] = v.y * qscale; q[g][6] = v.z * qscale; q[g][7] = v.w * qscale;
    }

    // ---- pass 1: scores (log2 domain) into shared memory, running max per head ----
    float mloc[GROUP];
    #pragma unroll
    for (int g = 0; g < GROUP; ++g) mloc[g] = -INFINITY;
    // The loop bound is warp-uniform (both half-warps of a warp run the same iterations):
    // the shuffles below use the full mask. Keys past cnt load as zero and are not stored.
    const int warp_first = hw & ~1;
    for (int it = warp_first; it < cnt; it += HALF_WARPS * UNROLL) {
        const int base = it + (hw & 1);
        uint4 kr[UNROLL];
        #pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int t = base + u * HALF_WARPS;
            if (t < cnt) kr[u] = __ldg(reinterpret_cast<const uint4*>(Kp + (size_t)(k0 + t) * D) + sl);
            else kr[u] = make_uint4(0, 0, 0, 0);
        }
        // partial dot products: value i = u * GROUP + g (key u of this step, query head g)
        float v[UNROLL * GROUP];
        #pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            float kf[8]; unpack8(kr[u], kf);
            #pragma unroll
            for (int g = 0; g < GROUP; ++g) {
                float acc = 0.f;
                #pragma unroll
                for (int e = 0; e < 8; ++e) acc = fmaf(q[g][e], kf[e], acc);
                v[u * GROUP + g] = acc;
            }
        }
        // transpose-reduce over the 16 lanes of the half-warp: each exchange halves the
        // number of values a lane carries (4 + 2 + 1 + 1 shuffles for 8 sums instead of 32)
        const bool b3 = sl & 8, b2 = sl & 4, b1 = sl & 2;
        float w4[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float send = b3 ? v[i] : v[i + 4];
            const float keep = b3 ? v[i + 4] : v[i];
            w4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        float w2[2];
        #pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float send = b2 ? w4[i] : w4[i + 2];
            const float keep = b2 ? w4[i + 2] : w4[i];
            w2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        float y;
        {
            const float send = b1 ? w2[0] : w2[1];
            const float keep = b1 ? w2[1] : w2[0];
            y = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        // this lane now holds key my_u, head my_g
        const int my_u = (b3 ? 2 : 0) + (b2 ? 1 : 0), my_g = b1 ? 1 : 0;
        const int t = base + my_u * HALF_WARPS;
        if (t < cnt) {
            if (my_g == 0) mloc[0] = fmaxf(mloc[0], y); else mloc[1] = fmaxf(mloc[1], y);
            if ((sl & 1) == 0) scores[my_g * a.keys_per_split + t] = y;
        }
    }
    // block max per head
    #pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        float m = mloc[g];
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (lane == 0) red[g][warp] = m;
    }
    __syncthreads();
    if (tid < GROUP) {
        float m = red[tid][0];
        #pragma unroll
        for (int w = 1; w < THREADS / 32; ++w) m = fmaxf(m, red[tid][w]);
        stat[tid] = m;
    }
    __syncthreads();

    // ---- softmax numerators and sums ----
    float lsum[GROUP];
    #pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        const float m = stat[g];
        float acc = 0.f;
        for (int t = tid; t < cnt; t += THREADS) {
            const float p = exp2f(scores[g * a.keys_per_split + t] - m);
            scores[g * a.keys_per_split + t] = p;
            acc += p;
        }
        lsum[g] = acc;
    }
    #pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        float v = lsum[g];
        #pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[g][warp] = v;
    }
    __syncthreads();
    if (tid < GROUP) {
        float v = 0.f;
        #pragma unroll
        for (int w = 0; w < THREADS / 32; ++w) v += red[tid][w];
        stat[GROUP + tid] = v;
    }

    // ---- pass 2: PV over the split's keys ----
    float acc[GROUP][8];
    #pragma unroll
    for (int g = 0; g < GROUP; ++g)
        #pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
    for (int it = warp_first; it < cnt; it += HALF_WARPS * UNROLL) {
        const int base = it + (hw & 1);
        uint4 vr[UNROLL];
        #pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int t = base + u * HALF_WARPS;
            if (t < cnt) vr[u] = __ldg(reinterpret_cast<const uint4*>(Vp + (size_t)(k0 + t) * D) + sl);
            else vr[u] = make_uint4(0, 0, 0, 0);
        }
        #pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int t = base + u * HALF_WARPS;
            if (t < cnt) {
                float vf[8]; unpack8(vr[u], vf);
                #pragma unroll
                for (int g = 0; g < GROUP; ++g) {
                    const float p = scores[g * a.keys_per_split + t];
                    #pragma unroll
                    for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vf[e], acc[g][e]);
                }
            }
        }
    }
    #pragma unroll
    for (int g = 0; g < GROUP; ++g)
        #pragma unroll
        for (int e = 0; e < 8; ++e) accbuf[hw][g][sl * 8 + e] = acc[g][e];
    __syncthreads();

    // reduce the 8 half-warps: thread t owns outputs (g, j) = (t / 64 ... ) over GROUP*D = 256
    float o[GROUP * D / THREADS];
    #pragma unroll
    for (int i = 0; i < GROUP * D / THREADS; ++i) {
        const int idx = tid + i * THREADS, g = idx / D, j = idx % D;
        float v = 0.f;
        #pragma unroll
        for (int h = 0; h < HALF_WARPS; ++h) v += accbuf[h][g][j];
        o[i] = v;
    }

    if (splits == 1) {
        #pragma unroll
        for (int i = 0; i < GROUP * D / THREADS; ++i) {
            const int idx = tid + i * THREADS, g = idx / D, j = idx % D;
            a.out[(qrow + g) * D + j] = o[i] / stat[GROUP + g];
        }
        return;
    }

    // ---- split > 1: publish this split's record, the last CTA of the unit merges ----
    float* rec = a.partial + ((size_t)unit * splits + split) * PARTIAL_FLOATS;
    if (tid < 2 * GROUP) rec[tid] = stat[tid];
    #pragma unroll
    for (int i = 0; i < GROUP * D / THREADS; ++i) rec[4 + tid + i * THREADS] = o[i];
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int done = atomicAdd(&a.counters[unit], 1);
        is_last = (done == splits - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();

    const float* recs = a.partial + (size_t)unit * splits * PARTIAL_FLOATS;
    float mall[GROUP], lall[GROUP];
    #pragma unroll
    for (int g = 0; g < GROUP; ++g) {
        float m = -INFINITY;
        for (int s = 0; s < splits; ++s) m = fmaxf(m, __ldcg(recs + (size_t)s * PARTIAL_FLOATS + g));
        mall[g] = m;
        float lv = 0.f;
        for (int s = 0; s < splits; ++s) {
            const float ms = __ldcg(recs + (size_t)s * PARTIAL_FLOATS + g);
            lv += (ms == -INFINITY) ? 0.f : exp2f(ms - m) * __ldcg(recs + (size_t)s * PARTIAL_FLOATS + GROUP + g);
        }
        lall[g] = lv;
    }
    #pragma unroll
    for (int i = 0; i < GROUP * D / THREADS; ++i) {
        const int idx = tid + i * THREADS, g = idx / D, j = idx % D;
        float v = 0.f;
        for (int s = 0; s < splits; ++s) {
            const float ms = __ldcg(recs + (size_t)s * PARTIAL_FLOATS + g);
            if (ms != -INFINITY) v += exp2f(ms - mall[g]) * __ldcg(recs + (size_t)s * PARTIAL_FLOATS + 4 + idx);
        }
        a.out[(qrow + g) * D + j] = v / lall[g];
    }
    if (tid == 0) a.counters[unit] = 0;      // ready for the next call on this stream
}

}  // namespace

void launch_attn_rows(const RowsArgs& a, cudaStream_t s) {
    const int rows = a.row_end - a.row_begin;
    const long long units = (long long)a.n_layers * rows * a.hkv;
    const unsigned blocks = (unsigned)(units * a.splits);
    const size_t smem = (size_t)GROUP * a.keys_per_split * sizeof(float);
    attn_rows_kernel<<<blocks, THREADS, smem, s>>>(a);
}

cudaError_t prepare_attn_rows() {
    cudaFuncAttributes attr{};
    return cudaFuncGetAttributes(&attr, attn_rows_kernel);     // loads the kernel's module now
}

}  // namespace qattn
