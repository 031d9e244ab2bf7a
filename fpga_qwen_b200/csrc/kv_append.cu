// kv_append.cu — fused QK-RMSNorm + RoPE + FP16 KV write.
//
// Reference arithmetic (tampajohn/fpga-qwen engine/core.cpp), reproduced bit for bit:
//   norm  :207-215  square = x*x (FP32); sum = Σ double(square) in ascending j (FP64);
//                   inv = 1 / sqrt(float(sum)/128 + 1e-6); out = (x*inv)*w
//   rope  :216-218  x[j] = a*c - b*s; x[j+64] = b*c + a*s  (unfused products)
//   store :399-405  K, V -> FP16 round-to-nearest-even at (layer, pos+b, head)
// Every rounding step is written with an explicit _rn intrinsic so that no compiler
// contraction can change a result.
//
// Layout: one "row" is one head vector of 128 FP32 values. Per token there are hq query
// rows, hkv key rows and hkv value rows. A block of ROWS threads owns ROWS consecutive
// rows: it stages them in shared memory with coalesced 16-byte loads (one warp reads one
// 512-byte row), then each thread runs the sequential FP64 sum of its own row (the order
// the reference fixes), normalises and rotates in place, and the block writes back with
// coalesced stores: FP32 query rows to q_out, FP16 K/V rows into the HBM KV store.
// The kernel is HBM-bound: 28,672 algorithmic bytes per (token, layer) at hq=16, hkv=8.
#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int ROWS = 64;          // rows (threads) per block
constexpr int STRIDE = 132;       // padded row stride in floats: conflict-free float4 access

__global__ void __launch_bounds__(ROWS) kv_append_kernel(const AppendArgs a) {
    __shared__ __align__(16) float tile[ROWS * STRIDE];
    const int R = a.hq + 2 * a.hkv;                       // rows per token
    const int per_layer = a.n * R;                        // <= 4096 * 32
    const int total = per_layer * a.n_layers;             // <= 28 * 4096 * 32 < 2^31
    const int g0 = blockIdx.x * ROWS;

    auto src_row = [&](int g, int& kind, int& l, int& b, int& head) -> const float* {
        l = (unsigned)g / (unsigned)per_layer;
        const int rem = g - l * per_layer;
        b = (unsigned)rem / (unsigned)R;
        const int r = rem - b * R;
        const size_t tok = (size_t)l * a.n + b;
        if (r < a.hq) { kind = 0; head = r; return a.q_pre + (tok * a.hq + head) * D; }
        if (r < a.hq + a.hkv) { kind = 1; head = r - a.hq; return a.k_pre + (tok * a.hkv + head) * D; }
        kind = 2; head = r - a.hq - a.hkv; return a.v_pre + (tok * a.hkv + head) * D;
    };

    // ---- stage: warp w reads rows w, w+warps, ... ; lane c reads 16-byte chunk c ----
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int WARPS = ROWS / 32;
    float4 staged[ROWS / WARPS];
    #pragma unroll
    for (int i = 0; i < ROWS / WARPS; ++i) {
        const int g = g0 + warp + i * WARPS;
        if (g < total) {
            int kind, l, b, head;
            const float* src = src_row(g, kind, l, b, head);
            staged[i] = __ldg(reinterpret_cast<const float4*>(src) + lane);
        }
    }
    #pragma unroll
    for (int i = 0; i < ROWS / WARPS; ++i) {
        const int row = warp + i * WARPS;
        if (g0 + row < total) *reinterpret_cast<float4*>(&tile[row * STRIDE + lane * 4]) = staged[i];
    }
    __syncthreads();

    // ---- per-row arithmetic: thread t owns row t ----
    const int g = g0 + threadIdx.x;
    if (g < total) {
        int kind, l, b, head;
        (void)src_row(g, kind, l, b, head);
        if (kind < 2) {
            float* x = &tile[threadIdx.x * STRIDE];
            double precise_sum = 0.0;
            #pragma unroll 4
            for (int j = 0; j < D; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(x + j);
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.x, v.x));
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.y, v.y));
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.z, v.z));
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.w, v.w));
            }
            const float sum = __double2float_rn(precise_sum);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), a.eps)));
            const float* w = a.norms + ((size_t)(a.layer0 + l) * 2 + kind) * D;
            const int pos = a.pos0 + b;
            const float* cs = a.cosines + (size_t)pos * 64;
            const float* sn = a.sines + (size_t)pos * 64;
            #pragma unroll 2
            for (int j = 0; j < 64; j += 4) {
                const float4 xa = *reinterpret_cast<const float4*>(x + j);
                const float4 xb = *reinterpret_cast<const float4*>(x + j + 64);
                const float4 wa = __ldg(reinterpret_cast<const float4*>(w + j));
                const float4 wb = __ldg(reinterpret_cast<const float4*>(w + j + 64));
                const float4 c = __ldg(reinterpret_cast<const float4*>(cs + j));
                const float4 s = __ldg(reinterpret_cast<const float4*>(sn + j));
                float na[4] = {__fmul_rn(__fmul_rn(xa.x, inv), wa.x), __fmul_rn(__fmul_rn(xa.y, inv), wa.y),
                               __fmul_rn(__fmul_rn(xa.z, inv), wa.z), __fmul_rn(__fmul_rn(xa.w, inv), wa.w)};
                float nb[4] = {__fmul_rn(__fmul_rn(xb.x, inv), wb.x), __fmul_rn(__fmul_rn(xb.y, inv), wb.y),
                               __fmul_rn(__fmul_rn(xb.z, inv), wb.z), __fmul_rn(__fmul_rn(xb.w, inv), wb.w)};
                const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
                float ra[4], rb[4];
                #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    ra[e] = __fsub_rn(__fmul_rn(na[e], cc[e]), __fmul_rn(nb[e], ss[e]));
                    rb[e] = __fadd_rn(__fmul_rn(nb[e], cc[e]), __fmul_rn(na[e], ss[e]));
                }
                *reinterpret_cast<float4*>(x + j) = make_float4(ra[0], ra[1], ra[2], ra[3]);
                *reinterpret_cast<float4*>(x + j + 64) = make_float4(rb[0], rb[1], rb[2], rb[3]);
            }
        }
    }
    __syncthreads();

    // ---- write back: query rows as FP32 (32 chunks), K/V rows as FP16 (16 chunks) ----
    for (int row = warp; row < ROWS; row += WARPS) {
        const int gr = g0 + row;
        if (gr >= total) break;
        int kind, l, b, head;
        (void)src_row(gr, kind, l, b, head);
        const float* x = &tile[row * STRIDE];
        if (kind == 0) {
            float* dst = a.q_out + (((size_t)l * a.n + b) * a.hq + head) * D;
            reinterpret_cast<float4*>(dst)[lane] = *reinterpret_cast<const float4*>(x + lane * 4);
        } else if (lane < 16) {
            const float4 lo = *reinterpret_cast<const float4*>(x + lane * 8);
            const float4 hi = *reinterpret_cast<const float4*>(x + lane * 8 + 4);
            __half2 h0 = __floats2half2_rn(lo.x, lo.y), h1 = __floats2half2_rn(lo.z, lo.w);
            __half2 h2 = __floats2half2_rn(hi.x, hi.y), h3 = __floats2half2_rn(hi.z, hi.w);
            uint4 packed;
            packed.x = *reinterpret_cast<uint32_t*>(&h0); packed.y = *reinterpret_cast<uint32_t*>(&h1);
            packed.z = *reinterpret_cast<uint32_t*>(&h2); packed.w = *reinterpret_cast<uint32_t*>(&h3);
            __half* dst = a.kv.plane(a.seq, a.layer0 + l, kind - 1, head) + (size_t)(a.pos0 + b) * D;
            reinterpret_cast<uint4*>(dst)[lane] = packed;
        }
    }
}

}  // namespace

void launch_kv_append(const AppendArgs& a, cudaStream_t s) {
    const int total = a.n_layers * a.n * (a.hq + 2 * a.hkv);
    const unsigned blocks = (unsigned)((total + ROWS - 1) / ROWS);
    kv_append_kernel<<<blocks, ROWS, 0, s>>>(a);
}

}  // namespace qattn
