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
// rows, hkv key rows and hkv value rows. A block owns TPB consecutive tokens of one layer,
// one thread per row. It stages the rows in shared memory with 16-byte cp.async copies (no
// registers held, all copies in flight at once), together with the RoPE cos/sin rows and
// the layer's q_norm/k_norm weights, so the per-row arithmetic reads only shared memory.
// Each thread then runs the reference's sequential FP64 sum of squares for its own row
// (the squares and their FP64 conversions are independent; only the 128 additions form a
// chain), normalises and rotates in place. The block writes back with coalesced stores:
// FP32 query rows to q_out, FP16 K/V rows into the HBM KV store.
// HBM-bound: 28,672 algorithmic bytes per (token, layer) at hq=16, hkv=8.
#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr int STRIDE = 132;       // padded row stride in floats: conflict-free float4 access
constexpr int SLOT = 384;         // staged floats per token: cos[64] sin[64] q_norm[128] k_norm[128]

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// One block = TPB consecutive tokens of one layer; R = 4*HKV rows per token (2*HKV query
// rows, HKV key rows, HKV value rows); one thread per row. HKV is a template parameter so
// every row/token index below divides by a constant.
template <int HKV, int TPB>
__global__ void __launch_bounds__(TPB * 4 * HKV) kv_append_kernel(const AppendArgs a) {
    constexpr int HQ = GROUP * HKV, R = HQ + 2 * HKV, ROWS = TPB * R, WARPS = (ROWS + 31) / 32;
    extern __shared__ __align__(16) float smem[];
    float* tile = smem;                                   // [ROWS][STRIDE]
    float* slots = smem + ROWS * STRIDE;                  // [TPB][SLOT]
    const int l = blockIdx.y;
    const int b0 = blockIdx.x * TPB;
    const int ntok = min(TPB, a.n - b0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t tok_base = (size_t)l * a.n + b0;

    // ---- stage rows: warp w copies rows w, w+WARPS, ...; lane c copies 16-byte chunk c ----
    for (int row = warp; row < ntok * R; row += WARPS) {
        const int tb = row / R, r = row - tb * R;
        const size_t tok = tok_base + tb;
        const float* src = r < HQ ? a.q_pre + (tok * HQ + r) * D
                         : r < HQ + HKV ? a.k_pre + (tok * HKV + (r - HQ)) * D
                                        : a.v_pre + (tok * HKV + (r - HQ - HKV)) * D;
        cp_async16(&tile[row * STRIDE + lane * 4], src + lane * 4);
    }
    // ---- stage per-token tables: cos, sin of the position; q_norm, k_norm of the layer ----
    for (int i = threadIdx.x; i < ntok * (SLOT / 4); i += ROWS) {
        const int tb = i / (SLOT / 4), c = i - tb * (SLOT / 4);   // 96 chunks of 16 bytes per token
        const int pos = a.rows.pos_of(b0 + tb, a.pos0);
        const float* src = c < 16 ? a.cosines + (size_t)pos * 64 + c * 4
                         : c < 32 ? a.sines + (size_t)pos * 64 + (c - 16) * 4
                                  : a.norms + (size_t)(a.layer0 + l) * 2 * D + (c - 32) * 4;
        cp_async16(&slots[tb * SLOT + c * 4], src);
    }
    cp_async_wait_all();
    __syncthreads();

    // ---- per-row arithmetic: thread t owns row t ----
    {
        const int row = threadIdx.x;
        const int tb = row / R, r = row - tb * R;
        const int kind = r < HQ ? 0 : (r < HQ + HKV ? 1 : 2);
        if (tb < ntok && kind < 2) {
            float* x = &tile[row * STRIDE];
            const float* slot = &slots[tb * SLOT];
            const float* cs = slot;
            const float* sn = slot + 64;
            const float* w = slot + 128 + kind * D;
            // FP32 squares and their FP64 values are independent; only the adds chain
            double precise_sum = 0.0;
            #pragma unroll 8
            for (int j = 0; j < D; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(x + j);
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.x, v.x));
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.y, v.y));
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.z, v.z));
                precise_sum = __dadd_rn(precise_sum, (double)__fmul_rn(v.w, v.w));
            }
            const float sum = __double2float_rn(precise_sum);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), a.eps)));
            #pragma unroll 4
            for (int j = 0; j < 64; j += 4) {
                const float4 xa = *reinterpret_cast<const float4*>(x + j);
                const float4 xb = *reinterpret_cast<const float4*>(x + j + 64);
                const float4 wa = *reinterpret_cast<const float4*>(w + j);
                const float4 wb = *reinterpret_cast<const float4*>(w + j + 64);
                const float4 c = *reinterpret_cast<const float4*>(cs + j);
                const float4 s = *reinterpret_cast<const float4*>(sn + j);
                const float na[4] = {__fmul_rn(__fmul_rn(xa.x, inv), wa.x), __fmul_rn(__fmul_rn(xa.y, inv), wa.y),
                                     __fmul_rn(__fmul_rn(xa.z, inv), wa.z), __fmul_rn(__fmul_rn(xa.w, inv), wa.w)};
                const float nb[4] = {__fmul_rn(__fmul_rn(xb.x, inv), wb.x), __fmul_rn(__fmul_rn(xb.y, inv), wb.y),
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
    for (int row = warp; row < ntok * R; row += WARPS) {
        const int tb = row / R, r = row - tb * R;
        const float* x = &tile[row * STRIDE];
        if (r < HQ) {
            float* dst = a.q_out + ((tok_base + tb) * HQ + r) * D;
            reinterpret_cast<float4*>(dst)[lane] = *reinterpret_cast<const float4*>(x + lane * 4);
        } else if (lane < 16) {
            const int kind = r < HQ + HKV ? 1 : 2;
            const int head = kind == 1 ? r - HQ : r - HQ - HKV;
            const float4 lo = *reinterpret_cast<const float4*>(x + lane * 8);
            const float4 hi = *reinterpret_cast<const float4*>(x + lane * 8 + 4);
            __half2 h0 = __floats2half2_rn(lo.x, lo.y), h1 = __floats2half2_rn(lo.z, lo.w);
            __half2 h2 = __floats2half2_rn(hi.x, hi.y), h3 = __floats2half2_rn(hi.z, hi.w);
            uint4 packed;
            packed.x = *reinterpret_cast<uint32_t*>(&h0); packed.y = *reinterpret_cast<uint32_t*>(&h1);
            packed.z = *reinterpret_cast<uint32_t*>(&h2); packed.w = *reinterpret_cast<uint32_t*>(&h3);
            __half* dst = a.kv.plane(a.rows.seq_of(b0 + tb, a.seq), a.layer0 + l, kind - 1, head) +
                          (size_t)a.rows.pos_of(b0 + tb, a.pos0) * D;
            reinterpret_cast<uint4*>(dst)[lane] = packed;
        }
    }
}

template <int HKV, int TPB>
void launch_append_t(const AppendArgs& a, cudaStream_t s) {
    constexpr int ROWS = TPB * 4 * HKV;
    const size_t smem = ((size_t)ROWS * STRIDE + (size_t)TPB * SLOT) * sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(kv_append_kernel<HKV, TPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = true;
    }
    const dim3 grid((a.n + TPB - 1) / TPB, a.n_layers);
    kv_append_kernel<HKV, TPB><<<grid, ROWS, smem, s>>>(a);
}

}  // namespace

void launch_kv_append(const AppendArgs& a, cudaStream_t s) {
    // 64 rows per block for decode-sized calls; 128 for long prefills
    const bool big = (long long)a.n * a.n_layers >= 4096;
    switch (a.hkv) {
        case 8: big ? launch_append_t<8, 4>(a, s) : launch_append_t<8, 2>(a, s); break;
        case 4: big ? launch_append_t<4, 8>(a, s) : launch_append_t<4, 4>(a, s); break;
        case 2: big ? launch_append_t<2, 16>(a, s) : launch_append_t<2, 8>(a, s); break;
        case 1: big ? launch_append_t<1, 32>(a, s) : launch_append_t<1, 16>(a, s); break;
        default: break;   // rejected at context creation
    }
}

}  // namespace qattn
