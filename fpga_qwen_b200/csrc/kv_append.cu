// kv_append.cu — fused QK-RMSNorm + RoPE + FP16 KV write.
//
// Reference arithmetic (tampajohn/fpga-qwen engine/core.cpp), reproduced bit for bit:
//   norm  :207-215 and rope :216-218 through norm_rope.cuh (shared with the fused decode
//                  step, so both paths write the same bits)
//   store :399-405  K, V -> FP16 round-to-nearest-even at (layer, pos+b, head)
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
#include "norm_rope.cuh"

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
            const float inv = rms_inv(x, a.eps);
            #pragma unroll 4
            for (int j = 0; j < 64; j += 4) {
                const float4 xa = *reinterpret_cast<const float4*>(x + j);
                const float4 xb = *reinterpret_cast<const float4*>(x + j + 64);
                const float4 wa = *reinterpret_cast<const float4*>(w + j);
                const float4 wb = *reinterpret_cast<const float4*>(w + j + 64);
                const float4 c = *reinterpret_cast<const float4*>(cs + j);
                const float4 s = *reinterpret_cast<const float4*>(sn + j);
                float ra[4], rb[4];
                norm_rope_pair(xa.x, xb.x, wa.x, wb.x, c.x, s.x, inv, ra[0], rb[0]);
                norm_rope_pair(xa.y, xb.y, wa.y, wb.y, c.y, s.y, inv, ra[1], rb[1]);
                norm_rope_pair(xa.z, xb.z, wa.z, wb.z, c.z, s.z, inv, ra[2], rb[2]);
                norm_rope_pair(xa.w, xb.w, wa.w, wb.w, c.w, s.w, inv, ra[3], rb[3]);
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
    // 64 rows per block for decode-sized calls; 32 for long prefills, where twelve blocks per SM
    // (18 KB of shared memory each) keep copies in flight while other blocks run their sequential
    // FP64 sums (0.57 ms against 0.64 ms with 128-row blocks for 3968 rows x 28 layers)
    const bool big = (long long)a.n * a.n_layers >= 4096;
    switch (a.hkv) {
        case 8: big ? launch_append_t<8, 1>(a, s) : launch_append_t<8, 2>(a, s); break;
        case 4: big ? launch_append_t<4, 2>(a, s) : launch_append_t<4, 4>(a, s); break;
        case 2: big ? launch_append_t<2, 4>(a, s) : launch_append_t<2, 8>(a, s); break;
        case 1: big ? launch_append_t<1, 8>(a, s) : launch_append_t<1, 16>(a, s); break;
        default: break;   // rejected at context creation
    }
}

}  // namespace qattn
