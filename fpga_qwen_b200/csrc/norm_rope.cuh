// norm_rope.cuh — the reference's QK-RMSNorm and RoPE arithmetic for one 128-channel row,
// shared by every kernel that appends KV rows, so all of them produce the same bits.
//
// tampajohn/fpga-qwen engine/core.cpp:
//   norm  :207-215  square = x*x (FP32); sum = sum of double(square) over j = 0..127 in
//                   ascending order (FP64); inv = 1 / sqrt(float(sum)/128 + eps); out = (x*inv)*w
//   rope  :216-218  x[j] = a*c - b*s; x[j+64] = b*c + a*s  (unfused products)
// Every rounding step is an explicit _rn intrinsic so no compiler contraction can change a
// result.
#pragma once

#include "qattn_common.cuh"

namespace qattn {

// inv of one row x[0..127] (any address space). Only the FP64 additions form a dependency
// chain; the squares and conversions are independent.
__device__ __forceinline__ float rms_inv(const float* x, float eps) {
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
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), eps)));
}

// Channel pair (j, j+64), j < 64: normalise with inv and weights (wa, wb), rotate by (c, s).
__device__ __forceinline__ void norm_rope_pair(float xa, float xb, float wa, float wb, float c, float s, float inv,
                                               float& ra, float& rb) {
    const float na = __fmul_rn(__fmul_rn(xa, inv), wa);
    const float nb = __fmul_rn(__fmul_rn(xb, inv), wb);
    ra = __fsub_rn(__fmul_rn(na, c), __fmul_rn(nb, s));
    rb = __fadd_rn(__fmul_rn(nb, c), __fmul_rn(na, s));
}

}  // namespace qattn
