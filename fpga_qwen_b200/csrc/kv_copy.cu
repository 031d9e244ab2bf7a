// kv_copy.cu — canonical prefix reuse by device block copy, and the seeded synthetic
// input generator.
//
// Prefix copy: the reference retains a canonical 512-token prefix by rewinding the same
// process's KV (tools/native_cpu_chat.py:189-216 -> engine/core.cpp:722-726). Here a
// prefix held by one sequence slot is copied into another slot: for every
// (layer, K|V, head) plane, rows [0, ntok) — 256 bytes each — are copied with 16-byte
// vector loads and stores, one grid-stride pass over all planes. The copy is HBM-bound:
// 2 * 114,688 * ntok bytes at 28 layers and 8 KV heads.
#include "qattn_common.cuh"

namespace qattn {
namespace {

__global__ void kv_copy_kernel(const KVLayout kv, int src_seq, int dst_seq, int ntok) {
    const size_t chunks_per_plane = (size_t)ntok * (D * sizeof(__half) / 16);      // 16 per row
    const size_t planes = (size_t)kv.layers * 2 * kv.hkv;
    const size_t total = chunks_per_plane * planes;
    const uint4* src = reinterpret_cast<const uint4*>(kv.base + kv.slot_elems() * src_seq);
    uint4* dst = reinterpret_cast<uint4*>(kv.base + kv.slot_elems() * dst_seq);
    const size_t plane_chunks = kv.plane_elems() * sizeof(__half) / 16;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t plane = i / chunks_per_plane, c = i - plane * chunks_per_plane;
        const size_t off = plane * plane_chunks + c;
        dst[off] = __ldcs(src + off);
    }
}

// SplitMix64 finaliser (Steele, Lea, Flood 2014).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void synth_kernel(float* dst, uint64_t seed, int kind, int layer0, int n_layers, int pos0,
                             int n, int head0, int heads, float mean, float stdev) {
    const size_t total = (size_t)n_layers * n * heads * D;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int j = int(i % D);
        size_t r = i / D;
        const int h = int(r % heads); r /= heads;
        const int b = int(r % n);
        const int l = int(r / n);
        const uint64_t key = ((((uint64_t)kind * 64 + (layer0 + l)) * 8192 + (pos0 + b)) * 64 + (head0 + h)) * D + j;
        const uint64_t x = mix64(seed * 0x9E3779B97F4A7C15ull + mix64(key + 0x632BE59BD9B4E019ull));
        const float u1 = ((float)(x >> 40) + 0.5f) * (1.0f / 16777216.0f);        // (0,1)
        const float u2 = (float)((x >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);    // [0,1)
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);               // Box-Muller
        dst[i] = mean + stdev * z;
    }
}

}  // namespace

void launch_kv_copy(const KVLayout& kv, int src_seq, int dst_seq, int ntok, cudaStream_t s) {
    kv_copy_kernel<<<NUM_SMS_B200 * 4, 512, 0, s>>>(kv, src_seq, dst_seq, ntok);
}

void launch_synth(float* dst, uint64_t seed, int kind, int layer0, int n_layers, int pos0, int n,
                  int head0, int heads, float mean, float stdev, cudaStream_t s) {
    synth_kernel<<<NUM_SMS_B200 * 8, 256, 0, s>>>(dst, seed, kind, layer0, n_layers, pos0, n, head0, heads,
                                                  mean, stdev);
}

}  // namespace qattn
