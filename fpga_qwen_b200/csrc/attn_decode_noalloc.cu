// attn_decode_noalloc.cu — split-context decode attention for callers that cannot allocate.
//
// Some hosts hand this library device memory they already own and forbid it from calling
// cudaMalloc: a serving runtime that reserves all HBM for its own arena at start-up (where
// a cudaMalloc fails, or synchronises the whole device and stalls other streams), or an
// engine that embeds the attention path as a plugin with a fixed memory budget. For them,
// qa_attn_decode_noalloc runs the same split-context decode kernel as qa_attn_decode, but
// its scratch — one (max, sum, 2x128 partial output) record per (layer, row, KV head,
// split) and one arrival counter per (layer, row, KV head) — lives in the file-scope device
// array below instead of memory from qa_create. The caller passes the KV slot, the
// queries and the output buffer; the call allocates nothing.
//
// The array is QA_NOALLOC_SCRATCH_BYTES (4 MiB). With lazy module loading (the CUDA default)
// the module holding it is loaded onto a GPU when its address is first looked up, and the
// kernel's module at its first launch; qa_create does both for its device, so a host that
// creates its context before it reserves the rest of HBM meets no load (and no allocation) at
// its first call. The GPU then holds the array until the process exits.
// Every call shares it and it keeps the last call's contents: each call clears the counters
// it uses before its launch, and calls that overlap on the GPU (for example on two streams at
// once) race on it.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/qattn.h"
#include "qattn_common.cuh"

namespace qattn {
namespace {

constexpr size_t SCRATCH_BYTES = QA_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
// Device address of g_scratch per device ordinal, and the CUDA context it was looked up in: a
// device reset or a new primary context invalidates the address, so it is looked up again then.
void* g_scratch_addr[MAX_DEVICES] = {};
CUcontext g_scratch_ctx[MAX_DEVICES] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        CtxGetCurrentFn f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", reinterpret_cast<void**>(&f), cudaEnableDefault, &q) !=
            cudaSuccess)
            f = nullptr;
        return f;
    }();
    CUcontext c = nullptr;
    if (fn) fn(&c);
    return c;
}

// Looks up the device address of g_scratch on the current device. In host code `g_scratch`
// names a host-side stand-in, not device memory, so it is never passed to a kernel directly.
cudaError_t scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_mu);
    const CUcontext cur = current_context();
    if (!cur || !g_scratch_addr[device] || g_scratch_ctx[device] != cur) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);   // initialises the context if needed
        if (e != cudaSuccess) return e;
        g_scratch_addr[device] = p;
        g_scratch_ctx[device] = current_context();
    }
    *out = g_scratch_addr[device];
    return cudaSuccess;
}

}  // namespace

cudaError_t noalloc_prepare(int device) {
    if (device < 0 || device >= MAX_DEVICES) return cudaErrorInvalidDevice;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return e;
    void* p = nullptr;
    if ((e = scratch_address(device, &p)) != cudaSuccess) return e;
    return prepare_attn_rows();                 // the kernel the entry point launches, loaded too
}

}  // namespace qattn

using namespace qattn;

extern "C" int qa_attn_decode_noalloc(const void* kv_slot, int n_layers_total, int n_kv_heads, int context,
                                      int layer, int n_layers, int pos0, int n, const float* q, float* out,
                                      void* stream) {
    // ---- validation: nothing is launched or written unless all of it passes ----
    if (!kv_slot || !q || !out) return QA_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(kv_slot) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
        return QA_ERR_INVALID;                                   // 16-byte vector accesses
    if (n_layers_total < 1 || n_kv_heads < 1 || context < 1 || context > QA_MAX_CONTEXT) return QA_ERR_INVALID;
    if (layer < 0 || n_layers < 1 || layer + n_layers > n_layers_total) return QA_ERR_INVALID;
    if (n < 1 || n > QA_MAX_DECODE_ROWS) return QA_ERR_INVALID;
    if (pos0 < 0 || n > context - pos0) return QA_ERR_CAPACITY;
    const long long units = (long long)n_layers * n * n_kv_heads;
    const size_t record = (size_t)PARTIAL_FLOATS * sizeof(float);
    const size_t counter_bytes = ((size_t)units * sizeof(int) + 255) / 256 * 256;
    if (counter_bytes + (size_t)units * record > SCRATCH_BYTES) return QA_ERR_CAPACITY;   // beyond the fixed array

    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= MAX_DEVICES) return QA_ERR_CUDA;
    void* base = nullptr;
    if (scratch_address(device, &base) != cudaSuccess) return QA_ERR_CUDA;

    // splits: as many as the fixed array holds, up to the qa_attn_decode choice
    const long long max_len = pos0 + n;
    const long long fit = (long long)((SCRATCH_BYTES - counter_bytes) / record) / units;
    long long s = std::max<long long>(1, ((long long)NUM_SMS_B200 * 8 + units - 1) / units);
    s = std::min<long long>(s, (max_len + 63) / 64);
    s = std::max<long long>(1, std::min(s, fit));
    const int kps = (int)(((max_len + s - 1) / s + 31) / 32 * 32);
    const int splits = (int)((max_len + kps - 1) / kps);

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* counters = static_cast<int*>(base);
    float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + counter_bytes);
    // the array keeps the previous call's contents: start every counter this call uses at zero
    if (cudaMemsetAsync(counters, 0, (size_t)units * sizeof(int), st) != cudaSuccess) return QA_ERR_CUDA;

    RowsArgs r{};
    r.q = q; r.out = out;
    r.kv.base = static_cast<__half*>(const_cast<void*>(kv_slot));
    r.kv.layers = n_layers_total; r.kv.hkv = n_kv_heads; r.kv.ctx = context;
    r.seq = 0; r.layer0 = layer; r.n_layers = n_layers; r.pos0 = pos0; r.n = n;
    r.hq = GROUP * n_kv_heads; r.hkv = n_kv_heads; r.row_begin = 0; r.row_end = n;
    r.splits = splits; r.keys_per_split = kps; r.partial = partial; r.counters = counters;
    launch_attn_rows(r, st);
    return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_CUDA;
}
