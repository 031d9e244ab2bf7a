// qattn_dist.cu — multi-GPU entry points: KV-head sharding with an all-gather of the
// attention outputs, and the prefill -> decode KV-block handoff, over NCCL on NVLink.
//
// The reference runs on one host (no distributed backend). Here the 8 KV heads split over
// 1/2/4/8 GPUs (each GPU keeps the 2 query heads of its KV heads and the outputs
// [pos, 16, 128] are gathered over NVLink), independent requests spread over GPUs (no
// collective), and prefilled KV blocks move from prefill GPUs to decode GPUs.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2 — the copy a PyTorch process has
// already loaded, or the system one), so the library links neither NCCL nor PyTorch.
// One communicator per context; every call runs on the context's stream.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/qattn.h"
#include "qattn_common.cuh"
#include "sm100.cuh"

namespace qattn {
namespace {

struct NcclApi {
    bool ok = false;
    std::string err;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) { api.err = std::string("cannot load libnccl.so.2: ") + dlerror(); return; }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
        api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
        api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
        api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
        api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllGather && api.Send && api.Recv &&
                 api.GroupStart && api.GroupEnd && api.GetErrorString;
        if (!api.ok) api.err = "libnccl.so.2 lacks a required symbol";
    });
    return api;
}

// full[l][b][r*hq_local + h][:] = gathered[r][l][b][h][:]
__global__ void permute_heads_kernel(const float4* gathered, float4* full, int nranks, int n_layers, int n, int hq_local) {
    const size_t per_rank = (size_t)n_layers * n * hq_local * (D / 4);
    const size_t total = per_rank * nranks;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % (D / 4));
        size_t rr = i / (D / 4);
        const int h = (int)(rr % hq_local); rr /= hq_local;
        const int b = (int)(rr % n); rr /= n;
        const int l = (int)(rr % n_layers);
        const int r = (int)(rr / n_layers);
        const size_t dst = (((size_t)l * n + b) * (hq_local * nranks) + (size_t)r * hq_local + h) * (D / 4) + c;
        full[dst] = gathered[i];
    }
}

// Slot rows [pos0, pos0 + ntok) of every (layer, K|V, head) plane <-> contiguous
// [planes][ntok][128] (the KV handoff's staging buffer, or a block of the prefix pool).
__global__ void pack_kv_kernel(const KVLayout kv, int seq, int pos0, int ntok, uint4* buf, int unpack) {
    const size_t chunks_per_row = D * sizeof(__half) / 16;
    const size_t chunks_per_plane = (size_t)ntok * chunks_per_row;
    const size_t planes = (size_t)kv.layers * 2 * kv.hkv;
    const size_t total = chunks_per_plane * planes;
    uint4* slot = reinterpret_cast<uint4*>(kv.base + kv.slot_elems() * seq) + (size_t)pos0 * chunks_per_row;
    const size_t plane_chunks = kv.plane_elems() * sizeof(__half) / 16;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t plane = i / chunks_per_plane, c = i - plane * chunks_per_plane;
        if (unpack) slot[plane * plane_chunks + c] = buf[i];
        else buf[i] = slot[plane * plane_chunks + c];
    }
}

// One CTA per slice of the landing buffer: thread 0 waits until every rank has marked `step`
// done (acquire at system scope; bounded by the context's peer-wait limit, 2 s by default, error
// code 51 on expiry), then the CTA copies its slice. Peers wrote the landing buffer over
// NVLink before their release.
__global__ void gather_wait_copy_kernel(const unsigned* flags, int nranks, unsigned step, const float4* landing,
                                        float4* out, size_t n4, int* error) {
    // Launched as a programmatic dependent of the decode step, this grid starts while that step
    // runs (it needs nothing from it but the flags it waits for), and lets the next step launch.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = 1;
        const uint64_t t0 = sm100::globaltimer(), limit = peer_wait_limit_ns(error);
        for (int r = 0; r < nranks && ok; ++r) {
            for (;;) {
                unsigned v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
                if ((int)(v - step) >= 0) break;
                if (sm100::globaltimer() - t0 > limit) { ok = 0; atomicCAS(error, 0, 51); break; }
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __ldcg(landing + i);
}

// ---- prefill head gather through peer memory ----
// Every rank's flag array (its own memory, mapped by the peers) holds PF_READY + r ("rank r's
// rows of call k are in this rank's landing buffer") and PF_ACK + r ("rank r has copied call k
// out of its own landing buffer, so this rank may write the next call there"). Marks only
// grow; comparisons wrap.
struct PeerFlags { unsigned* p[MAX_RANKS]; };

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded by the context's peer-wait limit (2 s by default): every rank other than `rank` has
// marks[r] at or past target.
__device__ bool wait_marks(const unsigned* marks, int nranks, int rank, unsigned target, const int* error) {
    const uint64_t t0 = sm100::globaltimer(), limit = peer_wait_limit_ns(error);
    for (int r = 0; r < nranks; ++r) {
        if (r == rank) continue;
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(marks + r) : "memory");
            if ((int)(v - target) >= 0) break;
            if (sm100::globaltimer() - t0 > limit) return false;
        }
    }
    return true;
}

__global__ void prefill_gate_kernel(PeerFlags flags, int nranks, int rank, unsigned call, int* error) {
    for (int r = 0; r < nranks; ++r)                       // the copy of call - 1 ran before this launch
        if (r != rank) st_release_sys(flags.p[r] + PF_ACK + rank, call - 1);
    if (!wait_marks(flags.p[rank] + PF_ACK, nranks, rank, call - 1, error)) atomicCAS(error, 0, 52);
}

__global__ void prefill_signal_kernel(PeerFlags flags, int nranks, int rank, unsigned call) {
    __threadfence_system();                                 // the prefill kernels' stores end with one too
    for (int r = 0; r < nranks; ++r)
        if (r != rank) st_release_sys(flags.p[r] + PF_READY + rank, call);
}

// Copies the rows of the other ranks' heads: lb = layer * n + row, foreign head fh in
// [0, HQ - hq_local) maps to head fh below this rank's heads and fh + hq_local above them.
__global__ void prefill_wait_copy_kernel(const unsigned* mine, int nranks, int rank, unsigned call,
                                         const float4* landing, float4* full, size_t lb_rows, int hq_local,
                                         int* error) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = wait_marks(mine + PF_READY, nranks, rank, call, error);
        if (!ok) atomicCAS(error, 0, 53);
    }
    __syncthreads();
    if (!ok) return;
    const int hq_all = hq_local * nranks, foreign = hq_all - hq_local, first = rank * hq_local;
    const size_t total = lb_rows * foreign * (D / 4);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % (D / 4));
        const size_t rr = i / (D / 4);
        const int fh = (int)(rr % foreign);
        const size_t lb = rr / foreign;
        const int h = fh < first ? fh : fh + hq_local;
        const size_t idx = (lb * hq_all + h) * (D / 4) + c;
        full[idx] = __ldcg(landing + idx);
    }
}

}  // namespace

void launch_prefill_gate(unsigned* const* peer_flags, int nranks, int rank, unsigned call, int* error,
                         cudaStream_t s) {
    PeerFlags f{};
    for (int r = 0; r < nranks && r < MAX_RANKS; ++r) f.p[r] = peer_flags[r];
    prefill_gate_kernel<<<1, 1, 0, s>>>(f, nranks, rank, call, error);
}

void launch_prefill_signal(unsigned* const* peer_flags, int nranks, int rank, unsigned call, cudaStream_t s) {
    PeerFlags f{};
    for (int r = 0; r < nranks && r < MAX_RANKS; ++r) f.p[r] = peer_flags[r];
    prefill_signal_kernel<<<1, 1, 0, s>>>(f, nranks, rank, call);
}

void launch_prefill_wait_copy(const unsigned* my_flags, int nranks, int rank, unsigned call, const float* landing,
                              float* full, int n_layers, int n, int hq_local, int* error, cudaStream_t s) {
    const size_t lb_rows = (size_t)n_layers * n;
    const size_t n4 = lb_rows * (size_t)hq_local * (nranks - 1) * (D / 4);
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>((size_t)NUM_SMS_B200 * 4, (n4 + 255) / 256));
    prefill_wait_copy_kernel<<<blocks, 256, 0, s>>>(my_flags, nranks, rank, call,
                                                    reinterpret_cast<const float4*>(landing),
                                                    reinterpret_cast<float4*>(full), lb_rows, hq_local, error);
}

void launch_gather_wait_copy(const unsigned* flags, int nranks, unsigned step, const float* landing, float* out,
                             size_t floats, int* error, cudaStream_t s) {
    const size_t n4 = floats / 4;
    const int blocks = (int)std::max<size_t>(1, std::min<size_t>(64, (n4 + 255) / 256));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(blocks); cfg.blockDim = dim3(256); cfg.dynamicSmemBytes = 0; cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, gather_wait_copy_kernel, flags, nranks, step, reinterpret_cast<const float4*>(landing),
                       reinterpret_cast<float4*>(out), n4, error);
}

void launch_permute_heads(const float* gathered, float* full, int nranks, int n_layers, int n, int hq_local,
                          cudaStream_t s) {
    permute_heads_kernel<<<NUM_SMS_B200 * 4, 256, 0, s>>>(reinterpret_cast<const float4*>(gathered),
                                                         reinterpret_cast<float4*>(full), nranks, n_layers, n,
                                                         hq_local);
}
void launch_pack_kv(const KVLayout& kv, int seq, int pos0, int ntok, void* buf, bool unpack, cudaStream_t s) {
    pack_kv_kernel<<<NUM_SMS_B200 * 4, 512, 0, s>>>(kv, seq, pos0, ntok, reinterpret_cast<uint4*>(buf), unpack ? 1 : 0);
}

const char* nccl_load_error() { return nccl().ok ? nullptr : nccl().err.c_str(); }

int nccl_unique_id(char out[128]) {
    if (!nccl().ok) return QA_ERR_NCCL;
    ncclUniqueId id;
    if (nccl().GetUniqueId(&id) != ncclSuccess) return QA_ERR_NCCL;
    std::memcpy(out, id.internal, 128);
    return QA_OK;
}

int nccl_comm_init(void** comm, int nranks, int rank, const char id_bytes[128], std::string& err) {
    if (!nccl().ok) { err = nccl().err; return QA_ERR_NCCL; }
    ncclUniqueId id;
    std::memcpy(id.internal, id_bytes, 128);
    ncclComm_t c = nullptr;
    const ncclResult_t r = nccl().CommInitRank(&c, nranks, id, rank);
    if (r != ncclSuccess) { err = nccl().GetErrorString(r); return QA_ERR_NCCL; }
    *comm = c;
    return QA_OK;
}

void nccl_comm_destroy(void* comm) {
    if (comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(comm));
}

int nccl_all_gather_f32(void* comm, const float* send, float* recv, size_t count, cudaStream_t s, std::string& err) {
    const ncclResult_t r = nccl().AllGather(send, recv, count, ncclFloat32, static_cast<ncclComm_t>(comm), s);
    if (r != ncclSuccess) { err = nccl().GetErrorString(r); return QA_ERR_NCCL; }
    return QA_OK;
}

int nccl_all_gather_bytes(void* comm, const void* send, void* recv, size_t bytes, cudaStream_t s, std::string& err) {
    const ncclResult_t r = nccl().AllGather(send, recv, bytes, ncclUint8, static_cast<ncclComm_t>(comm), s);
    if (r != ncclSuccess) { err = nccl().GetErrorString(r); return QA_ERR_NCCL; }
    return QA_OK;
}

int nccl_send_recv_bytes(void* comm, void* buf, size_t bytes, int peer, bool send, cudaStream_t s, std::string& err) {
    const ncclResult_t r = send ? nccl().Send(buf, bytes, ncclUint8, peer, static_cast<ncclComm_t>(comm), s)
                                : nccl().Recv(buf, bytes, ncclUint8, peer, static_cast<ncclComm_t>(comm), s);
    if (r != ncclSuccess) { err = nccl().GetErrorString(r); return QA_ERR_NCCL; }
    return QA_OK;
}

}  // namespace qattn
