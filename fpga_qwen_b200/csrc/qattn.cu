// qattn.cu — context, validation and the C ABI of libqattn.so (declared in include/qattn.h).
//
// The context owns everything the reference's Model::Impl owns for this path
// (engine/core.cpp:223-232, :277, :287-288): the FP16 KV history (here in HBM, one slot per
// sequence), the RoPE tables, the per-layer q_norm/k_norm weights and the logical position
// `pos` of each sequence. All validation happens on the host before any launch, so a call
// that fails validation leaves the state unchanged (core.hpp:32-33, :41).
#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/qattn.h"
#include "../../include/qattn_synth.h"
#include "qattn_common.cuh"

using namespace qattn;

namespace qattn {
int nccl_unique_id(char out[128]);
int nccl_comm_init(void** comm, int nranks, int rank, const char id_bytes[128], std::string& err);
void nccl_comm_destroy(void* comm);
int nccl_all_gather_f32(void* comm, const float* send, float* recv, size_t count, cudaStream_t s, std::string& err);
int nccl_send_recv_bytes(void* comm, void* buf, size_t bytes, int peer, bool send, cudaStream_t s, std::string& err);
int nccl_all_gather_bytes(void* comm, const void* send, void* recv, size_t bytes, cudaStream_t s, std::string& err);
}  // namespace qattn

struct qa_ctx {
    qa_config cfg{};
    int hq = 0, hkv = 0;                   // local heads
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    KVLayout kv{};
    float* norms = nullptr;                // [L][2][128]
    float* cosines = nullptr;              // [ctx][64]
    float* sines = nullptr;
    std::vector<int> pos;                  // committed position per sequence
    std::vector<std::vector<int>> appended;  // per sequence, per layer: rows written through
    void* proj_scratch = nullptr;          // the tensor-core projections' split input rows (project_mma.cu)
    float* partial = nullptr;              // split-context records, sized at creation for any call
    size_t partial_floats = 0;
    int* counters = nullptr;
    int max_units = 0;                     // counters held
    // One device allocation made at creation: [error block (ERR_BLOCK_BYTES)][staging]. io_host
    // contexts stage [outputs: io_out_floats][inputs: io_in_floats]; device-pointer contexts keep
    // the query rows of the fused decode step's two-launch form there.
    char* io_dev = nullptr;
    float* staging = nullptr;
    size_t staging_floats = 0, io_out_floats = 0, io_in_floats = 0;
    char* io_pin = nullptr;                // io_host: pinned [error block][outputs][inputs] of packed copies
    CUtensorMap kv_map{};                  // 3-D view {128 ch, ctx, planes} of the KV store, 64x128 boxes
    int* error = nullptr;                  // device error block (qattn_common.cuh: ERR_*), at io_dev
    int* prefill_tiles = nullptr;          // work-item counter of the persistent prefill kernel
    float* prefill_split = nullptr;        // partial rows of prefill items split over key segments
    // The FP32 rows below position 128 run on a second stream next to the persistent tensor-core
    // kernel (fork: aux waits for the context stream; join: the context stream waits for aux).
    cudaStream_t aux_stream = nullptr;
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    void* comm = nullptr;                  // NCCL communicator (multi-GPU)
    cudaStream_t comm_stream = nullptr;    // NCCL work runs here, ordered after/before the context stream
    cudaEvent_t comm_ev[2] = {nullptr, nullptr};
    int nranks = 1, rank = 0;
    float* gather_buf = nullptr;           // all-gather landing buffer
    size_t gather_floats = 0;
    // KV handoff staging: two buffers used alternately, so the pack (or unpack) of one request
    // overlaps the NVLink transfer of the previous one. kv_comm_done[b]: the NCCL op that used
    // buffer b has finished (comm stream); kv_unpacked[b]: the unpack from buffer b has finished
    // (context stream).
    void* kv_buf[2] = {nullptr, nullptr};
    size_t kv_buf_bytes[2] = {0, 0};
    cudaEvent_t kv_comm_done[2] = {nullptr, nullptr};
    cudaEvent_t kv_unpacked[2] = {nullptr, nullptr};
    cudaEvent_t kv_packed = nullptr;
    int kv_next = 0;
    // Head gather through peer memory: one allocation per rank, [landing 0][landing 1][flags],
    // mapped into every other rank with CUDA IPC. Landing buffers alternate by step.
    char* peer_block = nullptr;
    size_t landing_bytes = 0, flags_off = 0;
    char* peer_base[MAX_RANKS] = {};       // every rank's allocation (this rank's at [rank])
    bool peer_ok = false;
    size_t peer_min_bytes = 0;             // every rank's allocation (equal on all ranks)
    unsigned* gather_done = nullptr;       // CTAs of the gathering launch that finished
    unsigned gather_step = 0;
    float* step_out = nullptr;             // local output of the NCCL fallback
    // Prefill head gather through peer memory: a landing buffer per rank for the other ranks'
    // heads ([layers][context][all heads][128] FP32), mapped like the decode one on first use.
    char* pf_block = nullptr;
    char* pf_base[MAX_RANKS] = {};
    bool pf_tried = false, pf_ok = false;
    unsigned pf_call = 0;
    size_t pf_min_bytes = 0;               // smallest rank's prefill landing buffer
    float* pf_local = nullptr;             // local output of the NCCL fallback
    size_t pf_local_bytes = 0;
    // Prefix block pool (qa_block_pool): block b holds one 512-row chunk of every plane,
    // [planes][512][128] FP16; pool_chunk[b] is the chunk index it was saved from (-1: empty).
    __half* pool = nullptr;
    std::vector<int> pool_chunk;
    bool step_overlap = false;             // qa_set_step_overlap
    bool last_fused_step = false;          // the last launch on the stream was a fused decode step
    size_t step_out_bytes = 0;
    std::string err;
};

namespace {

void close_mappings(char* (&base)[MAX_RANKS], const char* own) {
    for (int r = 0; r < MAX_RANKS; ++r) {
        if (base[r] && base[r] != own) cudaIpcCloseMemHandle(base[r]);
        base[r] = nullptr;
    }
}

void peer_release(qa_ctx* ctx) {
    close_mappings(ctx->pf_base, ctx->pf_block);
    cudaFree(ctx->pf_block);
    ctx->pf_block = nullptr; ctx->pf_ok = false; ctx->pf_tried = false;
    close_mappings(ctx->peer_base, ctx->peer_block);
    cudaFree(ctx->peer_block);
    cudaFree(ctx->gather_done);
    ctx->peer_block = nullptr; ctx->gather_done = nullptr; ctx->peer_ok = false;
}

int fail(qa_ctx* c, int status, const char* fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap; va_start(ap, fmt); vsnprintf(buf, sizeof buf, fmt, ap); va_end(ap);
        c->err = buf;
    }
    return status;
}

int cuda_fail(qa_ctx* c, cudaError_t e, const char* what) {
    return fail(c, e == cudaErrorMemoryAllocation ? QA_ERR_OOM : QA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define QA_CUDA(call)                                                  \
    do {                                                               \
        cudaError_t e_ = (call);                                       \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call);       \
    } while (0)

// After a launch or device error the affected sequence restarts from position 0, like the
// engine's "Errors ... reset all model ... state" (engine/INTERFACE.md error contract).
int after_launch(qa_ctx* ctx, int seq, const char* what) {
    ctx->last_fused_step = false;
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return QA_OK;
    if (seq >= 0 && seq < (int)ctx->pos.size()) {
        ctx->pos[seq] = 0;
        std::fill(ctx->appended[seq].begin(), ctx->appended[seq].end(), 0);
    }
    return cuda_fail(ctx, e, what);
}

int check_seq(qa_ctx* ctx, int seq) {
    if (seq < 0 || seq >= ctx->cfg.max_seqs) return fail(ctx, QA_ERR_INVALID, "sequence %d out of range [0,%d)", seq, ctx->cfg.max_seqs);
    return QA_OK;
}

int check_layers(qa_ctx* ctx, int layer, int n_layers) {
    if (layer < 0 || n_layers < 1 || layer + n_layers > ctx->cfg.n_layers)
        return fail(ctx, QA_ERR_INVALID, "layer range [%d,%d) outside [0,%d)", layer, layer + n_layers, ctx->cfg.n_layers);
    return QA_OK;
}

// Common validation of the hot-path calls: rows [pos0, pos0+n) at the committed position.
int check_rows(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n) {
    int st;
    if ((st = check_seq(ctx, seq))) return st;
    if ((st = check_layers(ctx, layer, n_layers))) return st;
    if (n < 1) return fail(ctx, QA_ERR_INVALID, "empty input (n=%d)", n);
    if (pos0 != ctx->pos[seq])
        return fail(ctx, QA_ERR_STATE, "pos0 %d differs from the sequence position %d", pos0, ctx->pos[seq]);
    if (n > ctx->cfg.context - pos0)
        return fail(ctx, QA_ERR_CAPACITY, "context capacity exceeded: %d + %d > %d", pos0, n, ctx->cfg.context);
    return QA_OK;
}

int check_appended(qa_ctx* ctx, int seq, int layer, int n_layers, int end) {
    for (int l = layer; l < layer + n_layers; ++l)
        if (ctx->appended[seq][l] < end)
            return fail(ctx, QA_ERR_STATE, "layer %d holds rows through %d, attention needs %d", l, ctx->appended[seq][l], end);
    return QA_OK;
}

// ---- host-buffer (io_host) calls -----------------------------------------------------------------
// A host-buffer call copies its inputs into the device staging, launches, then copies its outputs
// back together with the device error block, and waits for the stream: one host->device and one
// device->host copy when the inputs and the outputs each fit IO_PACK_BYTES (packed through the
// pinned mirror io_pin), one copy per tensor otherwise. Calls whose rows x layers exceed the
// staging made at creation run in chunks of whole layers (every layer is independent). A bounded
// wait that ran out during the call fails it with QA_ERR_TIMEOUT and resets the sequence.
// Pinned host buffers (cudaHostAlloc, cudaHostRegister, torch's pin_memory) are reachable from the
// device: when every host buffer of a call is pinned, 16-byte aligned, and the call moves at most
// IO_DIRECT_BYTES, the kernels read the inputs and write the outputs over PCIe themselves and
// only the error block is copied back, which saves the staging copies and their latency on
// decode-sized calls.
constexpr size_t IO_PACK_BYTES = size_t(64) << 10;      // above this, one copy per tensor is faster
constexpr size_t IO_DIRECT_BYTES = size_t(8) << 20;

// A decode launch splits the keys of its n_layers x n x hkv units evenly over 2 CTAs per SM, and
// every CTA that covers part of a unit reads the unit's input rows: with at least one unit per
// SM the rows are read about once or twice; a one-layer call splits each unit over ~37 CTAs.
bool decode_inputs_read_once(int n_layers, int n, int hkv) { return (long long)n_layers * n * hkv >= NUM_SMS_B200; }

// The device address of pinned host memory at p, or null (pageable, device memory, misaligned).
const void* pinned_device_address(const void* p) {
    cudaPointerAttributes at{};
    if (!p || (reinterpret_cast<uintptr_t>(p) & 15)) return nullptr;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (at.type != cudaMemoryTypeHost || !at.devicePointer || (reinterpret_cast<uintptr_t>(at.devicePointer) & 15))
        return nullptr;
    return at.devicePointer;
}

struct IoCall {
    const float* in[3] = {};       // host inputs, [n_layers][...] layer-major
    size_t in_floats[3] = {};      // floats per layer of each input (0: unused)
    float* out[2] = {};            // host outputs: out[0] always, out[1] optional (may be null)
    size_t out_floats[2] = {};     // floats per layer (device room for out[1] is kept even when null)
    // the kernels read each input row about once, so pinned buffers may be used in place over
    // PCIe; false where many CTAs read the same rows (a decode whose units are split many ways),
    // which then goes through the staging copies (measured faster for one-layer decode calls)
    bool inputs_read_once = true;
};

// launch(l0, nl, din, dout) enqueues the work of layers [l0, l0 + nl) on device pointers and
// returns a status (after_launch).
template <class Launch>
int io_host_call(qa_ctx* ctx, int seq, int layer, int n_layers, const IoCall& c, Launch&& launch) {
    const size_t in_pl = c.in_floats[0] + c.in_floats[1] + c.in_floats[2];
    const size_t out_pl = c.out_floats[0] + c.out_floats[1];
    size_t fit = (size_t)n_layers;
    if (in_pl) fit = std::min(fit, ctx->io_in_floats / in_pl);
    if (out_pl) fit = std::min(fit, ctx->io_out_floats / out_pl);
    int* const h_err = reinterpret_cast<int*>(ctx->io_pin);
    // the error block came back with the call's outputs: a wait that ran out fails the call
    auto check_error = [&]() -> int {
        if (const int code = h_err[ERR_CODE]) {
            QA_CUDA(cudaMemsetAsync(ctx->error + ERR_CODE, 0, sizeof(int), ctx->stream));
            QA_CUDA(cudaStreamSynchronize(ctx->stream));
            if (seq >= 0 && seq < (int)ctx->pos.size()) {
                ctx->pos[seq] = 0;
                std::fill(ctx->appended[seq].begin(), ctx->appended[seq].end(), 0);
            }
            return fail(ctx, QA_ERR_TIMEOUT, "a device-side wait expired (code %d); the call's results are invalid", code);
        }
        return QA_OK;
    };
    if (c.inputs_read_once && (in_pl + out_pl) * n_layers * sizeof(float) <= IO_DIRECT_BYTES) {
        const float* din[3] = {};
        float* dout[2] = {};
        bool direct = true;
        for (int i = 0; i < 3; ++i)
            if (c.in_floats[i]) direct = direct && (din[i] = static_cast<const float*>(pinned_device_address(c.in[i])));
        for (int j = 0; j < 2; ++j)
            if (c.out[j]) direct = direct && (dout[j] = static_cast<float*>(const_cast<void*>(pinned_device_address(c.out[j]))));
        if (direct) {
            int st = launch(layer, n_layers, din, dout);
            if (st) return st;
            QA_CUDA(cudaMemcpyAsync(h_err, ctx->io_dev, ERR_BLOCK_BYTES, cudaMemcpyDeviceToHost, ctx->stream));
            QA_CUDA(cudaStreamSynchronize(ctx->stream));
            return check_error();
        }
    }
    if (fit < 1) return fail(ctx, QA_ERR_CAPACITY, "one layer of this call exceeds the host-buffer staging");
    const int chunk = (int)fit;
    float* const d_out = ctx->staging;
    float* const d_in = ctx->staging + ctx->io_out_floats;
    float* const h_out = reinterpret_cast<float*>(ctx->io_pin + ERR_BLOCK_BYTES);
    float* const h_in = h_out + IO_PACK_BYTES / sizeof(float);
    for (int l0 = layer; l0 < layer + n_layers; l0 += chunk) {
        const int nl = std::min(chunk, layer + n_layers - l0);
        const size_t lo = (size_t)(l0 - layer);
        const float* din[3] = {};
        float* dout[2] = {};
        size_t in_total = 0, back = 0;
        for (int i = 0; i < 3; ++i)
            if (c.in_floats[i]) { din[i] = d_in + in_total; in_total += c.in_floats[i] * nl; }
        dout[0] = d_out;
        if (c.out_floats[1]) dout[1] = d_out + c.out_floats[0] * nl;
        back = c.out_floats[0] * nl + (c.out[1] ? c.out_floats[1] * nl : 0);
        const bool pack = in_total * sizeof(float) <= IO_PACK_BYTES && back * sizeof(float) <= IO_PACK_BYTES;
        if (pack) {
            size_t o = 0;
            for (int i = 0; i < 3; ++i)
                if (c.in_floats[i]) {
                    std::memcpy(h_in + o, c.in[i] + lo * c.in_floats[i], c.in_floats[i] * nl * sizeof(float));
                    o += c.in_floats[i] * nl;
                }
            if (in_total) QA_CUDA(cudaMemcpyAsync(d_in, h_in, in_total * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
        } else {
            for (int i = 0; i < 3; ++i)
                if (c.in_floats[i])
                    QA_CUDA(cudaMemcpyAsync(const_cast<float*>(din[i]), c.in[i] + lo * c.in_floats[i],
                                            c.in_floats[i] * nl * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
        }
        int st = launch(l0, nl, din, dout);
        if (st) return st;
        if (pack) {
            QA_CUDA(cudaMemcpyAsync(h_err, ctx->io_dev, ERR_BLOCK_BYTES + back * sizeof(float), cudaMemcpyDeviceToHost,
                                    ctx->stream));
        } else {
            QA_CUDA(cudaMemcpyAsync(h_err, ctx->io_dev, ERR_BLOCK_BYTES, cudaMemcpyDeviceToHost, ctx->stream));
            for (int j = 0; j < 2; ++j)
                if (c.out[j])
                    QA_CUDA(cudaMemcpyAsync(c.out[j] + lo * c.out_floats[j], dout[j], c.out_floats[j] * nl * sizeof(float),
                                            cudaMemcpyDeviceToHost, ctx->stream));
        }
        QA_CUDA(cudaStreamSynchronize(ctx->stream));
        if (pack) {
            size_t o = 0;
            for (int j = 0; j < 2; ++j)
                if (c.out_floats[j]) {
                    if (c.out[j]) std::memcpy(c.out[j] + lo * c.out_floats[j], h_out + o, c.out_floats[j] * nl * sizeof(float));
                    o += c.out_floats[j] * nl;
                }
        }
        if ((st = check_error())) return st;
    }
    return QA_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// TMA descriptor of the KV store: planes of [ctx][128] FP16 rows; rows past ctx read as zero.
int make_kv_map(qa_ctx* ctx) {
    EncodeTiledFn encode = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &q) !=
            cudaSuccess || !encode)
        return fail(ctx, QA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t planes = (cuuint64_t)ctx->cfg.max_seqs * ctx->cfg.n_layers * 2 * ctx->hkv;
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)ctx->cfg.context, planes};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)ctx->cfg.context * D * 2};
    cuuint32_t box[3] = {64, 128, 1}, elem[3] = {1, 1, 1};
    CUresult r = encode(&ctx->kv_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ctx->kv.base, dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ctx, QA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QA_OK;
}

// Reads and clears the device error flag of the bounded waits.
int check_device_error(qa_ctx* ctx) {
    int code = 0;
    QA_CUDA(cudaMemcpyAsync(&code, ctx->error, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    if (code) {
        QA_CUDA(cudaMemsetAsync(ctx->error, 0, sizeof(int), ctx->stream));
        return fail(ctx, QA_ERR_TIMEOUT, "a device-side wait expired (code %d); results of the last calls are invalid", code);
    }
    return QA_OK;
}

// Runs `launch` on the caller's device pointers, or through the host-buffer staging (io_host).
template <class Launch>
int run_call(qa_ctx* ctx, int seq, int layer, int n_layers, const IoCall& c, Launch&& launch) {
    if (ctx->cfg.io_host) return io_host_call(ctx, seq, layer, n_layers, c, launch);
    const float* din[3] = {c.in[0], c.in[1], c.in[2]};
    float* dout[2] = {c.out[0], c.out[1]};
    return launch(layer, n_layers, din, dout);
}

}  // namespace

extern "C" {

const char* qa_version(void) { return "qattn 0.1 sm_100a"; }

const char* qa_status_string(int status) {
    switch (status) {
        case QA_OK: return "ok";
        case QA_ERR_INVALID: return "invalid argument";
        case QA_ERR_CAPACITY: return "context capacity exceeded";
        case QA_ERR_STATE: return "invalid state";
        case QA_ERR_CUDA: return "CUDA error";
        case QA_ERR_NCCL: return "NCCL error";
        case QA_ERR_TIMEOUT: return "device wait timed out";
        case QA_ERR_OOM: return "out of device memory";
        case QA_ERR_UNSUPPORTED: return "unsupported";
        default: return "unknown status";
    }
}

void qa_default_config(qa_config* c) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->n_layers = 28; c->n_q_heads = 16; c->n_kv_heads = 8; c->head_dim = 128;
    c->context = QA_MAX_CONTEXT; c->max_seqs = 1; c->kv_head_begin = 0; c->kv_head_count = 0;
    c->rope_theta = 1000000.0; c->norm_eps = 1e-6f; c->device = 0; c->io_host = 0;
}

const char* qa_last_error(const qa_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int qa_create(const qa_config* cfg, qa_ctx** out) {
    if (!cfg || !out) return QA_ERR_INVALID;
    *out = nullptr;
    qa_config c = *cfg;
    if (c.kv_head_count == 0) c.kv_head_count = c.n_kv_heads;
    // Shape limits: Qwen3-0.6B attention (core.cpp:28, :236-237).
    if (c.head_dim != D) return QA_ERR_UNSUPPORTED;
    if (c.n_kv_heads < 1 || c.n_q_heads != GROUP * c.n_kv_heads) return QA_ERR_UNSUPPORTED;
    if (c.n_layers < 1 || c.n_layers > 64) return QA_ERR_INVALID;
    if (c.context < 1 || c.context > QA_MAX_CONTEXT) return QA_ERR_INVALID;
    if (c.max_seqs < 1 || c.max_seqs > 4096) return QA_ERR_INVALID;
    if (c.kv_head_begin < 0 || c.kv_head_count < 1 || c.kv_head_begin + c.kv_head_count > c.n_kv_heads) return QA_ERR_INVALID;
    // kernels are specialised for 1, 2, 4 or 8 KV heads per context (Qwen3-0.6B: 8 over 1/2/4/8 GPUs)
    if (c.kv_head_count != 1 && c.kv_head_count != 2 && c.kv_head_count != 4 && c.kv_head_count != 8)
        return QA_ERR_UNSUPPORTED;
    if (!(c.rope_theta > 1.0) || !(c.norm_eps > 0.f)) return QA_ERR_INVALID;

    qa_ctx* ctx = new (std::nothrow) qa_ctx();
    if (!ctx) return QA_ERR_OOM;
    ctx->cfg = c;
    ctx->hkv = c.kv_head_count;
    ctx->hq = GROUP * c.kv_head_count;
    auto cleanup = [&](int st) { qa_destroy(ctx); return st; };

    if (cudaSetDevice(c.device) != cudaSuccess) return cleanup(QA_ERR_CUDA);
    if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess) return cleanup(QA_ERR_CUDA);
    ctx->stream = ctx->own_stream;

    ctx->kv.layers = c.n_layers; ctx->kv.hkv = ctx->hkv; ctx->kv.ctx = c.context;
    const size_t kv_bytes = ctx->kv.slot_elems() * sizeof(__half) * c.max_seqs;
    if (cudaMalloc(&ctx->kv.base, kv_bytes) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMemset(ctx->kv.base, 0, kv_bytes) != cudaSuccess) return cleanup(QA_ERR_CUDA);

    // RoPE tables exactly as core.cpp:288 computes them (FP64 angle, FP64 cos/sin, FP32 store).
    std::vector<float> cs((size_t)c.context * 64), sn(cs.size());
    for (int p = 0; p < c.context; ++p)
        for (int j = 0; j < 64; ++j) {
            const double angle = p / std::pow(c.rope_theta, 2.0 * j / D);
            cs[(size_t)p * 64 + j] = (float)std::cos(angle);
            sn[(size_t)p * 64 + j] = (float)std::sin(angle);
        }
    if (cudaMalloc(&ctx->cosines, cs.size() * sizeof(float)) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMalloc(&ctx->sines, sn.size() * sizeof(float)) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMemcpy(ctx->cosines, cs.data(), cs.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) return cleanup(QA_ERR_CUDA);
    if (cudaMemcpy(ctx->sines, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) return cleanup(QA_ERR_CUDA);

    std::vector<float> ones((size_t)c.n_layers * 2 * D, 1.0f);
    if (cudaMalloc(&ctx->norms, ones.size() * sizeof(float)) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMemcpy(ctx->norms, ones.data(), ones.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) return cleanup(QA_ERR_CUDA);

    // Split-context records and counters sized for the largest decode plan any call can make
    // (QA_MAX_DECODE_ROWS rows, or a batch of up to min(max_seqs, QA_MAX_BATCH) sequences, over
    // all layers), so that no hot call allocates.
    const int n_max = std::min(QA_MAX_BATCH, std::max(c.max_seqs, QA_MAX_DECODE_ROWS));
    ctx->max_units = c.n_layers * n_max * ctx->hkv;
    ctx->partial_floats = decode_partial_floats_bound(c.n_layers, ctx->hkv, n_max);
    if (cudaMalloc(&ctx->partial, ctx->partial_floats * sizeof(float)) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMalloc(&ctx->counters, (size_t)ctx->max_units * sizeof(int)) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMemset(ctx->counters, 0, (size_t)ctx->max_units * sizeof(int)) != cudaSuccess) return cleanup(QA_ERR_CUDA);

    // Error block + staging. io_host: room for io_rows rows of every tensor of one layer
    // (io_rows = max(context, QA_MAX_BATCH)); larger calls run in layer chunks. Device pointers:
    // the normalised query rows of the fused decode step's two-launch form (all layers, n_max rows).
    if (c.io_host) {
        const size_t io_rows = (size_t)std::max(c.context, QA_MAX_BATCH);
        ctx->io_out_floats = io_rows * 2 * ctx->hq * D;
        ctx->io_in_floats = io_rows * (ctx->hq + 2 * ctx->hkv) * D;
        ctx->staging_floats = ctx->io_out_floats + ctx->io_in_floats;
        if (cudaMallocHost(&ctx->io_pin, ERR_BLOCK_BYTES + 2 * IO_PACK_BYTES) != cudaSuccess) return cleanup(QA_ERR_OOM);
    } else {
        ctx->staging_floats = (size_t)c.n_layers * n_max * ctx->hq * D;
    }
    if (cudaMalloc(&ctx->io_dev, ERR_BLOCK_BYTES + ctx->staging_floats * sizeof(float)) != cudaSuccess)
        return cleanup(QA_ERR_OOM);
    if (cudaMemset(ctx->io_dev, 0, ERR_BLOCK_BYTES) != cudaSuccess) return cleanup(QA_ERR_CUDA);
    ctx->error = reinterpret_cast<int*>(ctx->io_dev);
    ctx->staging = reinterpret_cast<float*>(ctx->io_dev + ERR_BLOCK_BYTES);
    // the prefill's work counter and finished-CTA count: zero here, reset by each launch's last CTA
    if (cudaMalloc(&ctx->prefill_tiles, 2 * sizeof(int)) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMemset(ctx->prefill_tiles, 0, 2 * sizeof(int)) != cudaSuccess) return cleanup(QA_ERR_CUDA);
    if (cudaMalloc(&ctx->prefill_split, prefill_split_scratch_bytes()) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaMalloc(&ctx->proj_scratch, project_gemm_scratch_bytes()) != cudaSuccess) return cleanup(QA_ERR_OOM);
    if (cudaStreamCreateWithFlags(&ctx->aux_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->fork_ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->join_ev, cudaEventDisableTiming) != cudaSuccess)
        return cleanup(QA_ERR_CUDA);
    // the device address of qa_attn_decode_noalloc's fixed scratch, looked up now (it loads that
    // module onto the GPU) rather than at its first call, when the host may own all free memory
    if (noalloc_prepare(c.device) != cudaSuccess) return cleanup(QA_ERR_CUDA);
    if (make_kv_map(ctx) != QA_OK) return cleanup(QA_ERR_CUDA);

    ctx->pos.assign(c.max_seqs, 0);
    ctx->appended.assign(c.max_seqs, std::vector<int>(c.n_layers, 0));
    if (cudaDeviceSynchronize() != cudaSuccess) return cleanup(QA_ERR_CUDA);
    *out = ctx;
    return QA_OK;
}

void qa_destroy(qa_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->cfg.device);
    if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
    if (ctx->stream && ctx->stream != ctx->own_stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->kv.base); cudaFree(ctx->cosines); cudaFree(ctx->sines); cudaFree(ctx->norms);
    cudaFree(ctx->partial); cudaFree(ctx->counters); cudaFree(ctx->io_dev); cudaFreeHost(ctx->io_pin);
    cudaFree(ctx->prefill_tiles); cudaFree(ctx->prefill_split); cudaFree(ctx->proj_scratch);
    if (ctx->aux_stream) { cudaStreamSynchronize(ctx->aux_stream); cudaStreamDestroy(ctx->aux_stream); }
    if (ctx->fork_ev) cudaEventDestroy(ctx->fork_ev);
    if (ctx->join_ev) cudaEventDestroy(ctx->join_ev);
    cudaFree(ctx->gather_buf); cudaFree(ctx->kv_buf[0]); cudaFree(ctx->kv_buf[1]);
    for (cudaEvent_t e : ctx->kv_comm_done) if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->kv_unpacked) if (e) cudaEventDestroy(e);
    if (ctx->kv_packed) cudaEventDestroy(ctx->kv_packed);
    peer_release(ctx);
    cudaFree(ctx->step_out); cudaFree(ctx->pf_local); cudaFree(ctx->pool);
    nccl_comm_destroy(ctx->comm);
    if (ctx->comm_stream) cudaStreamDestroy(ctx->comm_stream);
    for (cudaEvent_t e : ctx->comm_ev) if (e) cudaEventDestroy(e);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
}

int qa_set_stream(qa_ctx* ctx, void* s) {
    if (!ctx) return QA_ERR_INVALID;
    ctx->stream = s ? static_cast<cudaStream_t>(s) : ctx->own_stream;
    ctx->last_fused_step = false;
    return QA_OK;
}

int qa_sync(qa_ctx* ctx) {
    if (!ctx) return QA_ERR_INVALID;
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->comm_stream) QA_CUDA(cudaStreamSynchronize(ctx->comm_stream));
    return check_device_error(ctx);
}

int qa_set_wait_limit(qa_ctx* ctx, int microseconds) {
    if (!ctx) return QA_ERR_INVALID;
    if (microseconds < 0) return fail(ctx, QA_ERR_INVALID, "negative wait limit %d", microseconds);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const unsigned us = (unsigned)microseconds;
    QA_CUDA(cudaMemcpyAsync(ctx->error + ERR_WAIT_US, &us, sizeof us, cudaMemcpyHostToDevice, ctx->stream));
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    return QA_OK;
}

int qa_selftest_timeout(qa_ctx* ctx) {
    if (!ctx) return QA_ERR_INVALID;
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    // the head gather's wait kernel, waiting for one rank's mark of step 1 in a word that stays 0
    launch_gather_wait_copy(reinterpret_cast<const unsigned*>(ctx->error + ERR_NEVER), 1, 1u, nullptr, nullptr, 0,
                            ctx->error, ctx->stream);
    return after_launch(ctx, -1, "selftest_timeout");
}

int qa_set_norms(qa_ctx* ctx, int layer, const float* q_norm, const float* k_norm) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_layers(ctx, layer, 1))) return st;
    if (!q_norm || !k_norm) return fail(ctx, QA_ERR_INVALID, "null norm weights");
    for (int j = 0; j < D; ++j)
        if (!std::isfinite(q_norm[j]) || !std::isfinite(k_norm[j]))
            return fail(ctx, QA_ERR_INVALID, "nonfinite norm weight in layer %d", layer);  // core.cpp:271
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    float* dst = ctx->norms + (size_t)layer * 2 * D;
    QA_CUDA(cudaMemcpyAsync(dst, q_norm, D * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    QA_CUDA(cudaMemcpyAsync(dst + D, k_norm, D * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    return QA_OK;
}

int qa_position(const qa_ctx* ctx, int seq, int* pos) {
    if (!ctx || !pos) return QA_ERR_INVALID;
    if (seq < 0 || seq >= ctx->cfg.max_seqs) return QA_ERR_INVALID;
    *pos = ctx->pos[seq];
    return QA_OK;
}

int qa_reset(qa_ctx* ctx, int seq) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, seq))) return st;
    ctx->pos[seq] = 0;
    std::fill(ctx->appended[seq].begin(), ctx->appended[seq].end(), 0);
    return QA_OK;
}

int qa_truncate(qa_ctx* ctx, int seq, int pos) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, seq))) return st;
    if (pos < 0 || pos > ctx->pos[seq])
        return fail(ctx, QA_ERR_STATE, "Rewind position out of range: %d not in [0,%d]", pos, ctx->pos[seq]);  // core.cpp:723
    ctx->pos[seq] = pos;
    for (int& a : ctx->appended[seq]) a = std::min(a, pos);
    return QA_OK;
}

int qa_commit(qa_ctx* ctx, int seq, int n) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, seq))) return st;
    if (n < 1) return fail(ctx, QA_ERR_INVALID, "commit count %d < 1", n);
    if (n > ctx->cfg.context - ctx->pos[seq]) return fail(ctx, QA_ERR_CAPACITY, "commit past context capacity");
    if ((st = check_appended(ctx, seq, 0, ctx->cfg.n_layers, ctx->pos[seq] + n))) return st;
    ctx->pos[seq] += n;
    return QA_OK;
}


int qa_append(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n,
              const float* q_pre, const float* k_pre, const float* v, float* q_out) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_rows(ctx, seq, layer, n_layers, pos0, n))) return st;
    if (!q_pre || !k_pre || !v || !q_out) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t qn = (size_t)n * ctx->hq * D, kn = (size_t)n * ctx->hkv * D;     // floats per layer
    IoCall c;
    c.in[0] = q_pre; c.in[1] = k_pre; c.in[2] = v; c.in_floats[0] = qn; c.in_floats[1] = kn; c.in_floats[2] = kn;
    c.out[0] = q_out; c.out_floats[0] = qn;
    st = run_call(ctx, seq, layer, n_layers, c, [&](int l0, int nl, const float* const* din, float* const* dout) {
        AppendArgs a{};
        a.q_pre = din[0]; a.k_pre = din[1]; a.v_pre = din[2]; a.q_out = dout[0];
        a.kv = ctx->kv; a.seq = seq; a.layer0 = l0; a.n_layers = nl; a.pos0 = pos0; a.n = n;
        a.hq = ctx->hq; a.hkv = ctx->hkv; a.norms = ctx->norms; a.cosines = ctx->cosines; a.sines = ctx->sines;
        a.eps = ctx->cfg.norm_eps;
        launch_kv_append(a, ctx->stream);
        return after_launch(ctx, seq, "kv_append");
    });
    if (st) return st;
    for (int l = layer; l < layer + n_layers; ++l) ctx->appended[seq][l] = pos0 + n;
    return QA_OK;
}

// The split-decode scratch is sized at creation for every plan a call can make (see
// decode_partial_floats_bound); a plan beyond it would be an internal error, refused here.
static int check_decode_scratch(qa_ctx* ctx, const DecodePlan& plan) {
    if (plan.partial_floats() > ctx->partial_floats || plan.units > ctx->max_units)
        return fail(ctx, QA_ERR_CAPACITY, "decode plan (%d units, %zu record floats) beyond the scratch made at creation",
                    plan.units, plan.partial_floats());
    return QA_OK;
}

// Prefill rows go to `gather` when given (full-head layout here and on the peers), else to out.
static int attend(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n, const float* q, float* out,
                  bool decode, const OutRows* gather = nullptr) {
    int st;
    if ((st = check_rows(ctx, seq, layer, n_layers, pos0, n))) return st;
    if (decode && n > QA_MAX_DECODE_ROWS)
        return fail(ctx, QA_ERR_INVALID, "decode takes at most %d rows, got %d", QA_MAX_DECODE_ROWS, n);
    if (!q || !out) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    if ((st = check_appended(ctx, seq, layer, n_layers, pos0 + n))) return st;
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t qn = (size_t)n * ctx->hq * D;
    IoCall c;
    c.in[0] = q; c.in_floats[0] = qn;
    c.out[0] = out; c.out_floats[0] = qn;
    c.inputs_read_once = !decode || decode_inputs_read_once(n_layers, n, ctx->hkv);
    return run_call(ctx, seq, layer, n_layers, c, [&](int l0, int nl, const float* const* din, float* const* dout) {
        int s2;
        if (decode) {
            int seqs[QA_MAX_DECODE_ROWS], pos[QA_MAX_DECODE_ROWS];
            for (int b = 0; b < n; ++b) { seqs[b] = seq; pos[b] = pos0 + b; }
            const DecodePlan plan = plan_attn_decode(nl, ctx->hkv, n, pos);
            if ((s2 = check_decode_scratch(ctx, plan))) return s2;
            launch_attn_decode_sm100(plan, ctx->kv, din[0], dout[0], l0, nl, n, seqs, pos, ctx->hq, ctx->hkv,
                                     ctx->partial, ctx->counters, ctx->error, ctx->stream);
        } else {
            RowsArgs r{};
            r.q = din[0]; r.out = dout[0]; r.kv = ctx->kv; r.seq = seq; r.layer0 = l0; r.n_layers = nl;
            r.pos0 = pos0; r.n = n; r.hq = ctx->hq; r.hkv = ctx->hkv; r.row_begin = 0; r.row_end = n;
            // rows below position TC_MIN_POSITION: FP32 CUDA cores; the rest: tcgen05 tensor cores
            const int tc_begin = std::min(n, std::max(0, TC_MIN_POSITION - pos0));
            OutRows o{};
            if (gather) o = *gather;
            else { o.out = dout[0]; o.heads = ctx->hq; }
            const bool both = tc_begin > 0 && tc_begin < n;
            if (both) {
                // the FP32 rows on the aux stream, submitted first, so their CTAs and the persistent
                // kernel's share the GPU (the tensor-core CTAs start on the SMs they leave free)
                QA_CUDA(cudaEventRecord(ctx->fork_ev, ctx->stream));
                QA_CUDA(cudaStreamWaitEvent(ctx->aux_stream, ctx->fork_ev, 0));
            }
            if (tc_begin > 0) {
                r.row_end = tc_begin;
                launch_attn_head_rows(r, o, both ? ctx->aux_stream : ctx->stream);
            }
            // beside a short persistent launch (one or two layers, as an engine's layer loop makes
            // them) the head-rows launch (one CTA per layer and KV head) keeps its SMs, so that it
            // runs alongside rather than after it; longer launches leave it their tail
            const int head_ctas = both && nl <= 2 ? nl * ctx->hkv : 0;
            const int lr = launch_attn_prefill_sm100(ctx->kv_map, din[0], o, seq, l0, nl, pos0, n, ctx->hq, ctx->hkv,
                                                     ctx->cfg.n_layers, tc_begin, ctx->prefill_tiles,
                                                     ctx->prefill_split, head_ctas <= NUM_SMS_B200 / 4 ? head_ctas : 0,
                                                     ctx->error, ctx->stream);
            if (lr == -1)
                return fail(ctx, QA_ERR_UNSUPPORTED, "tensor-core prefill kernel cannot launch (unexpected register allocation or shared-memory limit)");
            if (lr) return fail(ctx, QA_ERR_CUDA, "tensor-core prefill launch failed: %s", cudaGetErrorString(cudaGetLastError()));
            if (both) {
                QA_CUDA(cudaEventRecord(ctx->join_ev, ctx->aux_stream));
                QA_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->join_ev, 0));
            }
        }
        return after_launch(ctx, seq, decode ? "attn_decode" : "attn_prefill");
    });
}

int qa_attn_prefill(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n, const float* q, float* out) {
    if (!ctx) return QA_ERR_INVALID;
    return attend(ctx, seq, layer, n_layers, pos0, n, q, out, false);
}

int qa_attn_decode(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n, const float* q, float* out) {
    if (!ctx) return QA_ERR_INVALID;
    return attend(ctx, seq, layer, n_layers, pos0, n, q, out, true);
}

// ---- batched decode: one row for each of n sequences, each at its own position ----------------
static int check_batch(qa_ctx* ctx, const int* seqs, int n, int layer, int n_layers) {
    int st;
    if (!seqs) return fail(ctx, QA_ERR_INVALID, "null sequence list");
    if (n < 1 || n > QA_MAX_BATCH) return fail(ctx, QA_ERR_INVALID, "batch of %d sequences (1..%d)", n, QA_MAX_BATCH);
    if ((st = check_layers(ctx, layer, n_layers))) return st;
    for (int b = 0; b < n; ++b) {
        if ((st = check_seq(ctx, seqs[b]))) return st;
        for (int c = 0; c < b; ++c)
            if (seqs[c] == seqs[b]) return fail(ctx, QA_ERR_INVALID, "sequence %d listed twice", seqs[b]);
        if (ctx->pos[seqs[b]] >= ctx->cfg.context)
            return fail(ctx, QA_ERR_CAPACITY, "sequence %d is at context capacity", seqs[b]);
    }
    return QA_OK;
}

int qa_append_batch(qa_ctx* ctx, const int* seqs, int n, int layer, int n_layers, const float* q_pre,
                    const float* k_pre, const float* v, float* q_out) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_batch(ctx, seqs, n, layer, n_layers))) return st;
    if (!q_pre || !k_pre || !v || !q_out) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t qn = (size_t)n * ctx->hq * D, kn = (size_t)n * ctx->hkv * D;
    IoCall c;
    c.in[0] = q_pre; c.in[1] = k_pre; c.in[2] = v; c.in_floats[0] = qn; c.in_floats[1] = kn; c.in_floats[2] = kn;
    c.out[0] = q_out; c.out_floats[0] = qn;
    st = run_call(ctx, -1, layer, n_layers, c, [&](int l0, int nl, const float* const* din, float* const* dout) {
        AppendArgs a{};
        a.q_pre = din[0]; a.k_pre = din[1]; a.v_pre = din[2]; a.q_out = dout[0];
        a.kv = ctx->kv; a.seq = seqs[0]; a.layer0 = l0; a.n_layers = nl; a.pos0 = 0; a.n = n;
        a.hq = ctx->hq; a.hkv = ctx->hkv; a.norms = ctx->norms; a.cosines = ctx->cosines; a.sines = ctx->sines;
        a.eps = ctx->cfg.norm_eps;
        a.rows.batched = 1;
        for (int b = 0; b < n; ++b) { a.rows.seq[b] = seqs[b]; a.rows.pos[b] = ctx->pos[seqs[b]]; }
        launch_kv_append(a, ctx->stream);
        return after_launch(ctx, -1, "kv_append_batch");
    });
    if (st) return st;
    for (int b = 0; b < n; ++b)
        for (int l = layer; l < layer + n_layers; ++l) ctx->appended[seqs[b]][l] = ctx->pos[seqs[b]] + 1;
    return QA_OK;
}

int qa_attn_decode_batch(qa_ctx* ctx, const int* seqs, int n, int layer, int n_layers, const float* q, float* out) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_batch(ctx, seqs, n, layer, n_layers))) return st;
    if (!q || !out) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    int pos[QA_MAX_BATCH];
    for (int b = 0; b < n; ++b) {
        pos[b] = ctx->pos[seqs[b]];
        if ((st = check_appended(ctx, seqs[b], layer, n_layers, pos[b] + 1))) return st;
    }
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t qn = (size_t)n * ctx->hq * D;
    IoCall c;
    c.in[0] = q; c.in_floats[0] = qn;
    c.out[0] = out; c.out_floats[0] = qn;
    c.inputs_read_once = decode_inputs_read_once(n_layers, n, ctx->hkv);
    return run_call(ctx, -1, layer, n_layers, c, [&](int l0, int nl, const float* const* din, float* const* dout) {
        const DecodePlan plan = plan_attn_decode(nl, ctx->hkv, n, pos);
        int s2;
        if ((s2 = check_decode_scratch(ctx, plan))) return s2;
        launch_attn_decode_sm100(plan, ctx->kv, din[0], dout[0], l0, nl, n, seqs, pos, ctx->hq, ctx->hkv, ctx->partial,
                                 ctx->counters, ctx->error, ctx->stream);
        return after_launch(ctx, -1, "attn_decode_batch");
    });
}

// ---- fused decode step: append of one new row per sequence + decode attention, one launch ----
static int decode_step(qa_ctx* ctx, const int* seqs, const int* pos, int n, int layer, int n_layers,
                       const float* q_pre, const float* k_pre, const float* v, float* q_out, float* out,
                       const GatherArgs* gather = nullptr) {
    int st;
    if (!q_pre || !k_pre || !v || !out) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t qn = (size_t)n * ctx->hq * D, kn = (size_t)n * ctx->hkv * D;
    IoCall c;
    c.in[0] = q_pre; c.in[1] = k_pre; c.in[2] = v; c.in_floats[0] = qn; c.in_floats[1] = kn; c.in_floats[2] = kn;
    c.out[0] = out; c.out_floats[0] = qn;
    c.out[1] = q_out; c.out_floats[1] = qn;
    c.inputs_read_once = decode_inputs_read_once(n_layers, n, ctx->hkv);
    bool fused = false;
    const int seq1 = n == 1 ? seqs[0] : -1;
    st = run_call(ctx, seq1, layer, n_layers, c, [&](int l0, int nl, const float* const* din, float* const* dout) {
        StepInputs in{};
        in.q_pre = din[0]; in.k_pre = din[1]; in.v_pre = din[2]; in.q_out = dout[1];
        in.norms = ctx->norms; in.cosines = ctx->cosines; in.sines = ctx->sines; in.eps = ctx->cfg.norm_eps;
        // overlap with the previous step only right after a fused step of this context on this stream
        // (or the gather wait that followed one)
        in.pdl = ctx->step_overlap && ctx->last_fused_step && !ctx->cfg.io_host ? 1 : 0;
        const DecodePlan plan = plan_attn_decode(nl, ctx->hkv, n, pos);
        int s2;
        if ((s2 = check_decode_scratch(ctx, plan))) return s2;
        if (plan.max_units_per_cta <= FUSED_MAX_UNITS) {
            launch_attn_decode_sm100(plan, ctx->kv, nullptr, dout[0], l0, nl, n, seqs, pos, ctx->hq, ctx->hkv,
                                     ctx->partial, ctx->counters, ctx->error, ctx->stream, &in, gather);
            fused = true;
        } else {
            // Short contexts or many sequences per CTA range: the same results as append + decode,
            // run as those two launches (the normalised query rows go to q_out or to staging).
            float* qrows = in.q_out ? in.q_out : ctx->staging;
            AppendArgs ap{};
            ap.q_pre = in.q_pre; ap.k_pre = in.k_pre; ap.v_pre = in.v_pre; ap.q_out = qrows;
            ap.kv = ctx->kv; ap.seq = seqs[0]; ap.layer0 = l0; ap.n_layers = nl; ap.pos0 = 0; ap.n = n;
            ap.hq = ctx->hq; ap.hkv = ctx->hkv; ap.norms = ctx->norms; ap.cosines = ctx->cosines;
            ap.sines = ctx->sines; ap.eps = ctx->cfg.norm_eps;
            ap.rows.batched = 1;
            for (int b = 0; b < n; ++b) { ap.rows.seq[b] = seqs[b]; ap.rows.pos[b] = pos[b]; }
            launch_kv_append(ap, ctx->stream);
            launch_attn_decode_sm100(plan, ctx->kv, qrows, dout[0], l0, nl, n, seqs, pos, ctx->hq, ctx->hkv,
                                     ctx->partial, ctx->counters, ctx->error, ctx->stream, nullptr, gather);
            fused = false;
        }
        return after_launch(ctx, seq1, "attn_decode_step");
    });
    if (st) return st;
    ctx->last_fused_step = fused;
    for (int b = 0; b < n; ++b)
        for (int l = layer; l < layer + n_layers; ++l) ctx->appended[seqs[b]][l] = pos[b] + 1;
    return QA_OK;
}

int qa_decode_step(qa_ctx* ctx, int seq, int layer, int n_layers, int pos, const float* q_pre, const float* k_pre,
                   const float* v, float* q_out, float* out) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_rows(ctx, seq, layer, n_layers, pos, 1))) return st;
    return decode_step(ctx, &seq, &pos, 1, layer, n_layers, q_pre, k_pre, v, q_out, out);
}

int qa_decode_step_batch(qa_ctx* ctx, const int* seqs, int n, int layer, int n_layers, const float* q_pre,
                         const float* k_pre, const float* v, float* q_out, float* out) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_batch(ctx, seqs, n, layer, n_layers))) return st;
    int pos[QA_MAX_BATCH];
    for (int b = 0; b < n; ++b) pos[b] = ctx->pos[seqs[b]];
    return decode_step(ctx, seqs, pos, n, layer, n_layers, q_pre, k_pre, v, q_out, out);
}

int qa_commit_batch(qa_ctx* ctx, const int* seqs, int n) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_batch(ctx, seqs, n, 0, ctx->cfg.n_layers))) return st;
    for (int b = 0; b < n; ++b)
        if ((st = check_appended(ctx, seqs[b], 0, ctx->cfg.n_layers, ctx->pos[seqs[b]] + 1))) return st;
    for (int b = 0; b < n; ++b) ctx->pos[seqs[b]] += 1;
    return QA_OK;
}

int qa_copy_prefix(qa_ctx* ctx, int src, int dst, int ntok) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, src)) || (st = check_seq(ctx, dst))) return st;
    if (src == dst) return fail(ctx, QA_ERR_INVALID, "prefix copy onto itself");
    if (ntok < QA_PREFIX_CHUNK || ntok % QA_PREFIX_CHUNK)
        return fail(ctx, QA_ERR_INVALID, "prefix length %d is not a positive multiple of %d", ntok, QA_PREFIX_CHUNK);
    if (ntok > ctx->pos[src]) return fail(ctx, QA_ERR_STATE, "source holds %d committed rows, copy wants %d", ctx->pos[src], ntok);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    launch_kv_copy(ctx->kv, src, dst, ntok, ctx->stream);
    if ((st = after_launch(ctx, dst, "kv_copy"))) return st;
    ctx->pos[dst] = ntok;
    std::fill(ctx->appended[dst].begin(), ctx->appended[dst].end(), ntok);
    return QA_OK;
}

static size_t block_bytes(const qa_ctx* ctx) {
    return (size_t)ctx->cfg.n_layers * 2 * ctx->hkv * QA_PREFIX_CHUNK * D * sizeof(__half);
}

int qa_block_pool(qa_ctx* ctx, int n_blocks) {
    if (!ctx) return QA_ERR_INVALID;
    if (n_blocks < 0) return fail(ctx, QA_ERR_INVALID, "negative block count %d", n_blocks);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    QA_CUDA(cudaStreamSynchronize(ctx->stream));      // no queued copy still uses the old pool
    cudaFree(ctx->pool);
    ctx->pool = nullptr;
    ctx->pool_chunk.clear();
    if (n_blocks == 0) return QA_OK;
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)n_blocks * block_bytes(ctx)) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, QA_ERR_CAPACITY, "no device memory for %d prefix blocks of %zu bytes", n_blocks,
                    block_bytes(ctx));
    }
    ctx->pool = static_cast<__half*>(p);
    ctx->pool_chunk.assign(n_blocks, -1);
    return QA_OK;
}

static int check_block(qa_ctx* ctx, int seq, int chunk, int block) {
    int st;
    if ((st = check_seq(ctx, seq))) return st;
    if (block < 0 || block >= (int)ctx->pool_chunk.size())
        return fail(ctx, QA_ERR_INVALID, "block %d outside the pool of %zu", block, ctx->pool_chunk.size());
    if (chunk < 0 || (size_t)(chunk + 1) * QA_PREFIX_CHUNK > (size_t)ctx->cfg.context)
        return fail(ctx, QA_ERR_INVALID, "chunk %d outside the context", chunk);
    return QA_OK;
}

int qa_block_save(qa_ctx* ctx, int seq, int chunk, int block) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_block(ctx, seq, chunk, block))) return st;
    const int end = (chunk + 1) * QA_PREFIX_CHUNK;
    if (ctx->pos[seq] < end)
        return fail(ctx, QA_ERR_STATE, "sequence %d holds %d committed rows, chunk %d needs %d", seq, ctx->pos[seq], chunk, end);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    launch_pack_kv(ctx->kv, seq, chunk * QA_PREFIX_CHUNK, QA_PREFIX_CHUNK,
                   reinterpret_cast<char*>(ctx->pool) + (size_t)block * block_bytes(ctx), false, ctx->stream);
    if ((st = after_launch(ctx, -1, "block_save"))) return st;
    ctx->pool_chunk[block] = chunk;
    return QA_OK;
}

int qa_block_load(qa_ctx* ctx, int seq, int chunk, int block) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_block(ctx, seq, chunk, block))) return st;
    if (ctx->pool_chunk[block] != chunk)
        return fail(ctx, QA_ERR_STATE, "block %d holds chunk %d, not chunk %d (keys carry their positions)", block,
                    ctx->pool_chunk[block], chunk);
    if (ctx->pos[seq] != chunk * QA_PREFIX_CHUNK)
        return fail(ctx, QA_ERR_STATE, "sequence %d is at position %d, chunk %d starts at %d", seq, ctx->pos[seq], chunk,
                    chunk * QA_PREFIX_CHUNK);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    launch_pack_kv(ctx->kv, seq, chunk * QA_PREFIX_CHUNK, QA_PREFIX_CHUNK,
                   reinterpret_cast<char*>(ctx->pool) + (size_t)block * block_bytes(ctx), true, ctx->stream);
    if ((st = after_launch(ctx, seq, "block_load"))) return st;
    const int end = (chunk + 1) * QA_PREFIX_CHUNK;
    ctx->pos[seq] = end;
    std::fill(ctx->appended[seq].begin(), ctx->appended[seq].end(), end);
    return QA_OK;
}

int qa_read_kv(qa_ctx* ctx, int seq, int layer, int kv, int head, int pos0, int n, uint16_t* dst) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, seq)) || (st = check_layers(ctx, layer, 1))) return st;
    if (kv < 0 || kv > 1 || head < 0 || head >= ctx->hkv) return fail(ctx, QA_ERR_INVALID, "bad kv/head selector");
    if (pos0 < 0 || n < 0 || pos0 + n > ctx->cfg.context) return fail(ctx, QA_ERR_INVALID, "rows outside the context");
    if (!dst && n) return fail(ctx, QA_ERR_INVALID, "null destination");
    if (!n) return QA_OK;
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const __half* src = ctx->kv.plane(seq, layer, kv, head) + (size_t)pos0 * D;
    QA_CUDA(cudaMemcpyAsync(dst, src, (size_t)n * D * sizeof(__half), cudaMemcpyDeviceToHost, ctx->stream));
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    return QA_OK;
}

int qa_kv_pointer(qa_ctx* ctx, int seq, int layer, int kv, int head, void** ptr) {
    if (!ctx || !ptr) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, seq)) || (st = check_layers(ctx, layer, 1))) return st;
    if (kv < 0 || kv > 1 || head < 0 || head >= ctx->hkv) return fail(ctx, QA_ERR_INVALID, "bad kv/head selector");
    *ptr = ctx->kv.plane(seq, layer, kv, head);
    return QA_OK;
}

int qa_kv_slot_bytes(const qa_ctx* ctx, size_t* bytes) {
    if (!ctx || !bytes) return QA_ERR_INVALID;
    *bytes = ctx->kv.slot_elems() * sizeof(__half);
    return QA_OK;
}

}  // extern "C"

// ---- projections: decode GEMVs (project.cu) and batched prompt rows (project_mma.cu) -------------
namespace {
int project_call(qa_ctx* ctx, int n_mats, const uint16_t* const* w, const int* rows, int cols, const float* x,
                 int batch, float* const* y, bool gemm) {
    if (!ctx) return QA_ERR_INVALID;
    if (n_mats < 1 || n_mats > MAX_PROJECT_MATS || !w || !rows || !y)
        return fail(ctx, QA_ERR_INVALID, "%d matrices (1..%d) or null arrays", n_mats, MAX_PROJECT_MATS);
    if (cols < 8 || cols % 8) return fail(ctx, QA_ERR_INVALID, "columns %d: a positive multiple of 8", cols);
    if (batch < 1 || (!gemm && batch > QA_MAX_BATCH))
        return fail(ctx, QA_ERR_INVALID, "batch %d outside 1..%d", batch, gemm ? INT32_MAX : QA_MAX_BATCH);
    if (!x) return fail(ctx, QA_ERR_INVALID, "null input");
    if (!ctx->cfg.io_host && (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(ctx, QA_ERR_INVALID, "input rows must be 16-byte aligned");
    size_t out_floats = 0;
    ProjectArgs a{};
    a.n_mats = n_mats; a.cols = cols; a.batch = batch;
    for (int m = 0; m < n_mats; ++m) {
        if (!w[m] || !y[m] || rows[m] < 1) return fail(ctx, QA_ERR_INVALID, "matrix %d: null pointer or %d rows", m, rows[m]);
        if (reinterpret_cast<uintptr_t>(w[m]) & 15) return fail(ctx, QA_ERR_INVALID, "matrix %d is not 16-byte aligned", m);
        a.w[m] = reinterpret_cast<const __half*>(w[m]);
        a.rows[m] = rows[m];
        out_floats += (size_t)rows[m] * batch;
    }
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    // the tensor-core path where the shape allows it; otherwise the CUDA-core kernels, whose
    // eight-lane sums are one of the FP32 summation orders the batched form admits
    auto launch = [&]() {
        if (!gemm || launch_project_gemm(a, ctx->proj_scratch, ctx->error, ctx->stream) < 0) launch_project(a, ctx->stream);
    };
    const size_t in_floats = (size_t)batch * cols;
    if (!ctx->cfg.io_host) {
        a.x = x;
        for (int m = 0; m < n_mats; ++m) a.y[m] = y[m];
        launch();
        return after_launch(ctx, -1, "project");
    }
    // host buffers: x into the staging inputs, every y from the staging outputs (one copy each
    // way through the pinned mirror when they fit IO_PACK_BYTES)
    if (in_floats > ctx->io_in_floats || out_floats > ctx->io_out_floats)
        return fail(ctx, QA_ERR_CAPACITY, "projection of %zu outputs beyond the host-buffer staging", out_floats);
    float* d_out = ctx->staging;
    float* d_in = ctx->staging + ctx->io_out_floats;
    int* h_err = reinterpret_cast<int*>(ctx->io_pin);
    float* h_out = reinterpret_cast<float*>(ctx->io_pin + ERR_BLOCK_BYTES);
    float* h_in = h_out + IO_PACK_BYTES / sizeof(float);
    const bool pack_in = in_floats * sizeof(float) <= IO_PACK_BYTES, pack_out = out_floats * sizeof(float) <= IO_PACK_BYTES;
    if (pack_in) {
        std::memcpy(h_in, x, in_floats * sizeof(float));
        QA_CUDA(cudaMemcpyAsync(d_in, h_in, in_floats * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    } else {
        QA_CUDA(cudaMemcpyAsync(d_in, x, in_floats * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    }
    a.x = d_in;
    size_t off = 0;
    for (int m = 0; m < n_mats; ++m) { a.y[m] = d_out + off; off += (size_t)rows[m] * batch; }
    launch();
    int st;
    if ((st = after_launch(ctx, -1, "project"))) return st;
    if (pack_out) {
        QA_CUDA(cudaMemcpyAsync(h_err, ctx->io_dev, ERR_BLOCK_BYTES + out_floats * sizeof(float), cudaMemcpyDeviceToHost,
                                ctx->stream));
    } else {
        QA_CUDA(cudaMemcpyAsync(h_err, ctx->io_dev, ERR_BLOCK_BYTES, cudaMemcpyDeviceToHost, ctx->stream));
        for (int m = 0; m < n_mats; ++m)
            QA_CUDA(cudaMemcpyAsync(y[m], a.y[m], (size_t)rows[m] * batch * sizeof(float), cudaMemcpyDeviceToHost,
                                    ctx->stream));
    }
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    if (pack_out) {
        off = 0;
        for (int m = 0; m < n_mats; ++m) {
            std::memcpy(y[m], h_out + off, (size_t)rows[m] * batch * sizeof(float));
            off += (size_t)rows[m] * batch;
        }
    }
    if (const int code = h_err[ERR_CODE]) {
        QA_CUDA(cudaMemsetAsync(ctx->error + ERR_CODE, 0, sizeof(int), ctx->stream));
        QA_CUDA(cudaStreamSynchronize(ctx->stream));
        return fail(ctx, QA_ERR_TIMEOUT, "a device-side wait expired (code %d); results of the last calls are invalid", code);
    }
    return QA_OK;
}

}  // namespace

extern "C" {

int qa_project_group(qa_ctx* ctx, int n_mats, const uint16_t* const* w, const int* rows, int cols, const float* x,
                     int batch, float* const* y) {
    return project_call(ctx, n_mats, w, rows, cols, x, batch, y, false);
}
int qa_project(qa_ctx* ctx, const uint16_t* w, int rows, int cols, const float* x, int batch, float* y) {
    return project_call(ctx, 1, &w, &rows, cols, x, batch, &y, false);
}
int qa_project_group_gemm(qa_ctx* ctx, int n_mats, const uint16_t* const* w, const int* rows, int cols, const float* x,
                          int batch, float* const* y) {
    return project_call(ctx, n_mats, w, rows, cols, x, batch, y, true);
}
int qa_project_gemm(qa_ctx* ctx, const uint16_t* w, int rows, int cols, const float* x, int batch, float* y) {
    return project_call(ctx, 1, &w, &rows, cols, x, batch, &y, true);
}

int qa_synth_fill(float* dst, uint64_t seed, int kind, int layer0, int n_layers, int pos0, int n, int head0,
                  int heads, float mean, float stdev, void* stream) {
    if (!dst || kind < 0 || kind > 4 || layer0 < 0 || layer0 + n_layers > 64 || n_layers < 1 || pos0 < 0 || n < 1 ||
        pos0 + n > 8192 || head0 < 0 || heads < 1 || head0 + heads > 64)
        return QA_ERR_INVALID;
    launch_synth(dst, seed, kind, layer0, n_layers, pos0, n, head0, heads, mean, stdev, static_cast<cudaStream_t>(stream));
    return cudaGetLastError() == cudaSuccess ? QA_OK : QA_ERR_CUDA;
}

}  // extern "C"

// ---- multi-GPU ---------------------------------------------------------------------------------
namespace {
int grow(qa_ctx* ctx, void** buf, size_t& have, size_t need) {
    if (need <= have) return QA_OK;
    QA_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->comm_stream) QA_CUDA(cudaStreamSynchronize(ctx->comm_stream));
    cudaFree(*buf);
    *buf = nullptr; have = 0;
    QA_CUDA(cudaMalloc(buf, need));
    have = need;
    return QA_OK;
}
}  // namespace

// Exchanges CUDA IPC handles of `block` (this rank's allocation of `bytes`, or null when it
// could not be made) over the context's communicator, opens the peers', then agrees: *ok is
// set only if every rank mapped every other rank's block; *min_bytes is the smallest block
// (every store into a peer's block stays below it); with same_size, blocks of different sizes
// count as a failure. Collective. CUDA IPC failures are not errors; on disagreement the
// mappings are closed.
int ipc_exchange(qa_ctx* ctx, char* block, size_t bytes, bool same_size, char* (&base)[MAX_RANKS], bool* ok_out,
                 size_t* min_bytes) {
    const int R = ctx->nranks;
    struct Slot { cudaIpcMemHandle_t h; unsigned long long bytes; int ok; int pad[1]; };
    Slot mine{};
    mine.bytes = bytes;
    mine.ok = block && cudaIpcGetMemHandle(&mine.h, block) == cudaSuccess;
    cudaGetLastError();
    // exchange handles (one all-gather), open the peers', then agree (a second all-gather)
    Slot* dslots = nullptr;
    QA_CUDA(cudaMalloc(&dslots, sizeof(Slot) * R));
    std::vector<Slot> slots(R);
    std::string err;
    int st = QA_OK;
    bool agreed = false;
    do {
        if (cudaMemcpy(dslots + ctx->rank, &mine, sizeof(Slot), cudaMemcpyHostToDevice) != cudaSuccess) { st = QA_ERR_CUDA; break; }
        if ((st = nccl_all_gather_bytes(ctx->comm, dslots + ctx->rank, dslots, sizeof(Slot), ctx->comm_stream, err))) break;
        if (cudaStreamSynchronize(ctx->comm_stream) != cudaSuccess) { st = QA_ERR_CUDA; break; }
        if (cudaMemcpy(slots.data(), dslots, sizeof(Slot) * R, cudaMemcpyDeviceToHost) != cudaSuccess) { st = QA_ERR_CUDA; break; }
        int ok = 1;
        *min_bytes = bytes;
        for (int r = 0; r < R; ++r) {
            ok &= slots[r].ok;
            *min_bytes = std::min<size_t>(*min_bytes, slots[r].bytes);
            if (same_size && slots[r].bytes != bytes) ok = 0;
        }
        if (ok) {
            base[ctx->rank] = block;
            for (int r = 0; r < R && ok; ++r) {
                if (r == ctx->rank) continue;
                void* p = nullptr;
                if (cudaIpcOpenMemHandle(&p, slots[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) { ok = 0; cudaGetLastError(); }
                else base[r] = static_cast<char*>(p);
            }
        }
        mine.ok = ok;
        if (cudaMemcpy(dslots + ctx->rank, &mine, sizeof(Slot), cudaMemcpyHostToDevice) != cudaSuccess) { st = QA_ERR_CUDA; break; }
        if ((st = nccl_all_gather_bytes(ctx->comm, dslots + ctx->rank, dslots, sizeof(Slot), ctx->comm_stream, err))) break;
        if (cudaStreamSynchronize(ctx->comm_stream) != cudaSuccess) { st = QA_ERR_CUDA; break; }
        if (cudaMemcpy(slots.data(), dslots, sizeof(Slot) * R, cudaMemcpyDeviceToHost) != cudaSuccess) { st = QA_ERR_CUDA; break; }
        ok = 1;
        for (int r = 0; r < R; ++r) ok &= slots[r].ok;
        agreed = ok != 0;
    } while (false);
    cudaFree(dslots);
    if (!agreed) close_mappings(base, block);
    *ok_out = agreed;
    if (st) return fail(ctx, st, "peer memory set-up: %s", err.empty() ? "CUDA error" : err.c_str());
    return QA_OK;
}

// Maps every rank's decode-gather allocation into every other rank (collective over the
// context's communicator). The peer path is used only if every rank succeeded; otherwise the
// gathering decode step falls back to the NCCL all-gather.
int peer_setup(qa_ctx* ctx) {
    const int R = ctx->nranks;
    if (R < 2 || R > MAX_RANKS) return QA_OK;
    ctx->landing_bytes = ((size_t)ctx->cfg.n_layers * ctx->hq * R * D * sizeof(float) + 255) & ~size_t(255);
    ctx->flags_off = 2 * ctx->landing_bytes;
    const size_t total = ctx->flags_off + 256;
    bool local_ok = cudaMalloc(&ctx->peer_block, total) == cudaSuccess &&
                    cudaMalloc(&ctx->gather_done, sizeof(unsigned)) == cudaSuccess &&
                    cudaMemset(ctx->peer_block, 0, total) == cudaSuccess &&
                    cudaMemset(ctx->gather_done, 0, sizeof(unsigned)) == cudaSuccess;
    cudaGetLastError();
    // the flag words sit at an offset derived from the size: every rank's block must match
    const int st = ipc_exchange(ctx, local_ok ? ctx->peer_block : nullptr, total, true, ctx->peer_base,
                                &ctx->peer_ok, &ctx->peer_min_bytes);
    if (!ctx->peer_ok) peer_release(ctx);
    return st;
}

// The prefill landing buffer, mapped on the first gathering prefill (collective).
int prefill_peer_setup(qa_ctx* ctx) {
    ctx->pf_tried = true;
    if (!ctx->peer_ok) return QA_OK;
    const size_t bytes = (size_t)ctx->cfg.n_layers * ctx->cfg.context * ctx->hq * ctx->nranks * D * sizeof(float);
    bool local_ok = cudaMalloc(&ctx->pf_block, bytes) == cudaSuccess;
    if (!local_ok) ctx->pf_block = nullptr;
    cudaGetLastError();
    const int st = ipc_exchange(ctx, ctx->pf_block, bytes, false, ctx->pf_base, &ctx->pf_ok, &ctx->pf_min_bytes);
    if (!ctx->pf_ok) { cudaFree(ctx->pf_block); ctx->pf_block = nullptr; }
    return st;
}

// NCCL runs on the context's own communication stream: it waits for the work already on the
// context stream, and the context stream waits for it (any stream handle works, including
// the legacy default stream).
int comm_enter(qa_ctx* ctx) {
    QA_CUDA(cudaEventRecord(ctx->comm_ev[0], ctx->stream));
    QA_CUDA(cudaStreamWaitEvent(ctx->comm_stream, ctx->comm_ev[0], 0));
    return QA_OK;
}
int comm_leave(qa_ctx* ctx) {
    QA_CUDA(cudaEventRecord(ctx->comm_ev[1], ctx->comm_stream));
    QA_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->comm_ev[1], 0));
    return QA_OK;
}

extern "C" {

int qa_comm_unique_id(char id[128]) {
    if (!id) return QA_ERR_INVALID;
    return nccl_unique_id(id);
}

int qa_comm_init(qa_ctx* ctx, int nranks, int rank, const char id[128]) {
    if (!ctx || !id) return QA_ERR_INVALID;
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(ctx, QA_ERR_INVALID, "rank %d of %d", rank, nranks);
    if (ctx->comm) return fail(ctx, QA_ERR_STATE, "communicator already initialised");
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    if (!ctx->comm_stream) {
        QA_CUDA(cudaStreamCreateWithFlags(&ctx->comm_stream, cudaStreamNonBlocking));
        QA_CUDA(cudaEventCreateWithFlags(&ctx->comm_ev[0], cudaEventDisableTiming));
        QA_CUDA(cudaEventCreateWithFlags(&ctx->comm_ev[1], cudaEventDisableTiming));
        for (int b = 0; b < 2; ++b) {
            QA_CUDA(cudaEventCreateWithFlags(&ctx->kv_comm_done[b], cudaEventDisableTiming));
            QA_CUDA(cudaEventCreateWithFlags(&ctx->kv_unpacked[b], cudaEventDisableTiming));
        }
        QA_CUDA(cudaEventCreateWithFlags(&ctx->kv_packed, cudaEventDisableTiming));
    }
    std::string err;
    const int st = nccl_comm_init(&ctx->comm, nranks, rank, id, err);
    if (st) return fail(ctx, st, "ncclCommInitRank: %s", err.c_str());
    ctx->nranks = nranks; ctx->rank = rank;
    return peer_setup(ctx);
}

int qa_set_step_overlap(qa_ctx* ctx, int enable) {
    if (!ctx) return QA_ERR_INVALID;
    ctx->step_overlap = enable != 0;
    ctx->last_fused_step = false;
    return QA_OK;
}

int qa_comm_info(const qa_ctx* ctx, int* nranks, int* rank, int* peer_mapped) {
    if (!ctx || !nranks || !rank || !peer_mapped) return QA_ERR_INVALID;
    *nranks = ctx->nranks; *rank = ctx->rank; *peer_mapped = ctx->peer_ok ? 1 : 0;
    return QA_OK;
}

int qa_comm_destroy(qa_ctx* ctx) {
    if (!ctx) return QA_ERR_INVALID;
    if (ctx->comm) {
        cudaSetDevice(ctx->cfg.device);
        cudaStreamSynchronize(ctx->stream);
        if (ctx->comm_stream) cudaStreamSynchronize(ctx->comm_stream);
        peer_release(ctx);
        nccl_comm_destroy(ctx->comm);
        ctx->comm = nullptr;
    }
    ctx->nranks = 1; ctx->rank = 0;
    return QA_OK;
}

static int gather_heads(qa_ctx* ctx, int n_layers, int n, const float* local, float* full, bool async) {
    if (!ctx) return QA_ERR_INVALID;
    if (!ctx->comm) return fail(ctx, QA_ERR_STATE, "no communicator (qa_comm_init)");
    if (ctx->cfg.io_host) return fail(ctx, QA_ERR_UNSUPPORTED, "qa_gather_heads takes device pointers");
    if (!local || !full) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    if (n_layers < 1 || n < 1 || n_layers > ctx->cfg.n_layers || n > ctx->cfg.context)
        return fail(ctx, QA_ERR_INVALID, "bad shape %d x %d", n_layers, n);
    if (ctx->cfg.kv_head_begin != ctx->rank * ctx->hkv || ctx->nranks * ctx->hkv != ctx->cfg.n_kv_heads)
        return fail(ctx, QA_ERR_STATE, "rank %d holds KV heads [%d,%d): not the head shard the gather expects",
                    ctx->rank, ctx->cfg.kv_head_begin, ctx->cfg.kv_head_begin + ctx->hkv);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t count = (size_t)n_layers * n * ctx->hq * D;
    int st;
    {
        void* buf = ctx->gather_buf;
        size_t have = ctx->gather_floats * sizeof(float);
        if ((st = grow(ctx, &buf, have, count * ctx->nranks * sizeof(float)))) return st;
        ctx->gather_buf = static_cast<float*>(buf);
        ctx->gather_floats = have / sizeof(float);
    }
    std::string err;
    if ((st = comm_enter(ctx))) return st;
    if ((st = nccl_all_gather_f32(ctx->comm, local, ctx->gather_buf, count, ctx->comm_stream, err)))
        return fail(ctx, st, "ncclAllGather: %s", err.c_str());
    if (async) {
        // the permute stays on the communication stream; the context stream moves on
        launch_permute_heads(ctx->gather_buf, full, ctx->nranks, n_layers, n, ctx->hq, ctx->comm_stream);
        return after_launch(ctx, -1, "permute_heads");
    }
    if ((st = comm_leave(ctx))) return st;
    launch_permute_heads(ctx->gather_buf, full, ctx->nranks, n_layers, n, ctx->hq, ctx->stream);
    return after_launch(ctx, -1, "permute_heads");
}

int qa_gather_heads(qa_ctx* ctx, int n_layers, int n, const float* local, float* full) {
    return gather_heads(ctx, n_layers, n, local, full, false);
}

int qa_gather_heads_async(qa_ctx* ctx, int n_layers, int n, const float* local, float* full) {
    return gather_heads(ctx, n_layers, n, local, full, true);
}

int qa_attn_prefill_gather(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n, const float* q,
                           float* full) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_rows(ctx, seq, layer, n_layers, pos0, n))) return st;
    if (!ctx->comm) return fail(ctx, QA_ERR_STATE, "no communicator (qa_comm_init)");
    if (ctx->cfg.io_host) return fail(ctx, QA_ERR_UNSUPPORTED, "qa_attn_prefill_gather takes device pointers");
    if (!q || !full) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    if ((st = check_appended(ctx, seq, layer, n_layers, pos0 + n))) return st;
    if (ctx->cfg.kv_head_begin != ctx->rank * ctx->hkv || ctx->nranks * ctx->hkv != ctx->cfg.n_kv_heads)
        return fail(ctx, QA_ERR_STATE, "rank %d holds KV heads [%d,%d): not the head shard the gather expects",
                    ctx->rank, ctx->cfg.kv_head_begin, ctx->cfg.kv_head_begin + ctx->hkv);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    if (!ctx->pf_tried && (st = prefill_peer_setup(ctx))) return st;     // collective, first call only
    if (!ctx->pf_ok) {
        // no peer mapping: local prefill, then the NCCL all-gather
        const size_t bytes = (size_t)n_layers * n * ctx->hq * D * sizeof(float);
        void* buf = ctx->pf_local;
        if ((st = grow(ctx, &buf, ctx->pf_local_bytes, bytes))) return st;
        ctx->pf_local = static_cast<float*>(buf);
        if ((st = attend(ctx, seq, layer, n_layers, pos0, n, q, ctx->pf_local, false))) return st;
        return qa_gather_heads(ctx, n_layers, n, ctx->pf_local, full);
    }
    if ((size_t)n_layers * n * ctx->hq * ctx->nranks * D * sizeof(float) > ctx->pf_min_bytes)
        return fail(ctx, QA_ERR_INVALID, "%d x %d rows exceed the smallest rank's landing buffer", n_layers, n);
    const unsigned call = ++ctx->pf_call;
    unsigned* flags[MAX_RANKS] = {};
    OutRows o{};
    o.out = full; o.heads = ctx->hq * ctx->nranks; o.head0 = ctx->rank * ctx->hq;
    for (int r = 0; r < ctx->nranks; ++r) {
        flags[r] = reinterpret_cast<unsigned*>(ctx->peer_base[r] + ctx->flags_off);
        if (r != ctx->rank) o.peers[o.n_peers++] = reinterpret_cast<float*>(ctx->pf_base[r]);
    }
    launch_prefill_gate(flags, ctx->nranks, ctx->rank, call, ctx->error, ctx->stream);
    if ((st = after_launch(ctx, -1, "prefill_gate"))) return st;
    if ((st = attend(ctx, seq, layer, n_layers, pos0, n, q, full, false, &o))) return st;
    launch_prefill_signal(flags, ctx->nranks, ctx->rank, call, ctx->stream);
    if ((st = after_launch(ctx, -1, "prefill_signal"))) return st;
    launch_prefill_wait_copy(flags[ctx->rank], ctx->nranks, ctx->rank, call, reinterpret_cast<const float*>(ctx->pf_block),
                             full, n_layers, n, ctx->hq, ctx->error, ctx->stream);
    return after_launch(ctx, -1, "prefill_wait_copy");
}

int qa_decode_step_gather(qa_ctx* ctx, int seq, int layer, int n_layers, int pos, const float* q_pre,
                          const float* k_pre, const float* v, float* q_out, float* full) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_rows(ctx, seq, layer, n_layers, pos, 1))) return st;
    if (!ctx->comm) return fail(ctx, QA_ERR_STATE, "no communicator (qa_comm_init)");
    if (ctx->cfg.io_host) return fail(ctx, QA_ERR_UNSUPPORTED, "qa_decode_step_gather takes device pointers");
    if (!q_pre || !k_pre || !v || !full) return fail(ctx, QA_ERR_INVALID, "null tensor pointer");
    if (ctx->cfg.kv_head_begin != ctx->rank * ctx->hkv || ctx->nranks * ctx->hkv != ctx->cfg.n_kv_heads)
        return fail(ctx, QA_ERR_STATE, "rank %d holds KV heads [%d,%d): not the head shard the gather expects",
                    ctx->rank, ctx->cfg.kv_head_begin, ctx->cfg.kv_head_begin + ctx->hkv);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    if (!ctx->peer_ok) {
        // no peer mapping on this machine: local decode step, then the NCCL all-gather
        const size_t bytes = (size_t)n_layers * ctx->hq * D * sizeof(float);
        void* buf = ctx->step_out;
        if ((st = grow(ctx, &buf, ctx->step_out_bytes, bytes))) return st;
        ctx->step_out = static_cast<float*>(buf);
        if ((st = decode_step(ctx, &seq, &pos, 1, layer, n_layers, q_pre, k_pre, v, q_out, ctx->step_out))) return st;
        return qa_gather_heads(ctx, n_layers, 1, ctx->step_out, full);
    }
    const unsigned step = ++ctx->gather_step;
    const size_t par = (size_t)(step & 1) * ctx->landing_bytes;
    GatherArgs g{};
    g.out_hq = ctx->hq * ctx->nranks;
    g.out_h0 = ctx->rank * ctx->hq;
    for (int r = 0; r < ctx->nranks; ++r) {
        if (r != ctx->rank) g.peer_out[g.n_peers++] = reinterpret_cast<float*>(ctx->peer_base[r] + par);
        g.flags[g.n_flags++] = reinterpret_cast<unsigned*>(ctx->peer_base[r] + ctx->flags_off) + ctx->rank;
    }
    g.done = ctx->gather_done;
    g.step = step;
    float* landing = reinterpret_cast<float*>(ctx->peer_block + par);
    if ((st = decode_step(ctx, &seq, &pos, 1, layer, n_layers, q_pre, k_pre, v, q_out, landing, &g))) return st;
    const bool chain = ctx->last_fused_step;           // the wait reads no KV rows: the chain goes on
    launch_gather_wait_copy(reinterpret_cast<const unsigned*>(ctx->peer_block + ctx->flags_off), ctx->nranks, step,
                            landing, full, (size_t)n_layers * g.out_hq * D, ctx->error, ctx->stream);
    st = after_launch(ctx, -1, "gather_wait_copy");
    ctx->last_fused_step = chain && st == QA_OK;
    return st;
}

static int kv_transfer(qa_ctx* ctx, int seq, int ntok, int peer, bool send) {
    if (!ctx) return QA_ERR_INVALID;
    int st;
    if ((st = check_seq(ctx, seq))) return st;
    if (!ctx->comm) return fail(ctx, QA_ERR_STATE, "no communicator (qa_comm_init)");
    if (peer < 0 || peer >= ctx->nranks || peer == ctx->rank) return fail(ctx, QA_ERR_INVALID, "bad peer %d", peer);
    if (ntok < 1 || ntok > ctx->cfg.context) return fail(ctx, QA_ERR_INVALID, "bad row count %d", ntok);
    if (send && ntok > ctx->pos[seq])
        return fail(ctx, QA_ERR_STATE, "sequence holds %d committed rows, send wants %d", ctx->pos[seq], ntok);
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    const size_t bytes = (size_t)ctx->cfg.n_layers * 2 * ctx->hkv * ntok * D * sizeof(__half);
    const int b = ctx->kv_next;
    if ((st = grow(ctx, &ctx->kv_buf[b], ctx->kv_buf_bytes[b], bytes))) return st;
    void* buf = ctx->kv_buf[b];
    std::string err;
    if (send) {
        // pack on the context stream once the previous NCCL op on this buffer is done; the
        // send then runs on the communication stream while the context stream moves on
        QA_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->kv_comm_done[b], 0));
        launch_pack_kv(ctx->kv, seq, 0, ntok, buf, false, ctx->stream);
        if ((st = after_launch(ctx, -1, "pack_kv"))) return st;
        QA_CUDA(cudaEventRecord(ctx->kv_packed, ctx->stream));
        QA_CUDA(cudaStreamWaitEvent(ctx->comm_stream, ctx->kv_packed, 0));
        if ((st = nccl_send_recv_bytes(ctx->comm, buf, bytes, peer, true, ctx->comm_stream, err)))
            return fail(ctx, st, "ncclSend: %s", err.c_str());
        QA_CUDA(cudaEventRecord(ctx->kv_comm_done[b], ctx->comm_stream));
    } else {
        // receive on the communication stream once the previous unpack from this buffer is
        // done; the unpack follows on the context stream
        QA_CUDA(cudaStreamWaitEvent(ctx->comm_stream, ctx->kv_unpacked[b], 0));
        if ((st = nccl_send_recv_bytes(ctx->comm, buf, bytes, peer, false, ctx->comm_stream, err)))
            return fail(ctx, st, "ncclRecv: %s", err.c_str());
        QA_CUDA(cudaEventRecord(ctx->kv_comm_done[b], ctx->comm_stream));
        QA_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->kv_comm_done[b], 0));
        launch_pack_kv(ctx->kv, seq, 0, ntok, buf, true, ctx->stream);
        if ((st = after_launch(ctx, seq, "unpack_kv"))) return st;
        QA_CUDA(cudaEventRecord(ctx->kv_unpacked[b], ctx->stream));
        ctx->pos[seq] = ntok;
        std::fill(ctx->appended[seq].begin(), ctx->appended[seq].end(), ntok);
    }
    ctx->kv_next = b ^ 1;
    return QA_OK;
}

int qa_kv_send(qa_ctx* ctx, int seq, int ntok, int peer) { return kv_transfer(ctx, seq, ntok, peer, true); }
int qa_kv_recv(qa_ctx* ctx, int seq, int ntok, int peer) { return kv_transfer(ctx, seq, ntok, peer, false); }

int qa_comm_join(qa_ctx* ctx) {
    if (!ctx) return QA_ERR_INVALID;
    if (!ctx->comm_stream) return QA_OK;
    QA_CUDA(cudaSetDevice(ctx->cfg.device));
    return comm_leave(ctx);
}

}  // extern "C"
