// Shared definitions of the qattn CUDA library: KV layout, launch argument blocks and
// the kernel launchers implemented in the per-kernel .cu files.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace qattn {

constexpr int D = 128;          // head_dim
constexpr int GROUP = 2;        // query heads per KV head (Qwen3-0.6B: 16 / 8)
constexpr int NUM_SMS_B200 = 148;

// HBM KV store: [seq][layer][K|V][kv_head][pos][128] FP16 (256-byte rows).
struct KVLayout {
    __half* base = nullptr;
    int layers = 0, hkv = 0, ctx = 0;
    __host__ __device__ size_t plane_elems() const { return size_t(ctx) * D; }
    __host__ __device__ size_t slot_elems() const { return size_t(layers) * 2 * hkv * plane_elems(); }
    __host__ __device__ __half* plane(int seq, int layer, int kv, int head) const {
        return base + ((((size_t(seq) * layers + layer) * 2 + kv) * hkv + head) * size_t(ctx)) * D;
    }
};

// Sequence slot and absolute position of each row of a call. Plain calls use (seq, pos0 + b);
// batched decode calls give every row its own sequence (one row per sequence).
constexpr int MAX_BATCH = 64;
struct RowMap {
    int batched;
    int seq[MAX_BATCH];
    int pos[MAX_BATCH];
    __host__ __device__ int seq_of(int b, int seq0) const { return batched ? seq[b] : seq0; }
    __host__ __device__ int pos_of(int b, int pos0) const { return batched ? pos[b] : pos0 + b; }
};

struct AppendArgs {
    const float* q_pre; const float* k_pre; const float* v_pre; float* q_out;
    KVLayout kv; int seq; int layer0; int n_layers; int pos0; int n; int hq; int hkv;
    RowMap rows;
    const float* norms;      // [layers][2][128]: q_norm, k_norm
    const float* cosines;    // [ctx][64]
    const float* sines;      // [ctx][64]
    float eps;
};

// Split-context attention over explicit rows. Row b of the call sits at absolute position
// pos0+b and attends to keys [0, pos0+b]. Rows [row_begin, row_end) are computed.
struct RowsArgs {
    const float* q; float* out;     // [n_layers][n][hq][128]
    KVLayout kv; int seq; int layer0; int n_layers; int pos0; int n; int hq; int hkv;
    int row_begin, row_end;
    int splits, keys_per_split;
    float* partial;                 // [units][splits][4 + 2*128] when splits > 1
    int* counters;                  // [units], zero between calls
};

constexpr int MAX_RANKS = 8;

// Device error block of a context (256 bytes, zeroed at creation):
//   word ERR_CODE     first error code recorded by a bounded wait (0 = none); read and cleared
//                     by qa_sync and by every host-buffer call
//   word ERR_WAIT_US  limit of the waits on other GPUs' flags, in microseconds (0 = 2 s)
//   word ERR_NEVER    a flag word that nothing ever sets (qa_selftest_timeout waits on it)
constexpr int ERR_CODE = 0, ERR_WAIT_US = 1, ERR_NEVER = 2;
constexpr size_t ERR_BLOCK_BYTES = 256;
__device__ __forceinline__ unsigned long long peer_wait_limit_ns(const int* error) {
    const unsigned us = *reinterpret_cast<const volatile unsigned*>(error + ERR_WAIT_US);
    return us ? us * 1000ull : 2000000000ull;
}

// Destination of prefill output rows: row b of layer l, query head h of this context, goes to
// out[((l * n + b) * heads + head0 + h) * 128 ...] and to the same offset of every peers[i]
// (other GPUs' buffers, written over NVLink). {out, hq, 0, 0} is the plain local layout.
// With peers, every CTA ends with a system-scope fence, so a later launch on the stream may
// publish the rows to the peers with a release store.
struct OutRows {
    float* out = nullptr;
    int heads = 0, head0 = 0;
    int n_peers = 0;
    float* peers[MAX_RANKS - 1] = {};
};

void launch_kv_append(const AppendArgs& a, cudaStream_t s);
void launch_attn_rows(const RowsArgs& a, cudaStream_t s);
// Loads attn_rows_kernel's module onto the current device (lazy module loading defers that to
// the first launch, which may then need device memory).
cudaError_t prepare_attn_rows();
// FP32 attention of prefill rows [0, row_end) whose positions are all below 128.
void launch_attn_head_rows(const RowsArgs& a, const OutRows& o, cudaStream_t s);
void launch_kv_copy(const KVLayout& kv, int src_seq, int dst_seq, int ntok, cudaStream_t s);
// Tensor-core prefill for rows [row_begin, n) (all with absolute position >= 128).
// Returns non-zero (and launches nothing) if the kernel was not built with the expected registers.
int launch_attn_prefill_sm100(const CUtensorMap& map, const float* q, const OutRows& o, int seq, int layer0,
                              int n_layers, int pos0, int n, int hq, int hkv, int layers_total, int row_begin,
                              int* tile_counter, float* split_scratch, int reserve_sms, int* error,
                              cudaStream_t s);
// Device scratch for launches whose items are split over key segments (sized at context creation).
size_t prefill_split_scratch_bytes();
// TMA-streamed split-context decode. Row b of the call is sequence rows.seq[b] at position
// rows.pos[b] (context rows.pos[b] + 1), b < n <= MAX_BATCH.
struct DecodePlan {
    int ctas, max_keys, max_records, units;
    int max_units_per_cta;            // bound on the units one CTA range touches
    long long total_keys;
    size_t partial_floats() const;
};
DecodePlan plan_attn_decode(int n_layers, int hkv, int n, const int* pos);
// Upper bound of DecodePlan::partial_floats() over every plan of at most n_layers layers and
// n_max rows (any positions): the record count units * max_records is at most
// n_max * ctas + 2 * units, because total_keys >= n_layers_call * hkv * max_len.
size_t decode_partial_floats_bound(int n_layers, int hkv, int n_max);
// Inputs of a fused decode step (append of the one new row per sequence + decode attention).
// The fused kernel prepares the rows of at most FUSED_MAX_UNITS units per CTA before it
// streams; plans with more units per CTA run as append + decode.
constexpr int FUSED_MAX_UNITS = 4;
// Head gather through peer memory (decode step on KV-head shards): the kernel stores each
// output row into the landing buffer of every rank (its own and, over NVLink, its peers'),
// at this rank's head offset in the full-head layout, then its last CTA marks the step done
// in every rank's flag array.
struct GatherArgs {
    int out_hq = 0, out_h0 = 0;                  // heads per output row, this rank's first head
    int n_peers = 0;
    float* peer_out[MAX_RANKS] = {};             // other ranks' landing buffers (peer pointers)
    int n_flags = 0;
    unsigned* flags[MAX_RANKS] = {};             // word "rank me finished step" in each rank's flags
    unsigned* done = nullptr;                    // CTAs finished (this GPU), zero between launches
    unsigned step = 0;
};
struct StepInputs {
    const float* q_pre = nullptr; const float* k_pre = nullptr; const float* v_pre = nullptr;   // [L][n][h][128]
    float* q_out = nullptr;                                    // optional
    const float* norms = nullptr; const float* cosines = nullptr; const float* sines = nullptr;
    float eps = 0.f;
    int pdl = 0;                                               // programmatic dependent launch
};
void launch_attn_decode_sm100(const DecodePlan& plan, const KVLayout& kv, const float* q, float* out, int layer0,
                              int n_layers, int n, const int* seq, const int* pos, int hq, int hkv, float* partial,
                              int* counters, int* error, cudaStream_t s,
                              const StepInputs* step = nullptr, const GatherArgs* gather = nullptr);
// Waits (bounded) until every rank marked `step` done in `flags`, then copies the landing
// buffer to the caller's output. Error code 51 in *error when the wait runs out.
void launch_gather_wait_copy(const unsigned* flags, int nranks, unsigned step, const float* landing, float* out,
                             size_t floats, int* error, cudaStream_t s);
// Prefill head gather through peer memory. Each rank's flag array holds, per rank r, the word
// "r's rows of call k are in your landing buffer" (PF_READY + r) and "r has copied call k out
// of its landing buffer" (PF_ACK + r).
constexpr int PF_READY = 16, PF_ACK = 32;
// One thread: tells every peer that this rank's landing buffer is free of call `call` - 1 (its
// copy ran earlier on the stream), then waits (bounded, error 52) until every peer said the same.
// peer_flags[r]: rank r's flag array as mapped here (peer_flags[rank]: this rank's own).
void launch_prefill_gate(unsigned* const* peer_flags, int nranks, int rank, unsigned call, int* error,
                         cudaStream_t s);
// One thread: marks call `call` ready in every peer's flag array (system-scope release).
void launch_prefill_signal(unsigned* const* peer_flags, int nranks, int rank, unsigned call, cudaStream_t s);
// Waits (bounded, error 53) for every peer's ready mark of `call`, then copies the other ranks'
// heads of every row from the landing buffer ([n_layers][n][hq_local * nranks][128]) to full.
void launch_prefill_wait_copy(const unsigned* my_flags, int nranks, int rank, unsigned call, const float* landing,
                              float* full, int n_layers, int n, int hq_local, int* error, cudaStream_t s);
// Rows at absolute positions below this go to the FP32 CUDA-core kernel.
constexpr int TC_MIN_POSITION = 128;
void launch_synth(float* dst, uint64_t seed, int kind, int layer0, int n_layers, int pos0, int n,
                  int head0, int heads, float mean, float stdev, cudaStream_t s);

// Multi-GPU helpers (qattn_dist.cu).
void launch_permute_heads(const float* gathered, float* full, int nranks, int n_layers, int n, int hq_local,
                          cudaStream_t s);
// Rows [pos0, pos0 + ntok) of every plane of slot seq <-> contiguous [planes][ntok][128] at buf.
void launch_pack_kv(const KVLayout& kv, int seq, int pos0, int ntok, void* buf, bool unpack, cudaStream_t s);

// Partial record size (floats) of one split in RowsArgs::partial.
constexpr int PARTIAL_FLOATS = 4 + GROUP * D;

// Decode projections (project.cu): y[m][b][r] = eight-lane dot of x[b] and row r of the FP16
// matrix w[m] ([rows[m]][cols], cols % 8 == 0, 16-byte aligned), for n_mats matrices sharing
// one input x [batch][cols]. tile0 is filled by the launcher.
constexpr int MAX_PROJECT_MATS = 8;
struct ProjectArgs {
    int n_mats = 0;
    const __half* w[MAX_PROJECT_MATS] = {};
    int rows[MAX_PROJECT_MATS] = {};
    float* y[MAX_PROJECT_MATS] = {};
    int tile0[MAX_PROJECT_MATS + 1] = {};
    int cols = 0, batch = 0;
    const float* x = nullptr;
};
void launch_project(ProjectArgs a, cudaStream_t s);
// Batched projections on the tensor cores (project_mma.cu): the rows are split into FP16 halves
// in a scratch area of project_gemm_scratch_bytes() (made at context creation), GEMM_CHUNK_ROWS
// input rows at a time. Returns 0, or < 0 when the shape does not fit (cols > GEMM_MAX_COLS) or
// a tensor map cannot be made. Bounded-wait expiry codes go to *error.
constexpr int GEMM_CHUNK_ROWS = 512, GEMM_MAX_COLS = 8192;
size_t project_gemm_scratch_bytes();
int launch_project_gemm(const ProjectArgs& a, void* scratch, int* error, cudaStream_t s);

// Looks up, for `device` and its current context, the device address of the fixed scratch array
// behind qa_attn_decode_noalloc (attn_decode_noalloc.cu). Makes `device` current.
cudaError_t noalloc_prepare(int device);

}  // namespace qattn
