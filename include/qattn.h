/* qattn.h — C ABI of the B200 attention + KV-cache library (libqattn.so).
 *
 * Drop-in boundary for the attention and KV-cache hot path of tampajohn/fpga-qwen's C++
 * Qwen3-0.6B engine. The engine's Model::Impl (engine/core.cpp) keeps its projections,
 * MLP, sampler and protocol; the lines that own the FP16 KV history and compute
 * QK-RMSNorm, RoPE, the FP16 KV write and causal GQA attention become calls below.
 * Each declaration names the reference code it replaces.
 *
 * Conventions
 *   - Every entry point returns int status (QA_OK == 0). Validation happens before any
 *     state change or launch: a call that fails validation leaves the context unchanged
 *     (engine/core.hpp:32-33, :41; core.cpp:708-710, :723). qa_last_error() describes
 *     the most recent failure.
 *   - One host thread per context at a time ("One caller at a time", core.hpp:23).
 *   - Tensor arguments are FP32, row-major, heads innermost-but-one:
 *        q      [n_layers][n][hq_local][128]
 *        k, v   [n_layers][n][hkv_local][128]
 *        out    [n_layers][n][hq_local][128]
 *     where hkv_local = kv_head_count and hq_local = kv_head_count * (n_q_heads/n_kv_heads).
 *     Device pointers when the context was created with io_host = 0 (calls are
 *     asynchronous on the context's stream); host pointers when io_host = 1 (the call
 *     stages through device buffers made at qa_create, returns after the results are in
 *     host memory, and reports a device-side wait that ran out as QA_ERR_TIMEOUT with the
 *     sequence reset). Small calls move their inputs in one host->device copy and their
 *     outputs in one device->host copy through pinned memory of the context.
 *   - No hot call allocates device memory or synchronises beyond its own stream: the KV
 *     store, split-context scratch and staging are sized at qa_create for every call the
 *     context accepts (up to min(max_seqs, QA_MAX_BATCH) rows of a batched decode).
 *   - KV history lives in HBM, one slot per sequence, laid out
 *        [seq][layer][K|V][kv_head][pos][128] FP16, 256-byte rows
 *     (reference: two arrays [layer][head][pos][128], core.cpp:223, :277, :350-352).
 */
#ifndef QATTN_H
#define QATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    QA_OK = 0,
    QA_ERR_INVALID = 1,     /* bad argument; nothing changed                         */
    QA_ERR_CAPACITY = 2,    /* context capacity exceeded (core.cpp:709); nothing changed */
    QA_ERR_STATE = 3,       /* not valid in the sequence's current state; nothing changed */
    QA_ERR_CUDA = 4,        /* CUDA error; the sequence is reset to position 0        */
    QA_ERR_NCCL = 5,        /* NCCL error                                             */
    QA_ERR_TIMEOUT = 6,     /* a bounded device-side wait expired                     */
    QA_ERR_OOM = 7,         /* device allocation failed                               */
    QA_ERR_UNSUPPORTED = 8  /* shape or feature this build does not support           */
};

#define QA_HEAD_DIM 128
#define QA_MAX_CONTEXT 4096
#define QA_PREFIX_CHUNK 512       /* canonical prefix-reuse granule, core.hpp:10 */
#define QA_MAX_DECODE_ROWS 4      /* rows per qa_attn_decode call (1 = step, 2 = B2 verify) */

typedef struct qa_config {
    int n_layers;        /* 28                                                       */
    int n_q_heads;       /* 16 (global)                                              */
    int n_kv_heads;      /* 8 (global); GQA group = n_q_heads / n_kv_heads           */
    int head_dim;        /* must be 128                                              */
    int context;         /* 1..4096 positions per sequence (core.cpp:237)            */
    int max_seqs;        /* sequence slots held in HBM                               */
    int kv_head_begin;   /* first global KV head this context holds (head sharding)  */
    int kv_head_count;   /* KV heads held; 0 means all n_kv_heads                    */
    double rope_theta;   /* 1e6 (core.cpp:288)                                       */
    float norm_eps;      /* 1e-6 (core.cpp:213)                                      */
    int device;          /* CUDA device ordinal                                      */
    int io_host;         /* 0: tensor pointers are device memory; 1: host memory     */
} qa_config;

typedef struct qa_ctx qa_ctx;

/* Fills the Qwen3-0.6B defaults: 28 layers, 16/8 heads, 128, context 4096, 1 slot. */
void qa_default_config(qa_config* cfg);

/* Allocates the HBM KV store, RoPE tables and norm weights.
 * Replaces Model::Impl's KV allocation and table set-up, core.cpp:236-237, :277, :287-288. */
int qa_create(const qa_config* cfg, qa_ctx** out);
void qa_destroy(qa_ctx* ctx);

const char* qa_last_error(const qa_ctx* ctx);
const char* qa_status_string(int status);
/* Library build identification, e.g. "qattn sm_100a". */
const char* qa_version(void);

/* Limit of the bounded device-side waits on other GPUs (the flag waits of the head gathers,
 * qa_attn_prefill_gather and qa_decode_step_gather), in microseconds; 0 restores the default
 * of 2 s. A wait that runs out records QA_ERR_TIMEOUT, which qa_sync and the next host-buffer
 * call report, instead of holding the GPU. No counterpart in the reference (one CPU host). */
int qa_set_wait_limit(qa_ctx* ctx, int microseconds);
/* Self-test of that failure path on a single GPU: launches the head gather's wait kernel on a
 * flag word of this context that nothing ever sets. After the wait limit the kernel gives up
 * and records the timeout exactly as when a peer GPU stops answering; the next qa_sync (or
 * host-buffer call, which then resets its sequence) returns QA_ERR_TIMEOUT and clears it.
 * Asynchronous on the context stream. No counterpart in the reference. */
int qa_selftest_timeout(qa_ctx* ctx);

/* Runs subsequent work on an external cudaStream_t (NULL restores the context's own). */
int qa_set_stream(qa_ctx* ctx, void* cuda_stream);
/* Blocks until all work issued on the context's stream has finished. */
int qa_sync(qa_ctx* ctx);

/* Per-layer q_norm / k_norm weights [128] FP32, host pointers (pack tensors
 * self_attn.q_norm / k_norm, core.cpp:244, :395). Default: all ones. */
int qa_set_norms(qa_ctx* ctx, int layer, const float* q_norm, const float* k_norm);

/* Logical KV state: `pos` is the only validity state (core.cpp:232).
 * qa_position  -> Model::position, core.cpp:758
 * qa_reset     -> Model::reset, core.cpp:718-721 (O(1), no KV work)
 * qa_truncate  -> Model::truncate, core.cpp:722-726 (0 <= pos <= current, else QA_ERR_STATE)
 * qa_commit    -> the `pos += batch` after all layers, core.cpp:643, and
 *                 Model::commit_verified's `pos += count`, core.cpp:749. Every layer must
 *                 have been appended through pos+n. */
int qa_position(const qa_ctx* ctx, int seq, int* pos);
int qa_reset(qa_ctx* ctx, int seq);
int qa_truncate(qa_ctx* ctx, int seq, int pos);
int qa_commit(qa_ctx* ctx, int seq, int n);

/* Fused KV append: per-head QK-RMSNorm (eps 1e-6, FP64 sum of FP32 squares), RoPE at
 * absolute positions pos0..pos0+n-1, FP32->FP16 round-to-nearest-even K/V write into
 * rows [pos0, pos0+n) of layers [layer, layer+n_layers). Writes the normed, roped
 * query to q_out. pos0 must equal the sequence's committed position.
 * Replaces core.cpp:395-406 (and the B2 copy :659-670). Bit-exact with that arithmetic. */
int qa_append(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n,
              const float* q_pre, const float* k_pre, const float* v, float* q_out);

/* Causal GQA attention of n new rows: row b (position pos0+b) of query head h attends to
 * keys [0, pos0+b] of KV head h/group, softmax(q.k/sqrt(128)) . V, FP32 out.
 * Rows [pos0, pos0+n) of every layer in range must have been appended.
 * Replaces the batched-prefill attention, core.cpp:357-381 and :407-605.
 * Within max-abs 1e-3 / RMS 1e-4 of that arithmetic. */
int qa_attn_prefill(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n,
                    const float* q, float* out);

/* Same contract for 1 <= n <= QA_MAX_DECODE_ROWS rows with split-context
 * (flash-decoding) parallelism. n == 1 replaces the decode attention, core.cpp:606-624;
 * n == 2 replaces the B2 verify attention, core.cpp:671-689. */
int qa_attn_decode(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n,
                   const float* q, float* out);

/* Batched decode over independent sequences (multi-request serving). Row b of the tensors
 * belongs to sequence seqs[b] (host array of 1..QA_MAX_BATCH distinct slots) at that
 * sequence's committed position; q_pre/k_pre/v/q_out/out use the layouts above with
 * n = n_seqs. Each row is exactly one reference decode step (core.cpp:395-406 then
 * :606-624) for its sequence; the batch runs as one append launch and one attention launch
 * whose key work is split evenly over the GPU. qa_commit_batch advances every listed
 * sequence by one position (core.cpp:643 for batch 1). */
#define QA_MAX_BATCH 64
int qa_append_batch(qa_ctx* ctx, const int* seqs, int n_seqs, int layer, int n_layers,
                    const float* q_pre, const float* k_pre, const float* v, float* q_out);
int qa_attn_decode_batch(qa_ctx* ctx, const int* seqs, int n_seqs, int layer, int n_layers,
                         const float* q, float* out);
int qa_commit_batch(qa_ctx* ctx, const int* seqs, int n_seqs);

/* Fused decode step: qa_append of one new row followed by qa_attn_decode of that row, in a
 * single launch (the per-token work of core.cpp:395-406 then :606-624 for every requested
 * layer). Same tensors and layouts as those two calls with n = 1; q_out (the normalised,
 * rotated query rows) may be NULL when the caller does not need it. K/V rows and q_out are
 * bit-identical to qa_append; out matches qa_attn_decode. pos must be the sequence's
 * committed position; qa_commit advances it afterwards, as after qa_append.
 * The batch form takes one row per listed sequence at its committed position (layouts of
 * qa_append_batch / qa_attn_decode_batch). */
int qa_decode_step(qa_ctx* ctx, int seq, int layer, int n_layers, int pos, const float* q_pre,
                   const float* k_pre, const float* v, float* q_out, float* out);
/* Opt-in overlap of consecutive decode steps (default off). When on, a qa_decode_step launched
 * right after another fused decode step of this context on the same stream starts while the
 * previous one finishes (programmatic dependent launch): it sets up and copies KV rows older
 * than the previous step's new row early, and reads its inputs, and everything the previous
 * step wrote, only once that step's grid has completed. The caller promises that no kernel
 * of its own writes this context's KV store between two such steps (the library's own
 * launches of other kinds end the overlap by themselves). No effect in io_host mode. */
int qa_set_step_overlap(qa_ctx* ctx, int enable);
int qa_decode_step_batch(qa_ctx* ctx, const int* seqs, int n_seqs, int layer, int n_layers,
                         const float* q_pre, const float* k_pre, const float* v, float* q_out,
                         float* out);

/* Canonical prefix reuse by device block copy: copies KV rows [0, ntok) of every layer,
 * K/V and head from slot src_seq to slot dst_seq and sets dst's position to ntok.
 * ntok must be a positive multiple of QA_PREFIX_CHUNK and <= src's position.
 * Replaces the adapter's `rewind` of a retained prefix (tools/native_cpu_chat.py:189-216,
 * engine/INTERFACE.md:151-168) for a prefix held by another sequence slot. */
int qa_copy_prefix(qa_ctx* ctx, int src_seq, int dst_seq, int ntok);

/* Device-resident pool of canonical prefix blocks, for a prefix cache that outlives the
 * sequence slots (cross-session reuse of engine/INTERFACE.md:151-168's 512-token granule).
 * A block holds rows [512*chunk, 512*chunk + 512) of every layer, K/V and head of one
 * sequence: 512 * 114,688 bytes at 28 layers and 8 KV heads. The keys carry RoPE of their
 * absolute positions, so a block loads back only at the chunk index it was saved from.
 * qa_block_pool (re)allocates n_blocks (0 frees the pool; existing blocks are dropped;
 * synchronises the context stream). */
int qa_block_pool(qa_ctx* ctx, int n_blocks);
/* Copies chunk `chunk` of sequence seq (committed rows: position >= 512*(chunk+1)) into
 * pool block `block`. */
int qa_block_save(qa_ctx* ctx, int seq, int chunk, int block);
/* Sequence seq, at position 512*chunk, receives the block's rows (saved from the same chunk
 * index) and advances to 512*(chunk+1): qa_copy_prefix for one chunk, from the pool. */
int qa_block_load(qa_ctx* ctx, int seq, int chunk, int block);

/* Reads FP16 KV rows [pos0, pos0+n) of (layer, kv = 0 for K / 1 for V, local head) into
 * dst (host memory, n*128 uint16). Synchronous. Diagnostic / parity access to the store. */
int qa_read_kv(qa_ctx* ctx, int seq, int layer, int kv, int head, int pos0, int n,
               uint16_t* dst);

/* Device address of the KV rows of (seq, layer, kv, local head) at position 0, and the
 * byte size of one whole sequence slot. For peer copies and external consumers. */
int qa_kv_pointer(qa_ctx* ctx, int seq, int layer, int kv, int head, void** ptr);
int qa_kv_slot_bytes(const qa_ctx* ctx, size_t* bytes);

/* ---- Projections over FP16 matrices (the engine's GEMVs around attention) ------------------
 * y[b][r] = dot(x[b], W[r]) for an FP16 matrix W [rows][cols] (cols a multiple of 8, W and a
 * device x 16-byte aligned, W DEVICE memory in every context: weights stay resident), FP32 x [batch][cols] and
 * y [batch][rows] (device pointers, or host pointers in io_host contexts), 1 <= batch <=
 * QA_MAX_BATCH. Every output follows the reference's eight-lane dot bit for bit: two 4-lane
 * FP32 accumulators over channels j..j+3 and j+4..j+7, fused multiply-adds with j ascending by
 * 8, then (s0+s1)+(s2+s3) of their lane-wise sums (core.cpp:119-147). That is the arithmetic
 * of Model::Impl::project for one row (core.cpp:292-301), of the verification projections for
 * two (project_verify, dot_verify_pair / dot_verify_two_rows, :182-206, :321-349) and of the
 * FP16-only vocabulary head at any batch (:705, :713). (Batched prefill projections over the
 * FP32 copies of the layer matrices, cblas_sgemm at :294, sum in an unpublished order; this
 * call gives them within FP32 rounding.) Asynchronous on the context stream. */
int qa_project(qa_ctx* ctx, const uint16_t* w, int rows, int cols, const float* x, int batch, float* y);
/* The same for n_mats (1..8) matrices of equal width that share the input x, as one launch:
 * q/k/v or gate/up (project_group / project_group_verify, core.cpp:302-320, :388-389, :629,
 * :657, :693). y[m] receives [batch][rows[m]]. */
int qa_project_group(qa_ctx* ctx, int n_mats, const uint16_t* const* w, const int* rows, int cols,
                     const float* x, int batch, float* const* y);
/* Batched projections of prompt rows on the tensor cores: Model::Impl::project and
 * project_group with more than one row (core.cpp:292-320, the cblas_sgemm at :294 over the FP32
 * widening of the FP16 matrices; :387-394, :625-641 for a prompt chunk). Each input row is split
 * into two FP16 halves (22 bits of its significand, after an exact power-of-two scale) and both
 * are multiplied by W with FP32 accumulation, so y lies within FP32 accumulation rounding of the
 * exact product, as sgemm's does (no bit-exact claim: sgemm's summation order is unpublished).
 * Same arguments and alignment rules as qa_project / qa_project_group; any batch >= 1 (host
 * buffers: up to the staging made at creation). Widths above 8192 columns run on the CUDA-core
 * kernels instead. Asynchronous on the context stream. */
int qa_project_gemm(qa_ctx* ctx, const uint16_t* w, int rows, int cols, const float* x, int batch, float* y);
int qa_project_group_gemm(qa_ctx* ctx, int n_mats, const uint16_t* const* w, const int* rows, int cols,
                          const float* x, int batch, float* const* y);

/* ---- Multi-GPU: KV-head sharding and prefill -> decode handoff (NCCL over NVLink) -------
 * No counterpart in the reference, a single-host CPU engine. One process per GPU; each
 * context holds KV heads [kv_head_begin, kv_head_begin + kv_head_count) with their GQA
 * query heads. NCCL is loaded at run time (libnccl.so.2). */

/* Writes a new NCCL unique id (128 bytes) for qa_comm_init; call on one rank, share it. */
int qa_comm_unique_id(char id[128]);
/* Joins the communicator of nranks contexts (collective: every rank must call it). */
int qa_comm_init(qa_ctx* ctx, int nranks, int rank, const char id[128]);
int qa_comm_destroy(qa_ctx* ctx);
/* All-gather of head-sharded attention outputs. Rank r must hold KV heads
 * [r*kv_head_count, (r+1)*kv_head_count) and nranks*kv_head_count == n_kv_heads.
 * local: [n_layers][n][hq_local][128] device FP32; full: [n_layers][n][n_q_heads][128]
 * device FP32 with heads in global order (the layout the reference's o_proj reads,
 * core.cpp:625). Collective; asynchronous on the context's stream. */
int qa_gather_heads(qa_ctx* ctx, int n_layers, int n, const float* local, float* full);
/* The same gather without holding the context stream: the all-gather and the permute run on
 * the context's communication stream, so work queued next on the context stream (the next
 * layers' prefill) overlaps them. `local` must stay unchanged and `full` unread until
 * qa_comm_join or qa_sync. Consecutive gathers run in call order. */
int qa_gather_heads_async(qa_ctx* ctx, int n_layers, int n, const float* local, float* full);
/* Prefill attention with the head gather done by the kernels themselves, for KV-head shards:
 * qa_attn_prefill of this rank's heads, with every output row stored straight into `full`
 * ([n_layers][n][all query heads][128], device) at this rank's head offset and, over NVLink,
 * into every other rank's landing buffer; then a wait for all ranks' "rows stored" marks and a
 * copy of the other ranks' heads into `full`. Bit-identical to qa_attn_prefill followed by
 * qa_gather_heads. Collective: every rank calls it with the same layer range, pos0 and n.
 * The first call maps the landing buffers ([layers][context][all heads][128] FP32 per rank).
 * Bounded waits: QA_ERR_TIMEOUT (read by qa_sync) after 2 s. Where the machine offers no peer
 * mapping, it runs qa_attn_prefill + qa_gather_heads (NCCL), with the same results.
 * Replaces the batched-prefill attention (core.cpp:357-381, :407-605) on a KV-head shard and
 * hands o_proj the full-head rows. */
int qa_attn_prefill_gather(qa_ctx* ctx, int seq, int layer, int n_layers, int pos0, int n, const float* q,
                           float* full);
/* Prefill -> decode KV handoff. qa_kv_send ships KV rows [0, ntok) of every layer, K|V and
 * local head of sequence `seq` to rank `peer`; the peer's matching qa_kv_recv stores them in
 * its slot `seq` and sets that sequence's position to ntok. Both contexts must hold the
 * same heads. 114,688*ntok bytes at 28 layers and 8 KV heads.
 * Asynchronous and pipelined: the rows are packed on the context stream into one of two
 * staging buffers and cross NVLink on the context's communication stream, so consecutive
 * handoffs overlap (pack of request i+1 / unpack of request i-1 with the transfer of
 * request i). Work queued later on the context stream is ordered after the pack (sender)
 * or the unpack (receiver); the sender's context stream does not wait for the transfer
 * itself: qa_comm_join or qa_sync does. */
int qa_kv_send(qa_ctx* ctx, int seq, int ntok, int peer);
int qa_kv_recv(qa_ctx* ctx, int seq, int ntok, int peer);
/* Communicator shape of a context and whether the other ranks' gather buffers are mapped
 * into this process (1: qa_decode_step_gather stores over NVLink; 0: it uses NCCL). */
int qa_comm_info(const qa_ctx* ctx, int* nranks, int* rank, int* peer_mapped);
/* Makes the context stream wait for all communication queued so far (no host wait). */
int qa_comm_join(qa_ctx* ctx);

/* Fused decode step with the head gather done by the kernel itself, for KV-head shards
 * (the layout qa_gather_heads expects): qa_decode_step of one row on this rank's heads, with
 * every output row stored straight into every rank's landing buffer over NVLink (peer
 * stores into memory mapped at qa_comm_init), then a wait for all ranks' "step done" marks
 * and a copy into `full` ([n_layers][1][all query heads][128], device). Collective: every
 * rank calls it for the same step. A rank whose peers stop answering records
 * QA_ERR_TIMEOUT (read by qa_sync) after 2 s instead of waiting forever. Where the
 * machine offers no peer mapping, it runs qa_decode_step + qa_gather_heads (NCCL) instead,
 * with the same results. Replaces, per token, core.cpp:395-406 + :606-624 and hands o_proj
 * (core.cpp:625) the full-head rows. */
int qa_decode_step_gather(qa_ctx* ctx, int seq, int layer, int n_layers, int pos, const float* q_pre,
                          const float* k_pre, const float* v, float* q_out, float* full);

/* Size of the fixed device array behind qa_attn_decode_noalloc: 4 MiB per GPU. It is loaded
 * onto a GPU when qa_create runs on that device (or, without a context, at the first
 * qa_attn_decode_noalloc call there) and held until the process exits. */
#define QA_NOALLOC_SCRATCH_BYTES (4u << 20)

/* Split-context decode attention that allocates nothing. It has no counterpart in the
 * reference: it exists for hosts that own all device memory themselves (a serving
 * runtime's pre-reserved arena, an engine with a fixed HBM budget) and do not let this
 * library call cudaMalloc, which would fail there or synchronise the whole device.
 * Same arithmetic and tolerance as qa_attn_decode, on caller-owned memory:
 *   kv_slot  one sequence slot of the KV store, [n_layers_total][K|V][n_kv_heads][context][128]
 *            FP16 (what qa_kv_pointer(ctx, seq, 0, 0, 0, &p) returns), device memory
 *   q, out   [n_layers][n][2*n_kv_heads][128] FP32, device memory; rows at positions
 *            pos0..pos0+n-1 of layers [layer, layer+n_layers), 1 <= n <= QA_MAX_DECODE_ROWS
 *   stream   cudaStream_t (NULL: the legacy default stream)
 * Scratch lives in one static device array of QA_NOALLOC_SCRATCH_BYTES; requests whose
 * (layer, row, head) records do not fit return QA_ERR_CAPACITY before anything runs.
 * qa_create looks up that array's address for its device, which loads it onto the GPU; a
 * host that reserves the rest of HBM for its own arena should create its context first.
 * Without a context on the device, the first call there does the look-up (make it before
 * any stream capture). After a device reset the address is looked up again.
 * Every call shares the array: calls that overlap on the GPU race, so issue them on one
 * stream or order them. Asynchronous on `stream`. */
int qa_attn_decode_noalloc(const void* kv_slot, int n_layers_total, int n_kv_heads, int context,
                           int layer, int n_layers, int pos0, int n, const float* q, float* out,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QATTN_H */
