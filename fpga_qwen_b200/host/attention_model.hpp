// attention_model.hpp — C++ host mirror of qwen_cpu::Model's attention/KV path over libqattn.
//
// tampajohn/fpga-qwen engine/core.hpp:25-56 and engine/core.cpp:707-752 define the model's
// state machine, kept here for one sequence slot of a qa_ctx:
//   prefill / step    append rows and advance the position (core.cpp:707-714, :727-728);
//   verify_two        evaluates two rows without advancing and blocks inference until
//                     commit_verified, reset or truncate (core.cpp:729-752, core.hpp:38-45);
//   reset / truncate  O(1) logical operations (core.cpp:718-726);
//   errors            std::runtime_error. Validation failures (the reference's messages)
//                     leave the state unchanged; execution failures reset the logical
//                     state and rethrow (core.cpp:740, :751).
// Inputs are the attention rows (pre-norm q, k, v) instead of token ids, because the
// projections stay in the host engine (core.cpp:292-349). Tensor layouts are those of
// include/qattn.h: q and out [layers][n][q_heads][128], k and v [layers][n][kv_heads][128]
// FP32, device memory or (Options::host_buffers) host memory.
//
// Two forms of the same passes:
//   all layers at once  prefill / step / verify_two take every layer's rows in one call (a
//                       caller whose layers are independent, such as a benchmark);
//   layer by layer      begin_rows(n) / layer_rows(layer, ...) / end_rows(): the engine's own
//                       loop (core.cpp:383-645), where layer l+1's q, k, v come from layer l's
//                       attention output through o_proj and the MLP, so the rows of one layer
//                       are appended and attended (core.cpp:395-406, :407-624) before the
//                       next layer's projections run; the position advances once, after the
//                       last layer (core.cpp:643), or the rows wait for commit_verified.
//
// Header-only; link libqattn.so. C++17.
#pragma once

#include <stdexcept>
#include <string>

#include "qattn.h"

namespace qattn_host {

inline constexpr int prefix_reuse_chunk = QA_PREFIX_CHUNK;

struct Options {
    int layers = 28;
    int context = 4096;
    int max_sequences = 1;
    int device = 0;
    int kv_head_begin = 0;
    int kv_head_count = 0;       // 0: all KV heads
    bool host_buffers = false;   // tensor pointers are host memory (the library stages them)
};

class AttentionModel {
public:
    explicit AttentionModel(const Options& options, int sequence = 0) : seq_(sequence) {
        if (sequence < 0 || sequence >= options.max_sequences) throw std::runtime_error("Sequence slot out of range");
        qa_config cfg;
        qa_default_config(&cfg);
        cfg.n_layers = options.layers;
        cfg.context = options.context;
        cfg.max_seqs = options.max_sequences;
        cfg.device = options.device;
        cfg.kv_head_begin = options.kv_head_begin;
        cfg.kv_head_count = options.kv_head_count;
        cfg.io_host = options.host_buffers ? 1 : 0;
        const int st = qa_create(&cfg, &ctx_);
        if (st != QA_OK) throw std::runtime_error(std::string("qa_create: ") + qa_status_string(st));
        layers_ = options.layers;
        context_ = options.context;
    }
    ~AttentionModel() { qa_destroy(ctx_); }
    AttentionModel(const AttentionModel&) = delete;
    AttentionModel& operator=(const AttentionModel&) = delete;

    qa_ctx* context() const { return ctx_; }
    int layers() const { return layers_; }

    void set_norms(int layer, const float* q_norm, const float* k_norm) {
        check(qa_set_norms(ctx_, layer, q_norm, k_norm), false);
    }

    int position() const {
        int p = 0;
        qa_position(ctx_, seq_, &p);
        return p;
    }

    void reset() {
        check(qa_reset(ctx_, seq_), false);
        verification_pending_ = false;
        pass_rows_ = 0;
    }

    void truncate(int position) {
        require(position >= 0 && position <= this->position(), "Rewind position out of range");
        check(qa_truncate(ctx_, seq_, position), false);
        verification_pending_ = false;
        pass_rows_ = 0;
    }

    // Appends n rows at the current position and writes their attention outputs; q_rows
    // receives the normalised, rotated query rows (same layout as q).
    void prefill(int n, const float* q, const float* k, const float* v, float* q_rows, float* out) {
        require(pass_rows_ == 0, "A layer pass is already open");
        if (verification_pending_) throw std::runtime_error("Commit or discard pending verification before inference");
        require(n > 0, "Empty token input");
        require(n <= context_ - position(), "Context capacity exceeded");
        const int pos = position();
        run([&] {
            int st = qa_append(ctx_, seq_, 0, layers_, pos, n, q, k, v, q_rows);
            if (st == QA_OK)   // one row: the split-context decode kernel (core.cpp:606-624)
                st = n == 1 ? qa_attn_decode(ctx_, seq_, 0, layers_, pos, n, q_rows, out)
                            : qa_attn_prefill(ctx_, seq_, 0, layers_, pos, n, q_rows, out);
            if (st == QA_OK) st = qa_commit(ctx_, seq_, n);
            return st;
        });
    }

    // One decode row through the fused step (append + attention in one launch).
    void step(const float* q, const float* k, const float* v, float* out) {
        require(pass_rows_ == 0, "A layer pass is already open");
        if (verification_pending_) throw std::runtime_error("Commit or discard pending verification before inference");
        require(1 <= context_ - position(), "Context capacity exceeded");
        const int pos = position();
        run([&] {
            int st = qa_decode_step(ctx_, seq_, 0, layers_, pos, q, k, v, nullptr, out);
            if (st == QA_OK) st = qa_commit(ctx_, seq_, 1);
            return st;
        });
    }

    // Two rows evaluated at the current position without advancing it; returns that base
    // position. Their KV rows stay appended for commit_verified.
    int verify_two(const float* q, const float* k, const float* v, float* q_rows, float* out) {
        require(pass_rows_ == 0, "A layer pass is already open");
        require(!verification_pending_, "Verification already pending");
        require(position() <= context_ - 2, "Context capacity exceeded");
        const int pos = position();
        run([&] {
            int st = qa_append(ctx_, seq_, 0, layers_, pos, 2, q, k, v, q_rows);
            if (st == QA_OK) st = qa_attn_decode(ctx_, seq_, 0, layers_, pos, 2, q_rows, out);
            return st;
        });
        verification_pending_ = true;
        return pos;
    }

    void commit_verified(int count) {
        require(verification_pending_, "No verification pending");
        require(count == 1 || count == 2, "Commit count must be one or two");
        run([&] { return qa_commit(ctx_, seq_, count); });
        verification_pending_ = false;
    }

    bool verification_pending() const { return verification_pending_; }

    // ---- layer by layer ------------------------------------------------------------------
    // Opens a pass of n new rows at the current position (n == 1: a decode step; verify: the
    // two rows of verify_two). Returns the base position. The same checks as the all-layer
    // calls, before anything runs.
    int begin_rows(int n, bool verify = false) {
        if (verification_pending_) throw std::runtime_error("Commit or discard pending verification before inference");
        require(pass_rows_ == 0, "A layer pass is already open");
        require(n > 0, "Empty token input");
        if (verify) require(n == 2, "Verification takes two rows");
        require(n <= context_ - position(), "Context capacity exceeded");
        pass_rows_ = n;
        pass_verify_ = verify;
        pass_layer_ = 0;
        pass_pos_ = position();
        return pass_pos_;
    }

    // Appends the open pass's rows of `layer` (tensors of that one layer: q [n][q_heads][128],
    // k and v [n][kv_heads][128]) and writes their attention outputs to out. Layers run in
    // order 0, 1, ... . q_rows receives the normalised, rotated query rows; it may be null for
    // a decode step, which runs as one fused launch.
    void layer_rows(int layer, const float* q, const float* k, const float* v, float* q_rows, float* out) {
        require(pass_rows_ > 0, "No layer pass is open");
        require(layer == pass_layer_, "Layers must run in order");
        const int n = pass_rows_, pos = pass_pos_;
        require(n == 1 || q_rows != nullptr, "Query rows buffer required");
        run([&] {
            if (n == 1) return qa_decode_step(ctx_, seq_, layer, 1, pos, q, k, v, q_rows, out);
            int st = qa_append(ctx_, seq_, layer, 1, pos, n, q, k, v, q_rows);
            if (st == QA_OK)
                st = pass_verify_ ? qa_attn_decode(ctx_, seq_, layer, 1, pos, n, q_rows, out)
                                  : qa_attn_prefill(ctx_, seq_, layer, 1, pos, n, q_rows, out);
            return st;
        });
        ++pass_layer_;
    }

    // Closes the pass after its last layer: prefill and step rows are committed; verify rows
    // become pending for commit_verified.
    void end_rows() {
        require(pass_rows_ > 0, "No layer pass is open");
        require(pass_layer_ == layers_, "Every layer must run before the pass ends");
        const int n = pass_rows_;
        const bool verify = pass_verify_;
        pass_rows_ = 0;
        if (verify) {
            verification_pending_ = true;
            return;
        }
        run([&] { return qa_commit(ctx_, seq_, n); });
    }

    bool layer_pass_open() const { return pass_rows_ > 0; }

    // Blocks until the queued work has finished; reports a device-side wait that expired.
    void sync() { run([&] { return qa_sync(ctx_); }); }

private:
    static void require(bool yes, const char* message) {
        if (!yes) throw std::runtime_error(message);
    }
    // Validation statuses leave the state as it was; anything else (CUDA, NCCL, an expired
    // device wait) resets the sequence, as the reference resets after an execution failure.
    void check(int st, bool reset_on_failure) {
        if (st == QA_OK) return;
        std::string msg = qa_last_error(ctx_);
        if (msg.empty()) msg = qa_status_string(st);
        const bool validation = st == QA_ERR_INVALID || st == QA_ERR_CAPACITY || st == QA_ERR_STATE;
        if (reset_on_failure && !validation) {
            qa_reset(ctx_, seq_);
            verification_pending_ = false;
            pass_rows_ = 0;
        }
        throw std::runtime_error(msg);
    }
    template <class F>
    void run(F&& work) {
        check(work(), true);
    }

    qa_ctx* ctx_ = nullptr;
    int seq_ = 0;
    int layers_ = 0;
    int context_ = 0;
    bool verification_pending_ = false;
    int pass_rows_ = 0, pass_layer_ = 0, pass_pos_ = 0;   // the open layer-by-layer pass
    bool pass_verify_ = false;
};

}  // namespace qattn_host
