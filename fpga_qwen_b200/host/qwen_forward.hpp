// qwen_forward.hpp — x86 host build of the reference engine's forward pass over libqattn.
//
// tampajohn/fpga-qwen engine/core.cpp's Model::Impl::chunk (:353-646), verify_chunk
// (:647-706) and append (:707-714), with the host keeping the reference's glue and the GPU
// doing the rest through the C ABI:
//   host   embedding lookup (:382-383), RMSNorm of the residual (norm, :207-215, with the
//          reference's FP64 sum of FP32 squares), residual adds (:626, :641), the MLP gate
//          g * (0.5 + 0.5 tanh(g/2)) * up (:636-639; std::tanh for Accelerate's vvtanhf);
//   GPU    every projection (qa_project / qa_project_group: q/k/v and gate/up grouped as at
//          :388-389, :629; the eight-lane dot per output, bit-exact with the reference's for one
//          row, for verification and for the FP16-only vocabulary head; prompt chunks of more
//          than one row take qa_project_gemm / qa_project_group_gemm on the tensor cores, where
//          the reference uses cblas_sgemm, :294), QK-RMSNorm + RoPE +
//          FP16 KV write and attention (AttentionModel's layer-by-layer pass: qa_append +
//          qa_attn_prefill / qa_attn_decode, or the fused qa_decode_step for one row).
// Layer l+1's projections consume layer l's attention output, exactly the engine's order; the
// position advances once per chunk after the last layer (:643). Prompts are processed in
// chunks of QA_PREFIX_CHUNK rows (the engine's prefill_chunk, core.hpp:10, core.cpp:712).
// Activations stay in host vectors as in Model::Impl (the context uses host buffers); the
// matrices are device pointers (uploaded once by the caller), the per-layer norm vectors and
// the embedding rows used for the lookup are host pointers.
//
// Header-only; link libqattn.so. C++17.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "attention_model.hpp"

namespace qattn_host {

struct LayerWeights {
    const uint16_t* q = nullptr;      // device FP16 [q_heads*128][hidden]
    const uint16_t* k = nullptr;      // device FP16 [kv_heads*128][hidden]
    const uint16_t* v = nullptr;      // device FP16 [kv_heads*128][hidden]
    const uint16_t* o = nullptr;      // device FP16 [hidden][q_heads*128]
    const uint16_t* gate = nullptr;   // device FP16 [intermediate][hidden]
    const uint16_t* up = nullptr;     // device FP16 [intermediate][hidden]
    const uint16_t* down = nullptr;   // device FP16 [hidden][intermediate]
    const float* input_norm = nullptr;      // host [hidden]
    const float* post_norm = nullptr;       // host [hidden]
    const float* q_norm = nullptr;          // host [128]
    const float* k_norm = nullptr;          // host [128]
};

struct ForwardWeights {
    int hidden = 1024, intermediate = 3072, vocab = 151936;
    const uint16_t* embed_device = nullptr;   // FP16 [vocab][hidden], the tied output head
    const uint16_t* embed_host = nullptr;     // the same rows in host memory, for the lookup
    const float* final_norm = nullptr;        // host [hidden]
    std::vector<LayerWeights> layers;
};

class QwenForward {
public:
    QwenForward(const ForwardWeights& weights, Options options) : w_(weights), attn_(with_host_buffers(options)) {
        const int L = attn_.layers();
        if ((int)w_.layers.size() != L) throw std::runtime_error("Layer count differs from the weights");
        for (int l = 0; l < L; ++l) attn_.set_norms(l, w_.layers[l].q_norm, w_.layers[l].k_norm);
        qd_ = 16 * 128;
        kd_ = 8 * 128;
    }

    int position() const { return attn_.position(); }
    void reset() { attn_.reset(); }
    void truncate(int position) { attn_.truncate(position); }

    // Model::prefill / Model::step: the logits of the last row (core.cpp:707-714).
    std::vector<float> prefill(const std::vector<int>& ids) {
        if (ids.empty()) throw std::runtime_error("Empty token input");
        for (int id : ids) check_id(id);
        std::vector<float> hidden;
        for (size_t begin = 0; begin < ids.size(); begin += QA_PREFIX_CHUNK) {
            const int n = (int)std::min<size_t>(QA_PREFIX_CHUNK, ids.size() - begin);
            hidden = chunk(ids.data() + begin, n, false);
        }
        return logits(hidden.data(), 1);
    }
    std::vector<float> step(int id) { return prefill(std::vector<int>{id}); }

    // Model::verify_two: both rows' logits [2][vocab]; the rows wait for commit_verified.
    std::vector<float> verify_two(int first, int second) {
        check_id(first);
        check_id(second);
        const int ids[2] = {first, second};
        const std::vector<float> hidden = chunk(ids, 2, true);
        return logits(hidden.data(), 2);
    }
    void commit_verified(int count) { attn_.commit_verified(count); }

private:
    static Options with_host_buffers(Options o) {
        o.host_buffers = true;
        return o;
    }
    void check_id(int id) const {
        if (id < 0 || id >= w_.vocab) throw std::runtime_error("Token ID out of range");
    }
    void run(int st) {
        if (st != QA_OK) throw std::runtime_error(qa_last_error(attn_.context()));
    }
    // core.cpp:207-215: FP32 squares summed in FP64, one FP32 rounding, (x * inv) * w.
    static void norm(const float* x, const float* w, float* out, int n) {
        double precise = 0;
        for (int j = 0; j < n; ++j) {
            const float square = x[j] * x[j];
            precise += static_cast<double>(square);
        }
        const float sum = static_cast<float>(precise);
        const float inv = 1.0f / std::sqrt(sum / n + 1e-6f);
        for (int j = 0; j < n; ++j) out[j] = (x[j] * inv) * w[j];
    }

    // n new rows through every layer; returns the final-normed hidden rows the caller needs
    // (the last row, or both rows of a verification).
    std::vector<float> chunk(const int* ids, int n, bool verify) {
        const int H = w_.hidden, F = w_.intermediate, L = attn_.layers();
        x_.assign((size_t)n * H, 0.f);
        for (int b = 0; b < n; ++b)
            for (int j = 0; j < H; ++j) x_[(size_t)b * H + j] = half_to_float(w_.embed_host[(size_t)ids[b] * H + j]);
        h_.resize(x_.size()); q_.resize((size_t)n * qd_); k_.resize((size_t)n * kd_); v_.resize(k_.size());
        qrows_.resize(q_.size()); att_.resize(q_.size()); res_.resize(x_.size());
        gate_.resize((size_t)n * F); up_.resize(gate_.size());
        qa_ctx* ctx = attn_.context();
        attn_.begin_rows(n, verify);
        try {
            layers(ctx, n, H, F, L, n > 1 && !verify);
        } catch (...) {
            attn_.reset();                 // as Model::verify_two / commit_verified do (core.cpp:740, :751)
            throw;
        }
        attn_.end_rows();
        const int first = verify ? 0 : n - 1, count = verify ? 2 : 1;
        std::vector<float> hidden((size_t)count * H);
        for (int b = 0; b < count; ++b) norm(&x_[(size_t)(first + b) * H], w_.final_norm, &hidden[(size_t)b * H], H);
        return hidden;
    }

    // batched: a prompt chunk (core.cpp:294's sgemm); otherwise one row or a verification pair
    void layers(qa_ctx* ctx, int n, int H, int F, int L, bool batched) {
        auto project = [&](const uint16_t* w, int rows, int cols, const float* x, float* y) {
            run(batched ? qa_project_gemm(ctx, w, rows, cols, x, n, y) : qa_project(ctx, w, rows, cols, x, n, y));
        };
        auto project_group = [&](int k, const uint16_t* const* ws, const int* rows, int cols, const float* x,
                                 float* const* ys) {
            run(batched ? qa_project_group_gemm(ctx, k, ws, rows, cols, x, n, ys)
                        : qa_project_group(ctx, k, ws, rows, cols, x, n, ys));
        };
        for (int l = 0; l < L; ++l) {
            const LayerWeights& lw = w_.layers[l];
            for (int b = 0; b < n; ++b) norm(&x_[(size_t)b * H], lw.input_norm, &h_[(size_t)b * H], H);
            {
                const uint16_t* ws[3] = {lw.q, lw.k, lw.v};
                const int rows[3] = {qd_, kd_, kd_};
                float* ys[3] = {q_.data(), k_.data(), v_.data()};
                project_group(3, ws, rows, H, h_.data(), ys);
            }
            attn_.layer_rows(l, q_.data(), k_.data(), v_.data(), n == 1 ? nullptr : qrows_.data(), att_.data());
            project(lw.o, H, qd_, att_.data(), res_.data());
            for (size_t j = 0; j < x_.size(); ++j) x_[j] += res_[j];
            for (int b = 0; b < n; ++b) norm(&x_[(size_t)b * H], lw.post_norm, &h_[(size_t)b * H], H);
            {
                const uint16_t* ws[2] = {lw.gate, lw.up};
                const int rows[2] = {F, F};
                float* ys[2] = {gate_.data(), up_.data()};
                project_group(2, ws, rows, H, h_.data(), ys);
            }
            for (size_t j = 0; j < gate_.size(); ++j) {
                const float t = std::tanh(gate_[j] * 0.5f);
                gate_[j] = gate_[j] * (0.5f + 0.5f * t) * up_[j];
            }
            project(lw.down, H, F, gate_.data(), res_.data());
            for (size_t j = 0; j < x_.size(); ++j) x_[j] += res_[j];
        }
    }

    // The tied vocabulary head over the FP16 embedding matrix (core.cpp:705, :713).
    std::vector<float> logits(const float* hidden, int rows) {
        std::vector<float> out((size_t)rows * w_.vocab);
        run(qa_project(attn_.context(), w_.embed_device, w_.vocab, w_.hidden, hidden, rows, out.data()));
        return out;
    }

    static float half_to_float(uint16_t h) {
        const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1f, mant = h & 0x3ffu;
        uint32_t bits;
        if (exp == 0) {
            if (mant == 0) {
                bits = sign;
            } else {                                   // subnormal: normalise
                int e = -1;
                uint32_t m = mant;
                do { ++e; m <<= 1; } while (!(m & 0x400u));
                bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
            }
        } else if (exp == 31) {
            bits = sign | 0x7f800000u | (mant << 13);
        } else {
            bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
        }
        float f;
        std::memcpy(&f, &bits, 4);
        return f;
    }

    ForwardWeights w_;
    AttentionModel attn_;
    int qd_ = 0, kd_ = 0;
    std::vector<float> x_, h_, q_, k_, v_, qrows_, att_, res_, gate_, up_;
};

}  // namespace qattn_host
