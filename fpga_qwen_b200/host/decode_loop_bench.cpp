// decode_loop_bench.cpp — end-to-end decode timing from C++ through the C ABI with host buffers,
// in the two call patterns an x86 engine can use (built and run by bench.py; any host can
// build it the same way):
//   per layer  the engine's own order (tampajohn/fpga-qwen engine/core.cpp:383-645): per token,
//              28 qa_decode_step calls of one layer each (the projections would run between
//              them), then qa_commit;
//   fused      one qa_decode_step over all 28 layers per token (an engine that batches its
//              layers' attention).
// The buffers are std::vector (pageable), as Model::Impl holds its activations. The context
// first takes a 3968-row history (appended layer by layer, then committed); each pattern then
// decodes 128 tokens from there. Prints one JSON line: microseconds per token of each pattern.
//
//   g++ -O2 -std=c++17 -I include fpga_qwen_b200/host/decode_loop_bench.cpp \
//       -L fpga_qwen_b200 -lqattn -Wl,-rpath,fpga_qwen_b200 -o decode_loop_bench
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "qattn.h"

namespace {

constexpr int L = 28, HQ = 16, HKV = 8, D = 128, PREFILL = 3968, TOKENS = 128;

struct Rng {
    uint64_t s;
    float next() {            // uniform in [-2, 2): xorshift64, top 24 bits
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        return (float)(s >> 40) * (4.0f / 16777216.0f) - 2.0f;
    }
};

void check(int st, qa_ctx* ctx, const char* what) {
    if (st != QA_OK) {
        std::fprintf(stderr, "%s: %s\n", what, ctx ? qa_last_error(ctx) : qa_status_string(st));
        std::exit(1);
    }
}

void fill(std::vector<float>& v, Rng& r) {
    for (float& x : v) x = r.next();
}

// the 3968-row history, one layer per call (65 MB of host rows per layer)
void prefill(qa_ctx* ctx, Rng& r) {
    check(qa_reset(ctx, 0), ctx, "reset");
    std::vector<float> q((size_t)PREFILL * HQ * D), k((size_t)PREFILL * HKV * D), v(k.size()), qn(q.size());
    for (int l = 0; l < L; ++l) {
        fill(q, r); fill(k, r); fill(v, r);
        check(qa_append(ctx, 0, l, 1, 0, PREFILL, q.data(), k.data(), v.data(), qn.data()), ctx, "append");
    }
    check(qa_commit(ctx, 0, PREFILL), ctx, "commit");
}

double seconds_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

int main() {
    qa_config cfg;
    qa_default_config(&cfg);
    cfg.io_host = 1;
    qa_ctx* ctx = nullptr;
    check(qa_create(&cfg, &ctx), nullptr, "create");
    Rng r{0x9e3779b97f4a7c15ull};
    std::vector<float> qw(D), kw(D);
    for (int l = 0; l < L; ++l) {
        for (int j = 0; j < D; ++j) { qw[j] = 1.0f + 0.05f * r.next(); kw[j] = 1.0f + 0.05f * r.next(); }
        check(qa_set_norms(ctx, l, qw.data(), kw.data()), ctx, "norms");
    }
    // per-token rows of every layer: [token][layer][heads][128]
    std::vector<float> tq((size_t)TOKENS * L * HQ * D), tk((size_t)TOKENS * L * HKV * D), tv(tk.size());
    fill(tq, r); fill(tk, r); fill(tv, r);
    std::vector<float> out((size_t)L * HQ * D);

    double per_layer = 0, fused = 0;
    for (int rep = 0; rep < 2; ++rep) {               // the first pass of each pattern warms up
        prefill(ctx, r);
        auto t0 = std::chrono::steady_clock::now();
        for (int s = 0; s < TOKENS; ++s) {
            for (int l = 0; l < L; ++l) {
                const size_t o = (size_t)s * L + l;
                check(qa_decode_step(ctx, 0, l, 1, PREFILL + s, &tq[o * HQ * D], &tk[o * HKV * D], &tv[o * HKV * D],
                                     nullptr, &out[(size_t)l * HQ * D]),
                      ctx, "decode_step (one layer)");
            }
            check(qa_commit(ctx, 0, 1), ctx, "commit");
        }
        per_layer = seconds_since(t0);
        prefill(ctx, r);
        t0 = std::chrono::steady_clock::now();
        for (int s = 0; s < TOKENS; ++s) {
            // a token's rows of all layers are contiguous: the layer-major layout of a 28-layer call
            const size_t o = (size_t)s * L;
            check(qa_decode_step(ctx, 0, 0, L, PREFILL + s, &tq[o * HQ * D], &tk[o * HKV * D], &tv[o * HKV * D], nullptr,
                                 out.data()),
                  ctx, "decode_step (28 layers)");
            check(qa_commit(ctx, 0, 1), ctx, "commit");
        }
        fused = seconds_since(t0);
    }
    std::printf("{\"per_layer_us_per_token\": %.2f, \"fused_us_per_token\": %.2f, \"tokens\": %d, \"context\": %d}\n",
                per_layer / TOKENS * 1e6, fused / TOKENS * 1e6, TOKENS, PREFILL);
    qa_destroy(ctx);
    return 0;
}
