// Test driver for fpga_qwen_b200/host/attention_model.hpp (built and run by
// tests/test_host_model.py).
//   host_model_main nogpu           constructing a model where no GPU is usable throws
//                                   std::runtime_error (prints "caught: ...", exit 0)
//   host_model_main gpu <out.bin>   4 layers, context 512, host buffers: prefill 85 rows,
//                                   3 steps, verify_two, a step refused while verification is
//                                   pending, commit_verified(1), a refused and an accepted
//                                   truncate, one more step. Writes the norm weights and
//                                   every input and output (float32, in call order) for the
//                                   test to replay.
//   host_model_main engine <out.bin>
//                                   the engine's own loop (engine/core.cpp:383-645) with a
//                                   stand-in for the projections: per pass, every layer's q, k
//                                   and v are computed from a residual that the previous
//                                   layer's attention output updated, so layer l+1 depends on
//                                   layer l. Passes: prefill 85 rows, 3 decode steps, a
//                                   two-row verification committed by one; plus the refusals of
//                                   a layer out of order and of an all-layer call while a pass
//                                   is open. Writes the norm weights and, per pass, the
//                                   residual in and, per layer, q, k, v and the output.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "attention_model.hpp"

namespace {

constexpr int L = 4, HQ = 16, HKV = 8, D = 128;

struct Rng {
    uint64_t s;
    float next() {            // uniform in [-2, 2): xorshift64, top 24 bits
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        return (float)(s >> 40) * (4.0f / 16777216.0f) - 2.0f;
    }
};

struct Rows {
    std::vector<float> q, k, v, qn, out;
    Rows(int n, Rng& r) : q(size_t(L) * n * HQ * D), k(size_t(L) * n * HKV * D), v(k.size()), qn(q.size()), out(q.size()) {
        for (float& x : q) x = r.next();
        for (float& x : k) x = r.next();
        for (float& x : v) x = r.next();
    }
};

void dump(FILE* f, const std::vector<float>& a) { std::fwrite(a.data(), sizeof(float), a.size(), f); }

template <class F>
std::string refused(F&& f) {
    try {
        f();
    } catch (const std::runtime_error& e) {
        return e.what();
    }
    return "";
}

}  // namespace

// Stand-in for the engine's projections around attention (not the reference's arithmetic,
// only its data flow): q, k, v of layer l from the residual r [n][2048], and r += out / 2.
void project_stand_in(int layer, int n, const std::vector<float>& r, std::vector<float>& q, std::vector<float>& k,
                      std::vector<float>& v) {
    const float a = 1.0f + 0.01f * (float)layer, b = 0.001f * (float)layer;
    for (int i = 0; i < n * HQ * D; ++i) q[i] = r[i] * a + b;
    for (int row = 0; row < n; ++row)
        for (int i = 0; i < HKV * D; ++i) {
            k[size_t(row) * HKV * D + i] = r[size_t(row) * HQ * D + i] * 0.9f;
            v[size_t(row) * HKV * D + i] = r[size_t(row) * HQ * D + HKV * D + i] * 1.1f;
        }
}

int engine_mode(const char* path) {
    qattn_host::Options opt;
    opt.layers = L;
    opt.context = 512;
    opt.host_buffers = true;
    qattn_host::AttentionModel m(opt);
    FILE* f = std::fopen(path, "wb");
    if (!f) return 3;
    Rng rng{0xD1B54A32D192ED03ull};
    std::vector<float> qw(D), kw(D);
    for (int l = 0; l < L; ++l) {
        for (int j = 0; j < D; ++j) { qw[j] = 1.0f + 0.025f * rng.next(); kw[j] = 1.0f + 0.025f * rng.next(); }
        m.set_norms(l, qw.data(), kw.data());
        dump(f, qw); dump(f, kw);
    }
    std::string order_msg, open_msg;
    auto pass = [&](int n, bool verify) {
        std::vector<float> r(size_t(n) * HQ * D), q(r.size()), qn(r.size()), out(r.size());
        std::vector<float> k(size_t(n) * HKV * D), v(k.size());
        for (float& x : r) x = rng.next();
        dump(f, r);
        m.begin_rows(n, verify);
        for (int l = 0; l < L; ++l) {
            project_stand_in(l, n, r, q, k, v);
            if (l == 1 && order_msg.empty())
                order_msg = refused([&] { m.layer_rows(2, q.data(), k.data(), v.data(), qn.data(), out.data()); });
            if (l == 2 && open_msg.empty())
                open_msg = refused([&] { m.step(q.data(), k.data(), v.data(), out.data()); });
            m.layer_rows(l, q.data(), k.data(), v.data(), n == 1 ? nullptr : qn.data(), out.data());
            dump(f, q); dump(f, k); dump(f, v); dump(f, out);
            for (size_t i = 0; i < r.size(); ++i) r[i] = r[i] + 0.5f * out[i];     // stand-in o_proj + residual
        }
        m.end_rows();
    };
    pass(85, false);
    const int pos_prefill = m.position();
    for (int s = 0; s < 3; ++s) pass(1, false);
    const int pos_steps = m.position();
    pass(2, true);
    const bool pending = m.verification_pending();
    m.commit_verified(1);
    std::fclose(f);
    m.sync();
    std::printf("positions %d %d %d %d\n", pos_prefill, pos_steps, pending ? 1 : 0, m.position());
    std::printf("order_msg %s\n", order_msg.c_str());
    std::printf("open_msg %s\n", open_msg.c_str());
    return 0;
}

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "";
    if (mode == "engine" && argc > 2) return engine_mode(argv[2]);
    if (mode == "nogpu") {
        try {
            qattn_host::AttentionModel m(qattn_host::Options{});
        } catch (const std::runtime_error& e) {
            std::printf("caught: %s\n", e.what());
            return 0;
        }
        std::printf("no exception\n");
        return 1;
    }
    if (mode != "gpu" || argc < 3) return 2;
    qattn_host::Options opt;
    opt.layers = L;
    opt.context = 512;
    opt.host_buffers = true;
    qattn_host::AttentionModel m(opt);
    FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 3;
    Rng r{0x9E3779B97F4A7C15ull};
    std::vector<float> qw(D), kw(D);
    for (int l = 0; l < L; ++l) {
        for (int j = 0; j < D; ++j) { qw[j] = 1.0f + 0.025f * r.next(); kw[j] = 1.0f + 0.025f * r.next(); }
        m.set_norms(l, qw.data(), kw.data());
        dump(f, qw); dump(f, kw);
    }
    Rows pre(85, r);
    m.prefill(85, pre.q.data(), pre.k.data(), pre.v.data(), pre.qn.data(), pre.out.data());
    dump(f, pre.q); dump(f, pre.k); dump(f, pre.v); dump(f, pre.out);
    for (int s = 0; s < 3; ++s) {
        Rows st(1, r);
        m.step(st.q.data(), st.k.data(), st.v.data(), st.out.data());
        dump(f, st.q); dump(f, st.k); dump(f, st.v); dump(f, st.out);
    }
    Rows ver(2, r);
    const int base = m.verify_two(ver.q.data(), ver.k.data(), ver.v.data(), ver.qn.data(), ver.out.data());
    dump(f, ver.q); dump(f, ver.k); dump(f, ver.v); dump(f, ver.out);
    Rows blocked(1, r);
    const std::string pending_msg =
        refused([&] { m.step(blocked.q.data(), blocked.k.data(), blocked.v.data(), blocked.out.data()); });
    const int pos_pending = m.position();
    m.commit_verified(1);
    const int pos_commit = m.position();
    const std::string rewind_msg = refused([&] { m.truncate(200); });
    m.truncate(50);
    Rows last(1, r);
    m.step(last.q.data(), last.k.data(), last.v.data(), last.out.data());
    dump(f, last.q); dump(f, last.k); dump(f, last.v); dump(f, last.out);
    std::fclose(f);
    m.sync();
    std::printf("base %d pending_pos %d commit_pos %d final_pos %d\n", base, pos_pending, pos_commit, m.position());
    std::printf("pending_msg %s\n", pending_msg.c_str());
    std::printf("rewind_msg %s\n", rewind_msg.c_str());
    return 0;
}
