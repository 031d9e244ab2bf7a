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

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "";
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
