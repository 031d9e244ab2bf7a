// qattn_oracle.cpp — CPU restatement of the reference's attention + KV-cache path.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA library and the
// timed CPU baseline. Nothing in the shipped library links, loads or calls it; only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm do.
//
// What it restates (tampajohn/fpga-qwen, engine/core.cpp):
//   * norm            core.cpp:207-215  FP32 squares summed in FP64, one FP32 rounding,
//                                       inv = 1/sqrt(sum/n + 1e-6), out = (x*inv)*w
//   * rope            core.cpp:216-218  rotate-half over (j, j+64)
//   * RoPE tables     core.cpp:287-288  angle = p / 1e6^(2j/128) in FP64, cos/sin -> FP32
//   * KV write        core.cpp:399-405  K and V rounded to FP16 (round-to-nearest-even)
//   * dot             core.cpp:119-127  two 4-lane FMA accumulators (channels j..j+3 and
//                                       j+4..j+7, j ascending by 8), lane-wise add, then
//                                       (c0+c1)+(c2+c3)
//   * attention       core.cpp:606-624 (decode) and :407-605 (batched prefill; per output
//                                       the same formula, :128-130, :148-149, :548-550):
//                     s_t = dot(q,K_t) * (1/sqrt(128)); m = max s; e_t = exp(s_t - m);
//                     sum = sequential ascending FP32 sum; p_t = e_t/sum;
//                     out_j = fma(p_t, V_tj, out_j) ascending t.
//   * Pool partitions core.cpp:68 (count*i/n), prefill cost balance core.cpp:357-381.
//   * projections     core.cpp:292-301  y[b][r] = x[b] . W[r] over an FP16 matrix: one row
//                                       (or a matrix without an FP32 copy, :267) through the
//                                       eight-lane dot of :119-127 (dot4 :131-147 keeps the
//                                       order per row); batches over a layer matrix through
//                                       cblas_sgemm on the exact FP32 widening (:294)
//   * MLP gate        core.cpp:636-639  g * (0.5 + 0.5*tanh(g*0.5)) * up
//
// Substitutions, stated: the reference calls Apple Accelerate vvexpf (core.cpp:441,617);
// this file calls glibc expf. Likewise glibc tanhf for vvtanhf (:638), and for cblas_sgemm
// (:294), whose summation order Accelerate does not publish, an ascending-column FP32 sum
// (parity with those by tolerance). NEON intrinsics become x86 FMA/F16C intrinsics with the same
// lane-wise semantics (vfmaq_f32 == fused multiply-add per lane; vcvt_f32_f16 is exact).
// The reference's RoPE is built with -ffp-contract=fast (tools/build_native_cpu.py:45-46),
// which leaves fusion to the compiler; this restatement is compiled with
// -ffp-contract=off so RoPE is the explicit unfused form (two products, one add/sub),
// the same form the reference's NumPy oracle uses (tests/test_full_model.py:45-50).
//
// Parity pin: no golden attention vectors are committed in the reference; this file is
// checked against the reference's own NumPy oracle (tests/test_full_model.py:44-71),
// imported and run in the build container on synthetic weights, through the fixtures
// under tests/golden/ (see tests/golden/make_golden.py), plus known-answer tests.
#include <immintrin.h>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <thread>
#include <vector>

namespace {
constexpr int D = 128;

// ---- FP16 <-> FP32 ---------------------------------------------------------------
// float -> half, round to nearest even, written from the IEEE 754 binary16 definition.
inline uint16_t f32_to_f16(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mag = x & 0x7fffffffu;
    if (mag >= 0x7f800000u) {                       // inf / nan
        return uint16_t(sign | 0x7c00u | (mag > 0x7f800000u ? 0x200u : 0u));
    }
    if (mag >= 0x477ff000u) return uint16_t(sign | 0x7c00u);   // rounds to >= 65520 -> inf
    if (mag < 0x38800000u) {                        // result is subnormal (or zero)
        if (mag < 0x33000000u) return uint16_t(sign);          // < 2^-25: rounds to 0
        const uint32_t e = mag >> 23;                 // biased exponent, 102..112
        const uint32_t m = (mag & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;               // 14..24
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return uint16_t(sign | h);
    }
    // normal: rebias exponent 127 -> 15, keep 10 mantissa bits with RNE
    uint32_t h = ((mag >> 13) - ((127 - 15) << 10));
    const uint32_t rem = mag & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return uint16_t(sign | h);
}
inline float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu, x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {                                       // subnormal half -> normal float
            int s = 0; while (!(m & 0x400u)) { m <<= 1; ++s; }
            x = sign | (uint32_t(113 - s) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e + 112) << 23) | (m << 13);
    float f; std::memcpy(&f, &x, 4); return f;
}

// ---- restated scalar pieces ---------------------------------------------------------
// core.cpp:207-215
void norm(const float* x, const float* w, float* out, int n) {
    double precise_sum = 0;
    for (int j = 0; j < n; ++j) { const float square = x[j] * x[j]; precise_sum += static_cast<double>(square); }
    const float sum = static_cast<float>(precise_sum);
    const float inv = 1.0f / std::sqrt(sum / n + 1e-6f);
    for (int j = 0; j < n; ++j) out[j] = (x[j] * inv) * w[j];
}
// core.cpp:216-218 (unfused; this TU is compiled with -ffp-contract=off)
void rope(float* x, const float* cs, const float* sn) {
    for (int j = 0; j < 64; ++j) { float a = x[j], b = x[j + 64]; x[j] = a * cs[j] - b * sn[j]; x[j + 64] = b * cs[j] + a * sn[j]; }
}
// core.cpp:119-127: lanes 0..3 of the 8-wide accumulator are NEON's `a`, lanes 4..7 are `b`.
inline float dot_f16(const float* q, const uint16_t* key) {
    __m256 acc = _mm256_setzero_ps();
    for (int j = 0; j < D; j += 8) {
        const __m256 k = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(key + j)));
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(q + j), k, acc);
    }
    const __m128 c = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    alignas(16) float l[4]; _mm_store_ps(l, c);
    return (l[0] + l[1]) + (l[2] + l[3]);
}
// The same eight-lane order over n columns (n % 8 == 0): one projection output (core.cpp:298-299).
inline float dot_f16_n(const float* x, const uint16_t* w, int n) {
    __m256 acc = _mm256_setzero_ps();
    for (int j = 0; j < n; j += 8) {
        const __m256 k = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(w + j)));
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(x + j), k, acc);
    }
    const __m128 c = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    alignas(16) float l[4]; _mm_store_ps(l, c);
    return (l[0] + l[1]) + (l[2] + l[3]);
}
// out[j] = fma(p, V[j], out[j]) for the 128 channels of one value row (core.cpp:620-621).
inline void axpy_f16(float p, const uint16_t* val, float* out) {
    const __m256 pv = _mm256_set1_ps(p);
    for (int j = 0; j < D; j += 8) {
        const __m256 v = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(val + j)));
        _mm256_storeu_ps(out + j, _mm256_fmadd_ps(v, pv, _mm256_loadu_ps(out + j)));
    }
}

// One query row over n keys: the per-output formula shared by decode (:606-624) and
// every batched-prefill variant (:407-605).
void attend_one(const float* q, const uint16_t* kplane, const uint16_t* vplane, int n,
                float* scores, float* out) {
    const float scale = 1.0f / std::sqrt(float(D));
    float maximum = -std::numeric_limits<float>::infinity();
    for (int t = 0; t < n; ++t) { float s = dot_f16(q, kplane + size_t(t) * D) * scale; scores[t] = s; maximum = std::max(maximum, s); }
    for (int t = 0; t < n; ++t) scores[t] = std::exp(scores[t] - maximum);   // vvexpf -> expf
    float sum = 0; for (int t = 0; t < n; ++t) sum += scores[t];
    std::fill(out, out + D, 0.0f);
    for (int t = 0; t < n; ++t) { const float prob = scores[t] / sum; axpy_f16(prob, vplane + size_t(t) * D, out); }
}

// ---- a small persistent pool with the reference's contiguous split (core.cpp:68) ----
class Pool {
    int n_ = 1;
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_start_, cv_done_;
    uint64_t gen_ = 0; int pending_ = 0; bool stop_ = false;
    size_t count_ = 0;
    const std::function<void(size_t, size_t, int)>* job_ = nullptr;
    void work(int i) {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(mu_);
            cv_start_.wait(lk, [&] { return stop_ || gen_ != seen; });
            if (stop_) return;
            seen = gen_;
            const size_t count = count_; auto* job = job_;
            lk.unlock();
            (*job)(count * i / n_, count * (i + 1) / n_, i);
            lk.lock();
            if (--pending_ == 0) cv_done_.notify_one();
        }
    }
public:
    explicit Pool(int n) : n_(std::max(1, n)) { for (int i = 1; i < n_; ++i) threads_.emplace_back([this, i] { work(i); }); }
    ~Pool() { { std::lock_guard<std::mutex> lk(mu_); stop_ = true; } cv_start_.notify_all(); for (auto& t : threads_) t.join(); }
    int size() const { return n_; }
    void run(size_t count, const std::function<void(size_t, size_t, int)>& fn) {
        {
            std::lock_guard<std::mutex> lk(mu_);
            job_ = &fn; count_ = count; pending_ = n_ - 1; ++gen_;
        }
        cv_start_.notify_all();
        fn(0, count / n_, 0);
        std::unique_lock<std::mutex> lk(mu_);
        cv_done_.wait(lk, [&] { return pending_ == 0; });
        job_ = nullptr;
    }
};
std::mutex g_pool_mu;
Pool* g_pool = nullptr;
Pool& pool_for(int threads) {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (!g_pool || g_pool->size() != std::max(1, threads)) { delete g_pool; g_pool = new Pool(threads); }
    return *g_pool;
}
}  // namespace

extern "C" {

// RoPE tables [context][64] (core.cpp:287-288).
void qo_rope_tables(int context, float* cosines, float* sines) {
    for (int p = 0; p < context; ++p)
        for (int j = 0; j < 64; ++j) {
            double angle = p / std::pow(1000000.0, 2.0 * j / D);
            cosines[p * 64 + j] = float(std::cos(angle));
            sines[p * 64 + j] = float(std::sin(angle));
        }
}
void qo_norm(const float* x, const float* w, float* out, int n) { norm(x, w, out, n); }
void qo_rope(float* x, const float* cs, const float* sn) { rope(x, cs, sn); }
void qo_f32_to_f16(const float* x, uint16_t* h, size_t n) { for (size_t i = 0; i < n; ++i) h[i] = f32_to_f16(x[i]); }
void qo_f16_to_f32(const uint16_t* h, float* x, size_t n) { for (size_t i = 0; i < n; ++i) x[i] = f16_to_f32(h[i]); }

// KV append for one layer (core.cpp:395-406): rows b in [0,n) at absolute position pos0+b.
// q_pre [n][hq][128], k_pre/v_pre [n][hkv][128] FP32; qw/kw [128]; tables [ctx][64].
// Writes q_out [n][hq][128] (normed + roped) and kplane/vplane [hkv][ctx][128] FP16 bits.
void qo_append(int hq, int hkv, int ctx, int pos0, int n,
               const float* q_pre, const float* k_pre, const float* v_pre,
               const float* qw, const float* kw, const float* cosines, const float* sines,
               float* q_out, uint16_t* kplane, uint16_t* vplane) {
    std::vector<float> a(D);
    for (int b = 0; b < n; ++b) {
        const float* cs = cosines + size_t(pos0 + b) * 64; const float* sn = sines + size_t(pos0 + b) * 64;
        for (int h = 0; h < hq; ++h) {
            const float* src = q_pre + (size_t(b) * hq + h) * D; float* dst = q_out + (size_t(b) * hq + h) * D;
            norm(src, qw, dst, D); rope(dst, cs, sn);
        }
        for (int h = 0; h < hkv; ++h) {
            norm(k_pre + (size_t(b) * hkv + h) * D, kw, a.data(), D); rope(a.data(), cs, sn);
            const size_t dst = (size_t(h) * ctx + pos0 + b) * D;
            const float* vs = v_pre + (size_t(b) * hkv + h) * D;
            for (int j = 0; j < D; ++j) { kplane[dst + j] = f32_to_f16(a[j]); vplane[dst + j] = f32_to_f16(vs[j]); }
        }
    }
}

// Attention for one layer: row b (absolute position pos0+b) of every query head sees keys
// [0, pos0+b]. q [n][hq][128] FP32, planes [hkv][ctx][128] FP16, out [n][hq][128] FP32.
// GQA: query head h reads kv head h/(hq/hkv) (core.cpp:610). With threads > 1, work is
// split like the reference: n == 1 -> items (token, q-head) (:606); n > 1 -> items
// (row pair, kv head) with the causal-cost balanced ranges of :357-381. Per output the
// arithmetic is identical in both, so results do not depend on threads.
void qo_attention(int hq, int hkv, int ctx, int pos0, int n, const float* q,
                  const uint16_t* kplane, const uint16_t* vplane, float* out, int threads) {
    const int group = hq / hkv;
    Pool& pool = pool_for(threads);
    const int workers = pool.size();
    std::vector<float> scratch(size_t(workers) * (pos0 + n));
    const size_t stride = size_t(pos0 + n);
    if (n == 1) {
        pool.run(size_t(hq), [&](size_t begin, size_t end, int worker) {
            float* sc = scratch.data() + worker * stride;
            for (size_t item = begin; item < end; ++item) {
                const int h = int(item), kh = h / group;
                attend_one(q + size_t(h) * D, kplane + size_t(kh) * ctx * D, vplane + size_t(kh) * ctx * D,
                           pos0 + 1, sc, out + size_t(h) * D);
            }
        });
        return;
    }
    const size_t items = size_t((n + 1) / 2) * hkv;
    auto prefix_cost = [&](size_t item) -> uint64_t {
        const uint64_t b = std::min(uint64_t(n), uint64_t(2) * (item / hkv)), head = item % hkv;
        const uint64_t preceding = b * (uint64_t(2) * pos0 + b + 1) / 2;
        const uint64_t cost = pos0 + b + 1 + (b + 1 < uint64_t(n) ? pos0 + b + 2 : 0);
        return hkv * preceding + head * cost;
    };
    std::vector<size_t> ranges(workers + 1, 0);
    ranges[workers] = items;
    const uint64_t total = prefix_cost(items);
    for (int w = 1; w < workers; ++w) {
        const uint64_t target = total * w / workers;
        size_t lo = 0, hi = items;
        while (lo < hi) { const size_t mid = lo + (hi - lo) / 2; if (prefix_cost(mid) < target) lo = mid + 1; else hi = mid; }
        ranges[w] = lo;
    }
    pool.run(items, [&](size_t, size_t, int worker) {
        float* sc = scratch.data() + worker * stride;
        for (size_t item = ranges[worker]; item < ranges[worker + 1]; ++item) {
            const int b0 = 2 * int(item / hkv), kh = int(item % hkv);
            for (int b = b0; b < std::min(n, b0 + 2); ++b)
                for (int g = 0; g < group; ++g) {
                    const int h = kh * group + g;
                    attend_one(q + (size_t(b) * hq + h) * D, kplane + size_t(kh) * ctx * D,
                               vplane + size_t(kh) * ctx * D, pos0 + b + 1, sc, out + (size_t(b) * hq + h) * D);
                }
        }
    });
}

// Projection through an FP16 matrix w [rows][cols] (cols % 8 == 0): x [batch][cols] FP32 ->
// y [batch][rows] FP32 (core.cpp:292-301). sgemm == 0: the eight-lane dot per output, as for
// one row or the FP16-only embedding/vocabulary matrix; sgemm != 0 (batch > 1 over a layer
// matrix): FP32 products of the widened weights summed in ascending column order.
void qo_project(const float* x, const uint16_t* w, int rows, int cols, int batch, int sgemm, float* y,
                int threads) {
    Pool& pool = pool_for(threads);
    pool.run(size_t(batch) * rows, [&](size_t begin, size_t end, int) {
        for (size_t i = begin; i < end; ++i) {
            const size_t b = i / rows, r = i % rows;
            const float* xb = x + b * cols;
            const uint16_t* wr = w + r * cols;
            if (!sgemm) { y[i] = dot_f16_n(xb, wr, cols); continue; }
            float acc = 0.f;
            for (int j = 0; j < cols; ++j) acc = std::fma(xb[j], f16_to_f32(wr[j]), acc);
            y[i] = acc;
        }
    });
}

// The MLP gate of core.cpp:636-639 in place over n values: g = g * (0.5 + 0.5*tanh(g*0.5)) * up.
void qo_mlp_gate(float* gate, const float* up, size_t n) {
    for (size_t j = 0; j < n; ++j) {
        const float half = gate[j] * 0.5f;
        const float t = std::tanh(half);
        gate[j] = gate[j] * (0.5f + 0.5f * t) * up[j];
    }
}

void qo_release_pool() { std::lock_guard<std::mutex> lk(g_pool_mu); delete g_pool; g_pool = nullptr; }

}  // extern "C"
