// attn_decode_sm100.cu — decode / verify attention streamed from HBM by the TMA engine.
//
// Replaces the reference's single-token decode attention (tampajohn/fpga-qwen
// engine/core.cpp:606-624) and the B2 verify attention (:671-689): for each of the n new
// rows b (position pos0+b, context pos0+b+1) and query head h,
// out = softmax(q.K^T / sqrt(128)) V over the KV head h/2 of every requested layer.
//
// Decode is bound by HBM bandwidth: at 4K context one step reads 470 MB of FP16 K/V for
// 57 KFLOP-per-row of arithmetic. The kernel is built to keep HBM busy:
//   * Even work split (stream-K style). The keys of all (layer, row, KV head) units are laid
//     end to end and cut into C equal ranges, C a multiple of the SM count; CTA c takes range
//     c. A range can end inside one unit and continue in the next, so every CTA gets the
//     same number of keys and there is no tail wave.
//   * TMA bulk copies. K and V rows of one (layer, head) are contiguous, so a 64-key chunk
//     is one 16 KB cp.async.bulk. One thread keeps a 4-stage ring of chunks in flight
//     (64 KB per CTA, 2 CTAs per SM), so the CTA never waits on individual loads. The ring
//     runs over the CTA's whole chunk stream (segment after segment, K chunks then V chunks
//     of each), so it stays full across segment boundaries: a batched step over many short
//     sequences crosses dozens of them per CTA.
//   * Both GQA query heads share every K and V chunk (the reference pairs heads the same
//     way, core.cpp:150-159). Scores of the range stay in shared memory; the max and sum
//     over the range are exact; V is streamed after K.
// A range that covers a whole unit writes that unit's output directly. A unit split over
// several CTAs gets one (max, sum, 2x128 partial output) record per CTA; the last CTA to
// finish (one atomic counter, no waiting) merges them.
// Every wait is bounded (globaltimer): on expiry the CTA records an error code for the
// host, stops consuming, drains its outstanding copies and exits.
//
// Fused decode step (FUSED = true): the kernel also performs the append of the one new row
// per sequence (core.cpp:395-406 for a single token), so a decode step is one launch. Before
// its first segment the CTA normalises and rotates the query rows of every unit its range
// touches (at most FUSED_MAX_UNITS; the host falls back to append + decode otherwise) from the
// pre-norm input (norm_rope.cuh, the same arithmetic as kv_append, so q_out and the attention
// input are bit-identical to an append followed by a decode). Each row's sequential FP64 sum
// runs on its own lane, all rows at once, while the copy ring fills. The new row is the last
// key of its unit, so exactly one CTA reads it: that CTA builds the FP16 K and V rows, stores
// them in the KV store (and q_out), and patches them into the ring chunk that holds the stale
// row before scoring it.
#include <algorithm>

#include "norm_rope.cuh"
#include "qattn_common.cuh"
#include "sm100.cuh"

namespace qattn {
namespace {

using namespace sm100;

constexpr int THREADS = 128;                  // four warps (the merge's reductions read red[][0..3])
static_assert(THREADS == 128, "block reductions are written for four warps");
constexpr int HALF_WARPS = THREADS / 16;
constexpr int CH = 64;                        // keys per chunk
constexpr int NST = 4;                        // ring stages
constexpr uint32_t CHUNK_BYTES = CH * D * 2;  // 16 KB
constexpr int MAX_UNIT_KEYS = 4096;           // longest unit (QA_MAX_CONTEXT): a segment's scores fit in 2 x 16 KB
constexpr int FAST_MERGE = 4;                 // units split over at most this many CTAs merge in one load round

struct DecodeArgs {
    const float* q; float* out;               // [n_layers][n][hq][128]
    StepInputs step;                          // fused decode step only
    int pdl;                                  // launched as a programmatic dependent of the previous step
    GatherArgs g;                             // head gather through peer memory (out_hq == 0: off)
    KVLayout kv; int layer0, n_layers, n, hq, hkv;
    int seq[MAX_BATCH];                       // sequence slot of row b
    int pos[MAX_BATCH];                       // absolute position of row b (context pos+1)
    int start[MAX_BATCH + 1];                 // prefix sums of row context lengths
    long long total_keys;                     // T = Σ over units of their context length
    int ctas;                                 // C
    int max_keys;                             // max keys of one CTA range (scores capacity)
    int max_records;                          // records reserved per unit
    float* partial;                           // [units][max_records][PARTIAL_FLOATS]
    int* counters;                            // [units], zero between calls
    int* error;
};

struct Unit { int l, b, kh, len; long long off; };

// Unit containing global key g; units ordered (layer, row, KV head), unit (l, b, kh) holding
// keys [0, pos[b]] of row b's sequence.
__device__ __forceinline__ Unit unit_of(const DecodeArgs& a, long long g) {
    const long long layer_keys = (long long)a.hkv * a.start[a.n];
    Unit u;
    u.l = (int)(g / layer_keys);
    const long long r = g - (long long)u.l * layer_keys;
    int b = 0;
    while (b < a.n - 1 && (long long)a.hkv * a.start[b + 1] <= r) ++b;
    u.b = b;
    u.len = a.pos[b] + 1;
    const long long rr = r - (long long)a.hkv * a.start[b];
    u.kh = (int)(rr / u.len);
    u.off = (long long)u.l * layer_keys + (long long)a.hkv * a.start[b] + (long long)u.kh * u.len;
    return u;
}

// The unit after u in (layer, row, KV head) order, without divisions.
__device__ __forceinline__ void next_unit(const DecodeArgs& a, Unit& u) {
    u.off += u.len;
    if (++u.kh == a.hkv) {
        u.kh = 0;
        if (++u.b == a.n) { u.b = 0; ++u.l; }
        u.len = a.pos[u.b] + 1;
    }
}

// CTA whose range holds global key g: the largest c with floor(c*T/C) <= g.
__device__ __forceinline__ int cta_of(long long g, long long T, int C) { return (int)(((g + 1) * C - 1) / T); }

__device__ __forceinline__ void unpack8(const uint4 u, float f[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    #pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r, ua = *reinterpret_cast<unsigned long long*>(&a), ub = *reinterpret_cast<unsigned long long*>(&b),
                          uc = *reinterpret_cast<unsigned long long*>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(ua), "l"(ub), "l"(uc));
    return *reinterpret_cast<float2*>(&r);
}

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

template <bool FUSED>
__global__ void __launch_bounds__(THREADS, 2) attn_decode_sm100_kernel(const DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;                                              // NST x 16 KB
    float* scores = reinterpret_cast<float*>(smem + NST * CHUNK_BYTES);   // [GROUP][max_keys]
    __shared__ __align__(8) uint64_t full[NST];
    __shared__ float red[GROUP][THREADS / 32];
    __shared__ float stat[2 * GROUP];
    __shared__ __align__(16) float accbuf[HALF_WARPS][GROUP][D];
    __shared__ int is_last, abort_flag, never_abort;
    constexpr int QB = FUSED ? FUSED_MAX_UNITS : 1;
    __shared__ __align__(16) float s_q[QB][GROUP][D];      // fused: normalised query rows of unit i
    __shared__ __align__(16) __half s_new[QB][2][D];       // fused: the new K and V rows (FP16)
    __shared__ float s_inv[QB][3];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hw = tid >> 4, sl = tid & 15;
    const long long T = a.total_keys;
    const int C = a.ctas, c = blockIdx.x;
    const long long g_begin = (long long)c * T / C, g_end = (long long)(c + 1) * T / C;

    if (tid == 0) {
        abort_flag = 0; never_abort = 0;
        for (int s = 0; s < NST; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    uint32_t issued = 0, consumed = 0;                 // ring sequence numbers (thread 0 issues)
    const float qscale = 1.4426950408889634f * 0.08838834764831845f;   // log2(e)/sqrt(128)

    // Producer cursor (thread 0, in shared memory so that it holds no registers in the
    // consumer loop). The CTA's chunk stream is, segment after segment, the K chunks then the
    // V chunks of each segment (the part of one unit inside the range); the consumers walk
    // the same stream in the same order.
    __shared__ struct { Unit u; const __half* K; const __half* V; int j, nch, cnt, k0; } pc;
    // limited: before the previous step's grid has finished (programmatic dependent launch),
    // only chunks that hold neither that step's new row (key len-2 of its unit) nor this step's
    // (key len-1) may be copied; returns false, issuing nothing, at the first chunk that does.
    auto produce = [&](bool limited) {
        if (pc.j == 2 * pc.nch) {                      // next segment: the next unit from key 0
            next_unit(a, pc.u);
            if (pc.u.off >= g_end) return false;
            pc.cnt = (int)min((long long)pc.u.len, g_end - pc.u.off);
            pc.nch = (pc.cnt + CH - 1) / CH;
            pc.j = 0;
            pc.k0 = 0;
            const int layer = a.layer0 + pc.u.l;
            pc.K = a.kv.plane(a.seq[pc.u.b], layer, 0, pc.u.kh);
            pc.V = a.kv.plane(a.seq[pc.u.b], layer, 1, pc.u.kh);
        }
        const int stage = issued % NST;
        const bool is_v = pc.j >= pc.nch;
        const int jj = is_v ? pc.j - pc.nch : pc.j;
        const int keys = min(CH, pc.cnt - jj * CH);
        if (limited && pc.k0 + jj * CH + keys > pc.u.len - 2) return false;
        const __half* src = (is_v ? pc.V : pc.K) + (size_t)jj * CH * D;
        mbar_arrive_expect_tx(&full[stage], keys * D * 2);
        bulk_copy(ring + stage * CHUNK_BYTES, src, keys * D * 2, &full[stage]);
        ++issued;
        ++pc.j;
        return true;
    };
    Unit u = unit_of(a, g_begin);                      // consumers' unit cursor
    if (tid == 0) {
        // first segment: keys [g_begin - off, ...) of the unit holding g_begin
        const int k0 = (int)(g_begin - u.off);
        pc.u = u;
        pc.k0 = k0;
        pc.cnt = (int)min((long long)u.len, g_end - u.off) - k0;
        pc.nch = (pc.cnt + CH - 1) / CH;
        pc.j = 0;
        const int layer = a.layer0 + u.l;
        pc.K = a.kv.plane(a.seq[u.b], layer, 0, u.kh) + (size_t)k0 * D;
        pc.V = a.kv.plane(a.seq[u.b], layer, 1, u.kh) + (size_t)k0 * D;
        if (!FUSED)                                    // the fused kernel primes after its input copies
            for (int i = 0; i < NST && g_begin < g_end; ++i) produce(false);
    }

    if constexpr (FUSED) {
        // ---- append of the new rows of the units this range touches (i-th unit: unit_at(i)) ----
        auto unit_at = [&](int i) {
            Unit w = u;
            for (int k = 0; k < i; ++k) next_unit(a, w);
            return w;
        };
        // Inputs of unit i, staged in the score buffer (free until the first K chunk is scored,
        // so every ring stage streams K/V meanwhile; the launch sizes it for the staging):
        // [q0 | q1 | k | v | cos | sin | q_norm | k_norm] = 896 floats at i * 1024.
        float* stg = scores;
        // tables (RoPE rows, norm weights: constant during a step) or the step's inputs
        auto stage_inputs = [&](bool tables) {
            for (int i = 0; i < QB; ++i) {
                const Unit w = unit_at(i);
                if (w.off >= g_end) break;
                const bool owns = w.off + w.len <= g_end;
                const int layer = a.layer0 + w.l, pos = w.len - 1;
                const size_t qrow_w = ((size_t)w.l * a.n + w.b) * a.hq + (size_t)w.kh * GROUP;
                const size_t krow_w = ((size_t)w.l * a.n + w.b) * a.hkv + w.kh;
                for (int gidx = tid + (tables ? 128 : 0); gidx < (tables ? 224 : 128); gidx += THREADS) {
                    const float* src;                  // 16-byte granules
                    if (gidx < 64) src = a.step.q_pre + qrow_w * D + gidx * 4;
                    else if (gidx < 96) src = owns ? a.step.k_pre + krow_w * D + (gidx - 64) * 4 : nullptr;
                    else if (gidx < 128) src = owns ? a.step.v_pre + krow_w * D + (gidx - 96) * 4 : nullptr;
                    else if (gidx < 144) src = a.step.cosines + (size_t)pos * 64 + (gidx - 128) * 4;
                    else if (gidx < 160) src = a.step.sines + (size_t)pos * 64 + (gidx - 144) * 4;
                    else if (gidx < 192) src = a.step.norms + (size_t)layer * 2 * D + (gidx - 160) * 4;
                    else src = owns ? a.step.norms + (size_t)layer * 2 * D + D + (gidx - 192) * 4 : nullptr;
                    if (src)
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                     ::"r"(smem_u32(stg + i * 1024 + gidx * 4)), "l"(src) : "memory");
                }
            }
        };
        stage_inputs(true);
        if (a.pdl) {
            // Launched while the previous step may still run: copy only KV rows it cannot be
            // writing, then wait for its grid (and its memory) before touching this step's
            // inputs, records and rows, and let the next step launch.
            if (tid == 0)
                for (int i = 0; i < NST && g_begin < g_end; ++i)
                    if (!produce(true)) break;
            asm volatile("griddepcontrol.wait;" ::: "memory");
        }
        // a following overlapped step may launch now (it waits for this grid before it reads
        // anything this step writes)
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        stage_inputs(false);
        if (tid == 0)                                  // K/V stream behind the small input copies
            while ((int)issued < NST && produce(false)) {}
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        if (tid < 3 * QB) {                            // one lane per sequential FP64 chain
            const int i = tid / 3, r = tid - 3 * i;    // rows: query head 0, query head 1, key
            const Unit w = unit_at(i);
            if (w.off < g_end && (r < 2 || w.off + w.len <= g_end)) s_inv[i][r] = rms_inv(stg + i * 1024 + r * 128, a.step.eps);
        }
        __syncthreads();
        {
            // thread t: channel pair j = t % 64 of rows {h, 2 + h} (h = t / 64) of every unit
            const int j = tid & 63, h = tid >> 6;
            for (int i = 0; i < QB; ++i) {
                const Unit w = unit_at(i);
                if (w.off >= g_end) break;
                const bool owns = w.off + w.len <= g_end;
                const float* u8 = stg + i * 1024;
                const float c = u8[512 + j], sn = u8[576 + j];
                float ra, rb;
                norm_rope_pair(u8[h * 128 + j], u8[h * 128 + j + 64], u8[640 + j], u8[640 + j + 64], c, sn, s_inv[i][h],
                               ra, rb);
                s_q[i][h][j] = ra;
                s_q[i][h][j + 64] = rb;
                if (owns) {
                    if (a.step.q_out) {
                        const size_t qrow_w = ((size_t)w.l * a.n + w.b) * a.hq + (size_t)w.kh * GROUP;
                        a.step.q_out[(qrow_w + h) * D + j] = ra;
                        a.step.q_out[(qrow_w + h) * D + j + 64] = rb;
                    }
                    if (h == 0) {                      // key row: norm + rope, FP16
                        norm_rope_pair(u8[256 + j], u8[256 + j + 64], u8[768 + j], u8[768 + j + 64], c, sn, s_inv[i][2],
                                       ra, rb);
                        s_new[i][0][j] = __float2half_rn(ra);
                        s_new[i][0][j + 64] = __float2half_rn(rb);
                    } else {                           // value row: FP16 rounding only
                        s_new[i][1][j] = __float2half_rn(u8[384 + j]);
                        s_new[i][1][j + 64] = __float2half_rn(u8[384 + j + 64]);
                    }
                }
            }
        }
        __syncthreads();                               // the staging is read: the score buffer is free
        if (tid < QB * 32) {                          // store the new K and V rows, 16 B per lane
            const int i = tid >> 5, kv = (tid >> 4) & 1, c16 = tid & 15;
            const Unit w = unit_at(i);
            if (w.off < g_end && w.off + w.len <= g_end) {
                __half* dst = a.kv.plane(a.seq[w.b], a.layer0 + w.l, kv, w.kh) + (size_t)(w.len - 1) * D;
                reinterpret_cast<uint4*>(dst)[c16] = reinterpret_cast<const uint4*>(s_new[i][kv])[c16];
            }
        }
    }

    // final output of (unit u, head gq of its pair, channel jc): this GPU's output buffer, or
    // every rank's landing buffer when gathering heads through peer memory
    auto store_out = [&](const Unit& uu, int gq, int jc, float val) {
        if (a.g.out_hq == 0) {
            a.out[((((size_t)uu.l * a.n + uu.b) * a.hq + (size_t)uu.kh * GROUP) + gq) * D + jc] = val;
        } else {
            const size_t o = ((((size_t)uu.l * a.n + uu.b) * a.g.out_hq + a.g.out_h0 + (size_t)uu.kh * GROUP) + gq) * D + jc;
            a.out[o] = val;
            for (int p = 0; p < a.g.n_peers; ++p) a.g.peer_out[p][o] = val;
        }
    };

    int si = -1;                                       // segment index within this range
    for (long long g = g_begin; g < g_end;) {
        if (g != g_begin) next_unit(a, u);
        ++si;
        if (FUSED && si >= QB) {                       // the host bounds units per range; never expected
            if (tid == 0) atomicCAS(a.error, 0, 42);
            break;
        }
        const int k0 = (int)(g - u.off);
        const int cnt = (int)min((long long)u.len, g_end - u.off) - k0;
        const int nch = (cnt + CH - 1) / CH;
        g = u.off + k0 + cnt;
        const int total_chunks = 2 * nch;                // K chunks then V chunks
        const size_t qrow = ((size_t)u.l * a.n + u.b) * a.hq + (size_t)u.kh * GROUP;

        // the segment ends at the unit's last key: in a fused step that is the new row
        const bool owns_new = FUSED && k0 + cnt == u.len;
        float q[GROUP][8];
        if constexpr (FUSED) {
            #pragma unroll
            for (int gq = 0; gq < GROUP; ++gq)
                #pragma unroll
                for (int e = 0; e < 8; ++e) q[gq][e] = s_q[si][gq][sl * 8 + e] * qscale;
        } else {
            #pragma unroll
            for (int gq = 0; gq < GROUP; ++gq) {
                const float4* src = reinterpret_cast<const float4*>(a.q + (qrow + gq) * D + sl * 8);
                const float4 x = __ldg(src), y = __ldg(src + 1);
                q[gq][0] = x.x * qscale; q[gq][1] = x.y * qscale; q[gq][2] = x.z * qscale; q[gq][3] = x.w * qscale;
                q[gq][4] = y.x * qscale; q[gq][5] = y.y * qscale; q[gq][6] = y.z * qscale; q[gq][7] = y.w * qscale;
            }
        }
        float mloc0 = -INFINITY, mloc1 = -INFINITY;
        float acc[GROUP][8];
        #pragma unroll
        for (int gq = 0; gq < GROUP; ++gq)
            #pragma unroll
            for (int e = 0; e < 8; ++e) acc[gq][e] = 0.f;

        bool aborted = false;
        for (int j = 0; j < total_chunks; ++j) {
            const int stage = consumed % NST;
            const uint32_t parity = (consumed / NST) & 1;
            bool got = mbar_wait(&full[stage], parity, &abort_flag);
            if (!got) { abort_flag = 1; atomicCAS(a.error, 0, 41); }
            got = __all_sync(0xffffffffu, got);           // warp-uniform: the shuffles below need all lanes
            uint8_t* buf = ring + stage * CHUNK_BYTES;
            const bool is_v = j >= nch;
            const int jj = is_v ? j - nch : j;
            const int keys = min(CH, cnt - jj * CH);
            if (owns_new && jj == nch - 1) {
                // the last chunk of each pass holds the new row, copied before it was written:
                // replace it with the row built above (CTA-uniform branch)
                if (tid < 16)
                    reinterpret_cast<uint4*>(buf + (keys - 1) * 256)[tid] = reinterpret_cast<const uint4*>(s_new[si][is_v])[tid];
                __syncthreads();
            }
            if (got) {
                if (!is_v) {
                    // ---- scores: half-warp hw takes keys hw, hw+8, hw+16, hw+24 (+32) ----
                    #pragma unroll
                    for (int half = 0; half < CH / (HALF_WARPS * 4); ++half) {
                        float v[8];
                        #pragma unroll
                        for (int uu = 0; uu < 4; ++uu) {
                            const int t = half * 32 + uu * HALF_WARPS + hw;
                            uint4 kr = make_uint4(0, 0, 0, 0);
                            if (t < keys) kr = *reinterpret_cast<const uint4*>(buf + t * 256 + sl * 16);
                            float kf[8]; unpack8(kr, kf);
                            #pragma unroll
                            for (int gq = 0; gq < GROUP; ++gq) {
                                // even/odd channel partial sums with packed FP32 FMA
                                float2 s2 = make_float2(0.f, 0.f);
                                #pragma unroll
                                for (int e = 0; e < 8; e += 2)
                                    s2 = ffma2(make_float2(q[gq][e], q[gq][e + 1]), make_float2(kf[e], kf[e + 1]), s2);
                                v[uu * GROUP + gq] = s2.x + s2.y;
                            }
                        }
                        // transpose-reduce over the 16 lanes of the half-warp (8 shuffles for 8 sums)
                        const bool b3 = sl & 8, b2 = sl & 4, b1 = sl & 2;
                        float w4[4], w2[2], y;
                        #pragma unroll
                        for (int i = 0; i < 4; ++i)
                            w4[i] = (b3 ? v[i + 4] : v[i]) + __shfl_xor_sync(0xffffffffu, b3 ? v[i] : v[i + 4], 8);
                        #pragma unroll
                        for (int i = 0; i < 2; ++i)
                            w2[i] = (b2 ? w4[i + 2] : w4[i]) + __shfl_xor_sync(0xffffffffu, b2 ? w4[i] : w4[i + 2], 4);
                        y = (b1 ? w2[1] : w2[0]) + __shfl_xor_sync(0xffffffffu, b1 ? w2[0] : w2[1], 2);
                        y += __shfl_xor_sync(0xffffffffu, y, 1);
                        const int my_u = (b3 ? 2 : 0) + (b2 ? 1 : 0), my_g = b1 ? 1 : 0;
                        const int t = half * 32 + my_u * HALF_WARPS + hw;
                        if (t < keys) {
                            if (my_g == 0) mloc0 = fmaxf(mloc0, y); else mloc1 = fmaxf(mloc1, y);
                            if ((sl & 1) == 0) scores[my_g * a.max_keys + jj * CH + t] = y;
                        }
                    }
                } else {
                    // ---- PV: half-warp hw takes value rows hw, hw+8, ... of the chunk ----
                    #pragma unroll 4
                    for (int t = hw; t < keys; t += HALF_WARPS) {
                        float vf[8];
                        unpack8(*reinterpret_cast<const uint4*>(buf + t * 256 + sl * 16), vf);
                        const float p0 = scores[jj * CH + t], p1 = scores[a.max_keys + jj * CH + t];
                        const float2 pp0 = make_float2(p0, p0), pp1 = make_float2(p1, p1);
                        #pragma unroll
                        for (int e = 0; e < 8; e += 2) {
                            const float2 v2 = make_float2(vf[e], vf[e + 1]);
                            float2 a0 = ffma2(pp0, v2, make_float2(acc[0][e], acc[0][e + 1]));
                            float2 a1 = ffma2(pp1, v2, make_float2(acc[1][e], acc[1][e + 1]));
                            acc[0][e] = a0.x; acc[0][e + 1] = a0.y; acc[1][e] = a1.x; acc[1][e + 1] = a1.y;
                        }
                    }
                }
            }
            ++consumed;
            __syncthreads();                       // everyone is done with this stage
            if (abort_flag) { aborted = true; break; }
            if (tid == 0) produce(false);          // refill the freed stage (next segment's chunks too)
            if (j == nch - 1) {
                // ---- end of the K pass: exact max and exp-sum over this range ----
                float m0 = mloc0, m1 = mloc1;
                #pragma unroll
                for (int off = 16; off >= 1; off >>= 1) {
                    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
                    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
                }
                if (lane == 0) { red[0][warp] = m0; red[1][warp] = m1; }
                __syncthreads();
                if (tid < GROUP) {
                    float m = red[tid][0];
                    #pragma unroll
                    for (int w = 1; w < THREADS / 32; ++w) m = fmaxf(m, red[tid][w]);
                    stat[tid] = m;
                }
                __syncthreads();
                float s0 = 0.f, s1 = 0.f;
                const float mm0 = stat[0], mm1 = stat[1];
                for (int t = tid; t < cnt; t += THREADS) {
                    const float p0 = exp2f(scores[t] - mm0), p1 = exp2f(scores[a.max_keys + t] - mm1);
                    scores[t] = p0; scores[a.max_keys + t] = p1;
                    s0 += p0; s1 += p1;
                }
                #pragma unroll
                for (int off = 16; off >= 1; off >>= 1) {
                    s0 += __shfl_xor_sync(0xffffffffu, s0, off);
                    s1 += __shfl_xor_sync(0xffffffffu, s1, off);
                }
                __syncthreads();                   // red reuse
                if (lane == 0) { red[0][warp] = s0; red[1][warp] = s1; }
                __syncthreads();
                if (tid < GROUP) {
                    float s = 0.f;
                    #pragma unroll
                    for (int w = 0; w < THREADS / 32; ++w) s += red[tid][w];
                    stat[GROUP + tid] = s;
                }
                __syncthreads();
            }
        }
        if (aborted) break;

        // ---- combine the 8 half-warps' partial PV sums ----
        #pragma unroll
        for (int gq = 0; gq < GROUP; ++gq)
            #pragma unroll
            for (int e = 0; e < 8; ++e) accbuf[hw][gq][sl * 8 + e] = acc[gq][e];
        __syncthreads();
        float o[GROUP * D / THREADS];
        #pragma unroll
        for (int i = 0; i < GROUP * D / THREADS; ++i) {
            const int idx = tid + i * THREADS, gq = idx / D, jc = idx % D;
            float s = 0.f;
            #pragma unroll
            for (int h = 0; h < HALF_WARPS; ++h) s += accbuf[h][gq][jc];
            o[i] = s;
        }

        const int c_first = cta_of(u.off, T, C), c_last = cta_of(u.off + u.len - 1, T, C);
        if (c_first == c_last) {
            // this CTA holds the whole unit: normalise and store
            #pragma unroll
            for (int i = 0; i < GROUP * D / THREADS; ++i) {
                const int idx = tid + i * THREADS, gq = idx / D, jc = idx % D;
                store_out(u, gq, jc, o[i] / stat[GROUP + gq]);
            }
        } else {
            const int unit = (u.l * a.n + u.b) * a.hkv + u.kh;
            const int nrec = c_last - c_first + 1;
            float* rec = a.partial + ((size_t)unit * a.max_records + (c - c_first)) * PARTIAL_FLOATS;
            if (tid < 2 * GROUP) rec[tid] = stat[tid];
            #pragma unroll
            for (int i = 0; i < GROUP * D / THREADS; ++i) rec[4 + tid + i * THREADS] = o[i];
            __threadfence();
            __syncthreads();
            if (tid == 0) is_last = (atomicAdd(&a.counters[unit], 1) == nrec - 1);
            __syncthreads();
            if (is_last && nrec <= FAST_MERGE) {
                // Few records (a 28-layer step splits a unit over about 1.3 CTAs): every other
                // record's statistics and this thread's two output columns are loaded at once, one
                // L2 round trip; this CTA's own record is still in registers. The sum runs in
                // record order, so the result does not depend on which CTA arrives last.
                __threadfence();
                const float* recs = a.partial + (size_t)unit * a.max_records * PARTIAL_FLOATS;
                const int own = c - c_first;
                float4 st4[FAST_MERGE];
                float av[FAST_MERGE][GROUP * D / THREADS];
                #pragma unroll
                for (int sr = 0; sr < FAST_MERGE; ++sr) {
                    if (sr < nrec && sr != own) {
                        const float* rs = recs + (size_t)sr * PARTIAL_FLOATS;
                        st4[sr] = __ldcg(reinterpret_cast<const float4*>(rs));
                        #pragma unroll
                        for (int i = 0; i < GROUP * D / THREADS; ++i) av[sr][i] = __ldcg(rs + 4 + tid + i * THREADS);
                    } else {
                        st4[sr] = make_float4(stat[0], stat[1], stat[GROUP], stat[GROUP + 1]);
                        #pragma unroll
                        for (int i = 0; i < GROUP * D / THREADS; ++i) av[sr][i] = o[i];
                    }
                }
                float mm[GROUP] = {-INFINITY, -INFINITY};
                #pragma unroll
                for (int sr = 0; sr < FAST_MERGE; ++sr)
                    if (sr < nrec) { mm[0] = fmaxf(mm[0], st4[sr].x); mm[1] = fmaxf(mm[1], st4[sr].y); }
                float ll[GROUP] = {0.f, 0.f}, wt[FAST_MERGE][GROUP];
                #pragma unroll
                for (int sr = 0; sr < FAST_MERGE; ++sr) {
                    wt[sr][0] = sr < nrec ? exp2f(st4[sr].x - mm[0]) : 0.f;
                    wt[sr][1] = sr < nrec ? exp2f(st4[sr].y - mm[1]) : 0.f;
                    if (sr < nrec) { ll[0] += wt[sr][0] * st4[sr].z; ll[1] += wt[sr][1] * st4[sr].w; }
                }
                #pragma unroll
                for (int i = 0; i < GROUP * D / THREADS; ++i) {
                    const int idx = tid + i * THREADS, gq = idx / D, jc = idx % D;
                    float v = 0.f;
                    #pragma unroll
                    for (int sr = 0; sr < FAST_MERGE; ++sr)
                        if (sr < nrec) v += wt[sr][gq] * av[sr][i];
                    store_out(u, gq, jc, v / ll[gq]);
                }
                if (tid == 0) a.counters[unit] = 0;    // ready for the next call on this stream
            } else if (is_last) {
                // Merge the unit's nrec records (a unit split over many CTAs: one layer per call)
                // in rounds of `cap` records: a round copies its records into shared memory with
                // every copy in flight at once (one L2 round trip), then each thread folds its two
                // output columns over the round in record order, rescaling across rounds. The
                // ring holds 63 records when this is the range's last segment (nothing is left to
                // stream into it); otherwise the score buffer (this segment's scores are spent) or
                // accbuf holds a round.
                __threadfence();
                const float* recs = a.partial + (size_t)unit * a.max_records * PARTIAL_FLOATS;
                const int score_floats = FUSED ? max(GROUP * a.max_keys, FUSED_MAX_UNITS * 1024) : GROUP * a.max_keys;
                float* buf = &accbuf[0][0][0];
                int cap = HALF_WARPS * GROUP * D / PARTIAL_FLOATS;
                if (g >= g_end) {
                    buf = reinterpret_cast<float*>(ring);
                    cap = NST * (int)CHUNK_BYTES / (PARTIAL_FLOATS * 4);
                } else if (score_floats / PARTIAL_FLOATS > cap) {
                    buf = scores;
                    cap = score_floats / PARTIAL_FLOATS;
                }
                // per round: the two heads' maxima (warp 0), one weight per (record, head) into the
                // record's max slot, then every thread's columns and the sums over the weights
                float M[GROUP] = {-INFINITY, -INFINITY}, Ls[GROUP] = {0.f, 0.f};
                float V[GROUP * D / THREADS];
                #pragma unroll
                for (int i = 0; i < GROUP * D / THREADS; ++i) V[i] = 0.f;
                for (int r0 = 0; r0 < nrec; r0 += cap) {
                    const int nr = min(cap, nrec - r0);
                    __syncthreads();                   // the previous round (or accbuf's last use) is read
                    const float* src = recs + (size_t)r0 * PARTIAL_FLOATS;
                    for (int i = tid; i < nr * PARTIAL_FLOATS / 4; i += THREADS)
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                     ::"r"(smem_u32(buf + 4 * i)), "l"(src + 4 * i) : "memory");
                    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
                    __syncthreads();
                    if (warp == 0) {
                        float m0 = M[0], m1 = M[1];
                        for (int sr = lane; sr < nr; sr += 32) {
                            m0 = fmaxf(m0, buf[sr * PARTIAL_FLOATS]);
                            m1 = fmaxf(m1, buf[sr * PARTIAL_FLOATS + 1]);
                        }
                        #pragma unroll
                        for (int off = 16; off >= 1; off >>= 1) {
                            m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, off));
                            m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, off));
                        }
                        if (lane == 0) { stat[0] = m0; stat[1] = m1; }
                    }
                    __syncthreads();
                    const float n0 = stat[0], n1 = stat[1];
                    for (int k = tid; k < GROUP * nr; k += THREADS) {      // weight of record k / 2, head k % 2
                        float* slot = buf + (k >> 1) * PARTIAL_FLOATS + (k & 1);
                        *slot = exp2f(*slot - ((k & 1) ? n1 : n0));
                    }
                    const float sc0 = M[0] == -INFINITY ? 0.f : exp2f(M[0] - n0);
                    const float sc1 = M[1] == -INFINITY ? 0.f : exp2f(M[1] - n1);
                    M[0] = n0; M[1] = n1;
                    Ls[0] *= sc0; Ls[1] *= sc1;
                    #pragma unroll
                    for (int i = 0; i < GROUP * D / THREADS; ++i) V[i] *= ((tid + i * THREADS) / D) ? sc1 : sc0;
                    __syncthreads();                   // weights in place
                    for (int sr = 0; sr < nr; ++sr) {
                        const float* rb = buf + sr * PARTIAL_FLOATS;
                        const float w0 = rb[0], w1 = rb[1];
                        Ls[0] += w0 * rb[GROUP];
                        Ls[1] += w1 * rb[GROUP + 1];
                        #pragma unroll
                        for (int i = 0; i < GROUP * D / THREADS; ++i) {
                            const int idx = tid + i * THREADS;
                            V[i] += (idx / D ? w1 : w0) * rb[4 + idx];
                        }
                    }
                }
                #pragma unroll
                for (int i = 0; i < GROUP * D / THREADS; ++i) {
                    const int idx = tid + i * THREADS, gq = idx / D, jc = idx % D;
                    store_out(u, gq, jc, V[i] / Ls[gq]);
                }
                if (tid == 0) a.counters[unit] = 0;    // ready for the next call on this stream
            }
        }
        __syncthreads();                               // accbuf / stat reuse by the next segment
    }

    // drain: copies issued but never consumed (abort path) must land before the CTA exits
    if (tid == 0) {
        while (consumed < issued) {
            mbar_wait(&full[consumed % NST], (consumed / NST) & 1, &never_abort, 500000000ull);
            ++consumed;
        }
    }
    if (a.g.n_flags > 0) {
        // The CTA's output stores (peers' memory included) are ordered before its count by the
        // barrier and one system-scope acquire-release add (cumulative over the CTA's stores);
        // the last CTA, having acquired every count, marks the step done in every rank's flags
        // with release stores.
        __syncthreads();
        if (tid == 0) {
            unsigned prev;
            asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.g.done) : "memory");
            if (prev == gridDim.x - 1) {
                *a.g.done = 0;                         // ready for the next launch, before anyone may start it
                for (int r = 0; r < a.g.n_flags; ++r)
                    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.g.flags[r]), "r"(a.g.step) : "memory");
            }
        }
    }
}

}  // namespace

size_t DecodePlan::partial_floats() const { return (size_t)units * max_records * PARTIAL_FLOATS; }

size_t decode_partial_floats_bound(int n_layers, int hkv, int n_max) {
    const size_t ctas = (size_t)NUM_SMS_B200 * 2, units = (size_t)n_layers * n_max * hkv;
    return ((size_t)n_max * ctas + 2 * units) * PARTIAL_FLOATS;
}

// Even split: C ranges of T/C keys, C = 2 CTAs per SM (one wave) unless that makes a range
// shorter than 64 keys. A segment (one range within one unit) holds at most
// min(ceil(T/C), longest unit) keys, which sizes the score buffer.
DecodePlan plan_attn_decode(int n_layers, int hkv, int n, const int* pos) {
    DecodePlan p{};
    long long row_keys = 0;
    int max_len = 0;
    for (int b = 0; b < n; ++b) { row_keys += pos[b] + 1; max_len = std::max(max_len, pos[b] + 1); }
    p.total_keys = (long long)n_layers * hkv * row_keys;
    // Two CTAs per SM with at least 64 keys each. (One CTA per SM for launches under 512 keys
    // per CTA, halving the records of a one-layer call, measured slower: 461 against 374 us per
    // token of 28 one-layer steps, the longer per-CTA streams cost more than the merges save.)
    long long ctas = (long long)NUM_SMS_B200 * 2;
    ctas = std::min<long long>(ctas, std::max<long long>(1, p.total_keys / 64));
    p.ctas = (int)ctas;
    p.max_keys = (int)std::min<long long>((p.total_keys + ctas - 1) / ctas + 1, max_len);
    // a unit of len keys meets at most floor(len*C/T) + 2 of the C ranges
    p.max_records = (int)(((long long)max_len * ctas) / p.total_keys) + 2;
    p.units = n_layers * n * hkv;
    // a range of R keys meets at most ceil(R / shortest unit) + 1 units
    int min_len = max_len;
    for (int b = 0; b < n; ++b) min_len = std::min(min_len, pos[b] + 1);
    const long long range = (p.total_keys + ctas - 1) / ctas;
    p.max_units_per_cta = (int)std::min<long long>((range + min_len - 1) / min_len + 1, 1 << 30);
    return p;
}

void launch_attn_decode_sm100(const DecodePlan& plan, const KVLayout& kv, const float* q, float* out, int layer0,
                              int n_layers, int n, const int* seq, const int* pos, int hq, int hkv, float* partial,
                              int* counters, int* error, cudaStream_t s, const StepInputs* step,
                              const GatherArgs* gather) {
    DecodeArgs a{};
    a.q = q; a.out = out; a.kv = kv; a.layer0 = layer0; a.n_layers = n_layers; a.n = n; a.hq = hq; a.hkv = hkv;
    if (step) a.step = *step;
    if (gather) a.g = *gather;
    a.start[0] = 0;
    for (int b = 0; b < n; ++b) { a.seq[b] = seq[b]; a.pos[b] = pos[b]; a.start[b + 1] = a.start[b] + pos[b] + 1; }
    a.total_keys = plan.total_keys; a.ctas = plan.ctas; a.max_keys = plan.max_keys;
    a.max_records = plan.max_records;
    a.partial = partial; a.counters = counters; a.error = error;
    // ring + score buffer; a fused step stages its inputs (1024 floats per unit) in the score buffer
    const size_t score_bytes = std::max((size_t)GROUP * a.max_keys * sizeof(float),
                                        step ? (size_t)FUSED_MAX_UNITS * 1024 * sizeof(float) : (size_t)0);
    const size_t smem = (size_t)NST * CHUNK_BYTES + score_bytes;
    static bool attr = false;
    if (!attr) {
        const int max_smem = NST * CHUNK_BYTES + GROUP * MAX_UNIT_KEYS * (int)sizeof(float);
        cudaFuncSetAttribute(attn_decode_sm100_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        cudaFuncSetAttribute(attn_decode_sm100_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        attr = true;
    }
    if (step && step->pdl) {
        a.pdl = 1;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(a.ctas); cfg.blockDim = dim3(THREADS); cfg.dynamicSmemBytes = smem; cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr; cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, attn_decode_sm100_kernel<true>, a);
    } else if (step) attn_decode_sm100_kernel<true><<<a.ctas, THREADS, smem, s>>>(a);
    else attn_decode_sm100_kernel<false><<<a.ctas, THREADS, smem, s>>>(a);
}

}  // namespace qattn
