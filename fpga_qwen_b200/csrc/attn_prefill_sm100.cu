// attn_prefill_sm100.cu — causal GQA prefill attention on the 5th-generation tensor cores.
//
// Replaces the reference's batched-prefill attention (tampajohn/fpga-qwen engine/core.cpp
// :357-381, :407-605): for each new row b (position pos0+b) and query head h,
// out = softmax(q.K^T / sqrt(128)) V over keys [0, pos0+b] of KV head h/2.
//
// Work item = (layer, KV head, 128-row query tile). The kernel is persistent: one CTA per SM
// takes work items from a global counter (a two-slot tile queue in shared memory hands each
// item to all warps), keeps its TMEM, barriers and K/V ring across items, and streams the
// next item's K/V while the current one finishes. Both query heads of the GQA pair live in
// the CTA and share every K/V tile (the reference pairs heads for the same reason,
// core.cpp:150-159). Rows whose absolute position is below 128 are not handled here: they
// attend to few keys, where FP16 probabilities are not accurate enough, and go to the
// FP32 CUDA-core kernel (attn_head_rows.cu).
//
// Warp roles (384 threads, three warpgroups):
//   warps 0-3  softmax group for query head 0 (thread t owns query row t of the tile)
//   warps 4-7  softmax group for query head 1
//   warp  8    MMA issuer (the warp runs the issue sequences, one elected lane issues
//              tcgen05.mma; the warp zeroes stale V rows)
//   warp  9    TMA producer (one thread); warps 10-11 idle
// setmaxnreg moves registers from the control warpgroup to the softmax warpgroups so each
// softmax thread holds its 128-column S row in registers.
// Per 128-key tile j:
//   S_h = Q_h K_j^T         tcgen05.mma kind::f16, M=128 N=128 K=128, FP32 accumulate in TMEM
//   softmax group h: tcgen05.ld S_h row, causal mask, running max (log2 domain, lazy
//   rescale when the max grows by more than 8), P = 2^(s - m) -> FP16 written back into the
//   first 64 TMEM columns of S_h with tcgen05.st (two FP16 keys per 32-bit column)
//   O_h += P_h V_j          tcgen05.mma with A = P from TMEM, B = V (MN-major, shared memory)
// The MMA thread issues PV_h(j) then S_h(j+1) for h = 0, 1, so the tensor pipe works on one
// head while the other head's softmax runs. S_h(j+1) overwrites P_h(j) only after PV_h(j)
// has read it: MMAs issued by one thread execute in order. The commit that announces S_h(j)
// also covers PV_h(j-1), so the softmax group may rescale O_h without another barrier.
// Key tiles above the diagonal of the query tile are skipped; tiles crossing it are masked
// per element.
//
// Memory: Q_0, Q_1 (FP16, 32 KB each) and a 5-stage K/V ring (32 KB stages) = 224 KB of
// shared memory; TMEM 512 columns = S_0/P_0, S_1/P_1, O_0, O_1 (128 FP32 columns each).
// K/V tiles come from the HBM KV store through one 3-D tensor map
// {128 channels, ctx positions, planes} with 64x128 boxes and 128-byte swizzle; loads run
// up to 2.5 tiles ahead of the tensor pipe.
// Q rows are read with coalesced 512-byte row loads. At an item boundary the softmax warps
// first store the next item's Q (the head's Q buffer is free once the last QK of the item has
// completed), so its first QK runs on the tensor pipe while they write this item's output rows
// straight from TMEM (16x256b loads: every store writes whole 32-byte sectors). The peer-store
// instantiation instead stages rows in the Q buffer for 128-byte writes over NVLink and stores
// the next Q after its epilogue.
//
// Launches with fewer items than SMs (a prompt chunk of a few hundred rows attended one layer
// per call) split every item's key tiles into segments (the <false, true> instantiation): each
// segment leaves unnormalised rows and their running max and sum in a scratch, and
// prefill_merge_kernel combines them. Single-GPU launches are programmatic dependents of the
// previous kernel (set-up overlaps it; griddepcontrol.wait precedes every read of its output),
// and the last CTA of each launch resets the work counter for the next one.
//
// Every wait is bounded (globaltimer, 2 s): on expiry the CTA raises an abort flag, writes
// an error code to the host-visible flag, drains what it issued and frees its TMEM.
#include <algorithm>

#include "qattn_common.cuh"
#include "sm100.cuh"

namespace qattn {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128;
constexpr int THREADS = 384;                              // 12 warps = 3 warpgroups
// Register split: launched at 168 per thread (384 x 168 = 64,512); the control warpgroup
// (MMA + TMA warps) drops to 72 and the two softmax warpgroups rise to 216:
// 2 x 128 x 216 + 128 x 72 = 64,512, the launch total.
constexpr int REGS_LAUNCH = 168, REGS_SOFTMAX = 216, REGS_CONTROL = 72;
static_assert(2 * 128 * REGS_SOFTMAX + 128 * REGS_CONTROL == THREADS * REGS_LAUNCH, "register split must match launch");
constexpr uint32_t TILE_BYTES = BN * D * 2;               // 32 KB FP16 K or V tile
// K and V tiles share one 5-stage ring in load order K0, V0, K1, V1, ...: item i = 2j (K_j)
// or 2j+1 (V_j) lives in stage i % 5, so every load is issued about 2.5 tiles before use.
constexpr int RING = 5;
constexpr int OFF_Q = 0, OFF_RING = 65536, OFF_BAR = OFF_RING + RING * 32768;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;          // + barriers + alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
constexpr float RESCALE_THRESHOLD = 8.0f;                 // log2 units

constexpr int TQ = 2;                                     // tile queue slots
enum {
    B_Q0, B_Q1, B_FULL0, B_EMPTY0 = B_FULL0 + RING, B_SF0 = B_EMPTY0 + RING, B_SF1, B_PF0, B_PF1, B_OD0, B_OD1,
    B_OF0, B_OF1,                                         // O_h read by the epilogue (free for the next tile)
    B_TF0, B_TE0 = B_TF0 + TQ,                            // tile queue slot filled / read by every consumer
    B_DRAIN = B_TE0 + TQ, B_COUNT
};
static_assert(B_COUNT * 8 + 4 + 4 * TQ <= 256, "barrier area");

struct PrefillArgs {
    const float* q;                   // [n_layers][n][hq][128]
    OutRows o;                        // output rows: local layout, or full-head layout here and on peers
    int seq, layer0, n_layers, pos0, n, hq, hkv, layers_total;
    int row_begin, n_qtiles, n_tiles;
    int size_major;                   // 1: items ordered by size across all (layer, KV head) groups
    int kseg;                         // key segments per item (work units = items x kseg); 1: no split
    float* part;                      // kseg > 1: [unit][2 heads][128 rows][128] unnormalised O rows
    float* part_ml;                   // kseg > 1: [unit][2 heads][128 rows] (running max, sum)
    int* tile_counter;                // [0] next unit to hand out, [1] CTAs finished; zero between launches
    int* error;
};

// Tile t of the launch. Launches whose K/V exceed a share of L2: the query tiles of one (layer,
// KV head) are consecutive, heaviest first, so CTAs running at the same time read the same K/V
// planes and hit in L2. Launches whose K/V fit in L2 (a layer or two, as an engine calls it):
// heaviest first across all groups (the longest items start first, so the launch ends evenly).
// With kseg > 1 (launches with fewer items than SMs) unit t is segment t % kseg of item
// t / kseg: key tiles [j0, j0 + nj) of the item's nk, an even share.
// SPLIT is the kernel instantiation for such launches (the others compile without the division).
struct TileInfo { int l, kh, r0, nk, valid_keys, plane_k, j0, nj; };
template <bool SPLIT>
__device__ __forceinline__ TileInfo tile_info(const PrefillArgs& a, int t) {
    TileInfo ti;
    const int item = SPLIT ? t / a.kseg : t, seg = SPLIT ? t - item * a.kseg : 0;
    const int groups = a.hkv * a.n_layers;
    const int lh = a.size_major ? item % groups : item / a.n_qtiles;
    const int tile = a.n_qtiles - 1 - (a.size_major ? item / groups : item % a.n_qtiles);
    ti.kh = lh % a.hkv;
    ti.l = lh / a.hkv;
    ti.r0 = a.row_begin + tile * BM;                          // first query row of the tile
    ti.valid_keys = a.pos0 + min(ti.r0 + BM, a.n);            // keys visible to the tile's last row
    ti.nk = (ti.valid_keys + BN - 1) / BN;                    // causal key tiles
    ti.plane_k = ((a.seq * a.layers_total + a.layer0 + ti.l) * 2 + 0) * a.hkv + ti.kh;
    ti.j0 = SPLIT ? seg * ti.nk / a.kseg : 0;
    ti.nj = SPLIT ? (seg + 1) * ti.nk / a.kseg - ti.j0 : ti.nk;
    return ti;
}

__device__ __forceinline__ uint32_t swz(int row, int chunk16) {   // K-major, 128B swizzle, 2 atom columns
    return (uint32_t)((chunk16 >> 3) * 16384 + (row >> 3) * 1024 + (row & 7) * 128 + (((chunk16 & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// 2^x on the MUFU unit (PTX ex2.approx.ftz: relative error ~2^-22, inputs here are <= 8)
__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r, ua = *reinterpret_cast<unsigned long long*>(&a), ub = *reinterpret_cast<unsigned long long*>(&b),
                          uc = *reinterpret_cast<unsigned long long*>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(ua), "l"(ub), "l"(uc));
    return *reinterpret_cast<float2*>(&r);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long r, ua = *reinterpret_cast<unsigned long long*>(&a), ub = *reinterpret_cast<unsigned long long*>(&b);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(ua), "l"(ub));
    return *reinterpret_cast<float2*>(&r);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// The 32 rows of one warp's quarter of head h: lane i reads channels 4i..4i+3 of each row
// (coalesced 512-byte rows), all 32 rows in flight (one L2 round trip).
__device__ __forceinline__ void q_load_rows(const PrefillArgs& a, const TileInfo& ti, int h, int wq, int lane,
                                            float4 (&xr)[32]) {
    const float* base = a.q + (((size_t)ti.l * a.n) * a.hq + (size_t)ti.kh * 2 + h) * D + lane * 4;
    #pragma unroll
    for (int rr = 0; rr < 32; ++rr) {
        const int r = ti.r0 + wq * 32 + rr;
        xr[rr] = r < a.n ? __ldg(reinterpret_cast<const float4*>(base + (size_t)r * a.hq * D)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}
// ... as FP16 in the swizzled K-major layout of the head's Q buffer.
__device__ __forceinline__ void q_store_rows(uint8_t* Qs, int wq, int lane, const float4 (&xr)[32]) {
    #pragma unroll
    for (int rr = 0; rr < 32; ++rr)
        *reinterpret_cast<uint2*>(Qs + swz(wq * 32 + rr, lane >> 1) + (lane & 1) * 8) =
            make_uint2(pack_half2(xr[rr].x, xr[rr].y), pack_half2(xr[rr].z, xr[rr].w));
}

// PEERS: rows go where a.o says, peers included; otherwise the local layout {out, hq, 0}
// (the single-GPU path carries no peer-store code). SPLIT (single-GPU only): units are key
// segments of items, whose rows go unnormalised to the scratch for prefill_merge_kernel.
template <bool PEERS, bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
attn_prefill_sm100_kernel(const __grid_constant__ CUtensorMap kv_map, const PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + B_COUNT * 8);
    volatile int* tq = reinterpret_cast<volatile int*>(smem + OFF_BAR + B_COUNT * 8 + 4);
    __shared__ int abort_flag;
    __shared__ int never_abort;                              // for drains that must not give up early

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        abort_flag = 0;
        never_abort = 0;
        mbar_init(&bar[B_Q0], 128); mbar_init(&bar[B_Q1], 128);
        for (int i = 0; i < RING; ++i) { mbar_init(&bar[B_FULL0 + i], 1); mbar_init(&bar[B_EMPTY0 + i], 1); }
        mbar_init(&bar[B_SF0], 1); mbar_init(&bar[B_SF1], 1);
        mbar_init(&bar[B_PF0], 128); mbar_init(&bar[B_PF1], 128); mbar_init(&bar[B_OD0], 1); mbar_init(&bar[B_OD1], 1);
        mbar_init(&bar[B_OF0], 128); mbar_init(&bar[B_OF1], 128);
        for (int i = 0; i < TQ; ++i) { mbar_init(&bar[B_TF0 + i], 1); mbar_init(&bar[B_TE0 + i], 1 + 256); }
        mbar_init(&bar[B_DRAIN], 1);
        fence_mbar_init();
    }
    if (warp == 8) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (warp == 9 && lane == 0) prefetch_tmap(&kv_map);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Single-GPU launches are programmatic dependents: the set-up above overlaps the previous
    // kernel, and nothing that kernel writes (q, K/V, the work counter, the split scratch) is
    // read before this wait.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    volatile int* abortp = &abort_flag;
    if (warp < 8) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_SOFTMAX));
    else asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CONTROL));
    auto fail = [&](int code) { *abortp = 1; atomicCAS(a.error, 0, code); };

    if (warp < 8) {
        // ================================ softmax groups ================================
        const int h = warp >> 2;                             // query head within the pair
        const int wq = warp & 3;                             // this warp's 32-row quarter
        const int trow = tid & 127;                          // row within the tile
        uint8_t* Qs = smem + OFF_Q + h * 32768;
        const float scale = 1.4426950408889634f * 0.08838834764831845f;   // log2(e)/sqrt(128)
        const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
        const uint32_t s_col = tmem + lane_base + h * 128;   // S_h; P_h in its first 64 columns
        const uint32_t o_col = tmem + lane_base + 256 + h * 128;
        uint32_t kt = 0;                                     // key tiles processed (S, P phases)
        // the i-th work item from the tile queue (-1: none left; -2: the wait gave up)
        auto read_tile = [&](int i) {
            const int slot = i % TQ;
            if (!mbar_wait(&bar[B_TF0 + slot], (i / TQ) & 1, abortp)) { fail(14); return -2; }
            const int tt = tq[slot];
            mbar_arrive(&bar[B_TE0 + slot]);
            return tt;
        };
        // Q rows of this warp's quarter (q_load_rows / q_store_rows): all 32 loaded at once, then
        // stored as FP16 into this warp's own rows of the head's Q buffer (free when called).
        auto store_q = [&](const TileInfo& tn) {
            float4 xr[32];
            q_load_rows(a, tn, h, wq, lane, xr);
            q_store_rows(Qs, wq, lane, xr);
            fence_proxy_async_smem();
            mbar_arrive(&bar[B_Q0 + h]);
        };
        int tt = read_tile(0);
        if (tt >= 0) store_q(tile_info<SPLIT>(a, tt));
        for (int i = 0; tt >= 0; ++i) {
            const TileInfo ti = tile_info<SPLIT>(a, tt);
            const int row_pos = a.pos0 + ti.r0 + trow;
            float m = -INFINITY, lsum = 0.f;
            bool ok = true;
            for (int j = 0; j < ti.nj; ++j, ++kt) {
                if (!mbar_wait(&bar[B_SF0 + h], kt & 1, abortp)) { fail(11); ok = false; break; }
                tc_fence_after();
                // S row -> registers: four 32-column loads in flight, one wait; the empty asm pins
                // every use of the loaded registers after the wait
                uint32_t sr[4][32];
                #pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32(s_col + c * 32, sr[c]);
                tmem_wait_ld();
                #pragma unroll
                for (int c = 0; c < 4; ++c)
                    #pragma unroll
                    for (int e = 0; e < 32; ++e) asm volatile("" : "+r"(sr[c][e]));
                float* v = reinterpret_cast<float*>(&sr[0][0]);
                const int k0 = (ti.j0 + j) * BN;
                const int lim = row_pos - k0;                   // keys c > lim are in the future
                if (lim < BN - 1) {                             // tile crosses the diagonal
                    #pragma unroll
                    for (int c = 0; c < BN; ++c) v[c] = (c > lim) ? -INFINITY : v[c];
                }
                // row max: four independent 3-input max chains, then combined
                float mq[4];
                #pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const float* w = v + q4 * 32;
                    float x = fmax3(w[0], w[1], w[2]);
                    #pragma unroll
                    for (int c = 3; c < 31; c += 2) x = fmax3(x, w[c], w[c + 1]);
                    mq[q4] = fmaxf(x, w[31]);
                }
                float mt = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale;
                float alpha = 1.f;
                bool rescale = false;
                if (j == 0) m = mt;
                else if (mt > m + RESCALE_THRESHOLD) { alpha = ex2_approx(m - mt); m = mt; rescale = true; }
                // p = 2^(s*scale - m): packed FMA pairs, MUFU ex2, FP16 pairs into TMEM over S_h
                // (the first half is stored while the second half is computed)
                const float2 sc2 = make_float2(scale, scale), mn2 = make_float2(-m, -m);
                float2 ps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                #pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t pk[32];
                    #pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const int k = half * 64 + 2 * c;
                        const float2 x = ffma2(make_float2(v[k], v[k + 1]), sc2, mn2);
                        const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                        ps[c & 3] = fadd2(ps[c & 3], e);
                        pk[c] = pack_half2(e.x, e.y);
                    }
                    tmem_st32(s_col + half * 32, pk);
                }
                const float psum = (ps[0].x + ps[0].y) + (ps[1].x + ps[1].y) + (ps[2].x + ps[2].y) + (ps[3].x + ps[3].y);
                if (rescale) {
                    // O_h holds PV_h(0..j-1) (the commit that announced S_h(j) covered them); it is
                    // rescaled before PV_h(j) is allowed to accumulate into it
                    #pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t rr[32];
                        tmem_ld32(o_col + c * 32, rr);
                        tmem_wait_ld();
                        #pragma unroll
                        for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
                        tmem_st32(o_col + c * 32, rr);
                    }
                    lsum *= alpha;
                }
                lsum += psum;
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bar[B_PF0 + h]);
            }
            if (!ok) break;
            // the next work item (its Q rows were pulled into L2 by the producer when it took it)
            const int next = read_tile(i + 1);
            if constexpr (!PEERS) {
                // Q_h is free (QK_h of the last key tile completed before its S was announced):
                // the next item's Q rows go in now, so its first QK_h runs on the tensor pipe
                // while this item's epilogue runs
                if (next >= 0) store_q(tile_info<SPLIT>(a, next));
            }
            // ---- epilogue: O_h of this tile (all its MMAs, QK_h included, have completed) ----
            if (!mbar_wait(&bar[B_OD0 + h], i & 1, abortp)) { fail(13); break; }
            tc_fence_after();
            // a key segment of a split item leaves its rows unnormalised (weight 1) in the scratch,
            // with the row's running max and sum beside them, for prefill_merge_kernel
            constexpr bool split = SPLIT && !PEERS;
            const float inv = split ? 1.f : 1.f / lsum;
            if (split) {
                float* ml = a.part_ml + (((size_t)tt * 2 + h) * BM + trow) * 2;
                ml[0] = m;
                ml[1] = lsum;
            }
            if constexpr (!PEERS) {
                // Rows straight from TMEM in the 16x256b shape: a thread holds two adjacent
                // columns of rows t/4 and t/4 + 8 of a 16-row half, so each store instruction
                // writes eight rows x 32 contiguous bytes (whole sectors) and no shared memory
                // is involved. Row sums come from the thread that owns the row.
                uint32_t ro[2][64];
                tmem_ld_16x256b_x16(o_col, ro[0]);
                tmem_ld_16x256b_x16(o_col + (16u << 16), ro[1]);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(&bar[B_OF0 + h]);                // O_h read: the next item may overwrite it
                #pragma unroll
                for (int rh = 0; rh < 2; ++rh) {
                    const int ra = rh * 16 + (lane >> 2);    // rows ra and ra + 8 of the warp's quarter
                    const float ia = __shfl_sync(0xffffffffu, inv, ra), ib = __shfl_sync(0xffffffffu, inv, ra + 8);
                    const int r = ti.r0 + wq * 32 + ra;
                    const bool sa = split || r < a.n, sb = split || r + 8 < a.n;   // split: all 128 scratch rows
                    float* pa = split ? a.part + (((size_t)tt * 2 + h) * BM + wq * 32 + ra) * D + 2 * (lane & 3)
                                      : a.o.out + (((size_t)ti.l * a.n + r) * a.hq + (size_t)ti.kh * 2 + h) * D + 2 * (lane & 3);
                    float* pb = pa + (size_t)8 * (split ? D : a.hq * D);
                    #pragma unroll
                    for (int g = 0; g < 16; ++g) {
                        if (sa)
                            *reinterpret_cast<float2*>(pa + 8 * g) =
                                make_float2(__uint_as_float(ro[rh][4 * g]) * ia, __uint_as_float(ro[rh][4 * g + 1]) * ia);
                        if (sb)
                            *reinterpret_cast<float2*>(pb + 8 * g) =
                                make_float2(__uint_as_float(ro[rh][4 * g + 2]) * ib, __uint_as_float(ro[rh][4 * g + 3]) * ib);
                    }
                }
            } else {
                // Output rows leave through the 4 KB piece of this head's Q buffer that holds
                // the first 64 channels of this warp's own Q rows, 32 columns at a time: each
                // thread writes its normalised 128-byte row segment (8 chunks, XOR-swizzled by
                // row), then the warp stores four rows per instruction as 128-byte segments, the
                // peers' copies included (whole 128-byte writes over NVLink).
                uint8_t* stage = Qs + wq * 4096;
                #pragma unroll
                for (int part = 0; part < 4; ++part) {
                    uint32_t ro[32];
                    tmem_ld32(o_col + part * 32, ro);
                    tmem_wait_ld();
                    if (part == 3) {                          // O_h fully read: the next tile may overwrite it
                        tc_fence_before();
                        mbar_arrive(&bar[B_OF0 + h]);
                    }
                    #pragma unroll
                    for (int c = 0; c < 8; ++c)
                        *reinterpret_cast<float4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                            make_float4(__uint_as_float(ro[4 * c]) * inv, __uint_as_float(ro[4 * c + 1]) * inv,
                                        __uint_as_float(ro[4 * c + 2]) * inv, __uint_as_float(ro[4 * c + 3]) * inv);
                    __syncwarp();
                    #pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int rr = 4 * k + (lane >> 3), c = lane & 7;
                        const float4 val = *reinterpret_cast<const float4*>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
                        const int r = ti.r0 + wq * 32 + rr;
                        if (r < a.n) {
                            const size_t off = (((size_t)ti.l * a.n + r) * a.o.heads + a.o.head0 + ti.kh * 2 + h) * D +
                                               part * 32 + c * 4;
                            *reinterpret_cast<float4*>(a.o.out + off) = val;
                            #pragma unroll
                            for (int p = 0; p < MAX_RANKS - 1; ++p)
                                if (p < a.o.n_peers) *reinterpret_cast<float4*>(a.o.peers[p] + off) = val;
                        }
                    }
                    __syncwarp();
                }
                if (next >= 0) store_q(tile_info<SPLIT>(a, next));  // this warp's own Q rows, after its staging
            }
            tt = next;
        }
    } else if (warp == 8) {
        // ================================== MMA issuer ==================================
        const uint32_t idesc_qk = idesc_f16_f32(BM, BN, false);
        const uint32_t idesc_pv = idesc_f16_f32(BM, D, true);
        const uint32_t q_addr = smem_u32(smem + OFF_Q), ring_addr = smem_u32(smem + OFF_RING);
        // Descriptors as a fixed high word (stride offset, version, swizzle) and a low word
        // stepped by 32-bit adds (start address >> 4 in bits 0-13: shared addresses stay below
        // 256 KB, so the field never carries): cheaper to issue than rebuilding both words.
        const uint64_t dq = sw128_desc(q_addr, 16, 1024);
        const uint32_t d_hi = (uint32_t)(dq >> 32), lo_q = (uint32_t)dq;
        const uint32_t lo_k = (uint32_t)sw128_desc(ring_addr, 16, 1024), lo_v = (uint32_t)sw128_desc(ring_addr, 16384, 1024);
        bool ok = true;
        auto wait_item = [&](int it) {                   // ring item it has landed
            return mbar_wait(&bar[B_FULL0 + it % RING], (it / RING) & 1, abortp);
        };
        // The whole warp runs the issue sequences; the elected lane issues (sm100.cuh).
        const uint32_t leader = elect_one();
        auto release_item = [&](int it) {                // stage of item it free once prior MMAs finish
            mma_commit_warp(&bar[B_EMPTY0 + it % RING], leader);
        };
        auto issue_qk = [&](int it, int h) {             // 8 K-steps of 16 channels (32-byte column pairs)
            const uint32_t kb = lo_k + (uint32_t)((it % RING) * TILE_BYTES >> 4), qb = lo_q + (uint32_t)(h * 32768 >> 4);
            const uint32_t d = tmem + h * 128;
#define QK_STEP(S) mma_f16_ss_warp<(((S >> 2) * 16384 + (S & 3) * 32) >> 4), (((S >> 2) * 16384 + (S & 3) * 32) >> 4)>( \
        d, qb, kb, d_hi, idesc_qk, (S > 0), leader)
            QK_STEP(0); QK_STEP(1); QK_STEP(2); QK_STEP(3); QK_STEP(4); QK_STEP(5); QK_STEP(6); QK_STEP(7);
#undef QK_STEP
            mma_commit_warp(&bar[B_SF0 + h], leader);
        };
        auto issue_pv = [&](int it, int h, bool first, bool last) {   // A = P_h in TMEM: 8 columns per 16 keys
            const uint32_t vb = lo_v + (uint32_t)((it % RING) * TILE_BYTES >> 4);
            const uint32_t d = tmem + 256 + h * 128, p = tmem + h * 128, acc0 = first ? 0u : 1u;
#define PV_STEP(S) mma_f16_ts_warp<(S * 8), ((S * 2048) >> 4)>(d, p, vb, d_hi, idesc_pv, (S > 0 ? 1u : acc0), leader)
            PV_STEP(0); PV_STEP(1); PV_STEP(2); PV_STEP(3); PV_STEP(4); PV_STEP(5); PV_STEP(6); PV_STEP(7);
#undef PV_STEP
            if (last) mma_commit_warp(&bar[B_OD0 + h], leader);   // O_h final for the tile
        };
        int base = 0;                                    // ring item of the tile's K_0
        uint32_t kt = 0;                                 // key tiles processed (S, P phases)
        for (int i = 0; ok; ++i) {
            const int slot = i % TQ;
            if (!mbar_wait(&bar[B_TF0 + slot], (i / TQ) & 1, abortp)) { fail(20); break; }
            const int tt = tq[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar[B_TE0 + slot]);
            if (tt < 0) break;
            const TileInfo ti = tile_info<SPLIT>(a, tt);
            // tile prologue: S_0(0) as soon as Q_0 is in place, then S_1(0)
            if (!wait_item(base) || !mbar_wait(&bar[B_Q0], i & 1, abortp)) { fail(21); ok = false; break; }
            tc_fence_after();
            issue_qk(base, 0);
            if (!mbar_wait(&bar[B_Q1], i & 1, abortp)) { fail(21); ok = false; break; }
            tc_fence_after();
            issue_qk(base, 1);
            release_item(base);
            // Per key tile j and head h: O_h += P_h(j) V_j as soon as P_h(j) is written, then
            // S_h(j+1) = Q_h K_{j+1}^T over P_h(j) (ordered after PV_h(j), issued just before);
            // the tensor pipe works on one head while the other head's softmax runs.
            for (int j = 0; j < ti.nj && ok; ++j, ++kt) {
                const int iv = base + 2 * j + 1;
                if (!wait_item(iv)) { fail(22); ok = false; break; }
                if (ti.j0 + j == ti.nk - 1 && ti.valid_keys < (ti.j0 + j + 1) * BN) {
                    // Rows of the last V tile past the causal end hold stale data: zero them so
                    // that a zero probability never meets a non-finite value.
                    uint8_t* Vs = smem + OFF_RING + (iv % RING) * TILE_BYTES;
                    const int first = ti.valid_keys - (ti.j0 + j) * BN;
                    for (int idx = first * 16 + lane; idx < BN * 16; idx += 32) {
                        const int row = idx >> 4, c = idx & 15;    // c: 16-byte chunk of the 256-byte row
                        const int half_sel = c >> 3, cc = c & 7;
                        *reinterpret_cast<uint4*>(Vs + half_sel * 16384 + (row >> 3) * 1024 + (row & 7) * 128 +
                                                  ((cc ^ (row & 7)) << 4)) = make_uint4(0, 0, 0, 0);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                tc_fence_after();
                for (int h = 0; h < 2 && ok; ++h) {
                    if (!mbar_wait(&bar[B_PF0 + h], kt & 1, abortp)) { fail(23); ok = false; break; }
                    // the first PV of a tile overwrites O_h: the previous tile's epilogue has read it
                    if (j == 0 && i > 0 && !mbar_wait(&bar[B_OF0 + h], (i - 1) & 1, abortp)) { fail(27); ok = false; break; }
                    tc_fence_after();
                    issue_pv(iv, h, j == 0, j == ti.nj - 1);
                    if (h == 1) release_item(iv);                  // V_j free when PV_1(j) completes
                    if (j + 1 < ti.nj) {
                        const int ik = base + 2 * j + 2;
                        if (h == 0 && !wait_item(ik)) { fail(24); ok = false; break; }
                        tc_fence_after();
                        issue_qk(ik, h);
                        if (h == 1) release_item(ik);              // K_{j+1} free when QK_1(j+1) completes
                    }
                }
            }
            base += 2 * ti.nj;
        }
        // drain: every MMA this thread issued has completed before TMEM is released
        if (lane == 0) {
            mma_commit(&bar[B_DRAIN]);
            if (!mbar_wait(&bar[B_DRAIN], 0, &never_abort)) atomicCAS(a.error, 0, 29);
        }
        __syncwarp();
    } else if (warp == 9 && lane == 0) {
        // ========================= tile queue + TMA producer =========================
        int issued = 0;
        bool ok = true;
        for (int i = 0; ok; ++i) {
            const int slot = i % TQ;
            if (i >= TQ && !mbar_wait(&bar[B_TE0 + slot], ((i / TQ) - 1) & 1, abortp)) { fail(30); break; }
            int tt = atomicAdd(a.tile_counter, 1);
            if (tt >= a.n_tiles) tt = -1;
            tq[slot] = tt;
            mbar_arrive(&bar[B_TF0 + slot]);                 // the slot's value is visible to the waiters
            if (tt < 0) break;
            const TileInfo ti = tile_info<SPLIT>(a, tt);
            // the item's query rows (both heads of the pair: 1 KB per row) into L2, well before
            // the softmax warps load them
            for (int r = ti.r0; r < min(ti.r0 + BM, a.n); ++r)
                bulk_prefetch_l2(a.q + (((size_t)ti.l * a.n + r) * a.hq + (size_t)ti.kh * 2) * D, 2 * D * sizeof(float));
            for (int j2 = 0; j2 < 2 * ti.nj; ++j2) {
                const int st = issued % RING;
                if (issued >= RING && !mbar_wait(&bar[B_EMPTY0 + st], ((issued / RING) - 1) & 1, abortp)) {
                    fail(31); ok = false; break;
                }
                uint8_t* dst = smem + OFF_RING + st * TILE_BYTES;
                const int plane = (j2 & 1) ? ti.plane_k + a.hkv : ti.plane_k, key0 = (ti.j0 + (j2 >> 1)) * BN;
                mbar_arrive_expect_tx(&bar[B_FULL0 + st], TILE_BYTES);
                tma_load_3d(dst, &kv_map, 0, key0, plane, &bar[B_FULL0 + st]);
                tma_load_3d(dst + 16384, &kv_map, 64, key0, plane, &bar[B_FULL0 + st]);
                ++issued;
            }
        }
        if (!ok) {
            // drain the loads this thread issued (bounded, ignoring the abort flag)
            for (int it = std::max(0, issued - RING); it < issued; ++it)
                mbar_wait(&bar[B_FULL0 + it % RING], (it / RING) & 1, &never_abort, 500000000ull);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (tid == 0) {
        // this CTA takes no more items (on every path): the last CTA out resets the work counter
        // and this count for the next launch
        if (atomicAdd(a.tile_counter + 1, 1) == (int)gridDim.x - 1) {
            a.tile_counter[0] = 0;
            a.tile_counter[1] = 0;
        }
    }
    if (PEERS && a.o.n_peers && tid == 0) __threadfence_system();   // rows stored to peers: visible system-wide at exit
}

// Key-segment merge of split items: one warp per output row (item, head, row), lane l holding
// columns 4l..4l+3. Every segment's running max and sum and its piece of the row are loaded at
// once; the segments then combine in segment order with weights 2^(m_s - M) (the same log2
// domain as the kernel's softmax): out = sum_s w_s O_s / sum_s w_s l_s.
constexpr int MAX_KSEG = 16;
constexpr int SPLIT_UNITS = NUM_SMS_B200;     // scratch: at most one wave of units
__global__ void __launch_bounds__(256) prefill_merge_kernel(const PrefillArgs a) {
    asm volatile("griddepcontrol.wait;" ::: "memory");          // the partials are the prefill's output
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int w = (int)((blockIdx.x * 256u + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    const int n_items = a.n_tiles / a.kseg;
    if (w >= n_items * 2 * BM) return;
    const int item = w / (2 * BM), h = (w / BM) & 1, row = w % BM;
    const TileInfo ti = tile_info<true>(a, item * a.kseg);
    const int r = ti.r0 + row;
    if (r >= a.n) return;
    float m[MAX_KSEG], l[MAX_KSEG];
    float4 o[MAX_KSEG];
    #pragma unroll
    for (int sg = 0; sg < MAX_KSEG; ++sg)
        if (sg < a.kseg) {
            const size_t u = ((size_t)(item * a.kseg + sg) * 2 + h) * BM + row;
            m[sg] = __ldcg(a.part_ml + 2 * u);
            l[sg] = __ldcg(a.part_ml + 2 * u + 1);
            o[sg] = __ldcg(reinterpret_cast<const float4*>(a.part + u * D) + lane);
        }
    float M = -INFINITY;
    #pragma unroll
    for (int sg = 0; sg < MAX_KSEG; ++sg)
        if (sg < a.kseg) M = fmaxf(M, m[sg]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll
    for (int sg = 0; sg < MAX_KSEG; ++sg)
        if (sg < a.kseg) {
            const float wt = ex2_approx(m[sg] - M);
            L += wt * l[sg];
            acc.x += wt * o[sg].x; acc.y += wt * o[sg].y; acc.z += wt * o[sg].z; acc.w += wt * o[sg].w;
        }
    const float inv = 1.f / L;
    *reinterpret_cast<float4*>(a.o.out + (((size_t)ti.l * a.n + r) * a.hq + (size_t)ti.kh * 2 + h) * D + lane * 4) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

}  // namespace

size_t prefill_split_scratch_bytes() { return (size_t)SPLIT_UNITS * 2 * BM * (D + 2) * sizeof(float); }

// Host side --------------------------------------------------------------------------------------
int launch_attn_prefill_sm100(const CUtensorMap& map, const float* q, const OutRows& o, int seq, int layer0,
                              int n_layers, int pos0, int n, int hq, int hkv, int layers_total, int row_begin,
                              int* tile_counter, float* split_scratch, int reserve_sms, int* error,
                              cudaStream_t s) {
    if (row_begin >= n) return 0;
    const bool peers = o.n_peers > 0 || o.heads != hq || o.head0 != 0;
    PrefillArgs a{};
    a.q = q; a.o = o; a.seq = seq; a.layer0 = layer0; a.n_layers = n_layers; a.pos0 = pos0; a.n = n;
    a.hq = hq; a.hkv = hkv; a.layers_total = layers_total; a.row_begin = row_begin;
    a.n_qtiles = (n - row_begin + BM - 1) / BM; a.error = error;
    const int n_items = a.n_qtiles * hkv * n_layers;
    // K/V the launch reads (FP16 K and V rows of every (layer, head) up to the last row), against
    // a third of the 126 MB L2
    a.size_major = (double)n_layers * hkv * 2.0 * (pos0 + n) * D * 2 <= 42.0e6 ? 1 : 0;
    a.tile_counter = tile_counter;
    // persistent: one CTA per SM (225 KB of shared memory each) pulls tiles from the counter
    int dev = 0, sms = NUM_SMS_B200;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // SMs left to a kernel that runs beside this one (the FP32 head rows of a short launch), so
    // that its CTAs start at once instead of after the persistent CTAs
    sms = std::max(1, sms - std::max(0, reserve_sms));
    // Fewer items than SMs (a prompt chunk of a few hundred rows at an offset, one layer per call):
    // each item's key tiles split into kseg segments of at least two tiles, one unit per SM at
    // most, merged by prefill_merge_kernel.
    a.kseg = 1;
    if (!peers && split_scratch && n_items < sms) {
        const int nk_min = (pos0 + std::min(row_begin + BM, n) + BN - 1) / BN;   // the first row tile's key tiles
        const int k = std::min({sms / n_items, nk_min / 2, MAX_KSEG, SPLIT_UNITS / n_items});
        if (k >= 2) {
            a.kseg = k;
            a.part = split_scratch;
            a.part_ml = split_scratch + (size_t)SPLIT_UNITS * 2 * BM * D;
        }
    }
    a.n_tiles = n_items * a.kseg;
    const int which = peers ? 2 : a.kseg > 1 ? 1 : 0;
    void (*const kernels[3])(const CUtensorMap, const PrefillArgs) = {
        attn_prefill_sm100_kernel<false, false>, attn_prefill_sm100_kernel<false, true>,
        attn_prefill_sm100_kernel<true, false>};
    static int checked[3] = {0, 0, 0};           // per instantiation: 1 ready, -1 refused
    int& ck = checked[which];
    if (!ck) {
        // setmaxnreg.inc waits for registers the control warpgroup releases; the split is
        // only consistent with a launch at exactly REGS_LAUNCH registers per thread.
        const void* fn = (const void*)kernels[which];
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess || fa.numRegs != REGS_LAUNCH ||
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
            ck = -1;
        else
            ck = 1;
    }
    if (ck < 0) return -1;
    const unsigned blocks = (unsigned)std::min(a.n_tiles, sms);
    // single-GPU launches (and the merge after a split one) as programmatic dependents
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(blocks); cfg.blockDim = dim3(THREADS); cfg.dynamicSmemBytes = SMEM_BYTES; cfg.stream = s;
    cfg.attrs = attr; cfg.numAttrs = peers ? 0 : 1;
    if (cudaLaunchKernelEx(&cfg, kernels[which], map, a) != cudaSuccess) return -2;
    if (a.kseg > 1) {
        cudaLaunchConfig_t mc{};
        mc.gridDim = dim3((unsigned)(n_items * 2 * BM / 8)); mc.blockDim = dim3(256); mc.stream = s;
        mc.attrs = attr; mc.numAttrs = 1;
        if (cudaLaunchKernelEx(&mc, prefill_merge_kernel, a) != cudaSuccess) return -2;
    }
    return 0;
}

}  // namespace qattn
