/* qattn_synth.h — seeded synthetic workload generator exported by libqattn.so.
 *
 * No counterpart in the reference: its attention inputs come from projections of the
 * Qwen3-0.6B checkpoint, which is not available here. This generator produces the
 * stand-in inputs the benchmark configurations describe: pre-norm q [16,128] and k, v
 * [8,128] ~ N(0,1) per (layer, absolute position), and q_norm / k_norm weights
 * ~ N(1, 0.05) per layer.
 *
 * Each value is a pure function of (seed, kind, layer, position, global head, channel):
 * a SplitMix64 hash of that key feeds one Box-Muller draw. Regenerating a position
 * with the same seed therefore reproduces the same bits, whatever range is requested
 * (used for the canonical-prefix configuration, where a second request regenerates
 * positions 0..511 of the first).
 */
#ifndef QATTN_SYNTH_H
#define QATTN_SYNTH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { QA_SYNTH_Q = 0, QA_SYNTH_K = 1, QA_SYNTH_V = 2, QA_SYNTH_QNORM = 3, QA_SYNTH_KNORM = 4 };

/* Writes dst[n_layers][n][heads][128] (device memory) on `stream` (cudaStream_t, may be
 * NULL): value = mean + std * z(seed, kind, layer0+l, pos0+b, head0+h, j). */
int qa_synth_fill(float* dst, uint64_t seed, int kind, int layer0, int n_layers, int pos0,
                  int n, int head0, int heads, float mean, float std, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QATTN_SYNTH_H */
