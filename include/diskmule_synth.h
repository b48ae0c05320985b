/*
 * diskmule_synth.h -- seeded synthetic tensors for tests and benchmarks.
 *
 * No counterpart in the reference (its fixtures are written by its tests, e.g.
 * src/glm52/cpu.rs:1841-2063, and real checkpoints are not available here).
 * Block b of a tensor is a pure function of (seed, b): the host and the device
 * write identical bytes, and any slice (one expert) can be generated alone.
 *   dense kinds (DM_F32 / DM_F16 / DM_BF16): one element per block, N(0, sigma)
 *     (Irwin-Hall sum of 12 SplitMix64 uniforms, rounded to the kind);
 *   block kinds (DM_Q4_K / DM_Q6_K / DM_Q5_0 / DM_Q8_0): uniform random bytes with
 *     the f16 scale fields (d, and dmin for Q4_K) uniform in [lo, hi).
 */
#ifndef DISKMULE_SYNTH_H
#define DISKMULE_SYNTH_H

#include <stdint.h>

#ifndef DM_API
#if defined(__GNUC__)
#define DM_API __attribute__((visibility("default")))
#else
#define DM_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

DM_API int32_t dm_synth_fill_host(int32_t kind, uint64_t seed, uint64_t first_block,
                           uint64_t n_blocks, float sigma, float lo, float hi, void *dst);
DM_API int32_t dm_synth_fill_device(int32_t kind, uint64_t seed, uint64_t first_block,
                             uint64_t n_blocks, float sigma, float lo, float hi, void *dst,
                             void *stream);

#ifdef __cplusplus
}
#endif
#endif
