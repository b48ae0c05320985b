// dm_oracle_synth.cpp -- the seeded synthetic-input generator inside the oracle library.
//
// TEST INFRASTRUCTURE ONLY. The reference CPU arm of bench.py and the tests generate
// the synthetic layer's bytes (weights, token rows) with this function, so that timing
// or checking the oracle never loads the CUDA library. It evaluates the same
// counter-based generator the product's fills use (diskmule_b200/csrc/dm_synth.cuh,
// compiled here as plain C++), so host bytes equal device bytes by construction.
#include <stdint.h>

#include "../diskmule_b200/csrc/dm_synth.cuh"

extern "C" __attribute__((visibility("default"))) int32_t dmo_synth_fill(
    int32_t kind, uint64_t seed, uint64_t first_block, uint64_t n_blocks, float sigma,
    float lo, float hi, void *dst) {
  const int bytes = dm::synth::block_bytes(kind);
  if (bytes == 0) return -1;
  if (!dst && n_blocks) return -9;
  uint8_t *out = (uint8_t *)dst;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n_blocks; i++)
    dm::synth::fill_block(kind, seed, first_block + (uint64_t)i, sigma, lo, hi,
                          out + (uint64_t)i * bytes);
  return 0;
}
