// dm_synth.cu -- host and device fills of seeded synthetic tensors
// (include/diskmule_synth.h).
#include <cuda_runtime.h>

#include "../../include/diskmule_cuda.h"
#include "../../include/diskmule_synth.h"
#include "dm_synth.cuh"

namespace {

__global__ void synth_kernel(int kind, uint64_t seed, uint64_t first, uint64_t n, float sigma,
                             float lo, float hi, uint8_t *dst, int bytes) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint8_t block[256];
    dm::synth::fill_block(kind, seed, first + i, sigma, lo, hi, block);
    uint8_t *o = dst + i * bytes;
    for (int j = 0; j < bytes; j++) o[j] = block[j];
  }
}

}  // namespace

extern "C" {

int32_t dm_synth_fill_host(int32_t kind, uint64_t seed, uint64_t first_block, uint64_t n_blocks,
                           float sigma, float lo, float hi, void *dst) {
  int bytes = dm::synth::block_bytes(kind);
  if (bytes == 0) return DM_ERR_UNSUPPORTED_TENSOR_TYPE;
  if (!dst && n_blocks) return DM_ERR_INVALID_ARGUMENT;
  uint8_t *out = (uint8_t *)dst;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n_blocks; i++)
    dm::synth::fill_block(kind, seed, first_block + (uint64_t)i, sigma, lo, hi,
                          out + (uint64_t)i * bytes);
  return DM_OK;
}

int32_t dm_synth_fill_device(int32_t kind, uint64_t seed, uint64_t first_block, uint64_t n_blocks,
                             float sigma, float lo, float hi, void *dst, void *stream) {
  int bytes = dm::synth::block_bytes(kind);
  if (bytes == 0) return DM_ERR_UNSUPPORTED_TENSOR_TYPE;
  if (!dst && n_blocks) return DM_ERR_INVALID_ARGUMENT;
  if (n_blocks == 0) return DM_OK;
  uint64_t blocks = (n_blocks + 255) / 256;
  int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
  synth_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(kind, seed, first_block, n_blocks, sigma,
                                                       lo, hi, (uint8_t *)dst, bytes);
  return cudaGetLastError() == cudaSuccess ? DM_OK : DM_ERR_COMMAND;
}

}  // extern "C"
