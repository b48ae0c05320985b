// dm_stack.cu -- device glue of a GLM-shaped decode stack (include/diskmule_stack.h):
// embedding row, residual add + RMSNorm, output head + greedy argmax. Each reproduces
// its reference's floating-point operations in order, so a stack decoded here picks
// the reference's tokens whenever its MoE outputs agree.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/diskmule_stack.h"
#include "dm_internal.cuh"

using dmi::fail;

namespace {

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits) { return __uint_as_float(bits << 16); }

__global__ void embed_kernel(const void *table, int f32, int vocab, int hidden, const int32_t *token,
                             float *h, int32_t *status) {
  const int t = *token;
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && status) atomicOr(status, DM_STACK_BAD_TOKEN);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
      h[i] = __int_as_float(0x7fc00000);
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x) {
    if (f32) h[i] = reinterpret_cast<const float *>(table)[(size_t)t * hidden + i];
    else h[i] = bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(table)[(size_t)t * hidden + i]);
  }
}

// src/glm52/cpu.rs:912-924. The mean square is a sequential f64 sum (each f32 square
// is exact in f64), so one thread adds them in order; the rest is elementwise.
constexpr int kNormThreads = 1024;

__global__ void __launch_bounds__(kNormThreads)
add_rms_norm_kernel(float *h, const float *delta, const float *weight, int n, float epsilon,
                    float *out, int32_t *status) {
  extern __shared__ float v[];
  __shared__ float scale;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float x = h[i];
    if (delta) {
      x = __fadd_rn(x, delta[i]);
      h[i] = x;
    }
    v[i] = x;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) {
      const double x = (double)v[i];
      sum = __dadd_rn(sum, __dmul_rn(x, x));
    }
    const float ms = __double2float_rn(__ddiv_rn(sum, (double)n));
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, epsilon)));
    if (!isfinite(scale) && status) atomicOr(status, DM_STACK_NON_FINITE_NORM);
  }
  __syncthreads();
  const float s = scale;
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(v[i], s), weight[i]);
}

// Output head: one thread per row, each a sequential chain over the columns
// (acc = acc + w * x, from -0.0, no contraction). Rows are staged 64 columns at a time
// into shared memory (coalesced 16-byte copies, chunk index XOR-swizzled by row so the
// per-row reads spread over the banks) with a two-stage cp.async pipeline.
constexpr int kHeadRows = 128;
constexpr int kHeadCols = 64;  // 128 bytes of bf16 per row per stage

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes));
}

__device__ __forceinline__ uint64_t argmax_key(float v, int row) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ordered = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // total order
  return ((uint64_t)ordered << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)row);
}

__global__ void __launch_bounds__(kHeadRows)
lm_head_kernel(const uint16_t *__restrict__ w, int vocab, int hidden, const float *__restrict__ x,
               float *logits, unsigned long long *best, int32_t *status) {
  extern __shared__ __align__(16) uint8_t smem[];
  float *xs = reinterpret_cast<float *>(smem);
  uint8_t *tiles = smem + (size_t)hidden * 4;  // [2][kHeadRows][128 B]
  const int r0 = blockIdx.x * kHeadRows;
  const int tid = threadIdx.x;
  for (int i = tid; i < hidden; i += blockDim.x) xs[i] = x[i];
  const int ntiles = hidden / kHeadCols;
  auto stage = [&](int tile, int buf) {
    uint8_t *dst = tiles + buf * kHeadRows * 128;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int idx = tid + j * kHeadRows;  // 1024 16-byte chunks
      const int row = idx >> 3, c = idx & 7;
      const bool valid = r0 + row < vocab;
      const uint16_t *src = w + (size_t)(valid ? r0 + row : 0) * hidden + tile * kHeadCols + c * 8;
      cp_async16(dst + row * 128 + ((c ^ (row & 7)) << 4), src, valid);
    }
    asm volatile("cp.async.commit_group;");
  };
  stage(0, 0);
  __syncthreads();
  float acc = -0.0f;
  for (int t = 0; t < ntiles; t++) {
    if (t + 1 < ntiles) {
      stage(t + 1, (t + 1) & 1);
      asm volatile("cp.async.wait_group 1;");
    } else {
      asm volatile("cp.async.wait_group 0;");
    }
    __syncthreads();
    const uint8_t *rowp = tiles + (t & 1) * kHeadRows * 128 + tid * 128;
    const float *xt = xs + t * kHeadCols;
#pragma unroll
    for (int c = 0; c < 8; c++) {
      const uint4 q = *reinterpret_cast<const uint4 *>(rowp + ((c ^ (tid & 7)) << 4));
      const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(words[k] << 16), xt[c * 8 + 2 * k]));
        acc = __fadd_rn(acc, __fmul_rn(__uint_as_float(words[k] & 0xffff0000u), xt[c * 8 + 2 * k + 1]));
      }
    }
    __syncthreads();
  }
  const int row = r0 + tid;
  unsigned long long key = 0;
  if (row < vocab) {
    if (logits) logits[row] = acc;
    if (!isfinite(acc) && status) atomicOr(status, DM_STACK_NON_FINITE_LOGIT);
    key = argmax_key(acc, row);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other > key ? other : key;
  }
  if ((tid & 31) == 0 && key) atomicMax(best, key);
}

__global__ void argmax_finish_kernel(const unsigned long long *best, int32_t *token) {
  *token = (int32_t)(0xFFFFFFFFu - (uint32_t)(*best & 0xFFFFFFFFull));
}

}  // namespace

extern "C" {

int32_t dm_stack_embed(dm_cuda_context *ctx, const void *table, int32_t table_type, int32_t vocab,
                       int32_t hidden, const int32_t *token, float *h, int32_t *status,
                       void *stream) {
  if (!ctx || !table || !token || !h) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (table_type != DM_BF16 && table_type != DM_F32)
    return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "embedding tables are bf16 or f32");
  if (vocab <= 0 || hidden <= 0) return fail(DM_ERR_EMPTY_INPUT, "empty embedding table");
  cudaSetDevice(ctx->device);
  cudaStream_t s = (cudaStream_t)stream;
  embed_kernel<<<(hidden + 255) / 256, 256, 0, s>>>(table, table_type == DM_F32, vocab, hidden,
                                                     token, h, status);
  DM_CUDA(cudaGetLastError(), "embedding launch");
  return DM_OK;
}

int32_t dm_stack_add_rms_norm(dm_cuda_context *ctx, float *h, const float *delta,
                              const float *weight, int32_t hidden, float epsilon, float *out,
                              int32_t *status, void *stream) {
  if (!ctx || !h || !weight || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (hidden <= 0) return fail(DM_ERR_EMPTY_INPUT, "rms_norm of an empty vector");
  if (hidden > 48 * 1024) return fail(DM_ERR_ELEMENT_COUNT, "hidden %d is above 49152", hidden);
  if (!(epsilon > 0.0f) || epsilon != epsilon || epsilon > 3.4e38f)
    return fail(DM_ERR_POSITIVE_PARAMETER, "RMSNorm epsilon requires a finite positive parameter");
  cudaSetDevice(ctx->device);
  const size_t smem = (size_t)hidden * 4;
  if (smem > 48 * 1024)
    DM_CUDA(cudaFuncSetAttribute(add_rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem), "norm shared memory");
  add_rms_norm_kernel<<<1, kNormThreads, smem, (cudaStream_t)stream>>>(h, delta, weight, hidden,
                                                                       epsilon, out, status);
  DM_CUDA(cudaGetLastError(), "rms_norm launch");
  return DM_OK;
}

int32_t dm_stack_lm_head_argmax(dm_cuda_context *ctx, const void *weight, int32_t weight_type,
                                int32_t vocab, int32_t hidden, const float *x, float *logits,
                                int32_t *token, int32_t *status, void *stream) {
  if (!ctx || !weight || !x || !token) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (weight_type != DM_BF16) return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "the output head is bf16");
  if (vocab <= 0 || hidden <= 0) return fail(DM_ERR_EMPTY_INPUT, "argmax of an empty input");
  if (hidden % kHeadCols) return fail(DM_ERR_ELEMENT_COUNT, "hidden must be a multiple of 64");
  if ((uintptr_t)weight & 15) return fail(DM_ERR_INVALID_ARGUMENT, "head weights must be 16-byte aligned");
  const size_t smem = (size_t)hidden * 4 + 2 * kHeadRows * 128;
  if (smem > 200 * 1024) return fail(DM_ERR_ELEMENT_COUNT, "hidden %d is too large for the head", hidden);
  cudaSetDevice(ctx->device);
  cudaStream_t s = (cudaStream_t)stream;
  // the argmax key lives in the context's status buffer (bytes 64..71)
  unsigned long long *best = reinterpret_cast<unsigned long long *>(
      reinterpret_cast<uint8_t *>(ctx->status) + 64);
  DM_CUDA(cudaMemsetAsync(best, 0, 8, s), "argmax reset");
  if (smem > 48 * 1024)
    DM_CUDA(cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem), "head shared memory");
  lm_head_kernel<<<(vocab + kHeadRows - 1) / kHeadRows, kHeadRows, smem, s>>>(
      reinterpret_cast<const uint16_t *>(weight), vocab, hidden, x, logits, best, status);
  argmax_finish_kernel<<<1, 1, 0, s>>>(best, token);
  DM_CUDA(cudaGetLastError(), "output head launch");
  return DM_OK;
}

}  // extern "C"
