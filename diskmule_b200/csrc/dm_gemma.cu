// dm_gemma.cu -- Gemma 4's whole feed-forward block around the routed experts
// (dm_gemma_ffn_* in include/diskmule_cuda.h).
//
// src/gemma4/cpu.rs:547-620 per token:
//   shared = rms_norm(down(gelu_tanh(gate s) * up s), shared_post_norm),
//            s = rms_norm(x, feed_forward_norm)                       (:548-558, :693-712)
//   routed = rms_norm(routed branch of x, routed_post_norm)            (:559-613)
//   hidden = (x + rms_norm(shared + routed, post_feed_forward_norm)) * layer_output_scale
// The dense shared FFN runs through the grouped expert kernels as a one-expert layer (its
// gate and up rows copied once into the fused [2W][H] layout of Gemma's expert tensors,
// every token a row of that expert), the routed branch is dm_moe_forward, and two row
// kernels do the norms: one CTA per token, block-wide sums of squares (the outputs are
// held to the 1e-3 relative-L2 bar; the router's own inputs keep their exact
// sequential chains inside dm_moe_forward).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>

#include "dm_internal.cuh"

using dmi::cuda_fail;
using dmi::fail;

namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) red[0] = s;
  }
  __syncthreads();
  return red[0];
}

// 1 / sqrt(mean(v^2) + eps), the rms_norm factor (src/cpu.rs:99-143)
__device__ __forceinline__ float inv_rms(float sumsq, int n, float eps) {
  return __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)n), eps)));
}

// out[t] = rms_norm(x[t], w): (x * w) * inv, one CTA per token
__global__ void __launch_bounds__(kRowThreads) weighted_norm_rows_kernel(const float *x,
                                                                         const float *w, float *out,
                                                                         int H, float eps,
                                                                         int32_t *status) {
  __shared__ float red[32];
  const float *row = x + (size_t)blockIdx.x * H;
  float s = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) s = fmaf(row[i], row[i], s);
  const float inv = inv_rms(block_sum(s, red), H, eps);
  if (threadIdx.x == 0 && !isfinite(inv)) atomicExch(status, dm::kStatusNonFiniteNorm);
  float *o = out + (size_t)blockIdx.x * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(row[i], w[i]), inv);
}

// hidden[t] = (x + rms_norm(rms_norm(shared, sp) + rms_norm(routed, rp), pf)) * scale.
// The CTA keeps the combined row in shared memory between the passes.
__global__ void __launch_bounds__(kRowThreads) gemma_finalize_kernel(
    const float *x, const float *shared, const float *routed, const float *sp, const float *rp,
    const float *pf, float scale, float *hidden, int H, float eps, int32_t *status) {
  extern __shared__ float comb[];
  __shared__ float red[32];
  const size_t base = (size_t)blockIdx.x * H;
  float ss = 0.0f, sr = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    ss = fmaf(shared[base + i], shared[base + i], ss);
    sr = fmaf(routed[base + i], routed[base + i], sr);
  }
  const float inv_s = inv_rms(block_sum(ss, red), H, eps);
  const float inv_r = inv_rms(block_sum(sr, red), H, eps);
  float sc = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float a = __fmul_rn(__fmul_rn(shared[base + i], sp[i]), inv_s);
    const float b = __fmul_rn(__fmul_rn(routed[base + i], rp[i]), inv_r);
    const float c = __fadd_rn(a, b);
    comb[i] = c;
    sc = fmaf(c, c, sc);
  }
  const float inv_c = inv_rms(block_sum(sc, red), H, eps);
  if (threadIdx.x == 0 && !(isfinite(inv_s) && isfinite(inv_r) && isfinite(inv_c)))
    atomicExch(status, dm::kStatusNonFiniteNorm);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float c = __fmul_rn(__fmul_rn(comb[i], pf[i]), inv_c);
    hidden[base + i] = __fmul_rn(__fadd_rn(x[base + i], c), scale);
  }
}

}  // namespace

struct dm_gemma_ffn {
  dm_moe_layer *routed = nullptr;  // the caller's routed layer (not owned)
  dm_moe_layer *dense = nullptr;   // one-expert layer over the shared FFN (owned)
  void *owned = nullptr;           // fused gate/up copy, the dense layer's unit vectors
  dm_gemma_ffn_desc desc{};
  float epsilon = 1e-6f;
  int hidden = 0;
  // per-call scratch
  void *scratch = nullptr;
  int capacity = 0;
  float *shared_in = nullptr, *shared_raw = nullptr, *routed_out = nullptr;
  int32_t *ids = nullptr, *status = nullptr;
};

extern "C" {

void dm_gemma_ffn_destroy(dm_gemma_ffn *B) {
  if (!B) return;
  if (B->routed) cudaSetDevice(B->routed->ctx->device);
  if (B->dense) dm_moe_layer_destroy(B->dense);
  if (B->owned) cudaFree(B->owned);
  if (B->scratch) cudaFree(B->scratch);
  cudaGetLastError();
  delete B;
}

int32_t dm_gemma_ffn_create(dm_moe_layer *routed, const dm_gemma_ffn_desc *desc,
                            dm_gemma_ffn **out) {
  if (!routed || !desc || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  const dm_moe_desc &rd = routed->desc;
  if (rd.family != DM_FAMILY_GEMMA4)
    return fail(DM_ERR_INVALID_ARGUMENT, "the routed layer is not a Gemma 4 layer");
  if (routed->local_experts != rd.experts)
    return fail(DM_ERR_INVALID_ARGUMENT, "the routed layer must hold every expert");
  const int H = rd.hidden, W = desc->width;
  if (W <= 0 || W % 32) return fail(DM_ERR_ELEMENT_COUNT, "feed-forward width must be a positive multiple of 32");
  if (!desc->gate || !desc->up || !desc->down || !desc->feed_forward_norm ||
      !desc->shared_post_norm || !desc->routed_post_norm || !desc->post_feed_forward_norm)
    return fail(DM_ERR_INVALID_ARGUMENT, "null weight pointer");
  if (desc->gate_type != desc->up_type)
    return fail(DM_ERR_INVALID_ARGUMENT, "the shared FFN's gate and up must share a type");
  if (!std::isfinite(desc->layer_output_scale))
    return fail(DM_ERR_NON_FINITE, "layer_output_scale must be finite");
  const uint64_t gate_rb = dm::row_bytes(desc->gate_type, H);
  if (gate_rb == 0 || dm::row_bytes(desc->down_type, W) == 0)
    return fail(DM_ERR_ELEMENT_COUNT, "shared FFN rows are not a whole number of blocks");
  DM_CUDA(cudaSetDevice(routed->ctx->device), "cudaSetDevice");
  dm_gemma_ffn *B = new dm_gemma_ffn();
  B->routed = routed;
  B->desc = *desc;
  B->epsilon = rd.epsilon;
  B->hidden = H;
  // fused [gate rows; up rows] copy and unit vectors / a zero router row for the
  // one-expert layer (its router is never run: every token is a row of expert 0)
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t gu = (size_t)W * gate_rb;
  const size_t bytes = al(2 * gu) + al((size_t)H * 4) + 2 * al((size_t)H * 4) + al(4);
  if (cudaMalloc(&B->owned, bytes) != cudaSuccess) {
    B->owned = nullptr;
    dm_gemma_ffn_destroy(B);
    return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes for the shared FFN", bytes);
  }
  uint8_t *fused = (uint8_t *)B->owned;
  float *router = (float *)(fused + al(2 * gu));
  float *ones = (float *)((uint8_t *)router + al((size_t)H * 4));
  float *one = (float *)((uint8_t *)ones + al((size_t)H * 4));
  cudaStream_t s = routed->ctx->stream;
  cudaError_t err = cudaMemcpyAsync(fused, desc->gate, gu, cudaMemcpyDeviceToDevice, s);
  if (err == cudaSuccess) err = cudaMemcpyAsync(fused + gu, desc->up, gu, cudaMemcpyDeviceToDevice, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(router, 0, (size_t)H * 4, s);
  std::vector<float> h_ones(H, 1.0f);
  if (err == cudaSuccess) err = cudaMemcpyAsync(ones, h_ones.data(), (size_t)H * 4, cudaMemcpyHostToDevice, s);
  if (err == cudaSuccess) err = cudaMemcpyAsync(one, h_ones.data(), 4, cudaMemcpyHostToDevice, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess) {
    dm_gemma_ffn_destroy(B);
    return cuda_fail(err, "shared FFN set-up");
  }
  dm_moe_desc d{};
  d.family = DM_FAMILY_GEMMA4;
  d.hidden = H;
  d.intermediate = W;
  d.experts = 1;
  d.top_k = 1;
  d.n_groups = 1;
  d.topk_groups = 1;
  d.routed_scale = 1.0f;
  d.epsilon = rd.epsilon;
  d.input_type = DM_F32;
  d.router_type = DM_F32;
  d.router = router;
  d.router_scale = ones;
  d.routed_pre_norm = ones;
  d.expert_scale = one;
  d.gate_type = desc->gate_type;
  d.up_type = desc->gate_type;
  d.down_type = desc->down_type;
  d.gate = fused;
  d.up = nullptr;
  d.down = desc->down;
  int32_t rc = dm_moe_layer_create(routed->ctx, &d, &B->dense);
  if (rc != DM_OK) {
    B->dense = nullptr;
    dm_gemma_ffn_destroy(B);
    return rc;
  }
  *out = B;
  return DM_OK;
}

int32_t dm_gemma_ffn_forward(dm_gemma_ffn *B, const float *x, float *hidden, int32_t tokens,
                             uint32_t *sel_idx, float *sel_weight, void *stream) {
  if (!B || !x || !hidden) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  if (((uintptr_t)x | (uintptr_t)hidden) & 15)
    return fail(DM_ERR_INVALID_ARGUMENT, "x and hidden must be 16-byte aligned device pointers");
  const int H = B->hidden;
  DM_CUDA(cudaSetDevice(B->routed->ctx->device), "cudaSetDevice");
  if (tokens > B->capacity) {
    if (B->scratch) {
      cudaDeviceSynchronize();
      cudaFree(B->scratch);
    }
    B->scratch = nullptr;
    B->capacity = 0;
    auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t rows = (size_t)tokens * H * 4;
    const size_t bytes = 3 * al(rows) + al((size_t)tokens * 4) + al(4);
    if (cudaMalloc(&B->scratch, bytes) != cudaSuccess) {
      B->scratch = nullptr;
      return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of block scratch", bytes);
    }
    uint8_t *p = (uint8_t *)B->scratch;
    B->shared_in = (float *)p;
    B->shared_raw = (float *)(p + al(rows));
    B->routed_out = (float *)(p + 2 * al(rows));
    B->ids = (int32_t *)(p + 3 * al(rows));
    B->status = (int32_t *)(p + 3 * al(rows) + al((size_t)tokens * 4));
    DM_CUDA(cudaMemset(B->ids, 0, (size_t)tokens * 4), "expert ids");  // every row: expert 0
    B->capacity = tokens;
  }
  cudaStream_t s = (cudaStream_t)stream;
  DM_CUDA(cudaMemsetAsync(B->status, 0, 4, s), "status reset");
  weighted_norm_rows_kernel<<<tokens, kRowThreads, 0, s>>>(x, B->desc.feed_forward_norm,
                                                           B->shared_in, H, B->epsilon, B->status);
  int32_t rc = dm_moe_expert_rows(B->dense, B->shared_in, B->ids, tokens, B->shared_raw, stream);
  if (rc != DM_OK) return rc;
  rc = dm_moe_forward(B->routed, x, B->routed_out, tokens, sel_idx, sel_weight, stream);
  if (rc != DM_OK) return rc;
  const size_t smem = (size_t)H * 4;
  if (smem > 48 * 1024) dm::ensure_smem_limit((const void *)gemma_finalize_kernel);
  gemma_finalize_kernel<<<tokens, kRowThreads, smem, s>>>(
      x, B->shared_raw, B->routed_out, B->desc.shared_post_norm, B->desc.routed_post_norm,
      B->desc.post_feed_forward_norm, B->desc.layer_output_scale, hidden, H, B->epsilon,
      B->status);
  DM_CUDA(cudaGetLastError(), "Gemma feed-forward block");
  return DM_OK;
}

int32_t dm_gemma_ffn_status(dm_gemma_ffn *B, void *stream) {
  if (!B) return fail(DM_ERR_INVALID_ARGUMENT, "null block");
  DM_CUDA(cudaSetDevice(B->routed->ctx->device), "cudaSetDevice");
  int32_t st[2] = {0, 0};
  cudaStream_t s = (cudaStream_t)stream;
  if (B->status) DM_CUDA(cudaMemcpyAsync(&st[0], B->status, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaMemcpyAsync(&st[1], B->routed->args.status, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaStreamSynchronize(s), "Gemma feed-forward block");
  for (int32_t v : st) {
    if (v == dm::kStatusNonFiniteRouter) return fail(DM_ERR_NON_FINITE, "router produced a non-finite score");
    if (v == dm::kStatusNonFiniteNorm) return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");
    if (v == dm::kStatusTimeout) return fail(DM_ERR_TIMEOUT, "a bounded wait ran out");
  }
  return DM_OK;
}

}  // extern "C"
