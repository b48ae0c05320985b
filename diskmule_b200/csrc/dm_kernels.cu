// dm_kernels.cu -- sm_100a kernels of the routed-expert path (router -> top-k ->
// dispatch -> expert gate/up -> expert down -> combine) and the Metal-style
// operators (matvec, top-k softmax, gelu/silu multiply, rms_norm).
//
// Bit-exactness rules (the parts the reference's selection depends on):
//   * router logits are one sequential chain per (token, expert) in column order:
//     fma for the GGUF path (src/cpu.rs:389-397), multiply-then-add for GLM
//     (src/glm52/cpu.rs:1177-1185); every op uses an explicit _rn intrinsic so
//     nothing is contracted or reassociated;
//   * Gemma's router input reproduces src/cpu.rs:99-143 and src/gemma4/cpu.rs:562-573;
//   * top-k orders by (value desc, index asc) under the IEEE total order.
// Expert products accumulate in f32 in a different order than the reference and
// are held to the relative-L2 tolerance instead.
#include "dm_kernels.cuh"
#include "dm_tc.cuh"

#include <algorithm>
#include <mutex>
#include <cstdio>
#include <set>
#include <utility>

namespace dm {

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  return v;
}

__device__ __forceinline__ float load_as_f32(const void *p, size_t i, bool bf16) {
  if (bf16) return bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(p)[i]);
  return reinterpret_cast<const float *>(p)[i];
}

cudaError_t ensure_smem_limit(const void *kernel) {
  static std::mutex lock;
  static std::set<std::pair<const void *, int>> done;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> guard(lock);
  if (done.count({kernel, device})) return cudaSuccess;
  int optin = 0;
  cudaFuncAttributes attr;
  err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (err == cudaSuccess) err = cudaFuncGetAttributes(&attr, kernel);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               optin - (int)attr.sharedSizeBytes);
  if (err == cudaSuccess) done.insert({kernel, device});
  return err;
}

// Raise the kernel's limit when `bytes` needs it; a failure stays recorded as the
// last CUDA error, so the caller's launch check reports it.
template <typename F>
static void set_smem(F *kernel, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaError_t err = ensure_smem_limit((const void *)kernel);
    if (err != cudaSuccess) fprintf(stderr, "diskmule_cuda: shared memory limit: %s\n", cudaGetErrorString(err));
  }
}

// ---------------------------------------------------------------------------
// router transpose (layer set-up): [E][H] -> [H][E1], optional extra column E
// ---------------------------------------------------------------------------

// columns >= E1 of the [H][ld] result are zero
__global__ void transpose_router_kernel(const void *src, int bf16, int E, int H,
                                        const float *extra, void *dst, int E1, int ld) {
  size_t n = (size_t)H * ld;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n;
       idx += (size_t)gridDim.x * blockDim.x) {
    int h = (int)(idx / ld), e = (int)(idx % ld);
    if (bf16) {
      uint16_t v = e < E ? reinterpret_cast<const uint16_t *>(src)[(size_t)e * H + h] : 0;
      reinterpret_cast<uint16_t *>(dst)[idx] = v;
    } else {
      float v = e < E ? reinterpret_cast<const float *>(src)[(size_t)e * H + h]
                      : (e < E1 ? extra[h] : 0.0f);
      reinterpret_cast<float *>(dst)[idx] = v;
    }
  }
}

int launch_transpose_router(const void *src, int src_bf16, int E, int H, const float *extra_col,
                            void *dst, cudaStream_t stream) {
  int E1 = E + (extra_col ? 1 : 0);
  int ld = router_ld(E1);
  size_t n = (size_t)H * ld;
  int blocks = (int)std::min<size_t>((n + 255) / 256, 4096);
  transpose_router_kernel<<<blocks, 256, 0, stream>>>(src, src_bf16, E, H, extra_col, dst, E1, ld);
  return 1;
}

// ---------------------------------------------------------------------------
// Gemma router / expert input (src/gemma4/cpu.rs:559-573, rms_norm src/cpu.rs:99-143)
// ---------------------------------------------------------------------------

// Gemma router and expert inputs (src/gemma4/cpu.rs:559-573, rms_norm src/cpu.rs:99-143).
// The sum of squares is the reference's sequential fma fold, so each token's chain is one
// thread: a CTA takes 16 tokens, streams their rows through a 3-stage ring of 256-column
// chunks (cp.async, all threads), and warp 0 runs the 16 chains at fma latency; then all
// threads write both outputs (x re-read from L2).
constexpr int kPrepTokens = 16;
constexpr int kPrepChunk = 256;
constexpr int kPrepStages = 3;
constexpr int kPrepLd = kPrepChunk + 4;  // padded row: lane t reads row t at one column

__device__ __forceinline__ void prep_cp16(float *dst, const float *src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

__global__ void __launch_bounds__(256) gemma_prep_kernel(ForwardArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float ring[];  // [kPrepStages][kPrepTokens][kPrepLd]
  __shared__ float inv_s[kPrepTokens];
  const int H = a.H;
  const int t0 = blockIdx.x * kPrepTokens;
  const int nt = min(kPrepTokens, a.T - t0);
  const float *x = reinterpret_cast<const float *>(a.x);
  // the norm vectors are read by every token of the CTA: ask L2 for them now
  for (int i = threadIdx.x * 32; i < H; i += blockDim.x * 32) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a.router_scale + i));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a.routed_pre_norm + i));
  }
  // Few tokens: whole rows fit the buffer ([nt][H + 4]), all requested at once.
  // Otherwise 256-column chunks through the ring.
  const int HP = H + 4;
  const bool flat = nt * HP <= kPrepStages * kPrepTokens * kPrepLd;
  const int nchunks = flat ? 1 : (H + kPrepChunk - 1) / kPrepChunk;
  const int cw = flat ? H : kPrepChunk, ld = flat ? HP : kPrepLd;
  auto issue = [&](int c) {
    if (c < nchunks) {
      const int c0 = c * cw, w4 = min(cw, H - c0) / 4;
      float *st = ring + (flat ? 0 : (c % kPrepStages) * kPrepTokens * kPrepLd);
      for (int idx = threadIdx.x; idx < nt * w4; idx += blockDim.x) {
        const int tt = idx / w4, q = idx - tt * w4;
        prep_cp16(st + tt * ld + 4 * q, x + (size_t)(t0 + tt) * H + c0 + 4 * q);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int c = 0; c < kPrepStages - 1; c++) issue(c);
  float s = 0.0f;
  for (int c = 0; c < nchunks; c++) {
    issue(c + kPrepStages - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(kPrepStages - 1) : "memory");
    __syncthreads();
    if (threadIdx.x < nt) {
      const float *row = ring + (flat ? 0 : (c % kPrepStages) * kPrepTokens * kPrepLd) + threadIdx.x * ld;
      const int w = min(cw, H - c * cw);
      // 16-byte reads (padded rows spread the banks) from two register sets of 16 values:
      // the next 16 load while the current 16 feed the chain (w % 32 == 0)
      float va[16], vb[16];
      auto load16 = [&](int i, float *v) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 q = *reinterpret_cast<const float4 *>(row + i + 4 * j);
          v[4 * j] = q.x, v[4 * j + 1] = q.y, v[4 * j + 2] = q.z, v[4 * j + 3] = q.w;
        }
      };
      load16(0, va);
      for (int i = 0; i < w; i += 32) {
        load16(i + 16, vb);
#pragma unroll
        for (int j = 0; j < 16; j++) s = __fmaf_rn(va[j], va[j], s);
        load16(i + 32 < w ? i + 32 : i, va);  // last pass: a harmless reload
#pragma unroll
        for (int j = 0; j < 16; j++) s = __fmaf_rn(vb[j], vb[j], s);
      }
    }
    __syncthreads();  // the stage is refilled by the next iteration's issue
  }
  if (threadIdx.x < nt) {
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), a.epsilon)));
    if (!isfinite(inv)) atomicExch(a.status, kStatusNonFiniteNorm);
    inv_s[threadIdx.x] = inv;
  }
  __syncthreads();
  // outputs: four independent 16-byte pieces per thread and pass, so the L2 reads overlap
  const int h4 = H / 4, n4 = nt * h4;
  for (int base = threadIdx.x; base < n4; base += 4 * blockDim.x) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int idx = base + u * blockDim.x;
      if (idx < n4) {
        const int tt = idx / h4, q = idx - tt * h4;
        v[u] = *reinterpret_cast<const float4 *>(x + (size_t)(t0 + tt) * H + 4 * q);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int idx = base + u * blockDim.x;
      if (idx >= n4) break;
      const int tt = idx / h4, q = idx - tt * h4;
      const size_t o = (size_t)(t0 + tt) * H + 4 * q;
      const float inv = inv_s[tt];
      const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      float ri[4], ei[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {  // caller vectors: 4-byte alignment only
        const float rr = a.router_scale[4 * q + j], pp = a.routed_pre_norm[4 * q + j];
        ri[j] = __fmul_rn(__fmul_rn(vv[j], inv), __fmul_rn(rr, a.inv_sqrt_hidden));
        ei[j] = __fmul_rn(__fmul_rn(vv[j], pp), inv);
      }
      *reinterpret_cast<float4 *>(a.router_in + o) = make_float4(ri[0], ri[1], ri[2], ri[3]);
      *reinterpret_cast<float4 *>(a.expert_in + o) = make_float4(ei[0], ei[1], ei[2], ei[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// router logits: one sequential chain per (token, expert)
// ---------------------------------------------------------------------------

// Few tokens: a CTA owns EPC <= 8 experts and up to RT <= 4 tokens; EPC*RT threads of
// warp 0 run the sequential chains. EPC is chosen so that the grid spreads the router rows
// over most SMs. The experts' router rows ([E1][H] f32 copy made at set-up, so one row is
// contiguous) are requested up front as 1-D bulk copies in chunks of kRsChunk columns,
// each chunk completing an mbarrier, and land in rows padded by 16 bytes (threads of one
// token read different rows at the same column without bank conflicts). The token rows
// arrive the same way, f32 or bf16 as given (a bf16 value is widened in the chain thread,
// off the chain's critical path). A chain runs at the dependent-add latency (about 4.2
// cycles per column on B200): weights and inputs for the next 32 or 64 columns are loaded
// while the current ones feed the chain, and the GLM family's products are formed before
// their sums.
constexpr int kSmallExperts = 8;
constexpr int kRsChunk = 1024;
constexpr int kRsMaxChunks = 12;  // H <= 12288

__device__ __forceinline__ void rs_bulk(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Bounded wait for the phase with parity 0 of a router barrier; on timeout the status
// word records it and the caller goes on (its sums are then discarded by the host).
__device__ __forceinline__ void rs_wait(uint32_t bar, int32_t *status) {
  const long long start = clock64();
  uint32_t done = 0;
  while (!done) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar)
        : "memory");
    if (!done && clock64() - start > 200000000ll) {
      atomicExch(status, kStatusTimeout);
      break;
    }
  }
}

// Eight inputs of a token row in shared memory, as f32, from column h (h % 8 == 0).
template <bool XBF16>
__device__ __forceinline__ void rs_x8(const void *xr, int h, float *v) {
  if (XBF16) {
    const uint4 u = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(xr) + h);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(xr) + h);
    const float4 b = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(xr) + h + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

template <int N, bool XBF16>
__device__ __forceinline__ void rs_load(const float *wr, const void *xr, int h, float *w, float *xv) {
#pragma unroll
  for (int i = 0; i < N / 4; i++) {
    const float4 a = *reinterpret_cast<const float4 *>(wr + h + 4 * i);
    w[4 * i] = a.x, w[4 * i + 1] = a.y, w[4 * i + 2] = a.z, w[4 * i + 3] = a.w;
  }
#pragma unroll
  for (int i = 0; i < N / 8; i++) rs_x8<XBF16>(xr, h + 8 * i, xv + 8 * i);
}

// Columns [h0, h1) of one chain (h1 - h0 a multiple of 32), in order.
template <bool GLM, bool XBF16>
__device__ __forceinline__ float rs_chain(const float *wr, const void *xr, int h0, int h1, float s) {
  if (GLM) {
    // products of 64 columns first, then their sums; the next 64 columns load meanwhile
    constexpr int B = 64;
    int h = h0;
    if (h + B <= h1) {
      float w[B], xv[B];
      rs_load<B, XBF16>(wr, xr, h, w, xv);
      for (; h + B <= h1; h += B) {
        float p[B];
#pragma unroll
        for (int j = 0; j < B; j++) p[j] = __fmul_rn(w[j], xv[j]);
        const int hn = h + 2 * B <= h1 ? h + B : h;  // last batch: a harmless reload
        rs_load<B, XBF16>(wr, xr, hn, w, xv);
#pragma unroll
        for (int j = 0; j < B; j++) s = __fadd_rn(s, p[j]);
      }
    }
    for (; h < h1; h += 32) {  // a 32-column tail
      float w[32], xv[32];
      rs_load<32, XBF16>(wr, xr, h, w, xv);
#pragma unroll
      for (int j = 0; j < 32; j++) s = __fadd_rn(s, __fmul_rn(w[j], xv[j]));
    }
    return s;
  }
  // fma chain: two register sets of 16 columns, one loading while the other feeds the chain
  float wa[16], xa[16], wb[16], xb[16];
  rs_load<16, XBF16>(wr, xr, h0, wa, xa);
  for (int h = h0; h < h1; h += 32) {
    rs_load<16, XBF16>(wr, xr, h + 16, wb, xb);
#pragma unroll
    for (int j = 0; j < 16; j++) s = __fmaf_rn(wa[j], xa[j], s);
    const int hn = h + 32 < h1 ? h + 32 : h;  // last pass: a harmless reload
    rs_load<16, XBF16>(wr, xr, hn, wa, xa);
#pragma unroll
    for (int j = 0; j < 16; j++) s = __fmaf_rn(wb[j], xb[j], s);
  }
  return s;
}

template <bool GLM, bool XBF16>
__global__ void __launch_bounds__(256) router_small_kernel(const float *rows, const void *x, int T,
                                                          int H, int E1, int RT, int EPC,
                                                          const float *lbias, int E,
                                                          float *logits, int32_t *status) {
  extern __shared__ __align__(16) float smem[];
  __shared__ __align__(8) unsigned long long bars[kRsMaxChunks + 1];  // chunks, then x
  constexpr int kXb = XBF16 ? 2 : 4;                       // bytes per input value
  const int HP = H + 4;                                     // padded weight rows (16 bytes)
  const int XP = H + 16 / kXb;                              // padded token rows (16 bytes)
  float *ws = smem;                                         // [EPC][H + 4] f32
  uint8_t *xs = reinterpret_cast<uint8_t *>(ws + EPC * HP);  // [RT][XP] f32 or bf16
  const int e0 = blockIdx.x * EPC, t0 = blockIdx.y * RT;
  const int nt = min(RT, T - t0);
  const int ne = min(EPC, E1 - e0);
  const int nchunks = (H + kRsChunk - 1) / kRsChunk;
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(bars);
  const uint32_t xbar = (uint32_t)__cvta_generic_to_shared(&bars[kRsMaxChunks]);
  if (threadIdx.x == 0) {
    for (int c = 0; c < nchunks; c++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * c));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(xbar));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // One thread of warp 1 (no chain runs there) issues the copies: issuing stalls while the
  // copy engine's queue is full, so it stays off the chain warp. The rows are layer
  // weights, so the first chunk is requested before pdl_wait(), while the kernel that
  // writes the token rows still runs; then the token rows, then the other chunks.
  const uint32_t wbase = (uint32_t)__cvta_generic_to_shared(ws);
  const uint32_t xbase = (uint32_t)__cvta_generic_to_shared(xs);
  constexpr int kIssuer = 32;
  auto issue_chunks = [&](int c_begin, int c_end) {
    for (int c = c_begin; c < c_end; c++) {
      const int h0 = c * kRsChunk, w = min(kRsChunk, H - h0);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar0 + 8 * c),
                   "r"((uint32_t)(ne * w * 4))
                   : "memory");
      for (int el = 0; el < ne; el++)
        rs_bulk(wbase + (uint32_t)(el * HP + h0) * 4, rows + (size_t)(e0 + el) * H + h0,
                (uint32_t)w * 4, bar0 + 8 * c);
    }
  };
  if (threadIdx.x == kIssuer) issue_chunks(0, 1);
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == kIssuer) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(xbar),
                 "r"((uint32_t)(nt * H * kXb))
                 : "memory");
    for (int tt = 0; tt < nt; tt++)
      rs_bulk(xbase + (uint32_t)(tt * XP * kXb),
              reinterpret_cast<const uint8_t *>(x) + (size_t)(t0 + tt) * H * kXb, (uint32_t)(H * kXb),
              xbar);
    issue_chunks(1, nchunks);
  }
  const int el = threadIdx.x % EPC, tl = threadIdx.x / EPC;
  if (tl < nt && el < ne) {
    const void *xr = xs + (size_t)tl * XP * kXb;
    const float *wr = ws + el * HP;
    rs_wait(xbar, status);
    float s = GLM ? -0.0f : 0.0f;
    for (int c = 0; c < nchunks; c++) {
      rs_wait(bar0 + 8 * c, status);  // its copies complete by themselves
      const int h0 = c * kRsChunk;
      s = rs_chain<GLM, XBF16>(wr, xr, h0, min(H, h0 + kRsChunk), s);
    }
    if (lbias && e0 + el < E) s = __fadd_rn(s, lbias[e0 + el]);
    logits[(size_t)(t0 + tl) * E1 + e0 + el] = s;
  }
}

// router [E][H] (f32 or bf16) + optional extra row (Qwen shared gate) -> [E1][H] f32
__global__ void router_rows_kernel(const void *src, int bf16, int E, int H, const float *extra,
                                   float *dst) {
  const size_t n = (size_t)(E + (extra ? 1 : 0)) * H;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t e = idx / H, h = idx % H;
    dst[idx] = e < (size_t)E ? load_as_f32(src, idx, bf16 != 0) : extra[h];
  }
}

int launch_router_rows(const void *router, int bf16, int E, int H, const float *extra_col,
                       float *dst, cudaStream_t stream) {
  const size_t n = (size_t)(E + (extra_col ? 1 : 0)) * H;
  router_rows_kernel<<<(int)std::min<size_t>((n + 255) / 256, 4096), 256, 0, stream>>>(
      router, bf16, E, H, extra_col, dst);
  return 1;
}

// Many tokens: register-tiled SIMT matmul. A CTA computes a 32-token x 64-expert tile;
// thread (tx, ty) holds tokens 4ty.. x experts 4tx.. = 16 chains, each still one
// sequential chain over h in the reference's order (so logits stay bit-exact), computed
// two experts at a time with packed f32x2 instructions (one rounding per element, as
// scalar code). Operands come from x transposed once per forward, [h][t] (a 16-byte load
// yields a thread's four tokens, each paired with itself in registers for the packed
// steps: 32 bytes of shared memory per 8 packed steps), and the router padded to f32
// [h][128k] at set-up, through a 3-stage cp.async pipeline of
// 64-wide h chunks (one block barrier per 64 steps of the chains); operands are read with
// plain shared-memory loads, so the compiler can issue the next step's loads ahead of the
// current step's FMAs.
//
// Step arithmetic. The softmax families' reference chains are fused multiply-adds. GLM's
// is `s + w * x` with the product rounded first (src/glm52/cpu.rs:1121-1187). When w and
// x are both bf16 (8 significant bits each) the product has at most 16 significant bits,
// so it is an exact f32 value unless it leaves the normal range; with every nonzero |w|
// and |x| in [2^-60, 2^60) it cannot, the first rounding is the identity, and
// fma(w, x, s) == s + w * x bit for bit. The GLM kernels then take the fused step (half
// the FP32 instructions); otherwise (an f32 router or input, or a tile holding a value
// outside that range) they keep the two-instruction step.
constexpr int kRgTokens = 32, kRgExperts = 64, kRgChunk = 64, kRgThreads = 128, kRgStages = 3;
constexpr int kRgXBytes = kRgChunk * kRgTokens * 4;
constexpr int kRgStageBytes = kRgXBytes + kRgChunk * kRgExperts * 4;

template <bool FMA>
__device__ __forceinline__ uint64_t rg_step(uint64_t w, uint64_t x, uint64_t s) {
  uint64_t r;
  if (!FMA) {
    uint64_t p;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(w), "l"(x));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(s), "l"(p));
  } else {
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(w), "l"(x), "l"(s));
  }
  return r;
}

__device__ __forceinline__ bool outside_exact_range(float v) {
  const float a = fabsf(v);
  return v != 0.0f && !(a >= 0x1p-60f && a < 0x1p60f);  // NaN and inf fail the range test
}

// Whether a GLM router CTA over token tile `tile` may take the fused step: the layer's
// router is in range and no 32x32 input tile of its tokens holds a value out of range.
__device__ __forceinline__ bool router_fused_step(bool glm, int exact_products,
                                                  const uint8_t *tiny, int tile, int hblocks) {
  if (!glm) return true;
  int bad = !exact_products || !tiny;
  if (!bad)
    for (int i = threadIdx.x; i < hblocks; i += blockDim.x) bad |= tiny[(size_t)tile * hblocks + i];
  return !__syncthreads_or(bad);
}

__global__ void bf16_range_check_kernel(const uint16_t *v, size_t n, int32_t *flag) {
  bool bad = false;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    bad |= outside_exact_range(__uint_as_float((uint32_t)v[i] << 16));
  if (__syncthreads_or(bad) && threadIdx.x == 0) *flag = 1;
}

int launch_bf16_range_check(const uint16_t *v, size_t n, int32_t *flag, cudaStream_t stream) {
  bf16_range_check_kernel<<<(int)std::min<size_t>((n + 255) / 256, 1184), 256, 0, stream>>>(
      v, n, flag);
  return 1;
}

__device__ __forceinline__ void rg_cp16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// (v, v) as an f32 pair for a packed step
__device__ __forceinline__ uint64_t pair_same(float v) {
  const uint64_t u = __float_as_uint(v);
  return (u << 32) | u;
}

template <bool FMA>
__device__ __forceinline__ void router_gemm_chains(uint64_t (&acc)[4][2], const float *w32,
                                                   int wld, const float *xT1, int xld, int H,
                                                   uint8_t *rg_smem) {
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kRgExperts, t0 = blockIdx.y * kRgTokens;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(rg_smem);
  const int nchunks = H / kRgChunk;
  auto issue = [&](int c) {
    if (c < nchunks) {
      const uint32_t st = sbase + (uint32_t)(c % kRgStages) * kRgStageBytes;
      const int h0 = c * kRgChunk;
#pragma unroll
      for (int i = 0; i < kRgChunk * 8 / kRgThreads; i++) {  // x: rows of 32 tokens x 4 bytes
        const int f = tid + kRgThreads * i, row = f >> 3, piece = f & 7;
        rg_cp16(st + row * 128 + piece * 16, xT1 + (size_t)(h0 + row) * xld + t0 + 4 * piece);
      }
#pragma unroll
      for (int i = 0; i < kRgChunk * 16 / kRgThreads; i++) {  // w: rows of 64 experts x 4 bytes
        const int f = tid + kRgThreads * i, row = f >> 4, piece = f & 15;
        rg_cp16(st + kRgXBytes + row * 256 + piece * 16, w32 + (size_t)(h0 + row) * wld + e0 + 4 * piece);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int c = 0; c < kRgStages - 1; c++) issue(c);
  for (int c = 0; c < nchunks; c++) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kRgStages - 2) : "memory");
    __syncthreads();  // chunk c is in; every thread is done with chunk c - 1
    issue(c + kRgStages - 1);
    const uint8_t *stp = rg_smem + (size_t)(c % kRgStages) * kRgStageBytes;
#pragma unroll
    for (int kk = 0; kk < kRgChunk; kk++) {
      const float4 xv = *reinterpret_cast<const float4 *>(stp + kk * 128 + ty * 16);
      const ulonglong2 w = *reinterpret_cast<const ulonglong2 *>(stp + kRgXBytes + kk * 256 + tx * 16);
      const uint64_t xp[4] = {pair_same(xv.x), pair_same(xv.y), pair_same(xv.z), pair_same(xv.w)};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        acc[i][0] = rg_step<FMA>(w.x, xp[i], acc[i][0]);
        acc[i][1] = rg_step<FMA>(w.y, xp[i], acc[i][1]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <bool GLM>
__global__ void __launch_bounds__(kRgThreads) router_gemm_kernel(const float *w32, int wld,
                                                                 const float *xT1, int xld, int T,
                                                                 int H, int E1, const float *lbias,
                                                                 int E, float *logits,
                                                                 const uint8_t *tiny,
                                                                 int exact_products) {
  pdl_wait();
  extern __shared__ __align__(16) uint8_t rg_smem[];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kRgExperts, t0 = blockIdx.y * kRgTokens;
  uint64_t acc[4][2];  // token 4ty + i, experts (4tx + 2jp, 4tx + 2jp + 1)
  const float z = GLM ? -0.0f : 0.0f;
  const uint64_t z2 = ((uint64_t)__float_as_uint(z) << 32) | __float_as_uint(z);
#pragma unroll
  for (int i = 0; i < 4; i++) acc[i][0] = acc[i][1] = z2;
  if (router_fused_step(GLM, exact_products, tiny, blockIdx.y, (H + 31) / 32))
    router_gemm_chains<true>(acc, w32, wld, xT1, xld, H, rg_smem);
  else
    router_gemm_chains<false>(acc, w32, wld, xT1, xld, H, rg_smem);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = t0 + 4 * ty + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int e = e0 + 4 * tx + j;
      const float v = __uint_as_float((uint32_t)(acc[i][j >> 1] >> (32 * (j & 1))));
      if (e < E1) logits[(size_t)t * E1 + e] = (lbias && e < E) ? __fadd_rn(v, lbias[e]) : v;
    }
  }
}

// The wide form for many tokens and experts: a CTA computes 32 tokens x 128 experts and
// thread (tx, ty) holds tokens 4ty.. x experts {4tx.., 64 + 4tx..} = 32 chains (the two
// expert quads sit 256 bytes apart in shared memory, so a quarter-warp's 16-byte loads
// cover 128 contiguous bytes). Per step of h a thread loads 64 bytes and issues 16
// packed steps, twice the work per shared-memory byte of the 16-chain form; 16-wide h
// chunks in 4 stages keep a CTA at 48 KB so four fit on an SM. Chains, operands and the
// step arithmetic are those of router_gemm_kernel.
constexpr int kRwTokens = 32, kRwExperts = 128, kRwChunk = 16, kRwThreads = 128, kRwStages = 4;
constexpr int kRwXBytes = kRwChunk * kRwTokens * 8;
constexpr int kRwStageBytes = kRwXBytes + kRwChunk * kRwExperts * 4;

template <bool FMA>
__device__ __forceinline__ void router_wide_chains(uint64_t (&acc)[4][4], const float *w32,
                                                   int wld, const float *xT2, int xld, int H,
                                                   uint8_t *smem) {
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kRwExperts, t0 = blockIdx.y * kRwTokens;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const int nchunks = H / kRwChunk;
  auto issue = [&](int c) {
    if (c < nchunks) {
      const uint32_t st = sbase + (uint32_t)(c % kRwStages) * kRwStageBytes;
      const int h0 = c * kRwChunk;
#pragma unroll
      for (int i = 0; i < kRwChunk * 16 / kRwThreads; i++) {  // x: rows of 32 tokens x 8 bytes
        const int f = tid + kRwThreads * i, row = f >> 4, piece = f & 15;
        rg_cp16(st + row * 256 + piece * 16, xT2 + ((size_t)(h0 + row) * xld + t0) * 2 + 4 * piece);
      }
#pragma unroll
      for (int i = 0; i < kRwChunk * 32 / kRwThreads; i++) {  // w: rows of 128 experts x 4 bytes
        const int f = tid + kRwThreads * i, row = f >> 5, piece = f & 31;
        rg_cp16(st + kRwXBytes + row * 512 + piece * 16, w32 + (size_t)(h0 + row) * wld + e0 + 4 * piece);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int c = 0; c < kRwStages - 1; c++) issue(c);
  for (int c = 0; c < nchunks; c++) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kRwStages - 2) : "memory");
    __syncthreads();  // chunk c is in; every thread is done with chunk c - 1
    issue(c + kRwStages - 1);
    const uint8_t *stp = smem + (size_t)(c % kRwStages) * kRwStageBytes;
#pragma unroll
    for (int kk = 0; kk < kRwChunk; kk++) {
      const ulonglong2 xa = *reinterpret_cast<const ulonglong2 *>(stp + kk * 256 + ty * 32);
      const ulonglong2 xb = *reinterpret_cast<const ulonglong2 *>(stp + kk * 256 + ty * 32 + 16);
      const uint8_t *wrow = stp + kRwXBytes + kk * 512 + tx * 16;
      const ulonglong2 wa = *reinterpret_cast<const ulonglong2 *>(wrow);
      const ulonglong2 wb = *reinterpret_cast<const ulonglong2 *>(wrow + 256);
      const uint64_t xp[4] = {xa.x, xa.y, xb.x, xb.y};
      const uint64_t wp[4] = {wa.x, wa.y, wb.x, wb.y};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = rg_step<FMA>(wp[j], xp[i], acc[i][j]);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <bool GLM>
__global__ void __launch_bounds__(kRwThreads) router_wide_kernel(const float *w32, int wld,
                                                                 const float *xT2, int xld, int T,
                                                                 int H, int E1, const float *lbias,
                                                                 int E, float *logits,
                                                                 const uint8_t *tiny,
                                                                 int exact_products) {
  pdl_wait();
  extern __shared__ __align__(16) uint8_t rw_smem[];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kRwExperts, t0 = blockIdx.y * kRwTokens;
  uint64_t acc[4][4];  // token 4ty + i; experts (4tx + 2j, +1) for j < 2, (64 + 4tx + 2(j-2), +1)
  const float z = GLM ? -0.0f : 0.0f;
  const uint64_t z2 = ((uint64_t)__float_as_uint(z) << 32) | __float_as_uint(z);
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = z2;
  if (router_fused_step(GLM, exact_products, tiny, blockIdx.y, (H + 31) / 32))
    router_wide_chains<true>(acc, w32, wld, xT2, xld, H, rw_smem);
  else
    router_wide_chains<false>(acc, w32, wld, xT2, xld, H, rw_smem);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = t0 + 4 * ty + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int eb = e0 + (j < 2 ? 4 * tx + 2 * j : 64 + 4 * tx + 2 * (j - 2));
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const int e = eb + q;
        const float v = __uint_as_float((uint32_t)(acc[i][j] >> (32 * q)));
        if (e < E1) logits[(size_t)t * E1 + e] = (lbias && e < E) ? __fadd_rn(v, lbias[e]) : v;
      }
    }
  }
}

// The widest form (GLM prefill): a CTA of 64 threads computes 32 tokens x 128 experts and
// thread (tx, ty) holds tokens 8ty .. 8ty+7 x experts {4tx.., 64 + 4tx..} = 64 chains. The
// input comes once per value ([H][xld] f32) and is paired in registers for the packed
// steps, so a step of h loads 64 bytes for 32 packed steps: half the shared-memory bytes
// per step of router_wide_kernel, whose operand traffic bounded it (shared memory 85%
// busy). Chains, operands and the step arithmetic are those of router_gemm_kernel.
constexpr int kRxTokens = 32, kRxExperts = 128, kRxChunk = 16, kRxThreads = 64, kRxStages = 4;
constexpr int kRxXBytes = kRxChunk * kRxTokens * 4;
constexpr int kRxStageBytes = kRxXBytes + kRxChunk * kRxExperts * 4;

template <bool FMA>
__device__ __forceinline__ void router_x8_chains(uint64_t (&acc)[8][4], const float *w32, int wld,
                                                 const float *xT1, int xld, int H, uint8_t *smem) {
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kRxExperts, t0 = blockIdx.y * kRxTokens;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const int nchunks = H / kRxChunk;
  auto issue = [&](int c) {
    if (c < nchunks) {
      const uint32_t st = sbase + (uint32_t)(c % kRxStages) * kRxStageBytes;
      const int h0 = c * kRxChunk;
#pragma unroll
      for (int i = 0; i < kRxChunk * 8 / kRxThreads; i++) {  // x: rows of 32 tokens x 4 bytes
        const int f = tid + kRxThreads * i, row = f >> 3, piece = f & 7;
        rg_cp16(st + row * 128 + piece * 16, xT1 + (size_t)(h0 + row) * xld + t0 + 4 * piece);
      }
#pragma unroll
      for (int i = 0; i < kRxChunk * 32 / kRxThreads; i++) {  // w: rows of 128 experts x 4 bytes
        const int f = tid + kRxThreads * i, row = f >> 5, piece = f & 31;
        rg_cp16(st + kRxXBytes + row * 512 + piece * 16, w32 + (size_t)(h0 + row) * wld + e0 + 4 * piece);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int c = 0; c < kRxStages - 1; c++) issue(c);
  for (int c = 0; c < nchunks; c++) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kRxStages - 2) : "memory");
    __syncthreads();  // chunk c is in; every thread is done with chunk c - 1
    issue(c + kRxStages - 1);
    const uint8_t *stp = smem + (size_t)(c % kRxStages) * kRxStageBytes;
#pragma unroll
    for (int kk = 0; kk < kRxChunk; kk++) {
      const float4 xa = *reinterpret_cast<const float4 *>(stp + kk * 128 + ty * 32);
      const float4 xb = *reinterpret_cast<const float4 *>(stp + kk * 128 + ty * 32 + 16);
      const uint8_t *wrow = stp + kRxXBytes + kk * 512 + tx * 16;
      const ulonglong2 wa = *reinterpret_cast<const ulonglong2 *>(wrow);
      const ulonglong2 wb = *reinterpret_cast<const ulonglong2 *>(wrow + 256);
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      const uint64_t wp[4] = {wa.x, wa.y, wb.x, wb.y};
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint64_t xp = ((uint64_t)__float_as_uint(xv[i]) << 32) | __float_as_uint(xv[i]);
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = rg_step<FMA>(wp[j], xp, acc[i][j]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <bool GLM>
__global__ void __launch_bounds__(kRxThreads) router_x8_kernel(const float *w32, int wld,
                                                               const float *xT1, int xld, int T,
                                                               int H, int E1, const float *lbias,
                                                               int E, float *logits,
                                                               const uint8_t *tiny,
                                                               int exact_products) {
  pdl_wait();
  extern __shared__ __align__(16) uint8_t rx_smem[];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kRxExperts, t0 = blockIdx.y * kRxTokens;
  uint64_t acc[8][4];  // token 8ty + i; experts (4tx + 2j, +1) for j < 2, (64 + 4tx + 2(j-2), +1)
  const float z = GLM ? -0.0f : 0.0f;
  const uint64_t z2 = ((uint64_t)__float_as_uint(z) << 32) | __float_as_uint(z);
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = z2;
  if (router_fused_step(GLM, exact_products, tiny, blockIdx.y, (H + 31) / 32))
    router_x8_chains<true>(acc, w32, wld, xT1, xld, H, rx_smem);
  else
    router_x8_chains<false>(acc, w32, wld, xT1, xld, H, rx_smem);
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int t = t0 + 8 * ty + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int eb = e0 + (j < 2 ? 4 * tx + 2 * j : 64 + 4 * tx + 2 * (j - 2));
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const int e = eb + q;
        const float v = __uint_as_float((uint32_t)(acc[i][j] >> (32 * q)));
        if (e < E1) logits[(size_t)t * E1 + e] = (lbias && e < E) ? __fadd_rn(v, lbias[e]) : v;
      }
    }
  }
}

// x [T][H] (f32 or bf16) -> xT2 [H][xld][2] f32, each value twice; tokens T..xld-1 zero.
// With `tiny`, block (bx, by) also writes tiny[by * gridDim.x + bx]: whether its 32x32 tile
// holds a nonzero |x| outside [2^-60, 2^60) (see the router's step arithmetic).
__global__ void __launch_bounds__(256) transpose_x_kernel(const void *x, int bf16, int T, int H,
                                                         int xld, float *xT2, uint8_t *tiny,
                                                         int single) {
  pdl_wait();
  __shared__ float tile[32][33];
  const int h0 = blockIdx.x * 32, t0 = blockIdx.y * 32;
  const int c = threadIdx.x & 31, r0 = threadIdx.x >> 5;
  bool bad = false;
  for (int r = r0; r < 32; r += 8) {
    const int t = t0 + r, h = h0 + c;
    float v = 0.0f;
    if (t < T && h < H) v = load_as_f32(x, (size_t)t * H + h, bf16 != 0);
    bad |= outside_exact_range(v);
    tile[r][c] = v;
  }
  const int any = __syncthreads_or(bad);  // also the barrier before the tile is read
  if (tiny && threadIdx.x == 0) tiny[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = any ? 1 : 0;
  for (int r = r0; r < 32; r += 8) {
    const int h = h0 + r, t = t0 + c;
    const float v = tile[c][r];
    if (h < H && t < xld) {
      if (single) xT2[(size_t)h * xld + t] = v;
      else reinterpret_cast<float2 *>(xT2)[(size_t)h * xld + t] = make_float2(v, v);
    }
  }
}

// router [H][ld] (f32 or bf16) -> [H][dld] f32 (zero past ld)
__global__ void pad_router_kernel(const void *src, int bf16, int H, int ld, int dld, float *dst) {
  const size_t n = (size_t)H * dld;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int h = (int)(idx / dld), e = (int)(idx % dld);
    dst[idx] = e < ld ? load_as_f32(src, (size_t)h * ld + e, bf16 != 0) : 0.0f;
  }
}

int launch_dup_router(const void *router_t, int bf16, int H, int E1, float *dst,
                      cudaStream_t stream) {
  const int dld = router_dup_ld(E1);
  const size_t n = (size_t)H * dld;
  pad_router_kernel<<<(int)std::min<size_t>((n + 255) / 256, 4096), 256, 0, stream>>>(
      router_t, bf16, H, router_ld(E1), dld, dst);
  return 1;
}

// ---------------------------------------------------------------------------
// top-k: one warp per token
// ---------------------------------------------------------------------------

constexpr int kTopkWarps = 4;
constexpr int kMaxGlmExperts = 1024;

// softmax family: src/cpu.rs:234-260 (+ softmax_in_place :196-231). With REG the
// token's logits (E <= 1024) stay in registers across the k selection rounds.
template <bool REG>
__global__ void __launch_bounds__(32 * kTopkWarps) topk_softmax_kernel(
    const float *logits, int T, int E1, int E, int k, uint32_t *sel_idx, float *sel_w,
    int32_t *status) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kTopkWarps + warp;
  if (t >= T) return;
  const float *lg = logits + (size_t)t * E1;
  constexpr int kPer = REG ? 32 : 1;
  float v[kPer];
  bool bad = false;
  if (REG) {
#pragma unroll
    for (int j = 0; j < kPer; j++) {
      int e = lane + 32 * j;
      v[j] = e < E ? lg[e] : 0.0f;
      bad |= e < E && !isfinite(v[j]);
    }
  } else {
    for (int e = lane; e < E; e += 32) bad |= !isfinite(lg[e]);
  }
  if (__any_sync(0xffffffffu, bad)) {
    // flag the error and leave an in-range selection so later kernels stay in bounds
    if (lane == 0) atomicExch(status, kStatusNonFiniteRouter);
    for (int r = lane; r < k; r += 32) {
      sel_idx[(size_t)t * k + r] = (uint32_t)r;
      sel_w[(size_t)t * k + r] = 0.0f;
    }
    return;
  }
  unsigned long long last = ~0ull;
  float vals[32];
  uint32_t idxs[32];
  for (int r = 0; r < k; r++) {
    unsigned long long best = 0;
    if (REG) {
#pragma unroll
      for (int j = 0; j < kPer; j++) {
        int e = lane + 32 * j;
        unsigned long long key = e < E ? rank_key(v[j], (uint32_t)e) : 0ull;
        if (key < last && key > best) best = key;
      }
    } else {
      for (int e = lane; e < E; e += 32) {
        unsigned long long key = rank_key(lg[e], (uint32_t)e);
        if (key < last && key > best) best = key;
      }
    }
    best = warp_max_u64(best);
    last = best;
    uint32_t idx = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
    if (idx >= (uint32_t)E) idx = 0;  // unreachable for k <= E; keeps reads in range
    if (r < 32) {
      idxs[r] = idx;
      vals[r] = __uint_as_float((uint32_t)(best >> 32) ^ 0x80000000u);
    }
  }
  if (lane == 0) {
    // undo rank_key's order-preserving map to recover the selected logits exactly
    for (int r = 0; r < k; r++) {
      int32_t key = __float_as_int(vals[r]);
      vals[r] = __int_as_float(key ^ (int32_t)(((uint32_t)(key >> 31)) >> 1));
    }
    float maximum = -INFINITY, sum = 0.0f;
    for (int r = 0; r < k; r++) maximum = fmaxf(maximum, vals[r]);
    for (int r = 0; r < k; r++) {
      vals[r] = exp_f32_cr(__fsub_rn(vals[r], maximum));
      sum = __fadd_rn(sum, vals[r]);
    }
    for (int r = 0; r < k; r++) {
      sel_idx[(size_t)t * k + r] = idxs[r];
      sel_w[(size_t)t * k + r] = __fdiv_rn(vals[r], sum);
    }
  }
}

// softmax family for the forward (E <= 1023): one CTA per token, one thread per logit.
// Two-level rank selection: each thread ranks its key within its warp (shuffles), each
// warp's k best become candidates, and every candidate's rank among all candidates is
// its selection position (keys are unique: value, then lower index). Then the
// reference's softmax over the k winners (src/cpu.rs:196-231: max, exp, sequential sum
// in selection order, divide).
__global__ void __launch_bounds__(1024) topk_rank_softmax_kernel(const float *logits, int T, int E1,
                                                                int E, int k, uint32_t *sel_idx,
                                                                float *sel_w, int32_t *status) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(16) unsigned long long cand[32 * 32];
  __shared__ unsigned long long chosen[32];
  __shared__ int bad_s;
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  if (tid == 0) bad_s = 0;
  __syncthreads();
  const float v = tid < E ? logits[(size_t)t * E1 + tid] : 0.0f;
  if (tid < E && !isfinite(v)) bad_s = 1;
  const unsigned long long key = tid < E ? rank_key(v, (uint32_t)tid) : 0ull;
  int wr = 0;
#pragma unroll
  for (int j = 0; j < 32; j++) wr += __shfl_sync(0xffffffffu, key, j) > key ? 1 : 0;
  // Lanes past E hold key 0 and tie, so they all land on one slot: clear the warp's k
  // slots first. A zero key loses to every finite logit, and with at least k valid
  // candidates the zeros never reach the top k.
  if (lane < k) cand[warp * k + lane] = 0ull;
  __syncwarp();
  if (wr < k) cand[warp * k + wr] = key;
  __syncthreads();
  if (bad_s) {
    // flag the error and leave an in-range selection so later kernels stay in bounds
    if (tid == 0) atomicExch(status, kStatusNonFiniteRouter);
    if (tid < k) {
      sel_idx[(size_t)t * k + tid] = (uint32_t)tid;
      sel_w[(size_t)t * k + tid] = 0.0f;
    }
    return;
  }
  const int C = nwarps * k;
  const ulonglong2 *cand2 = reinterpret_cast<const ulonglong2 *>(cand);
  for (int c = tid; c < C; c += blockDim.x) {
    const unsigned long long mine = cand[c];
    int r = (C & 1) && cand[C - 1] > mine ? 1 : 0;
#pragma unroll 8
    for (int j = 0; j < C / 2; j++) {  // two keys per 16-byte load, loads pipelined
      const ulonglong2 q = cand2[j];
      r += (q.x > mine ? 1 : 0) + (q.y > mine ? 1 : 0);
    }
    if (r < k) chosen[r] = mine;
  }
  __syncthreads();
  if (warp == 0) {
    float val = -INFINITY;
    uint32_t idx = 0;
    if (lane < k) {
      const unsigned long long best = chosen[lane];
      idx = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
      const int32_t kb = (int32_t)((uint32_t)(best >> 32) ^ 0x80000000u);
      val = __int_as_float(kb ^ (int32_t)(((uint32_t)(kb >> 31)) >> 1));
    }
    float m = val;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float ex = lane < k ? exp_f32_cr(__fsub_rn(val, m)) : 0.0f;
    float sum = 0.0f;
    for (int r = 0; r < k; r++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, r));
    if (lane < k) {
      sel_idx[(size_t)t * k + lane] = idx;
      sel_w[(size_t)t * k + lane] = __fdiv_rn(ex, sum);
    }
  }
}

int launch_topk_softmax(const float *logits, int n, int k, uint32_t *idx, float *prob,
                        int32_t *status, cudaStream_t stream) {
  if (n <= 1024)
    topk_softmax_kernel<true><<<1, 32 * kTopkWarps, 0, stream>>>(logits, 1, n, n, k, idx, prob, status);
  else
    topk_softmax_kernel<false><<<1, 32 * kTopkWarps, 0, stream>>>(logits, 1, n, n, k, idx, prob, status);
  return 1;
}

// ---------------------------------------------------------------------------
// dispatch: one CTA, stable counting sort of the T*k pairs by expert
// ---------------------------------------------------------------------------

constexpr int kDispatchThreads = 1024, kDispatchWarps = kDispatchThreads / 32;

__device__ __forceinline__ int warp_inclusive_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Exclusive scans of three values over all threads of a kDispatchThreads block;
// also returns the three totals to every thread.
__device__ __forceinline__ void block_exclusive_scan3(int &a, int &b, int &c, int &ta, int &tb,
                                                      int &tc) {
  __shared__ int ws[3][kDispatchWarps];
  __shared__ int tot[3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ia = warp_inclusive_scan(a), ib = warp_inclusive_scan(b), ic = warp_inclusive_scan(c);
  if (lane == 31) {
    ws[0][warp] = ia;
    ws[1][warp] = ib;
    ws[2][warp] = ic;
  }
  __syncthreads();
  if (warp == 0) {
    const int x = ws[0][lane], y = ws[1][lane], z = ws[2][lane];
    const int sx = warp_inclusive_scan(x), sy = warp_inclusive_scan(y), sz = warp_inclusive_scan(z);
    ws[0][lane] = sx - x;
    ws[1][lane] = sy - y;
    ws[2][lane] = sz - z;
    if (lane == 31) {
      tot[0] = sx;
      tot[1] = sy;
      tot[2] = sz;
    }
  }
  __syncthreads();
  a = ws[0][warp] + ia - a;
  b = ws[1][warp] + ib - b;
  c = ws[2][warp] + ic - c;
  ta = tot[0];
  tb = tot[1];
  tc = tot[2];
  __syncthreads();
}

// Rows mode (expert-parallel rows): sel_idx holds explicit expert ids where id E is the
// shared expert, so E + 1 buckets are counted and no shared pairs are added.
__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(ForwardArgs a) {
  pdl_wait();
  extern __shared__ int32_t sm[];
  const int E = a.E, P = a.T * a.k;
  const int EB = E + (a.rows_mode ? 1 : 0);      // buckets counted from sel_idx
  int32_t *wc = sm;                              // [warps][EB]
  int32_t *total = sm + kDispatchWarps * (E + 1);  // [E + 1]
  int32_t *flags = total + (E + 1);              // [E + 1] scan scratch
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // contiguous chunks of whole warps' worth of pairs: few pairs use few warps
  const int chunk = max(32, (((P + kDispatchWarps - 1) / kDispatchWarps) + 31) & ~31);
  const int nw = (P + chunk - 1) / chunk;
  for (int i = threadIdx.x; i < nw * EB; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  const int begin = min(P, warp * chunk), end = min(P, begin + chunk);
  for (int p = begin + lane; p < end; p += 32) {
    uint32_t e = a.sel_idx[p];
    if (e < (uint32_t)EB) atomicAdd(&wc[warp * EB + e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < EB; e += blockDim.x) {
    int running = 0;
    for (int w = 0; w < nw; w++) {
      int c = wc[w * EB + e];
      wc[w * EB + e] = running;
      running += c;
    }
    total[e] = running;
  }
  __syncthreads();
  // Block-wide exclusive scans over the experts (one thread per expert, the shared
  // expert as index E): token offsets, the compacted active list and the work list
  // of (expert, first token, position, tokens) chunks of `a.chunk` tokens.
  {
    const int e = threadIdx.x;  // E + 1 <= kDispatchThreads
    const int count = e < EB ? total[e] : (e == E && a.shared ? a.T : 0);
    const int items = (count + a.chunk - 1) / a.chunk;
    int s_count = count, s_active = count > 0, s_items = items;
    int tot_count, tot_active, tot_items;
    block_exclusive_scan3(s_count, s_active, s_items, tot_count, tot_active, tot_items);
    if (e <= E) {
      a.counts[e] = count;
      a.offsets[e] = s_count;
      if (e < EB) flags[e] = s_count;
      if (count > 0) a.active[s_active] = e;
      if (a.balanced_items && items > 1) {
        // items of base or base + 1 tokens, the larger ones first
        const int base = count / items, rem = count - base * items;
        for (int j = 0; j < items; j++) {
          const int first = j * base + min(j, rem);
          a.items[s_items + j] = make_int4(e, first, s_count + first, base + (j < rem ? 1 : 0));
        }
      } else {
        for (int j = 0; j < items; j++)
          a.items[s_items + j] = make_int4(e, j * a.chunk, s_count + j * a.chunk,
                                           min(a.chunk, count - j * a.chunk));
      }
    }
    if (e == 0) {
      a.offsets[E + 1] = tot_count;
      *a.n_active = tot_active;
      *a.n_items = tot_items;
    }
  }
  __syncthreads();
  for (int base = begin; base < end; base += 32) {
    int p = base + lane;
    bool valid = p < end;
    unsigned vmask = __ballot_sync(0xffffffffu, valid);
    if (valid && a.drop_invalid && a.sel_idx[p] >= (uint32_t)EB) {
      a.inverse[p] = -1;  // a slot this rank does not run
      valid = false;
    }
    vmask = __ballot_sync(0xffffffffu, valid);
    if (valid) {
      uint32_t e = a.sel_idx[p];
      if (e >= (uint32_t)EB) e = 0;  // rejected upstream; keep indices in range
      unsigned peers = __match_any_sync(vmask, e);
      int rank = __popc(peers & ((1u << lane) - 1u));
      int pos = flags[e] + wc[warp * EB + e] + rank;
      a.sorted[pos] = p;
      a.inverse[p] = pos;
      __syncwarp(vmask);
      if (rank == 0) wc[warp * EB + e] += __popc(peers);
    }
    __syncwarp();
  }
  if (a.shared) {
    for (int t = threadIdx.x; t < a.T; t += blockDim.x) {
      a.sorted[P + t] = P + t;
      a.inverse[P + t] = P + t;
    }
  }
}

// ---------------------------------------------------------------------------
// expert products (CUDA cores): a warp owns a row, lanes split its 32-element
// units, each unit is dequantised once into registers and applied to a chunk of
// up to TT tokens staged in shared memory ([TT][units][36] floats, padded so the
// float4 reads of 32 lanes hit distinct banks).
// ---------------------------------------------------------------------------

constexpr int kExpertThreads = 256, kExpertWarps = kExpertThreads / 32, kUnitStride = 36;

__device__ __forceinline__ int pair_token(const ForwardArgs &a, int pair) {
  int P = a.T * a.k;
  return pair < P ? pair / a.k : pair - P;
}

__device__ __forceinline__ float expert_input(const ForwardArgs &a, int token, int col) {
  size_t o = (size_t)token * a.H + col;
  if (a.family == kGemma) return a.expert_in[o];
  return load_as_f32(a.x, o, a.input_bf16);
}

__device__ __forceinline__ float activate(const ForwardArgs &a, int expert, float g, float u) {
  if (a.family == kGemma) return __fmul_rn(gelu_tanh(g), u);
  if (a.family == kQwen) return __fmul_rn(qwen_silu(g), u);
  if (expert == a.E) return __fmul_rn(glm_silu(g), u);  // GLM shared `mlp`
  return __fmul_rn(glm_cached_silu(g), u);               // GLM routed experts
}

template <int TT>
__device__ __forceinline__ void unit_dot(const float *w, const float *xs, int units, int u,
                                         int nt, float *acc) {
#pragma unroll
  for (int t = 0; t < TT; t++) {
    if (t < nt) {
      const float4 *xv = reinterpret_cast<const float4 *>(xs + ((size_t)t * units + u) * kUnitStride);
      float s = acc[t];
#pragma unroll
      for (int v = 0; v < 8; v++) {
        float4 q = xv[v];
        s = fmaf(w[4 * v], q.x, s);
        s = fmaf(w[4 * v + 1], q.y, s);
        s = fmaf(w[4 * v + 2], q.z, s);
        s = fmaf(w[4 * v + 3], q.w, s);
      }
      acc[t] = s;
    }
  }
}

template <class U, int TT>
__global__ void __launch_bounds__(kExpertThreads) expert_up_kernel(ForwardArgs a,
                                                                  int rows_per_cta) {
  pdl_wait();
  extern __shared__ __align__(16) float xs[];
  const int slot = blockIdx.y;
  if (slot >= *a.n_active) return;
  const int e = a.active[slot];
  const int n = a.counts[e], base = a.offsets[e];
  const int I = a.I, H = a.H, units = H / 32;
  const int row0 = blockIdx.x * rows_per_cta;
  if (row0 >= I) return;
  const uint64_t rb = row_bytes(a.gate_type, H);
  const uint8_t *G = e < a.E ? a.gate + (size_t)e * a.gate_stride : a.sh_gate;
  const uint8_t *Up = e < a.E ? a.up + (size_t)e * a.up_stride : a.sh_up;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c0 = 0; c0 < n; c0 += TT) {
    const int nt = min(TT, n - c0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < nt * H; idx += blockDim.x) {
      int tt = idx / H, col = idx - tt * H;
      int tok = pair_token(a, a.sorted[base + c0 + tt]);
      xs[((size_t)tt * units + (col >> 5)) * kUnitStride + (col & 31)] = expert_input(a, tok, col);
    }
    __syncthreads();
    for (int r = warp; r < rows_per_cta; r += kExpertWarps) {
      const int i = row0 + r;
      if (i >= I) break;
      float ag[TT], au[TT];
#pragma unroll
      for (int t = 0; t < TT; t++) ag[t] = au[t] = 0.0f;
      const uint8_t *grow = G + (size_t)i * rb, *urow = Up + (size_t)i * rb;
      for (int u = lane; u < units; u += 32) {
        float w[32];
        U::decode(grow, u, w);
        unit_dot<TT>(w, xs, units, u, nt, ag);
        U::decode(urow, u, w);
        unit_dot<TT>(w, xs, units, u, nt, au);
      }
#pragma unroll
      for (int t = 0; t < TT; t++) {
        ag[t] = warp_sum(ag[t]);
        au[t] = warp_sum(au[t]);
      }
      if (lane == 0) {
        for (int t = 0; t < nt; t++)
          a.h[(size_t)(base + c0 + t) * I + i] = activate(a, e, ag[t], au[t]);
      }
    }
  }
}

template <class U, int TT>
__global__ void __launch_bounds__(kExpertThreads) expert_down_kernel(ForwardArgs a,
                                                                    int rows_per_cta) {
  pdl_wait();
  extern __shared__ __align__(16) float xs[];
  const int slot = blockIdx.y;
  if (slot >= *a.n_active) return;
  const int e = a.active[slot];
  const int n = a.counts[e], base = a.offsets[e];
  const int I = a.I, H = a.H, units = I / 32;
  const int row0 = blockIdx.x * rows_per_cta;
  if (row0 >= H) return;
  const uint64_t rb = row_bytes(a.down_type, I);
  const uint8_t *D = e < a.E ? a.down + (size_t)e * a.down_stride : a.sh_down;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c0 = 0; c0 < n; c0 += TT) {
    const int nt = min(TT, n - c0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < nt * I; idx += blockDim.x) {
      int tt = idx / I, col = idx - tt * I;
      xs[((size_t)tt * units + (col >> 5)) * kUnitStride + (col & 31)] =
          a.h[(size_t)(base + c0 + tt) * I + col];
    }
    __syncthreads();
    for (int r = warp; r < rows_per_cta; r += kExpertWarps) {
      const int row = row0 + r;
      if (row >= H) break;
      float acc[TT];
#pragma unroll
      for (int t = 0; t < TT; t++) acc[t] = 0.0f;
      const uint8_t *drow = D + (size_t)row * rb;
      for (int u = lane; u < units; u += 32) {
        float w[32];
        U::decode(drow, u, w);
        unit_dot<TT>(w, xs, units, u, nt, acc);
      }
#pragma unroll
      for (int t = 0; t < TT; t++) acc[t] = warp_sum(acc[t]);
      if (lane == 0) {
        for (int t = 0; t < nt; t++) a.ysorted[(size_t)(base + c0 + t) * H + row] = acc[t];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// weighted combine: selection order, deterministic, no atomics
// ---------------------------------------------------------------------------

constexpr int kCombineThreads = 64;

__global__ void __launch_bounds__(kCombineThreads) combine_kernel(ForwardArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ int pos_s[32];
  __shared__ float w_s[32];
  __shared__ float gate_s;
  const int t = blockIdx.x;
  const int H = a.H, k = a.k, P = a.T * a.k;
  if (threadIdx.x < k) {
    const int p = t * k + threadIdx.x;
    pos_s[threadIdx.x] = a.inverse[p];
    float w = a.sel_w[p];
    if (a.family == kGemma) w = __fmul_rn(w, a.expert_scale[a.sel_idx[p]]);  // p * scale[e]
    w_s[threadIdx.x] = w;
  }
  if (threadIdx.x == 32)
    gate_s = a.shared && a.family == kQwen ? qwen_sigmoid(a.logits[(size_t)t * a.E1 + a.E]) : 0.0f;
  __syncthreads();
  const float gate = gate_s;
  const int i4 = blockIdx.y * blockDim.x + threadIdx.x;
  if (i4 < H / 4) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    // selection order; the rows of up to 8 pairs are loaded before they are added
    for (int j0 = 0; j0 < k; j0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j0 + j < k)
          v[j] = *reinterpret_cast<const float4 *>(a.ysorted + (size_t)pos_s[j0 + j] * H + 4 * i4);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (j0 + j < k) {
          const float vv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
          const float w = w_s[j0 + j];
#pragma unroll
          for (int c = 0; c < 4; c++) {
            if (a.family == kGlm)
              acc[c] = __fadd_rn(acc[c], __fmul_rn(__fmul_rn(vv[c], w), a.routed_scale));
            else
              acc[c] = __fmaf_rn(vv[c], w, acc[c]);
          }
        }
      }
    }
    if (a.shared) {
      const float4 v = *reinterpret_cast<const float4 *>(a.ysorted + (size_t)(P + t) * H + 4 * i4);
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; c++)
        acc[c] = a.family == kQwen ? __fmaf_rn(vv[c], gate, acc[c]) : __fadd_rn(acc[c], vv[c]);
    }
    *reinterpret_cast<float4 *>(a.y + (size_t)t * H + 4 * i4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
}

// ---------------------------------------------------------------------------
// forward orchestration
// ---------------------------------------------------------------------------

template <template <class, int> class K, int TT>
static void *pick_kernel(int kind) {
  switch (kind) {
    case DM_Q4_K: return (void *)K<Q4KUnit, TT>::fn();
    case DM_Q6_K: return (void *)K<Q6KUnit, TT>::fn();
    case DM_Q5_0: return (void *)K<Q50Unit, TT>::fn();
    case DM_Q8_0: return (void *)K<Q80Unit, TT>::fn();
    case DM_BF16: return (void *)K<BF16Unit, TT>::fn();
    case DM_F16: return (void *)K<F16Unit, TT>::fn();
    case DM_F32: return (void *)K<F32Unit, TT>::fn();
    default: return nullptr;
  }
}

template <class U, int TT>
struct UpK {
  static decltype(&expert_up_kernel<U, TT>) fn() { return &expert_up_kernel<U, TT>; }
};
template <class U, int TT>
struct DownK {
  static decltype(&expert_down_kernel<U, TT>) fn() { return &expert_down_kernel<U, TT>; }
};

typedef void (*ExpertFn)(ForwardArgs, int);

static int choose_tt(int columns) {
  size_t per_token = (size_t)(columns / 32) * kUnitStride * sizeof(float);
  return per_token * 8 <= 112 * 1024 ? 8 : 4;
}

static ExpertFn expert_fn(bool up, int kind, int tt) {
  if (up) return (ExpertFn)(tt == 8 ? pick_kernel<UpK, 8>(kind) : pick_kernel<UpK, 4>(kind));
  return (ExpertFn)(tt == 8 ? pick_kernel<DownK, 8>(kind) : pick_kernel<DownK, 4>(kind));
}

// The same dispatch for at most kSmallPairs pairs (decode) in one CTA with a thread per
// bucket: counts in shared memory, one block-wide exclusive scan over the E + 1 buckets
// for the offsets, the active list and the work items, and each pair's position from
// the pairs before it with the same expert (stable: expert, then pair index).
constexpr int kSmallPairs = 64;

struct SmallDispatchSmem {
  int32_t cnt[1024];        // bucket counts, then first positions
  uint32_t sel[kSmallPairs];
  int32_t wsum[3][32];      // per-warp totals of counts, active buckets, items
};

// The dispatch of the pairs in sm.sel (already in range, P = T*k of them).
__device__ __forceinline__ void dispatch_small_body(const ForwardArgs &a, SmallDispatchSmem &sm) {
  const int E = a.E, P = a.T * a.k, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int32_t *cnt = sm.cnt;
  if (tid <= E) cnt[tid] = 0;
  __syncthreads();
  if (tid < P) atomicAdd(&cnt[sm.sel[tid]], 1);
  __syncthreads();
  if (a.shared && tid == 0) cnt[E] = a.T;
  __syncthreads();
  // one thread per bucket: a block-wide exclusive scan of counts, active flags and items
  const int e = tid;
  const int c = e <= E ? cnt[e] : 0;
  const int items = (c + a.chunk - 1) / a.chunk;
  int c_inc = c, a_inc = c > 0, i_inc = items;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int cc = __shfl_up_sync(0xffffffffu, c_inc, o);
    const int ac = __shfl_up_sync(0xffffffffu, a_inc, o);
    const int ic = __shfl_up_sync(0xffffffffu, i_inc, o);
    if (lane >= o) c_inc += cc, a_inc += ac, i_inc += ic;
  }
  if (lane == 31) sm.wsum[0][warp] = c_inc, sm.wsum[1][warp] = a_inc, sm.wsum[2][warp] = i_inc;
  __syncthreads();
  if (warp == 0) {
    const int nw = (int)(blockDim.x >> 5);
    int x0 = lane < nw ? sm.wsum[0][lane] : 0, x1 = lane < nw ? sm.wsum[1][lane] : 0,
        x2 = lane < nw ? sm.wsum[2][lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y0 = __shfl_up_sync(0xffffffffu, x0, o), y1 = __shfl_up_sync(0xffffffffu, x1, o),
                y2 = __shfl_up_sync(0xffffffffu, x2, o);
      if (lane >= o) x0 += y0, x1 += y1, x2 += y2;
    }
    if (lane < nw) sm.wsum[0][lane] = x0, sm.wsum[1][lane] = x1, sm.wsum[2][lane] = x2;  // inclusive
  }
  __syncthreads();
  const int wb0 = warp ? sm.wsum[0][warp - 1] : 0, wb1 = warp ? sm.wsum[1][warp - 1] : 0,
            wb2 = warp ? sm.wsum[2][warp - 1] : 0;
  const int c_off = wb0 + c_inc - c, a_off = wb1 + a_inc - (c > 0), i_off = wb2 + i_inc - items;
  __syncthreads();  // every count is read before it becomes a position
  if (e <= E) {
    a.counts[e] = c;
    a.offsets[e] = c_off;
    if (c > 0) a.active[a_off] = e;
    for (int j = 0; j < items; j++)
      a.items[i_off + j] = make_int4(e, j * a.chunk, c_off + j * a.chunk, min(a.chunk, c - j * a.chunk));
    cnt[e] = c_off;  // becomes the bucket's first position
  }
  if (tid == (int)blockDim.x - 1) {
    a.offsets[E + 1] = sm.wsum[0][(blockDim.x >> 5) - 1];
    *a.n_active = sm.wsum[1][(blockDim.x >> 5) - 1];
    *a.n_items = sm.wsum[2][(blockDim.x >> 5) - 1];
  }
  __syncthreads();
  // pair p goes after the earlier pairs of its bucket (stable order)
  if (tid < P) {
    const uint32_t ep = sm.sel[tid];
    int before = 0;
    for (int q = 0; q < tid; q++) before += sm.sel[q] == ep;
    const int pos = cnt[ep] + before;
    a.sorted[pos] = tid;
    a.inverse[tid] = pos;
  }
  if (a.shared)
    for (int t = tid; t < a.T; t += blockDim.x) {
      a.sorted[P + t] = P + t;
      a.inverse[P + t] = P + t;
    }
}

__global__ void __launch_bounds__(1024) dispatch_small_kernel(ForwardArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ SmallDispatchSmem sm;
  const int EB = a.E + (a.rows_mode ? 1 : 0);
  if ((int)threadIdx.x < a.T * a.k) {
    uint32_t e = a.sel_idx[threadIdx.x];
    if (e >= (uint32_t)EB) e = 0;  // rejected upstream; keep indices in range
    sm.sel[threadIdx.x] = e;
  }
  dispatch_small_body(a, sm);
}

// One decode token (T = 1) of the softmax families: the rank top-k of
// topk_rank_softmax_kernel, then the small dispatch of its k pairs, in one CTA.
__global__ void __launch_bounds__(1024) topk_dispatch1_kernel(ForwardArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ SmallDispatchSmem sm;
  __shared__ __align__(16) unsigned long long cand[32 * 32];
  __shared__ unsigned long long chosen[32];
  __shared__ int bad_s;
  const int E = a.E, k = a.k, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  if (tid == 0) bad_s = 0;
  __syncthreads();
  const float v = tid < E ? a.logits[tid] : 0.0f;
  if (tid < E && !isfinite(v)) bad_s = 1;
  const unsigned long long key = tid < E ? rank_key(v, (uint32_t)tid) : 0ull;
  int wr = 0;
#pragma unroll
  for (int j = 0; j < 32; j++) wr += __shfl_sync(0xffffffffu, key, j) > key ? 1 : 0;
  // Lanes past E hold key 0 and tie, so they all land on one slot: clear the warp's k
  // slots first. A zero key loses to every finite logit, and with at least k valid
  // candidates the zeros never reach the top k.
  if (lane < k) cand[warp * k + lane] = 0ull;
  __syncwarp();
  if (wr < k) cand[warp * k + wr] = key;
  __syncthreads();
  if (bad_s) {
    // flag the error and dispatch an in-range selection so later kernels stay in bounds
    if (tid == 0) atomicExch(a.status, kStatusNonFiniteRouter);
    if (tid < k) {
      a.sel_idx[tid] = (uint32_t)tid;
      a.sel_w[tid] = 0.0f;
      sm.sel[tid] = (uint32_t)tid;
    }
  } else {
    const int C = nwarps * k;
    const ulonglong2 *cand2 = reinterpret_cast<const ulonglong2 *>(cand);
    for (int c = tid; c < C; c += blockDim.x) {
      const unsigned long long mine = cand[c];
      int r = (C & 1) && cand[C - 1] > mine ? 1 : 0;
#pragma unroll 8
      for (int j = 0; j < C / 2; j++) {  // two keys per 16-byte load, loads pipelined
        const ulonglong2 q = cand2[j];
        r += (q.x > mine ? 1 : 0) + (q.y > mine ? 1 : 0);
      }
      if (r < k) chosen[r] = mine;
    }
    __syncthreads();
    if (warp == 0) {
      float val = -INFINITY;
      uint32_t idx = 0;
      if (lane < k) {
        const unsigned long long best = chosen[lane];
        idx = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
        const int32_t kb = (int32_t)((uint32_t)(best >> 32) ^ 0x80000000u);
        val = __int_as_float(kb ^ (int32_t)(((uint32_t)(kb >> 31)) >> 1));
      }
      float m = val;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float ex = lane < k ? exp_f32_cr(__fsub_rn(val, m)) : 0.0f;
      float sum = 0.0f;
      for (int r = 0; r < k; r++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, r));
      if (lane < k) {
        a.sel_idx[lane] = idx;
        a.sel_w[lane] = __fdiv_rn(ex, sum);
        sm.sel[lane] = idx < (uint32_t)E ? idx : 0u;  // the dispatch indexes by it
      }
    }
  }
  __syncthreads();
  dispatch_small_body(a, sm);
}

// Per-row outputs of the rows mode: out[r] = ysorted[inverse[r]] (k = 1, unweighted).
__global__ void __launch_bounds__(128) scatter_rows_kernel(ForwardArgs a) {
  pdl_wait();
  const int r = blockIdx.x, i4 = blockIdx.y * blockDim.x + threadIdx.x;
  if (i4 >= a.H / 4) return;
  const float4 v = *reinterpret_cast<const float4 *>(a.ysorted + (size_t)a.inverse[r] * a.H + 4 * i4);
  *reinterpret_cast<float4 *>(a.y + (size_t)r * a.H + 4 * i4) = v;
}

// the identity position map used when pair outputs arrive already in pair order
__global__ void iota_kernel(int32_t *v, int n) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) v[i] = i;
}

// GLM routing with one token per CTA and a thread per expert: sigmoid + correction
// choices computed once (src/glm52/cpu.rs:731-754), group scores (top1 + top2 of the
// group's choices, the topk_groups best groups kept; restated), then each eligible
// expert's rank among the eligible ones by key (choice descending, index ascending) --
// the selection and order of repeated argmax -- and the weights normalised by their sum
// in selection order. FUSED (one token): the small dispatch follows in the same CTA.
template <bool FUSED>
__global__ void __launch_bounds__(1024) topk_sigmoid_rank_kernel(ForwardArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long key_s[kMaxGlmExperts];
  __shared__ unsigned long long cmp_s[kMaxGlmExperts];
  __shared__ float w_s[kMaxGlmExperts];
  __shared__ float c_s[kMaxGlmExperts];
  __shared__ unsigned long long gkey_s[32];
  __shared__ unsigned char keep_s[32];
  __shared__ uint32_t idx_s[32];
  __shared__ float selw_s[32];
  __shared__ float sum_s;
  __shared__ int bad_s;
  __shared__ SmallDispatchSmem sm;
  const int t = blockIdx.x, tid = threadIdx.x, E = a.E, k = a.k;
  const float *lg = a.logits + (size_t)t * a.E1;
  if (tid == 0) bad_s = 0;
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const float w = glm_sigmoid(lg[e]);
    const float c = __fadd_rn(w, a.bias[e]);
    if (!isfinite(w) || !isfinite(c)) bad_s = 1;
    w_s[e] = w;
    c_s[e] = c;
    key_s[e] = rank_key(c, (uint32_t)e);
  }
  __syncthreads();
  if (bad_s) {
    // flag the error and leave an in-range selection so later kernels stay in bounds
    if (tid == 0) atomicExch(a.status, kStatusNonFiniteRouter);
    if (tid < k) {
      a.sel_idx[(size_t)t * k + tid] = (uint32_t)tid;
      a.sel_w[(size_t)t * k + tid] = 0.0f;
      if (FUSED) sm.sel[tid] = (uint32_t)tid;
    }
  } else {
    const int ng = a.n_groups > 1 ? a.n_groups : 1, pg = E / ng;
    if (ng > 1) {
      if (tid < ng) {
        unsigned long long k1 = 0, k2 = 0;
        for (int i = 0; i < pg; i++) {
          const unsigned long long key = key_s[tid * pg + i];
          if (key > k1) {
            k2 = k1;
            k1 = key;
          } else if (key > k2) {
            k2 = key;
          }
        }
        const float c1 = c_s[0xffffffffu - (uint32_t)(k1 & 0xffffffffu)];
        const float c2 = c_s[0xffffffffu - (uint32_t)(k2 & 0xffffffffu)];
        gkey_s[tid] = rank_key(__fadd_rn(c1, c2), (uint32_t)tid);
      }
      __syncthreads();
      if (tid < ng) {
        int rank = 0;
        for (int g = 0; g < ng; g++) rank += gkey_s[g] > gkey_s[tid];
        keep_s[tid] = rank < a.topk_groups;
      }
      __syncthreads();
    }
    // the eligible experts' keys, compacted (kept groups in order) into cmp_s
    int n_elig = E;
    if (ng > 1) {
      int kept_before = 0, kept = 0;
      for (int g = 0; g < ng; g++) kept += keep_s[g];
      n_elig = kept * pg;
      for (int e = tid; e < E; e += blockDim.x) {
        const int g = e / pg;
        if (!keep_s[g]) continue;
        kept_before = 0;
        for (int h = 0; h < g; h++) kept_before += keep_s[h];
        cmp_s[kept_before * pg + (e - g * pg)] = key_s[e];
      }
    } else {
      for (int e = tid; e < E; e += blockDim.x) cmp_s[e] = key_s[e];
    }
    __syncthreads();
    for (int i = tid; i < n_elig; i += blockDim.x) {
      const unsigned long long key = cmp_s[i];
      int r = 0;
      for (int j = 0; j < n_elig; j++) r += cmp_s[j] > key;
      if (r < k) {
        const uint32_t e = 0xffffffffu - (uint32_t)(key & 0xffffffffu);
        idx_s[r] = e;
        selw_s[r] = w_s[e < (uint32_t)E ? e : 0u];
      }
    }
    __syncthreads();
    if (tid == 0) {
      float sum = -0.0f;
      for (int r = 0; r < k; r++) sum = __fadd_rn(sum, selw_s[r]);
      sum_s = __fadd_rn(sum, 1e-20f);
    }
    __syncthreads();
    if (tid < k) {
      const uint32_t idx = idx_s[tid] < (uint32_t)E ? idx_s[tid] : 0u;
      a.sel_idx[(size_t)t * k + tid] = idx;
      a.sel_w[(size_t)t * k + tid] = a.normalize ? __fdiv_rn(selw_s[tid], sum_s) : selw_s[tid];
      if (FUSED) sm.sel[tid] = idx;
    }
  }
  if (FUSED) {
    __syncthreads();
    dispatch_small_body(a, sm);
  }
}

// ydest[pos] = the output row of sorted position pos in its source rank's output table
// (EpReturnMap); positions past the received count are left alone.
__global__ void __launch_bounds__(256) ep_dest_kernel(ForwardArgs a) {
  pdl_wait();
  const int count = a.offsets[a.E + 1];
  const EpReturnMap m = a.ret;
  for (int pos = blockIdx.x * blockDim.x + threadIdx.x; pos < count; pos += gridDim.x * blockDim.x) {
    const int p = a.sorted[pos];
    const int r = p / m.k1, j = p - r * m.k1;
    const int s = r / m.tmax, t = r - s * m.tmax;
    const size_t row = j < m.k ? (size_t)t * m.k + j : (size_t)m.tokens[s] * m.k + t;
    a.ydest[pos] = reinterpret_cast<float *>(m.peer[s] + m.off_ret) + row * a.H;
  }
}

int launch_forward(const ForwardArgs &a, cudaStream_t stream, cudaEvent_t *ev,
                   const GemvPlan *gemv, const TcPlan *tc, int mode) {
  int launches = 0;
  if (mode & kRunIdentity) {  // pair outputs given in pair order (expert-parallel combine)
    const int n = a.T * a.k + (a.shared ? a.T : 0);
    launch_pdl(iota_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, a.inverse, n);
    launches++;
  }
  const bool glm = a.family == kGlm;
  // one decode token of a softmax family: top-k and dispatch in one kernel
  const bool fused_dispatch = (mode & kRunRoute) && (mode & kRunExperts) && !a.rows_mode &&
                              a.T == 1 && a.k <= kSmallPairs && a.E + 1 <= 1024;
  auto mark = [&](int stage) {
    if (ev) cudaEventRecord(ev[stage], stream);
  };
  if (mode & kRunRoute) {
  // 1. Gemma router / expert inputs
  mark(kStagePrep);
  const void *router_x = a.x;
  bool router_x_bf16 = a.input_bf16;
  if (a.family == kGemma) {
    size_t smem = (size_t)kPrepStages * kPrepTokens * kPrepLd * sizeof(float);
    set_smem(gemma_prep_kernel, smem);
    launch_pdl(gemma_prep_kernel, dim3((a.T + kPrepTokens - 1) / kPrepTokens), dim3(256), smem, stream, a);
    launches++;
    router_x = a.router_in;
    router_x_bf16 = false;
  }
  // 2. router logits
  mark(kStageRouter);
  if (a.T <= 16 || !a.xT || !a.router_dup || a.H % kRgChunk) {
    int RT = std::min(4, a.T);
    const int epc = std::max(1, std::min(kSmallExperts, a.E1 / 256));
    const int xb = router_x_bf16 ? 2 : 4;
    auto bytes = [&](int rt) {
      return (size_t)epc * (a.H + 4) * 4 + (size_t)rt * (a.H + 16 / xb) * xb;
    };
    while (RT > 1 && bytes(RT) > 200 * 1024) RT >>= 1;
    const size_t smem = bytes(RT);
    dim3 grid((a.E1 + epc - 1) / epc, (a.T + RT - 1) / RT);
#define DM_ROUTER_SMALL(G, X)                                                               \
  {                                                                                         \
    auto fn = router_small_kernel<G, X>;                                                    \
    set_smem(fn, smem);                                                                     \
    launch_pdl(fn, grid, dim3(256), smem, stream, (const float *)a.router_rows, router_x, a.T,  \
               a.H, a.E1, RT, epc, a.logit_bias, a.E, a.logits, a.status);                  \
  }
    if (glm && router_x_bf16) DM_ROUTER_SMALL(true, true)
    else if (glm) DM_ROUTER_SMALL(true, false)
    else DM_ROUTER_SMALL(false, false)
#undef DM_ROUTER_SMALL
  } else {
    const int xld = (a.T + kRgTokens - 1) / kRgTokens * kRgTokens;
    // GLM with a bf16 router and bf16 input may take the fused step; the transpose marks
    // the input tiles that rule it out
    const int exact = glm && router_x_bf16 && a.router_exact_products;
    uint8_t *tiny = exact ? a.x_tiny : nullptr;
    // 32 x 128 tiles when there are enough of them to fill the SMs, else 32 x 64
    static const int n_sm = [] {
      int dev = 0, n = 148;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      return n;
    }();
    const int wide_tiles = (a.E1 + kRwExperts - 1) / kRwExperts * (xld / kRwTokens);
    const bool wide = a.E1 >= kRwExperts && a.H % kRwChunk == 0 && wide_tiles >= n_sm;
    // the wide tiles with 64 chains per thread read the input once per value
    // (DISKMULE_CUDA_ROUTER_X8=0 keeps the 32-chain form over the doubled input)
    static const bool x8_on = [] {
      const char *e = getenv("DISKMULE_CUDA_ROUTER_X8");
      return !(e && e[0] == '0');
    }();
    const bool x8 = wide && x8_on;
    // every router form but the 32-chain wide one reads the input once per value
    const bool doubled = wide && !x8;
    launch_pdl(transpose_x_kernel, dim3((a.H + 31) / 32, xld / 32), dim3(256), 0, stream, router_x,
               router_x_bf16 ? 1 : 0, a.T, a.H, xld, a.xT, tiny, doubled ? 0 : 1);
    launches++;
#define DM_ROUTER_TILED(KERNEL, G, EXPERTS, THREADS, SMEM)                                     \
  {                                                                                          \
    auto fn = KERNEL<G>;                                                                     \
    set_smem(fn, SMEM);                                                                      \
    launch_pdl(fn, dim3((a.E1 + EXPERTS - 1) / EXPERTS, xld / kRgTokens), dim3(THREADS), SMEM, \
               stream, (const float *)a.router_dup, router_dup_ld(a.E1), (const float *)a.xT,  \
               xld, a.T, a.H, a.E1, a.logit_bias, a.E, a.logits, (const uint8_t *)tiny, exact); \
  }
    const size_t rg_smem = (size_t)kRgStages * kRgStageBytes;
    const size_t rw_smem = (size_t)kRwStages * kRwStageBytes;
    const size_t rx_smem = (size_t)kRxStages * kRxStageBytes;
    if (x8 && glm) DM_ROUTER_TILED(router_x8_kernel, true, kRxExperts, kRxThreads, rx_smem)
    else if (x8) DM_ROUTER_TILED(router_x8_kernel, false, kRxExperts, kRxThreads, rx_smem)
    else if (wide && glm) DM_ROUTER_TILED(router_wide_kernel, true, kRwExperts, kRwThreads, rw_smem)
    else if (wide) DM_ROUTER_TILED(router_wide_kernel, false, kRwExperts, kRwThreads, rw_smem)
    else if (glm) DM_ROUTER_TILED(router_gemm_kernel, true, kRgExperts, kRgThreads, rg_smem)
    else DM_ROUTER_TILED(router_gemm_kernel, false, kRgExperts, kRgThreads, rg_smem)
#undef DM_ROUTER_TILED
  }
  launches++;
  // 3. top-k
  mark(kStageTopk);
  if (glm && fused_dispatch)
    launch_pdl(topk_sigmoid_rank_kernel<true>, dim3(1),
               dim3(std::max(kSmallPairs, (a.E + 1 + 31) / 32 * 32)), 0, stream, a);
  else if (glm)
    launch_pdl(topk_sigmoid_rank_kernel<false>, dim3(a.T), dim3(std::min(1024, (a.E + 31) / 32 * 32)),
               0, stream, a);
  else if (fused_dispatch)
    launch_pdl(topk_dispatch1_kernel, dim3(1),
               dim3(std::max(kSmallPairs, (a.E + 1 + 31) / 32 * 32)), 0, stream, a);
  else
    launch_pdl(topk_rank_softmax_kernel, dim3(a.T), dim3(32 * ((a.E + 31) / 32)), 0, stream,
               (const float *)a.logits, a.T, a.E1, a.E, a.k, a.sel_idx, a.sel_w, a.status);
  launches++;
  }
  if (mode & kRunExperts) {
  // 4. dispatch (already done with the top-k of one decode token)
  mark(kStageDispatch);
  if (fused_dispatch) {
    launches--;  // counted with the top-k
  } else if (a.T * a.k <= kSmallPairs && !a.drop_invalid) {
    launch_pdl(dispatch_small_kernel, dim3(1), dim3(std::max(kSmallPairs, (a.E + 1 + 31) / 32 * 32)),
               0, stream, a);
  } else {
    size_t dsmem = ((size_t)kDispatchWarps * (a.E + 1) + 2 * (a.E + 1)) * sizeof(int32_t);
    set_smem(dispatch_kernel, dsmem);
    launch_pdl(dispatch_kernel, dim3(1), dim3(kDispatchThreads), dsmem, stream, a);
  }
  launches++;
  if (a.ydest) {  // expert-parallel return: each sorted row's destination in peer memory
    const int n = a.T * a.k;
    launch_pdl(ep_dest_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, a);
    launches++;
  }
  // 5. gate/up (+activation) and 6. down, over the active experts
  const int max_active = std::min(a.E + (a.shared ? 1 : 0), a.T * a.k + (a.shared ? 1 : 0));
  mark(kStageUp);
  if (gemv && tc) {
    int n = launch_tc_experts(a, *tc, *tc->weights, stream, ev ? ev[kStageDown] : nullptr);
    if (n < 0) return -1;
    launches += n;
  } else if (gemv) {
    int n = launch_gemv_experts(a, *gemv, stream, ev ? ev[kStageDown] : nullptr);
    if (n < 0) return -1;
    launches += n;
  } else {
  {
    int tt = choose_tt(a.H);
    ExpertFn fn = expert_fn(true, a.gate_type, tt);
    size_t smem = (size_t)tt * (a.H / 32) * kUnitStride * sizeof(float);
    set_smem(fn, smem);
    int rows_per_cta = kExpertWarps * 4;
    dim3 grid((a.I + rows_per_cta - 1) / rows_per_cta, max_active);
    fn<<<grid, kExpertThreads, smem, stream>>>(a, rows_per_cta);
    launches++;
  }
  mark(kStageDown);
  {
    int tt = choose_tt(a.I);
    ExpertFn fn = expert_fn(false, a.down_type, tt);
    size_t smem = (size_t)tt * (a.I / 32) * kUnitStride * sizeof(float);
    set_smem(fn, smem);
    int rows_per_cta = kExpertWarps * 8;
    dim3 grid((a.H + rows_per_cta - 1) / rows_per_cta, max_active);
    fn<<<grid, kExpertThreads, smem, stream>>>(a, rows_per_cta);
    launches++;
  }
  }
  }
  // 7. combine (or the per-row outputs of the rows mode)
  mark(kStageCombine);
  if (mode & kRunCombine) {
    launch_pdl(combine_kernel, dim3(a.T, (a.H / 4 + kCombineThreads - 1) / kCombineThreads),
               dim3(kCombineThreads), 0, stream, a);
    launches++;
  }
  if (mode & kRunScatter) {
    launch_pdl(scatter_rows_kernel, dim3(a.T, (a.H / 4 + 127) / 128), dim3(128), 0, stream, a);
    launches++;
  }
  mark(kStageCount);
  return launches;
}

// ---------------------------------------------------------------------------
// Metal-style operators
// ---------------------------------------------------------------------------

template <class U>
__global__ void __launch_bounds__(256) gemv_unit_kernel(const uint8_t *w, int rows, int cols,
                                                       uint64_t rb, const float *x, float *y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const uint8_t *row = w + (size_t)warp * rb;
  float acc = 0.0f;
  for (int u = lane; u < cols / 32; u += 32) {
    float wv[32];
    U::decode(row, u, wv);
#pragma unroll
    for (int j = 0; j < 32; j++) acc = fmaf(wv[j], x[u * 32 + j], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[warp] = acc;
}

// dense rows of any width (F32 / F16 / BF16), element by element
__global__ void __launch_bounds__(256) gemv_dense_kernel(const uint8_t *w, int kind, int rows,
                                                        int cols, const float *x, float *y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float acc = 0.0f;
  for (int c = lane; c < cols; c += 32) {
    size_t i = (size_t)warp * cols + c;
    float v;
    if (kind == DM_F32) v = reinterpret_cast<const float *>(w)[i];
    else if (kind == DM_F16) v = f16_bits_to_f32(reinterpret_cast<const uint16_t *>(w)[i]);
    else v = bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(w)[i]);
    acc = fmaf(v, x[c], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[warp] = acc;
}

// GLM-5.2 checkpoint encodings, one warp per row (lanes stride the columns, so a
// warp's byte loads are one coalesced 32-byte piece), products summed with fma and a
// warp reduction (a tolerance-bound result, like the reference's Metal kernels,
// metal/kernels.metal:273-344):
//   kQuantI8Row:  w = int8 * scales[row]
//   kQuantI4:     w = (nibble - 8) * scales[row * ceil(cols / group) + col / group],
//                 low nibble for even columns
//   kQuantF8:     w = e4m3fn(byte) * scales[(row / 128) * ceil(cols / 128) + col / 128],
//                 decoded through a 256-entry table built per block; the two invalid
//                 codes (exponent 15, fraction 7) decode to NaN.
__global__ void __launch_bounds__(256) quant_gemv_kernel(int enc, const uint8_t *w,
                                                        const float *scales, int rows, int cols,
                                                        int group, const float *x, float *y) {
  __shared__ float lut[256];
  if (enc == kQuantF8) {
    const int v = threadIdx.x;
    const int e = (v >> 3) & 15, f = v & 7;
    const float mag = e == 0 ? (float)f * 0.001953125f
                             : __fmul_rn(1.0f + (float)f * 0.125f, ldexpf(1.0f, e - 7));
    lut[v] = (e == 15 && f == 7) ? __int_as_float(0x7fc00000) : ((v & 0x80) ? -mag : mag);
    __syncthreads();
  }
  const int row = (int)(blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  float acc = 0.0f;
  if (enc == kQuantI8Row) {
    const int8_t *q = reinterpret_cast<const int8_t *>(w) + (size_t)row * cols;
    const float s = scales[row];
    for (int c = lane; c < cols; c += 32) acc = fmaf(__fmul_rn((float)q[c], s), x[c], acc);
  } else if (enc == kQuantI4) {
    const int rb = (cols + 1) / 2, sc = (cols + group - 1) / group;
    const uint8_t *q = w + (size_t)row * rb;
    const float *srow = scales + (size_t)row * sc;
    for (int c = lane; c < cols; c += 32) {
      const uint8_t b = q[c >> 1];
      const int nib = (c & 1) ? (b >> 4) : (b & 15);
      acc = fmaf(__fmul_rn((float)(nib - 8), srow[c / group]), x[c], acc);
    }
  } else {
    const uint8_t *q = w + (size_t)row * cols;
    const float *srow = scales + (size_t)(row / 128) * ((cols + 127) / 128);
    for (int c = lane; c < cols; c += 32)
      acc = fmaf(__fmul_rn(lut[q[c]], srow[c >> 7]), x[c], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

int launch_quant_gemv(int enc, const uint8_t *w, const float *scales, int rows, int cols,
                      int group, const float *x, float *y, cudaStream_t stream) {
  quant_gemv_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(enc, w, scales, rows, cols, group, x, y);
  return 1;
}

int launch_gemv(int kind, const uint8_t *w, int rows, int cols, const float *x, float *y,
                cudaStream_t stream) {
  int blocks = (rows + 7) / 8;
  uint64_t rb = row_bytes(kind, cols);
  bool aligned16 = ((uintptr_t)w % 16) == 0 && rb % 16 == 0;
  switch (kind) {
    case DM_Q4_K:
      if (!aligned16) return -1;
      gemv_unit_kernel<Q4KUnit><<<blocks, 256, 0, stream>>>(w, rows, cols, rb, x, y);
      break;
    case DM_Q6_K: gemv_unit_kernel<Q6KUnit><<<blocks, 256, 0, stream>>>(w, rows, cols, rb, x, y); break;
    case DM_Q5_0: gemv_unit_kernel<Q50Unit><<<blocks, 256, 0, stream>>>(w, rows, cols, rb, x, y); break;
    case DM_Q8_0: gemv_unit_kernel<Q80Unit><<<blocks, 256, 0, stream>>>(w, rows, cols, rb, x, y); break;
    case DM_F32:
    case DM_F16:
    case DM_BF16: gemv_dense_kernel<<<blocks, 256, 0, stream>>>(w, kind, rows, cols, x, y); break;
    default: return -1;
  }
  return 1;
}

__global__ void elementwise_kernel(int op, const float *a, const float *b, float *out, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float g = a[i];
    // Metal gelu_mul / silu_mul (metal/kernels.metal:96-122) against the CPU forms
    out[i] = op == kOpGeluMul ? __fmul_rn(gelu_tanh(g), b[i]) : __fmul_rn(glm_cached_silu(g), b[i]);
  }
}

// rms_norm as src/cpu.rs:99-143: one sequential fma chain for the sum of squares
__global__ void rms_norm_kernel(const float *x, const float *w, float *out, int n, float eps,
                                int32_t *status) {
  __shared__ float inv_s;
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s = __fmaf_rn(x[i], x[i], s);
    float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)n), eps)));
    if (!isfinite(inv)) *status = kStatusNonFiniteNorm;
    inv_s = inv;
  }
  __syncthreads();
  float inv = inv_s;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[i] = w ? __fmul_rn(__fmul_rn(x[i], w[i]), inv) : __fmul_rn(x[i], inv);
}

int launch_elementwise(int op, const float *a, const float *b, float *out, int n, float,
                       cudaStream_t stream) {
  int blocks = std::min((n + 255) / 256, 1024);
  elementwise_kernel<<<blocks, 256, 0, stream>>>(op, a, b, out, n);
  return 1;
}

int launch_rms_norm(const float *x, const float *w, float *out, int n, float eps,
                    int32_t *status, cudaStream_t stream) {
  rms_norm_kernel<<<1, 256, 0, stream>>>(x, w, out, n, eps, status);
  return 1;
}

}  // namespace dm
