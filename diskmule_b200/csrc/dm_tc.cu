// dm_tc.cu -- tcgen05 grouped expert GEMM (see dm_tc.cuh).
//
// Kernel structure (one CTA = 9 warps, one 128-row A tile, two producer threads per row):
//   warps 0..7 (producers), per K step ks on stage s = ks % 2:
//       wait empty[s] (the MMAs of step ks-2 are done with the stage); load step ks+1's
//       raw quant blocks into registers; dequantise step ks into swizzled smem;
//       fence.proxy.async; one arrival per warp on full[s]
//   warp 8, lane 0 (control): wait empty[s]; TMA of the B tile (hi, lo) -> tma[s];
//       wait tma[s] and full[s]; tcgen05.mma chain; tcgen05.commit -> empty[s]
//   epilogue: wait for the last commit; warps 0..3 tcgen05.ld their 32 lanes; write.
// No block-wide barrier in the main loop. Every mbarrier wait is bounded (about 0.1 s
// of SM clock); on expiry the kernel records kStatusTimeout (which stops every other
// CTA too), waits (bounded) for its own work in flight, frees its tensor memory and
// returns.
#include <cudaTypedefs.h>

#include <algorithm>

#include "dm_kernels.cuh"
#include "dm_tc.cuh"

namespace dm {
namespace tc {

constexpr long long kWaitCycles = 200000000ll;  // ~0.1 s at 2 GHz; real waits take microseconds

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Wait for the phase with parity `parity` to complete; false after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const long long start = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - start > kWaitCycles) return false;
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, f32 accumulate
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 16 consecutive f32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: fp16 A and B (K-major), f32 D, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ uint4 ldg16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Store 8 fp16 values (one 16-byte chunk `c` of the 128-byte row `r` of an atom)
// with the 128-byte swizzle: chunk c lands at c ^ (r & 7).
__device__ __forceinline__ void st_chunk(uint32_t atom, int r, int c, uint4 v) {
  const uint32_t addr = atom + (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------
// f32 pair arithmetic (packed .f32x2 instructions of sm_100) and fp16 packing
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t pair(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// f32 pair -> half2 (one rounding each), low element in the low half
__device__ __forceinline__ uint32_t to_h2(uint64_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;"
      : "=r"(h)
      : "f"(__uint_as_float((uint32_t)(v >> 32))), "f"(__uint_as_float((uint32_t)v)));
  return h;
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// bytes c and c+1 of w as the f32 pair (0.5 + byte/256): exact for bytes below 128
__device__ __forceinline__ uint64_t magic2(uint32_t w, int c) {
  const uint32_t lo = __byte_perm(w, 0x3F000000u, 0x7044u | ((uint32_t)c << 8));
  const uint32_t hi = __byte_perm(w, 0x3F000000u, 0x7044u | ((uint32_t)(c + 1) << 8));
  return ((uint64_t)hi << 32) | lo;
}

// ---------------------------------------------------------------------------
// producers: one A row's part of a K step, dequantised in f32 and rounded once to
// fp16, stored in the swizzled layout. A quant byte q becomes f = 0.5 + q/256
// (exact), so a value alpha*q + beta is fma(f, 256*alpha, beta - 128*alpha): one
// packed f32x2 fma per two weights, f32-accurate before the fp16 rounding.
// ---------------------------------------------------------------------------

// One group pair gp of a Q4_K super-block (src/cpu.rs:585-616) -> one atom: chunks
// 0..3 = low nibbles (sub-block 2gp), chunks 4..7 = high nibbles (sub-block 2gp+1),
// in element order. value = (d*sc)*q - dmin*m. A high nibble is read shifted right by
// one bit (byte 8*q, below 128 as the magic needs): f = 0.5 + q/32.
__device__ __forceinline__ void produce_q4k(uint4 hd, uint4 qa, uint4 qb, int gp, uint32_t atom,
                                            int r) {
  const float d = f16_bits_to_f32((uint16_t)(hd.x & 0xffff));
  const float dmin = f16_bits_to_f32((uint16_t)(hd.x >> 16));
  const uint32_t sca = hd.y & 0x3F3F3F3Fu, ma = hd.z & 0x3F3F3F3Fu;
  const uint32_t scb = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
  const uint32_t mb = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
  const int jl = 2 * gp, jh = jl + 1;
  const uint32_t scl = jl < 4 ? (sca >> (8 * jl)) & 0xff : (scb >> (8 * (jl - 4))) & 0xff;
  const uint32_t ml = jl < 4 ? (ma >> (8 * jl)) & 0xff : (mb >> (8 * (jl - 4))) & 0xff;
  const uint32_t sch = jh < 4 ? (sca >> (8 * jh)) & 0xff : (scb >> (8 * (jh - 4))) & 0xff;
  const uint32_t mh = jh < 4 ? (ma >> (8 * jh)) & 0xff : (mb >> (8 * (jh - 4))) & 0xff;
  const float al = __fmul_rn(d, (float)scl), bl = __fmul_rn(dmin, (float)ml);
  const float ah = __fmul_rn(d, (float)sch), bh = __fmul_rn(dmin, (float)mh);
  // low nibble: v = al*q - bl = fma(f, 256 al, -(128 al + bl))
  const uint64_t Ml = pair(256.0f * al, 256.0f * al);
  const float cl = -(128.0f * al + bl);
  const uint64_t Cl = pair(cl, cl);
  // high nibble (byte = 8 q): v = ah*q - bh = fma(f, 32 ah, -(16 ah + bh))
  const uint64_t Mh = pair(32.0f * ah, 32.0f * ah);
  const float ch = -(16.0f * ah + bh);
  const uint64_t Ch = pair(ch, ch);
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const uint32_t wl = w[2 * c + k] & 0x0F0F0F0Fu, wh = (w[2 * c + k] >> 1) & 0x78787878u;
      lo[2 * k] = to_h2(fma2(magic2(wl, 0), Ml, Cl));
      lo[2 * k + 1] = to_h2(fma2(magic2(wl, 2), Ml, Cl));
      hi[2 * k] = to_h2(fma2(magic2(wh, 0), Mh, Ch));
      hi[2 * k + 1] = to_h2(fma2(magic2(wh, 2), Mh, Ch));
    }
    st_chunk(atom, r, c, make_uint4(lo[0], lo[1], lo[2], lo[3]));
    st_chunk(atom, r, c + 4, make_uint4(hi[0], hi[1], hi[2], hi[3]));
  }
}

// Atom g of half h of a Q6_K super-block (src/cpu.rs:618-645), split layout:
// elements 128h + 64g + j, i.e. quarters 2g and 2g+1. ql = the half's 64 low-bit bytes
// (16 words), qh = its 32 high-bit bytes (8 words), sw = the word holding the atom's
// four scales (scale index 8h + 4g + (j / 16)). value = (d*sc)*(q-32) =
// fma(f, 256 s, -160 s). Quarter 2g+u takes nibble 4g of ql[8u + i] and high bits
// 2(2g+u) of qh[i].
__device__ __forceinline__ void produce_q6k(const uint32_t *ql, const uint32_t *qh, uint32_t sw,
                                            float d, int g, uint32_t atom, int r) {
  const int nsh = 4 * g;
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const int u = c >> 2;          // quarter 2g + u
    const int idx0 = 8 * (c & 3);  // first idx of the chunk within the quarter
    const int sb = (idx0 >> 4) + 2 * u;
    const float s = __fmul_rn(d, (float)(int8_t)((sw >> (8 * sb)) & 0xff));
    const uint64_t M = pair(256.0f * s, 256.0f * s), C = pair(-160.0f * s, -160.0f * s);
    uint32_t out[4];
#pragma unroll
    for (int wi = 0; wi < 2; wi++) {
      const int i = idx0 / 4 + wi;
      const uint32_t src = u ? ql[8 + i] : ql[i];
      const uint32_t hg = g ? qh[i] : (qh[i] << 4);
      const uint32_t q = ((src >> nsh) & 0x0F0F0F0Fu) | ((hg >> (2 * u)) & 0x30303030u);
      out[2 * wi] = to_h2(fma2(magic2(q, 0), M, C));
      out[2 * wi + 1] = to_h2(fma2(magic2(q, 2), M, C));
    }
    st_chunk(atom, r, c, make_uint4(out[0], out[1], out[2], out[3]));
  }
}

__device__ __forceinline__ uint32_t spread4(uint32_t v) {
  return ((v & 0xfu) * 0x02040810u) & 0x10101010u;
}

// Q5_0 block b (0 or 1) of a 64-value atom (src/cpu.rs:560-574), split layout ->
// chunks 4b..4b+3. value = d*(q-16) = fma(f, 256 d, -144 d).
__device__ __forceinline__ void produce_q50(uint4 qs, uint32_t hb, float d, int b, uint32_t atom,
                                            int r) {
  const uint64_t M = pair(256.0f * d, 256.0f * d), C = pair(-144.0f * d, -144.0f * d);
  const uint32_t w[4] = {qs.x, qs.y, qs.z, qs.w};
  uint32_t lo[4], hi[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    lo[i] = (w[i] & 0x0F0F0F0Fu) | spread4(hb >> (4 * i));
    hi[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | spread4(hb >> (16 + 4 * i));
  }
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    o[2 * i] = to_h2(fma2(magic2(lo[i], 0), M, C));
    o[2 * i + 1] = to_h2(fma2(magic2(lo[i], 2), M, C));
  }
  st_chunk(atom, r, 4 * b + 0, make_uint4(o[0], o[1], o[2], o[3]));
  st_chunk(atom, r, 4 * b + 1, make_uint4(o[4], o[5], o[6], o[7]));
#pragma unroll
  for (int i = 0; i < 4; i++) {
    o[2 * i] = to_h2(fma2(magic2(hi[i], 0), M, C));
    o[2 * i + 1] = to_h2(fma2(magic2(hi[i], 2), M, C));
  }
  st_chunk(atom, r, 4 * b + 2, make_uint4(o[0], o[1], o[2], o[3]));
  st_chunk(atom, r, 4 * b + 3, make_uint4(o[4], o[5], o[6], o[7]));
}

// ---------------------------------------------------------------------------
// pack: sorted activation rows -> fp16 hi + lo pair with a power-of-two scale
// ---------------------------------------------------------------------------

__device__ __forceinline__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// scale s = 2^(13 - floor(log2 max)) puts the row's largest magnitude in [2^13, 2^14)
__device__ __forceinline__ float pow2_scale(float m) {
  if (!(m > 0.0f) || !isfinite(m)) return 1.0f;
  return exp2f((float)(13 - ilogbf(m)));
}

// Row `pos` of the packed matrix: hi = fp16(x*s) in row pos, lo = fp16(x*s - hi) in
// row pos + lo_offset; x*s = hi + lo to about 2^-22 relative.
template <bool INPUT>
__global__ void __launch_bounds__(256) pack_kernel(ForwardArgs a, __half *out, float *inv, int K,
                                                  int lo_offset) {
  __shared__ float red[8];
  const int pos = blockIdx.x;
  if (pos >= a.offsets[a.E + 1]) return;
  const float *src;
  if (INPUT) {
    const int P = a.T * a.k, pr = a.sorted[pos];
    const int tok = pr < P ? pr / a.k : pr - P;
    src = (a.family == kGemma ? a.expert_in : reinterpret_cast<const float *>(a.x)) +
          (size_t)tok * K;
  } else {
    src = a.h + (size_t)pos * K;
  }
  float m = 0.0f;
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4 *>(src + i);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  const float s = pow2_scale(block_max(m, red));
  for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4 *>(src + i);
    const float xs[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
    __half hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      hi[j] = __float2half_rn(xs[j]);
      lo[j] = __float2half_rn(xs[j] - __half2float(hi[j]));
    }
    *reinterpret_cast<uint2 *>(out + (size_t)pos * K + i) =
        make_uint2(h2u(__halves2half2(hi[0], hi[1])), h2u(__halves2half2(hi[2], hi[3])));
    *reinterpret_cast<uint2 *>(out + (size_t)(pos + lo_offset) * K + i) =
        make_uint2(h2u(__halves2half2(lo[0], lo[1])), h2u(__halves2half2(lo[2], lo[3])));
  }
  if (threadIdx.x == 0) inv[pos] = 1.0f / s;
}

// ---------------------------------------------------------------------------
// GEMM kernels (warp-specialised)
// ---------------------------------------------------------------------------

__device__ __forceinline__ float activate(const ForwardArgs &a, int expert, float g, float u) {
  if (a.family == kGemma) return __fmul_rn(gelu_tanh(g), u);
  if (a.family == kQwen) return __fmul_rn(qwen_silu(g), u);
  if (expert == a.E) return __fmul_rn(glm_silu(g), u);
  return __fmul_rn(glm_cached_silu(g), u);
}

// 8 producer warps (two threads per A row: row t & 127, part t >> 7) and one
// control warp (TMA + MMA issue); warps 0..3 also own the TMEM lanes for the epilogue.
constexpr int kProducerThreads = 256;
constexpr int kProducerWarps = kProducerThreads / 32;
constexpr int kTcThreads = kProducerThreads + 32;
constexpr int kStages = 2;

// Stage s: A tile at base + s*stage, B tile (hi | lo) after it; barriers after the
// stages: tma[s] (B tile landed, transaction bytes), full[s] (A tile written, one
// arrival per producer warp), empty[s] (stage consumed, tcgen05.commit).
struct Smem {
  uint32_t base, stage, a_bytes, bars;
  uint8_t *generic;  // generic pointer of the aligned base
  __device__ __forceinline__ uint32_t a(int s) const { return base + (uint32_t)s * stage; }
  __device__ __forceinline__ uint32_t b(int s) const { return a(s) + a_bytes; }
  __device__ __forceinline__ uint32_t tma(int s) const { return bars + 8u * s; }
  __device__ __forceinline__ uint32_t full(int s) const { return bars + 8u * (kStages + s); }
  __device__ __forceinline__ uint32_t empty(int s) const { return bars + 8u * (2 * kStages + s); }
  __device__ __forceinline__ uint32_t slot() const { return bars + 8u * 3 * kStages; }
};

template <int ATOMS, int NT>
struct Layout {
  static constexpr uint32_t kA = ATOMS * 16384u;         // 128 rows x 128 B per atom
  static constexpr uint32_t kBHalf = ATOMS * NT * 128u;  // one of hi / lo
  static constexpr uint32_t kStage = kA + 2 * kBHalf;
  static constexpr size_t kSmem = 1024 + kStages * (size_t)kStage + 128;
};

template <int ATOMS, int NT>
__device__ __forceinline__ Smem carve(uint8_t *dsm) {
  using L = Layout<ATOMS, NT>;
  Smem s;
  const uint32_t raw = smem_u32(dsm);
  s.base = (raw + 1023u) & ~1023u;
  s.generic = dsm + (s.base - raw);
  s.stage = L::kStage;
  s.a_bytes = L::kA;
  s.bars = s.base + kStages * L::kStage;
  return s;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool aborted(const int *abort_flag, const int32_t *status) {
  return *reinterpret_cast<const volatile int *>(abort_flag) ||
         *reinterpret_cast<const volatile int32_t *>(status) == kStatusTimeout;
}

// Bounded wait that also gives up as soon as another thread of the CTA has aborted.
__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, const int *abort_flag) {
  const long long start = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (*reinterpret_cast<const volatile int *>(abort_flag)) return false;
    if (clock64() - start > kWaitCycles) return false;
  }
}

// Producer side: `P` supplies `Raw load(int ks)` and `void store(const Raw &, int ks,
// uint32_t a_base)`; step ks+1 is loaded while step ks is dequantised. The decision to
// stop is taken per warp (vote), so every lane leaves the loop at the same step.
template <int ATOMS, int NT, class P>
__device__ __forceinline__ void producer_loop(const Smem &sm, int nsteps, P &prod, int *abort_flag,
                                              const int32_t *status) {
  const int lane = threadIdx.x & 31;
  auto cur = prod.load(0);
  for (int ks = 0; ks < nsteps; ks++) {
    const int s = ks % kStages, use = ks / kStages;
    bool stop = ks >= kStages && !mbar_wait_or_abort(sm.empty(s), (uint32_t)((use - 1) & 1), abort_flag);
    stop = stop || aborted(abort_flag, status);
    if (__any_sync(0xffffffffu, stop)) {
      if (lane == 0) atomicExch(abort_flag, 1);
      break;
    }
    auto nxt = prod.load(ks + 1 < nsteps ? ks + 1 : ks);
    prod.store(cur, ks, sm.a(s));
    cur = nxt;
    fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.full(s));
  }
}

// Control side (one thread): TMA of the B tiles and the MMA chain.
template <int ATOMS, int NT>
__device__ __forceinline__ void control_loop(const Smem &sm, uint32_t tmem, const CUtensorMap *bmap,
                                             int pos0, int lo_offset, int nsteps, int *abort_flag,
                                             const int32_t *status, int *issued) {
  using L = Layout<ATOMS, NT>;
  constexpr uint32_t idesc = idesc_f16(NT);
  for (int ks = 0; ks < nsteps; ks++) {
    const int s = ks % kStages, use = ks / kStages;
    if ((ks >= kStages && !mbar_wait_or_abort(sm.empty(s), (uint32_t)((use - 1) & 1), abort_flag)) ||
        aborted(abort_flag, status)) {
      atomicExch(abort_flag, 1);
      break;
    }
    mbar_expect_tx(sm.tma(s), 2 * L::kBHalf);
#pragma unroll
    for (int at = 0; at < ATOMS; at++) {
      const int k0 = (ks * ATOMS + at) * 64;
      tma_load_2d(sm.b(s) + at * (NT * 128u), bmap, k0, pos0, sm.tma(s));
      tma_load_2d(sm.b(s) + L::kBHalf + at * (NT * 128u), bmap, k0, pos0 + lo_offset, sm.tma(s));
    }
    if (!mbar_wait(sm.tma(s), (uint32_t)(use & 1)) ||
        !mbar_wait_or_abort(sm.full(s), (uint32_t)(use & 1), abort_flag)) {
      atomicExch(abort_flag, 1);
      break;
    }
    fence_after();
#pragma unroll
    for (int kk = 0; kk < 4 * ATOMS; kk++) {
      const uint64_t ad = sw128_desc(sm.a(s) + (kk >> 2) * 16384u + (kk & 3) * 32u);
      const uint32_t boff = (kk >> 2) * (NT * 128u) + (kk & 3) * 32u;
      mma_f16(tmem, ad, sw128_desc(sm.b(s) + boff), idesc, (ks == 0 && kk == 0) ? 0u : 1u);
      mma_f16(tmem, ad, sw128_desc(sm.b(s) + L::kBHalf + boff), idesc, 1u);
    }
    mma_commit(sm.empty(s));
    *issued = ks;
  }
}

// Barriers and tensor memory (warp 0 allocates). A CTA that starts after another
// has timed out begins aborted (decided by one thread, seen by all after the barrier).
template <int NT>
__device__ __forceinline__ uint32_t setup(const Smem &sm, int *abort_flag, int *issued,
                                          const int32_t *status) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    *abort_flag = *reinterpret_cast<const volatile int32_t *>(status) == kStatusTimeout;
    *issued = -1;
    for (int s = 0; s < kStages; s++) {
      mbar_init(sm.tma(s), 1);
      mbar_init(sm.full(s), kProducerWarps);
      mbar_init(sm.empty(s), 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if ((tid >> 5) == 0) tmem_alloc(sm.slot(), (uint32_t)(NT < 32 ? 32 : NT));
  fence_before();
  __syncthreads();
  fence_after();
  return *reinterpret_cast<volatile uint32_t *>(sm.generic + (sm.slot() - smem_u32(sm.generic)));
}

// After both loops: wait for the last issued MMAs, decide (uniformly) whether the
// accumulator is complete.
template <int NT>
__device__ __forceinline__ bool finish(const Smem &sm, int nsteps, int *abort_flag, int *issued,
                                       int32_t *status) {
  __syncthreads();
  const int last = *issued;
  bool ok = !*abort_flag && last == nsteps - 1;
  if (last >= 0 && !mbar_wait(sm.empty(last % kStages), (uint32_t)((last / kStages) & 1)))
    ok = false;
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (!ok && threadIdx.x == 0) atomicExch(status, kStatusTimeout);
  fence_after();
  return ok;
}

template <int NT>
__device__ __forceinline__ void read_columns(uint32_t tmem, float *v) {
  const uint32_t lane_base = ((uint32_t)((threadIdx.x >> 5) & 3) * 32u) << 16;
#pragma unroll
  for (int c = 0; c < NT; c += 16) tmem_ld16(tmem + lane_base + c, reinterpret_cast<uint32_t *>(v + c));
  tmem_wait_ld();
}

template <int NT>
__device__ __forceinline__ void teardown(uint32_t tmem) {
  fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) {
    fence_after();
    tmem_dealloc(tmem, (uint32_t)(NT < 32 ? 32 : NT));
  }
}

// gate/up producer: A row r = gate row i0+r/2 (even r) or up row i0+r/2 (odd r);
// a K step is half a Q4_K super-block (2 atoms = group pairs 2h, 2h+1); thread part p
// produces group pair 2h+p into atom p.
struct Q4KProducer {
  const uint4 *row;  // this row's super-blocks (9 uint4 each)
  int r, part;
  struct Raw {
    uint4 hd, qa, qb;
  };
  __device__ __forceinline__ Raw load(int ks) const {
    const uint4 *blk = row + (ks >> 1) * 9;
    const int gp = 2 * (ks & 1) + part;
    return {ldg16(blk), ldg16(blk + 1 + 2 * gp), ldg16(blk + 2 + 2 * gp)};
  }
  __device__ __forceinline__ void store(const Raw &w, int ks, uint32_t a_base) const {
    const int gp = 2 * (ks & 1) + part;
    produce_q4k(w.hd, w.qa, w.qb, gp, a_base + (uint32_t)part * 16384u, r);
  }
};

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_up_q4k_kernel(
    const __grid_constant__ CUtensorMap xmap, ForwardArgs a, const float *x_inv, int lo_offset) {
  extern __shared__ uint8_t dsm[];
  __shared__ int abort_flag, issued;
  if ((int)blockIdx.y >= *a.n_items) return;
  const int2 item = a.items[blockIdx.y];
  const int e = item.x, c0 = item.y;
  const int pos0 = a.offsets[e] + c0;
  const int ntok = min(NT, a.counts[e] - c0);
  const int i0 = blockIdx.x * 64;
  const Smem sm = carve<2, NT>(dsm);
  const int tid = threadIdx.x, r = tid & 127;
  const uint32_t tmem = setup<NT>(sm, &abort_flag, &issued, a.status);
  const int nsteps = a.H / 128;
  const int orow = i0 + (r >> 1);
  if (tid < kProducerThreads) {
    const bool shared = e == a.E;
    const uint8_t *mat = (r & 1) ? (shared ? a.sh_up : a.up + (size_t)e * a.up_stride)
                                 : (shared ? a.sh_gate : a.gate + (size_t)e * a.gate_stride);
    Q4KProducer prod{reinterpret_cast<const uint4 *>(mat + (size_t)orow * row_bytes(DM_Q4_K, a.H)),
                     r, tid >> 7};
    producer_loop<2, NT>(sm, nsteps, prod, &abort_flag, a.status);
  } else if (tid == kProducerThreads) {
    control_loop<2, NT>(sm, tmem, &xmap, pos0, lo_offset, nsteps, &abort_flag, a.status, &issued);
  }
  const bool ok = finish<NT>(sm, nsteps, &abort_flag, &issued, a.status);
  if (ok && tid < 128) {
    float v[NT];
    read_columns<NT>(tmem, v);
    const int lane = tid & 31;
#pragma unroll
    for (int n = 0; n < NT; n++) {
      const float u = __shfl_down_sync(0xffffffffu, v[n], 1);
      if (!(lane & 1) && n < ntok) {
        const float inv = x_inv[pos0 + n];
        a.h[(size_t)(pos0 + n) * a.I + orow] = activate(a, e, v[n] * inv, u * inv);
      }
    }
  }
  teardown<NT>(tmem);
}

// down producers: row r of the down tile; a K step is half a Q6_K super-block
// (2 atoms, part p -> atom p) or two Q5_0 blocks (1 atom, part p -> block p).
struct Q6KProducer {
  const uint8_t *quant;  // split quant region of this row's first super-block
  const uint16_t *d;     // f16 d of this row's first super-block
  int r, part;
  struct Raw {
    uint4 ql[4], qh[2];
    uint32_t sw;
    uint16_t d;
  };
  __device__ __forceinline__ Raw load(int ks) const {
    const uint4 *q = reinterpret_cast<const uint4 *>(quant + (size_t)(ks >> 1) * 208);
    const int h = ks & 1;
    Raw w;
#pragma unroll
    for (int i = 0; i < 4; i++) w.ql[i] = ldg16(q + 4 * h + i);
#pragma unroll
    for (int i = 0; i < 2; i++) w.qh[i] = ldg16(q + 8 + 2 * h + i);
    const uint4 sc = ldg16(q + 12);
    const uint32_t lo = h ? sc.z : sc.x, hi = h ? sc.w : sc.y;
    w.sw = part ? hi : lo;
    w.d = d[ks >> 1];
    return w;
  }
  __device__ __forceinline__ void store(const Raw &w, int, uint32_t a_base) const {
    produce_q6k(reinterpret_cast<const uint32_t *>(w.ql), reinterpret_cast<const uint32_t *>(w.qh),
                w.sw, f16_bits_to_f32(w.d), part, a_base + (uint32_t)part * 16384u, r);
  }
};

struct Q50Producer {
  const uint8_t *quant, *qh;  // split regions at this row's first block
  const uint16_t *d;
  int r, part;
  struct Raw {
    uint4 qs;
    uint32_t hb;
    uint16_t d;
  };
  __device__ __forceinline__ Raw load(int ks) const {
    const int blk = 2 * ks + part;
    return {ldg16(quant + (size_t)blk * 16), *reinterpret_cast<const uint32_t *>(qh + (size_t)blk * 4),
            d[blk]};
  }
  __device__ __forceinline__ void store(const Raw &w, int, uint32_t a_base) const {
    produce_q50(w.qs, w.hb, f16_bits_to_f32(w.d), part, a_base, r);
  }
};

template <int KIND, int NT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_down_kernel(
    const __grid_constant__ CUtensorMap hmap, ForwardArgs a, SplitTensor down,
    SplitTensor sh_down, const float *h_inv, int lo_offset) {
  constexpr int ATOMS = KIND == DM_Q6_K ? 2 : 1;
  extern __shared__ uint8_t dsm[];
  __shared__ int abort_flag, issued;
  if ((int)blockIdx.y >= *a.n_items) return;
  const int2 item = a.items[blockIdx.y];
  const int e = item.x, c0 = item.y;
  const int pos0 = a.offsets[e] + c0;
  const int ntok = min(NT, a.counts[e] - c0);
  const int m0 = blockIdx.x * 128;
  const Smem sm = carve<ATOMS, NT>(dsm);
  const int tid = threadIdx.x, r = tid & 127;
  const uint32_t tmem = setup<NT>(sm, &abort_flag, &issued, a.status);
  const int row = m0 + r;
  const int nsteps = a.I / (64 * ATOMS);
  if (tid < kProducerThreads) {
    const bool shared = e == a.E;
    const SplitTensor &D = shared ? sh_down : down;
    const int ex = shared ? 0 : e;
    if (KIND == DM_Q6_K) {
      const uint64_t g0 = ((uint64_t)ex * a.H + row) * (a.I / 256);
      Q6KProducer prod{D.quant + g0 * 208, D.d + g0, r, tid >> 7};
      producer_loop<ATOMS, NT>(sm, nsteps, prod, &abort_flag, a.status);
    } else {
      const uint64_t g0 = ((uint64_t)ex * a.H + row) * (a.I / 32);
      Q50Producer prod{D.quant + g0 * 16, D.qh + g0 * 4, D.d + g0, r, tid >> 7};
      producer_loop<ATOMS, NT>(sm, nsteps, prod, &abort_flag, a.status);
    }
  } else if (tid == kProducerThreads) {
    control_loop<ATOMS, NT>(sm, tmem, &hmap, pos0, lo_offset, nsteps, &abort_flag, a.status, &issued);
  }
  const bool ok = finish<NT>(sm, nsteps, &abort_flag, &issued, a.status);
  if (ok && tid < 128) {
    float v[NT];
    read_columns<NT>(tmem, v);
#pragma unroll
    for (int n = 0; n < NT; n++)
      if (n < ntok) a.ysorted[(size_t)(pos0 + n) * a.H + row] = v[n] * h_inv[pos0 + n];
  }
  teardown<NT>(tmem);
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

bool tc_supported(int gate_type, int down_type, int H, int I) {
  if (gate_type != DM_Q4_K) return false;
  if (down_type != DM_Q6_K && down_type != DM_Q5_0) return false;
  if (H % 256 || H % 128 || I % 64) return false;
  if (down_type == DM_Q6_K && I % 256) return false;
  return true;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  }
  return fn;
}

static bool encode(CUtensorMap *map, void *base, int cols, int rows, int nt) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)nt};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// x16 / h16 hold 2*rows rows: the hi halves in [0, rows), the lo halves in [rows, 2*rows).
int make_tc_maps(TcPlan &p, int H, int I, int nt) {
  if (!encode(&p.x_map, p.x16, H, 2 * p.rows, nt)) return -1;
  if (!encode(&p.h_map, p.h16, I, 2 * p.rows, nt)) return -1;
  return 0;
}

template <int NT>
static int launch_nt(const ForwardArgs &a, const TcPlan &p, const GemvPlan &g, cudaStream_t s,
                     cudaEvent_t down_mark) {
  const int rows_bound = a.T * a.k + (a.shared ? a.T : 0);
  tc::pack_kernel<true><<<rows_bound, 256, 0, s>>>(a, p.x16, p.x_inv, a.H, p.rows);
  {
    auto fn = tc::tc_up_q4k_kernel<NT>;
    ensure_smem_limit((const void *)fn);
    fn<<<dim3(a.I / 64, p.max_items), tc::kTcThreads, tc::Layout<2, NT>::kSmem, s>>>(
        p.x_map, a, p.x_inv, p.rows);
  }
  if (down_mark) cudaEventRecord(down_mark, s);
  tc::pack_kernel<false><<<rows_bound, 256, 0, s>>>(a, p.h16, p.h_inv, a.I, p.rows);
  if (a.down_type == DM_Q6_K) {
    auto fn = tc::tc_down_kernel<DM_Q6_K, NT>;
    ensure_smem_limit((const void *)fn);
    fn<<<dim3(a.H / 128, p.max_items), tc::kTcThreads, tc::Layout<2, NT>::kSmem, s>>>(
        p.h_map, a, g.down, g.sh_down, p.h_inv, p.rows);
  } else {
    auto fn = tc::tc_down_kernel<DM_Q5_0, NT>;
    ensure_smem_limit((const void *)fn);
    fn<<<dim3(a.H / 128, p.max_items), tc::kTcThreads, tc::Layout<1, NT>::kSmem, s>>>(
        p.h_map, a, g.down, g.sh_down, p.h_inv, p.rows);
  }
  return 4;
}

int launch_tc_experts(const ForwardArgs &a, const TcPlan &p, const GemvPlan &g, cudaStream_t s,
                      cudaEvent_t down_mark) {
  switch (p.nt) {
    case 16: return launch_nt<16>(a, p, g, s, down_mark);
    case 32: return launch_nt<32>(a, p, g, s, down_mark);
    case 64: return launch_nt<64>(a, p, g, s, down_mark);
    default: return -1;
  }
}

}  // namespace dm
