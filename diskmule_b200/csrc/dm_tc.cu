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
#include <cstdlib>
#include <cstring>

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

// One try_wait on the phase with parity `parity`; the warp may sleep in it (up to
// about a millisecond) until the phase completes instead of spinning.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(1000000u)
      : "memory");
  return done != 0;
}

// Wait for the phase with parity `parity` to complete; false after ~0.1 s.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const long long start = clock64();
  while (true) {
    if (mbar_try(bar, parity)) return true;
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

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4}], [%5];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
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
// dequantisation of one 256-wide K step of one weight row into tensor memory.
// A quant byte q (< 128) becomes f = 0.5 + q/256 exactly (PRMT into the mantissa of
// 0.5), so a value alpha*q + beta is fma(f, 256*alpha, beta - 128*alpha): one packed
// f32x2 fma per two weights, f32-accurate, then a single rounding to fp16. Two
// consecutive K values share one 32-bit TMEM column (lower K in the low half); the
// row is this thread's TMEM lane.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint4 lds16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds4(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds8(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint16_t lds2(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// 16 columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// four bytes (each below 128) -> two fp16-pair columns
__device__ __forceinline__ void deq4(uint32_t w, uint64_t M, uint64_t C, uint32_t *out) {
  out[0] = to_h2(fma2(magic2(w, 0), M, C));
  out[1] = to_h2(fma2(magic2(w, 2), M, C));
}

// Each K step of a row is split between two producer threads: half hf dequantises K
// values [128 hf, 128 hf + 128) of the step into 64 columns from tcol, reading the row's
// raw blocks from the step's shared-memory stage.

// Q4_K super-block (src/cpu.rs:585-616) at s: 16-byte header (d, dmin, 12 scale bytes),
// qs[128]. Half hf = group pairs 2hf, 2hf+1. Group pair gp: low nibbles of
// qs[32gp .. 32gp+32) are elements 64gp + i (sub-block 2gp), high nibbles elements
// 64gp + 32 + i (sub-block 2gp+1). value = d*(sc*q) - dmin*m, built in fp16 without
// the ALU pipe's byte shuffles:
//   one LOP3 turns the nibbles of bytes 0 and 2 (or 1 and 3) of a word into the fp16 pair
//   1024 + q (low nibble) or 1024 + 16q (high nibble), exact;
//   fma(1024 + q, sc, -1024 sc) (or fma(1024 + 16q, sc/16, -64 sc)) = sc*q exactly
//   (the product is exact inside the fma and sc*q <= 945 is an fp16 integer);
//   fma(sc*q, d, fp16(-dmin*m)) with d the block's own fp16 value: one rounding of the
//   product, the same as rounding the f32 value once to fp16, plus the rounding of the
//   small bias term.
// A column therefore holds K values (4j, 4j+2) or (4j+1, 4j+3) of a group of four; the
// activation tiles are packed in the same order (pack_kernel<true>).
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t h2dup(float v) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(h) : "f"(v));
  return h;
}

__device__ __forceinline__ void deq_q4k(uint32_t s, int hf, uint32_t tcol) {
  const uint4 hd = lds16(s);
  const uint32_t D = __byte_perm(hd.x, 0, 0x1010);  // (d, d) as fp16x2
  const float dmin = f16_bits_to_f32((uint16_t)(hd.x >> 16));
  // scale/min bytes of sub-blocks 4hf .. 4hf+3 (get_scale_min_k4)
  const uint32_t sc = hf ? ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u)) : (hd.y & 0x3F3F3F3Fu);
  const uint32_t mn = hf ? (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u))
                         : (hd.z & 0x3F3F3F3Fu);
#pragma unroll
  for (int g = 0; g < 2; g++) {
    const float scl = (float)((sc >> (16 * g)) & 0xff), sch = (float)((sc >> (16 * g + 8)) & 0xff);
    const float mnl = (float)((mn >> (16 * g)) & 0xff), mnh = (float)((mn >> (16 * g + 8)) & 0xff);
    const uint32_t SL = h2dup(scl), CL = h2dup(-1024.0f * scl);
    const uint32_t SH = h2dup(0.0625f * sch), CH = h2dup(-64.0f * sch);
    const uint32_t BL = h2dup(-(dmin * mnl)), BH = h2dup(-(dmin * mnh));  // dmin*m exact in f32
    const uint4 qa = lds16(s + 16 + 64 * hf + 32 * g), qb = lds16(s + 32 + 64 * hf + 32 * g);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint32_t lo[16], hi[16];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const uint32_t w8 = w[k] >> 8;
      lo[2 * k] = hfma2(hfma2((w[k] & 0x000F000Fu) | 0x64006400u, SL, CL), D, BL);
      lo[2 * k + 1] = hfma2(hfma2((w8 & 0x000F000Fu) | 0x64006400u, SL, CL), D, BL);
      hi[2 * k] = hfma2(hfma2((w[k] & 0x00F000F0u) | 0x64006400u, SH, CH), D, BH);
      hi[2 * k + 1] = hfma2(hfma2((w8 & 0x00F000F0u) | 0x64006400u, SH, CH), D, BH);
    }
    tmem_st16(tcol + 32 * g, lo);
    tmem_st16(tcol + 32 * g + 16, hi);
  }
}

// Q6_K super-block (src/cpu.rs:618-645), split layout at s: ql[128] qh[64] sc[16]; d
// given. Half h = hf (elements 128h + ...): quarter qq, index l < 32: element
// 128h + 32qq + l = low nibble (qq < 2) or high nibble of ql[64h + 32(qq&1) + l] | bits 2qq
// of qh[32h + l] << 4, scale sc[8h + l/16 + 2qq]. value = (d*sc)*(q-32) =
// fma(f, 256 s, -160 s).
__device__ __forceinline__ void deq_q6k(uint32_t s, int h, float d, uint32_t tcol) {
  const uint2 scw = lds8(s + 192 + 8 * h);
  const uint32_t sc[2] = {scw.x, scw.y};
  uint32_t ql[16], qh[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint4 v = lds16(s + 64 * h + 16 * i);
    ql[4 * i] = v.x, ql[4 * i + 1] = v.y, ql[4 * i + 2] = v.z, ql[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const uint4 v = lds16(s + 128 + 32 * h + 16 * i);
    qh[4 * i] = v.x, qh[4 * i + 1] = v.y, qh[4 * i + 2] = v.z, qh[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int qq = 0; qq < 4; qq++) {
    uint32_t out[16];
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int si = half + 2 * qq;
      const float sv = __fmul_rn(d, (float)(int8_t)((sc[si >> 2] >> (8 * (si & 3))) & 0xff));
      const uint64_t M = pair(256.0f * sv, 256.0f * sv), C = pair(-160.0f * sv, -160.0f * sv);
#pragma unroll
      for (int ii = 0; ii < 4; ii++) {
        const int i = 4 * half + ii;
        const uint32_t src = ql[8 * (qq & 1) + i];
        const uint32_t lo4 = (qq < 2 ? src : src >> 4) & 0x0F0F0F0Fu;
        const uint32_t hb = qq == 0 ? (qh[i] << 4) : qq == 1 ? (qh[i] << 2) : qq == 2 ? qh[i] : (qh[i] >> 2);
        deq4(lo4 | (hb & 0x30303030u), M, C, out + 2 * i);
      }
    }
    tmem_st16(tcol + 16 * qq, out);
  }
}

__device__ __forceinline__ uint32_t spread4(uint32_t v) {
  return ((v & 0xfu) * 0x02040810u) & 0x10101010u;
}

// nb (<= 4) Q5_0 blocks (src/cpu.rs:560-574): qs[16 nb] at sq, qh words at sh, f16 d at
// sd. Block b: elements 32b + j (j < 16) = low nibble of qs[j] | qh bit j << 4, elements
// 32b + 16 + j = high nibble | qh bit 16 + j << 4. value = d*(q-16) = fma(f, 256 d, -144 d).
// Columns 16b.
__device__ __forceinline__ void deq_q50(uint32_t sq, uint32_t sh, uint32_t sd, int nb,
                                        uint32_t tcol) {
#pragma unroll
  for (int b = 0; b < 4; b++) {
    if (b < nb) {
      const uint4 qs = lds16(sq + 16 * b);
      const uint32_t hb = lds4(sh + 4 * b);
      const uint32_t dw = lds4(sd + 4 * (b >> 1));
      const float d = f16_bits_to_f32((uint16_t)((b & 1) ? dw >> 16 : dw & 0xffff));
      const uint64_t M = pair(256.0f * d, 256.0f * d), C = pair(-144.0f * d, -144.0f * d);
      const uint32_t w[4] = {qs.x, qs.y, qs.z, qs.w};
      uint32_t out[16];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        deq4((w[i] & 0x0F0F0F0Fu) | spread4(hb >> (4 * i)), M, C, out + 2 * i);
        deq4(((w[i] >> 4) & 0x0F0F0F0Fu) | spread4(hb >> (16 + 4 * i)), M, C, out + 8 + 2 * i);
      }
      tmem_st16(tcol + 16 * b, out);
    }
  }
}

__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// nb (<= 4) Q5_0 blocks whose quants were widened at layer set-up to one byte per value,
// q5 = low nibble | high bit << 4 (src/cpu.rs:560-574), 32 bytes per block at sq; f16 d
// at sd. value = d*(q5 - 16): a PRMT puts two bytes under an f16 exponent (1024 + q5,
// exact), an f16x2 add of -1040 leaves q5 - 16 (exact), an f16x2 multiply by d rounds
// once -- the value deq_q50 rounds once from f32 -- in three instructions per two values
// instead of the bit assembly of the 5-bit layout. Columns 16b, natural K order.
__device__ __forceinline__ void deq_q50b(uint32_t sq, uint32_t sd, int nb, uint32_t tcol) {
  constexpr uint32_t kMinus1040 = 0xE410E410u;  // (-1040, -1040) as f16x2
#pragma unroll
  for (int b = 0; b < 4; b++) {
    if (b < nb) {
      const uint4 u0 = lds16(sq + 32 * b), u1 = lds16(sq + 32 * b + 16);
      const uint32_t dw = lds4(sd + 4 * (b >> 1));
      const uint32_t dh = (b & 1) ? dw >> 16 : dw & 0xffffu;
      const uint32_t D = dh | (dh << 16);
      const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint32_t out[16];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        out[2 * i] = hmul2(hadd2(__byte_perm(w[i], 0x64646464u, 0x4140u), kMinus1040), D);
        out[2 * i + 1] = hmul2(hadd2(__byte_perm(w[i], 0x64646464u, 0x4342u), kMinus1040), D);
      }
      tmem_st16(tcol + 16 * b, out);
    }
  }
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
  // capped at 2^126 so that the scale and its inverse stay finite for rows below 2^-113
  return exp2f((float)min(13 - ilogbf(m), 126));
}

// GLM's silu(g) * u with the hardware exponential and a fast divide: the CUDA-core
// activations above evaluate exp in double for the reference's exact rounding, which the
// intermediate h, rounded to fp16 right after, does not need (|error| ~1e-6 relative against
// fp16's 5e-4). Used where the epilogue of a tensor-core product applies the activation:
// four warps per SM there, so latency, not throughput, bounds it.
__device__ __forceinline__ float glm_silu_mul_fast(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__device__ __forceinline__ float activate(const ForwardArgs &a, int expert, float g, float u) {
  if (a.family == kGemma) return __fmul_rn(gelu_tanh(g), u);
  if (a.family == kQwen) return __fmul_rn(qwen_silu(g), u);
  if (expert == a.E) return __fmul_rn(glm_silu(g), u);
  return __fmul_rn(glm_cached_silu(g), u);
}

constexpr int kMaxPackI = 2048;  // intermediate rows staged in shared memory by pack_kernel

// Sorted row `pos` -> hi = fp16(x*s) and lo = fp16(x*s - hi), x*s = hi + lo to about
// 2^-22 relative. With `split` the two halves are rows 2 pos and 2 pos + 1 (one tile of
// 2 NT rows then feeds both halves to a single MMA); without it row pos holds hi alone.
// INPUT: x is the expert input row. Otherwise x = act(gate, up) of the row's gate/up
// outputs gu[pos][2i] (gate) and gu[pos][2i + 1] (up), i < K.
// One warp per row (8 rows per CTA): lane l takes the 16-byte pieces l, l + 32, ...;
// the row maximum is a shuffle reduction; an input row is read twice (L2), an
// intermediate row is activated once into the warp's shared-memory row.
constexpr int kPackRows = 8;

template <bool INPUT>
__global__ void __launch_bounds__(32 * kPackRows) pack_kernel(ForwardArgs a, const float *gu,
                                                             __half *out, float *inv, int K,
                                                             int split) {
  extern __shared__ __align__(16) float hrows[];  // [kPackRows][K] (intermediates only)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = blockIdx.x * kPackRows + warp;
  if (pos >= a.offsets[a.E + 1]) return;
  const float *src;
  const int P = a.T * a.k, pr = a.sorted[pos];
  const int k4 = K / 4;
  if (INPUT) {
    const int tok = pr < P ? pr / a.k : pr - P;
    src = (a.family == kGemma ? a.expert_in : reinterpret_cast<const float *>(a.x)) +
          (size_t)tok * K;
  } else {
    const int e = pr < P ? (int)a.sel_idx[pr] : a.E;
    const float *row = gu + (size_t)pos * 2 * K;
    float *h = hrows + (size_t)warp * K;
#pragma unroll 4
    for (int q = lane; q < k4; q += 32) {
      const float4 g0 = *reinterpret_cast<const float4 *>(row + 8 * q);
      const float4 g1 = *reinterpret_cast<const float4 *>(row + 8 * q + 4);
      *reinterpret_cast<float4 *>(h + 4 * q) =
          make_float4(activate(a, e, g0.x, g0.y), activate(a, e, g0.z, g0.w),
                      activate(a, e, g1.x, g1.y), activate(a, e, g1.z, g1.w));
    }
    __syncwarp();
    src = h;
  }
  // (loops unrolled so that each lane has several 16-byte loads in flight: an input row
  // comes from L2, one latency per batch instead of per piece)
  float m = 0.0f;
#pragma unroll 8
  for (int q = lane; q < k4; q += 32) {
    const float4 v = *reinterpret_cast<const float4 *>(src + 4 * q);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s = pow2_scale(m);
  // expert inputs feed the Q4_K gate/up tiles, whose columns pair K values (0, 2) and
  // (1, 3) of each group of four (deq_q4k): the same order here
  const int a1 = INPUT ? 2 : 1, a2 = INPUT ? 1 : 2;
  const size_t orow = split ? 2 * (size_t)pos : (size_t)pos;
#pragma unroll 4
  for (int q = lane; q < k4; q += 32) {
    const float4 v = *reinterpret_cast<const float4 *>(src + 4 * q);
    const float xs[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
    __half hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      hi[j] = __float2half_rn(xs[j]);
      lo[j] = __float2half_rn(xs[j] - __half2float(hi[j]));
    }
    *reinterpret_cast<uint2 *>(out + orow * K + 4 * q) =
        make_uint2(h2u(__halves2half2(hi[0], hi[a1])), h2u(__halves2half2(hi[a2], hi[3])));
    if (split)
      *reinterpret_cast<uint2 *>(out + (orow + 1) * K + 4 * q) =
          make_uint2(h2u(__halves2half2(lo[0], lo[a1])), h2u(__halves2half2(lo[a2], lo[3])));
  }
  if (lane == 0) inv[pos] = 1.0f / s;
}

// ---------------------------------------------------------------------------
// persistent grouped expert GEMM
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool aborted(const int *abort_flag) {
  return *reinterpret_cast<const volatile int *>(abort_flag) != 0;
}

// Bounded wait that also gives up once another thread of the CTA has aborted. The abort
// flag and the clock are checked every 8 tries, so a spinning warp issues few
// instructions besides the try itself (the producers share the issue slots); SLEEP_NS > 0
// backs off between tries, for waits that have slack (the epilogue's accumulator wait,
// the TMA warps' free-slot waits).
template <int SLEEP_NS = 0>
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, const int *abort_flag) {
  const long long start = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; i++) {
      if (mbar_try(bar, parity)) return true;
      if (SLEEP_NS > 0) __nanosleep(SLEEP_NS);
    }
    if (*reinterpret_cast<const volatile int *>(abort_flag)) return false;
    if (clock64() - start > kWaitCycles) return false;
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, fp16 inputs, f32 accumulate; A row m is TMEM lane m.
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp roles: 0..3 epilogue (TMEM lane quarter = warp); 4..19 producers, two groups of
// eight (group g dequantises the steps t = g mod 2; in a group, warp 4 + 8g + 4hf + q
// covers lanes 32q.. and half hf of the K step); 20 TMA of the activation tiles; 21 TMA
// of the raw weight tiles; 22..25 MMA issue (one tcgen05.mma issuer is latency-bound at
// ~45 cycles per instruction in isolation and ~120 beside busy producer warps; up to four
// issuers, one per SM sub-partition, each into its own accumulator, raise the rate; the
// epilogue adds their partial sums in issuer order, so results stay deterministic).
constexpr int kEpilogueWarps = 4;
constexpr int kProducerWarps = 16;
constexpr int kTmaWarp = kEpilogueWarps + kProducerWarps;  // 20
constexpr int kRawWarp = kTmaWarp + 1;                     // 21
constexpr int kMmaWarp = kRawWarp + 1;                     // 22 .. 25
constexpr int kMaxIssuers = 4;
constexpr int kTcThreads = (kMmaWarp + kMaxIssuers) * 32;  // 832
constexpr int kStepK = 256;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in per block
constexpr int kBarBytes = 512;
constexpr int kMaxRaw = 8;          // raw stages

enum TcKind { kUpQ4K = 0, kDownQ6K = 1, kDownQ50 = 2 };

// Raw stage of one K step, 128 weight rows, filled by TMA:
//   Q4_K: row r (gate/up interleaved) at 144 r: one super-block;
//   Q6_K: row r at 208 r: ql qh sc of one super-block; then the 128 f16 d;
//   Q5_0: row r at 272 r: the 256 quant bytes (one per value, widened at set-up) of 8
//         blocks (+16 bytes of the next step, unused); then d[128][8 f16].
// Row strides are odd multiples of 16 bytes, so a warp's 16-byte loads of 32 rows are
// free of bank conflicts.
template <int KIND>
struct RawTile {
  static constexpr int kRowBytes = KIND == kDownQ6K ? 208 : KIND == kDownQ50 ? 272 : 144;
  static constexpr int kQuant = 128 * kRowBytes;
  static constexpr int kSide = KIND == kDownQ6K ? 256 : KIND == kDownQ50 ? 128 * 16 : 0;
  static constexpr int kBytes = kQuant + kSide;
  static constexpr int kStage = (kBytes + 1023) / 1024 * 1024;
};

// Tile of NT tokens: B rows NB = NT, or 2 NT with the hi + lo split (interleaved), so
// one MMA of N = NB covers both halves (an M=128, K=16 MMA costs the same for N <= 64).
// TMEM (512 columns): NA A buffers of 128 columns, then 2 (double buffer) x NI (issuers)
// accumulators of NB columns.
template <int KIND, int NT, bool SPLIT>
struct Cfg {
  static constexpr int NB = SPLIT ? 2 * NT : NT;
  // Tensor memory (512 columns): NA A stages of 128 columns, then AB accumulator buffers
  // of NI issuers x NB columns. Four issuers (one per SM sub-partition) when their
  // accumulators fit beside three A stages, single-buffered if need be (the epilogue
  // then reads all partial sums before it stores); otherwise two or one, double-buffered.
  // The down products (K = I: two or three K steps per unit) use two issuers with
  // double-buffered accumulators at NB = 32 instead: a unit boundary every few steps costs
  // more than the slower issue (measured on the Qwen shape: 189 -> 178 us).
  static constexpr bool kShortK = KIND != kUpQ4K && NB == 32;
  static constexpr int NI4_AB =
      kShortK ? 0 : (3 * 128 + 2 * 4 * NB <= 512 ? 2 : (3 * 128 + 4 * NB <= 512 ? 1 : 0));
  static constexpr int NA = kShortK ? 3 : (NI4_AB ? 3 : (3 * 128 + 4 * NB <= 512 ? 3 : 2));
  static constexpr int NI = kShortK ? 2 : (NI4_AB ? 4 : (NA * 128 + 4 * NB <= 512 ? 2 : 1));
  static constexpr int AB = kShortK ? 2 : (NI4_AB ? NI4_AB : 2);
  static_assert(NB % 16 == 0 && NA * 128 + AB * NI * NB <= 512, "tensor memory layout");
  static constexpr int kAccCol = NA * 128;
  static constexpr int kBStage = (kStepK / 64) * NB * 128;  // 4 swizzle atoms of NB rows
  static constexpr int kFixed = 1024 + NA * kBStage + kBarBytes;
  static constexpr int kRSfit = (kSmemLimit - kFixed) / RawTile<KIND>::kStage;
  static constexpr int kRS = kRSfit < kMaxRaw ? kRSfit : kMaxRaw;  // raw stages
  static constexpr int kSmem = kFixed + kRS * RawTile<KIND>::kStage;
  static constexpr bool kFits = kRS >= 3;
};

// Stage i: afull (A written: one arrival per producer warp of the group), bfull (B tile
// landed: TMA bytes), empty (the stage's MMAs are done: one commit per issuer); raw
// stage j: rawfull (TMA bytes), rawempty (one arrival per producer warp that read it).
struct Bars {
  uint32_t base;
  __device__ __forceinline__ uint32_t afull(int i) const { return base + 8u * i; }
  __device__ __forceinline__ uint32_t bfull(int i) const { return base + 8u * (3 + i); }
  __device__ __forceinline__ uint32_t empty(int i) const { return base + 8u * (6 + i); }
  __device__ __forceinline__ uint32_t accfull(int i) const { return base + 8u * (9 + i); }
  __device__ __forceinline__ uint32_t accempty(int i) const { return base + 8u * (11 + i); }
  __device__ __forceinline__ uint32_t drain() const { return base + 8u * 13; }
  __device__ __forceinline__ uint32_t rawfull(int i) const { return base + 8u * (14 + i); }
  __device__ __forceinline__ uint32_t rawempty(int i) const { return base + 8u * (14 + kMaxRaw + i); }
  __device__ __forceinline__ uint32_t slot() const { return base + 8u * (14 + 2 * kMaxRaw); }
};

// One issuer's MMAs of one K step: slices s = I, I + NI, ... (all 16 on the fast path).
// desc(addr + off) = desc(addr) + off / 16 while addresses stay below 256 KB.
template <int NB, int NI, int I>
__device__ __forceinline__ void issue_step(uint32_t dcol, uint32_t acol, uint32_t bst, int slices,
                                           bool first) {
  constexpr uint32_t idesc = idesc_f16(NB);
  const uint64_t b0 = sw128_desc(bst);
  if (slices == kStepK / 16) {
#pragma unroll
    for (int s = I; s < kStepK / 16; s += NI) {
      const uint32_t boff = (uint32_t)(s >> 2) * (NB * 128u) + (uint32_t)(s & 3) * 32u;
      mma_ts(dcol, acol + 8u * s, b0 + (boff >> 4), idesc, (first && s == I) ? 0u : 1u);
    }
  } else {
#pragma unroll
    for (int s = I; s < kStepK / 16; s += NI) {
      if (s < slices) {
        const uint32_t boff = (uint32_t)(s >> 2) * (NB * 128u) + (uint32_t)(s & 3) * 32u;
        mma_ts(dcol, acol + 8u * s, b0 + (boff >> 4), idesc, (first && s == I) ? 0u : 1u);
      }
    }
  }
}

struct Unit {
  int e, pos0, ntok, tile;
};

__device__ __forceinline__ Unit make_unit(int4 rec, int u, int n_tiles) {
  Unit r;
  r.e = rec.x;
  r.pos0 = rec.z;
  r.ntok = rec.w;
  r.tile = u % n_tiles;
  return r;
}

// Unit records of one CTA's units in order: the record of unit lu + 1 is loaded when
// unit lu is first asked for, so its latency hides behind a unit of work.
struct UnitWalk {
  const int4 *items;
  int first, stride, n_tiles, count;
  int lu = -1;
  Unit cur;
  int4 next;
  __device__ __forceinline__ int4 load(int l) const {
    return l < count ? items[(first + l * stride) / n_tiles] : make_int4(0, 0, 0, 0);
  }
  __device__ __forceinline__ const Unit &at(int l) {
    if (l != lu) {
      const int4 rec = (lu >= 0 && l == lu + 1) ? next : load(l);
      cur = make_unit(rec, first + l * stride, n_tiles);
      lu = l;
      next = load(l + 1);
    }
    return cur;
  }
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4, %5}], [%6];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

template <int KIND, int NT, bool SPLIT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_kernel(
    const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap wmap,
    const __grid_constant__ CUtensorMap sh_wmap, ForwardArgs a, TcSide side, const float *b_inv,
    float *gu) {
  using C = Cfg<KIND, NT, SPLIT>;
  using RT = RawTile<KIND>;
  constexpr int NB = C::NB, NA = C::NA, NI = C::NI, RS = C::kRS;
  extern __shared__ uint8_t dsm[];
  __shared__ int abort_flag;
  const int K = KIND == kUpQ4K ? a.H : a.I;
  const int n_tiles = KIND == kUpQ4K ? a.I / 64 : a.H / 128;
  const int n_units = *a.n_items * n_tiles;
  if ((int)blockIdx.x >= n_units) return;
  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nsteps = (K + kStepK - 1) / kStepK;
  const int total = my_units * nsteps;

  const uint32_t raw = smem_u32(dsm);
  const uint32_t b_base = (raw + 1023u) & ~1023u;
  const uint32_t w_base = b_base + NA * C::kBStage;
  const Bars bars{w_base + RS * RT::kStage};
  uint8_t *generic = dsm + (bars.slot() - raw);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    abort_flag = *reinterpret_cast<const volatile int32_t *>(a.status) == kStatusTimeout;
    for (int i = 0; i < 3; i++) {
      mbar_init(bars.afull(i), kProducerWarps / 2);
      mbar_init(bars.bfull(i), 1);
      mbar_init(bars.empty(i), NI);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(bars.accfull(i), NI);
      mbar_init(bars.accempty(i), kEpilogueWarps);
    }
    mbar_init(bars.drain(), NI);
    for (int i = 0; i < kMaxRaw; i++) {
      mbar_init(bars.rawfull(i), 1);
      mbar_init(bars.rawempty(i), kProducerWarps / 2);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(bars.slot(), 512);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(generic);
  const uint32_t unit_stride = gridDim.x;

  if (warp >= kEpilogueWarps && warp < kTmaWarp) {
    // ---- producers ----
    const int pw = warp - kEpilogueWarps;  // 0..15
    const int g = pw >> 3, hf = (pw >> 2) & 1, q = warp & 3, r = 32 * q + lane;
    for (int t = g; t < total; t += 2) {
      const int rs = t % RS, ab = t % NA;
      bool ok = wait_or_abort(bars.rawfull(rs), (uint32_t)((t / RS) & 1), &abort_flag);
      ok = ok && (t < NA || wait_or_abort(bars.empty(ab), (uint32_t)((t / NA - 1) & 1), &abort_flag));
      ok = ok && !aborted(&abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicExch(&abort_flag, 1);
        break;
      }
      fence_after();
      const uint32_t st = w_base + (uint32_t)rs * RT::kStage;
      const uint32_t tcol = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)ab * 128u + 64u * hf;
      const int ks = t % nsteps;
      if (KIND == kUpQ4K) {
        deq_q4k(st + r * 144u, hf, tcol);
      } else if (KIND == kDownQ6K) {
        const float d = f16_bits_to_f32(lds2(st + RT::kQuant + 2u * r));
        deq_q6k(st + r * 208u, hf, d, tcol);
      } else {
        const uint32_t sq = st + r * 272u + 128u * hf;
        const uint32_t sd = st + RT::kQuant + r * 16u + 8u * hf;
        deq_q50b(sq, sd, min(4, (K - kStepK * ks) / 32 - 4 * hf), tcol);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.rawempty(rs));  // this warp's reads of the stage are done
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.afull(ab));
    }
  } else if (warp == kTmaWarp || warp == kRawWarp) {
    // ---- TMA: activation tiles (warp 20) and raw weight tiles (warp 21) ----
    if (lane == 0) {
      const bool is_b = warp == kTmaWarp;
      const int depth = is_b ? NA : RS;
      int t = 0;
      bool stop = false;
      UnitWalk walk{a.items, (int)blockIdx.x, (int)unit_stride, n_tiles, my_units};
      for (int lu = 0; lu < my_units && !stop; lu++) {
        const Unit un = walk.at(lu);
        // another CTA's timeout stops this one too (checked once per unit)
        if (*reinterpret_cast<const volatile int32_t *>(a.status) == kStatusTimeout)
          atomicExch(&abort_flag, 1);
        const bool shared = un.e == a.E;
        for (int ks = 0; ks < nsteps; ks++, t++) {
          const int i = t % depth;
          const uint32_t free_bar = is_b ? bars.empty(i) : bars.rawempty(i);
          if ((t >= depth && !wait_or_abort<64>(free_bar, (uint32_t)((t / depth - 1) & 1), &abort_flag)) ||
              aborted(&abort_flag)) {
            atomicExch(&abort_flag, 1);
            stop = true;
            break;
          }
          if (is_b) {
            // one box of 4 atoms x NB rows (atoms past K read as zeros, unused)
            mbar_expect_tx(bars.bfull(i), (uint32_t)C::kBStage);
            tma_load_3d(b_base + (uint32_t)i * C::kBStage, &bmap, 0, SPLIT ? 2 * un.pos0 : un.pos0,
                        (kStepK / 64) * ks, bars.bfull(i));
          } else {
            const uint32_t dst = w_base + (uint32_t)i * RT::kStage, bar = bars.rawfull(i);
            const CUtensorMap *map = shared ? &sh_wmap : &wmap;
            const int ex = shared ? 0 : un.e;
            mbar_expect_tx(bar, (uint32_t)RT::kBytes);
            if (KIND == kUpQ4K) {
              tma_load_4d(dst, map, 144 * ks, 0, un.tile * 64, ex, bar);
            } else {
              const int row0 = ex * a.H + un.tile * 128;
              // x: Q6_K in bytes; Q5_0 in 2-byte elements (a 136-element box is its 272 bytes)
              tma_load_2d(dst, map, KIND == kDownQ6K ? 208 * ks : 128 * ks, row0, bar);
              const size_t side_row = ((size_t)ex * nsteps + ks) * a.H + un.tile * 128;
              if (KIND == kDownQ6K) {
                bulk_load(dst + RT::kQuant, (shared ? side.sh_d_t : side.d_t) + side_row * 2, 256, bar);
              } else {
                bulk_load(dst + RT::kQuant, (shared ? side.sh_d_t : side.d_t) + side_row * 16,
                          128 * 16, bar);
              }
            }
          }
        }
      }
      // every armed stage has landed before the CTA may exit
      for (int i = max(0, t - depth); i < t; i++)
        mbar_wait(is_b ? bars.bfull(i % depth) : bars.rawfull(i % depth), (uint32_t)((i / depth) & 1));
    }
  } else if (warp >= kMmaWarp) {
    // ---- MMA issue: issuer i takes the K slices s = i mod NI into its own accumulator ----
    const int issuer = warp - kMmaWarp;
    if (lane == 0 && issuer < NI) {
      int t = 0;
      bool stop = false;
      for (int lu = 0; lu < my_units && !stop; lu++) {
        const int acc = lu % C::AB;
        if (lu >= C::AB &&
            !wait_or_abort(bars.accempty(acc), (uint32_t)((lu / C::AB - 1) & 1), &abort_flag)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        fence_after();
        const uint32_t dcol = tmem + C::kAccCol + (uint32_t)((acc * NI + issuer) * NB);
        for (int ks = 0; ks < nsteps; ks++, t++) {
          const int ab = t % NA;
          if (!wait_or_abort(bars.afull(ab), (uint32_t)((t / NA) & 1), &abort_flag) ||
              !wait_or_abort(bars.bfull(ab), (uint32_t)((t / NA) & 1), &abort_flag)) {
            atomicExch(&abort_flag, 1);
            stop = true;
            break;
          }
          fence_after();
          const int slices = min(kStepK, K - kStepK * ks) / 16;
          const uint32_t acol = tmem + (uint32_t)ab * 128u;
          const uint32_t bst = b_base + (uint32_t)ab * C::kBStage;
          switch (issuer) {
            case 0: issue_step<NB, NI, 0>(dcol, acol, bst, slices, ks == 0); break;
            case 1: issue_step<NB, NI, 1 % NI>(dcol, acol, bst, slices, ks == 0); break;
            case 2: issue_step<NB, NI, 2 % NI>(dcol, acol, bst, slices, ks == 0); break;
            default: issue_step<NB, NI, 3 % NI>(dcol, acol, bst, slices, ks == 0); break;
          }
          mma_commit(bars.empty(ab));
        }
        if (!stop) mma_commit(bars.accfull(acc));
      }
      mma_commit(bars.drain());
      if (!mbar_wait(bars.drain(), 0)) atomicExch(&abort_flag, 1);
    }
  } else {
    // ---- epilogue: warp q owns TMEM lanes 32q..32q+31 ----
    const int q = warp, r = 32 * q + lane;
    UnitWalk walk{a.items, (int)blockIdx.x, (int)unit_stride, n_tiles, my_units};
    for (int lu = 0; lu < my_units; lu++) {
      const int acc = lu % C::AB;
      const Unit un = walk.at(lu);
      // the unit's row scales, one token per lane (loaded before the wait)
      const float inv_a = lane < un.ntok ? b_inv[un.pos0 + lane] : 0.0f;
      const float inv_b = NT > 32 && lane + 32 < un.ntok ? b_inv[un.pos0 + 32 + lane] : 0.0f;
      const bool ok = wait_or_abort<128>(bars.accfull(acc), (uint32_t)((lu / C::AB) & 1), &abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicExch(&abort_flag, 1);
        break;
      }
      fence_after();
      // column n of each issuer's accumulator: token n (or, with the split, hi of token
      // n/2 at even n and lo at odd n); the issuers' partial sums are added in order
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + C::kAccCol + (uint32_t)(acc * NI * NB);
      // columns per chunk and issuer (a tcgen05.ld here moves 16 columns)
      constexpr int CW = NB < 16 ? NB : (32 / NI < 16 ? 16 : 32 / NI);
      constexpr int TPC = SPLIT ? CW / 2 : CW;         // tokens per chunk
      // gate/up rows: A rows 2i and 2i+1 hold index 0 and 1 of the gate|up axis
      const bool swapped = un.e == a.E ? side.sh_up_swapped : side.up_swapped;
      float *out = KIND == kUpQ4K ? gu : a.ysorted;
      const int ld = KIND == kUpQ4K ? 2 * a.I : a.H;
      const int col = KIND == kUpQ4K ? un.tile * 128 + (r ^ (swapped ? 1 : 0)) : un.tile * 128 + r;
      if constexpr (C::AB == 1) {
        // single accumulator buffer: add the issuers' partial sums (in issuer order) into
        // registers, free the accumulators for the next unit, then store
        float v[NB];
#pragma unroll
        for (int i = 0; i < NI; i++) {
#pragma unroll
          for (int c0 = 0; c0 < NB; c0 += 16) {
            float w[16];
            tmem_ld16(taddr + i * NB + c0, reinterpret_cast<uint32_t *>(w));
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; c++) v[c0 + c] = i == 0 ? w[c] : v[c0 + c] + w[c];
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bars.accempty(acc));
#pragma unroll
        for (int j = 0; j < (SPLIT ? NB / 2 : NB); j++) {
          const float val = SPLIT ? v[2 * j] + v[2 * j + 1] : v[j];
          const float inv = __shfl_sync(0xffffffffu, j < 32 ? inv_a : inv_b, j & 31);
          if (j < un.ntok) out[(size_t)(un.pos0 + j) * ld + col] = val * inv;
        }
        continue;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < NB; c0 += CW) {
        float w[NI][CW];
#pragma unroll
        for (int i = 0; i < NI; i++)
#pragma unroll
          for (int c = 0; c < CW; c += 16)
            tmem_ld16(taddr + i * NB + c0 + c, reinterpret_cast<uint32_t *>(&w[i][c]));
        tmem_wait_ld();
        if (c0 + CW >= NB) {  // the accumulators are free for the unit after next
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bars.accempty(acc));
        }
        float v[CW];
#pragma unroll
        for (int c = 0; c < CW; c++) {
          v[c] = w[0][c];
#pragma unroll
          for (int i = 1; i < NI; i++) v[c] += w[i][c];
        }
        const int nbase = SPLIT ? c0 / 2 : c0;
        // up: gate of i at gu column 2i, up at 2i + 1 (a warp writes 128 contiguous bytes)
#pragma unroll
        for (int j = 0; j < TPC; j++) {
          const float val = SPLIT ? v[2 * j] + v[2 * j + 1] : v[j];
          const int n = nbase + j;
          const float inv = __shfl_sync(0xffffffffu, n < 32 ? inv_a : inv_b, n & 31);
          if (n < un.ntok) out[(size_t)(un.pos0 + n) * ld + col] = val * inv;
        }
      }
    }
  }

  __syncthreads();
  if (tid == 0 && abort_flag) atomicExch(a.status, kStatusTimeout);
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per-step transposes of the down side arrays: Q6_K d -> [expert][step][row] f16;
// Q5_0: quants widened to one byte per value, q5 = low nibble | high bit << 4, at
// qh_t [expert][row][I]; d -> [expert][step][row][8 f16] (zero past the last block of a
// ragged step).
__global__ void side_transpose_kernel(int kind, SplitTensor src, int experts, int H, int I,
                                      uint8_t *qh_t, uint8_t *d_t) {
  const int nsteps = (I + kStepK - 1) / kStepK;
  const size_t n = (size_t)experts * nsteps * H;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx % H);
    const int ks = (int)((idx / H) % nsteps);
    const size_t e = idx / ((size_t)H * nsteps);
    const size_t grow = e * H + row;
    if (kind == DM_Q6_K) {
      reinterpret_cast<uint16_t *>(d_t)[idx] = src.d[grow * (I / 256) + ks];
    } else {
      const int nbr = I / 32;
      for (int b = 0; b < 8; b++) {
        const int blk = 8 * ks + b;
        const bool in = blk < nbr;
        reinterpret_cast<uint16_t *>(d_t)[idx * 8 + b] = in ? src.d[grow * nbr + blk] : (uint16_t)0;
        if (!in) continue;
        const uint8_t *qs = src.quant + (grow * nbr + blk) * 16;
        const uint32_t qh = *reinterpret_cast<const uint32_t *>(src.qh + (grow * nbr + blk) * 4);
        uint8_t *q5 = qh_t + grow * I + 32 * blk;
        for (int j = 0; j < 16; j++) {
          q5[j] = (uint8_t)((qs[j] & 0x0F) | (((qh >> j) & 1u) << 4));
          q5[16 + j] = (uint8_t)((qs[j] >> 4) | (((qh >> (16 + j)) & 1u) << 4));
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// bf16 grouped GEMM (GLM): the weights need no dequantisation, so A (128 weight rows x
// 64 K, 128-byte swizzle) and B (the tile's tokens) both come by TMA into shared memory
// and one thread issues tcgen05.mma (kind::f16 with bf16 operands, f32 accumulate).
// Products of bf16 values are exact in f32, so only the summation order differs from
// the reference's sequential w*x sum.
//   warps 0..3 epilogue, warp 4 TMA, warp 5 MMA issue.
// ---------------------------------------------------------------------------

// L2 eviction policies for TMA loads. In the CTA-pair gate/up kernel the token tiles are
// read again by every weight tile of their item, so they load as evict-last and the
// weight stream (normal priority: an expert's second work item runs at the same time and
// reads the same weight tiles) does not push them out between those reads (measured at
// config 4: 17.8 -> 16.6 GB of DRAM reads; evict-first weights raised it to 21.5 GB).
__device__ __forceinline__ uint64_t l2_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t dst, const CUtensorMap *map, int c0,
                                                      int c1, uint32_t bar_cluster, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar_cluster), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair_hint(uint32_t dst, const CUtensorMap *map, int c0,
                                                      int c1, int c2, int c3, uint32_t bar_cluster,
                                                      uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar_cluster), "l"(pol)
      : "memory");
}

constexpr int kBfThreads = 6 * 32;
constexpr int kBfStepK = 64;

template <int NB>
struct BfCfg {
  static constexpr int kA = 128 * 128;        // 128 rows x 64 bf16
  static constexpr int kB = NB * 128;         // NB rows x 64 bf16
  static constexpr int kStage = kA + kB;
  static constexpr int kStages = (kSmemLimit - 1024 - 256) / kStage < 6 ? (kSmemLimit - 1024 - 256) / kStage : 6;
  static constexpr int kSmem = 1024 + kStages * kStage + 256;
};

__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// UP: gate/up rows (64 gate + 64 up interleaved), K = H, output gu; else down rows, K = I,
// output ysorted. SPLIT: B rows are hi/lo pairs (2 per token). HALVES = 2: a work item
// holds up to 2 x TPT tokens and each (item, row tile) is two units of TPT tokens; a unit
// without tokens is skipped by every warp role alike, and the accumulator buffers and
// barrier phases follow the count of units actually run.
// F16 (down only): A = fp16 copies of the down weights, B = single fp16 intermediate rows
// scaled by a power of two per row (row_inv = 1 / scale, applied in the epilogue).
template <bool UP, int NB, bool SPLIT, int HALVES, bool F16 = false>
__global__ void __launch_bounds__(kBfThreads, 1) tc_bf16_kernel(
    const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap wmap,
    const __grid_constant__ CUtensorMap sh_wmap, ForwardArgs a, TcSide side, float *gu,
    const float *row_inv) {
  using C = BfCfg<NB>;
  constexpr int S = C::kStages;
  constexpr int TPT = SPLIT ? NB / 2 : NB;  // tokens per tile
  extern __shared__ uint8_t dsm[];
  __shared__ int abort_flag;
  const int K = UP ? a.H : a.I;
  const int n_tiles = UP ? a.I / 64 : a.H / 128;
  const int n_units = *a.n_items * n_tiles * HALVES;
  if ((int)blockIdx.x >= n_units) return;
  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nsteps = K / kBfStepK;
  // the record of the unit after this one is requested while this one runs
  int4 rec_next = make_int4(0, 0, 0, 0);
  int item_next = -1;
  auto unit_at = [&](int lu) {
    const int u = (int)blockIdx.x + lu * (int)gridDim.x;
    const int item = u / (n_tiles * HALVES), rem = u - item * (n_tiles * HALVES);
    const int half = rem / n_tiles;  // every tile of the first half, then of the second
    const int4 rec = item == item_next ? rec_next : a.items[item];
    const int un_next = u + (int)gridDim.x;
    if (un_next < n_units) {
      item_next = un_next / (n_tiles * HALVES);
      rec_next = a.items[item_next];
    }
    Unit un;
    un.e = rec.x;
    un.tile = rem - half * n_tiles;
    un.pos0 = rec.z + half * TPT;
    un.ntok = min(TPT, rec.w - half * TPT);
    return un;
  };

  const uint32_t raw = smem_u32(dsm);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + S * C::kStage;  // full[S], empty[S], accfull[2], accempty[2], slot
  auto full = [&](int i) { return bars + 8u * i; };
  auto empty = [&](int i) { return bars + 8u * (S + i); };
  auto accfull = [&](int i) { return bars + 8u * (2 * S + i); };
  auto accempty = [&](int i) { return bars + 8u * (2 * S + 2 + i); };
  const uint32_t slot = bars + 8u * (2 * S + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    abort_flag = *reinterpret_cast<const volatile int32_t *>(a.status) == kStatusTimeout;
    for (int i = 0; i < S; i++) {
      mbar_init(full(i), 1);
      mbar_init(empty(i), 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(accfull(i), 1);
      mbar_init(accempty(i), 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  constexpr uint32_t kCols = 2 * NB <= 32 ? 32 : 2 * NB;  // power of two: 2 accumulators
  if (warp == 0) tmem_alloc(slot, kCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(dsm + (slot - raw));

  if (warp == 4) {
    if (lane == 0) {
      int t = 0;
      bool stop = false;
      for (int lu = 0; lu < my_units && !stop; lu++) {
        const Unit un = unit_at(lu);
        if (un.ntok <= 0) continue;
        if (*reinterpret_cast<const volatile int32_t *>(a.status) == kStatusTimeout)
          atomicExch(&abort_flag, 1);
        const bool shared = un.e == a.E;
        const int ex = shared ? 0 : un.e;
        for (int ks = 0; ks < nsteps; ks++, t++) {
          const int i = t % S;
          if ((t >= S && !wait_or_abort<64>(empty(i), (uint32_t)((t / S - 1) & 1), &abort_flag)) ||
              aborted(&abort_flag)) {
            atomicExch(&abort_flag, 1);
            stop = true;
            break;
          }
          const uint32_t st = base + (uint32_t)i * C::kStage;
          mbar_expect_tx(full(i), (uint32_t)C::kStage);
          if (UP)
            tma_load_4d(st, shared ? &sh_wmap : &wmap, kBfStepK * ks, 0, un.tile * 64, ex, full(i));
          else
            tma_load_2d(st, shared ? &sh_wmap : &wmap, kBfStepK * ks, ex * a.H + un.tile * 128, full(i));
          tma_load_2d(st + C::kA, &bmap, kBfStepK * ks, SPLIT ? 2 * un.pos0 : un.pos0, full(i));
        }
      }
      for (int i = max(0, t - S); i < t; i++) mbar_wait(full(i % S), (uint32_t)((i / S) & 1));
    }
  } else if (warp == 5) {
    if (lane == 0) {
      int t = 0, pu = 0;
      bool stop = false;
      for (int lu = 0; lu < my_units && !stop; lu++) {
        const Unit un = unit_at(lu);
        if (un.ntok <= 0) continue;
        const int acc = pu & 1;
        if (pu >= 2 && !wait_or_abort(accempty(acc), (uint32_t)(((pu >> 1) - 1) & 1), &abort_flag)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        pu++;
        fence_after();
        // N sized to the unit's tokens (a multiple of 16): ragged tiles cost less
        const int rows = SPLIT ? 2 * un.ntok : un.ntok;
        const int n = min(NB, (rows + 15) & ~15);
        const uint32_t idesc = F16 ? idesc_f16(n) : idesc_bf16(n);
        const uint32_t dcol = tmem + (uint32_t)(acc * NB);
        for (int ks = 0; ks < nsteps; ks++, t++) {
          const int i = t % S;
          if (!wait_or_abort(full(i), (uint32_t)((t / S) & 1), &abort_flag)) {
            atomicExch(&abort_flag, 1);
            stop = true;
            break;
          }
          fence_after();
          const uint32_t st = base + (uint32_t)i * C::kStage;
          const uint64_t a0 = sw128_desc(st), b0 = sw128_desc(st + C::kA);
#pragma unroll
          for (int s = 0; s < kBfStepK / 16; s++)
            mma_ss(dcol, a0 + 2u * s, b0 + 2u * s, idesc, (ks | s) ? 1u : 0u);
          mma_commit(empty(i));
        }
        if (!stop) mma_commit(accfull(acc));
      }
      // every issued MMA is done before the CTA may exit (the last commit covers them all)
      if (t > 0) mbar_wait(empty((t - 1) % S), (uint32_t)(((t - 1) / S) & 1));
    }
  } else if (warp < 4) {
    const int q = warp, r = 32 * q + lane;
    int pu = 0;
    for (int lu = 0; lu < my_units; lu++) {
      const Unit un = unit_at(lu);
      if (un.ntok <= 0) continue;
      const int acc = pu & 1;
      const bool ok = wait_or_abort<128>(accfull(acc), (uint32_t)((pu >> 1) & 1), &abort_flag);
      pu++;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicExch(&abort_flag, 1);
        break;
      }
      fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * NB);
      const bool swapped = un.e == a.E ? side.sh_up_swapped : side.up_swapped;
      float *out = UP ? gu : a.ysorted;
      const int ld = UP ? 2 * a.I : a.H;
      const int col = UP ? un.tile * 128 + (r ^ (swapped ? 1 : 0)) : un.tile * 128 + r;
      const int rows = SPLIT ? 2 * un.ntok : un.ntok;
#pragma unroll 1
      for (int c0 = 0; c0 < NB; c0 += 32) {
        if (c0 < rows) {
          float w[32];
          tmem_ld16(taddr + c0, reinterpret_cast<uint32_t *>(w));
          tmem_ld16(taddr + c0 + 16, reinterpret_cast<uint32_t *>(w + 16));
          tmem_wait_ld();
          const int nbase = SPLIT ? c0 / 2 : c0;
          // the chunk's row scales and destination rows, one per lane, fetched before the
          // loop so that its stores wait on no load
          const bool mine = nbase + lane < un.ntok;
          const float rv = (F16 && mine) ? row_inv[un.pos0 + nbase + lane] : 1.0f;
          // expert-parallel receivers store the row into its source rank's memory
          float *dp = !mine ? nullptr
                            : (!UP && a.ydest) ? a.ydest[un.pos0 + nbase + lane]
                                               : out + (size_t)(un.pos0 + nbase + lane) * ld;
#pragma unroll
          for (int j = 0; j < (SPLIT ? 16 : 32); j++) {
            const int n = nbase + j;
            float v = SPLIT ? w[2 * j] + w[2 * j + 1] : w[j];
            if (F16) v *= __shfl_sync(0xffffffffu, rv, j);  // exact: a power of two
            float *orow = reinterpret_cast<float *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dp), j));
            if (n < un.ntok) orow[col] = v;
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty(acc));
    }
  }
  // stores into other GPUs' memory are visible system-wide before the kernel ends (the
  // signal that follows it raises the ranks' done flags)
  if (!UP && a.ydest) __threadfence_system();
  __syncthreads();
  if (tid == 0 && abort_flag) atomicExch(a.status, kStatusTimeout);
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ---------------------------------------------------------------------------
// The same bf16 / fp16 grouped GEMM on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on two SMs computes a 256-row x up-to-256-token unit: CTA r holds
// the 128 weight rows of tile 2 pt + r and half of the unit's tokens (each CTA loads only
// its own halves, with plain non-multicast TMA), and one thread of CTA 0 issues
// M = 256 MMAs that read both CTAs' shared memory and accumulate into both CTAs' tensor
// memory (each its 128 rows x N tokens). Per K step and SM that moves 32 KB for the
// 4.2 MFLOP the SM's tensor core does (48 KB on the single-CTA kernel), and seven 32 KB
// stages fit where four 48 KB ones did, so more of the L2 / HBM latency is covered.
//   full[s]     (CTA 0) CTA 0's producer expects both CTAs' bytes; both CTAs' TMA loads
//               complete on it
//   empty[s]    (each CTA) the MMA issuer's commit arrives on both CTAs' copies
//   accfull[b]  (each CTA) the last commit of a unit arrives on both
//   accempty[b] (CTA 0) the four epilogue warps of each CTA arrive (CTA 1's remotely)
// Token split of a unit of n tokens: h = n/2 rounded up to 16; CTA 0's B rows are tokens
// 0..h-1, CTA 1's tokens h..2h-1, so accumulator column c is token c (N = 2h).
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int c0,
                                                 int c1, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap *map, int c0,
                                                 int c1, int c2, int c3, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

// completion of this thread's MMAs so far arrives once on the barrier at cluster address
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

__device__ __forceinline__ void mma_ss_pair(uint32_t d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// M = 256 (two CTAs x 128 rows), N = n, f32 D; bf16 or fp16 A and B (one type for both)
__host__ __device__ constexpr uint32_t idesc_pair(int n, bool f16) {
  return (1u << 4) | (f16 ? 0u : (1u << 7) | (1u << 10)) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(256 >> 4) << 24);
}

struct PairCfg {
  static constexpr int kA = 128 * 128;  // 128 rows x 64 elements
  static constexpr int kB = 128 * 128;  // 128 tokens x 64 elements
  static constexpr int kStage = kA + kB;
  static constexpr int kStages = 7;
  static constexpr int kSmem = 1024 + kStages * kStage + 256;
  static_assert(kSmem <= kSmemLimit, "stages exceed shared memory");
};

// With UP the epilogue applies the activation: the gate and up rows of an intermediate
// index sit in adjacent lanes, a lane pair trades one value per two tokens, and each lane
// writes h = act(gate, up) * h_scale[row] as fp16 (h_out [rows][I], the down product's
// operand) for one of the two tokens. h_scale is a power of two per row chosen before the
// product from a bound on |h| (gather_bf16_kernel), so no pass over h is needed to scale it.
template <bool UP, bool F16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kBfThreads, 1) tc_bf16_pair_kernel(
    const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap wmap,
    const __grid_constant__ CUtensorMap sh_wmap, ForwardArgs a, TcSide side, float *gu,
    const float *row_inv, __half *h_out, const float *h_scale) {
  using C = PairCfg;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t dsm[];
  __shared__ int abort_flag;
  const uint32_t rank = cluster_rank();
  const int K = UP ? a.H : a.I;
  const int n_pt = UP ? a.I / 128 : a.H / 256;  // pair tiles of 256 weight rows
  const int n_units = *a.n_items * n_pt;
  const int cid = (int)blockIdx.x >> 1, nclusters = (int)gridDim.x >> 1;
  const int my_units = cid < n_units ? (n_units - cid + nclusters - 1) / nclusters : 0;
  const int nsteps = K / kBfStepK;
  auto unit_at = [&](int lu) {
    const int u = cid + lu * nclusters;
    const int item = u / n_pt;
    const int4 rec = a.items[item];
    Unit un;
    un.e = rec.x;
    un.tile = 2 * (u - item * n_pt) + (int)rank;  // this CTA's 128-row tile
    un.pos0 = rec.z;
    un.ntok = min(256, rec.w);
    return un;
  };
  auto half_of = [](int ntok) { return (((ntok + 1) >> 1) + 15) & ~15; };

  const uint32_t raw = smem_u32(dsm);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + S * C::kStage;  // full[S], empty[S], accfull[2], accempty[2], slot
  auto full = [&](int i) { return bars + 8u * i; };
  auto empty = [&](int i) { return bars + 8u * (S + i); };
  auto accfull = [&](int i) { return bars + 8u * (2 * S + i); };
  auto accempty = [&](int i) { return bars + 8u * (2 * S + 2 + i); };
  const uint32_t slot = bars + 8u * (2 * S + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    abort_flag = *reinterpret_cast<const volatile int32_t *>(a.status) == kStatusTimeout;
    for (int i = 0; i < S; i++) {
      mbar_init(full(i), 1);
      mbar_init(empty(i), 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(accfull(i), 1);
      mbar_init(accempty(i), 8);  // four epilogue warps in each CTA (used in CTA 0)
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  constexpr uint32_t kCols = 512;  // two 256-column accumulators
  if (warp == 0) tmem_alloc_pair(slot, kCols);
  fence_before();
  cluster_sync();  // barriers and tensor memory of both CTAs ready
  fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(dsm + (slot - raw));

  if (warp == 4) {
    if (lane == 0) {
      const uint64_t pol_w = l2_evict_normal(), pol_b = l2_evict_last();
      int t = 0;
      bool stop = false;
      for (int lu = 0; lu < my_units && !stop; lu++) {
        const Unit un = unit_at(lu);
        if (un.ntok <= 0) continue;
        if (*reinterpret_cast<const volatile int32_t *>(a.status) == kStatusTimeout)
          atomicExch(&abort_flag, 1);
        const bool shared = un.e == a.E;
        const int ex = shared ? 0 : un.e;
        const int h = half_of(un.ntok);
        const int brow = un.pos0 + (int)rank * h;
        for (int ks = 0; ks < nsteps; ks++, t++) {
          const int i = t % S;
          if ((t >= S && !wait_or_abort<64>(empty(i), (uint32_t)((t / S - 1) & 1), &abort_flag)) ||
              aborted(&abort_flag)) {
            atomicExch(&abort_flag, 1);
            stop = true;
            break;
          }
          const uint32_t st = base + (uint32_t)i * C::kStage;
          const uint32_t fb = map_to_rank(full(i), 0);
          if (rank == 0) mbar_expect_tx(full(i), (uint32_t)(2 * C::kStage));
          if (UP)
            tma_load_4d_pair_hint(st, shared ? &sh_wmap : &wmap, kBfStepK * ks, 0, un.tile * 64, ex,
                                  fb, pol_w);
          else
            tma_load_2d_pair_hint(st, shared ? &sh_wmap : &wmap, kBfStepK * ks,
                                  ex * a.H + un.tile * 128, fb, pol_w);
          tma_load_2d_pair_hint(st + C::kA, &bmap, kBfStepK * ks, brow, fb, pol_b);
        }
      }
      // CTA 0 drains both CTAs' loads in flight (they all complete on its full barriers)
      if (rank == 0)
        for (int i = max(0, t - S); i < t; i++) mbar_wait(full(i % S), (uint32_t)((i / S) & 1));
    }
  } else if (warp == 5) {
    if (lane == 0 && rank == 0) {
      int t = 0, pu = 0;
      bool stop = false;
      for (int lu = 0; lu < my_units && !stop; lu++) {
        const Unit un = unit_at(lu);
        if (un.ntok <= 0) continue;
        const int acc = pu & 1;
        if (pu >= 2 && !wait_or_abort(accempty(acc), (uint32_t)(((pu >> 1) - 1) & 1), &abort_flag)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        pu++;
        fence_after();
        const int n = 2 * half_of(un.ntok);
        const uint32_t idesc = idesc_pair(n, F16);
        const uint32_t dcol = tmem + (uint32_t)(acc * 256);
        for (int ks = 0; ks < nsteps; ks++, t++) {
          const int i = t % S;
          if (!wait_or_abort(full(i), (uint32_t)((t / S) & 1), &abort_flag)) {
            atomicExch(&abort_flag, 1);
            stop = true;
            break;
          }
          fence_after();
          const uint32_t st = base + (uint32_t)i * C::kStage;
          const uint64_t a0 = sw128_desc(st), b0 = sw128_desc(st + C::kA);
#pragma unroll
          for (int s = 0; s < kBfStepK / 16; s++)
            mma_ss_pair(dcol, a0 + 2u * s, b0 + 2u * s, idesc, (ks | s) ? 1u : 0u);
          mma_commit_pair(empty(i));
          mma_commit_pair(map_to_rank(empty(i), 1));
        }
        if (!stop) {
          mma_commit_pair(accfull(acc));
          mma_commit_pair(map_to_rank(accfull(acc), 1));
        }
      }
      // every issued MMA is done before either CTA may free its stages or exit
      if (t > 0) mbar_wait(empty((t - 1) % S), (uint32_t)(((t - 1) / S) & 1));
    }
  } else if (warp < 4) {
    const int q = warp, r = 32 * q + lane;
    const uint32_t ae0 = map_to_rank(accempty(0), 0), ae1 = map_to_rank(accempty(1), 0);
    int pu = 0;
    for (int lu = 0; lu < my_units; lu++) {
      const Unit un = unit_at(lu);
      if (un.ntok <= 0) continue;
      const int acc = pu & 1;
      const bool ok = wait_or_abort<128>(accfull(acc), (uint32_t)((pu >> 1) & 1), &abort_flag);
      pu++;
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) atomicExch(&abort_flag, 1);
        break;
      }
      fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * 256);
      const bool swapped = un.e == a.E ? side.sh_up_swapped : side.up_swapped;
      // UP: gate|up row `gr` of the tile; even rows are gates
      const int gr = r ^ (swapped ? 1 : 0);
      const bool is_gate = (gr & 1) == 0;
      __half *hcol = h_out + un.tile * 64 + (gr >> 1);
      const int col = un.tile * 128 + r;
#pragma unroll 1
      for (int c0 = 0; c0 < un.ntok; c0 += 32) {
        float w[32];
        tmem_ld16(taddr + c0, reinterpret_cast<uint32_t *>(w));
        tmem_ld16(taddr + c0 + 16, reinterpret_cast<uint32_t *>(w + 16));
        tmem_wait_ld();
        if (UP) {
          // the chunk's 32 row scales, one per lane (no load waits inside the loop below)
          const float sc = c0 + lane < un.ntok ? h_scale[un.pos0 + c0 + lane] : 0.0f;
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            // the gate lane takes token c0 + j, the up lane token c0 + j + 1
            const float recv = __shfl_xor_sync(0xffffffffu, is_gate ? w[j + 1] : w[j], 1);
            const float s_n = __shfl_sync(0xffffffffu, sc, is_gate ? j : j + 1);
            const float g = is_gate ? w[j] : recv, u = is_gate ? recv : w[j + 1];
            const int n = c0 + j + (is_gate ? 0 : 1);
            if (n < un.ntok)
              hcol[(size_t)(un.pos0 + n) * a.I] = __float2half_rn(glm_silu_mul_fast(g, u) * s_n);
          }
        } else {
          const float rv = (F16 && c0 + lane < un.ntok) ? row_inv[un.pos0 + c0 + lane] : 1.0f;
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int n = c0 + j;
            float v = w[j];
            if (F16) v *= __shfl_sync(0xffffffffu, rv, j);  // exact: a power of two
            if (n < un.ntok) a.ysorted[(size_t)(un.pos0 + n) * a.H + col] = v;
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? ae1 : ae0);
    }
  }
  fence_before();
  cluster_sync();  // no CTA frees tensor memory or leaves while its pair still works
  if (tid == 0 && abort_flag) atomicExch(a.status, kStatusTimeout);
  if (warp == 0) {
    fence_after();
    tmem_dealloc_pair(tmem, kCols);
  }
}

// bf16 inputs gathered into sorted order: out[pos] = x[token of pos] (bf16 copy).
//
// With h_scale, also the power of two that scales row pos of the intermediate h into fp16.
// |gate_i| <= |gate row i| |x| and |up_i| <= |up row i| |x| (Cauchy-Schwarz), |silu(g)| <= |g|,
// so |h_i| <= B = gate_norm[e] up_norm[e] |x|^2 for every i of the row. The scale is
// 2^(13 - floor(log2 B)): every scaled |h| stays below 2^14, a quarter of fp16's largest
// finite value (room for rounding in the products), and values within 2^24 of the bound
// keep fp16's full 11-bit precision. h_inv[pos] = 1 / scale (exact).
__global__ void __launch_bounds__(256) gather_bf16_kernel(ForwardArgs a, __nv_bfloat16 *out,
                                                          TcSide side, float *h_scale,
                                                          float *h_inv) {
  const int pos = blockIdx.x;
  if (pos >= a.offsets[a.E + 1]) return;
  const int P = a.T * a.k, pr = a.sorted[pos];
  const int tok = pr < P ? pr / a.k : pr - P;
  const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(a.x) + (size_t)tok * a.H);
  uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)pos * a.H);
  float ss = 0.0f;
  for (int i = threadIdx.x; i < a.H / 8; i += blockDim.x) {
    const uint4 v = src[i];
    dst[i] = v;
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float lo = __uint_as_float(p[j] << 16), hi = __uint_as_float(p[j] & 0xffff0000u);
      ss = fmaf(lo, lo, fmaf(hi, hi, ss));
    }
  }
  if (!h_scale) return;
  __shared__ float part[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) sum += part[w];
    const int e = pr < P ? (int)a.sel_idx[pr] : a.E;
    const float bound = side.gate_norm[e] * side.up_norm[e] * sum;
    float s = 1.0f;
    if (!isfinite(bound)) s = 0x1p-126f;
    else if (bound > 0.0f) s = exp2f((float)max(-126, min(126, 13 - ilogbf(bound))));
    h_scale[pos] = s;
    h_inv[pos] = 1.0f / s;
  }
}

// out[e] = max over the rows of expert e of the row's L2 norm (a warp per row).
__global__ void row_norm_max_kernel(const uint8_t *w, uint64_t expert_stride, int experts,
                                    int rows, int K, float *out) {
  const int lane = threadIdx.x & 31;
  const uint64_t nrows = (uint64_t)experts * rows;
  const uint64_t step = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t r = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5; r < nrows; r += step) {
    const int e = (int)(r / rows), i = (int)(r % rows);
    const uint4 *row = reinterpret_cast<const uint4 *>(w + e * expert_stride + (uint64_t)i * K * 2);
    float ss = 0.0f;
    for (int q = lane; q < K / 8; q += 32) {
      const uint4 v = row[q];
      const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float lo = __uint_as_float(p[j] << 16), hi = __uint_as_float(p[j] & 0xffff0000u);
        ss = fmaf(lo, lo, fmaf(hi, hi, ss));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    // norms are not negative, so their bit patterns order as integers; a NaN or inf norm
    // (a non-finite weight) pins the bound at inf
    if (lane == 0) atomicMax(reinterpret_cast<int *>(out + e), __float_as_int(fminf(sqrtf(ss), INFINITY)));
  }
}

// h = act(gate, up) from gu, as bf16 hi (row 2 pos) + lo (row 2 pos + 1).
__global__ void __launch_bounds__(256) pack_h_bf16_kernel(ForwardArgs a, const float *gu,
                                                         __nv_bfloat16 *out) {
  const int pos = blockIdx.x;
  if (pos >= a.offsets[a.E + 1]) return;
  const int P = a.T * a.k, pr = a.sorted[pos];
  const int e = pr < P ? (int)a.sel_idx[pr] : a.E;
  const int I = a.I;
  const float *row = gu + (size_t)pos * 2 * I;
  for (int i = threadIdx.x * 2; i < I; i += blockDim.x * 2) {
    const float4 v = *reinterpret_cast<const float4 *>(row + 2 * i);
    const float h0 = activate(a, e, v.x, v.y), h1 = activate(a, e, v.z, v.w);
    const __nv_bfloat16 a0 = __float2bfloat16_rn(h0), a1 = __float2bfloat16_rn(h1);
    const __nv_bfloat16 b0 = __float2bfloat16_rn(h0 - __bfloat162float(a0));
    const __nv_bfloat16 b1 = __float2bfloat16_rn(h1 - __bfloat162float(a1));
    *reinterpret_cast<__nv_bfloat162 *>(out + (size_t)2 * pos * I + i) = __halves2bfloat162(a0, a1);
    *reinterpret_cast<__nv_bfloat162 *>(out + (size_t)(2 * pos + 1) * I + i) = __halves2bfloat162(b0, b1);
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

bool tc_supported(int gate_type, int down_type, int H, int I) {
  if (gate_type == DM_BF16 && down_type == DM_BF16) return H % 128 == 0 && I % 64 == 0;
  if (gate_type != DM_Q4_K) return false;
  if (down_type != DM_Q6_K && down_type != DM_Q5_0) return false;
  if (H % 256 || I % 64) return false;  // Q4_K rows of whole super-blocks; 128-row down tiles
  if (I > tc::kMaxPackI) return false;
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

// View of a packed [rows][K] fp16 matrix as (64 elements, row, K/64 atoms): one box of
// {64, nb, 4} lands as 4 swizzled atoms of nb rows each, the B tile of one K step.
static bool encode(CUtensorMap *map, void *base, int K, int rows, int nb) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(K / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)nb, 4};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KIND>
static bool fits_split(int nt) {
  switch (nt) {
    case 16: return tc::Cfg<KIND, 16, true>::kFits;
    case 32: return tc::Cfg<KIND, 32, true>::kFits;
    default: return tc::Cfg<KIND, 64, true>::kFits;
  }
}

// x16 / h16 hold 2*rows rows (hi and lo interleaved with the split, hi alone without).
// The split of a matrix is dropped where its kernel's tiles would not fit shared memory.
static bool encode_bf16_rows(CUtensorMap *map, const void *base, int K, uint64_t rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int make_tc_maps(TcPlan &p, int H, int I, int down_type, int nt) {
  if (down_type == DM_BF16) {  // gathered bf16 inputs; intermediates as hi/lo row pairs
    p.bf16 = true;
    p.split_x = false;
    p.split_h = true;
    // x tiles: nt tokens; h tiles: nt rows = nt / 2 tokens as hi/lo pairs
    if (!encode_bf16_rows(&p.x_map, p.x16, H, (uint64_t)p.rows, nt)) return -1;
    if (!encode_bf16_rows(&p.h_map, p.h16, I, 2 * (uint64_t)p.rows, nt)) return -1;
    // the same buffer as single fp16 rows (2-byte elements either way for the copy)
    if (!encode_bf16_rows(&p.h1_map, p.h16, I, (uint64_t)p.rows, nt)) return -1;
    // CTA pairs load half a 256-token tile each: 128-row boxes
    if (!encode_bf16_rows(&p.x_map_pair, p.x16, H, (uint64_t)p.rows, 128)) return -1;
    if (!encode_bf16_rows(&p.h1_map_pair, p.h16, I, (uint64_t)p.rows, 128)) return -1;
    return 0;
  }
  p.split_x = p.split && fits_split<tc::kUpQ4K>(nt);
  p.split_h = p.split && (down_type == DM_Q6_K ? fits_split<tc::kDownQ6K>(nt)
                                               : fits_split<tc::kDownQ50>(nt));
  if (!encode(&p.x_map, p.x16, H, p.split_x ? 2 * p.rows : p.rows, p.split_x ? 2 * nt : nt))
    return -1;
  if (!encode(&p.h_map, p.h16, I, p.split_h ? 2 * p.rows : p.rows, p.split_h ? 2 * nt : nt))
    return -1;
  return 0;
}

template <int KIND, int NT>
static bool launch_kind(const CUtensorMap &map, const ForwardArgs &a, const TcWeights &w,
                        const float *inv, const TcPlan &p, bool split, cudaStream_t s) {
  const int n_tiles = KIND == tc::kUpQ4K ? a.I / 64 : a.H / 128;
  const int grid = std::max(1, std::min(p.n_sm, p.max_items * n_tiles));
  const CUtensorMap &wm = KIND == tc::kUpQ4K ? w.up : w.down;
  const CUtensorMap &sm = KIND == tc::kUpQ4K ? w.sh_up : w.sh_down;
  if (split) {
    if constexpr (tc::Cfg<KIND, NT, true>::kFits) {
      auto fn = tc::tc_expert_kernel<KIND, NT, true>;
      ensure_smem_limit((const void *)fn);
      fn<<<grid, tc::kTcThreads, tc::Cfg<KIND, NT, true>::kSmem, s>>>(map, wm, sm, a, w.side, inv,
                                                                       p.gu);
    }
  } else {
    static_assert(tc::Cfg<KIND, NT, false>::kFits, "tile configuration exceeds shared memory");
    auto fn = tc::tc_expert_kernel<KIND, NT, false>;
    ensure_smem_limit((const void *)fn);
    fn<<<grid, tc::kTcThreads, tc::Cfg<KIND, NT, false>::kSmem, s>>>(map, wm, sm, a, w.side, inv,
                                                                      p.gu);
  }
  return true;
}

template <int NT>
static int launch_nt(const ForwardArgs &a, const TcPlan &p, const TcWeights &w, cudaStream_t s,
                     cudaEvent_t down_mark) {
  const int rows_bound = a.T * a.k + (a.shared ? a.T : 0);
  tc::pack_kernel<true><<<(rows_bound + tc::kPackRows - 1) / tc::kPackRows, 32 * tc::kPackRows, 0, s>>>(
      a, nullptr, p.x16, p.x_inv, a.H, p.split_x ? 1 : 0);
  launch_kind<tc::kUpQ4K, NT>(p.x_map, a, w, p.x_inv, p, p.split_x, s);
  if (down_mark) cudaEventRecord(down_mark, s);
  {
    const size_t hsmem = (size_t)tc::kPackRows * a.I * sizeof(float);
    if (hsmem > 48 * 1024) ensure_smem_limit((const void *)tc::pack_kernel<false>);
    tc::pack_kernel<false><<<(rows_bound + tc::kPackRows - 1) / tc::kPackRows, 32 * tc::kPackRows,
                             hsmem, s>>>(a, p.gu, p.h16, p.h_inv, a.I, p.split_h ? 1 : 0);
  }
  if (a.down_type == DM_Q6_K)
    launch_kind<tc::kDownQ6K, NT>(p.h_map, a, w, p.h_inv, p, p.split_h, s);
  else
    launch_kind<tc::kDownQ50, NT>(p.h_map, a, w, p.h_inv, p, p.split_h, s);
  return 4;
}

// Work items of up to 256 tokens: gate/up takes a whole item per unit (N = 256, every
// weight tile read once per item); down, whose hi/lo rows double N, takes each item as
// two units of 128 tokens.
// Persistent grid of CTA pairs for tc_bf16_pair_kernel: at most one pair per two SMs.
static int pair_grid(const TcPlan &p, int tiles) {
  const int pairs = std::max(1, std::min(p.n_sm / 2, p.max_items * tiles));
  return 2 * pairs;
}

static bool use_pairs() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("DISKMULE_CUDA_TC_PAIRS");
    v = !(e && (!strcmp(e, "0") || !strcmp(e, "false")));
  }
  return v == 1;
}

static int launch_bf16(const ForwardArgs &a, const TcPlan &p, const TcWeights &w, cudaStream_t s,
                       cudaEvent_t down_mark) {
  constexpr int NT = 256;
  if (p.nt != NT) return -1;
  const int rows_bound = a.T * a.k + (a.shared ? a.T : 0);
  // (the pair epilogue applies GLM's activation)
  const bool pairs = use_pairs() && a.family == kGlm && w.f16_down && w.side.gate_norm &&
                     a.I % 128 == 0 && a.H % 256 == 0;
  // with CTA pairs, the gather also sets each row's intermediate scale (p.x_inv holds the
  // scales, p.h_inv their inverses)
  tc::gather_bf16_kernel<<<rows_bound, 256, 0, s>>>(a, reinterpret_cast<__nv_bfloat16 *>(p.x16),
                                                    w.side, pairs ? p.x_inv : nullptr, p.h_inv);
  if (pairs) {
    // CTA pairs for the gate/up product: 256-row weight tiles, activation in the epilogue
    // (DISKMULE_CUDA_TC_PAIRS=0 turns them off)
    auto up = tc::tc_bf16_pair_kernel<true, false>;
    ensure_smem_limit((const void *)up);
    up<<<pair_grid(p, a.I / 128), tc::kBfThreads, tc::PairCfg::kSmem, s>>>(
        p.x_map_pair, w.up, w.sh_up, a, w.side, nullptr, nullptr, p.h16, p.x_inv);
    if (down_mark) cudaEventRecord(down_mark, s);
    // the down product (K = I: few K steps per unit) measured faster on single CTAs
    auto down = tc::tc_bf16_kernel<false, NT, false, 1, true>;
    ensure_smem_limit((const void *)down);
    const int grid = std::max(1, std::min(p.n_sm, p.max_items * (a.H / 128)));
    down<<<grid, tc::kBfThreads, tc::BfCfg<NT>::kSmem, s>>>(p.h1_map, w.down16, w.sh_down16, a,
                                                                w.side, p.gu, p.h_inv);
    return 3;
  }
  {
    auto fn = tc::tc_bf16_kernel<true, NT, false, 1>;
    ensure_smem_limit((const void *)fn);
    const int grid = std::max(1, std::min(p.n_sm, p.max_items * (a.I / 64)));
    fn<<<grid, tc::kBfThreads, tc::BfCfg<NT>::kSmem, s>>>(p.x_map, w.up, w.sh_up, a, w.side, p.gu,
                                                              nullptr);
  }
  if (down_mark) cudaEventRecord(down_mark, s);
  if (w.f16_down) {
    // h = act(gate, up) as one fp16 row per pair, scaled by a power of two per row
    const size_t hsmem = (size_t)tc::kPackRows * a.I * sizeof(float);
    if (hsmem > 48 * 1024) ensure_smem_limit((const void *)tc::pack_kernel<false>);
    tc::pack_kernel<false><<<(rows_bound + tc::kPackRows - 1) / tc::kPackRows, 32 * tc::kPackRows,
                             hsmem, s>>>(a, p.gu, p.h16, p.h_inv, a.I, 0);
    auto fn = tc::tc_bf16_kernel<false, NT, false, 1, true>;
    ensure_smem_limit((const void *)fn);
    const int grid = std::max(1, std::min(p.n_sm, p.max_items * (a.H / 128)));
    fn<<<grid, tc::kBfThreads, tc::BfCfg<NT>::kSmem, s>>>(p.h1_map, w.down16, w.sh_down16, a,
                                                              w.side, p.gu, p.h_inv);
    return 4;
  }
  tc::pack_h_bf16_kernel<<<rows_bound, 256, 0, s>>>(a, p.gu, reinterpret_cast<__nv_bfloat16 *>(p.h16));
  {
    auto fn = tc::tc_bf16_kernel<false, NT, true, 2>;
    ensure_smem_limit((const void *)fn);
    const int grid = std::max(1, std::min(p.n_sm, 2 * p.max_items * (a.H / 128)));
    fn<<<grid, tc::kBfThreads, tc::BfCfg<NT>::kSmem, s>>>(p.h_map, w.down, w.sh_down, a, w.side,
                                                              p.gu, nullptr);
  }
  return 4;
}

// Self-test: the bounded wait of the kernels above on a barrier nothing arrives on.
__global__ void selftest_wait_kernel(long long cycles, int32_t *status) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t b = (uint32_t)__cvta_generic_to_shared(&bar);
  tc::mbar_init(b, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const long long start = clock64();
  bool done = false;
  while (!done) {
    done = tc::mbar_try(b, 0);
    if (!done && clock64() - start > cycles) break;
  }
  *status = done ? 0 : kStatusTimeout;
}

void launch_selftest_wait(long long cycles, int32_t *status, cudaStream_t s) {
  selftest_wait_kernel<<<1, 1, 0, s>>>(cycles, status);
}

int launch_tc_experts(const ForwardArgs &a, const TcPlan &p, const TcWeights &w, cudaStream_t s,
                      cudaEvent_t down_mark) {
  if (p.bf16) return launch_bf16(a, p, w, s, down_mark);
  switch (p.nt) {
    case 16: return launch_nt<16>(a, p, w, s, down_mark);
    case 32: return launch_nt<32>(a, p, w, s, down_mark);
    case 64: return launch_nt<64>(a, p, w, s, down_mark);
    default: return -1;
  }
}

void tc_side_bytes(int down_type, uint64_t experts, int H, int I, uint64_t *qh_bytes,
                   uint64_t *d_bytes) {
  const uint64_t rows = experts * (uint64_t)((I + tc::kStepK - 1) / tc::kStepK) * H;
  *qh_bytes = down_type == DM_Q5_0 ? experts * (uint64_t)H * I : 0;  // one byte per value
  *d_bytes = down_type == DM_Q5_0 ? rows * 16 : rows * 2;
}

// gate/up rows as {row bytes, gate|up, row, expert}: the lower of the two base addresses
// is the origin and the other sits one "gate|up" stride away.
static bool encode_up(CUtensorMap *map, const uint8_t *gate, const uint8_t *up, uint64_t row_bytes,
                      int I, int experts, uint64_t expert_stride, int *swapped) {
  auto fn = encode_fn();
  if (!fn || !gate || !up) return false;
  const uint8_t *origin = gate < up ? gate : up;
  *swapped = gate < up ? 0 : 1;
  cuuint64_t dims[4] = {row_bytes, 2, (cuuint64_t)I, (cuuint64_t)experts};
  cuuint64_t strides[3] = {(cuuint64_t)(gate < up ? up - gate : gate - up), row_bytes,
                           expert_stride};
  cuuint32_t box[4] = {144, 2, 64, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void *)origin, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// down quant bytes as {row bytes, row}, box {box_x, 128}
static bool encode_rows(CUtensorMap *map, const uint8_t *base, uint64_t row_bytes, uint64_t rows,
                        uint32_t box_x) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_x, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// widened Q5_0 rows ({I bytes, row}) as 2-byte elements, box {136, 128}: the 256 bytes of
// one K step plus 16 more, so that rows land 272 bytes apart in shared memory (an odd
// multiple of 16: conflict-free 16-byte reads of 32 rows); past I the box reads zeros
static bool encode_rows16(CUtensorMap *map, const uint8_t *base, int row_bytes, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn || !base || row_bytes % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes / 2, rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {136, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void *)base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 gate/up rows as {K, gate|up, row, expert} (box {64, 2, 64, 1}, 128-byte swizzle):
// 64 interleaved gate/up row pairs of one 64-wide K step.
static bool encode_up_bf16(CUtensorMap *map, const uint8_t *gate, const uint8_t *up, int H, int I,
                           int experts, uint64_t expert_stride, int *swapped) {
  auto fn = encode_fn();
  if (!fn || !gate || !up) return false;
  const uint8_t *origin = gate < up ? gate : up;
  *swapped = gate < up ? 0 : 1;
  cuuint64_t dims[4] = {(cuuint64_t)H, 2, (cuuint64_t)I, (cuuint64_t)experts};
  cuuint64_t strides[3] = {(cuuint64_t)(gate < up ? up - gate : gate - up), (cuuint64_t)H * 2,
                           expert_stride};
  cuuint32_t box[4] = {64, 2, 64, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, (void *)origin, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int make_tc_weights_bf16(TcWeights &w, const uint8_t *gate, const uint8_t *up, uint64_t expert_stride,
                         const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *down,
                         const uint8_t *sh_down, int experts, int H, int I,
                         const uint8_t *down16, const uint8_t *sh_down16) {
  if (!encode_up_bf16(&w.up, gate, up, H, I, experts, expert_stride, &w.side.up_swapped)) return -1;
  if (!encode_bf16_rows(&w.down, down, I, (uint64_t)experts * H, 128)) return -1;
  const bool shared = sh_gate != nullptr;
  if (shared) {
    if (!encode_up_bf16(&w.sh_up, sh_gate, sh_up, H, I, 1, (uint64_t)I * H * 2, &w.side.sh_up_swapped))
      return -1;
    if (!encode_bf16_rows(&w.sh_down, sh_down, I, (uint64_t)H, 128)) return -1;
  } else {
    w.sh_up = w.up;
    w.sh_down = w.down;
  }
  w.f16_down = false;
  if (down16 && (!shared || sh_down16)) {
    if (!encode_bf16_rows(&w.down16, down16, I, (uint64_t)experts * H, 128)) return -1;
    if (shared) {
      if (!encode_bf16_rows(&w.sh_down16, sh_down16, I, (uint64_t)H, 128)) return -1;
    } else {
      w.sh_down16 = w.down16;
    }
    w.f16_down = true;
  }
  return 0;
}

namespace tc {
__global__ void bf16_to_f16_kernel(const uint4 *src, uint4 *dst, uint64_t n8) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float lo = __uint_as_float(in[j] << 16), hi = __uint_as_float(in[j] & 0xffff0000u);
      o[j] = h2u(__halves2half2(__float2half_rn(lo), __float2half_rn(hi)));
    }
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}
}  // namespace tc

void launch_row_norm_max(const void *w, uint64_t expert_stride, int experts, int rows, int K,
                         float *out, cudaStream_t stream) {
  tc::row_norm_max_kernel<<<148 * 8, 256, 0, stream>>>((const uint8_t *)w, expert_stride, experts,
                                                       rows, K, out);
}

void launch_bf16_to_f16(const void *src, void *dst, uint64_t n, cudaStream_t stream) {
  const uint64_t n8 = n / 8;  // callers pass whole 16-byte pieces (rows of 8k elements)
  tc::bf16_to_f16_kernel<<<148 * 8, 256, 0, stream>>>((const uint4 *)src, (uint4 *)dst, n8);
}

int make_tc_weights(TcWeights &w, const uint8_t *gate, const uint8_t *up, uint64_t expert_stride,
                    const uint8_t *sh_gate, const uint8_t *sh_up, const SplitTensor &down,
                    const SplitTensor &sh_down, int down_type, int experts, int H, int I,
                    uint8_t *qh_t, uint8_t *d_t, uint8_t *sh_qh_t, uint8_t *sh_d_t,
                    cudaStream_t stream) {
  const uint64_t up_row = (uint64_t)(H / 256) * 144;
  if (!encode_up(&w.up, gate, up, up_row, I, experts, expert_stride, &w.side.up_swapped)) return -1;
  const bool shared = sh_gate != nullptr;
  if (shared && !encode_up(&w.sh_up, sh_gate, sh_up, up_row, I, 1, up_row * I, &w.side.sh_up_swapped))
    return -1;
  const bool q6 = down_type == DM_Q6_K;
  if (q6) {
    const uint64_t down_row = (uint64_t)(I / 256) * 208;
    if (!encode_rows(&w.down, down.quant, down_row, (uint64_t)experts * H, 208)) return -1;
    if (shared && !encode_rows(&w.sh_down, sh_down.quant, down_row, (uint64_t)H, 208)) return -1;
  } else {
    // Q5_0 rows widened to I bytes (side_transpose_kernel, below, fills them first)
    if (!encode_rows16(&w.down, qh_t, I, (uint64_t)experts * H)) return -1;
    if (shared && !encode_rows16(&w.sh_down, sh_qh_t, I, (uint64_t)H)) return -1;
  }
  if (!shared) {  // the kernels take both maps; the shared ones are never used
    w.sh_up = w.up;
    w.sh_down = w.down;
  }
  const int threads = 256;
  tc::side_transpose_kernel<<<1024, threads, 0, stream>>>(down_type, down, experts, H, I, qh_t, d_t);
  if (shared)
    tc::side_transpose_kernel<<<256, threads, 0, stream>>>(down_type, sh_down, 1, H, I, sh_qh_t,
                                                          sh_d_t);
  w.side.qh_t = qh_t;
  w.side.d_t = d_t;
  w.side.sh_qh_t = sh_qh_t;
  w.side.sh_d_t = sh_d_t;
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace dm
