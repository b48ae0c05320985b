// dm_synth.cuh -- counter-based synthetic GGUF / safetensors tensors.
//
// Every byte of a tensor is a pure function of (seed, block index), so the host
// and the device produce identical bytes and any expert's slice can be generated
// alone. The generator is SplitMix64 (the reference's sampler, src/runtime.rs:
// 1017-1031) evaluated at counter n: the n-th output of a SplitMix64 seeded with
// `seed`. Only integer operations, one correctly rounded int->float conversion and
// fmaf are used, so host and device agree bit for bit.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define DM_HD __host__ __device__ __forceinline__
#else
#define DM_HD inline
#endif

namespace dm {
namespace synth {

DM_HD uint64_t splitmix(uint64_t seed, uint64_t n) {
  uint64_t z = seed + (n + 1) * 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

DM_HD float int_to_float_rn(int64_t v) {
#ifdef __CUDA_ARCH__
  return __ll2float_rn(v);
#else
  return (float)v;  // round-to-nearest-even (default rounding mode)
#endif
}

DM_HD float fma_rn(float a, float b, float c) {
#ifdef __CUDA_ARCH__
  return __fmaf_rn(a, b, c);
#else
  return __builtin_fmaf(a, b, c);
#endif
}

DM_HD float mul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  volatile float r = a * b;
  return r;
#endif
}

DM_HD uint32_t f32_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}

// uniform in [0, 1) with 24 random bits
DM_HD float uniform24(uint64_t r) { return int_to_float_rn((int64_t)(r >> 40)) * 5.9604644775390625e-08f; }

// approximately N(0, 1): Irwin-Hall sum of 12 uniforms (24 bits each) minus 6,
// summed exactly in integers and rounded once.
DM_HD float normal(uint64_t seed, uint64_t element) {
  int64_t s = 0;
  for (int j = 0; j < 6; j++) {
    uint64_t r = splitmix(seed, element * 6 + j);
    s += (int64_t)(r >> 40) + (int64_t)((r >> 8) & 0xffffffull);
  }
  return int_to_float_rn(s - 6 * (int64_t)16777216) * 5.9604644775390625e-08f;
}

// IEEE f32 -> binary16, round to nearest even (finite inputs).
DM_HD uint16_t f32_to_f16_bits(float f) {
  uint32_t x = f32_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t mant = x & 0x7fffffu;
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - exp);
    uint32_t half = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t half = sign | ((uint32_t)exp << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1))) half++;
  return (uint16_t)half;
}

DM_HD uint16_t f32_to_bf16_bits(float f) {
  uint32_t x = f32_bits(f);
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

// f16 scale uniform in [lo, hi)
DM_HD uint16_t scale_f16(uint64_t r, float lo, float hi) {
  float u = uniform24(r);
  return f32_to_f16_bits(fma_rn(u, hi - lo, lo));
}

// Bytes per block and elements per block of the synthetic formats.
DM_HD int block_bytes(int kind) {
  switch (kind) {
    case 0: return 4;     // F32
    case 1: return 2;     // F16
    case 30: return 2;    // BF16
    case 6: return 22;    // Q5_0
    case 8: return 34;    // Q8_0
    case 12: return 144;  // Q4_K
    case 14: return 210;  // Q6_K
    default: return 0;
  }
}

// Write block `b` of a tensor of type `kind`. Dense types: one element drawn
// from N(0, sigma). Block types: random bytes with the f16 scale fields drawn
// uniformly from [lo, hi).
DM_HD void fill_block(int kind, uint64_t seed, uint64_t b, float sigma, float lo, float hi,
                      uint8_t *out) {
  switch (kind) {
    case 0: {
      uint32_t v = f32_bits(mul_rn(normal(seed, b), sigma));
      out[0] = (uint8_t)v; out[1] = (uint8_t)(v >> 8); out[2] = (uint8_t)(v >> 16); out[3] = (uint8_t)(v >> 24);
      return;
    }
    case 1: {
      uint16_t v = f32_to_f16_bits(mul_rn(normal(seed, b), sigma));
      out[0] = (uint8_t)v; out[1] = (uint8_t)(v >> 8);
      return;
    }
    case 30: {
      uint16_t v = f32_to_bf16_bits(mul_rn(normal(seed, b), sigma));
      out[0] = (uint8_t)v; out[1] = (uint8_t)(v >> 8);
      return;
    }
    default: break;
  }
  const int bytes = block_bytes(kind);
  const uint64_t draws = (uint64_t)(bytes + 7) / 8;
  for (int i = 0; i < bytes; i++) {
    uint64_t r = splitmix(seed, b * draws + (uint64_t)(i >> 3));
    out[i] = (uint8_t)(r >> (8 * (i & 7)));
  }
  const uint64_t scale_seed = seed ^ 0x5ca1ab1e0ddba11ull;
  uint64_t r0 = splitmix(scale_seed, 2 * b), r1 = splitmix(scale_seed, 2 * b + 1);
  uint16_t d = scale_f16(r0, lo, hi);
  switch (kind) {
    case 12: {  // Q4_K: d, dmin at bytes 0..3
      uint16_t dmin = scale_f16(r1, lo, hi);
      out[0] = (uint8_t)d; out[1] = (uint8_t)(d >> 8);
      out[2] = (uint8_t)dmin; out[3] = (uint8_t)(dmin >> 8);
      return;
    }
    case 14:  // Q6_K: d at bytes 208..209
      out[208] = (uint8_t)d; out[209] = (uint8_t)(d >> 8);
      return;
    case 6:
    case 8:  // Q5_0 / Q8_0: d at bytes 0..1
      out[0] = (uint8_t)d; out[1] = (uint8_t)(d >> 8);
      return;
    default:
      return;
  }
}

}  // namespace synth
}  // namespace dm
