// dm_common.cuh -- shared definitions for the sm_100a MoE kernels.
//
// Weight formats are GGUF blocks (src/gguf.rs:321-342) and safetensors rows. The
// decoders below restate src/cpu.rs:546-660 on the device; the arithmetic order of
// the per-element value follows the reference (e.g. Q4_K: (d*sc)*q - dmin*m).
#pragma once

#include <utility>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/diskmule_cuda.h"

namespace dm {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// exact helpers shared with the CPU reference
// ---------------------------------------------------------------------------

// src/cpu.rs:647-660 -- f16 bits to f32 (subnormals as fraction * 2^-24).
__host__ __device__ inline float f16_bits_to_f32(uint16_t value) {
  uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  uint32_t exponent = (value >> 10) & 0x1fu;
  uint32_t fraction = value & 0x03ffu;
  uint32_t bits;
  if (exponent == 0 && fraction == 0) {
    bits = sign;
  } else if (exponent == 0) {
    float magnitude = (float)fraction * 5.9604644775390625e-08f;  // exact
    return sign ? -magnitude : magnitude;
  } else if (exponent == 0x1f) {
    bits = sign | 0x7f800000u | (fraction << 13);
  } else {
    bits = sign | ((exponent + 112u) << 23) | (fraction << 13);
  }
#ifdef __CUDA_ARCH__
  return __uint_as_float(bits);
#else
  float f;
  memcpy(&f, &bits, 4);
  return f;
#endif
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t bits) {
  return __uint_as_float((uint32_t)bits << 16);
}

// exp rounded once from a double evaluation: the correctly rounded f32 result
// except when exp(x) lies within ~1e-16 of a rounding midpoint.
__device__ __forceinline__ float exp_f32_cr(float x) { return (float)exp((double)x); }

// src/glm52/cpu.rs:980-982
__device__ __forceinline__ float glm_sigmoid(float v) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32_cr(-v)));
}
// src/glm52/cpu.rs:984-986 (shared expert `mlp`)
__device__ __forceinline__ float glm_silu(float v) { return __fmul_rn(v, glm_sigmoid(v)); }
// src/glm52/expert.rs:264 (routed experts, CachedExpert::mlp)
__device__ __forceinline__ float glm_cached_silu(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, exp_f32_cr(-v)));
}
// src/qwen35/cpu.rs:982-993
__device__ __forceinline__ float qwen_sigmoid(float v) {
  if (v >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32_cr(-v)));
  float e = exp_f32_cr(v);
  return __fdiv_rn(e, __fadd_rn(1.0f, e));
}
__device__ __forceinline__ float qwen_silu(float v) { return __fmul_rn(v, qwen_sigmoid(v)); }
// src/cpu.rs:145-150 (gelu_tanh); tanh from CUDA (tolerance-level parity).
__device__ __forceinline__ float gelu_tanh(float v) {
  float cube = __fmul_rn(v, __fmul_rn(v, v));
  float arg = __fmul_rn(0.7978846f, __fadd_rn(v, __fmul_rn(0.044715f, cube)));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(arg)));
}

// Rust f32::total_cmp as a signed key (IEEE total order).
__host__ __device__ inline int32_t total_key(float v) {
#ifdef __CUDA_ARCH__
  int32_t bits = __float_as_int(v);
#else
  int32_t bits;
  memcpy(&bits, &v, 4);
#endif
  return bits ^ (int32_t)(((uint32_t)(bits >> 31)) >> 1);
}

// Ordering key used by every top-k: larger value first, then smaller index.
// Packed so that a single unsigned 64-bit max picks the winner.
__device__ __forceinline__ unsigned long long rank_key(float v, uint32_t index) {
  uint32_t k = (uint32_t)total_key(v) ^ 0x80000000u;  // order-preserving to unsigned
  return ((unsigned long long)k << 32) | (unsigned long long)(0xffffffffu - index);
}

// ---------------------------------------------------------------------------
// formats
// ---------------------------------------------------------------------------

__host__ __device__ inline bool block_layout(int kind, int *elements, int *bytes) {
  switch (kind) {
    case DM_F32: *elements = 1; *bytes = 4; return true;
    case DM_F16: *elements = 1; *bytes = 2; return true;
    case DM_BF16: *elements = 1; *bytes = 2; return true;
    case DM_Q5_0: *elements = 32; *bytes = 22; return true;
    case DM_Q8_0: *elements = 32; *bytes = 34; return true;
    case DM_Q4_K: *elements = 256; *bytes = 144; return true;
    case DM_Q6_K: *elements = 256; *bytes = 210; return true;
    default: return false;
  }
}

// Row byte length of `columns` elements (src/gguf.rs:352-358); 0 when the column
// count is not a whole number of blocks.
__host__ __device__ inline uint64_t row_bytes(int kind, uint64_t columns) {
  int e = 0, b = 0;
  if (!block_layout(kind, &e, &b)) return 0;
  if (columns % (uint64_t)e) return 0;
  return columns / (uint64_t)e * (uint64_t)b;
}

// ---------------------------------------------------------------------------
// device-side unit decoders: 32 consecutive elements of one row.
// `row` points at the first byte of the row in the reference layout; `unit` is
// the index of the 32-element group within the row.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
  return (uint16_t)p[0] | ((uint16_t)p[1] << 8);
}

// src/cpu.rs:585-616: sub-block `sb` (0..7) of super-block `blk`. Low nibbles of
// quant bytes [32*(sb/2), +32) for even sb, high nibbles for odd sb.
struct Q4KUnit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const uint8_t *block = row + (unit >> 3) * 144;
    int sb = unit & 7;
    float d = f16_bits_to_f32(ld_u16(block));
    float dmin = f16_bits_to_f32(ld_u16(block + 2));
    const uint8_t *scales = block + 4;
    uint32_t sc, m;
    if (sb < 4) {
      sc = scales[sb] & 63;
      m = scales[sb + 4] & 63;
    } else {
      sc = (scales[sb + 4] & 0x0f) | ((scales[sb - 4] >> 6) << 4);
      m = (scales[sb + 4] >> 4) | ((scales[sb] >> 6) << 4);
    }
    float a = __fmul_rn(d, (float)sc);
    float b = __fmul_rn(dmin, (float)m);
    const uint4 *q = reinterpret_cast<const uint4 *>(block + 16 + 32 * (sb >> 1));
    int shift = (sb & 1) * 4;
#pragma unroll
    for (int v = 0; v < 2; v++) {
      uint4 chunk = q[v];
      uint32_t words[4] = {chunk.x, chunk.y, chunk.z, chunk.w};
#pragma unroll
      for (int i = 0; i < 16; i++) {
        uint32_t nib = (words[i >> 2] >> (8 * (i & 3) + shift)) & 0xf;
        w[16 * v + i] = __fsub_rn(__fmul_rn(a, (float)nib), b);
      }
    }
  }
};

// src/cpu.rs:618-645: element e of a block: half = e/128, quarter = (e%128)/32,
// idx = e%32; q from ql[half*64 + idx + 32*(quarter&1)] (low nibble for quarter<2),
// qh[half*32 + idx] bits 2*quarter, scale sc[half*8 + idx/16 + 2*quarter].
struct Q6KUnit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const uint8_t *block = row + (unit >> 3) * 210;
    int u = unit & 7;
    int half = u >> 2, quarter = u & 3;
    const uint8_t *ql = block + half * 64 + 32 * (quarter & 1);
    const uint8_t *qh = block + 128 + half * 32;
    const int8_t *sc = reinterpret_cast<const int8_t *>(block + 192 + half * 8 + 2 * quarter);
    float d = f16_bits_to_f32(ld_u16(block + 208));
    float s0 = __fmul_rn(d, (float)sc[0]);
    float s1 = __fmul_rn(d, (float)sc[1]);
    int lshift = (quarter >> 1) * 4;
    int hshift = 2 * quarter;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      uint32_t q = ((ql[i] >> lshift) & 0xf) | (((qh[i] >> hshift) & 3) << 4);
      w[i] = __fmul_rn(i < 16 ? s0 : s1, __fsub_rn((float)q, 32.0f));
    }
  }
};

// src/cpu.rs:560-574
struct Q50Unit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const uint8_t *block = row + unit * 22;
    float d = f16_bits_to_f32(ld_u16(block));
    uint32_t hb = (uint32_t)ld_u16(block + 2) | ((uint32_t)ld_u16(block + 4) << 16);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      uint32_t packed = block[6 + i];
      uint32_t lo = (packed & 0x0f) | (((hb >> i) << 4) & 0x10);
      uint32_t hi = (packed >> 4) | ((hb >> (i + 12)) & 0x10);
      w[i] = __fmul_rn(d, (float)((int)lo - 16));
      w[i + 16] = __fmul_rn(d, (float)((int)hi - 16));
    }
  }
};

// src/cpu.rs:576-583
struct Q80Unit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const uint8_t *block = row + unit * 34;
    float d = f16_bits_to_f32(ld_u16(block));
#pragma unroll
    for (int i = 0; i < 32; i++) w[i] = __fmul_rn(d, (float)(int8_t)block[2 + i]);
  }
};

struct BF16Unit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const uint4 *p = reinterpret_cast<const uint4 *>(row + unit * 64);
#pragma unroll
    for (int v = 0; v < 4; v++) {
      uint4 c = p[v];
      uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        w[8 * v + 2 * i] = __uint_as_float(words[i] << 16);
        w[8 * v + 2 * i + 1] = __uint_as_float(words[i] & 0xffff0000u);
      }
    }
  }
};

struct F16Unit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const uint16_t *p = reinterpret_cast<const uint16_t *>(row + unit * 64);
#pragma unroll
    for (int i = 0; i < 32; i++) w[i] = f16_bits_to_f32(p[i]);
  }
};

struct F32Unit {
  __device__ __forceinline__ static void decode(const uint8_t *row, int unit, float *w) {
    const float4 *p = reinterpret_cast<const float4 *>(row + unit * 128);
#pragma unroll
    for (int v = 0; v < 8; v++) {
      float4 c = p[v];
      w[4 * v] = c.x;
      w[4 * v + 1] = c.y;
      w[4 * v + 2] = c.z;
      w[4 * v + 3] = c.w;
    }
  }
};

// Allow a kernel the full 227 KB of dynamic shared memory, once per (kernel,
// device): the attribute persists, and raising the limit alone does not change a
// launch's occupancy (that follows the shared memory it actually requests).
cudaError_t ensure_smem_limit(const void *kernel);

// Programmatic dependent launch along the forward chain: a kernel launched this way may
// be scheduled while its predecessor runs, so it reads nothing its predecessor writes
// before pdl_wait(), which returns once the predecessor has completed and its writes are
// visible (and at once when the kernel was launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Let the next kernel of the stream launch now. Called right after pdl_wait() by the
// latency-bound kernels of the decode chain: every CTA of this grid is then resident or
// done, so the successor's CTAs take only spare room on the SMs and wait there, and its
// launch latency overlaps this kernel's work. Not called by a kernel whose successor is a
// one-wave, throughput-bound grid (the many-token router after the input transpose): CTAs
// placed around a running grid would pile onto the SMs it leaves free.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Scratch carved from one device allocation, 256-byte aligned pieces.
// Carves 256-byte-aligned pieces from one allocation; a request past the capacity
// returns null and sets `overflow` (the caller checks it once after carving).
struct Arena {
  uint8_t *base = nullptr;
  size_t used = 0, capacity = 0;
  bool overflow = false;
  template <class T>
  T *take(size_t count) {
    size_t bytes = (count * sizeof(T) + 255) & ~size_t(255);
    if (used + bytes > capacity) {
      overflow = true;
      return nullptr;
    }
    T *p = reinterpret_cast<T *>(base + used);
    used += bytes;
    return p;
  }
};

}  // namespace dm
