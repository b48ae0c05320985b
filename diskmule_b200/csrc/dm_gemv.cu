// dm_gemv.cu -- HBM-bound expert GEMV for decode-sized batches (see dm_gemv.cuh).
#include <algorithm>
#include <cstdlib>

#include "dm_gemv.cuh"
#include "dm_kernels.cuh"

namespace dm {

// ---------------------------------------------------------------------------
// repack of the 2-byte-aligned block formats (layer set-up, pure byte moves)
// ---------------------------------------------------------------------------

__global__ void repack_kernel(int kind, const uint8_t *src, uint64_t blocks, SplitTensor dst) {
  for (uint64_t g = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; g < blocks;
       g += (uint64_t)gridDim.x * blockDim.x) {
    if (kind == DM_Q6_K) {
      const uint8_t *b = src + g * 210;
      uint8_t *q = dst.quant + g * 208;
      for (int i = 0; i < 208; i++) q[i] = b[i];
      dst.d[g] = (uint16_t)(b[208] | (b[209] << 8));
    } else if (kind == DM_Q5_0) {
      const uint8_t *b = src + g * 22;
      dst.d[g] = (uint16_t)(b[0] | (b[1] << 8));
      for (int i = 0; i < 4; i++) dst.qh[g * 4 + i] = b[2 + i];
      for (int i = 0; i < 16; i++) dst.quant[g * 16 + i] = b[6 + i];
    } else if (kind == DM_Q8_0) {
      const uint8_t *b = src + g * 34;
      dst.d[g] = (uint16_t)(b[0] | (b[1] << 8));
      for (int i = 0; i < 32; i++) dst.quant[g * 32 + i] = b[2 + i];
    }
  }
}

int launch_repack(int kind, const uint8_t *src, uint64_t blocks, SplitTensor dst,
                  cudaStream_t stream) {
  if (blocks == 0) return 0;
  int grid = (int)((blocks + 255) / 256 < 4096 ? (blocks + 255) / 256 : 4096);
  repack_kernel<<<grid, 256, 0, stream>>>(kind, src, blocks, dst);
  return 1;
}

// ---------------------------------------------------------------------------
// per-format task dot products
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint4 ldg16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// f = 0.5 + byte_c(v)/256, exact for byte values below 128
__device__ __forceinline__ float magic(uint32_t v, int c) {
  return __uint_as_float(__byte_perm(v, 0x3F000000u, 0x7044u | ((uint32_t)c << 8)));
}

// sum over 4 bytes of a word: f(byte) * x
__device__ __forceinline__ float dot4(uint32_t q, float4 x, float s) {
  s = fmaf(magic(q, 0), x.x, s);
  s = fmaf(magic(q, 1), x.y, s);
  s = fmaf(magic(q, 2), x.z, s);
  s = fmaf(magic(q, 3), x.w, s);
  return s;
}

__device__ __forceinline__ float byte_f(uint32_t v, int c) { return (float)((v >> (8 * c)) & 0xff); }

// elements per task and x padding group
template <int KIND> struct Task;
template <> struct Task<DM_Q4_K> { static constexpr int kElems = 256; };
template <> struct Task<DM_Q6_K> { static constexpr int kElems = 256; };
template <> struct Task<DM_Q5_0> { static constexpr int kElems = 32; };
// Q5_0 with two blocks per task (rows whose length is a multiple of 64): half the threads,
// each with two blocks' loads in flight. An internal kernel choice, not a format.
constexpr int kQ50Pair = 1000 + DM_Q5_0;
template <> struct Task<kQ50Pair> { static constexpr int kElems = 64; };
template <> struct Task<DM_Q8_0> { static constexpr int kElems = 32; };
template <> struct Task<DM_BF16> { static constexpr int kElems = 128; };
template <> struct Task<DM_F16> { static constexpr int kElems = 64; };
template <> struct Task<DM_F32> { static constexpr int kElems = 64; };

// Where a matrix lives: reference layout (`base`, `stride` bytes per expert,
// `row_bytes`) or a split layout (`split`, indexed by the global block number).
struct MatrixRef {
  const uint8_t *base;
  uint64_t stride;
  uint64_t row_bytes;
  SplitTensor split;
  int rows;  // rows per expert
};

// x: this task's first element for token 0, token stride `kp`; s16: sums of each
// 16 consecutive x values (token stride `sp`), first group of this task.
template <int KIND, int NT>
__device__ __forceinline__ void task_dot(const MatrixRef &m, int expert, int row, int task,
                                         const float *x, int kp, const float *s16, int sp,
                                         int nt, float *acc);

template <>
__device__ __forceinline__ void task_dot<DM_Q4_K, 1>(const MatrixRef &m, int expert, int row,
                                                     int task, const float *x, int kp,
                                                     const float *s16, int sp, int nt,
                                                     float *acc);

#define DM_TASK_DOT_Q4K(NT)                                                                     \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<DM_Q4_K, NT>(const MatrixRef &m, int expert, int row, \
                                                        int task, const float *x, int kp,       \
                                                        const float *s16, int sp, int nt,       \
                                                        float *acc) {                           \
    const uint8_t *blk = m.base + (uint64_t)expert * m.stride + (uint64_t)row * m.row_bytes +   \
                         (uint64_t)task * 144;                                                  \
    uint4 hd = ldg16(blk);                                                                      \
    uint4 q[8];                                                                                 \
    _Pragma("unroll") for (int i = 0; i < 8; i++) q[i] = ldg16(blk + 16 + 16 * i);             \
    const float d = f16_bits_to_f32((uint16_t)(hd.x & 0xffff));                                 \
    const float dmin = f16_bits_to_f32((uint16_t)(hd.x >> 16));                                 \
    const uint32_t sca = hd.y & 0x3F3F3F3Fu, ma = hd.z & 0x3F3F3F3Fu;                           \
    const uint32_t scb = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);                    \
    const uint32_t mb = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);              \
    _Pragma("unroll") for (int gp = 0; gp < 4; gp++) {                                          \
      const int jl = 2 * gp, jh = 2 * gp + 1;                                                   \
      const float al = __fmul_rn(d, jl < 4 ? byte_f(sca, jl) : byte_f(scb, jl - 4));            \
      const float bl = __fmul_rn(dmin, jl < 4 ? byte_f(ma, jl) : byte_f(mb, jl - 4));           \
      const float ah = __fmul_rn(d, jh < 4 ? byte_f(sca, jh) : byte_f(scb, jh - 4));            \
      const float bh = __fmul_rn(dmin, jh < 4 ? byte_f(ma, jh) : byte_f(mb, jh - 4));           \
      const uint32_t w[8] = {q[2 * gp].x,     q[2 * gp].y,     q[2 * gp].z,     q[2 * gp].w,   \
                             q[2 * gp + 1].x, q[2 * gp + 1].y, q[2 * gp + 1].z, q[2 * gp + 1].w}; \
      uint32_t lo[8], hi[8];                                                                    \
      _Pragma("unroll") for (int i = 0; i < 8; i++) {                                           \
        lo[i] = w[i] & 0x0F0F0F0Fu;                                                             \
        hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;                                                      \
      }                                                                                         \
      _Pragma("unroll") for (int t = 0; t < NT; t++) {                                          \
        if (t < nt) {                                                                           \
          const float *xl = x + t * kp + 64 * gp, *xh = xl + 32;                                \
          float sl = 0.0f, sh = 0.0f;                                                           \
          _Pragma("unroll") for (int i = 0; i < 8; i++) {                                       \
            sl = dot4(lo[i], *reinterpret_cast<const float4 *>(xl + 4 * i), sl);                \
            sh = dot4(hi[i], *reinterpret_cast<const float4 *>(xh + 4 * i), sh);                \
          }                                                                                     \
          const float *sg = s16 + t * sp + 4 * gp;                                              \
          const float xl_sum = sg[0] + sg[1], xh_sum = sg[2] + sg[3];                           \
          float r = acc[t];                                                                     \
          r = fmaf(al, 256.0f * fmaf(-0.5f, xl_sum, sl), r);                                    \
          r = fmaf(-bl, xl_sum, r);                                                             \
          r = fmaf(ah, 256.0f * fmaf(-0.5f, xh_sum, sh), r);                                    \
          r = fmaf(-bh, xh_sum, r);                                                             \
          acc[t] = r;                                                                           \
        }                                                                                       \
      }                                                                                         \
    }                                                                                           \
  }
DM_TASK_DOT_Q4K(1)
DM_TASK_DOT_Q4K(2)
DM_TASK_DOT_Q4K(4)
#undef DM_TASK_DOT_Q4K

#define DM_TASK_DOT_Q6K(NT)                                                                     \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<DM_Q6_K, NT>(const MatrixRef &m, int expert, int row, \
                                                        int task, const float *x, int kp,       \
                                                        const float *s16, int sp, int nt,       \
                                                        float *acc) {                           \
    const int nb = (int)(m.row_bytes / 210);                                                    \
    const uint64_t g = ((uint64_t)expert * m.rows + row) * nb + task;                           \
    const uint8_t *blk = m.split.quant + g * 208;                                               \
    uint4 v[13];                                                                                \
    _Pragma("unroll") for (int i = 0; i < 13; i++) v[i] = ldg16(blk + 16 * i);                  \
    const float d = f16_bits_to_f32(m.split.d[g]);                                              \
    const uint32_t *ql = reinterpret_cast<const uint32_t *>(v);                                 \
    const uint32_t *qh = ql + 32;                                                               \
    const uint32_t *sc = ql + 48;                                                               \
    _Pragma("unroll") for (int h = 0; h < 2; h++) {                                             \
      uint32_t q[4][8];                                                                         \
      _Pragma("unroll") for (int i = 0; i < 8; i++) {                                           \
        const uint32_t l0 = ql[16 * h + i], l1 = ql[16 * h + 8 + i], hh = qh[8 * h + i];        \
        q[0][i] = (l0 & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u);                               \
        q[1][i] = (l1 & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u);                               \
        q[2][i] = ((l0 >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u);                               \
        q[3][i] = ((l1 >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u);                        \
      }                                                                                         \
      _Pragma("unroll") for (int qq = 0; qq < 4; qq++) {                                        \
        _Pragma("unroll") for (int g16 = 0; g16 < 2; g16++) {                                   \
          const int scale_index = 8 * h + g16 + 2 * qq;                                         \
          const float s = __fmul_rn(                                                            \
              d, (float)(int8_t)((sc[scale_index >> 2] >> (8 * (scale_index & 3))) & 0xff));    \
          _Pragma("unroll") for (int t = 0; t < NT; t++) {                                      \
            if (t < nt) {                                                                       \
              const float *xp = x + t * kp + 128 * h + 32 * qq + 16 * g16;                      \
              float S = 0.0f;                                                                   \
              _Pragma("unroll") for (int i = 0; i < 4; i++)                                     \
                S = dot4(q[qq][4 * g16 + i], *reinterpret_cast<const float4 *>(xp + 4 * i), S); \
              const float sx = s16[t * sp + 8 * h + 2 * qq + g16];                              \
              acc[t] = fmaf(s, fmaf(256.0f, fmaf(-0.5f, sx, S), -32.0f * sx), acc[t]);          \
            }                                                                                   \
          }                                                                                     \
        }                                                                                       \
      }                                                                                         \
    }                                                                                           \
  }
DM_TASK_DOT_Q6K(1)
DM_TASK_DOT_Q6K(2)
DM_TASK_DOT_Q6K(4)
#undef DM_TASK_DOT_Q6K

__device__ __forceinline__ uint32_t spread4(uint32_t v) {
  return ((v & 0xfu) * 0x02040810u) & 0x10101010u;
}

// One Q5_0 block (global block g) dotted with up to NT tokens' 32 x values.
template <int NT>
__device__ __forceinline__ void q50_block_dot(const MatrixRef &m, uint64_t g, const float *x, int kp,
                                              const float *s16, int sp, int nt, float *acc) {
  const uint4 qs = ldg16(m.split.quant + g * 16);
  const uint32_t hb = *reinterpret_cast<const uint32_t *>(m.split.qh + g * 4);
  const float d = f16_bits_to_f32(m.split.d[g]);
  const uint32_t w[4] = {qs.x, qs.y, qs.z, qs.w};
  uint32_t lo[4], hi[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    lo[i] = (w[i] & 0x0F0F0F0Fu) | spread4(hb >> (4 * i));
    hi[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | spread4(hb >> (16 + 4 * i));
  }
#pragma unroll
  for (int t = 0; t < NT; t++) {
    if (t < nt) {
      const float *xp = x + t * kp;
      float sl = 0.0f, sh = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        sl = dot4(lo[i], *reinterpret_cast<const float4 *>(xp + 4 * i), sl);
        sh = dot4(hi[i], *reinterpret_cast<const float4 *>(xp + 16 + 4 * i), sh);
      }
      const float xl = s16[t * sp], xh = s16[t * sp + 1];
      float r = acc[t];
      r = fmaf(d, fmaf(256.0f, fmaf(-0.5f, xl, sl), -16.0f * xl), r);
      r = fmaf(d, fmaf(256.0f, fmaf(-0.5f, xh, sh), -16.0f * xh), r);
      acc[t] = r;
    }
  }
}

#define DM_TASK_DOT_Q50(NT)                                                                     \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<DM_Q5_0, NT>(const MatrixRef &m, int expert, int row, \
                                                        int task, const float *x, int kp,       \
                                                        const float *s16, int sp, int nt,       \
                                                        float *acc) {                           \
    const int nb = (int)(m.row_bytes / 22);                                                     \
    q50_block_dot<NT>(m, ((uint64_t)expert * m.rows + row) * nb + task, x, kp, s16, sp, nt, acc); \
  }                                                                                             \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<kQ50Pair, NT>(const MatrixRef &m, int expert, int row, \
                                                         int task, const float *x, int kp,      \
                                                         const float *s16, int sp, int nt,      \
                                                         float *acc) {                          \
    const int nb = (int)(m.row_bytes / 22);                                                     \
    const uint64_t g = ((uint64_t)expert * m.rows + row) * nb + 2 * (uint64_t)task;             \
    q50_block_dot<NT>(m, g, x, kp, s16, sp, nt, acc);                                           \
    q50_block_dot<NT>(m, g + 1, x + 32, kp, s16 + 2, sp, nt, acc);                              \
  }
DM_TASK_DOT_Q50(1)
DM_TASK_DOT_Q50(2)
DM_TASK_DOT_Q50(4)
#undef DM_TASK_DOT_Q50

#define DM_TASK_DOT_Q80(NT)                                                                     \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<DM_Q8_0, NT>(const MatrixRef &m, int expert, int row, \
                                                        int task, const float *x, int kp,       \
                                                        const float *s16, int sp, int nt,       \
                                                        float *acc) {                           \
    const int nb = (int)(m.row_bytes / 34);                                                     \
    const uint64_t g = ((uint64_t)expert * m.rows + row) * nb + task;                           \
    const uint4 a = ldg16(m.split.quant + g * 32), b = ldg16(m.split.quant + g * 32 + 16);      \
    const float d = f16_bits_to_f32(m.split.d[g]);                                              \
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};                             \
    _Pragma("unroll") for (int t = 0; t < NT; t++) {                                            \
      if (t < nt) {                                                                             \
        const float *xp = x + t * kp;                                                           \
        float s = 0.0f;                                                                         \
        _Pragma("unroll") for (int i = 0; i < 8; i++) {                                         \
          const float4 xv = *reinterpret_cast<const float4 *>(xp + 4 * i);                      \
          const uint32_t u = w[i] ^ 0x80808080u; /* q + 128 */                                  \
          s = fmaf(__uint_as_float(0x4B000000u | (u & 0xff)) - 8388736.0f, xv.x, s);            \
          s = fmaf(__uint_as_float(0x4B000000u | ((u >> 8) & 0xff)) - 8388736.0f, xv.y, s);     \
          s = fmaf(__uint_as_float(0x4B000000u | ((u >> 16) & 0xff)) - 8388736.0f, xv.z, s);    \
          s = fmaf(__uint_as_float(0x4B000000u | (u >> 24)) - 8388736.0f, xv.w, s);             \
        }                                                                                       \
        acc[t] = fmaf(d, s, acc[t]);                                                            \
      }                                                                                         \
    }                                                                                           \
  }
DM_TASK_DOT_Q80(1)
DM_TASK_DOT_Q80(2)
DM_TASK_DOT_Q80(4)
#undef DM_TASK_DOT_Q80

#define DM_TASK_DOT_DENSE(KIND, NT)                                                             \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<KIND, NT>(const MatrixRef &m, int expert, int row,    \
                                                     int task, const float *x, int kp,          \
                                                     const float *s16, int sp, int nt,          \
                                                     float *acc) {                              \
    constexpr int kBytes = KIND == DM_F32 ? 256 : (KIND == DM_BF16 ? 256 : 128);                \
    const uint8_t *p = m.base + (uint64_t)expert * m.stride + (uint64_t)row * m.row_bytes +     \
                       (uint64_t)task * kBytes;                                                 \
    uint4 v[kBytes / 16];                                                                       \
    _Pragma("unroll") for (int i = 0; i < kBytes / 16; i++) v[i] = ldg16(p + 16 * i);          \
    constexpr int kElems = Task<KIND>::kElems;                                                  \
    float wv[kElems];                                                                           \
    _Pragma("unroll") for (int i = 0; i < kBytes / 16; i++) {                                   \
      const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};                                   \
      _Pragma("unroll") for (int j = 0; j < 4; j++) {                                           \
        if (KIND == DM_F32) {                                                                   \
          wv[4 * i + j] = __uint_as_float(u[j]);                                                \
        } else if (KIND == DM_BF16) {                                                           \
          wv[8 * i + 2 * j] = __uint_as_float(u[j] << 16);                                      \
          wv[8 * i + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);                          \
        } else {                                                                                \
          wv[8 * i + 2 * j] = f16_bits_to_f32((uint16_t)(u[j] & 0xffff));                       \
          wv[8 * i + 2 * j + 1] = f16_bits_to_f32((uint16_t)(u[j] >> 16));                      \
        }                                                                                       \
      }                                                                                         \
    }                                                                                           \
    _Pragma("unroll") for (int t = 0; t < NT; t++) {                                            \
      if (t < nt) {                                                                             \
        const float *xp = x + t * kp;                                                           \
        float s = acc[t];                                                                       \
        _Pragma("unroll") for (int i = 0; i < kElems; i += 4) {                                 \
          const float4 xv = *reinterpret_cast<const float4 *>(xp + i);                          \
          s = fmaf(wv[i], xv.x, s);                                                             \
          s = fmaf(wv[i + 1], xv.y, s);                                                         \
          s = fmaf(wv[i + 2], xv.z, s);                                                         \
          s = fmaf(wv[i + 3], xv.w, s);                                                         \
        }                                                                                       \
        acc[t] = s;                                                                             \
      }                                                                                         \
    }                                                                                           \
  }
DM_TASK_DOT_DENSE(DM_BF16, 1)
DM_TASK_DOT_DENSE(DM_BF16, 2)
DM_TASK_DOT_DENSE(DM_BF16, 4)
DM_TASK_DOT_DENSE(DM_F32, 1)
DM_TASK_DOT_DENSE(DM_F32, 2)
DM_TASK_DOT_DENSE(DM_F32, 4)
DM_TASK_DOT_DENSE(DM_F16, 1)
DM_TASK_DOT_DENSE(DM_F16, 2)
DM_TASK_DOT_DENSE(DM_F16, 4)
#undef DM_TASK_DOT_DENSE

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------

constexpr int kGemvThreads = 256;

__host__ __device__ __forceinline__ int pad_index(int k, int group) { return k + (k / group) * 4; }

// Stage `nt` rows of x (gathered by `row_of(t)`) into padded shared memory and
// compute the 16-element group sums.
template <int NT, class Load>
__device__ __forceinline__ void stage_rows(float *xs, float *s16, int K, int group, int nt,
                                           Load load) {
  const int kp = pad_index(K, group), k4 = K / 4;
#pragma unroll 4
  for (int idx = threadIdx.x; idx < nt * k4; idx += blockDim.x) {
    int t = idx / k4, k = 4 * (idx - t * k4);
    *reinterpret_cast<float4 *>(xs + t * kp + pad_index(k, group)) = load(t, k);
  }
  __syncthreads();
  const int groups = K / 16;
  for (int idx = threadIdx.x; idx < nt * groups; idx += blockDim.x) {
    int t = idx / groups, g = idx - t * groups;
    const float *p = xs + t * kp + pad_index(16 * g, group);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) s += p[i];
    s16[t * groups + g] = s;
  }
  __syncthreads();
}

__device__ __forceinline__ float act_fn(const ForwardArgs &a, int expert, float g, float u);

// Ask for the bytes of this thread's first task before x is staged, so the weight fetch
// from HBM overlaps the staging and the barriers.
template <int KIND>
__device__ __forceinline__ void prefetch_task(const MatrixRef &m, int expert, int row, int task) {
  const uint8_t *p;
  int bytes;
  if (KIND == DM_Q6_K || KIND == DM_Q5_0 || KIND == kQ50Pair || KIND == DM_Q8_0) {
    const bool q50 = KIND == DM_Q5_0 || KIND == kQ50Pair;
    const int nb = (int)(m.row_bytes / (KIND == DM_Q6_K ? 210 : (q50 ? 22 : 34)));
    const uint64_t g = ((uint64_t)expert * m.rows + row) * nb +
                       (uint64_t)task * (KIND == DM_Q6_K ? 1 : Task<KIND>::kElems / 32);
    const int qb = KIND == DM_Q6_K ? 208 : (q50 ? 16 : 32);
    p = m.split.quant + g * qb;
    bytes = qb * (KIND == DM_Q6_K ? 1 : Task<KIND>::kElems / 32);
  } else {
    const int tb = KIND == DM_Q4_K ? 144 : Task<KIND>::kElems * (KIND == DM_F32 ? 4 : 2);
    p = m.base + (uint64_t)expert * m.stride + (uint64_t)row * m.row_bytes + (uint64_t)task * tb;
    bytes = tb;
  }
  // every 128-byte line the task touches, into L1 (and L2 on the way): the task's loads
  // then find it on the SM once x is staged
  const uintptr_t first = (uintptr_t)p & ~(uintptr_t)127, last = ((uintptr_t)p + bytes - 1) & ~(uintptr_t)127;
  for (uintptr_t l = first; l <= last; l += 128)
    asm volatile("prefetch.global.L1 [%0];" ::"l"(l));
}

template <int KIND, int NT>
__global__ void __launch_bounds__(kGemvThreads) gemv_up_kernel(ForwardArgs a, MatrixRef gate,
                                                              MatrixRef up, MatrixRef sh_gate,
                                                              MatrixRef sh_up, int up_row_offset,
                                                              int rows_per_cta) {
  extern __shared__ __align__(16) float smem[];
  const int H = a.H, I = a.I;
  constexpr int kTask = Task<KIND>::kElems;
  const int kp = pad_index(H, kTask), groups = H / 16;
  float *xs = smem;
  float *s16 = xs + NT * kp;
  float *part = s16 + NT * groups;
  // One token: every work item reads row 0 of the input (or of Gemma's routed input, which
  // a kernel before the predecessor wrote), so it is staged before the wait, while the
  // predecessor finishes, instead of after the chain items -> offsets -> sorted -> row.
  const bool one = NT == 1 && a.T == 1;
  if (one && blockIdx.x * rows_per_cta < I)
    stage_rows<1>(xs, s16, H, kTask, 1, [&](int, int k) {
      if (a.family == kGemma) return *reinterpret_cast<const float4 *>(a.expert_in + k);
      if (a.input_bf16) {
        const uint2 u = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(a.x) + k);
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                           __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
      }
      return *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + k);
    });
  pdl_wait();
  pdl_trigger();
  if ((int)blockIdx.y >= *a.n_items) return;
  const int4 item = a.items[blockIdx.y];  // (expert, first token of the chunk, ...)
  const int e = item.x, c0 = item.y;
  const int base = a.offsets[e];
  const int nt = one ? 1 : min(NT, a.counts[e] - c0);
  const int nb = H / kTask;
  const int i0 = blockIdx.x * rows_per_cta;
  if (i0 >= I) return;
  const int nrows = min(rows_per_cta, I - i0);
  const bool shared = e == a.E;
  const MatrixRef &G = shared ? sh_gate : gate;
  const MatrixRef &U = shared ? sh_up : up;
  const int ex = shared ? 0 : e;
  const int tasks = 2 * nrows * nb;
  const int P = a.T * a.k;
  if ((int)threadIdx.x < tasks) {
    const int which = threadIdx.x / (nrows * nb), rem = threadIdx.x - which * nrows * nb;
    prefetch_task<KIND>(which ? U : G, ex, i0 + rem / nb + (which ? up_row_offset : 0), rem % nb);
  }
  if (!one) stage_rows<NT>(xs, s16, H, kTask, nt, [&](int t, int k) {
    int pair = a.sorted[base + c0 + t];
    int tok = pair < P ? pair / a.k : pair - P;
    size_t o = (size_t)tok * H + k;
    if (a.family == kGemma) return *reinterpret_cast<const float4 *>(a.expert_in + o);
    if (a.input_bf16) {
      const uint2 u = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(a.x) + o);
      return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                         __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
    }
    return *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + o);
  });
  for (int tau = threadIdx.x; tau < tasks; tau += blockDim.x) {
    const int which = tau / (nrows * nb);
    const int rem = tau - which * nrows * nb;
    const int r = rem / nb, b = rem - r * nb;
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    const int row = i0 + r + (which ? up_row_offset : 0);
    task_dot<KIND, NT>(which ? U : G, ex, row, b, xs + pad_index(b * kTask, kTask), kp,
                       s16 + b * (kTask / 16), groups, nt, acc);
#pragma unroll
    for (int t = 0; t < NT; t++) part[tau * NT + t] = acc[t];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nrows * nt; idx += blockDim.x) {
    const int r = idx / nt, t = idx - r * nt;
    float g = 0.0f, u = 0.0f;
    for (int b = 0; b < nb; b++) {
      g += part[((r * nb) + b) * NT + t];
      u += part[((nrows * nb) + r * nb + b) * NT + t];
    }
    a.h[(size_t)(base + c0 + t) * I + i0 + r] = act_fn(a, e, g, u);
  }
}

template <int KIND, int NT>
__global__ void __launch_bounds__(kGemvThreads) gemv_down_kernel(ForwardArgs a, MatrixRef down,
                                                                MatrixRef sh_down,
                                                                int rows_per_cta) {
  extern __shared__ __align__(16) float smem[];
  const int H = a.H, I = a.I;
  constexpr int kTask = Task<KIND>::kElems;
  const int nb = I / kTask;
  const int r0 = blockIdx.x * rows_per_cta;
  const int nrows = min(rows_per_cta, H - r0);
  const int tasks = nrows * nb;
  // The work items come from the dispatch two launches back, which completed before the
  // gate/up kernel let this grid launch: while that kernel still runs, ask L2 for this
  // CTA's down rows (read through L2, and only as prefetch addresses, so a line cached
  // from an earlier call cannot turn into a wrong result).
  if (r0 < H && (int)blockIdx.y < __ldcg(a.n_items) && (int)threadIdx.x < tasks) {
    const int ep = min(max(__ldcg(&a.items[blockIdx.y].x), 0), a.E);
    prefetch_task<KIND>(ep == a.E ? sh_down : down, ep == a.E ? 0 : ep, r0 + threadIdx.x / nb,
                        threadIdx.x % nb);
  }
  pdl_wait();
  pdl_trigger();
  if ((int)blockIdx.y >= *a.n_items) return;
  const int4 item = a.items[blockIdx.y];
  const int e = item.x, c0 = item.y;
  const int base = a.offsets[e];
  const int nt = min(NT, a.counts[e] - c0);
  if (r0 >= H) return;
  const int kp = pad_index(I, kTask), groups = I / 16;
  float *xs = smem;
  float *s16 = xs + NT * kp;
  float *part = s16 + NT * groups;
  const bool shared = e == a.E;
  const MatrixRef &D = shared ? sh_down : down;
  const int ex = shared ? 0 : e;
  stage_rows<NT>(xs, s16, I, kTask, nt,
                 [&](int t, int k) {
                   return *reinterpret_cast<const float4 *>(a.h + (size_t)(base + c0 + t) * I + k);
                 });
  for (int tau = threadIdx.x; tau < tasks; tau += blockDim.x) {
    const int r = tau / nb, b = tau - r * nb;
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    task_dot<KIND, NT>(D, ex, r0 + r, b, xs + pad_index(b * kTask, kTask), kp,
                       s16 + b * (kTask / 16), groups, nt, acc);
#pragma unroll
    for (int t = 0; t < NT; t++) part[tau * NT + t] = acc[t];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nrows * nt; idx += blockDim.x) {
    const int r = idx / nt, t = idx - r * nt;
    float s = 0.0f;
    for (int b = 0; b < nb; b++) s += part[(r * nb + b) * NT + t];
    a.ysorted[(size_t)(base + c0 + t) * H + r0 + r] = s;
  }
}

__device__ __forceinline__ float act_fn(const ForwardArgs &a, int expert, float g, float u) {
  if (a.family == kGemma) return __fmul_rn(gelu_tanh(g), u);
  if (a.family == kQwen) return __fmul_rn(qwen_silu(g), u);
  if (expert == a.E) return __fmul_rn(glm_silu(g), u);
  return __fmul_rn(glm_cached_silu(g), u);
}

// ---------------------------------------------------------------------------
// Q4_K gate/up on tensor-core tiles (mma.sync m16n8k16, f16 in, f32 accumulate)
//
// The f32 dot products above spend about six instructions per weight (byte placement,
// FMA, shared-memory loads of x), so a decode token's 13 MB of Q4_K rows took 15 us on
// instruction issue, not on HBM. Here the dot product of a block (256 columns) with up
// to four tokens is 16 MMAs per 16 rows, and a weight costs about one instruction:
//
//   w = d * sc_j * q - dmin * m_j   (q a nibble, sc_j / m_j the 6-bit scale and min of
//                                    the 32-column sub-block j)
//   sum_i w_i x_i = d * sum_i (q_i sc_j) x_i - dmin * sum_j m_j X_j,  X_j = sum_{i in j} x_i
//
// q * sc_j <= 945 is an integer, exact in f16: a PRMT places two quant bytes under an
// f16 exponent (1024 + q, or 1024 + 16 q for a high nibble) and one f16x2 FMA with
// (sc, -1024 sc) or (sc / 16, -64 sc) leaves q * sc exactly. Each token's x, scaled by a
// power of two per block so its largest value lies in [2^14, 2^15), is split into f16
// hi + lo halves (x = hi + lo to ~2^-22), two B columns of the MMA; the products are
// exact and sum in f32. So the result carries no weight rounding at all.
//
// Work: a CTA takes 16 gate rows and the same 16 up rows of one (expert, token chunk)
// item; warp w takes blocks w, w + warps, ... of the row. Lane (r = lane / 4,
// q = lane % 4) holds rows r and r + 8 of the tile (the A fragment's rows) and bytes
// [16q, 16q + 16) and [16q + 64, 16q + 80) of each row's 128 quant bytes; the MMA's K
// order is a permutation of the block's columns (the same one in A and B): MMA c of a
// piece uses the lane's bytes 2c and 2c + 1, their low nibbles as k = 2q, 2q + 1 and
// their high nibbles as k = 2q + 8, 2q + 9. Every 128-byte line of the warp's blocks is
// first requested into L1 (no registers held by bytes in flight); the lane's six 16-byte
// loads per matrix and block (two rows: header and two quant pieces) then find them there.
// The x fragments of a block are built once by the whole warp (shared memory), and the min
// terms dmin * sum_j m_j X_j run one row per lane. The partial sums of a row are added in
// a fixed order (deterministic).
// ---------------------------------------------------------------------------

constexpr int kMmaMaxWarps = 8;

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// two f32 -> f16x2 (lo in bits 0-15), round to nearest even
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ float f16_round(float v) {
  uint16_t h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(v));
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}

// The same f16 value in both halves of a register (v exactly representable).
__device__ __forceinline__ uint32_t splat_f16(float v) { return pack_f16x2(v, v); }

// Q4_K 6-bit scale (j < 8) and min of a block header (bytes 4..15 in y, z, w).
__device__ __forceinline__ uint32_t q4k_sc(const uint4 &hd, int j) {
  return j < 4 ? (hd.y >> (8 * j)) & 0x3F
               : ((hd.w >> (8 * (j - 4))) & 0x0F) | (((hd.y >> (8 * (j - 4))) >> 2) & 0x30);
}
__device__ __forceinline__ uint32_t q4k_m(const uint4 &hd, int j) {
  return j < 4 ? (hd.z >> (8 * j)) & 0x3F
               : ((hd.w >> (8 * (j - 4) + 4)) & 0x0F) | (((hd.z >> (8 * (j - 4))) >> 2) & 0x30);
}

// x of up to NT tokens, scaled and split for the B fragments of one block; see the
// kernel. Only lanes 0 .. 8 NT - 1 hold nonzero B values (columns 2t, 2t + 1).
template <int NT>
struct MmaBlockX {
  uint2 frag[2][8][8 * NT];  // [piece slot][MMA][lane]: {b0b1, b2b3}
  float xsum[NT][8];         // [token][sub-block] unscaled sums
  float inv[NT];             // [token] 2^-s
};

template <int NT, class RowPtr>
__device__ __forceinline__ void mma_build_x(MmaBlockX<NT> &bx, int b, int nt, RowPtr row_ptr) {
  // Lane l converts columns [8l, 8l + 8) of the block for every token. Column e sits in
  // piece P = 2 (e / 64) + (e % 32) / 16 (lane q = P % 4, slot P / 4), MMA (e % 16) / 2,
  // register (e % 64) / 32 (low or high nibbles), half e % 2.
  const int lane = threadIdx.x & 31, e0 = 8 * lane;
  const int P = 2 * (e0 >> 6) + ((e0 & 31) >> 4);
  const int q = P & 3, ps = P >> 2, reg = (e0 & 63) >> 5, c0 = (e0 & 15) >> 1;
  uint32_t *frag = reinterpret_cast<uint32_t *>(&bx.frag[0][0][0]);
  for (int t = 0; t < nt && t < NT; t++) {
    const float *xr = row_ptr(t) + 256 * b + e0;
    const float4 u = *reinterpret_cast<const float4 *>(xr);
    const float4 w = *reinterpret_cast<const float4 *>(xr + 4);
    const float x[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
    float mx = 0.0f, sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      mx = fmaxf(mx, fabsf(x[i]));
      sum = __fadd_rn(sum, x[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // the 32-column sub-block (lanes 4s .. 4s + 3): sum of the four lanes' sums
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
    sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
    // scale 2^s with mx * 2^s in [2^14, 2^15); 1 for zero or non-finite rows
    int sh = 0;
    if (mx > 0.0f && mx <= 3.0e38f) {
      const int ex = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;
      sh = min(max(14 - ex, -126), 126);
    }
    const float scale = __uint_as_float((uint32_t)(127 + sh) << 23);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float v0 = x[2 * i] * scale, v1 = x[2 * i + 1] * scale;
      const float h0 = f16_round(v0), h1 = f16_round(v1);
      const int slot = ((ps * 8 + c0 + i) * (8 * NT) + 8 * t + q) * 2 + reg;
      frag[slot] = pack_f16x2(h0, h1);                                   // column 2t: hi
      frag[slot + 8] = pack_f16x2(__fsub_rn(v0, h0), __fsub_rn(v1, h1));  // column 2t + 1: lo
    }
    if ((lane & 3) == 0) bx.xsum[t][lane >> 2] = sum;
    if (lane == 0) bx.inv[t] = __uint_as_float((uint32_t)(127 - sh) << 23);
  }
}

template <int NT>
__global__ void __launch_bounds__(32 * kMmaMaxWarps, 3) gemv_up_q4k_mma_kernel(
    ForwardArgs a, MatrixRef gate, MatrixRef up, MatrixRef sh_gate, MatrixRef sh_up,
    int up_row_offset) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int H = a.H, I = a.I, nb = H / 256;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int q = lane & 3, rr = lane >> 2;
  MmaBlockX<NT> *bx = reinterpret_cast<MmaBlockX<NT> *>(smem_raw);    // [nb]
  float *part = reinterpret_cast<float *>(bx + nb);                   // [nw][NT][32]
  float *partm = part + nw * NT * 32;                                 // [nw][NT][32]
  const bool one = NT == 1 && a.T == 1;
  // One token: every item reads row 0 of the input, which does not depend on the
  // dispatch, so its fragments are built while the predecessor finishes.
  auto x_row = [&](int tok) -> const float * {
    return a.family == kGemma ? a.expert_in + (size_t)tok * H
                              : reinterpret_cast<const float *>(a.x) + (size_t)tok * H;
  };
  if (one)
    for (int b = warp; b < nb; b += nw) mma_build_x<NT>(bx[b], b, 1, [&](int) { return x_row(0); });
  pdl_wait();
  pdl_trigger();
  if ((int)blockIdx.y >= *a.n_items) return;
  // (expert, first token within it, its sorted position, tokens): no further lookups
  const int4 item = a.items[blockIdx.y];
  const int e = item.x, pos0 = item.z;
  const int nt = one ? 1 : min(NT, item.w);
  const int i0 = blockIdx.x * 16;
  const bool shared = e == a.E;
  const MatrixRef &G = shared ? sh_gate : gate;
  const MatrixRef &U = shared ? sh_up : up;
  const int ex = shared ? 0 : e;
  const uint8_t *gp0 = G.base + (uint64_t)ex * G.stride + (uint64_t)(i0 + rr) * G.row_bytes;
  const uint8_t *up0 =
      U.base + (uint64_t)ex * U.stride + (uint64_t)(i0 + rr + up_row_offset) * U.row_bytes;
  const uint64_t r8g = 8 * G.row_bytes, r8u = 8 * U.row_bytes;
  float val[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // gate r, gate r + 8, up r, up r + 8 (token q)
  // Lane l's row for the prefetches and the min terms: row l % 16 of gate (l < 16) or up.
  const uint8_t *row_l = lane < 16 ? gp0 + ((int64_t)(lane & 15) - rr) * (int64_t)G.row_bytes
                                   : up0 + ((int64_t)(lane & 15) - rr) * (int64_t)U.row_bytes;
  // Every line of the warp's blocks is requested into L1 first, so all of the bytes are in
  // flight without holding registers; the loads of each matrix then find them there.
  for (int b = warp; b < nb; b += nw) {
    const uint8_t *p = row_l + (uint64_t)b * 144;
    const uintptr_t first = (uintptr_t)p & ~(uintptr_t)127, last = ((uintptr_t)p + 143) & ~(uintptr_t)127;
    for (uintptr_t l = first; l <= last; l += 128) asm volatile("prefetch.global.L1 [%0];" ::"l"(l));
  }
  // several tokens: their rows come from the dispatch (built after the prefetches)
  if (!one) {
    const int P = a.T * a.k;
    for (int b = warp; b < nb; b += nw)
      mma_build_x<NT>(bx[b], b, nt, [&](int t) {
        const int pair = a.sorted[pos0 + t];
        return x_row(pair < P ? pair / a.k : pair - P);
      });
  }
  __syncwarp();
  float mval[NT];  // lane l's row: sum over blocks of dmin * sum_j m_j X_j, per token
#pragma unroll
  for (int t = 0; t < NT; t++) mval[t] = 0.0f;
  for (int b = warp; b < nb; b += nw) {
    const MmaBlockX<NT> &X = bx[b];
#pragma unroll
    for (int m = 0; m < 2; m++) {
      // [row][header, piece q, piece q + 4]
      uint4 v[2][3];
#pragma unroll
      for (int r = 0; r < 2; r++) {
        const uint8_t *p = (m ? up0 + (r ? r8u : 0) : gp0 + (r ? r8g : 0)) + (uint64_t)b * 144;
        v[r][0] = ldg16(p);
        v[r][1] = ldg16(p + 16 + 16 * q);
        v[r][2] = ldg16(p + 16 + 16 * (q + 4));
      }
      float dacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int ps = 0; ps < 2; ps++) {
        const int j = 2 * (ps * 2 + (q >> 1));  // sub-block of the low nibbles; j + 1 high
        uint32_t ml[2], al[2], mh[2], ah[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
          const float scl = (float)q4k_sc(v[r][0], j), sch = (float)q4k_sc(v[r][0], j + 1);
          ml[r] = splat_f16(scl);
          al[r] = splat_f16(-1024.0f * scl);
          mh[r] = splat_f16(0.0625f * sch);
          ah[r] = splat_f16(-64.0f * sch);
        }
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const uint32_t sel = (c & 1) ? 0x4342u : 0x4140u;
          uint32_t w[2];
#pragma unroll
          for (int r = 0; r < 2; r++) {
            const uint4 &pc = v[r][1 + ps];
            w[r] = __byte_perm(c < 2 ? pc.x : c < 4 ? pc.y : c < 6 ? pc.z : pc.w, 0x64646464u, sel);
          }
          const uint32_t a0 = hfma2_bits(w[0] & 0xFF0FFF0Fu, ml[0], al[0]);
          const uint32_t a1 = hfma2_bits(w[1] & 0xFF0FFF0Fu, ml[1], al[1]);
          const uint32_t a2 = hfma2_bits(w[0] & 0xFFF0FFF0u, mh[0], ah[0]);
          const uint32_t a3 = hfma2_bits(w[1] & 0xFFF0FFF0u, mh[1], ah[1]);
          const uint2 f = lane < 8 * NT ? X.frag[ps][c][lane] : make_uint2(0u, 0u);
          mma_16816(dacc, a0, a1, a2, a3, f.x, f.y);
        }
      }
      if (q < nt) {
        const float inv = X.inv[q];
#pragma unroll
        for (int r = 0; r < 2; r++) {
          const float d = f16_bits_to_f32((uint16_t)(v[r][0].x & 0xffff));
          const float dot = __fmul_rn(__fadd_rn(dacc[2 * r], dacc[2 * r + 1]), inv);
          val[2 * m + r] = __fmaf_rn(d, dot, val[2 * m + r]);
        }
      }
    }
    // the min terms, one row per lane
    {
      const uint4 hd = ldg16(row_l + (uint64_t)b * 144);
      const float dmin = f16_bits_to_f32((uint16_t)(hd.x >> 16));
      float mj[8];
#pragma unroll
      for (int j = 0; j < 8; j++) mj[j] = (float)q4k_m(hd, j);
#pragma unroll
      for (int t = 0; t < NT; t++) {
        if (t < nt) {
          float mins = 0.0f;
#pragma unroll
          for (int j = 0; j < 8; j++) mins = __fmaf_rn(mj[j], X.xsum[t][j], mins);
          mval[t] = __fmaf_rn(dmin, mins, mval[t]);
        }
      }
    }
  }
  if (q < nt) {
    float *pw = part + ((size_t)warp * NT + q) * 32;
    pw[rr] = val[0];
    pw[rr + 8] = val[1];
    pw[16 + rr] = val[2];
    pw[16 + rr + 8] = val[3];
  }
#pragma unroll
  for (int t = 0; t < NT; t++)
    if (t < nt) partm[((size_t)warp * NT + t) * 32 + lane] = mval[t];
  __syncthreads();
  for (int idx = threadIdx.x; idx < 16 * nt; idx += blockDim.x) {
    const int r = idx & 15, t = idx >> 4;
    float g = 0.0f, u = 0.0f;
    for (int w = 0; w < nw; w++) {
      const size_t o = ((size_t)w * NT + t) * 32;
      g = __fadd_rn(g, __fsub_rn(part[o + r], partm[o + r]));
      u = __fadd_rn(u, __fsub_rn(part[o + 16 + r], partm[o + 16 + r]));
    }
    a.h[(size_t)(pos0 + t) * I + i0 + r] = act_fn(a, e, g, u);
  }
}

// ---------------------------------------------------------------------------
// dense weights (BF16 / F16 / F32): one warp per row, coalesced 512-byte loads
//
// A warp streams a row as 512-byte pieces (lane l takes bytes 16·(l + 32i) .. +16), with
// four pieces in flight per matrix, and dots them with the x rows staged once per CTA in
// shared memory as f32; each CTA covers many rows, so the staging is a few percent of
// the weight bytes even at H = 6144. Row sums are a fixed shuffle tree (deterministic).
// ---------------------------------------------------------------------------

template <int KIND>
__device__ __forceinline__ void dense_unpack(const uint4 v, float *w) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; j++) {
    if (KIND == DM_BF16) {
      w[2 * j] = __uint_as_float(u[j] << 16);
      w[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
    } else if (KIND == DM_F16) {
      w[2 * j] = f16_bits_to_f32((uint16_t)(u[j] & 0xffff));
      w[2 * j + 1] = f16_bits_to_f32((uint16_t)(u[j] >> 16));
    } else {
      w[j] = __uint_as_float(u[j]);
    }
  }
}

// Elements per 16-byte piece.
template <int KIND> struct DenseElems { static constexpr int kN = KIND == DM_F32 ? 4 : 8; };

// acc[t] += row . x_t over one row of `chunks` 16-byte pieces (this lane's share).
template <int KIND, int NT>
__device__ __forceinline__ void dense_row_dot(const uint8_t *__restrict__ row, int chunks,
                                              const float *xs, int xld, int nt, float *acc) {
  constexpr int kE = DenseElems<KIND>::kN;
  const int lane = threadIdx.x & 31;
  constexpr int kU = 4;
  for (int c0 = lane; c0 < chunks; c0 += 32 * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; u++) {
      const int c = c0 + 32 * u;
      v[u] = c < chunks ? ldg16(row + 16 * (size_t)c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kU; u++) {
      const int c = c0 + 32 * u;
      if (c >= chunks) break;
      float w[kE];
      dense_unpack<KIND>(v[u], w);
#pragma unroll
      for (int t = 0; t < NT; t++) {
        if (t < nt) {
          const float *xp = xs + t * xld + c * kE;
          float s = acc[t];
#pragma unroll
          for (int i = 0; i < kE; i += 4) {
            const float4 xv = *reinterpret_cast<const float4 *>(xp + i);
            s = fmaf(w[i], xv.x, s);
            s = fmaf(w[i + 1], xv.y, s);
            s = fmaf(w[i + 2], xv.z, s);
            s = fmaf(w[i + 3], xv.w, s);
          }
          acc[t] = s;
        }
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kDenseThreads = 256;

template <int KIND, int NT>
__global__ void __launch_bounds__(kDenseThreads) dense_up_kernel(ForwardArgs a, MatrixRef gate,
                                                                 MatrixRef up, MatrixRef sh_gate,
                                                                 MatrixRef sh_up,
                                                                 int up_row_offset,
                                                                 int rows_per_cta) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float smem[];
  if ((int)blockIdx.y >= *a.n_items) return;
  const int4 item = a.items[blockIdx.y];
  const int e = item.x, c0 = item.y;
  const int base = a.offsets[e];
  const int nt = min(NT, a.counts[e] - c0);
  const int H = a.H, I = a.I;
  const int i0 = blockIdx.x * rows_per_cta;
  if (i0 >= I) return;
  const int nrows = min(rows_per_cta, I - i0);
  const bool shared = e == a.E;
  const MatrixRef &G = shared ? sh_gate : gate;
  const MatrixRef &U = shared ? sh_up : up;
  const int ex = shared ? 0 : e;
  const int P = a.T * a.k;
  const int xld = H + 4;
  float *xs = smem;
  // stage the x rows of this item's tokens as f32
  for (int idx = threadIdx.x; idx < nt * (H / 4); idx += blockDim.x) {
    const int t = idx / (H / 4), k = 4 * (idx - t * (H / 4));
    const int pair = a.sorted[base + c0 + t];
    const int tok = pair < P ? pair / a.k : pair - P;
    const size_t o = (size_t)tok * H + k;
    float4 v;
    if (a.family == kGemma) {
      v = *reinterpret_cast<const float4 *>(a.expert_in + o);
    } else if (a.input_bf16) {
      const uint2 q = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(a.x) + o);
      v = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xffff0000u),
                      __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xffff0000u));
    } else {
      v = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + o);
    }
    *reinterpret_cast<float4 *>(xs + t * xld + k) = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (int)(G.row_bytes / 16);
  for (int r = warp; r < nrows; r += kDenseThreads / 32) {
    const int row = i0 + r;
    float g[NT], u[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) g[t] = u[t] = 0.0f;
    dense_row_dot<KIND, NT>(G.base + (uint64_t)ex * G.stride + (uint64_t)row * G.row_bytes, chunks,
                            xs, xld, nt, g);
    dense_row_dot<KIND, NT>(U.base + (uint64_t)ex * U.stride +
                                (uint64_t)(row + up_row_offset) * U.row_bytes,
                            chunks, xs, xld, nt, u);
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float gs = warp_sum(g[t]), us = warp_sum(u[t]);
      if (lane == 0 && t < nt) a.h[(size_t)(base + c0 + t) * I + row] = act_fn(a, e, gs, us);
    }
  }
}

template <int KIND, int NT>
__global__ void __launch_bounds__(kDenseThreads) dense_down_kernel(ForwardArgs a, MatrixRef down,
                                                                   MatrixRef sh_down,
                                                                   int rows_per_cta) {
  extern __shared__ __align__(16) float smem[];
  const int H = a.H, I = a.I;
  const int r0 = blockIdx.x * rows_per_cta;
  const int nrows = min(rows_per_cta, H - r0);
  pdl_wait();
  pdl_trigger();
  if ((int)blockIdx.y >= *a.n_items) return;
  const int4 item = a.items[blockIdx.y];
  const int e = item.x, c0 = item.y;
  const int base = a.offsets[e];
  const int nt = min(NT, a.counts[e] - c0);
  if (r0 >= H) return;
  const bool shared = e == a.E;
  const MatrixRef &D = shared ? sh_down : down;
  const int ex = shared ? 0 : e;
  const int xld = I + 4;
  float *xs = smem;
  for (int idx = threadIdx.x; idx < nt * (I / 4); idx += blockDim.x) {
    const int t = idx / (I / 4), k = 4 * (idx - t * (I / 4));
    *reinterpret_cast<float4 *>(xs + t * xld + k) =
        *reinterpret_cast<const float4 *>(a.h + (size_t)(base + c0 + t) * I + k);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (int)(D.row_bytes / 16);
  for (int r = warp; r < nrows; r += kDenseThreads / 32) {
    const int row = r0 + r;
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t] = 0.0f;
    dense_row_dot<KIND, NT>(D.base + (uint64_t)ex * D.stride + (uint64_t)row * D.row_bytes, chunks,
                            xs, xld, nt, acc);
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float s = warp_sum(acc[t]);
      if (lane == 0 && t < nt) a.ysorted[(size_t)(base + c0 + t) * H + row] = s;
    }
  }
}

// ---------------------------------------------------------------------------
// launcher
// ---------------------------------------------------------------------------

static MatrixRef matrix(int kind, const uint8_t *base, uint64_t stride, int rows, int cols,
                        SplitTensor split) {
  MatrixRef m;
  m.base = base;
  m.stride = stride;
  m.row_bytes = row_bytes(kind == kQ50Pair ? DM_Q5_0 : kind, cols);
  m.split = split;
  m.rows = rows;
  return m;
}

constexpr bool is_dense(int kind) { return kind == DM_BF16 || kind == DM_F16 || kind == DM_F32; }

// Rows per CTA of the dense kernels: 32 rows make the x staging (one row of f32 per
// token) about 3% of the weight bytes; fewer when the grid would not fill the SMs twice.
static int dense_rows(int rows_total, int items) {
  int r = 32;
  while (r > 8 && (long)((rows_total + r - 1) / r) * items < 2L * 148) r /= 2;
  return r;
}

template <int KIND, int NT>
static void launch_dense_up(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  const int up_rows = a.family == kGemma ? 2 * a.I : a.I;
  MatrixRef g = matrix(KIND, a.gate, a.gate_stride, up_rows, a.H, p.gate);
  MatrixRef u = matrix(KIND, a.family == kGemma ? a.gate : a.up, a.up_stride, up_rows, a.H, p.up);
  MatrixRef sg = matrix(KIND, a.sh_gate, 0, a.I, a.H, p.sh_gate);
  MatrixRef su = matrix(KIND, a.sh_up, 0, a.I, a.H, p.sh_up);
  const int rows = dense_rows(a.I, p.max_items);
  const size_t smem = (size_t)NT * (a.H + 4) * 4;
  auto fn = dense_up_kernel<KIND, NT>;
  if (smem > 48 * 1024) ensure_smem_limit((const void *)fn);
  dim3 grid((a.I + rows - 1) / rows, p.max_items);
  launch_pdl(fn, grid, dim3(kDenseThreads), smem, s, a, g, u, sg, su, a.family == kGemma ? a.I : 0, rows);
}

template <int KIND, int NT>
static void launch_dense_down(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  MatrixRef d = matrix(KIND, a.down, a.down_stride, a.H, a.I, p.down);
  MatrixRef sd = matrix(KIND, a.sh_down, 0, a.H, a.I, p.sh_down);
  const int rows = dense_rows(a.H, p.max_items);
  const size_t smem = (size_t)NT * (a.I + 4) * 4;
  auto fn = dense_down_kernel<KIND, NT>;
  if (smem > 48 * 1024) ensure_smem_limit((const void *)fn);
  dim3 grid((a.H + rows - 1) / rows, p.max_items);
  launch_pdl(fn, grid, dim3(kDenseThreads), smem, s, a, d, sd, rows);
}

// Threads per CTA of the quantised GEMVs (a thread per task): halved from 256 while the
// grid has fewer than four CTAs per SM, so that few-token launches (a decode token reads
// k experts) spread evenly over the 148 SMs instead of leaving some SMs a third CTA
// while others idle.
static int quant_threads(int rows_total, int tasks_per_row, int items) {
  int threads = kGemvThreads;
  while (threads > 64) {
    const int rows = std::max(1, threads / tasks_per_row);
    if ((long)((rows_total + rows - 1) / rows) * items >= 4L * 148) break;
    threads >>= 1;
  }
  return threads;
}

// Q4_K gate/up through gemv_up_q4k_mma_kernel (DISKMULE_CUDA_GEMV_MMA=0 keeps the f32
// dot products): rows in tiles of 16, so I must be a multiple of 16, and the x fragments
// of a whole row (4.2 KB per 256 columns at four tokens) must fit shared memory.
static bool use_q4k_mma(const ForwardArgs &a) {
  static const bool enabled = [] {
    const char *env = getenv("DISKMULE_CUDA_GEMV_MMA");
    return !(env && env[0] == '0');
  }();
  const size_t smem_bound = (size_t)(a.H / 256) * sizeof(MmaBlockX<4>) +
                            (size_t)2 * kMmaMaxWarps * 4 * 32 * sizeof(float);
  return enabled && a.I % 16 == 0 && a.H % 256 == 0 && !a.input_bf16 && smem_bound <= 200 * 1024;
}

template <int NT>
static void launch_up_q4k_mma(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  const int nb = a.H / 256;
  const int per_warp = (nb + kMmaMaxWarps - 1) / kMmaMaxWarps;  // blocks of a row per warp
  const int warps = (nb + per_warp - 1) / per_warp;
  const size_t smem = (size_t)nb * sizeof(MmaBlockX<NT>) + (size_t)2 * warps * NT * 32 * sizeof(float);
  auto fn = gemv_up_q4k_mma_kernel<NT>;
  if (smem > 48 * 1024) ensure_smem_limit((const void *)fn);
  const int up_rows = a.family == kGemma ? 2 * a.I : a.I;
  MatrixRef g = matrix(DM_Q4_K, a.gate, a.gate_stride, up_rows, a.H, p.gate);
  MatrixRef u = matrix(DM_Q4_K, a.family == kGemma ? a.gate : a.up, a.up_stride, up_rows, a.H, p.up);
  MatrixRef sg = matrix(DM_Q4_K, a.sh_gate, 0, a.I, a.H, p.sh_gate);
  MatrixRef su = matrix(DM_Q4_K, a.sh_up, 0, a.I, a.H, p.sh_up);
  launch_pdl(fn, dim3(a.I / 16, p.max_items), dim3(32 * warps), smem, s, a, g, u, sg, su,
             a.family == kGemma ? a.I : 0);
}

template <int KIND, int NT>
static void launch_up(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  if (is_dense(KIND)) return launch_dense_up<KIND, NT>(a, p, s);
  if (KIND == DM_Q4_K && use_q4k_mma(a)) return launch_up_q4k_mma<NT>(a, p, s);
  constexpr int kTask = Task<KIND>::kElems;
  const int nb = a.H / kTask;
  const int threads = quant_threads(a.I, 2 * nb, p.max_items);
  const int rows = std::max(1, threads / (2 * nb));
  const size_t smem = (size_t)NT * (pad_index(a.H, kTask) + a.H / 16) * 4 +
                      (size_t)2 * rows * nb * NT * 4;
  auto fn = gemv_up_kernel<KIND, NT>;
  if (smem > 48 * 1024) ensure_smem_limit((const void *)fn);
  dim3 grid((a.I + rows - 1) / rows, p.max_items);
  const int up_rows = a.family == kGemma ? 2 * a.I : a.I;
  MatrixRef g = matrix(KIND, a.gate, a.gate_stride, up_rows, a.H, p.gate);
  MatrixRef u = matrix(KIND, a.family == kGemma ? a.gate : a.up, a.up_stride, up_rows, a.H, p.up);
  MatrixRef sg = matrix(KIND, a.sh_gate, 0, a.I, a.H, p.sh_gate);
  MatrixRef su = matrix(KIND, a.sh_up, 0, a.I, a.H, p.sh_up);
  launch_pdl(fn, grid, dim3(threads), smem, s, a, g, u, sg, su, a.family == kGemma ? a.I : 0, rows);
}

template <int KIND, int NT>
static void launch_down(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  if (is_dense(KIND)) return launch_dense_down<KIND, NT>(a, p, s);
  constexpr int kTask = Task<KIND>::kElems;
  const int nb = a.I / kTask;
  const int threads = quant_threads(a.H, nb, p.max_items);
  const int rows = std::max(1, threads / nb);
  const size_t smem = (size_t)NT * (pad_index(a.I, kTask) + a.I / 16) * 4 +
                      (size_t)rows * nb * NT * 4;
  auto fn = gemv_down_kernel<KIND, NT>;
  if (smem > 48 * 1024) ensure_smem_limit((const void *)fn);
  dim3 grid((a.H + rows - 1) / rows, p.max_items);
  MatrixRef d = matrix(KIND, a.down, a.down_stride, a.H, a.I, p.down);
  MatrixRef sd = matrix(KIND, a.sh_down, 0, a.H, a.I, p.sh_down);
  launch_pdl(fn, grid, dim3(threads), smem, s, a, d, sd, rows);
}

template <int NT>
static bool dispatch_up(int kind, const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  switch (kind) {
    case DM_Q4_K: launch_up<DM_Q4_K, NT>(a, p, s); return true;
    case DM_Q6_K: launch_up<DM_Q6_K, NT>(a, p, s); return true;
    case DM_Q5_0:
      if (a.H % 64 == 0) launch_up<kQ50Pair, NT>(a, p, s);
      else launch_up<DM_Q5_0, NT>(a, p, s);
      return true;
    case DM_Q8_0: launch_up<DM_Q8_0, NT>(a, p, s); return true;
    case DM_BF16: launch_up<DM_BF16, NT>(a, p, s); return true;
    case DM_F16: launch_up<DM_F16, NT>(a, p, s); return true;
    case DM_F32: launch_up<DM_F32, NT>(a, p, s); return true;
    default: return false;
  }
}

template <int NT>
static bool dispatch_down(int kind, const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  switch (kind) {
    case DM_Q4_K: launch_down<DM_Q4_K, NT>(a, p, s); return true;
    case DM_Q6_K: launch_down<DM_Q6_K, NT>(a, p, s); return true;
    case DM_Q5_0:
      if (a.I % 64 == 0) launch_down<kQ50Pair, NT>(a, p, s);
      else launch_down<DM_Q5_0, NT>(a, p, s);
      return true;
    case DM_Q8_0: launch_down<DM_Q8_0, NT>(a, p, s); return true;
    case DM_BF16: launch_down<DM_BF16, NT>(a, p, s); return true;
    case DM_F16: launch_down<DM_F16, NT>(a, p, s); return true;
    case DM_F32: launch_down<DM_F32, NT>(a, p, s); return true;
    default: return false;
  }
}

int launch_gemv_experts(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s,
                        cudaEvent_t down_mark) {
  bool ok;
  if (p.nt == 1) ok = dispatch_up<1>(a.gate_type, a, p, s);
  else if (p.nt == 2) ok = dispatch_up<2>(a.gate_type, a, p, s);
  else ok = dispatch_up<4>(a.gate_type, a, p, s);
  if (!ok) return -1;
  if (down_mark) cudaEventRecord(down_mark, s);
  if (p.nt == 1) ok = dispatch_down<1>(a.down_type, a, p, s);
  else if (p.nt == 2) ok = dispatch_down<2>(a.down_type, a, p, s);
  else ok = dispatch_down<4>(a.down_type, a, p, s);
  return ok ? 2 : -1;
}

}  // namespace dm
