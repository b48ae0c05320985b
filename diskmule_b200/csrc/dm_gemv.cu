// dm_gemv.cu -- HBM-bound expert GEMV for decode-sized batches (see dm_gemv.cuh).
#include <algorithm>

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

#define DM_TASK_DOT_Q50(NT)                                                                     \
  template <>                                                                                   \
  __device__ __forceinline__ void task_dot<DM_Q5_0, NT>(const MatrixRef &m, int expert, int row, \
                                                        int task, const float *x, int kp,       \
                                                        const float *s16, int sp, int nt,       \
                                                        float *acc) {                           \
    const int nb = (int)(m.row_bytes / 22);                                                     \
    const uint64_t g = ((uint64_t)expert * m.rows + row) * nb + task;                           \
    const uint4 qs = ldg16(m.split.quant + g * 16);                                             \
    const uint32_t hb = *reinterpret_cast<const uint32_t *>(m.split.qh + g * 4);                \
    const float d = f16_bits_to_f32(m.split.d[g]);                                              \
    const uint32_t w[4] = {qs.x, qs.y, qs.z, qs.w};                                             \
    uint32_t lo[4], hi[4];                                                                      \
    _Pragma("unroll") for (int i = 0; i < 4; i++) {                                             \
      lo[i] = (w[i] & 0x0F0F0F0Fu) | spread4(hb >> (4 * i));                                   \
      hi[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | spread4(hb >> (16 + 4 * i));                        \
    }                                                                                           \
    _Pragma("unroll") for (int t = 0; t < NT; t++) {                                            \
      if (t < nt) {                                                                             \
        const float *xp = x + t * kp;                                                           \
        float sl = 0.0f, sh = 0.0f;                                                             \
        _Pragma("unroll") for (int i = 0; i < 4; i++) {                                         \
          sl = dot4(lo[i], *reinterpret_cast<const float4 *>(xp + 4 * i), sl);                  \
          sh = dot4(hi[i], *reinterpret_cast<const float4 *>(xp + 16 + 4 * i), sh);             \
        }                                                                                       \
        const float xl = s16[t * sp], xh = s16[t * sp + 1];                                     \
        float r = acc[t];                                                                       \
        r = fmaf(d, fmaf(256.0f, fmaf(-0.5f, xl, sl), -16.0f * xl), r);                         \
        r = fmaf(d, fmaf(256.0f, fmaf(-0.5f, xh, sh), -16.0f * xh), r);                         \
        acc[t] = r;                                                                             \
      }                                                                                         \
    }                                                                                           \
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
  if (KIND == DM_Q6_K || KIND == DM_Q5_0 || KIND == DM_Q8_0) {
    const int nb = (int)(m.row_bytes / (KIND == DM_Q6_K ? 210 : (KIND == DM_Q5_0 ? 22 : 34)));
    const uint64_t g = ((uint64_t)expert * m.rows + row) * nb + task;
    const int qb = KIND == DM_Q6_K ? 208 : (KIND == DM_Q5_0 ? 16 : 32);
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
  m.row_bytes = row_bytes(kind, cols);
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

template <int KIND, int NT>
static void launch_up(const ForwardArgs &a, const GemvPlan &p, cudaStream_t s) {
  if (is_dense(KIND)) return launch_dense_up<KIND, NT>(a, p, s);
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
    case DM_Q5_0: launch_up<DM_Q5_0, NT>(a, p, s); return true;
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
    case DM_Q5_0: launch_down<DM_Q5_0, NT>(a, p, s); return true;
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
