/*
 * dm_oracle.c -- CPU restatement of DiskMule's routed-expert (MoE) path.
 *
 * TEST INFRASTRUCTURE ONLY (see dm_oracle.h).  Compiled with -ffp-contract=off so
 * that every f32 expression rounds once per operation, exactly as Rust does;
 * fmaf() appears only where the reference calls `mul_add`.
 *
 * Reference citations are `path:line` inside the DiskMule source tree.
 */
#include "dm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar decode helpers                                                    */
/* ------------------------------------------------------------------------ */

static float bits_to_f32(uint32_t bits) {
  float value;
  memcpy(&value, &bits, sizeof value);
  return value;
}

static uint32_t f32_to_bits(float value) {
  uint32_t bits;
  memcpy(&bits, &value, sizeof bits);
  return bits;
}

/* src/cpu.rs:647-660 (f16_to_f32); src/glm52/expert.rs:507-520 is identical. */
float dmo_f16_to_f32(uint16_t value) {
  uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  uint32_t exponent = (value >> 10) & 0x1fu;
  uint32_t fraction = value & 0x03ffu;
  if (exponent == 0 && fraction == 0) return bits_to_f32(sign);
  if (exponent == 0) {
    /* `fraction as f32 * 2.0_f32.powi(-24)`: 2^-24 is exact */
    float magnitude = (float)fraction * 5.9604644775390625e-08f;
    return sign == 0 ? magnitude : -magnitude;
  }
  if (exponent == 0x1f) return bits_to_f32(sign | 0x7f800000u | (fraction << 13));
  return bits_to_f32(sign | ((exponent + 112u) << 23) | (fraction << 13));
}

/* src/glm52/cpu.rs:1266-1271 (bf16 -> f32 is `bits << 16`). */
float dmo_bf16_to_f32(uint16_t bits) { return bits_to_f32((uint32_t)bits << 16); }

/* src/gguf.rs:321-342 (TensorType::layout) for the types on the path. */
int dmo_block_layout(int kind, uint64_t *block_elements, uint64_t *block_bytes) {
  uint64_t e, b;
  switch (kind) {
    case DMO_F32: e = 1; b = 4; break;
    case DMO_F16: e = 1; b = 2; break;
    case DMO_BF16: e = 1; b = 2; break;
    case DMO_Q5_0: e = 32; b = 22; break;
    case DMO_Q8_0: e = 32; b = 34; break;
    case DMO_Q4_K: e = 256; b = 144; break;
    case DMO_Q5_K: e = 256; b = 176; break;
    case DMO_Q6_K: e = 256; b = 210; break;
    default: return DMO_ERR_UNSUPPORTED;
  }
  if (block_elements) *block_elements = e;
  if (block_bytes) *block_bytes = b;
  return DMO_OK;
}

/* src/gguf.rs:352-358 (row_byte_len): None unless `elements % block_elements == 0`. */
int dmo_row_byte_len(int kind, uint64_t elements, uint64_t *out) {
  uint64_t e, b;
  if (dmo_block_layout(kind, &e, &b) != DMO_OK) return DMO_ERR_UNSUPPORTED;
  if (elements % e != 0) return DMO_ERR_ELEMENT_COUNT;
  uint64_t blocks = elements / e;
  if (b != 0 && blocks > UINT64_MAX / b) return DMO_ERR_OVERFLOW;
  *out = blocks * b;
  return DMO_OK;
}

/* src/cpu.rs:607-616 (scale_min_q4_k). */
void dmo_scale_min_q4_k(int index, const uint8_t *scales, uint8_t *scale, uint8_t *min) {
  if (index < 4) {
    *scale = scales[index] & 0x3f;
    *min = scales[index + 4] & 0x3f;
  } else {
    *scale = (uint8_t)((scales[index + 4] & 0x0f) | ((scales[index - 4] >> 6) << 4));
    *min = (uint8_t)((scales[index + 4] >> 4) | ((scales[index] >> 6) << 4));
  }
}

static uint16_t le16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* src/cpu.rs:546-550 */
static void decode_f32(const uint8_t *enc, float *out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    uint32_t bits = (uint32_t)enc[4 * i] | ((uint32_t)enc[4 * i + 1] << 8) |
                    ((uint32_t)enc[4 * i + 2] << 16) | ((uint32_t)enc[4 * i + 3] << 24);
    out[i] = bits_to_f32(bits);
  }
}

/* src/cpu.rs:552-558 */
static void decode_f16(const uint8_t *enc, float *out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = dmo_f16_to_f32(le16(enc + 2 * i));
}

static void decode_bf16(const uint8_t *enc, float *out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = dmo_bf16_to_f32(le16(enc + 2 * i));
}

/* src/cpu.rs:560-574 (decode_q5_0) */
static void decode_q5_0(const uint8_t *enc, float *out, size_t n) {
  for (size_t b = 0; b < n / 32; b++) {
    const uint8_t *block = enc + 22 * b;
    float *values = out + 32 * b;
    float delta = dmo_f16_to_f32(le16(block));
    uint32_t high_bits = (uint32_t)block[2] | ((uint32_t)block[3] << 8) |
                         ((uint32_t)block[4] << 16) | ((uint32_t)block[5] << 24);
    for (int index = 0; index < 16; index++) {
      uint8_t packed = block[6 + index];
      uint8_t low_high_bit = (uint8_t)(((high_bits >> index) << 4) & 0x10);
      uint8_t high_high_bit = (uint8_t)((high_bits >> (index + 12)) & 0x10);
      int32_t low = (int32_t)((packed & 0x0f) | low_high_bit) - 16;
      int32_t high = (int32_t)((packed >> 4) | high_high_bit) - 16;
      values[index] = delta * (float)low;
      values[index + 16] = delta * (float)high;
    }
  }
}

/* src/cpu.rs:576-583 (decode_q8_0) */
static void decode_q8_0(const uint8_t *enc, float *out, size_t n) {
  for (size_t b = 0; b < n / 32; b++) {
    const uint8_t *block = enc + 34 * b;
    float delta = dmo_f16_to_f32(le16(block));
    for (int i = 0; i < 32; i++) out[32 * b + i] = delta * (float)(int8_t)block[2 + i];
  }
}

/* src/cpu.rs:585-605 (decode_q4_k) */
static void decode_q4_k(const uint8_t *enc, float *out, size_t n) {
  for (size_t b = 0; b < n / 256; b++) {
    const uint8_t *block = enc + 144 * b;
    float *values = out + 256 * b;
    float delta = dmo_f16_to_f32(le16(block));
    float minimum = dmo_f16_to_f32(le16(block + 2));
    const uint8_t *scales = block + 4;
    const uint8_t *quants = block + 16;
    for (int group_pair = 0; group_pair < 4; group_pair++) {
      uint8_t scale_low, min_low, scale_high, min_high;
      dmo_scale_min_q4_k(group_pair * 2, scales, &scale_low, &min_low);
      dmo_scale_min_q4_k(group_pair * 2 + 1, scales, &scale_high, &min_high);
      int quant_offset = group_pair * 32;
      int value_offset = group_pair * 64;
      for (int index = 0; index < 32; index++) {
        uint8_t packed = quants[quant_offset + index];
        values[value_offset + index] = delta * (float)scale_low * (float)(packed & 0x0f) -
                                       minimum * (float)min_low;
        values[value_offset + index + 32] = delta * (float)scale_high * (float)(packed >> 4) -
                                            minimum * (float)min_high;
      }
    }
  }
}

/* src/cpu.rs:618-645 (decode_q6_k) */
static void decode_q6_k(const uint8_t *enc, float *out, size_t n) {
  for (size_t b = 0; b < n / 256; b++) {
    const uint8_t *block = enc + 210 * b;
    float delta = dmo_f16_to_f32(le16(block + 208));
    for (int half = 0; half < 2; half++) {
      const uint8_t *low = block + half * 64;
      const uint8_t *high = block + 128 + half * 32;
      const int8_t *scales = (const int8_t *)(block + 192 + half * 8);
      float *values = out + 256 * b + half * 128;
      for (int index = 0; index < 32; index++) {
        int scale_pair = index / 16;
        uint8_t q1 = (uint8_t)((low[index] & 0x0f) | ((high[index] & 0x03) << 4));
        uint8_t q2 = (uint8_t)((low[index + 32] & 0x0f) | (((high[index] >> 2) & 0x03) << 4));
        uint8_t q3 = (uint8_t)((low[index] >> 4) | (((high[index] >> 4) & 0x03) << 4));
        uint8_t q4 = (uint8_t)((low[index + 32] >> 4) | (((high[index] >> 6) & 0x03) << 4));
        values[index] = delta * (float)scales[scale_pair] * ((float)q1 - 32.0f);
        values[index + 32] = delta * (float)scales[scale_pair + 2] * ((float)q2 - 32.0f);
        values[index + 64] = delta * (float)scales[scale_pair + 4] * ((float)q3 - 32.0f);
        values[index + 96] = delta * (float)scales[scale_pair + 6] * ((float)q4 - 32.0f);
      }
    }
  }
}

/* src/cpu.rs:313-343 (dequantize): validation order is element count, byte length,
 * then the supported-type match. BF16 is not a GGUF CPU type in the reference. */
int dmo_dequantize(int kind, const uint8_t *encoded, size_t encoded_len, float *out,
                   size_t n) {
  uint64_t expected;
  int rc = dmo_row_byte_len(kind, (uint64_t)n, &expected);
  if (rc == DMO_ERR_UNSUPPORTED) return DMO_ERR_UNSUPPORTED;
  if (rc != DMO_OK) return rc;
  if ((uint64_t)encoded_len != expected) return DMO_ERR_BYTE_LENGTH;
  switch (kind) {
    case DMO_F32: decode_f32(encoded, out, n); break;
    case DMO_F16: decode_f16(encoded, out, n); break;
    case DMO_Q5_0: decode_q5_0(encoded, out, n); break;
    case DMO_Q8_0: decode_q8_0(encoded, out, n); break;
    case DMO_Q4_K: decode_q4_k(encoded, out, n); break;
    case DMO_Q6_K: decode_q6_k(encoded, out, n); break;
    default: return DMO_ERR_UNSUPPORTED;
  }
  return DMO_OK;
}

/* ------------------------------------------------------------------------ */
/* operators (src/cpu.rs)                                                   */
/* ------------------------------------------------------------------------ */

/* One row of src/cpu.rs:389-397: dequantize, then
 * `fold(0.0, |sum, (weight, value)| weight.mul_add(*value, sum))`. */
static int matvec_row(int kind, const uint8_t *row_bytes, size_t row_len, size_t columns,
                      const float *input, float *scratch, float *result) {
  int rc = dmo_dequantize(kind, row_bytes, row_len, scratch, columns);
  if (rc != DMO_OK) return rc;
  float sum = 0.0f;
  for (size_t c = 0; c < columns; c++) sum = fmaf(scratch[c], input[c], sum);
  *result = sum;
  return DMO_OK;
}

/* src/cpu.rs:346-399 (matvec). Rows run in parallel (rayon there, OpenMP here);
 * each row's dot product is one sequential fma chain in column order. */
int dmo_matvec(int kind, size_t rows, size_t columns, const uint8_t *encoded,
               size_t encoded_len, const float *input, size_t input_len, float *output,
               size_t output_len, int threads) {
  if (input_len != columns) return DMO_ERR_INPUT_LENGTH;
  if (output_len != rows) return DMO_ERR_OUTPUT_LENGTH;
  uint64_t row_bytes;
  int rc = dmo_row_byte_len(kind, (uint64_t)columns, &row_bytes);
  if (rc == DMO_ERR_UNSUPPORTED) return DMO_ERR_UNSUPPORTED;
  if (rc != DMO_OK) return rc;
  if (row_bytes != 0 && rows > UINT64_MAX / row_bytes) return DMO_ERR_OVERFLOW;
  if ((uint64_t)encoded_len != rows * row_bytes) return DMO_ERR_BYTE_LENGTH;
  int status = DMO_OK;
  if (threads < 1) threads = 1;
#pragma omp parallel num_threads(threads) if (threads > 1 && rows > 1)
  {
    float *scratch = (float *)malloc((columns ? columns : 1) * sizeof(float));
#pragma omp for schedule(static)
    for (long r = 0; r < (long)rows; r++) {
      int row_rc = matvec_row(kind, encoded + (size_t)r * row_bytes, (size_t)row_bytes,
                              columns, input, scratch, &output[r]);
      if (row_rc != DMO_OK) {
#pragma omp critical
        status = row_rc;
      }
    }
    free(scratch);
  }
  return status;
}

/* src/cpu.rs:99-143 (rms_norm) */
int dmo_rms_norm(const float *input, const float *weight, size_t n, float epsilon,
                 float *output) {
  if (n == 0) return DMO_ERR_EMPTY;
  if (!isfinite(epsilon) || epsilon <= 0.0f) return DMO_ERR_PARAM;
  float sum_squares = 0.0f;
  for (size_t i = 0; i < n; i++) sum_squares = fmaf(input[i], input[i], sum_squares);
  float inverse_rms = 1.0f / sqrtf(sum_squares / (float)n + epsilon);
  if (!isfinite(inverse_rms)) return DMO_ERR_NONFINITE;
  if (weight) {
    for (size_t i = 0; i < n; i++) output[i] = input[i] * weight[i] * inverse_rms;
  } else {
    for (size_t i = 0; i < n; i++) output[i] = input[i] * inverse_rms;
  }
  return DMO_OK;
}

/* src/cpu.rs:145-150 (gelu_tanh). `value.powi(3)` lowers to value*(value*value),
 * which equals (value*value)*value exactly because f32 multiplication commutes. */
float dmo_gelu_tanh(float value) {
  const float sqrt_two_over_pi = 0.7978846f;
  const float cubic = 0.044715f;
  float cube = value * (value * value);
  return 0.5f * value * (1.0f + tanhf(sqrt_two_over_pi * (value + cubic * cube)));
}

/* src/cpu.rs:196-231 (softmax_in_place) */
int dmo_softmax_in_place(float *values, size_t n) {
  if (n == 0) return DMO_ERR_EMPTY;
  for (size_t i = 0; i < n; i++)
    if (isnan(values[i]) || values[i] == INFINITY) return DMO_ERR_NONFINITE;
  float maximum = -INFINITY;
  for (size_t i = 0; i < n; i++) maximum = fmaxf(maximum, values[i]);
  if (maximum == -INFINITY) return DMO_ERR_NONFINITE;
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    values[i] = expf(values[i] - maximum);
    sum += values[i];
  }
  if (!isfinite(sum) || sum <= 0.0f) return DMO_ERR_NONFINITE;
  for (size_t i = 0; i < n; i++) values[i] /= sum;
  return DMO_OK;
}

/* Rust f32::total_cmp key: a signed integer whose order is the IEEE total order. */
static int32_t total_key(float value) {
  int32_t bits = (int32_t)f32_to_bits(value);
  bits ^= (int32_t)(((uint32_t)(bits >> 31)) >> 1);
  return bits;
}

typedef struct {
  uint32_t index;
  float value;
  float weight;
} scored;

/* Descending by value (total order), ties by ascending index: the comparator of
 * src/cpu.rs:247-252 and src/glm52/cpu.rs:742-747. */
static int cmp_desc_then_index(const void *a, const void *b) {
  const scored *l = (const scored *)a, *r = (const scored *)b;
  int32_t kl = total_key(l->value), kr = total_key(r->value);
  if (kl != kr) return kl > kr ? -1 : 1;
  return l->index < r->index ? -1 : (l->index > r->index);
}

/* src/cpu.rs:234-260 (top_k_softmax) */
int dmo_top_k_softmax(const float *logits, size_t n, size_t k, uint32_t *indices,
                      float *probabilities) {
  if (k == 0 || k > n) return DMO_ERR_TOPK;
  for (size_t i = 0; i < n; i++)
    if (!isfinite(logits[i])) return DMO_ERR_NONFINITE;
  scored *selected = (scored *)malloc(n * sizeof(scored));
  for (size_t i = 0; i < n; i++) {
    selected[i].index = (uint32_t)i;
    selected[i].value = logits[i];
  }
  qsort(selected, n, sizeof(scored), cmp_desc_then_index);
  float *probs = (float *)malloc(k * sizeof(float));
  for (size_t i = 0; i < k; i++) probs[i] = selected[i].value;
  int rc = dmo_softmax_in_place(probs, k);
  if (rc == DMO_OK) {
    for (size_t i = 0; i < k; i++) {
      indices[i] = selected[i].index;
      probabilities[i] = probs[i];
    }
  }
  free(probs);
  free(selected);
  return rc;
}

/* src/cpu.rs:276-293 (argmax): the first maximum under the total order. */
int dmo_argmax(const float *values, size_t n, size_t *index) {
  if (n == 0) return DMO_ERR_EMPTY;
  for (size_t i = 0; i < n; i++)
    if (!isfinite(values[i])) return DMO_ERR_NONFINITE;
  size_t best = 0;
  for (size_t i = 1; i < n; i++)
    if (total_key(values[i]) > total_key(values[best])) best = i;
  *index = best;
  return DMO_OK;
}

/* ------------------------------------------------------------------------ */
/* GLM-5.2 helpers                                                          */
/* ------------------------------------------------------------------------ */

/* src/glm52/cpu.rs:912-924: the mean square is a sequential f64 sum of the (exact)
 * squares divided by n in f64; scale = 1 / sqrt(ms as f32 + eps) in f32;
 * out = value * scale * weight, left to right. */
int dmo_glm_rms_norm(const float *input, const float *weight, size_t n, float epsilon,
                     float *output) {
  if (n == 0) return DMO_ERR_EMPTY;
  double sum = 0.0;
  for (size_t i = 0; i < n; i++) sum += (double)input[i] * (double)input[i];
  const float mean_square = (float)(sum / (double)n);
  const float scale = 1.0f / sqrtf(mean_square + epsilon);
  for (size_t i = 0; i < n; i++) output[i] = input[i] * scale * weight[i];
  return DMO_OK;
}

/* src/glm52/cpu.rs:980-982 */
float dmo_glm_sigmoid(float value) { return 1.0f / (1.0f + expf(-value)); }
/* src/glm52/cpu.rs:984-986 (used by the shared-expert `mlp`, :897-910) */
float dmo_glm_silu(float value) { return value * dmo_glm_sigmoid(value); }
/* src/glm52/expert.rs:260-267 (routed experts through CachedExpert::mlp) */
float dmo_glm_cached_silu(float value) { return value / (1.0f + expf(-value)); }

/* src/qwen35/cpu.rs:982-993 */
float dmo_qwen_sigmoid(float value) {
  if (value >= 0.0f) return 1.0f / (1.0f + expf(-value));
  float exponential = expf(value);
  return exponential / (1.0f + exponential);
}
float dmo_qwen_silu(float value) { return value * dmo_qwen_sigmoid(value); }

static int dense_row(int kind, const uint8_t *encoded, size_t row, size_t columns,
                     float *out) {
  switch (kind) {
    case DMO_F32: decode_f32(encoded + row * columns * 4, out, columns); return DMO_OK;
    case DMO_F16: decode_f16(encoded + row * columns * 2, out, columns); return DMO_OK;
    case DMO_BF16: decode_bf16(encoded + row * columns * 2, out, columns); return DMO_OK;
    default: return DMO_ERR_UNSUPPORTED;
  }
}

/* src/glm52/cpu.rs:1121-1187 (TensorReader::matvec_into, dense dtypes) and
 * src/glm52/expert.rs:370-387 (CachedTensor::matvec): per row, a sequential
 * non-fused sum of `weight * value` in column order. Rust's f32 `Sum` folds from
 * -0.0; CachedTensor starts from 0.0; the two differ only for an all -0.0 row. */
int dmo_glm_matvec(int kind, size_t rows, size_t columns, const uint8_t *encoded,
                   const float *input, float *output, int threads) {
  if (kind != DMO_F32 && kind != DMO_F16 && kind != DMO_BF16) return DMO_ERR_UNSUPPORTED;
  if (threads < 1) threads = 1;
#pragma omp parallel num_threads(threads) if (threads > 1 && rows > 1)
  {
    float *row = (float *)malloc((columns ? columns : 1) * sizeof(float));
#pragma omp for schedule(static)
    for (long r = 0; r < (long)rows; r++) {
      dense_row(kind, encoded, (size_t)r, columns, row);
      float sum = -0.0f;
      for (size_t c = 0; c < columns; c++) sum = sum + row[c] * input[c];
      output[r] = sum;
    }
    free(row);
  }
  return DMO_OK;
}

/* GLM-5.2 checkpoint encodings.
 * decode_f8_e4m3fn (src/glm52/cpu.rs:1397-1410): finite-only E4M3; 0x7f / 0xff (exponent
 * 15, fraction 7) are invalid. Subnormals fraction * 2^-9, normals (1 + f/8) * 2^(e-7). */
int dmo_f8_e4m3fn(uint8_t v, float *out) {
  const float sign = (v & 0x80) ? -1.0f : 1.0f;
  const int e = (v >> 3) & 0x0f, f = v & 0x07;
  if (e == 0x0f && f == 0x07) return DMO_ERR_NONFINITE;
  const float mag = e == 0 ? (float)f * ldexpf(1.0f, -9) : (1.0f + (float)f / 8.0f) * ldexpf(1.0f, e - 7);
  *out = sign * mag;
  return DMO_OK;
}

/* matching_quantizations + resolve_quantization (src/glm52/quant.rs:63-76, :148-176):
 * int8 rows when rows * columns bytes and one scale per row, else int4 grouped with the
 * first group size of {16, 32, 48, 64, 96, 128, 192, 256} whose scale count matches.
 * kind: 1 int8 row, 2 int4 grouped. */
int dmo_glm_u8_encoding(size_t rows, size_t columns, size_t encoded_bytes, size_t scales,
                        int *kind, int *group_size) {
  static const size_t groups[8] = {16, 32, 48, 64, 96, 128, 192, 256};
  if (rows * columns == encoded_bytes && scales == rows) {
    *kind = 1;
    *group_size = 0;
    return DMO_OK;
  }
  if (rows * ((columns + 1) / 2) == encoded_bytes) {
    for (int i = 0; i < 8; i++)
      if (rows * ((columns + groups[i] - 1) / groups[i]) == scales) {
        *kind = 2;
        *group_size = (int)groups[i];
        return DMO_OK;
      }
  }
  return DMO_ERR_BYTE_LENGTH;
}

/* One decoded row (read_quantized_row, src/glm52/cpu.rs:1339-1395; read_fp8_row,
 * :1278-1337). fp8: scales [ceil(rows/128)][ceil(columns/128)] of `scale_inv` values. */
static int quant_row(int enc, int group, size_t rows, size_t columns, const uint8_t *w,
                     const float *scales, size_t r, float *out) {
  if (enc == 1) {
    const uint8_t *q = w + r * columns;
    for (size_t c = 0; c < columns; c++) out[c] = (float)(int8_t)q[c] * scales[r];
  } else if (enc == 2) {
    const size_t rb = (columns + 1) / 2, sc = (columns + (size_t)group - 1) / (size_t)group;
    const uint8_t *q = w + r * rb;
    for (size_t c = 0; c < columns; c++) {
      const uint8_t b = q[c / 2];
      const int nib = (c % 2 == 0) ? (b & 0x0f) : (b >> 4);
      out[c] = ((float)nib - 8.0f) * scales[r * sc + c / (size_t)group];
    }
  } else {
    const size_t sc = (columns + 127) / 128;
    const uint8_t *q = w + r * columns;
    for (size_t c = 0; c < columns; c++) {
      float d;
      if (dmo_f8_e4m3fn(q[c], &d) != DMO_OK) return DMO_ERR_NONFINITE;
      out[c] = d * scales[(r / 128) * sc + c / 128];
    }
  }
  (void)rows;
  return DMO_OK;
}

/* TensorReader::matvec_into over the quantized dtypes (src/glm52/cpu.rs:1121-1187):
 * each row decoded, then a sequential non-fused sum of `weight * value` from -0.0.
 * fp8 != 0: F8_E4M3 weights [rows][columns] with block scales; otherwise U8 storage
 * (int8 row or int4 grouped, resolved as above) with `.qs` scales. */
int dmo_glm_quant_matvec(int fp8, size_t rows, size_t columns, const uint8_t *encoded,
                         size_t encoded_bytes, const float *scales, size_t n_scales,
                         const float *input, float *output, int threads) {
  int enc = 3, group = 0;
  if (!fp8) {
    int rc = dmo_glm_u8_encoding(rows, columns, encoded_bytes, n_scales, &enc, &group);
    if (rc != DMO_OK) return rc;
  } else {
    if (encoded_bytes != rows * columns) return DMO_ERR_BYTE_LENGTH;
    if (n_scales != ((rows + 127) / 128) * ((columns + 127) / 128)) return DMO_ERR_BYTE_LENGTH;
  }
  if (threads < 1) threads = 1;
  int bad = 0;
#pragma omp parallel num_threads(threads) if (threads > 1 && rows > 1) reduction(| : bad)
  {
    float *row = (float *)malloc((columns ? columns : 1) * sizeof(float));
#pragma omp for schedule(static)
    for (long r = 0; r < (long)rows; r++) {
      if (quant_row(enc, group, rows, columns, encoded, scales, (size_t)r, row) != DMO_OK) {
        bad = 1;
        continue;
      }
      float sum = -0.0f;
      for (size_t c = 0; c < columns; c++) sum = sum + row[c] * input[c];
      output[r] = sum;
    }
    free(row);
  }
  return bad ? DMO_ERR_NONFINITE : DMO_OK;
}

/* A decoded row (matrix_row_into) of the same encodings. */
int dmo_glm_quant_row(int fp8, size_t rows, size_t columns, const uint8_t *encoded,
                      size_t encoded_bytes, const float *scales, size_t n_scales, size_t r,
                      float *out) {
  int enc = 3, group = 0;
  if (!fp8) {
    int rc = dmo_glm_u8_encoding(rows, columns, encoded_bytes, n_scales, &enc, &group);
    if (rc != DMO_OK) return rc;
  }
  if (r >= rows) return DMO_ERR_OUTPUT_LENGTH;
  return quant_row(enc, group, rows, columns, encoded, scales, r, out);
}

/* Sigmoid + correction-bias selection.
 *   n_groups == 1: src/glm52/cpu.rs:731-754 exactly (sigmoid, `choice = weight +
 *   correction`, non-finite -> error, sort by choice desc / index asc, truncate,
 *   optional `w /= sum + 1e-20`).
 *   n_groups > 1: restated, parity unpinned (the reference rejects n_group != 1 at
 *   src/glm52.rs:228-234). Standard group-limited routing: a group's score is the
 *   sum of its two largest choices (top1 + top2), the `topk_groups` best groups are
 *   kept (ties -> lower group index) and experts outside them are not eligible.
 * Output order is selection order; weights are the (normalised) sigmoid scores. */
int dmo_glm_select(const float *logits, const float *correction, size_t experts,
                   size_t k, size_t n_groups, size_t topk_groups, int normalize,
                   uint32_t *indices, float *weights) {
  if (k == 0 || k > experts) return DMO_ERR_TOPK;
  if (n_groups == 0 || experts % n_groups != 0 || topk_groups == 0 || topk_groups > n_groups)
    return DMO_ERR_PARAM;
  size_t per_group = experts / n_groups;
  if (n_groups > 1 && per_group < 2) return DMO_ERR_PARAM;
  if (k > topk_groups * per_group) return DMO_ERR_TOPK;
  scored *choices = (scored *)malloc(experts * sizeof(scored));
  for (size_t e = 0; e < experts; e++) {
    float weight = dmo_glm_sigmoid(logits[e]);
    float choice = weight + correction[e];
    if (!isfinite(weight) || !isfinite(choice)) {
      free(choices);
      return DMO_ERR_NONFINITE;
    }
    choices[e].index = (uint32_t)e;
    choices[e].value = choice;
    choices[e].weight = weight;
  }
  size_t eligible = experts;
  scored *pool = choices;
  scored *kept = NULL;
  if (n_groups > 1) {
    scored *groups = (scored *)malloc(n_groups * sizeof(scored));
    for (size_t g = 0; g < n_groups; g++) {
      const scored *base = choices + g * per_group;
      size_t first = 0;
      for (size_t i = 1; i < per_group; i++)
        if (cmp_desc_then_index(&base[i], &base[first]) < 0) first = i;
      size_t second = first == 0 ? 1 : 0;
      for (size_t i = 0; i < per_group; i++)
        if (i != first && cmp_desc_then_index(&base[i], &base[second]) < 0) second = i;
      groups[g].index = (uint32_t)g;
      groups[g].value = base[first].value + base[second].value;
    }
    qsort(groups, n_groups, sizeof(scored), cmp_desc_then_index);
    kept = (scored *)malloc(topk_groups * per_group * sizeof(scored));
    eligible = 0;
    for (size_t e = 0; e < experts; e++) {
      size_t g = e / per_group;
      for (size_t j = 0; j < topk_groups; j++)
        if (groups[j].index == g) {
          kept[eligible++] = choices[e];
          break;
        }
    }
    free(groups);
    pool = kept;
  }
  qsort(pool, eligible, sizeof(scored), cmp_desc_then_index);
  float sum = -0.0f;
  for (size_t i = 0; i < k; i++) sum = sum + pool[i].weight;
  sum = sum + 1e-20f;
  for (size_t i = 0; i < k; i++) {
    indices[i] = pool[i].index;
    weights[i] = normalize ? pool[i].weight / sum : pool[i].weight;
  }
  free(kept);
  free(choices);
  return DMO_OK;
}

/* ------------------------------------------------------------------------ */
/* dispatch (new work: the reference loops over `selected` per token)       */
/* ------------------------------------------------------------------------ */

/* Counting sort of the T*k (token, slot) pairs p = t*k + j by expert. Within an
 * expert the order is ascending p, i.e. (token asc, slot asc). inverse[p] is the
 * position of pair p in sorted_pairs. */
int dmo_dispatch(const uint32_t *selected, size_t tokens, size_t k, size_t experts,
                 int32_t *counts, int32_t *offsets, int32_t *sorted_pairs,
                 int32_t *inverse) {
  size_t pairs = tokens * k;
  for (size_t e = 0; e < experts; e++) counts[e] = 0;
  for (size_t p = 0; p < pairs; p++) {
    if (selected[p] >= experts) return DMO_ERR_EXPERT;
    counts[selected[p]]++;
  }
  offsets[0] = 0;
  for (size_t e = 0; e < experts; e++) offsets[e + 1] = offsets[e] + counts[e];
  int32_t *cursor = (int32_t *)malloc((experts ? experts : 1) * sizeof(int32_t));
  for (size_t e = 0; e < experts; e++) cursor[e] = offsets[e];
  for (size_t p = 0; p < pairs; p++) {
    int32_t position = cursor[selected[p]]++;
    sorted_pairs[position] = (int32_t)p;
    inverse[p] = position;
  }
  free(cursor);
  return DMO_OK;
}

/* ------------------------------------------------------------------------ */
/* MoE blocks                                                               */
/* ------------------------------------------------------------------------ */

static size_t row_bytes_of(int kind, size_t columns) {
  uint64_t out = 0;
  dmo_row_byte_len(kind, (uint64_t)columns, &out);
  return (size_t)out;
}

/* Gemma 4 routed branch for one token: src/gemma4/cpu.rs:559-611, with
 * tensor_expert_matvec (src/cpu.rs:474-509) slicing expert `e` at
 * `e * rows * row_bytes`. Output is `routed` at :612 (before routed_post_norm). */
/* The Gemma 4 router for one token (src/gemma4/cpu.rs:562-576): unweighted rms_norm,
 * router_scale / sqrt(hidden), the f32 router matvec, the optional logit bias, then
 * top_k_softmax. */
static int gemma_route_token(const dmo_gemma_layer *L, const float *x, uint32_t *sel_idx,
                             float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, E = (size_t)L->experts, k = (size_t)L->top_k;
  float *router_input = (float *)malloc(H * sizeof(float));
  float *logits = (float *)malloc(E * sizeof(float));
  int rc = dmo_rms_norm(x, NULL, H, L->epsilon, router_input);
  if (rc == DMO_OK) {
    float inverse_hidden_scale = 1.0f / sqrtf((float)H);
    for (size_t i = 0; i < H; i++)
      router_input[i] = router_input[i] * (L->router_scale[i] * inverse_hidden_scale);
    rc = dmo_matvec(DMO_F32, E, H, (const uint8_t *)L->router, E * H * 4, router_input, H,
                    logits, E, threads);
  }
  if (rc == DMO_OK && L->router_logit_bias)
    for (size_t e = 0; e < E; e++) logits[e] = logits[e] + L->router_logit_bias[e];
  if (rc == DMO_OK) rc = dmo_top_k_softmax(logits, E, k, sel_idx, sel_prob);
  free(router_input); free(logits);
  return rc;
}

static int gemma_token(const dmo_gemma_layer *L, const float *x, float *routed,
                       uint32_t *sel_idx, float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, I = (size_t)L->intermediate;
  size_t k = (size_t)L->top_k;
  float *routed_input = (float *)malloc(H * sizeof(float));
  float *gate_up = (float *)malloc(2 * I * sizeof(float));
  float *activated = (float *)malloc(I * sizeof(float));
  float *expert_output = (float *)malloc(H * sizeof(float));
  int rc = dmo_rms_norm(x, L->routed_pre_norm, H, L->epsilon, routed_input);
  if (rc == DMO_OK) rc = gemma_route_token(L, x, sel_idx, sel_prob, threads);
  for (size_t i = 0; i < H; i++) routed[i] = 0.0f;
  size_t gu_row = row_bytes_of(L->gate_up_type, H), down_row = row_bytes_of(L->down_type, I);
  for (size_t j = 0; rc == DMO_OK && j < k; j++) {
    size_t e = sel_idx[j];
    size_t gu_bytes = 2 * I * gu_row, down_bytes = H * down_row;
    rc = dmo_matvec(L->gate_up_type, 2 * I, H, L->gate_up + e * gu_bytes, gu_bytes,
                    routed_input, H, gate_up, 2 * I, threads);
    if (rc != DMO_OK) break;
    for (size_t i = 0; i < I; i++) activated[i] = dmo_gelu_tanh(gate_up[i]) * gate_up[I + i];
    rc = dmo_matvec(L->down_type, H, I, L->down + e * down_bytes, down_bytes, activated, I,
                    expert_output, H, threads);
    if (rc != DMO_OK) break;
    float scale = sel_prob[j] * L->expert_scale[e];
    for (size_t i = 0; i < H; i++) routed[i] = fmaf(expert_output[i], scale, routed[i]);
  }
  free(routed_input); free(gate_up);
  free(activated); free(expert_output);
  return rc;
}

/* Tokens are independent (the reference runs one token per forward). With several
 * tokens the oracle parallelises over tokens; with one it parallelises matvec rows. */
#define TOKEN_LOOP(call)                                                         \
  int status = DMO_OK;                                                           \
  if (threads < 1) threads = 1;                                                  \
  if (tokens == 1) {                                                             \
    long t = 0;                                                                  \
    status = (call);                                                             \
  } else {                                                                       \
    _Pragma("omp parallel for schedule(dynamic, 1) num_threads(threads)")        \
    for (long t = 0; t < (long)tokens; t++) {                                    \
      int rc_t = (call);                                                         \
      if (rc_t != DMO_OK) {                                                      \
        _Pragma("omp critical") status = rc_t;                                   \
      }                                                                          \
    }                                                                            \
  }                                                                              \
  return status;

int dmo_gemma_moe(const dmo_gemma_layer *L, const float *x, size_t tokens, float *routed,
                  uint32_t *sel_idx, float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(gemma_token(L, x + t * H, routed + t * H, sel_idx + t * k, sel_prob + t * k,
                         tokens == 1 ? threads : 1))
}

int dmo_gemma_route(const dmo_gemma_layer *L, const float *x, size_t tokens, uint32_t *sel_idx,
                    float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(gemma_route_token(L, x + t * H, sel_idx + t * k, sel_prob + t * k,
                               tokens == 1 ? threads : 1))
}

/* One token of the whole Gemma 4 feed-forward block (src/gemma4/cpu.rs:547-620). */
static int gemma_ffn_token(const dmo_gemma_ffn *F, const dmo_gemma_layer *L, const float *x,
                           float *hidden, uint32_t *sel_idx, float *sel_prob, int threads) {
  const size_t H = (size_t)L->hidden, W = (size_t)F->width;
  float *shared_input = (float *)malloc(H * sizeof(float));
  float *gate = (float *)malloc(W * sizeof(float));
  float *up = (float *)malloc(W * sizeof(float));
  float *shared_raw = (float *)malloc(H * sizeof(float));
  float *shared = (float *)malloc(H * sizeof(float));
  float *routed_raw = (float *)malloc(H * sizeof(float));
  float *routed = (float *)malloc(H * sizeof(float));
  float *combined = (float *)malloc(H * sizeof(float));
  int rc = dmo_rms_norm(x, F->feed_forward_norm, H, L->epsilon, shared_input);
  if (rc == DMO_OK)
    rc = dmo_matvec(F->gate_type, W, H, F->gate, W * row_bytes_of(F->gate_type, H), shared_input,
                    H, gate, W, threads);
  if (rc == DMO_OK)
    rc = dmo_matvec(F->up_type, W, H, F->up, W * row_bytes_of(F->up_type, H), shared_input, H,
                    up, W, threads);
  if (rc == DMO_OK) {
    for (size_t i = 0; i < W; i++) gate[i] = dmo_gelu_tanh(gate[i]) * up[i];
    rc = dmo_matvec(F->down_type, H, W, F->down, H * row_bytes_of(F->down_type, W), gate, W,
                    shared_raw, H, threads);
  }
  if (rc == DMO_OK) rc = dmo_rms_norm(shared_raw, F->shared_post_norm, H, L->epsilon, shared);
  if (rc == DMO_OK) rc = gemma_token(L, x, routed_raw, sel_idx, sel_prob, threads);
  if (rc == DMO_OK) rc = dmo_rms_norm(routed_raw, F->routed_post_norm, H, L->epsilon, routed);
  if (rc == DMO_OK) {
    for (size_t i = 0; i < H; i++) routed_raw[i] = shared[i] + routed[i];  /* combined */
    rc = dmo_rms_norm(routed_raw, F->post_feed_forward_norm, H, L->epsilon, combined);
  }
  if (rc == DMO_OK)
    for (size_t i = 0; i < H; i++) hidden[i] = (x[i] + combined[i]) * F->layer_output_scale;
  free(shared_input); free(gate); free(up); free(shared_raw); free(shared);
  free(routed_raw); free(routed); free(combined);
  return rc;
}

int dmo_gemma_ffn_block(const dmo_gemma_ffn *F, const dmo_gemma_layer *L, const float *x,
                        size_t tokens, float *hidden, uint32_t *sel_idx, float *sel_prob,
                        int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(gemma_ffn_token(F, L, x + t * H, hidden + t * H, sel_idx + t * k, sel_prob + t * k,
                             tokens == 1 ? threads : 1))
}

/* dense SiLU-GLU expert on GGUF tensors: the Qwen3.5 FFN form of
 * src/qwen35/cpu.rs:415-428 (gate, up, silu(gate)*up, down). */
static int qwen_expert(int gate_type, int up_type, int down_type, const uint8_t *gate,
                       const uint8_t *up, const uint8_t *down, size_t H, size_t I,
                       const float *x, float *out, int threads) {
  float *g = (float *)malloc(I * sizeof(float));
  float *u = (float *)malloc(I * sizeof(float));
  int rc = dmo_matvec(gate_type, I, H, gate, I * row_bytes_of(gate_type, H), x, H, g, I,
                      threads);
  if (rc == DMO_OK)
    rc = dmo_matvec(up_type, I, H, up, I * row_bytes_of(up_type, H), x, H, u, I, threads);
  if (rc == DMO_OK) {
    for (size_t i = 0; i < I; i++) g[i] = dmo_qwen_silu(g[i]) * u[i];
    rc = dmo_matvec(down_type, H, I, down, H * row_bytes_of(down_type, I), g, I, out, H,
                    threads);
  }
  free(g);
  free(u);
  return rc;
}

/* Qwen3.5-shaped MoE block -- restated, parity unpinned (the reference's Qwen3.5
 * is dense, src/qwen35.rs:297-304). Definition used by this build:
 *   logits = matvec_f32(router, x)                     (src/cpu.rs:346-399)
 *   (e_j, p_j) = top_k_softmax(logits, k)              (src/cpu.rs:234-260)
 *   routed = fma(expert_{e_j}(x), p_j, routed)  in selection order
 *   g = qwen_sigmoid(fma-chain dot(shared_gate_vector, x))
 *   y = fma(shared(x), g, routed)
 * with expert(x) = down(silu(gate x) * (up x)). */
static int qwen_route_token(const dmo_qwen_layer *L, const float *x, uint32_t *sel_idx,
                            float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, E = (size_t)L->experts, k = (size_t)L->top_k;
  float *logits = (float *)malloc(E * sizeof(float));
  int rc = dmo_matvec(DMO_F32, E, H, (const uint8_t *)L->router, E * H * 4, x, H, logits, E,
                      threads);
  if (rc == DMO_OK && L->router_logit_bias)
    for (size_t e = 0; e < E; e++) logits[e] = logits[e] + L->router_logit_bias[e];
  if (rc == DMO_OK) rc = dmo_top_k_softmax(logits, E, k, sel_idx, sel_prob);
  free(logits);
  return rc;
}

static int qwen_token(const dmo_qwen_layer *L, const float *x, float *y, uint32_t *sel_idx,
                      float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, I = (size_t)L->intermediate;
  size_t k = (size_t)L->top_k;
  float *out = (float *)malloc(H * sizeof(float));
  int rc = qwen_route_token(L, x, sel_idx, sel_prob, threads);
  for (size_t i = 0; i < H; i++) y[i] = 0.0f;
  size_t gate_bytes = I * row_bytes_of(L->gate_type, H);
  size_t up_bytes = I * row_bytes_of(L->up_type, H);
  size_t down_bytes = H * row_bytes_of(L->down_type, I);
  for (size_t j = 0; rc == DMO_OK && j < k; j++) {
    size_t e = sel_idx[j];
    rc = qwen_expert(L->gate_type, L->up_type, L->down_type, L->gate + e * gate_bytes,
                     L->up + e * up_bytes, L->down + e * down_bytes, H, I, x, out, threads);
    if (rc != DMO_OK) break;
    for (size_t i = 0; i < H; i++) y[i] = fmaf(out[i], sel_prob[j], y[i]);
  }
  if (rc == DMO_OK && L->shared_intermediate > 0) {
    float gate_logit = 0.0f;
    for (size_t i = 0; i < H; i++) gate_logit = fmaf(L->shared_gate_vector[i], x[i], gate_logit);
    float g = dmo_qwen_sigmoid(gate_logit);
    rc = qwen_expert(L->gate_type, L->up_type, L->down_type, L->shared_gate, L->shared_up,
                     L->shared_down, H, (size_t)L->shared_intermediate, x, out, threads);
    if (rc == DMO_OK)
      for (size_t i = 0; i < H; i++) y[i] = fmaf(out[i], g, y[i]);
  }
  free(out);
  return rc;
}

int dmo_qwen_moe(const dmo_qwen_layer *L, const float *x, size_t tokens, float *y,
                 uint32_t *sel_idx, float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(qwen_token(L, x + t * H, y + t * H, sel_idx + t * k, sel_prob + t * k,
                        tokens == 1 ? threads : 1))
}

int dmo_qwen_route(const dmo_qwen_layer *L, const float *x, size_t tokens, uint32_t *sel_idx,
                   float *sel_prob, int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(qwen_route_token(L, x + t * H, sel_idx + t * k, sel_prob + t * k,
                              tokens == 1 ? threads : 1))
}

/* The GLM-5.2 router for one token (src/glm52/cpu.rs:731-754): the router matvec on
 * the raw hidden state, then the grouped sigmoid + correction-bias selection. */
static int glm_route_token(const dmo_glm_layer *L, const float *x, uint32_t *sel_idx,
                           float *sel_weight, int threads) {
  size_t H = (size_t)L->hidden, E = (size_t)L->experts, k = (size_t)L->top_k;
  float *logits = (float *)malloc(E * sizeof(float));
  int rc = dmo_glm_matvec(L->weight_type, E, H, L->router, x, logits, threads);
  if (rc == DMO_OK)
    rc = dmo_glm_select(logits, L->correction_bias, E, k, (size_t)L->n_groups,
                        (size_t)L->topk_groups, L->normalize, sel_idx, sel_weight);
  free(logits);
  return rc;
}

/* GLM-5.2 sparse feed-forward for one token: src/glm52/cpu.rs:711-778.
 * Routed experts go through CachedExpert::mlp (src/glm52/expert.rs:260-267, silu
 * written `g / (1 + exp(-g))`); the shared expert through `mlp`
 * (src/glm52/cpu.rs:897-910, silu written `g * sigmoid(g)`). */
static int glm_token(const dmo_glm_layer *L, const float *x, float *y, uint32_t *sel_idx,
                     float *sel_weight, int threads) {
  size_t H = (size_t)L->hidden, I = (size_t)L->intermediate;
  size_t k = (size_t)L->top_k;
  size_t width = L->weight_type == DMO_F32 ? 4 : 2;
  size_t SI = L->shared_intermediate > 0 ? (size_t)L->shared_intermediate : 0;
  size_t maxI = I > SI ? I : SI;
  float *gate = (float *)malloc(maxI * sizeof(float));
  float *up = (float *)malloc(maxI * sizeof(float));
  float *out = (float *)malloc(H * sizeof(float));
  int rc = glm_route_token(L, x, sel_idx, sel_weight, threads);
  for (size_t i = 0; i < H; i++) y[i] = 0.0f;
  size_t expert_in = I * H * width;
  for (size_t j = 0; rc == DMO_OK && j < k; j++) {
    size_t e = sel_idx[j];
    const uint8_t *wg = L->expert_blobs ? L->expert_blobs[e] : L->gate + e * expert_in;
    const uint8_t *wu = L->expert_blobs ? L->expert_blobs[e] + expert_in : L->up + e * expert_in;
    const uint8_t *wd = L->expert_blobs ? L->expert_blobs[e] + 2 * expert_in : L->down + e * expert_in;
    dmo_glm_matvec(L->weight_type, I, H, wg, x, gate, threads);
    dmo_glm_matvec(L->weight_type, I, H, wu, x, up, threads);
    for (size_t i = 0; i < I; i++) gate[i] = dmo_glm_cached_silu(gate[i]) * up[i];
    dmo_glm_matvec(L->weight_type, H, I, wd, gate, out, threads);
    for (size_t i = 0; i < H; i++) y[i] = y[i] + out[i] * sel_weight[j] * L->routed_scale;
  }
  if (rc == DMO_OK && SI > 0) {
    dmo_glm_matvec(L->weight_type, SI, H, L->shared_gate, x, gate, threads);
    dmo_glm_matvec(L->weight_type, SI, H, L->shared_up, x, up, threads);
    for (size_t i = 0; i < SI; i++) gate[i] = dmo_glm_silu(gate[i]) * up[i];
    dmo_glm_matvec(L->weight_type, H, SI, L->shared_down, gate, out, threads);
    for (size_t i = 0; i < H; i++) y[i] = y[i] + out[i];
  }
  free(gate); free(up); free(out);
  return rc;
}

int dmo_glm_moe(const dmo_glm_layer *L, const float *x, size_t tokens, float *y,
                uint32_t *sel_idx, float *sel_weight, int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(glm_token(L, x + t * H, y + t * H, sel_idx + t * k, sel_weight + t * k,
                       tokens == 1 ? threads : 1))
}

int dmo_glm_route(const dmo_glm_layer *L, const float *x, size_t tokens, uint32_t *sel_idx,
                  float *sel_weight, int threads) {
  size_t H = (size_t)L->hidden, k = (size_t)L->top_k;
  TOKEN_LOOP(glm_route_token(L, x + t * H, sel_idx + t * k, sel_weight + t * k,
                             tokens == 1 ? threads : 1))
}

/* ------------------------------------------------------------------------ */
/* expert residency                                                         */
/* ------------------------------------------------------------------------ */

typedef struct {
  int32_t expert; /* -1 = empty */
  uint64_t last_used;
  int32_t pinned;
} lru_slot;

struct dmo_lru {
  int32_t layers, experts, slots, global_clock, reads_per_miss;
  uint64_t expert_bytes;
  uint64_t *clocks; /* one per layer, or clocks[0] shared */
  lru_slot *table;  /* [layers][slots] */
  dmo_cache_stats stats;
};

dmo_lru *dmo_lru_create(int32_t layers, int32_t experts, int32_t slots, int32_t global_clock,
                        uint64_t expert_bytes, int32_t reads_per_miss) {
  if (slots <= 0 || layers <= 0) return NULL;
  dmo_lru *lru = (dmo_lru *)calloc(1, sizeof(dmo_lru));
  lru->layers = layers;
  lru->experts = experts;
  lru->slots = slots;
  lru->global_clock = global_clock;
  lru->reads_per_miss = reads_per_miss;
  lru->expert_bytes = expert_bytes;
  lru->clocks = (uint64_t *)calloc((size_t)layers, sizeof(uint64_t));
  lru->table = (lru_slot *)calloc((size_t)layers * (size_t)slots, sizeof(lru_slot));
  for (int32_t i = 0; i < layers * slots; i++) lru->table[i].expert = -1;
  /* src/expert.rs:104-115: the Metal slots are allocated up front, so resident
   * bytes start at slots * bytes; the GLM cache counts bytes as they load. */
  if (!global_clock) lru->stats.resident_bytes = (uint64_t)layers * (uint64_t)slots * expert_bytes;
  return lru;
}

void dmo_lru_destroy(dmo_lru *lru) {
  if (!lru) return;
  free(lru->clocks);
  free(lru->table);
  free(lru);
}

/* src/expert.rs:166-229 (per-layer clock, pinned slots skipped) and
 * src/glm52/expert.rs:183-256 (global clock). Victim = the minimum of
 * (occupied, last_used, index) over eligible slots. */
int dmo_lru_acquire(dmo_lru *lru, int32_t layer, int32_t expert, int32_t *slot,
                    int32_t *was_miss) {
  if (layer < 0 || layer >= lru->layers) return DMO_ERR_LAYER;
  if (expert < 0 || expert >= lru->experts) return DMO_ERR_EXPERT;
  uint64_t *clock = lru->global_clock ? &lru->clocks[0] : &lru->clocks[layer];
  *clock += 1;
  lru_slot *slots = lru->table + (size_t)layer * (size_t)lru->slots;
  for (int32_t i = 0; i < lru->slots; i++) {
    if (slots[i].expert == expert) {
      slots[i].last_used = *clock;
      lru->stats.hits++;
      *slot = i;
      *was_miss = 0;
      return DMO_OK;
    }
  }
  lru->stats.misses++;
  int32_t victim = -1;
  for (int32_t i = 0; i < lru->slots; i++) {
    if (!lru->global_clock && slots[i].pinned) continue;
    if (victim < 0) {
      victim = i;
      continue;
    }
    int occ_i = slots[i].expert >= 0, occ_v = slots[victim].expert >= 0;
    if (occ_i < occ_v || (occ_i == occ_v && slots[i].last_used < slots[victim].last_used))
      victim = i;
  }
  if (victim < 0) return DMO_ERR_ALL_PINNED;
  int evicting = slots[victim].expert >= 0;
  if (evicting) lru->stats.evictions++;
  lru->stats.reads += (uint64_t)lru->reads_per_miss;
  lru->stats.bytes_read += lru->expert_bytes;
  if (lru->global_clock) {
    lru->stats.resident_bytes = lru->stats.resident_bytes - (evicting ? lru->expert_bytes : 0) +
                                lru->expert_bytes;
  }
  slots[victim].expert = expert;
  slots[victim].last_used = *clock;
  *slot = victim;
  *was_miss = 1;
  return DMO_OK;
}

void dmo_lru_set_pinned(dmo_lru *lru, int32_t layer, int32_t slot, int32_t pinned) {
  lru->table[(size_t)layer * (size_t)lru->slots + (size_t)slot].pinned = pinned;
}

void dmo_lru_stats(const dmo_lru *lru, dmo_cache_stats *stats) { *stats = lru->stats; }
