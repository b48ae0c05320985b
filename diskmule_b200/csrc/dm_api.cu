// dm_api.cu -- the extern "C" boundary (include/diskmule_cuda.h).
//
// The host side mirrors MetalContext (src/metal.rs:179-1604): validation before
// any launch, in the reference's error order, then stream-ordered kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "../../include/diskmule_cuda.h"
#include "dm_internal.cuh"
#include "../../include/diskmule_selftest.h"

namespace dmi {

thread_local char g_message[512] = "";

int32_t fail(int32_t status, const char *fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_message, sizeof g_message, fmt, args);
  va_end(args);
  return status;
}

int32_t cuda_fail(cudaError_t err, const char *what) {
  return fail(DM_ERR_COMMAND, "%s: %s", what, cudaGetErrorString(err));
}

}  // namespace dmi

using dmi::cuda_fail;
using dmi::fail;
using dmi::g_message;
using dmi::release_context;
using dmi::retain_context;

extern "C" {

const char *dm_status_string(int32_t status) {
  switch (status) {
    case DM_OK: return "ok";
    case DM_ERR_NO_DEVICE: return "no CUDA device is available";
    case DM_ERR_ALLOCATION: return "device allocation failed";
    case DM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DM_ERR_UNSUPPORTED_TENSOR_TYPE: return "unsupported tensor type";
    case DM_ERR_ELEMENT_COUNT: return "element count is not a whole number of blocks";
    case DM_ERR_BYTE_LENGTH: return "encoded byte length does not match the shape";
    case DM_ERR_INPUT_LENGTH: return "matvec input length does not match the columns";
    case DM_ERR_OUTPUT_LENGTH: return "matvec output length does not match the rows";
    case DM_ERR_EMPTY_INPUT: return "empty input";
    case DM_ERR_NON_FINITE: return "non-finite value";
    case DM_ERR_TOP_K: return "top-k count out of range";
    case DM_ERR_MAPPED_RANGE: return "range exceeds the mapped buffer";
    case DM_ERR_OVERFLOW: return "size overflow";
    case DM_ERR_COMMAND: return "CUDA command failed";
    case DM_ERR_INVALID_EXPERT: return "invalid expert";
    case DM_ERR_INVALID_LAYER: return "invalid layer";
    case DM_ERR_ALL_SLOTS_PINNED: return "all expert slots are pinned";
    case DM_ERR_CANCELLED: return "cancelled";
    case DM_ERR_NO_SLOTS: return "expert cache requires at least one slot";
    case DM_ERR_VECTOR_LENGTH: return "vector length mismatch";
    case DM_ERR_POSITIVE_PARAMETER: return "parameter must be finite and positive";
    case DM_ERR_TIMEOUT: return "a bounded wait ran out";
    case DM_ERR_NOT_BUILT: return "component not built";
    case DM_ERR_COMMUNICATOR: return "expert-parallel exchange failed";
    case DM_ERR_IO: return "expert source read failed";
    case DM_ERR_FORMAT: return "malformed model file index";
    default: return "unknown status";
  }
}

const char *dm_last_error_message(void) { return g_message; }

int32_t dm_cuda_create(int32_t device_ordinal, dm_cuda_context **out) {
  if (!out) return fail(DM_ERR_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
    return fail(DM_ERR_NO_DEVICE, "no CUDA device is available");
  if (device_ordinal < 0 || device_ordinal >= count)
    return fail(DM_ERR_NO_DEVICE, "device %d is outside the %d visible devices", device_ordinal,
                count);
  DM_CUDA(cudaSetDevice(device_ordinal), "cudaSetDevice");
  auto *ctx = new (std::nothrow) dm_cuda_context();
  if (!ctx) return fail(DM_ERR_ALLOCATION, "host allocation failed");
  ctx->device = device_ordinal;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device_ordinal) == cudaSuccess)
    snprintf(ctx->name, sizeof ctx->name, "%s", prop.name);
  cudaError_t err = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  if (err == cudaSuccess) err = cudaMalloc(&ctx->status, 256);
  if (err != cudaSuccess) {
    delete ctx;
    return cuda_fail(err, "context set-up");
  }
  *out = ctx;
  return DM_OK;
}

}  // extern "C"

static void free_context(dm_cuda_context *ctx) {
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->status) cudaFree(ctx->status);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  cudaGetLastError();  // teardown leaves no error behind for unrelated calls
  delete ctx;
}

static std::mutex g_ctx_mutex;

void dmi::retain_context(dm_cuda_context *ctx) {
  std::lock_guard<std::mutex> lock(g_ctx_mutex);
  ctx->refs++;
}

void dmi::release_context(dm_cuda_context *ctx) {
  bool last = false;
  {
    std::lock_guard<std::mutex> lock(g_ctx_mutex);
    last = --ctx->refs == 0 && ctx->closed;
  }
  if (last) free_context(ctx);
}

extern "C" {

void dm_cuda_destroy(dm_cuda_context *ctx) {
  if (!ctx) return;
  bool now = false;
  {
    std::lock_guard<std::mutex> lock(g_ctx_mutex);
    ctx->closed = true;
    now = ctx->refs == 0;
  }
  if (now) free_context(ctx);
}

int32_t dm_cuda_device_name(const dm_cuda_context *ctx, char *name, size_t capacity) {
  if (!ctx || !name || capacity == 0) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  snprintf(name, capacity, "%s", ctx->name);
  return DM_OK;
}

int32_t dm_cuda_synchronize(dm_cuda_context *ctx) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  cudaSetDevice(ctx->device);
  DM_CUDA(cudaDeviceSynchronize(), "device synchronize");
  return DM_OK;
}

// ---- buffers ----

static int32_t new_buffer(dm_cuda_context *ctx, size_t length, bool read_only, dm_buffer **out) {
  if (!ctx || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (length == 0) return fail(DM_ERR_ALLOCATION, "could not allocate a 0-byte buffer");
  cudaSetDevice(ctx->device);
  void *p = nullptr;
  if (cudaMalloc(&p, length) != cudaSuccess)
    return fail(DM_ERR_ALLOCATION, "could not allocate a %zu-byte device buffer", length);
  auto *b = new (std::nothrow) dm_buffer();
  if (!b) {
    cudaFree(p);
    return fail(DM_ERR_ALLOCATION, "host allocation failed");
  }
  b->ctx = ctx;
  retain_context(ctx);
  b->device = p;
  b->length = length;
  b->read_only = read_only;
  *out = b;
  return DM_OK;
}

int32_t dm_cuda_map_read_only(dm_cuda_context *ctx, const void *host, size_t length,
                              dm_buffer **out) {
  if (!host) return fail(DM_ERR_INVALID_ARGUMENT, "null host mapping");
  int32_t rc = new_buffer(ctx, length, true, out);
  if (rc != DM_OK) return rc;
  cudaError_t err = cudaMemcpy((*out)->device, host, length, cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    dm_buffer_free(*out);
    *out = nullptr;
    return cuda_fail(err, "upload of a read-only mapping");
  }
  return DM_OK;
}

int32_t dm_cuda_new_owned_buffer(dm_cuda_context *ctx, size_t length, dm_buffer **out) {
  int32_t rc = new_buffer(ctx, length, false, out);
  if (rc != DM_OK) return rc;
  DM_CUDA(cudaMemset((*out)->device, 0, length), "zero a new buffer");
  return DM_OK;
}

static int32_t check_range(const dm_buffer *b, size_t offset, size_t length) {
  if (!b) return fail(DM_ERR_INVALID_ARGUMENT, "null buffer");
  size_t end = offset + length;
  if (end < offset) return fail(DM_ERR_OVERFLOW, "range overflows");
  if (end > b->length)
    return fail(DM_ERR_MAPPED_RANGE, "range %zu..%zu exceeds its %zu-byte buffer", offset, end,
                b->length);
  return DM_OK;
}

int32_t dm_buffer_write(dm_buffer *b, size_t offset, const void *source, size_t length) {
  int32_t rc = check_range(b, offset, length);
  if (rc != DM_OK) return rc;
  if (b->read_only) return fail(DM_ERR_INVALID_ARGUMENT, "buffer is read-only");
  if (length == 0) return DM_OK;
  cudaSetDevice(b->ctx->device);
  DM_CUDA(cudaMemcpy((uint8_t *)b->device + offset, source, length, cudaMemcpyHostToDevice),
          "buffer write");
  return DM_OK;
}

int32_t dm_buffer_read(const dm_buffer *b, size_t offset, void *destination, size_t length) {
  int32_t rc = check_range(b, offset, length);
  if (rc != DM_OK) return rc;
  if (length == 0) return DM_OK;
  cudaSetDevice(b->ctx->device);
  DM_CUDA(cudaMemcpy(destination, (const uint8_t *)b->device + offset, length,
                     cudaMemcpyDeviceToHost),
          "buffer read");
  return DM_OK;
}

size_t dm_buffer_length(const dm_buffer *b) { return b ? b->length : 0; }
void *dm_buffer_device_pointer(const dm_buffer *b) { return b ? b->device : nullptr; }

void dm_buffer_free(dm_buffer *b) {
  if (!b) return;
  dm_cuda_context *ctx = b->ctx;
  cudaSetDevice(ctx->device);
  cudaFree(b->device);
  cudaGetLastError();
  delete b;
  release_context(ctx);
}

// ---- operators ----

static bool supported_matvec_type(int32_t kind) {
  switch (kind) {
    case DM_F32: case DM_F16: case DM_BF16: case DM_Q5_0: case DM_Q8_0: case DM_Q4_K:
    case DM_Q6_K:
      return true;
    default:
      return false;
  }
}

// prepare_matvec (src/metal.rs:1513-1560): lengths, type, element count, bytes.
static int32_t prepare_matvec(int32_t kind, size_t rows, size_t columns, size_t encoded_length,
                              size_t input_length, size_t output_length, uint64_t *row_bytes) {
  if (input_length != columns)
    return fail(DM_ERR_INPUT_LENGTH, "matvec input has %zu columns; expected %zu", input_length,
                columns);
  if (output_length != rows)
    return fail(DM_ERR_OUTPUT_LENGTH, "matvec output has %zu rows; expected %zu", output_length,
                rows);
  if (!supported_matvec_type(kind))
    return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "matrix-vector multiplication does not support type %d", kind);
  uint64_t rb = dm::row_bytes(kind, columns);
  if (rb == 0 && columns != 0)
    return fail(DM_ERR_ELEMENT_COUNT, "output length %zu is not a whole number of blocks", columns);
  if (rb != 0 && rows > UINT64_MAX / rb) return fail(DM_ERR_OVERFLOW, "matrix size overflows");
  if ((uint64_t)encoded_length != rows * rb)
    return fail(DM_ERR_BYTE_LENGTH, "requires %llu encoded bytes, got %zu",
                (unsigned long long)(rows * rb), encoded_length);
  *row_bytes = rb;
  return DM_OK;
}

static int32_t run_matvec(dm_cuda_context *ctx, int32_t kind, size_t rows, size_t columns,
                          const uint8_t *device_matrix, const float *input, float *output) {
  if (rows > INT32_MAX || columns > INT32_MAX) return fail(DM_ERR_OVERFLOW, "shape too large");
  size_t in_bytes = (columns * 4 + 255) & ~size_t(255);
  size_t out_bytes = (rows * 4 + 255) & ~size_t(255);
  int32_t rc = ctx->ensure_scratch(in_bytes + out_bytes);
  if (rc != DM_OK) return rc;
  float *x = (float *)ctx->scratch;
  float *y = (float *)((uint8_t *)ctx->scratch + in_bytes);
  DM_CUDA(cudaMemcpyAsync(x, input, columns * 4, cudaMemcpyHostToDevice, ctx->stream), "input copy");
  if (dm::launch_gemv(kind, device_matrix, (int)rows, (int)columns, x, y, ctx->stream) < 0)
    return fail(DM_ERR_INVALID_ARGUMENT, "matrix rows are not 16-byte aligned");
  DM_CUDA(cudaGetLastError(), "matvec launch");
  DM_CUDA(cudaMemcpyAsync(output, y, rows * 4, cudaMemcpyDeviceToHost, ctx->stream), "output copy");
  DM_CUDA(cudaStreamSynchronize(ctx->stream), "matvec");
  return DM_OK;
}

int32_t dm_cuda_matvec(dm_cuda_context *ctx, int32_t kind, size_t rows, size_t columns,
                       const uint8_t *encoded, size_t encoded_length, const float *input,
                       size_t input_length, float *output, size_t output_length) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  uint64_t rb = 0;
  int32_t rc = prepare_matvec(kind, rows, columns, encoded_length, input_length, output_length, &rb);
  if (rc != DM_OK) return rc;
  if (rows == 0) return DM_OK;
  if (input_length == 0) return fail(DM_ERR_EMPTY_INPUT, "matvec requires a non-empty input");
  cudaSetDevice(ctx->device);
  void *matrix = nullptr;
  if (cudaMalloc(&matrix, encoded_length) != cudaSuccess)
    return fail(DM_ERR_ALLOCATION, "could not allocate a %zu-byte device buffer", encoded_length);
  cudaError_t err = cudaMemcpy(matrix, encoded, encoded_length, cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    cudaFree(matrix);
    return cuda_fail(err, "matrix upload");
  }
  rc = run_matvec(ctx, kind, rows, columns, (const uint8_t *)matrix, input, output);
  cudaFree(matrix);
  return rc;
}

int32_t dm_cuda_matvec_mapped(dm_cuda_context *ctx, int32_t kind, size_t rows, size_t columns,
                              const dm_buffer *mapped, size_t offset, size_t encoded_length,
                              const float *input, size_t input_length, float *output,
                              size_t output_length) {
  if (!ctx || !mapped) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  uint64_t rb = 0;
  int32_t rc = prepare_matvec(kind, rows, columns, encoded_length, input_length, output_length, &rb);
  if (rc != DM_OK) return rc;
  rc = check_range(mapped, offset, encoded_length);
  if (rc != DM_OK) return rc;
  if (rows == 0) return DM_OK;
  if (input_length == 0) return fail(DM_ERR_EMPTY_INPUT, "matvec requires a non-empty input");
  cudaSetDevice(ctx->device);
  return run_matvec(ctx, kind, rows, columns, (const uint8_t *)mapped->device + offset, input,
                    output);
}

// u8_matrix_encoding (src/metal.rs:1893-1942): int8 rows when rows * columns bytes and
// one scale per row; otherwise int4 with rows * ceil(columns / 2) bytes and one scale per
// row (one group spanning the row) or the first group size of {16, 32, 48, 64, 96, 128,
// 192, 256} (not above `columns`) whose scale count matches.
static int32_t u8_encoding(size_t rows, size_t columns, size_t encoded_length, size_t scales,
                           int *enc, int *group) {
  if (columns && rows > SIZE_MAX / columns) return fail(DM_ERR_OVERFLOW, "matrix size overflows");
  if (encoded_length == rows * columns && scales == rows) {
    *enc = dm::kQuantI8Row;
    *group = 0;
    return DM_OK;
  }
  const size_t int4_bytes = rows * ((columns + 1) / 2);
  if (encoded_length != int4_bytes)
    return fail(DM_ERR_BYTE_LENGTH, "U8 quantized matrix requires %zu encoded bytes, got %zu",
                int4_bytes, encoded_length);
  if (scales == rows) {
    *enc = dm::kQuantI4;
    *group = (int)std::max<size_t>(columns, 1);
    return DM_OK;
  }
  static const size_t groups[8] = {16, 32, 48, 64, 96, 128, 192, 256};
  for (size_t g : groups) {
    if (g > columns) break;
    if (scales == rows * ((columns + g - 1) / g)) {
      *enc = dm::kQuantI4;
      *group = (int)g;
      return DM_OK;
    }
  }
  return fail(DM_ERR_BYTE_LENGTH, "U8 quantization scales require %zu bytes, got %zu", rows * 4,
              scales * 4);
}

int32_t dm_cuda_matvec_safetensor(dm_cuda_context *ctx, int32_t dtype, size_t rows,
                                  size_t columns, const uint8_t *encoded, size_t encoded_length,
                                  const float *scales, size_t scale_count, const float *input,
                                  size_t input_length, float *output, size_t output_length) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  if (dtype == DM_F32 || dtype == DM_F16 || dtype == DM_BF16)
    return dm_cuda_matvec(ctx, dtype, rows, columns, encoded, encoded_length, input, input_length,
                          output, output_length);
  if (dtype != DM_U8_QUANT && dtype != DM_F8_E4M3)
    return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "safetensors dtype %d is not supported", dtype);
  if (input_length != columns)
    return fail(DM_ERR_INPUT_LENGTH, "matvec input has %zu columns; expected %zu", input_length,
                columns);
  if (output_length != rows)
    return fail(DM_ERR_OUTPUT_LENGTH, "matvec output has %zu rows; expected %zu", output_length,
                rows);
  int enc = dm::kQuantF8, group = 0;
  size_t expect_scales = 0;
  if (dtype == DM_U8_QUANT) {
    if (!scales)
      return fail(DM_ERR_BYTE_LENGTH, "U8 quantization scales require %zu bytes, got 0", rows * 4);
    int32_t rc = u8_encoding(rows, columns, encoded_length, scale_count, &enc, &group);
    if (rc != DM_OK) return rc;
    expect_scales = scale_count;
  } else {
    if (columns && rows > SIZE_MAX / columns) return fail(DM_ERR_OVERFLOW, "matrix size overflows");
    if (encoded_length != rows * columns)
      return fail(DM_ERR_BYTE_LENGTH, "F8_E4M3FN requires %zu encoded bytes, got %zu",
                  rows * columns, encoded_length);
    expect_scales = ((rows + 127) / 128) * ((columns + 127) / 128);
    if (!scales || scale_count != expect_scales)
      return fail(DM_ERR_VECTOR_LENGTH, "F8_E4M3FN matvec scales: expected %zu, got %zu",
                  expect_scales, scales ? scale_count : (size_t)0);
  }
  if (rows == 0) return DM_OK;
  if (input_length == 0) return fail(DM_ERR_EMPTY_INPUT, "safetensors matvec requires a non-empty input");
  if (rows > INT32_MAX || columns > INT32_MAX) return fail(DM_ERR_OVERFLOW, "shape too large");
  cudaSetDevice(ctx->device);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t need = al(encoded_length) + al(expect_scales * 4) + al(columns * 4) + al(rows * 4);
  int32_t rc = ctx->ensure_scratch(need);
  if (rc != DM_OK) return rc;
  uint8_t *w = (uint8_t *)ctx->scratch;
  float *sc = (float *)(w + al(encoded_length));
  float *x = (float *)((uint8_t *)sc + al(expect_scales * 4));
  float *y = (float *)((uint8_t *)x + al(columns * 4));
  cudaStream_t s = ctx->stream;
  DM_CUDA(cudaMemcpyAsync(w, encoded, encoded_length, cudaMemcpyHostToDevice, s), "matrix copy");
  DM_CUDA(cudaMemcpyAsync(sc, scales, expect_scales * 4, cudaMemcpyHostToDevice, s), "scale copy");
  DM_CUDA(cudaMemcpyAsync(x, input, columns * 4, cudaMemcpyHostToDevice, s), "input copy");
  dm::launch_quant_gemv(enc, w, sc, (int)rows, (int)columns, group, x, y, s);
  DM_CUDA(cudaGetLastError(), "matvec launch");
  DM_CUDA(cudaMemcpyAsync(output, y, rows * 4, cudaMemcpyDeviceToHost, s), "output copy");
  DM_CUDA(cudaStreamSynchronize(s), "matvec");
  return DM_OK;
}

int32_t dm_cuda_top_k_softmax(dm_cuda_context *ctx, const float *logits, size_t length, size_t k,
                              uint32_t *indices, float *probabilities) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  if (k == 0 || k > length) return fail(DM_ERR_TOP_K, "top-k count %zu is outside 1..=%zu", k, length);
  if (k > 32) return fail(DM_ERR_TOP_K, "top-k count %zu exceeds the kernel limit of 32", k);
  for (size_t i = 0; i < length; i++)
    if (!std::isfinite(logits[i])) return fail(DM_ERR_NON_FINITE, "top-k softmax received a non-finite value");
  if (length > INT32_MAX) return fail(DM_ERR_OVERFLOW, "input too large");
  cudaSetDevice(ctx->device);
  size_t in_bytes = (length * 4 + 255) & ~size_t(255);
  int32_t rc = ctx->ensure_scratch(in_bytes + 512);
  if (rc != DM_OK) return rc;
  float *lg = (float *)ctx->scratch;
  uint32_t *idx = (uint32_t *)((uint8_t *)ctx->scratch + in_bytes);
  float *prob = (float *)(idx + 64);
  DM_CUDA(cudaMemcpyAsync(lg, logits, length * 4, cudaMemcpyHostToDevice, ctx->stream), "copy");
  DM_CUDA(cudaMemsetAsync(ctx->status, 0, 4, ctx->stream), "status reset");
  dm::launch_topk_softmax(lg, (int)length, (int)k, idx, prob, ctx->status, ctx->stream);
  DM_CUDA(cudaGetLastError(), "top-k launch");
  DM_CUDA(cudaMemcpyAsync(indices, idx, k * 4, cudaMemcpyDeviceToHost, ctx->stream), "copy");
  DM_CUDA(cudaMemcpyAsync(probabilities, prob, k * 4, cudaMemcpyDeviceToHost, ctx->stream), "copy");
  DM_CUDA(cudaStreamSynchronize(ctx->stream), "top-k softmax");
  return DM_OK;
}

static int32_t run_elementwise(dm_cuda_context *ctx, int op, const char *name, const float *gate,
                               const float *up, float *output, size_t length) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  if (length == 0) return fail(DM_ERR_EMPTY_INPUT, "%s requires a non-empty input", name);
  if (length > INT32_MAX) return fail(DM_ERR_OVERFLOW, "input too large");
  cudaSetDevice(ctx->device);
  size_t bytes = (length * 4 + 255) & ~size_t(255);
  int32_t rc = ctx->ensure_scratch(3 * bytes);
  if (rc != DM_OK) return rc;
  float *g = (float *)ctx->scratch;
  float *u = (float *)((uint8_t *)ctx->scratch + bytes);
  float *o = (float *)((uint8_t *)ctx->scratch + 2 * bytes);
  DM_CUDA(cudaMemcpyAsync(g, gate, length * 4, cudaMemcpyHostToDevice, ctx->stream), "copy");
  DM_CUDA(cudaMemcpyAsync(u, up, length * 4, cudaMemcpyHostToDevice, ctx->stream), "copy");
  dm::launch_elementwise(op, g, u, o, (int)length, 0.0f, ctx->stream);
  DM_CUDA(cudaGetLastError(), "elementwise launch");
  DM_CUDA(cudaMemcpyAsync(output, o, length * 4, cudaMemcpyDeviceToHost, ctx->stream), "copy");
  DM_CUDA(cudaStreamSynchronize(ctx->stream), name);
  return DM_OK;
}

int32_t dm_cuda_gelu_mul(dm_cuda_context *ctx, const float *gate, const float *up, float *output,
                         size_t length) {
  return run_elementwise(ctx, dm::kOpGeluMul, "GELU multiply", gate, up, output, length);
}

int32_t dm_cuda_silu_mul(dm_cuda_context *ctx, const float *gate, const float *up, float *output,
                         size_t length) {
  return run_elementwise(ctx, dm::kOpSiluMul, "SiLU multiply", gate, up, output, length);
}

// MetalContext::rms_norm (src/metal.rs:435-476) validation; CPU arithmetic (bit-exact).
int32_t dm_cuda_rms_norm(dm_cuda_context *ctx, const float *input, const float *weight,
                         size_t length, float epsilon, float *output) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  if (length == 0) return fail(DM_ERR_EMPTY_INPUT, "RMSNorm requires a non-empty input");
  if (!std::isfinite(epsilon) || epsilon <= 0.0f)
    return fail(DM_ERR_POSITIVE_PARAMETER, "RMSNorm epsilon requires a finite positive parameter");
  for (size_t i = 0; i < length; i++)
    if (!std::isfinite(input[i])) return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");
  if (length > INT32_MAX) return fail(DM_ERR_OVERFLOW, "input too large");
  cudaSetDevice(ctx->device);
  size_t bytes = (length * 4 + 255) & ~size_t(255);
  int32_t rc = ctx->ensure_scratch(3 * bytes);
  if (rc != DM_OK) return rc;
  float *x = (float *)ctx->scratch;
  float *w = (float *)((uint8_t *)ctx->scratch + bytes);
  float *o = (float *)((uint8_t *)ctx->scratch + 2 * bytes);
  DM_CUDA(cudaMemcpyAsync(x, input, length * 4, cudaMemcpyHostToDevice, ctx->stream), "copy");
  if (weight)
    DM_CUDA(cudaMemcpyAsync(w, weight, length * 4, cudaMemcpyHostToDevice, ctx->stream), "copy");
  DM_CUDA(cudaMemsetAsync(ctx->status, 0, 4, ctx->stream), "status reset");
  dm::launch_rms_norm(x, weight ? w : nullptr, o, (int)length, epsilon, ctx->status, ctx->stream);
  DM_CUDA(cudaGetLastError(), "rms_norm launch");
  int32_t status = 0;
  DM_CUDA(cudaMemcpyAsync(output, o, length * 4, cudaMemcpyDeviceToHost, ctx->stream), "copy");
  DM_CUDA(cudaMemcpyAsync(&status, ctx->status, 4, cudaMemcpyDeviceToHost, ctx->stream), "copy");
  DM_CUDA(cudaStreamSynchronize(ctx->stream), "rms_norm");
  if (status) return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");
  return DM_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// MoE layer
// ---------------------------------------------------------------------------


namespace {

int32_t validate_desc(const dm_moe_desc *d) {
  if (!d) return fail(DM_ERR_INVALID_ARGUMENT, "null descriptor");
  if (d->family != DM_FAMILY_GEMMA4 && d->family != DM_FAMILY_QWEN35_MOE &&
      d->family != DM_FAMILY_GLM52)
    return fail(DM_ERR_INVALID_ARGUMENT, "unknown family %d", d->family);
  if (d->hidden <= 0 || d->intermediate <= 0 || d->experts <= 0)
    return fail(DM_ERR_INVALID_ARGUMENT, "hidden, intermediate and experts must be positive");
  if (d->hidden % 32 || d->intermediate % 32)
    return fail(DM_ERR_ELEMENT_COUNT, "hidden and intermediate must be multiples of 32");
  if (d->hidden > 12288)
    return fail(DM_ERR_ELEMENT_COUNT, "hidden %d is above the supported 12288", d->hidden);
  if (d->top_k <= 0 || d->top_k > d->experts || d->top_k > 32)
    return fail(DM_ERR_TOP_K, "top-k count %d is outside 1..=%d", d->top_k, std::min(d->experts, 32));
  if (d->experts > 1023) return fail(DM_ERR_INVALID_ARGUMENT, "at most 1023 experts");
  if (!d->router || !d->gate || !d->down) return fail(DM_ERR_INVALID_ARGUMENT, "null weight pointer");
  int types[3] = {d->gate_type, d->up_type, d->down_type};
  for (int i = 0; i < 3; i++) {
    if (i == 1 && d->family == DM_FAMILY_GEMMA4) continue;
    if (!supported_matvec_type(types[i]))
      return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "unsupported expert tensor type %d", types[i]);
  }
  if (d->family != DM_FAMILY_GEMMA4 && d->gate_type != d->up_type)
    return fail(DM_ERR_INVALID_ARGUMENT, "gate and up must share a type");
  if (dm::row_bytes(d->gate_type, d->hidden) == 0 || dm::row_bytes(d->down_type, d->intermediate) == 0)
    return fail(DM_ERR_ELEMENT_COUNT, "expert rows are not a whole number of blocks");
  if (d->family == DM_FAMILY_GEMMA4) {
    if (!d->router_scale || !d->routed_pre_norm || !d->expert_scale)
      return fail(DM_ERR_INVALID_ARGUMENT, "Gemma needs router_scale, routed_pre_norm, expert_scale");
    if (!std::isfinite(d->epsilon) || d->epsilon <= 0.0f)
      return fail(DM_ERR_POSITIVE_PARAMETER, "RMSNorm epsilon requires a finite positive parameter");
    if (d->router_type != DM_F32 || d->input_type != DM_F32)
      return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "Gemma router and input are f32");
  } else {
    if (!d->up) return fail(DM_ERR_INVALID_ARGUMENT, "null up pointer");
  }
  if (d->family == DM_FAMILY_QWEN35_MOE) {
    if (d->router_type != DM_F32 || d->input_type != DM_F32)
      return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "Qwen router and input are f32");
    if (d->shared_intermediate > 0 && !d->shared_gate_vector)
      return fail(DM_ERR_INVALID_ARGUMENT, "Qwen shared expert needs shared_gate_vector");
  }
  if (d->family == DM_FAMILY_GLM52) {
    if (!d->correction_bias) return fail(DM_ERR_INVALID_ARGUMENT, "GLM needs correction_bias");
    if (d->router_type != DM_BF16 && d->router_type != DM_F32)
      return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "GLM router must be bf16 or f32");
    if (d->input_type != DM_BF16 && d->input_type != DM_F32)
      return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "GLM input must be bf16 or f32");
    int g = d->n_groups <= 0 ? 1 : d->n_groups, kg = d->topk_groups <= 0 ? 1 : d->topk_groups;
    if (d->experts % g || kg > g || g > 32 || (g > 1 && d->experts / g < 2))
      return fail(DM_ERR_INVALID_ARGUMENT, "invalid expert groups %d/%d", g, kg);
    if (d->top_k > kg * (d->experts / g)) return fail(DM_ERR_TOP_K, "top-k exceeds the kept groups");
  }
  if (d->shared_intermediate > 0) {
    if (d->shared_intermediate != d->intermediate)
      return fail(DM_ERR_INVALID_ARGUMENT, "shared intermediate must equal the routed intermediate");
    if (!d->shared_gate || !d->shared_up || !d->shared_down)
      return fail(DM_ERR_INVALID_ARGUMENT, "null shared expert pointer");
    if (d->family == DM_FAMILY_GEMMA4)
      return fail(DM_ERR_INVALID_ARGUMENT, "Gemma's shared FFN is outside the routed branch");
  }
  // vector loads need 16-byte aligned rows for the block formats that use them
  auto aligned = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  if ((d->gate_type == DM_Q4_K || d->gate_type == DM_BF16 || d->gate_type == DM_F32) &&
      (!aligned(d->gate) || (d->up && !aligned(d->up)) ||
       (d->shared_gate && (!aligned(d->shared_gate) || !aligned(d->shared_up)))))
    return fail(DM_ERR_INVALID_ARGUMENT, "gate/up weights must be 16-byte aligned");
  if ((d->down_type == DM_Q4_K || d->down_type == DM_BF16 || d->down_type == DM_F32) &&
      (!aligned(d->down) || (d->shared_down && !aligned(d->shared_down))))
    return fail(DM_ERR_INVALID_ARGUMENT, "down weights must be 16-byte aligned");
  return DM_OK;
}

// Repack `blocks` blocks of a Q6_K / Q5_0 / Q8_0 tensor into the split layout.
int32_t make_split(dm_moe_layer *L, int kind, const void *src, uint64_t blocks,
                   dm::SplitTensor *out) {
  dm::SplitLayout s = dm::split_layout(kind);
  if (s.quant_bytes == 0 || !src) return DM_OK;
  auto al = [](uint64_t b) { return (b + 255) & ~uint64_t(255); };
  uint64_t bytes = al(blocks * s.quant_bytes) + al(blocks * s.qh_bytes) + al(blocks * 2);
  void *mem = nullptr;
  if (cudaMalloc(&mem, bytes) != cudaSuccess)
    return fail(DM_ERR_ALLOCATION, "could not allocate %llu bytes for a repacked tensor",
                (unsigned long long)bytes);
  L->owned.push_back(mem);
  uint8_t *p = (uint8_t *)mem;
  out->quant = p;
  out->qh = s.qh_bytes ? p + al(blocks * s.quant_bytes) : nullptr;
  out->d = (uint16_t *)(p + al(blocks * s.quant_bytes) + al(blocks * s.qh_bytes));
  dm::launch_repack(kind, (const uint8_t *)src, blocks, *out, L->ctx->stream);
  return DM_OK;
}

// Tensor-core weight views: TMA maps over the gate/up and down weights and the per-step
// transposed down side arrays. A refused map leaves the layer on the GEMV path.
int32_t build_tc_weights(dm_moe_layer *L) {
  const dm_moe_desc &d = L->desc;
  if (d.down_type == DM_BF16) {
    // fp16 copies of the down weights: bf16 -> fp16 is exact for magnitudes in fp16's
    // normal range, and the down product then takes one fp16 MMA per K step on single
    // fp16 intermediates instead of two bf16 MMAs on hi + lo halves
    uint8_t *down16 = nullptr, *sh_down16 = nullptr;
    if (L->tc_f16_down && ((uintptr_t)d.down | (uintptr_t)d.shared_down) % 16 == 0) {
      const uint64_t n = (uint64_t)L->local_experts * d.hidden * d.intermediate;
      const uint64_t n_sh = L->shared ? (uint64_t)d.hidden * d.intermediate : 0;
      void *mem = nullptr;
      if (cudaMalloc(&mem, (n + n_sh) * 2) == cudaSuccess) {
        L->owned.push_back(mem);
        down16 = (uint8_t *)mem;
        dm::launch_bf16_to_f16(d.down, down16, n, L->ctx->stream);
        if (n_sh) {
          sh_down16 = down16 + n * 2;
          dm::launch_bf16_to_f16(d.shared_down, sh_down16, n_sh, L->ctx->stream);
        }
      } else {
        cudaGetLastError();  // no room for the copies: the hi + lo bf16 down path
      }
    }
    if (dm::make_tc_weights_bf16(L->tcw, (const uint8_t *)d.gate, L->up_base, L->gate_stride,
                                 (const uint8_t *)d.shared_gate, (const uint8_t *)d.shared_up,
                                 (const uint8_t *)d.down, (const uint8_t *)d.shared_down,
                                 L->local_experts, d.hidden, d.intermediate, down16,
                                 sh_down16) != 0) {
      fprintf(stderr, "diskmule_cuda: tensor-core path off for this layer (weight maps refused)\n");
      L->tc_ok = false;
    }
    // the largest gate-row and up-row norms of each expert (index E: the shared expert),
    // from which the fused gate/up epilogue scales the intermediates into fp16
    const int E = L->local_experts;
    void *norms = nullptr;
    if (L->tc_ok && down16 && cudaMalloc(&norms, 2 * (size_t)(E + 1) * sizeof(float)) == cudaSuccess) {
      L->owned.push_back(norms);
      float *gn = (float *)norms, *un = gn + E + 1;
      cudaMemsetAsync(norms, 0, 2 * (size_t)(E + 1) * sizeof(float), L->ctx->stream);
      const int H = d.hidden, I = d.intermediate;
      dm::launch_row_norm_max(d.gate, L->gate_stride, E, I, H, gn, L->ctx->stream);
      dm::launch_row_norm_max(L->up_base, L->up_stride, E, I, H, un, L->ctx->stream);
      if (L->shared) {
        dm::launch_row_norm_max(d.shared_gate, 0, 1, I, H, gn + E, L->ctx->stream);
        dm::launch_row_norm_max(d.shared_up, 0, 1, I, H, un + E, L->ctx->stream);
      }
      L->tcw.side.gate_norm = gn;
      L->tcw.side.up_norm = un;
    } else {
      cudaGetLastError();  // without the norms the gate/up product keeps the separate pack
    }
    return DM_OK;
  }
  uint64_t qh_bytes = 0, d_bytes = 0, sh_qh_bytes = 0, sh_d_bytes = 0;
  dm::tc_side_bytes(d.down_type, L->local_experts, d.hidden, d.intermediate, &qh_bytes, &d_bytes);
  if (L->shared)
    dm::tc_side_bytes(d.down_type, 1, d.hidden, d.intermediate, &sh_qh_bytes, &sh_d_bytes);
  uint8_t *bufs[4] = {nullptr, nullptr, nullptr, nullptr};
  const uint64_t sizes[4] = {qh_bytes, d_bytes, sh_qh_bytes, sh_d_bytes};
  for (int i = 0; i < 4; i++) {
    if (!sizes[i]) continue;
    void *mem = nullptr;
    if (cudaMalloc(&mem, sizes[i]) != cudaSuccess)
      return fail(DM_ERR_ALLOCATION, "could not allocate %llu bytes for tensor-core side arrays",
                  (unsigned long long)sizes[i]);
    L->owned.push_back(mem);
    bufs[i] = (uint8_t *)mem;
  }
  if (dm::make_tc_weights(L->tcw, (const uint8_t *)d.gate, L->up_base, L->gate_stride,
                          (const uint8_t *)d.shared_gate, (const uint8_t *)d.shared_up,
                          L->plan.down, L->plan.sh_down, d.down_type, L->local_experts, d.hidden,
                          d.intermediate, bufs[0], bufs[1], bufs[2], bufs[3], L->ctx->stream) != 0) {
    fprintf(stderr, "diskmule_cuda: tensor-core path off for this layer (weight maps refused)\n");
    L->tc_ok = false;
  }
  return DM_OK;
}

int32_t build_plan(dm_moe_layer *L) {
  const dm_moe_desc &d = L->desc;
  const uint64_t E = L->local_experts, H = d.hidden, I = d.intermediate;
  int e = 0, b = 0;
  auto nblocks = [&](int kind, uint64_t rows, uint64_t cols) {
    dm::block_layout(kind, &e, &b);
    return rows * (cols / (uint64_t)e);
  };
  const bool fused = d.family == DM_FAMILY_GEMMA4;
  int32_t rc = DM_OK;
  const uint64_t up_rows = fused ? 2 * I : I;
  rc = make_split(L, d.gate_type, d.gate, E * nblocks(d.gate_type, up_rows, H), &L->plan.gate);
  if (rc == DM_OK && fused) L->plan.up = L->plan.gate;
  if (rc == DM_OK && !fused)
    rc = make_split(L, d.up_type, d.up, E * nblocks(d.up_type, I, H), &L->plan.up);
  if (rc == DM_OK)
    rc = make_split(L, d.down_type, d.down, E * nblocks(d.down_type, H, I), &L->plan.down);
  if (rc == DM_OK && L->shared) {
    rc = make_split(L, d.gate_type, d.shared_gate, nblocks(d.gate_type, I, H), &L->plan.sh_gate);
    if (rc == DM_OK)
      rc = make_split(L, d.up_type, d.shared_up, nblocks(d.up_type, I, H), &L->plan.sh_up);
    if (rc == DM_OK)
      rc = make_split(L, d.down_type, d.shared_down, nblocks(d.down_type, H, I), &L->plan.sh_down);
  }
  return rc;
}

}  // namespace

namespace dmi {

int32_t ensure_layer_scratch(dm_moe_layer *L, int tokens) {
  if (tokens <= L->capacity) return DM_OK;
  const dm_moe_desc &d = L->desc;
  size_t T = (size_t)std::max(tokens, 1), H = d.hidden, I = d.intermediate, E = d.experts,
         k = d.top_k;
  size_t pairs = T * k + (L->shared ? T : 0);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  size_t bytes = 0;
  if (d.family == DM_FAMILY_GEMMA4) bytes += 2 * al(T * H * 4);
  bytes += al(T * L->E1 * 4) + 2 * al(T * k * 4);
  bytes += al((E + 1) * 4) + al((E + 2) * 4) + 2 * al(pairs * 4) + al((E + 1) * 4) + 2 * al(4);
  bytes += al((pairs + E + 1) * sizeof(int4)) + al(4);
  bytes += al(pairs * I * 4) + al(pairs * H * 4);
  const uint64_t xld = (T + 31) / 32 * 32;  // transposed router input for many tokens
  bytes += al(H * xld * 8) + al((xld / 32) * ((H + 31) / 32));
  if (L->tc_ok)
    bytes += al(2 * pairs * H * 2) + al(2 * pairs * I * 2) + 2 * al(pairs * 4) + al(2 * pairs * I * 4);
  L->drop_graphs();
  if (L->scratch) {
    cudaDeviceSynchronize();
    cudaFree(L->scratch);
  }
  L->scratch = nullptr;
  L->capacity = 0;
  if (cudaMalloc(&L->scratch, bytes) != cudaSuccess)
    return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of layer scratch", bytes);
  L->scratch_bytes = bytes;
  dm::Arena arena{(uint8_t *)L->scratch, 0, bytes};
  dm::ForwardArgs &a = L->args;
  a.router_in = d.family == DM_FAMILY_GEMMA4 ? arena.take<float>(T * H) : nullptr;
  a.expert_in = d.family == DM_FAMILY_GEMMA4 ? arena.take<float>(T * H) : nullptr;
  a.logits = arena.take<float>(T * L->E1);
  a.xT = arena.take<float>(H * xld * 2);
  a.x_tiny = arena.take<uint8_t>((xld / 32) * ((H + 31) / 32));
  a.sel_idx = arena.take<uint32_t>(T * k);
  a.sel_w = arena.take<float>(T * k);
  a.counts = arena.take<int32_t>(E + 1);
  a.offsets = arena.take<int32_t>(E + 2);
  a.sorted = arena.take<int32_t>(pairs);
  a.inverse = arena.take<int32_t>(pairs);
  a.active = arena.take<int32_t>(E + 1);
  a.n_active = arena.take<int32_t>(1);
  a.status = arena.take<int32_t>(1);
  a.items = arena.take<int4>(pairs + E + 1);
  a.n_items = arena.take<int32_t>(1);
  a.h = arena.take<float>(pairs * I);
  a.ysorted = arena.take<float>(pairs * H);
  if (L->tc_ok) {
    __half *x16 = arena.take<__half>(2 * pairs * H);  // hi rows, then lo rows
    __half *h16 = arena.take<__half>(2 * pairs * I);
    float *x_inv = arena.take<float>(pairs);
    float *h_inv = arena.take<float>(pairs);
    float *gu = arena.take<float>(2 * pairs * I);
    // token tiles: 16/32/64 for quantised weights; bf16 (GLM) always 128
    const bool bf16 = d.down_type == DM_BF16;
    const int nts[3] = {bf16 ? 256 : 16, bf16 ? 256 : 32, bf16 ? 256 : 64};
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, L->ctx->device);
    // Activation rows as fp16 hi + lo halves (two MMAs per step) for the memory-bound
    // plans (up to 24 tokens per expert on average), where the second MMA is free; single
    // fp16 rows with a power-of-two row scale for the 64-token plan, where the products are
    // compute-bound (Gemma T = 4096: 2.96 -> 3.41 M tokens/s, layer rel-L2 2e-4 -> 5e-4
    // against the 1e-3 bar). DISKMULE_CUDA_TC_SPLIT=0 makes every plan single, =all split.
    const char *split_env = getenv("DISKMULE_CUDA_TC_SPLIT");
    const bool split_off = split_env && (!strcmp(split_env, "0") || !strcmp(split_env, "false"));
    const bool split_all = split_env && !strcmp(split_env, "all");
    for (int i = 0; i < 3; i++) {
      dm::TcPlan &p = L->tc[i];
      p.nt = nts[i];
      p.n_sm = n_sm;
      p.split = !split_off && (i < 2 || split_all);
      p.rows = (int)pairs;
      p.x16 = x16;
      p.h16 = h16;
      p.x_inv = x_inv;
      p.h_inv = h_inv;
      p.gu = gu;
      if (dm::make_tc_maps(p, (int)H, (int)I, d.down_type, p.nt) != 0) L->tc_ok = false;
    }
  }
  if (arena.overflow) return fail(DM_ERR_ALLOCATION, "layer scratch carve exceeded its allocation");
  L->capacity = tokens;
  return DM_OK;
}

}  // namespace dmi
using dmi::ensure_layer_scratch;

extern "C" {

static int32_t create_layer(dm_cuda_context *ctx, const dm_moe_desc *desc, int32_t first_expert,
                            int32_t local_experts, dm_moe_layer **out, bool cached = false);

int32_t dm_moe_layer_create(dm_cuda_context *ctx, const dm_moe_desc *desc, dm_moe_layer **out) {
  if (!desc) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  return create_layer(ctx, desc, 0, desc->experts, out);
}

int32_t dm_moe_layer_create_ep(dm_cuda_context *ctx, const dm_moe_desc *desc, int32_t first_expert,
                               int32_t local_experts, dm_moe_layer **out) {
  if (!desc) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (first_expert < 0 || local_experts <= 0 || first_expert + local_experts > desc->experts)
    return fail(DM_ERR_INVALID_ARGUMENT, "expert range [%d, %d) is outside 0..%d", first_expert,
                first_expert + local_experts, desc->experts);
  return create_layer(ctx, desc, first_expert, local_experts, out);
}

static int32_t create_layer(dm_cuda_context *ctx, const dm_moe_desc *desc, int32_t first_expert,
                            int32_t local_experts, dm_moe_layer **out, bool cached) {
  if (!ctx || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  int32_t rc = validate_desc(desc);
  if (rc != DM_OK) return rc;
  cudaSetDevice(ctx->device);
  auto *L = new (std::nothrow) dm_moe_layer();
  if (!L) return fail(DM_ERR_ALLOCATION, "host allocation failed");
  L->ctx = ctx;
  retain_context(ctx);
  L->desc = *desc;
  L->first_expert = first_expert;
  L->local_experts = local_experts;
  dm_moe_desc &d = L->desc;
  if (d.n_groups <= 0) d.n_groups = 1;
  if (d.topk_groups <= 0) d.topk_groups = 1;
  L->shared = d.shared_intermediate > 0;
  const bool qwen_gate = d.family == DM_FAMILY_QWEN35_MOE && L->shared;
  L->E1 = d.experts + (qwen_gate ? 1 : 0);
  const uint64_t H = d.hidden, I = d.intermediate;
  const bool fused = d.family == DM_FAMILY_GEMMA4;
  L->gate_stride = (fused ? 2 * I : I) * dm::row_bytes(d.gate_type, H);
  L->up_stride = L->gate_stride;
  L->up_base = fused ? (const uint8_t *)d.gate + I * dm::row_bytes(d.gate_type, H)
                     : (const uint8_t *)d.up;
  L->down_stride = H * dm::row_bytes(d.down_type, I);
  const int wbytes = d.router_type == DM_BF16 ? 2 : 4;
  if (cudaMalloc(&L->router_t, (size_t)H * dm::router_ld(L->E1) * wbytes) != cudaSuccess) {
    L->router_t = nullptr;
    dm_moe_layer_destroy(L);
    return fail(DM_ERR_ALLOCATION, "could not allocate the transposed router");
  }
  dm::launch_transpose_router(d.router, d.router_type == DM_BF16, d.experts, d.hidden,
                              qwen_gate ? d.shared_gate_vector : nullptr, L->router_t,
                              ctx->stream);
  if (cudaMalloc(&L->router_rows, (size_t)L->E1 * H * sizeof(float)) != cudaSuccess) {
    L->router_rows = nullptr;
    dm_moe_layer_destroy(L);
    return fail(DM_ERR_ALLOCATION, "could not allocate the router rows");
  }
  dm::launch_router_rows(d.router, d.router_type == DM_BF16, d.experts, d.hidden,
                         qwen_gate ? d.shared_gate_vector : nullptr, L->router_rows, ctx->stream);
  if (cudaMalloc(&L->router_dup, (size_t)H * dm::router_dup_ld(L->E1) * sizeof(float)) ==
      cudaSuccess)
    dm::launch_dup_router(L->router_t, d.router_type == DM_BF16, (int)H, L->E1, L->router_dup,
                          ctx->stream);
  else
    L->router_dup = nullptr;  // the many-token router then runs the chain-per-thread kernel
  if (d.family == DM_FAMILY_GLM52 && d.router_type == DM_BF16) {
    int32_t *flag = nullptr, bad = 1;
    if (cudaMalloc(&flag, sizeof(int32_t)) == cudaSuccess) {
      if (cudaMemsetAsync(flag, 0, sizeof(int32_t), ctx->stream) == cudaSuccess) {
        dm::launch_bf16_range_check((const uint16_t *)d.router, (size_t)d.experts * H, flag,
                                    ctx->stream);
        if (cudaMemcpyAsync(&bad, flag, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(ctx->stream) != cudaSuccess)
          bad = 1;
      }
      cudaFree(flag);
    }
    L->router_exact_products = bad == 0;
  }
  rc = build_plan(L);
  if (cudaStreamCreateWithFlags(&L->capture, cudaStreamNonBlocking) != cudaSuccess) L->capture = nullptr;
  {
    const char *env = getenv("DISKMULE_CUDA_GRAPHS");
    L->graphs_enabled = L->capture && !(env && (!strcmp(env, "0") || !strcmp(env, "false")));
    const char *tc_env = getenv("DISKMULE_CUDA_TC");
    // the tensor-core kernels copy weight blocks in 16-byte pieces
    const uintptr_t align = (uintptr_t)d.gate | (uintptr_t)L->up_base |
                            (uintptr_t)d.shared_gate | (uintptr_t)d.shared_up;
    // Slots of an expert cache change under the layer: only the bf16 kernels, which
    // read the weights through TMA maps alone, keep no per-expert side arrays.
    const char *f16_env = getenv("DISKMULE_CUDA_F16_DOWN");
    L->tc_f16_down = !cached && !(f16_env && (!strcmp(f16_env, "0") || !strcmp(f16_env, "false")));
    L->tc_ok = rc == DM_OK && align % 16 == 0 && (!cached || d.down_type == DM_BF16) &&
               dm::tc_supported(d.gate_type, d.down_type, d.hidden, d.intermediate) &&
               !(tc_env && (!strcmp(tc_env, "0") || !strcmp(tc_env, "false")));
    if (L->tc_ok) rc = build_tc_weights(L);
  }
  cudaError_t err = cudaStreamSynchronize(ctx->stream);
  if (err == cudaSuccess) err = cudaGetLastError();
  if (rc != DM_OK || err != cudaSuccess) {
    dm_moe_layer_destroy(L);
    return rc != DM_OK ? rc : cuda_fail(err, "layer set-up");
  }
  *out = L;
  return DM_OK;
}

void dm_moe_layer_destroy(dm_moe_layer *L) {
  if (!L) return;
  cudaSetDevice(L->ctx->device);
  cudaStreamSynchronize(L->ctx->stream);
  if (L->router_t) cudaFree(L->router_t);
  if (L->router_dup) cudaFree(L->router_dup);
  if (L->router_rows) cudaFree(L->router_rows);
  if (L->scratch) cudaFree(L->scratch);
  if (L->io) cudaFree(L->io);
  if (L->pipe_in) cudaStreamSynchronize(L->pipe_in);
  if (L->pipe_out) cudaStreamSynchronize(L->pipe_out);
  if (L->pipe) cudaFree(L->pipe);
  for (auto &e : L->pipe_ev)
    if (e) cudaEventDestroy(e);
  if (L->pipe_in) cudaStreamDestroy(L->pipe_in);
  if (L->pipe_out) cudaStreamDestroy(L->pipe_out);
  if (L->pipe_status) cudaFreeHost(L->pipe_status);
  for (auto &e : L->events)
    if (e) cudaEventDestroy(e);
  for (void *p : L->owned) cudaFree(p);
  L->drop_graphs();
  if (L->capture) cudaStreamDestroy(L->capture);
  dmi::release_cached_scratch(L->cached);
  if (L->cache) dmi::cache_release(L->cache);
  cudaGetLastError();  // teardown leaves no error behind for unrelated calls
  dm_cuda_context *ctx = L->ctx;
  delete L;
  release_context(ctx);
}

int32_t dm_moe_layer_create_cached(dm_cuda_context *ctx, const dm_moe_desc *desc,
                                   dm_expert_cache *cache, int32_t layer, dm_moe_layer **out) {
  if (!ctx || !desc || !cache || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (!dmi::cache_on_device(cache, ctx->device))
    return fail(DM_ERR_INVALID_ARGUMENT, "the expert cache does not hold its slots on this device");
  int tensors = 0, slots = 0;
  uint8_t *const *mem = nullptr;
  const uint64_t *bytes = nullptr;
  int32_t rc = dmi::cache_layer_view(cache, layer, &tensors, &slots, &mem, &bytes);
  if (rc != DM_OK) return rc;
  const bool fused = desc->family == DM_FAMILY_GEMMA4;
  if (tensors != (fused ? 2 : 3))
    return fail(DM_ERR_INVALID_ARGUMENT, "cache layer %d has %d tensors; the family needs %d", layer,
                tensors, fused ? 2 : 3);
  const uint64_t H = desc->hidden, I = desc->intermediate;
  const uint64_t gate_bytes = (fused ? 2 * I : I) * dm::row_bytes(desc->gate_type, H);
  const uint64_t down_bytes = H * dm::row_bytes(desc->down_type, I);
  const uint64_t want[3] = {gate_bytes, fused ? down_bytes : gate_bytes, down_bytes};
  for (int i = 0; i < tensors; i++)
    if (bytes[i] != want[i])
      return fail(DM_ERR_BYTE_LENGTH, "cache tensor %d holds %llu bytes per expert; the layer needs %llu",
                  i, (unsigned long long)bytes[i], (unsigned long long)want[i]);
  if (slots > 1023) return fail(DM_ERR_INVALID_ARGUMENT, "at most 1023 slots per layer");
  dm_moe_desc d = *desc;
  d.gate = mem[0];
  d.up = fused ? nullptr : mem[1];
  d.down = mem[fused ? 1 : 2];
  dm_moe_layer *L = nullptr;
  rc = create_layer(ctx, &d, 0, slots, &L, true);
  if (rc != DM_OK) return rc;
  L->cache = cache;
  L->cache_layer = layer;
  dmi::cache_retain(cache);
  *out = L;
  return DM_OK;
}

int32_t dm_moe_set_profiling(dm_moe_layer *L, int32_t enable) {
  if (!L) return fail(DM_ERR_INVALID_ARGUMENT, "null layer");
  cudaSetDevice(L->ctx->device);
  if (enable && !L->events[0]) {
    for (auto &e : L->events) DM_CUDA(cudaEventCreate(&e), "event create");
  }
  L->profiling = enable != 0;
  return DM_OK;
}

int32_t dm_moe_stage_times(dm_moe_layer *L, float *milliseconds, int32_t capacity) {
  if (!L || !milliseconds) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (!L->profiling || !L->events[0]) return fail(DM_ERR_INVALID_ARGUMENT, "profiling is off");
  cudaSetDevice(L->ctx->device);
  DM_CUDA(cudaEventSynchronize(L->events[dm::kStageCount]), "event sync");
  int n = std::min<int>(capacity, dm::kStageCount);
  for (int i = 0; i < n; i++)
    DM_CUDA(cudaEventElapsedTime(&milliseconds[i], L->events[i], L->events[i + 1]), "elapsed");
  return n;
}

const char *dm_moe_stage_name(int32_t stage) {
  static const char *names[dm::kStageCount] = {"prep", "router", "topk", "dispatch",
                                              "expert_up", "expert_down", "combine"};
  return stage >= 0 && stage < dm::kStageCount ? names[stage] : "";
}

}  // extern "C"

namespace dmi {

// Forward arguments for `tokens` rows of `x` (the scratch is already sized).
dm::ForwardArgs fill_args(dm_moe_layer *L, const void *x, float *y, int32_t tokens) {
  const dm_moe_desc &d = L->desc;
  dm::ForwardArgs a = L->args;
  a.balanced_items = 0;  // choose_plans turns it on for the tensor-core kernels
  a.family = d.family;
  a.T = tokens;
  a.H = d.hidden;
  a.I = d.intermediate;
  a.E = d.experts;
  a.k = d.top_k;
  a.E1 = L->E1;
  a.shared = L->shared;
  a.rows_mode = 0;
  a.n_groups = d.n_groups;
  a.topk_groups = d.topk_groups;
  a.normalize = d.normalize_topk;
  a.routed_scale = d.routed_scale;
  a.epsilon = d.epsilon;
  a.inv_sqrt_hidden = 1.0f / std::sqrt((float)d.hidden);
  a.input_bf16 = d.input_type == DM_BF16;
  a.x = x;
  a.y = y;
  a.router_bf16 = d.router_type == DM_BF16;
  a.router_t = L->router_t;
  a.router_dup = L->router_dup;
  a.router_exact_products = L->router_exact_products;
  a.router_rows = L->router_rows;
  a.bias = d.correction_bias;
  a.router_scale = d.router_scale;
  a.routed_pre_norm = d.routed_pre_norm;
  a.expert_scale = d.expert_scale;
  a.logit_bias = d.family == DM_FAMILY_GLM52 ? nullptr : d.router_logit_bias;
  a.gate_type = d.gate_type;
  a.up_type = d.family == DM_FAMILY_GEMMA4 ? d.gate_type : d.up_type;
  a.down_type = d.down_type;
  a.gate = (const uint8_t *)d.gate;
  a.up = L->up_base;
  a.down = (const uint8_t *)d.down;
  a.gate_stride = L->gate_stride;
  a.up_stride = L->up_stride;
  a.down_stride = L->down_stride;
  a.sh_gate = (const uint8_t *)d.shared_gate;
  a.sh_up = (const uint8_t *)d.shared_up;
  a.sh_down = (const uint8_t *)d.shared_down;
  return a;
}

// Expert-kernel plans for the dispatch described by `a` (tokens, k, experts, shared or
// rows mode); sets a.chunk. `gp` / `tp` are null when that path does not apply.
void choose_plans(dm_moe_layer *L, dm::ForwardArgs &a, Plans &P) {
  const dm_moe_desc &d = L->desc;
  const int pairs = a.T * a.k + (a.shared ? a.T : 0);
  const int buckets = a.E + ((a.shared || a.rows_mode) ? 1 : 0);
  P.plan = L->plan;
  P.plan.nt = a.T == 1 ? 1 : (a.T == 2 ? 2 : 4);
  P.plan.max_active = std::min(buckets, pairs + (a.shared ? 1 : 0));
  P.plan.max_items = std::min(pairs, (pairs + P.plan.nt - 1) / P.plan.nt + P.plan.max_active);
  a.chunk = P.plan.nt;
  // the GEMV kernels cover whole tasks: 256 elements (Q4_K/Q6_K), 32 (Q5_0/Q8_0),
  // 128 (BF16) or 64 (F16/F32) per row chunk
  auto task_elems = [](int kind) {
    switch (kind) {
      case DM_Q4_K: case DM_Q6_K: return 256;
      case DM_Q5_0: case DM_Q8_0: return 32;
      case DM_BF16: return 128;
      default: return 64;
    }
  };
  const bool gemv_ok = d.hidden % task_elems(a.gate_type) == 0 &&
                       d.intermediate % task_elems(a.down_type) == 0;
  P.gp = gemv_ok ? &P.plan : nullptr;
  P.tp = nullptr;
  // Enough tokens per expert -> the tcgen05 grouped GEMM.
  if (P.gp && L->tc_ok) {
    const double avg = a.rows_mode ? (double)pairs / buckets : (double)a.T * a.k / a.E;
    if (avg >= (d.down_type == DM_BF16 ? 16.0 : 4.0)) {
      P.tcp = L->tc[avg <= 12.0 ? 0 : (avg <= 24.0 ? 1 : 2)];
      P.tcp.weights = &L->tcw;
      P.tcp.max_items = std::min(pairs, (pairs + P.tcp.nt - 1) / P.tcp.nt + P.plan.max_active);
      a.chunk = P.tcp.nt;
      P.tp = &P.tcp;
      // the tensor-core kernels take an item's first position and token count from the
      // item itself, so an expert's tokens may be split evenly over its items
      static const int balanced = [] {
        const char *e = getenv("DISKMULE_CUDA_BALANCED_ITEMS");
        return e && e[0] == '0' ? 0 : 1;
      }();
      a.balanced_items = balanced;
    }
  }
}

}  // namespace dmi
using dmi::Plans;
using dmi::choose_plans;
using dmi::fill_args;

extern "C" {

int32_t dm_moe_forward(dm_moe_layer *L, const void *x, float *y, int32_t tokens,
                       uint32_t *sel_idx, float *sel_weight, void *stream) {
  if (!L || !x || !y) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  if (L->local_experts != L->desc.experts)
    return fail(DM_ERR_INVALID_ARGUMENT,
                "this layer holds experts %d..%d only: use dm_moe_route / dm_moe_expert_rows",
                L->first_expert, L->first_expert + L->local_experts - 1);
  if ((int64_t)tokens * L->desc.top_k > INT32_MAX / 2 || tokens > (1 << 22))
    return fail(DM_ERR_OVERFLOW, "too many tokens in one call (limit 4194304)");
  if (((uintptr_t)y & 15) || ((uintptr_t)x & 15))
    return fail(DM_ERR_INVALID_ARGUMENT, "x and y must be 16-byte aligned device pointers");
  cudaSetDevice(L->ctx->device);
  int32_t rc = ensure_layer_scratch(L, tokens);
  if (rc != DM_OK) return rc;
  dm::ForwardArgs a = fill_args(L, x, y, tokens);
  if (sel_idx) a.sel_idx = sel_idx;
  if (sel_weight) a.sel_w = sel_weight;
  cudaStream_t s = (cudaStream_t)stream;
  Plans plans;
  choose_plans(L, a, plans);
  const dm::GemvPlan *gp = plans.gp;
  const dm::TcPlan *tp = plans.tp;

  // A call that repeats with the same buffers (a decode loop) is captured once as a
  // CUDA graph on an internal stream and replayed on the caller's stream.
  dm_moe_layer::GraphEntry *g = nullptr;
  if (!L->profiling && L->graphs_enabled) {
    for (auto &e : L->graphs)
      if (e.x == x && e.y == y && e.tokens == tokens && e.sel_idx == sel_idx &&
          e.sel_weight == sel_weight)
        g = &e;
    if (!g && L->graphs.size() < 16) {
      L->graphs.push_back({x, y, tokens, sel_idx, sel_weight, 0, nullptr, 0});
      g = &L->graphs.back();
    }
  }
  int launches = 0;
  if (g && !g->exec && g->seen >= 1 && !g->failed) {
    cudaGraph_t graph = nullptr;
    cudaError_t err = cudaStreamBeginCapture(L->capture, cudaStreamCaptureModeThreadLocal);
    if (err == cudaSuccess) {
      cudaMemsetAsync(a.status, 0, 4, L->capture);
      launches = dm::launch_forward(a, L->capture, nullptr, gp, tp);
      err = cudaStreamEndCapture(L->capture, &graph);
    }
    if (err == cudaSuccess && launches > 0) err = cudaGraphInstantiate(&g->exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (err != cudaSuccess || launches <= 0) {
      cudaGetLastError();
      g->failed = 1;
      g->exec = nullptr;
    } else {
      g->launches = launches;
    }
  }
  if (g && g->exec) {
    DM_CUDA(cudaGraphLaunch(g->exec, s), "MoE graph launch");
    launches = g->launches;
  } else {
    if (g) g->seen++;
    DM_CUDA(cudaMemsetAsync(a.status, 0, 4, s), "status reset");
    launches = dm::launch_forward(a, s, L->profiling ? L->events : nullptr, gp, tp);
    if (launches < 0) return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "no expert kernel for this format");
    DM_CUDA(cudaGetLastError(), "MoE forward launch");
  }
  L->last_tokens = tokens;
  L->last_noalloc = 0;
  L->last_launches = launches;
  return DM_OK;
}

int32_t dm_moe_forward_host(dm_moe_layer *L, const void *x, float *y, int32_t tokens,
                            uint32_t *sel_idx, float *sel_weight) {
  if (!L || !x || !y) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  cudaSetDevice(L->ctx->device);
  const dm_moe_desc &d = L->desc;
  size_t xb = (size_t)tokens * d.hidden * (d.input_type == DM_BF16 ? 2 : 4);
  size_t yb = (size_t)tokens * d.hidden * 4;
  size_t need = ((xb + 255) & ~size_t(255)) + yb;
  if (need > L->io_bytes) {
    if (L->io) cudaFree(L->io);
    L->io = nullptr;
    L->io_bytes = 0;
    if (cudaMalloc(&L->io, need) != cudaSuccess)
      return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of staging", need);
    L->io_bytes = need;
  }
  void *xd = L->io;
  float *yd = (float *)((uint8_t *)L->io + ((xb + 255) & ~size_t(255)));
  cudaStream_t s = L->ctx->stream;
  DM_CUDA(cudaMemcpyAsync(xd, x, xb, cudaMemcpyHostToDevice, s), "input copy");
  int32_t rc = dm_moe_forward(L, xd, yd, tokens, nullptr, nullptr, s);
  if (rc != DM_OK) return rc;
  int32_t status = 0;
  DM_CUDA(cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, s), "output copy");
  if (sel_idx)
    DM_CUDA(cudaMemcpyAsync(sel_idx, L->args.sel_idx, (size_t)tokens * d.top_k * 4,
                            cudaMemcpyDeviceToHost, s), "selection copy");
  if (sel_weight)
    DM_CUDA(cudaMemcpyAsync(sel_weight, L->args.sel_w, (size_t)tokens * d.top_k * 4,
                            cudaMemcpyDeviceToHost, s), "weight copy");
  DM_CUDA(cudaMemcpyAsync(&status, L->args.status, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaStreamSynchronize(s), "MoE forward");
  if (status == dm::kStatusNonFiniteRouter)
    return fail(DM_ERR_NON_FINITE, "router produced a non-finite score");
  if (status == dm::kStatusTimeout)
    return fail(DM_ERR_TIMEOUT, "a bounded wait in the tensor-core GEMM ran out");
  if (status == dm::kStatusNonFiniteNorm)
    return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");
  return DM_OK;
}

int32_t dm_moe_forward_host_batches(dm_moe_layer *L, int32_t batches, const void *const *x,
                                    float *const *y, int32_t tokens) {
  if (!L || !x || !y) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (batches < 0 || tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative count");
  if (batches == 0 || tokens == 0) return DM_OK;
  for (int b = 0; b < batches; b++)
    if (!x[b] || !y[b]) return fail(DM_ERR_INVALID_ARGUMENT, "null batch pointer %d", b);
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  const dm_moe_desc &d = L->desc;
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t xb = (size_t)tokens * d.hidden * (d.input_type == DM_BF16 ? 2 : 4);
  const size_t yb = (size_t)tokens * d.hidden * 4;
  const size_t slot = al(xb) + al(yb);
  if (2 * slot > L->pipe_bytes) {
    if (L->pipe) cudaFree(L->pipe);
    L->pipe = nullptr;
    L->pipe_bytes = 0;
    if (cudaMalloc(&L->pipe, 2 * slot) != cudaSuccess)
      return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of staging", 2 * slot);
    L->pipe_bytes = 2 * slot;
  }
  if (!L->pipe_in) {
    DM_CUDA(cudaStreamCreateWithFlags(&L->pipe_in, cudaStreamNonBlocking), "copy-in stream");
    DM_CUDA(cudaStreamCreateWithFlags(&L->pipe_out, cudaStreamNonBlocking), "copy-out stream");
    for (auto &e : L->pipe_ev)
      DM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "pipeline event");
  }
  if (batches > L->pipe_status_n) {
    if (L->pipe_status) cudaFreeHost(L->pipe_status);
    L->pipe_status = nullptr;
    L->pipe_status_n = 0;
    DM_CUDA(cudaHostAlloc((void **)&L->pipe_status, (size_t)batches * 4, cudaHostAllocDefault),
            "status words");
    L->pipe_status_n = batches;
  }
  cudaStream_t cs = L->ctx->stream;
  cudaEvent_t *ev_in = L->pipe_ev, *ev_fwd = L->pipe_ev + 2, *ev_out = L->pipe_ev + 4;
  for (int b = 0; b < batches; b++) {
    const int s = b & 1;
    uint8_t *xd = (uint8_t *)L->pipe + s * slot;
    float *yd = (float *)(xd + al(xb));
    // slot s was last used by batch b-2: its forward must have read the input before
    // the copy-in overwrites it, and its copy-out must be done before the forward
    // overwrites the output
    if (b >= 2) DM_CUDA(cudaStreamWaitEvent(L->pipe_in, ev_fwd[s], 0), "wait");
    DM_CUDA(cudaMemcpyAsync(xd, x[b], xb, cudaMemcpyHostToDevice, L->pipe_in), "input copy");
    DM_CUDA(cudaEventRecord(ev_in[s], L->pipe_in), "record");
    DM_CUDA(cudaStreamWaitEvent(cs, ev_in[s], 0), "wait");
    if (b >= 2) DM_CUDA(cudaStreamWaitEvent(cs, ev_out[s], 0), "wait");
    int32_t rc = dm_moe_forward(L, xd, yd, tokens, nullptr, nullptr, cs);
    if (rc != DM_OK) {
      cudaStreamSynchronize(cs);
      cudaStreamSynchronize(L->pipe_in);
      cudaStreamSynchronize(L->pipe_out);
      return rc;
    }
    DM_CUDA(cudaMemcpyAsync(&L->pipe_status[b], L->args.status, 4, cudaMemcpyDeviceToHost, cs),
            "status copy");
    DM_CUDA(cudaEventRecord(ev_fwd[s], cs), "record");
    DM_CUDA(cudaStreamWaitEvent(L->pipe_out, ev_fwd[s], 0), "wait");
    DM_CUDA(cudaMemcpyAsync(y[b], yd, yb, cudaMemcpyDeviceToHost, L->pipe_out), "output copy");
    DM_CUDA(cudaEventRecord(ev_out[s], L->pipe_out), "record");
  }
  DM_CUDA(cudaStreamSynchronize(L->pipe_out), "output copies");
  DM_CUDA(cudaStreamSynchronize(cs), "MoE forward");
  for (int b = 0; b < batches; b++) {
    const int32_t status = L->pipe_status[b];
    if (status == dm::kStatusNonFiniteRouter)
      return fail(DM_ERR_NON_FINITE, "batch %d: router produced a non-finite score", b);
    if (status == dm::kStatusTimeout)
      return fail(DM_ERR_TIMEOUT, "batch %d: a bounded wait in the tensor-core GEMM ran out", b);
    if (status == dm::kStatusNonFiniteNorm)
      return fail(DM_ERR_NON_FINITE, "batch %d: RMSNorm received a non-finite value", b);
  }
  return DM_OK;
}

// ---------------------------------------------------------------------------
// expert parallelism: route, experts on received rows, combine of returned rows
// ---------------------------------------------------------------------------

namespace {

int32_t finish_launch(dm_moe_layer *L, int launches, int tokens) {
  if (launches < 0) return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "no expert kernel for this format");
  DM_CUDA(cudaGetLastError(), "MoE launch");
  L->last_tokens = tokens;
  L->last_noalloc = 0;
  L->last_launches = launches;
  return DM_OK;
}

}  // namespace

int32_t dm_moe_route(dm_moe_layer *L, const void *x, int32_t tokens, uint32_t *sel_idx,
                     float *sel_weight, float *expert_in, float *logits, void *stream) {
  if (!L || !x || !sel_idx || !sel_weight) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  if (tokens > (1 << 22)) return fail(DM_ERR_OVERFLOW, "too many tokens in one call (limit 4194304)");
  if ((uintptr_t)x & 15) return fail(DM_ERR_INVALID_ARGUMENT, "x must be 16-byte aligned");
  cudaSetDevice(L->ctx->device);
  int32_t rc = ensure_layer_scratch(L, tokens);
  if (rc != DM_OK) return rc;
  dm::ForwardArgs a = fill_args(L, x, nullptr, tokens);
  a.sel_idx = sel_idx;
  a.sel_w = sel_weight;
  cudaStream_t s = (cudaStream_t)stream;
  DM_CUDA(cudaMemsetAsync(a.status, 0, 4, s), "status reset");
  const int launches = dm::launch_forward(a, s, nullptr, nullptr, nullptr, dm::kRunRoute);
  const dm_moe_desc &d = L->desc;
  if (expert_in && d.family == DM_FAMILY_GEMMA4)
    DM_CUDA(cudaMemcpyAsync(expert_in, a.expert_in, (size_t)tokens * d.hidden * 4,
                            cudaMemcpyDeviceToDevice, s), "expert input copy");
  if (logits)
    DM_CUDA(cudaMemcpyAsync(logits, a.logits, (size_t)tokens * L->E1 * 4, cudaMemcpyDeviceToDevice,
                            s), "logit copy");
  return finish_launch(L, launches, tokens);
}

int32_t dm_moe_expert_rows(dm_moe_layer *L, const void *rows, const int32_t *expert_ids,
                           int32_t count, float *out, void *stream) {
  if (!L || !rows || !expert_ids || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (count < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative row count");
  if (count == 0) return DM_OK;
  if (count > (1 << 22)) return fail(DM_ERR_OVERFLOW, "too many rows in one call (limit 4194304)");
  if (((uintptr_t)rows & 15) || ((uintptr_t)out & 15))
    return fail(DM_ERR_INVALID_ARGUMENT, "rows and out must be 16-byte aligned device pointers");
  cudaSetDevice(L->ctx->device);
  int32_t rc = ensure_layer_scratch(L, count);
  if (rc != DM_OK) return rc;
  dm::ForwardArgs a = fill_args(L, rows, out, count);
  a.k = 1;
  a.E = L->local_experts;  // ids are local; id E is the shared expert
  a.shared = 0;
  a.rows_mode = 1;
  a.sel_idx = (uint32_t *)expert_ids;
  if (L->desc.family == DM_FAMILY_GEMMA4) a.expert_in = (float *)rows;  // pre-normalised rows
  cudaStream_t s = (cudaStream_t)stream;
  Plans plans;
  choose_plans(L, a, plans);
  DM_CUDA(cudaMemsetAsync(a.status, 0, 4, s), "status reset");
  const int launches = dm::launch_forward(a, s, nullptr, plans.gp, plans.tp,
                                          dm::kRunExperts | dm::kRunScatter);
  return finish_launch(L, launches, count);
}

int32_t dm_moe_combine_rows(dm_moe_layer *L, int32_t tokens, const uint32_t *sel_idx,
                            const float *sel_weight, const float *logits, const float *pair_out,
                            float *y, void *stream) {
  if (!L || !sel_idx || !sel_weight || !pair_out || !y)
    return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  if (L->desc.family == DM_FAMILY_QWEN35_MOE && L->shared && !logits)
    return fail(DM_ERR_INVALID_ARGUMENT, "the Qwen shared-expert gate needs the router logits");
  if (((uintptr_t)pair_out & 15) || ((uintptr_t)y & 15))
    return fail(DM_ERR_INVALID_ARGUMENT, "pair_out and y must be 16-byte aligned device pointers");
  cudaSetDevice(L->ctx->device);
  int32_t rc = ensure_layer_scratch(L, tokens);
  if (rc != DM_OK) return rc;
  dm::ForwardArgs a = fill_args(L, nullptr, y, tokens);
  a.sel_idx = (uint32_t *)sel_idx;
  a.sel_w = (float *)sel_weight;
  if (logits) a.logits = (float *)logits;
  a.ysorted = (float *)pair_out;
  cudaStream_t s = (cudaStream_t)stream;
  const int launches = dm::launch_forward(a, s, nullptr, nullptr, nullptr,
                                          dm::kRunIdentity | dm::kRunCombine);
  return finish_launch(L, launches, tokens);
}

int32_t dm_moe_local_experts(const dm_moe_layer *L, int32_t *first_expert, int32_t *count) {
  if (!L || !first_expert || !count) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *first_expert = L->first_expert;
  *count = L->local_experts;
  return DM_OK;
}

int32_t dm_moe_last_dispatch(dm_moe_layer *L, int32_t *counts, int32_t *offsets,
                             int32_t *sorted_pairs, int32_t *inverse) {
  if (!L) return fail(DM_ERR_INVALID_ARGUMENT, "null layer");
  if (L->last_noalloc)
    return fail(DM_ERR_INVALID_ARGUMENT,
                "the last call was dm_moe_forward_noalloc, whose dispatch lists are not kept");
  if (L->last_tokens == 0) return DM_OK;
  cudaSetDevice(L->ctx->device);
  const int E = L->desc.experts;
  const size_t P = (size_t)L->last_tokens * L->desc.top_k;
  DM_CUDA(cudaDeviceSynchronize(), "dispatch sync");
  if (counts) DM_CUDA(cudaMemcpy(counts, L->args.counts, E * 4, cudaMemcpyDeviceToHost), "copy");
  if (offsets) DM_CUDA(cudaMemcpy(offsets, L->args.offsets, (E + 1) * 4, cudaMemcpyDeviceToHost), "copy");
  if (sorted_pairs) DM_CUDA(cudaMemcpy(sorted_pairs, L->args.sorted, P * 4, cudaMemcpyDeviceToHost), "copy");
  if (inverse) DM_CUDA(cudaMemcpy(inverse, L->args.inverse, P * 4, cudaMemcpyDeviceToHost), "copy");
  return DM_OK;
}

int32_t dm_moe_last_launch_count(const dm_moe_layer *L) { return L ? L->last_launches : 0; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward without allocation.
//
// Some callers cannot call cudaMalloc when they run a layer: a host runtime that
// has already carved all of HBM into its own pools (expert slot pools sized to
// fill the device), or code on a latency-critical stream where cudaMalloc's
// implicit device-wide synchronisation would stall other streams. For them,
// dm_moe_forward_noalloc runs the same kernels as dm_moe_forward, but every piece
// of per-call scratch (router logits, selection, dispatch lists, expert
// intermediates) is carved from one fixed device array compiled into this
// library, so the call allocates nothing.
// ---------------------------------------------------------------------------

// 8 MiB per device, held by every GPU that loads the library until the process
// exits. In host code this name is only a stand-in for the symbol; kernels get
// the array's device address, fetched by cudaGetSymbolAddress below.
static constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_lock;
void *g_noalloc_address[64] = {};  // per device ordinal, filled on first use

// Device address of the array on `device` (which must be current). The first
// call on a device looks it up; later calls reuse it.
int32_t noalloc_scratch(int device, uint8_t **out) {
  if (device < 0 || device >= 64) return fail(DM_ERR_INVALID_ARGUMENT, "device ordinal out of range");
  std::lock_guard<std::mutex> guard(g_noalloc_lock);
  if (!g_noalloc_address[device]) {
    void *ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress of the static scratch");
    g_noalloc_address[device] = ptr;
  }
  *out = (uint8_t *)g_noalloc_address[device];
  return DM_OK;
}

}  // namespace

extern "C" int32_t dm_moe_forward_noalloc(dm_moe_layer *L, const void *x, float *y,
                                          int32_t tokens, uint32_t *sel_idx, float *sel_weight,
                                          void *stream) {
  if (!L || !x || !y) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  // The same refusals as dm_moe_forward: a layer holding only some experts (an
  // expert-parallel shard, or a cache layer's slots) would index weights it lacks.
  if (L->local_experts != L->desc.experts)
    return fail(DM_ERR_INVALID_ARGUMENT,
                "this layer holds experts %d..%d only: use dm_moe_route / dm_moe_expert_rows",
                L->first_expert, L->first_expert + L->local_experts - 1);
  if ((int64_t)tokens * L->desc.top_k > INT32_MAX / 2 || tokens > (1 << 22))
    return fail(DM_ERR_OVERFLOW, "too many tokens in one call (limit 4194304)");
  if (((uintptr_t)y & 15) || ((uintptr_t)x & 15))
    return fail(DM_ERR_INVALID_ARGUMENT, "x and y must be 16-byte aligned device pointers");
  const dm_moe_desc &d = L->desc;
  // the same scratch layout as the allocating forward, carved from the static array
  // after the status word, which sits at a fixed offset (0) so that
  // dm_moe_forward_noalloc_status can find it
  const size_t T = (size_t)tokens, H = d.hidden, I = d.intermediate, E = d.experts,
               k = d.top_k;
  const size_t pairs = T * k + (L->shared ? T : 0);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  size_t need = al(4);
  if (d.family == DM_FAMILY_GEMMA4) need += 2 * al(T * H * 4);
  need += al(T * L->E1 * 4) + 2 * al(T * k * 4);
  need += al((E + 1) * 4) + al((E + 2) * 4) + 2 * al(pairs * 4) + al((E + 1) * 4) + al(4);
  need += al((pairs + E + 1) * sizeof(int4)) + al(4);
  need += al(pairs * I * 4) + al(pairs * H * 4);
  if (need > kNoAllocScratchBytes)
    return fail(DM_ERR_OVERFLOW,
                "%d tokens need %zu bytes of scratch; the no-allocation forward has %zu "
                "(use dm_moe_forward or fewer tokens per call)",
                tokens, need, kNoAllocScratchBytes);
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  uint8_t *base = nullptr;
  int32_t rc = noalloc_scratch(L->ctx->device, &base);
  if (rc != DM_OK) return rc;
  dm::Arena arena{base, 0, kNoAllocScratchBytes};
  dm::ForwardArgs a{};
  a.status = arena.take<int32_t>(1);
  a.router_in = d.family == DM_FAMILY_GEMMA4 ? arena.take<float>(T * H) : nullptr;
  a.expert_in = d.family == DM_FAMILY_GEMMA4 ? arena.take<float>(T * H) : nullptr;
  a.logits = arena.take<float>(T * L->E1);
  a.sel_idx = arena.take<uint32_t>(T * k);
  a.sel_w = arena.take<float>(T * k);
  a.counts = arena.take<int32_t>(E + 1);
  a.offsets = arena.take<int32_t>(E + 2);
  a.sorted = arena.take<int32_t>(pairs);
  a.inverse = arena.take<int32_t>(pairs);
  a.active = arena.take<int32_t>(E + 1);
  a.n_active = arena.take<int32_t>(1);
  a.items = arena.take<int4>(pairs + E + 1);
  a.n_items = arena.take<int32_t>(1);
  a.h = arena.take<float>(pairs * I);
  a.ysorted = arena.take<float>(pairs * H);
  if (arena.overflow) return fail(DM_ERR_ALLOCATION, "scratch carve exceeded the static array");
  a.family = d.family;
  a.T = tokens;
  a.H = d.hidden;
  a.I = d.intermediate;
  a.E = d.experts;
  a.k = d.top_k;
  a.E1 = L->E1;
  a.shared = L->shared;
  a.n_groups = d.n_groups;
  a.topk_groups = d.topk_groups;
  a.normalize = d.normalize_topk;
  a.routed_scale = d.routed_scale;
  a.epsilon = d.epsilon;
  a.inv_sqrt_hidden = 1.0f / std::sqrt((float)d.hidden);
  a.input_bf16 = d.input_type == DM_BF16;
  a.x = x;
  a.y = y;
  a.router_bf16 = d.router_type == DM_BF16;
  a.router_t = L->router_t;
  a.router_rows = L->router_rows;
  a.bias = d.correction_bias;
  a.router_scale = d.router_scale;
  a.routed_pre_norm = d.routed_pre_norm;
  a.expert_scale = d.expert_scale;
  a.logit_bias = d.family == DM_FAMILY_GLM52 ? nullptr : d.router_logit_bias;
  a.gate_type = d.gate_type;
  a.up_type = d.family == DM_FAMILY_GEMMA4 ? d.gate_type : d.up_type;
  a.down_type = d.down_type;
  a.gate = (const uint8_t *)d.gate;
  a.up = L->up_base;
  a.down = (const uint8_t *)d.down;
  a.gate_stride = L->gate_stride;
  a.up_stride = L->up_stride;
  a.down_stride = L->down_stride;
  a.sh_gate = (const uint8_t *)d.shared_gate;
  a.sh_up = (const uint8_t *)d.shared_up;
  a.sh_down = (const uint8_t *)d.shared_down;
  if (sel_idx) a.sel_idx = sel_idx;
  if (sel_weight) a.sel_w = sel_weight;
  dm::GemvPlan plan = L->plan;
  plan.nt = tokens == 1 ? 1 : (tokens == 2 ? 2 : 4);
  plan.max_active = std::min(a.E + (a.shared ? 1 : 0), a.T * a.k + (a.shared ? 1 : 0));
  plan.max_items = std::min((int)pairs, ((int)pairs + plan.nt - 1) / plan.nt + plan.max_active);
  a.chunk = plan.nt;
  auto task_elems = [](int kind) {
    switch (kind) {
      case DM_Q4_K: case DM_Q6_K: return 256;
      case DM_Q5_0: case DM_Q8_0: return 32;
      case DM_BF16: return 128;
      default: return 64;
    }
  };
  const bool gemv_ok = d.hidden % task_elems(a.gate_type) == 0 &&
                       d.intermediate % task_elems(a.down_type) == 0;
  cudaStream_t s = (cudaStream_t)stream;
  // Every buffer above is written before it is read within a call, except the
  // status word, which must start at zero: the array keeps the last call's bytes.
  DM_CUDA(cudaMemsetAsync(a.status, 0, 4, s), "status reset");
  const int launches = dm::launch_forward(a, s, nullptr, gemv_ok ? &plan : nullptr);
  if (launches < 0) return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "no expert kernel for this format");
  DM_CUDA(cudaGetLastError(), "MoE forward (no allocation) launch");
  // The dispatch lists of this call live in the shared array, not in the layer's
  // scratch: dm_moe_last_dispatch refuses until the next allocating call.
  L->last_tokens = tokens;
  L->last_launches = launches;
  L->last_noalloc = 1;
  return DM_OK;
}

extern "C" int32_t dm_moe_forward_noalloc_status(dm_moe_layer *L, void *stream) {
  if (!L) return fail(DM_ERR_INVALID_ARGUMENT, "null layer");
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  uint8_t *base = nullptr;
  int32_t rc = noalloc_scratch(L->ctx->device, &base);
  if (rc != DM_OK) return rc;
  int32_t status = 0;  // a host stack word: the copy allocates nothing
  cudaStream_t s = (cudaStream_t)stream;
  DM_CUDA(cudaMemcpyAsync(&status, base, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaStreamSynchronize(s), "MoE forward (no allocation)");
  if (status == dm::kStatusNonFiniteRouter)
    return fail(DM_ERR_NON_FINITE, "router produced a non-finite score");
  if (status == dm::kStatusTimeout)
    return fail(DM_ERR_TIMEOUT, "a bounded wait in an expert kernel ran out");
  if (status == dm::kStatusNonFiniteNorm)
    return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");
  return status == 0 ? DM_OK : fail(DM_ERR_COMMAND, "unexpected status %d", status);
}

extern "C" int32_t dm_selftest_device_wait(dm_cuda_context *ctx, int64_t cycles) {
  if (!ctx) return fail(DM_ERR_INVALID_ARGUMENT, "null context");
  if (cycles <= 0 || cycles > 4000000000ll)
    return fail(DM_ERR_INVALID_ARGUMENT, "the wait limit must be 1..4e9 cycles");
  cudaSetDevice(ctx->device);
  int32_t *st = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(ctx->status) + 128);
  DM_CUDA(cudaMemsetAsync(st, 0, 4, ctx->stream), "status reset");
  dm::launch_selftest_wait((long long)cycles, st, ctx->stream);
  DM_CUDA(cudaGetLastError(), "self-test launch");
  int32_t status = 0;
  DM_CUDA(cudaMemcpyAsync(&status, st, 4, cudaMemcpyDeviceToHost, ctx->stream), "status copy");
  DM_CUDA(cudaStreamSynchronize(ctx->stream), "self-test");
  if (status == dm::kStatusTimeout)
    return fail(DM_ERR_TIMEOUT, "a bounded device wait gave up after %lld cycles", (long long)cycles);
  return status == 0 ? DM_OK : fail(DM_ERR_COMMAND, "unexpected self-test status %d", status);
}
