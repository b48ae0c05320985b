/*
 * diskmule_gguf.h -- GGUF tensor index and expert slices for the CUDA backend.
 *
 * Replaces the reader the reference's GPU path maps expert tensors through:
 *   - GgufFile::read_from_with_arrays (src/gguf.rs:460-607): the bounded index parse,
 *     with the same limits and the same checks in the same order (magic, version 2 or 3,
 *     entry and length limits, metadata types, general.alignment, tensor dimensions,
 *     GGML types and block shapes, byte-length overflow, data-section alignment,
 *     tensor alignment, file bounds, overlaps);
 *   - TensorSource (src/gguf.rs:610-723): the read-only whole-file mapping, tensor
 *     lookup by name and index, borrowed tensor bytes, bounded positional reads;
 *   - ExpertLayerLayout + bytes_per_expert (src/expert.rs:44-51,
 *     src/gemma4/metal.rs:175-199, :1101-1117): the per-expert byte ranges of a layer's
 *     fused expert tensors.
 * These calls are host-only: they work without a GPU. Errors return a dm_status and
 * set dm_last_error_message() to the reference's GgufError text. Format errors are
 * DM_ERR_FORMAT, I/O errors DM_ERR_IO, integer overflow DM_ERR_OVERFLOW and unknown
 * GGML types DM_ERR_UNSUPPORTED_TENSOR_TYPE.
 */
#ifndef DISKMULE_GGUF_H
#define DISKMULE_GGUF_H

#include <stddef.h>
#include <stdint.h>

#ifndef DM_API
#if defined(__GNUC__)
#define DM_API __attribute__((visibility("default")))
#else
#define DM_API
#endif
#endif

#include "diskmule_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct dm_gguf dm_gguf;

/* One tensor of the index (TensorInfo, src/gguf.rs:387-395). `name` stays valid until
 * dm_gguf_close. dims[0] is the GGUF first (contiguous) dimension. */
typedef struct {
  const char *name;
  uint32_t n_dims;
  uint64_t dims[4];
  int32_t type;             /* GGML type id (dm_tensor_type values and the other ids) */
  uint64_t offset;          /* relative to the data section */
  uint64_t absolute_offset; /* from the start of the file */
  uint64_t byte_len;
} dm_gguf_tensor_info;

/* Per-expert byte ranges of one layer's fused expert tensors (ExpertLayerLayout). */
typedef struct {
  int32_t expert_count;
  uint64_t gate_up_offset; /* absolute file offset of expert 0 */
  uint64_t gate_up_bytes;  /* bytes per expert */
  uint64_t down_offset;
  uint64_t down_bytes;
} dm_expert_layer_layout;

/* Open and index a GGUF file and map it read-only (TensorSource::open_with_arrays).
 * `capture_arrays`: NULL, or newline-separated metadata keys whose array values are
 * kept (all other arrays keep only their element type and length). */
DM_API int32_t dm_gguf_open(const char *path, const char *capture_arrays, dm_gguf **out);
/* Index an in-memory GGUF image (copied), as GgufFile::read_from does over a reader. */
DM_API int32_t dm_gguf_parse(const void *bytes, uint64_t length, const char *capture_arrays,
                             dm_gguf **out);
DM_API void dm_gguf_close(dm_gguf *gguf);

DM_API int32_t dm_gguf_header(const dm_gguf *gguf, uint32_t *version, uint32_t *alignment,
                              uint64_t *data_offset, uint64_t *file_len);
DM_API int64_t dm_gguf_tensor_count(const dm_gguf *gguf);
/* TensorSource::tensor: the index of `name`, or DM_ERR_FORMAT (TensorNotFound). */
DM_API int32_t dm_gguf_find_tensor(const dm_gguf *gguf, const char *name, int64_t *index);
DM_API int32_t dm_gguf_tensor(const dm_gguf *gguf, int64_t index, dm_gguf_tensor_info *out);
/* TensorSource::tensor_bytes_by_index: the tensor's bytes in the read-only mapping. */
DM_API int32_t dm_gguf_tensor_bytes(const dm_gguf *gguf, int64_t index, const void **data,
                                    uint64_t *length);
/* TensorSource::read_tensor_at: bounded positional read of `length` bytes at `offset`
 * within the tensor (safe from several threads at once). */
DM_API int32_t dm_gguf_read_tensor_at(const dm_gguf *gguf, const char *name, uint64_t offset,
                                      void *destination, uint64_t length);

/* Metadata (MetadataValue, src/gguf.rs:144-269). `type` is the GGUF value type id
 * (0 u8 .. 12 f64, 8 string, 9 array); arrays report their element type and length. */
DM_API int32_t dm_gguf_metadata_type(const dm_gguf *gguf, const char *key, uint32_t *type,
                                     uint32_t *element_type, uint64_t *length);
/* A scalar of an integer type as u64 / i64 (unsigned types fail on negatives). */
DM_API int32_t dm_gguf_metadata_u64(const dm_gguf *gguf, const char *key, uint64_t *value);
DM_API int32_t dm_gguf_metadata_f64(const dm_gguf *gguf, const char *key, double *value);
/* A string value, NUL-terminated (DM_ERR_OUTPUT_LENGTH when it does not fit). */
DM_API int32_t dm_gguf_metadata_string(const dm_gguf *gguf, const char *key, char *buffer,
                                       uint64_t capacity);
/* A captured array: numeric element types as a packed little-endian array of
 * `length` elements; string arrays as `length` NUL-terminated const char pointers. */
DM_API int32_t dm_gguf_metadata_array(const dm_gguf *gguf, const char *key,
                                      uint32_t *element_type, uint64_t *length,
                                      const void **values);

/* The per-expert layout of a layer's expert tensors `gate_up` and `down` (each holding
 * `expert_count` equal slices), as ExpertCache builds it (src/gemma4/metal.rs:175-199):
 * DM_ERR_FORMAT when a byte length does not split evenly over the experts. */
DM_API int32_t dm_gguf_expert_layout(const dm_gguf *gguf, const char *gate_up,
                                     const char *down, int32_t expert_count,
                                     dm_expert_layer_layout *out);

#ifdef __cplusplus
}
#endif
#endif
