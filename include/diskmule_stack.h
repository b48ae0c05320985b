/*
 * diskmule_stack.h -- the per-step glue of a GLM-shaped decode stack, on the device.
 *
 * Not part of the MoE boundary (include/diskmule_cuda.h): these restate the steps of
 * forward_token_inner that surround the routed block (src/glm52/cpu.rs:462-518) --
 * the embedding row, RMSNorm, the residual add, the output head and greedy argmax --
 * so that a stack of out-of-core MoE layers can decode token by token on the GPU
 * without host round trips. Each is bit-exact with its reference:
 *   embedding  bf16 -> f32 by `<< 16` (src/glm52/cpu.rs:1267-1271);
 *   RMSNorm    mean square as a sequential f64 sum, scale = 1 / sqrt(ms as f32 + eps)
 *              in f32, out = value * scale * weight (src/glm52/cpu.rs:912-924);
 *   residual   hidden[i] += delta[i] in f32 (add_in_place);
 *   head       per row a sequential, unfused f32 sum of weight * value in column
 *              order from -0.0 (TensorReader::matvec_into, src/glm52/cpu.rs:1177-1185);
 *   argmax     largest by total order, ties to the lowest index; a non-finite logit is
 *              an error (cpu::argmax, src/cpu.rs:276-292).
 * All calls are stream-ordered and allocate nothing. `status` (device int32, may be
 * NULL) receives DM_STACK_NON_FINITE_* bits instead of an error return.
 */
#ifndef DISKMULE_STACK_H
#define DISKMULE_STACK_H

#include <stdint.h>

#include "diskmule_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
  DM_STACK_NON_FINITE_NORM = 1,    /* an RMSNorm input or scale was not finite */
  DM_STACK_NON_FINITE_LOGIT = 2,   /* the output head produced a non-finite logit */
  DM_STACK_BAD_TOKEN = 4,          /* the embedding token was outside the vocabulary */
};

/* h [hidden] f32 = row `*token` (device int32) of table [vocab, hidden] (DM_BF16 or
 * DM_F32). */
DM_API int32_t dm_stack_embed(dm_cuda_context *ctx, const void *table, int32_t table_type,
                              int32_t vocab, int32_t hidden, const int32_t *token, float *h,
                              int32_t *status, void *stream);
/* h += delta (when delta is not NULL), then out = rms_norm(h, weight, epsilon). */
DM_API int32_t dm_stack_add_rms_norm(dm_cuda_context *ctx, float *h, const float *delta,
                                     const float *weight, int32_t hidden, float epsilon,
                                     float *out, int32_t *status, void *stream);
/* logits [vocab] = weight [vocab, hidden] (DM_BF16) . x; *token = argmax (device
 * int32). logits may be NULL. */
DM_API int32_t dm_stack_lm_head_argmax(dm_cuda_context *ctx, const void *weight,
                                       int32_t weight_type, int32_t vocab, int32_t hidden,
                                       const float *x, float *logits, int32_t *token,
                                       int32_t *status, void *stream);

#ifdef __cplusplus
}
#endif
#endif
