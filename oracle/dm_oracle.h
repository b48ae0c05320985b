/*
 * dm_oracle.h -- CPU restatement of DiskMule's routed-expert (MoE) path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (diskmule_b200/, include/)
 * links, loads or calls this library.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm may use it, and only as the checker or
 * as the timed CPU implementation of the reference path.
 *
 * Every function restates the arithmetic of the Rust reference (DiskMule) in
 * plain C with the same operation order:
 *   - Rust `a.mul_add(b, c)`  ->  fmaf(a, b, c)
 *   - every other f32 expression is evaluated left to right with one rounding
 *     per operation (the oracle is compiled with -ffp-contract=off)
 *   - Rust `f32::exp` / `f32::tanh` call the platform libm (glibc here).
 *
 * Parity is pinned by the reference's own known-answer tests (tests/golden),
 * except where a function is marked "restated, parity unpinned".
 */
#ifndef DM_ORACLE_H
#define DM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type ids (src/gguf.rs:295-318, TensorType::from_ggml). */
enum {
  DMO_F32 = 0,
  DMO_F16 = 1,
  DMO_Q5_0 = 6,
  DMO_Q8_0 = 8,
  DMO_Q4_K = 12,
  DMO_Q5_K = 13,
  DMO_Q6_K = 14,
  DMO_BF16 = 30,
};

/* Error codes mirror src/cpu.rs:10-97 (CpuError) variants that the path can raise. */
enum {
  DMO_OK = 0,
  DMO_ERR_UNSUPPORTED = -1,     /* CpuError::UnsupportedType */
  DMO_ERR_ELEMENT_COUNT = -2,   /* CpuError::InvalidElementCount */
  DMO_ERR_BYTE_LENGTH = -3,     /* CpuError::InvalidByteLength */
  DMO_ERR_INPUT_LENGTH = -4,    /* CpuError::InvalidInputLength */
  DMO_ERR_OUTPUT_LENGTH = -5,   /* CpuError::InvalidOutputLength */
  DMO_ERR_EMPTY = -6,           /* CpuError::EmptyInput */
  DMO_ERR_NONFINITE = -7,       /* CpuError::NonFinite / InvalidRouterScore */
  DMO_ERR_TOPK = -8,            /* CpuError::InvalidTopK */
  DMO_ERR_PARAM = -9,           /* CpuError::InvalidPositiveParameter */
  DMO_ERR_OVERFLOW = -10,       /* CpuError::Overflow */
  DMO_ERR_EXPERT = -11,         /* ExpertCacheError::InvalidExpert */
  DMO_ERR_LAYER = -12,          /* ExpertCacheError::InvalidLayer */
  DMO_ERR_ALL_PINNED = -13,     /* ExpertCacheError::AllSlotsPinned */
  DMO_ERR_NO_SLOTS = -14,       /* ExpertCacheError::NoSlots */
  DMO_ERR_CANCELLED = -15,      /* ExpertCacheError::Cancelled */
};

/* ---- scalar decode helpers (src/cpu.rs:546-660, src/glm52/cpu.rs:1266-1271) ---- */
float dmo_f16_to_f32(uint16_t bits);
float dmo_bf16_to_f32(uint16_t bits);
int dmo_block_layout(int kind, uint64_t *block_elements, uint64_t *block_bytes);
int dmo_row_byte_len(int kind, uint64_t elements, uint64_t *out);
void dmo_scale_min_q4_k(int index, const uint8_t *scales, uint8_t *scale, uint8_t *min);
int dmo_dequantize(int kind, const uint8_t *encoded, size_t encoded_len, float *out,
                   size_t n);

/* ---- operators (src/cpu.rs) ---- */
int dmo_matvec(int kind, size_t rows, size_t columns, const uint8_t *encoded,
               size_t encoded_len, const float *input, size_t input_len, float *output,
               size_t output_len, int threads);
int dmo_rms_norm(const float *input, const float *weight, size_t n, float epsilon,
                 float *output);
float dmo_gelu_tanh(float value);
int dmo_softmax_in_place(float *values, size_t n);
int dmo_top_k_softmax(const float *logits, size_t n, size_t k, uint32_t *indices,
                      float *probabilities);
int dmo_argmax(const float *values, size_t n, size_t *index);

/* ---- GLM-5.2 helpers (src/glm52/cpu.rs, src/glm52/expert.rs) ---- */
int dmo_glm_rms_norm(const float *input, const float *weight, size_t n, float epsilon,
                     float *output);
int dmo_f8_e4m3fn(uint8_t v, float *out);
int dmo_glm_u8_encoding(size_t rows, size_t columns, size_t encoded_bytes, size_t scales,
                        int *kind, int *group_size);
int dmo_glm_quant_matvec(int fp8, size_t rows, size_t columns, const uint8_t *encoded,
                         size_t encoded_bytes, const float *scales, size_t n_scales,
                         const float *input, float *output, int threads);
int dmo_glm_quant_row(int fp8, size_t rows, size_t columns, const uint8_t *encoded,
                      size_t encoded_bytes, const float *scales, size_t n_scales, size_t r,
                      float *out);
int dmo_glm_matvec(int kind, size_t rows, size_t columns, const uint8_t *encoded,
                   const float *input, float *output, int threads);
float dmo_glm_sigmoid(float value);
float dmo_glm_silu(float value);
float dmo_glm_cached_silu(float value);
int dmo_glm_select(const float *logits, const float *correction, size_t experts,
                   size_t k, size_t n_groups, size_t topk_groups, int normalize,
                   uint32_t *indices, float *weights);

/* ---- Qwen3.5 helpers (src/qwen35/cpu.rs:982-993) ---- */
float dmo_qwen_sigmoid(float value);
float dmo_qwen_silu(float value);

/* ---- token -> expert dispatch (new work; deterministic counting sort) ---- */
int dmo_dispatch(const uint32_t *selected, size_t tokens, size_t k, size_t experts,
                 int32_t *counts, int32_t *offsets, int32_t *sorted_pairs,
                 int32_t *inverse);

/* ---- MoE blocks ---- */
typedef struct {
  int32_t hidden, intermediate, experts, top_k;
  float epsilon;
  const float *router;          /* [experts, hidden] f32 (GGUF dims [hidden, experts]) */
  const float *router_scale;    /* [hidden] */
  const float *routed_pre_norm; /* [hidden] */
  int32_t gate_up_type;         /* fused gate/up, [experts][2*intermediate rows][hidden] */
  const uint8_t *gate_up;
  int32_t down_type;            /* [experts][hidden rows][intermediate] */
  const uint8_t *down;
  const float *expert_scale;    /* [experts] (ffn_down_exps.scale) */
  const float *router_logit_bias; /* optional [experts], added once after the router chain */
} dmo_gemma_layer;

int dmo_gemma_moe(const dmo_gemma_layer *layer, const float *x, size_t tokens,
                  float *routed, uint32_t *sel_idx, float *sel_prob, int threads);
/* The router and top-k alone (no expert weights read): selection of `tokens` tokens. */
int dmo_gemma_route(const dmo_gemma_layer *layer, const float *x, size_t tokens,
                    uint32_t *sel_idx, float *sel_prob, int threads);

/* The rest of Gemma 4's feed-forward block around the routed branch
 * (src/gemma4/cpu.rs:547-558, :613-620): the dense shared FFN on
 * rms_norm(x, feed_forward_norm) (feed_forward, :693-712: gelu_tanh(gate) * up, then
 * down), its post norm, the routed post norm, their sum, the post feed-forward norm,
 * the residual add and the layer output scale. */
typedef struct {
  int32_t width;                    /* feed_forward_length */
  int32_t gate_type, up_type, down_type;
  const uint8_t *gate, *up;         /* [width][hidden] GGUF rows */
  const uint8_t *down;              /* [hidden][width] */
  const float *feed_forward_norm, *shared_post_norm, *routed_post_norm,
      *post_feed_forward_norm;      /* [hidden] */
  float layer_output_scale;
} dmo_gemma_ffn;

int dmo_gemma_ffn_block(const dmo_gemma_ffn *ffn, const dmo_gemma_layer *layer, const float *x,
                        size_t tokens, float *hidden, uint32_t *sel_idx, float *sel_prob,
                        int threads);

typedef struct {
  int32_t hidden, intermediate, experts, top_k;
  const float *router;      /* [experts, hidden] f32 */
  int32_t gate_type, up_type, down_type;
  const uint8_t *gate;      /* [experts][intermediate][hidden] */
  const uint8_t *up;        /* [experts][intermediate][hidden] */
  const uint8_t *down;      /* [experts][hidden][intermediate] */
  int32_t shared_intermediate;
  const uint8_t *shared_gate, *shared_up, *shared_down; /* same types, one expert */
  const float *shared_gate_vector; /* [hidden] f32: sigmoid(x . v) scales the shared output */
  const float *router_logit_bias;  /* optional [experts], added once after the router chain */
} dmo_qwen_layer;

int dmo_qwen_moe(const dmo_qwen_layer *layer, const float *x, size_t tokens, float *y,
                 uint32_t *sel_idx, float *sel_prob, int threads);
int dmo_qwen_route(const dmo_qwen_layer *layer, const float *x, size_t tokens,
                   uint32_t *sel_idx, float *sel_prob, int threads);

typedef struct {
  int32_t hidden, intermediate, experts, top_k;
  int32_t n_groups, topk_groups, normalize;
  float routed_scale;
  int32_t weight_type;           /* DMO_BF16 or DMO_F32 for router / experts / shared */
  const uint8_t *router;         /* [experts, hidden] */
  const float *correction_bias;  /* [experts] */
  const uint8_t *gate, *up;      /* [experts][intermediate][hidden] */
  const uint8_t *down;           /* [experts][hidden][intermediate] */
  int32_t shared_intermediate;   /* 0 = no shared expert */
  const uint8_t *shared_gate, *shared_up, *shared_down;
  /* optional: expert e's weights as one blob gate | up | down (then gate/up/down
   * above are not read) -- the layout of an out-of-core expert pool */
  const uint8_t *const *expert_blobs;
} dmo_glm_layer;

int dmo_glm_moe(const dmo_glm_layer *layer, const float *x, size_t tokens, float *y,
                uint32_t *sel_idx, float *sel_weight, int threads);
int dmo_glm_route(const dmo_glm_layer *layer, const float *x, size_t tokens,
                  uint32_t *sel_idx, float *sel_weight, int threads);

/* ---- expert residency (src/expert.rs, src/glm52/expert.rs) ---- */
typedef struct {
  uint64_t hits, misses, evictions, reads, bytes_read, resident_bytes;
} dmo_cache_stats;

typedef struct dmo_lru dmo_lru;
/* global_clock=0: per-layer clock with pinning (src/expert.rs:166-229);
 * global_clock=1: one clock across layers, no pinning (src/glm52/expert.rs:183-256). */
dmo_lru *dmo_lru_create(int32_t layers, int32_t experts, int32_t slots, int32_t global_clock,
                        uint64_t expert_bytes, int32_t reads_per_miss);
void dmo_lru_destroy(dmo_lru *lru);
int dmo_lru_acquire(dmo_lru *lru, int32_t layer, int32_t expert, int32_t *slot,
                    int32_t *was_miss);
void dmo_lru_set_pinned(dmo_lru *lru, int32_t layer, int32_t slot, int32_t pinned);
void dmo_lru_stats(const dmo_lru *lru, dmo_cache_stats *stats);

#ifdef __cplusplus
}
#endif
#endif
