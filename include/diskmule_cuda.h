/*
 * diskmule_cuda.h -- C ABI of the B200 (sm_100a) backend for DiskMule's
 * routed-expert (MoE) path.
 *
 * The Rust host binds these symbols from a `src/cuda.rs` that sits beside
 * `src/metal.rs`; every entry point names the reference interface it replaces.
 * Conventions follow the Metal backend (src/metal.rs):
 *   - row-major [rows, columns] matrices, where GGUF dims are [columns, rows]
 *     (src/gemma4/metal.rs:866-875);
 *   - validation happens before any launch, with the error order of
 *     `prepare_matvec` (src/metal.rs:1513-1560);
 *   - `*_host` / operator calls take borrowed host slices and return after the
 *     GPU finished (src/metal.rs:1562-1604);
 *   - every call returns an int32_t status: 0 = ok, negative = dm_status.
 * A context is used from one thread at a time (src/runtime.rs:741-760).
 */
#ifndef DISKMULE_CUDA_H
#define DISKMULE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifndef DM_API
#if defined(__GNUC__)
#define DM_API __attribute__((visibility("default")))
#else
#define DM_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: MetalError (src/metal.rs:3-126), CpuError (src/cpu.rs:10-97)
 *      and ExpertCacheError (src/expert.rs:13-42) variants reachable on this path ---- */
typedef enum {
  DM_OK = 0,
  DM_ERR_NO_DEVICE = -1,              /* MetalError::NoDevice */
  DM_ERR_ALLOCATION = -2,             /* MetalError::BufferAllocation */
  DM_ERR_INVALID_ARGUMENT = -3,       /* null handle / pointer, bad descriptor */
  DM_ERR_UNSUPPORTED_TENSOR_TYPE = -4,/* MetalError::UnsupportedTensorType */
  DM_ERR_ELEMENT_COUNT = -5,          /* MetalError::InvalidElementCount */
  DM_ERR_BYTE_LENGTH = -6,            /* MetalError::InvalidByteLength */
  DM_ERR_INPUT_LENGTH = -7,           /* MetalError::InvalidInputLength */
  DM_ERR_OUTPUT_LENGTH = -8,          /* MetalError::InvalidOutputLength */
  DM_ERR_EMPTY_INPUT = -9,            /* MetalError::EmptyInput */
  DM_ERR_NON_FINITE = -10,            /* MetalError::NonFinite, Glm52CpuError::InvalidRouterScore */
  DM_ERR_TOP_K = -11,                 /* MetalError::InvalidTopK */
  DM_ERR_MAPPED_RANGE = -12,          /* MetalError::MappedRange */
  DM_ERR_OVERFLOW = -13,              /* MetalError::Overflow */
  DM_ERR_COMMAND = -14,               /* MetalError::Command (a CUDA launch/runtime error) */
  DM_ERR_INVALID_EXPERT = -15,        /* ExpertCacheError::InvalidExpert */
  DM_ERR_INVALID_LAYER = -16,         /* ExpertCacheError::InvalidLayer */
  DM_ERR_ALL_SLOTS_PINNED = -17,      /* ExpertCacheError::AllSlotsPinned */
  DM_ERR_CANCELLED = -18,             /* ExpertCacheError::Cancelled */
  DM_ERR_NO_SLOTS = -19,              /* ExpertCacheError::NoSlots */
  DM_ERR_VECTOR_LENGTH = -20,         /* MetalError::InvalidVectorLength */
  DM_ERR_POSITIVE_PARAMETER = -21,    /* MetalError::InvalidPositiveParameter */
  DM_ERR_TIMEOUT = -22,               /* a bounded device or host wait ran out */
  DM_ERR_NOT_BUILT = -23,             /* the call needs a component this build lacks */
  DM_ERR_COMMUNICATOR = -24,          /* NCCL / expert-parallel exchange failed */
  DM_ERR_IO = -25,                    /* ExpertCacheError::Io: a source read failed or was short */
  DM_ERR_FORMAT = -26,                /* GgufError: a malformed model-file index, a missing tensor */
} dm_status;

/* GGML tensor type ids (src/gguf.rs:295-318) on the path. */
typedef enum {
  DM_F32 = 0,
  DM_F16 = 1,
  DM_Q5_0 = 6,
  DM_Q8_0 = 8,
  DM_Q4_K = 12,
  DM_Q6_K = 14,
  DM_BF16 = 30,
  /* safetensors storage of the GLM-5.2 checkpoints (src/glm52/quant.rs, SafeDtype) */
  DM_U8_QUANT = 200, /* U8: int8 rows or grouped int4, with a flat F32 `.qs` scale tensor */
  DM_F8_E4M3 = 201,  /* F8_E4M3 with an F32 `_scale_inv` tensor of 128 x 128 blocks */
} dm_tensor_type;

typedef struct dm_cuda_context dm_cuda_context;
typedef struct dm_buffer dm_buffer;
typedef struct dm_moe_layer dm_moe_layer;

/* Human-readable name of a status code, and the detail message of the last
 * failing call on this thread (the Display text of the Rust error). */
DM_API const char *dm_status_string(int32_t status);
DM_API const char *dm_last_error_message(void);

/* ---- context: MetalContext::new (src/metal.rs:291-346), device_name (:348-352) ---- */
DM_API int32_t dm_cuda_create(int32_t device_ordinal, dm_cuda_context **out);
DM_API void dm_cuda_destroy(dm_cuda_context *ctx);
DM_API int32_t dm_cuda_device_name(const dm_cuda_context *ctx, char *name, size_t capacity);
/* Wait for all work on the context's device (the completion wait every Metal call
 * ends with, src/metal.rs:1562-1604, offered separately for stream-ordered use). */
DM_API int32_t dm_cuda_synchronize(dm_cuda_context *ctx);

/* ---- buffers ----
 * dm_cuda_map_read_only replaces MetalContext::map_read_only (src/metal.rs:354-392):
 * the bytes of a read-only host mapping (e.g. a GGUF/safetensors file) become an
 * immutable HBM buffer. dm_cuda_new_owned_buffer replaces new_owned_buffer
 * (:394-402), with dm_buffer_write / dm_buffer_read as the as_mut_bytes / as_bytes
 * accessors of MetalOwnedBuffer (:213-243). */
DM_API int32_t dm_cuda_map_read_only(dm_cuda_context *ctx, const void *host, size_t length,
                              dm_buffer **out);
DM_API int32_t dm_cuda_new_owned_buffer(dm_cuda_context *ctx, size_t length, dm_buffer **out);
DM_API int32_t dm_buffer_write(dm_buffer *buffer, size_t offset, const void *source, size_t length);
DM_API int32_t dm_buffer_read(const dm_buffer *buffer, size_t offset, void *destination,
                       size_t length);
DM_API size_t dm_buffer_length(const dm_buffer *buffer);
DM_API void *dm_buffer_device_pointer(const dm_buffer *buffer);
DM_API void dm_buffer_free(dm_buffer *buffer);

/* ---- operators (synchronous, host slices) ----
 * dm_cuda_matvec: MetalContext::matvec (src/metal.rs:648-683).
 * dm_cuda_matvec_mapped: matvec_mapped (:687-734) and matvec_owned (:1148-1194).
 * The encoded matrix is row-major GGUF blocks of `kind`; F32/F16/BF16/Q5_0/Q8_0/
 * Q4_K/Q6_K are supported. The result is an f32 dot product per row (within the
 * reference tolerance of src/metal.rs:2041-2050, not a bit-exact fma chain). */
DM_API int32_t dm_cuda_matvec(dm_cuda_context *ctx, int32_t kind, size_t rows, size_t columns,
                       const uint8_t *encoded, size_t encoded_length, const float *input,
                       size_t input_length, float *output, size_t output_length);
DM_API int32_t dm_cuda_matvec_mapped(dm_cuda_context *ctx, int32_t kind, size_t rows,
                              size_t columns, const dm_buffer *mapped, size_t offset,
                              size_t encoded_length, const float *input, size_t input_length,
                              float *output, size_t output_length);
/* MetalContext::matvec_safetensor (src/metal.rs:883-992, matvec_u8 :1070-1147):
 * F32 / F16 / BF16 as dm_cuda_matvec; DM_U8_QUANT resolved to int8 rows or grouped int4
 * from the byte and scale counts as u8_matrix_encoding does (src/metal.rs:1893-1942);
 * DM_F8_E4M3 with [ceil(rows/128)][ceil(columns/128)] scales. Values decode as the CPU
 * reference's rows (src/glm52/cpu.rs:1278-1410); the dot products are f32 (tolerance). */
DM_API int32_t dm_cuda_matvec_safetensor(dm_cuda_context *ctx, int32_t dtype, size_t rows,
                                         size_t columns, const uint8_t *encoded,
                                         size_t encoded_length, const float *scales,
                                         size_t scale_count, const float *input,
                                         size_t input_length, float *output,
                                         size_t output_length);
/* MetalContext::top_k_softmax (src/metal.rs:1392-1434); indices are bit-exact with
 * cpu::top_k_softmax (src/cpu.rs:234-260). */
DM_API int32_t dm_cuda_top_k_softmax(dm_cuda_context *ctx, const float *logits, size_t length,
                              size_t k, uint32_t *indices, float *probabilities);
/* MetalContext::gelu_mul (:530-552), silu_mul (:554-576), rms_norm (:435-476). */
DM_API int32_t dm_cuda_gelu_mul(dm_cuda_context *ctx, const float *gate, const float *up,
                         float *output, size_t length);
DM_API int32_t dm_cuda_silu_mul(dm_cuda_context *ctx, const float *gate, const float *up,
                         float *output, size_t length);
DM_API int32_t dm_cuda_rms_norm(dm_cuda_context *ctx, const float *input, const float *weight,
                         size_t length, float epsilon, float *output);

/* ---- the batched MoE layer (new: the reference applies one expert at a time) ----
 * A family fixes the routing, activation, shared expert and combine rules:
 *   DM_FAMILY_GEMMA4: src/gemma4/cpu.rs:559-611 -- router input rms_norm(x) *
 *     (router_scale / sqrt(H)), expert input rms_norm(x, routed_pre_norm), f32
 *     fma-chain router, softmax top-k, fused Q4_K gate_up [E][2I][H], GeGLU-tanh,
 *     down [E][H][I], combine routed = fma(out, p * expert_scale[e], routed).
 *     y is `routed` at src/gemma4/cpu.rs:612.
 *   DM_FAMILY_QWEN35_MOE: Qwen3.5-shaped block, restated (the reference's Qwen3.5
 *     is dense): f32 router, softmax top-k, SiLU-GLU experts (src/qwen35/cpu.rs:
 *     415-428, 982-993), y = fma(shared(x), sigmoid(x . shared_gate_vector),
 *     sum_j fma(expert_j(x), p_j, .)).
 *   DM_FAMILY_GLM52: src/glm52/cpu.rs:711-778 -- bf16 router with a sequential
 *     non-fused sum, sigmoid + correction bias, optional group limit (restated),
 *     norm_topk, routed SiLU g/(1+e^-g), y += out*w*routed_scale, + shared MLP.
 * Weight pointers are DEVICE addresses of the reference's own byte layouts (GGUF
 * blocks or safetensors rows, experts contiguous): e.g. dm_buffer_device_pointer of
 * a dm_cuda_map_read_only buffer plus the tensor's offset. They must stay valid
 * until dm_moe_layer_destroy. */
typedef enum {
  DM_FAMILY_GEMMA4 = 1,
  DM_FAMILY_QWEN35_MOE = 2,
  DM_FAMILY_GLM52 = 3,
} dm_moe_family;

typedef struct {
  int32_t family;
  int32_t hidden, intermediate, experts, top_k;
  int32_t n_groups, topk_groups, normalize_topk; /* GLM; 1/1 = reference routing */
  float routed_scale;                             /* GLM routed_scaling_factor */
  float epsilon;                                  /* Gemma rms_norm epsilon */
  int32_t input_type;                             /* DM_F32, or DM_BF16 for GLM */
  int32_t router_type;                            /* DM_F32 (Gemma/Qwen), DM_BF16 or DM_F32 (GLM) */
  const void *router;                             /* [experts, hidden] */
  const float *correction_bias;                   /* GLM [experts] */
  const float *router_scale;                      /* Gemma [hidden] */
  const float *routed_pre_norm;                   /* Gemma [hidden] */
  const float *expert_scale;                      /* Gemma [experts] */
  int32_t gate_type, up_type, down_type;
  const void *gate; /* [experts][intermediate][hidden]; Gemma: fused [experts][2I][hidden] */
  const void *up;   /* [experts][intermediate][hidden]; NULL for Gemma */
  const void *down; /* [experts][hidden][intermediate] */
  int32_t shared_intermediate;                    /* 0 = no shared expert */
  const void *shared_gate, *shared_up, *shared_down;
  const float *shared_gate_vector;                /* Qwen [hidden] */
  /* Optional per-expert logit offset for the softmax families, added once after the
   * router chain (benchmark knob for skewed routing; NULL = the reference router). */
  const float *router_logit_bias;                 /* [experts] or NULL */
} dm_moe_desc;

DM_API int32_t dm_moe_layer_create(dm_cuda_context *ctx, const dm_moe_desc *desc,
                            dm_moe_layer **out);
DM_API void dm_moe_layer_destroy(dm_moe_layer *layer);

/* Stream-ordered forward on device pointers: x [tokens, hidden] (input_type),
 * y [tokens, hidden] f32, optional sel_idx / sel_weight [tokens, top_k] (selection
 * order, bit-exact indices). `stream` is a cudaStream_t (NULL = the legacy stream).
 * No host synchronisation happens inside. Replaces the per-layer routed block of
 * src/gemma4/metal.rs:694-777, src/gemma4/cpu.rs:559-611, src/glm52/cpu.rs:711-778. */
DM_API int32_t dm_moe_forward(dm_moe_layer *layer, const void *x, float *y, int32_t tokens,
                       uint32_t *sel_idx, float *sel_weight, void *stream);
/* The same on host slices, synchronous (the Metal call convention). */
DM_API int32_t dm_moe_forward_host(dm_moe_layer *layer, const void *x, float *y, int32_t tokens,
                            uint32_t *sel_idx, float *sel_weight);
/* `batches` independent forwards of `tokens` rows each on host slices x[b] -> y[b],
 * pipelined: the input copy of batch b+1 and the output copy of batch b-1 run on their
 * own streams while batch b computes (two device staging slots). Synchronous: returns
 * when every output is on the host, with the first failing batch's status. Page-locked
 * host slices make the copies overlap. The reference runs one token at a time through
 * `forward_token_inner` (src/gemma4/cpu.rs:358-378, src/glm52/cpu.rs:462-524); this is
 * the streaming form of that loop for a host that holds whole batches. */
DM_API int32_t dm_moe_forward_host_batches(dm_moe_layer *layer, int32_t batches,
                                           const void *const *x, float *const *y,
                                           int32_t tokens);
/* Token -> expert dispatch of the last forward, copied to the host: counts[experts],
 * offsets[experts + 1], sorted_pairs[tokens * top_k] (pair p = t*top_k + j, ordered by
 * expert, then p) and inverse[tokens * top_k]. Synchronous. */
DM_API int32_t dm_moe_last_dispatch(dm_moe_layer *layer, int32_t *counts, int32_t *offsets,
                             int32_t *sorted_pairs, int32_t *inverse);
/* Per-stage device timers of a forward: the CUDA analog of the phase timers in
 * GenerationProfile (src/generation.rs:119-141). With profiling on, events are
 * recorded on the forward's stream at every stage boundary; dm_moe_stage_times
 * waits for the last forward and writes up to `capacity` stage durations (ms),
 * returning the number written. Stage names: prep, router, topk, dispatch,
 * expert_up, expert_down, combine. */
DM_API int32_t dm_moe_set_profiling(dm_moe_layer *layer, int32_t enable);
DM_API int32_t dm_moe_stage_times(dm_moe_layer *layer, float *milliseconds, int32_t capacity);
DM_API const char *dm_moe_stage_name(int32_t stage);
/* Kernel launches issued by the last forward (a count for benchmarks). */
DM_API int32_t dm_moe_last_launch_count(const dm_moe_layer *layer);

/* dm_moe_forward without any allocation. No counterpart in the reference.
 * For callers that cannot call cudaMalloc while running a layer: a runtime that
 * has carved all device memory into its own pools (expert slot pools sized to fill
 * HBM), or a latency-critical stream where cudaMalloc's implicit device-wide
 * synchronisation is not acceptable. The call runs the same kernels as
 * dm_moe_forward with the same arguments, but all per-call scratch comes from one
 * fixed 8 MiB array compiled into the library (held by every GPU that loads it
 * until the process exits); a token count whose scratch exceeds 8 MiB is rejected
 * with DM_ERR_OVERFLOW. The first call on a device looks up the array's device
 * address, so make that first call before any stream capture. All calls share the
 * array: calls whose GPU work overlaps in time (other streams, other threads) race
 * on it and must be serialised by the caller. Layers holding only some experts
 * (expert-parallel shards, cache layers) are refused with DM_ERR_INVALID_ARGUMENT,
 * as by dm_moe_forward. The call returns once its kernels are queued; it does not
 * wait for them, so device-side failures (a non-finite router score, a bounded wait
 * that ran out) are read with dm_moe_forward_noalloc_status. dm_moe_last_dispatch
 * refuses after a no-allocation call: its dispatch lists are not kept. */
DM_API int32_t dm_moe_forward_noalloc(dm_moe_layer *layer, const void *x, float *y,
                                      int32_t tokens, uint32_t *sel_idx, float *sel_weight,
                                      void *stream);
/* Outcome of the last dm_moe_forward_noalloc on the layer's device: waits for
 * `stream`, then returns DM_OK, DM_ERR_NON_FINITE (a non-finite router score or
 * RMSNorm input) or DM_ERR_TIMEOUT (a bounded device wait ran out), as
 * dm_moe_forward_host reports them. Allocates nothing. No counterpart in the
 * reference. */
DM_API int32_t dm_moe_forward_noalloc_status(dm_moe_layer *layer, void *stream);

/* ---- expert parallelism --------------------------------------------------------
 * The reference runs every expert of a layer in one process (src/glm52/cpu.rs:711-778,
 * src/glm52/expert.rs:183-267); these calls split that block so expert weights can be
 * sharded over GPUs, with the token rows exchanged by the caller (NCCL all-to-all):
 *   dm_moe_route        router + top-k on local tokens (global expert ids)
 *   dm_moe_expert_rows  gate/up/down of received rows on this GPU's experts
 *   dm_moe_combine_rows weighted combine of the returned rows + shared expert
 * Composed, they give the same result as dm_moe_forward on one GPU. */

/* A layer holding the weights of experts [first_expert, first_expert + local_experts)
 * only: desc->gate/up/down point at those experts (local_experts x the per-expert
 * stride); the router, correction bias and shared expert are whole (desc->experts
 * columns). dm_moe_forward refuses such a layer unless it holds every expert. */
DM_API int32_t dm_moe_layer_create_ep(dm_cuda_context *ctx, const dm_moe_desc *desc,
                                      int32_t first_expert, int32_t local_experts,
                                      dm_moe_layer **out);
/* Experts held by the layer. */
DM_API int32_t dm_moe_local_experts(const dm_moe_layer *layer, int32_t *first_expert,
                                    int32_t *count);
/* Router logits and top-k of x [tokens, hidden] (device): sel_idx / sel_weight
 * [tokens, top_k] as in dm_moe_forward. Optional copies: the Gemma expert inputs
 * (expert_in [tokens, hidden] f32, the rows to send) and the router logits
 * (logits [tokens, experts (+1 Qwen shared gate)] f32). */
DM_API int32_t dm_moe_route(dm_moe_layer *layer, const void *x, int32_t tokens,
                            uint32_t *sel_idx, float *sel_weight, float *expert_in,
                            float *logits, void *stream);
/* Expert products of `count` rows (device, [count, hidden], input_type; Gemma: the
 * expert inputs from dm_moe_route) on this layer's experts: expert_ids[r] is the
 * local expert of row r (0..local_experts-1) or local_experts for the shared
 * expert. out [count, hidden] f32 receives each row's unweighted expert output. */
DM_API int32_t dm_moe_expert_rows(dm_moe_layer *layer, const void *rows,
                                  const int32_t *expert_ids, int32_t count, float *out,
                                  void *stream);
/* y [tokens, hidden] f32 = the weighted combine of pair_out, which holds the expert
 * output of pair p = t*top_k + j in row p and the shared expert's output of token t in
 * row tokens*top_k + t (when the layer has one); sel_idx / sel_weight / logits are
 * dm_moe_route's (logits needed for the Qwen shared gate only). */
DM_API int32_t dm_moe_combine_rows(dm_moe_layer *layer, int32_t tokens, const uint32_t *sel_idx,
                                   const float *sel_weight, const float *logits,
                                   const float *pair_out, float *y, void *stream);

/* ---- Gemma 4's whole feed-forward block ---------------------------------------------
 * The routed layer above plus what surrounds it in the reference (src/gemma4/cpu.rs:
 * 547-558, :613-620): the dense shared FFN on rms_norm(x, feed_forward_norm)
 * (feed_forward, :693-712: gelu_tanh(gate) * up, then down), its post norm, the routed
 * branch's post norm, their sum and post feed-forward norm, the residual add and the
 * layer output scale. x and hidden are [tokens, hidden] f32 device rows; sel_idx /
 * sel_weight as in dm_moe_forward. Weight pointers are device memory in GGUF row
 * layout ([width][hidden] gate and up, [hidden][width] down); norm vectors [hidden] f32.
 * The block keeps pointers, not copies (the gate and up rows are copied once into one
 * fused buffer). dm_gemma_ffn_status waits for `stream` and reports a non-finite norm. */
typedef struct {
  int32_t width;                 /* feed_forward_length */
  int32_t gate_type, up_type, down_type;
  const void *gate, *up, *down;
  const float *feed_forward_norm, *shared_post_norm, *routed_post_norm, *post_feed_forward_norm;
  float layer_output_scale;
} dm_gemma_ffn_desc;
typedef struct dm_gemma_ffn dm_gemma_ffn;
DM_API int32_t dm_gemma_ffn_create(dm_moe_layer *routed, const dm_gemma_ffn_desc *desc,
                                   dm_gemma_ffn **out);
DM_API int32_t dm_gemma_ffn_forward(dm_gemma_ffn *block, const float *x, float *hidden,
                                    int32_t tokens, uint32_t *sel_idx, float *sel_weight,
                                    void *stream);
DM_API int32_t dm_gemma_ffn_status(dm_gemma_ffn *block, void *stream);
DM_API void dm_gemma_ffn_destroy(dm_gemma_ffn *block);

/* ---- expert parallelism over NVLink peer memory -----------------------------------
 * The same split as above with the token exchange done by this library's own kernels:
 * each rank stores token rows straight into the other ranks' memory (CUDA IPC mappings
 * over NVLink / NVSwitch) and raises per-rank epoch flags, so a forward has no host
 * synchronisation and no collective-library call. The reference runs every expert in
 * one process (src/glm52/cpu.rs:711-778, src/glm52/expert.rs:183-267); composed over
 * the ranks, a forward gives dm_moe_forward's result for each rank's tokens (the
 * combine is the same selection-order kernel on the same pair outputs).
 *
 * dm_ep_create takes a layer made by dm_moe_layer_create_ep for experts
 * [rank*E/world, (rank+1)*E/world) and sizes an exchange region for up to
 * `max_tokens` tokens per rank per forward. Every rank then connects to every other:
 * dm_ep_ipc_handle writes this rank's 64-byte handle, and dm_ep_connect_ipc takes all
 * ranks' handles [world][64] (exchanged by the caller, e.g. an all-gather); ranks
 * that live in one process use dm_ep_connect_local with every rank's dm_ep. All ranks
 * must be connected before any rank starts a forward, and stay alive until every rank
 * has finished its last one.
 *
 * A forward is dm_ep_forward on every rank (or its three phases in order: dispatch,
 * experts, combine). Every rank runs the same number of forwards; a rank with no
 * tokens passes tokens = 0. Waits on other ranks are bounded (about two seconds):
 * dm_ep_status returns DM_ERR_TIMEOUT after a forward in which a rank's rows or
 * outputs did not arrive. Ranks on one GPU are run phase by phase in one stream
 * (every rank's dispatch, then every rank's experts, then every rank's combine), so no
 * kernel ever waits on a kernel launched after it. */
typedef struct dm_ep dm_ep;
DM_API int32_t dm_ep_create(dm_moe_layer *layer, int32_t rank, int32_t world,
                            int32_t max_tokens, dm_ep **out);
DM_API int32_t dm_ep_ipc_handle(dm_ep *ep, void *handle);
DM_API int32_t dm_ep_connect_ipc(dm_ep *ep, const void *handles);
DM_API int32_t dm_ep_connect_local(dm_ep *ep, dm_ep *const *peers);
/* Router + top-k of x [tokens, hidden] (input_type, device) and the send of rows. */
DM_API int32_t dm_ep_dispatch(dm_ep *ep, const void *x, int32_t tokens, void *stream);
/* Wait for every rank's rows, run this rank's experts on them, return the outputs. */
DM_API int32_t dm_ep_experts(dm_ep *ep, void *stream);
/* Wait for every rank's outputs and combine them into y [tokens, hidden] f32;
 * optional copies of the selection [tokens, top_k]. */
DM_API int32_t dm_ep_combine(dm_ep *ep, float *y, uint32_t *sel_idx, float *sel_weight,
                             void *stream);
DM_API int32_t dm_ep_forward(dm_ep *ep, const void *x, float *y, int32_t tokens,
                             uint32_t *sel_idx, float *sel_weight, void *stream);
/* Waits for `stream`; DM_OK, DM_ERR_TIMEOUT (a rank did not arrive) or the layer's own
 * device status (non-finite router score, tensor-core wait) of the last forward. */
DM_API int32_t dm_ep_status(dm_ep *ep, void *stream);
/* Kernel launches of the last forward (a count for benchmarks). */
DM_API int32_t dm_ep_last_launch_count(const dm_ep *ep);
DM_API void dm_ep_destroy(dm_ep *ep);

/* ---- pinned host memory ----------------------------------------------------------
 * The out-of-core expert pool lives in page-locked host memory so that a cache miss
 * is one DMA copy over PCIe (the reference reads the file with pread instead,
 * src/expert.rs:241-256). dm_cuda_host_alloc returns new pinned memory
 * (cudaHostAlloc, portable across devices); dm_cuda_host_register pins an existing
 * range, e.g. a read-only mapping of the model file. */
DM_API int32_t dm_cuda_host_alloc(dm_cuda_context *ctx, size_t length, void **out);
DM_API void dm_cuda_host_free(dm_cuda_context *ctx, void *host);
DM_API int32_t dm_cuda_host_register(dm_cuda_context *ctx, void *host, size_t length);
DM_API int32_t dm_cuda_host_unregister(dm_cuda_context *ctx, void *host);

/* ---- expert residency ------------------------------------------------------------
 * dm_expert_cache replaces ExpertCache (src/expert.rs:64-229, per-layer clock, slots
 * pinned during use, two reads per miss) and Glm52ExpertCache
 * (src/glm52/expert.rs:66-256, one clock across layers, three reads per miss):
 * `global_clock` selects the GLM rules. Each layer holds `slots_per_layer` slots in
 * HBM, one contiguous array per tensor ([slots][bytes[i]]). acquire() keeps the
 * reference's bookkeeping exactly -- clock += 1; a hit sets last_used; a miss takes
 * the unpinned slot with the smallest (occupied, last_used, index), counts an
 * eviction if it was occupied, then reads the expert -- and counts hits, misses,
 * evictions, reads, bytes_read and resident_bytes as the reference does. The read is
 * a cudaMemcpyAsync from the pinned source on the cache's own copy stream, ordered
 * after the work that last read the slot (release_slot) and before the work that
 * waits for it (wait_slot), so fills overlap compute on other slots.
 *
 * A source is either pinned host memory described by the layout, or a read callback
 * (dm_expert_cache_set_reader) that the cache calls on the host into its own pinned
 * staging, as the reference's pread. All of an expert's tensors are read before any
 * slot byte changes, so a failed or short read leaves the slot as it was; the counters
 * then stand as the reference leaves them (misses and evictions counted, reads and
 * bytes not). With ctx == NULL the slots are host memory and fills are memcpy: the
 * same bookkeeping, usable without a GPU. */
typedef struct dm_expert_cache dm_expert_cache;

/* One layer's experts. Tensor i (i < tensor_count <= 4; Gemma/GGUF: gate_up, down;
 * GLM/Qwen: gate, up, down) of expert e is bytes[i] bytes at
 *   expert_host[e] + offset[i]          when expert_host is set (one blob per expert),
 *   host + offset[i] + e * bytes[i]     otherwise (the GGUF layout: ExpertLayerLayout,
 *                                        src/expert.rs:44-51).
 * Neither is read when the cache has a reader callback. */
typedef struct {
  int32_t expert_count;
  int32_t tensor_count;
  uint64_t bytes[4];
  uint64_t offset[4];
  const void *host;
  const void *const *expert_host;
} dm_expert_layout;

/* ExpertCacheStats (src/expert.rs:53-62) / Glm52ExpertCacheStats
 * (src/glm52/expert.rs:55-64), plus what the copy engine did. io_wait_ns is the
 * device time of the fills (the reference's time spent in reads). */
typedef struct {
  uint64_t hits, misses, evictions, reads, bytes_read;
  uint64_t io_wait_ns;
  uint64_t resident_bytes;
  uint64_t h2d_bytes;  /* bytes copied host -> slot */
  uint64_t fills;      /* fills issued */
} dm_expert_cache_stats;

/* Reader callback: fill `destination` with `length` bytes of tensor `tensor` of
 * (layer, expert); return the number of bytes read (less = a short read) or a
 * negative errno. */
typedef int64_t (*dm_expert_read_fn)(void *user, int32_t layer, int32_t expert, int32_t tensor,
                                     void *destination, uint64_t length);

/* ExpertCache::new (src/expert.rs:87-128) / Glm52ExpertCache::new
 * (src/glm52/expert.rs:103-148): zero slots -> DM_ERR_NO_SLOTS. A layout's host source
 * must be page-locked (dm_cuda_host_alloc / dm_cuda_host_register) for a device
 * cache. */
DM_API int32_t dm_expert_cache_create(dm_cuda_context *ctx, const dm_expert_layout *layouts,
                                      int32_t layers, int32_t slots_per_layer,
                                      int32_t global_clock, dm_expert_cache **out);
DM_API int32_t dm_expert_cache_set_reader(dm_expert_cache *cache, dm_expert_read_fn read,
                                          void *user);
/* Layers created on the cache keep it alive until they are destroyed. */
DM_API void dm_expert_cache_destroy(dm_expert_cache *cache);
DM_API int32_t dm_expert_cache_slots_per_layer(const dm_expert_cache *cache);
/* Base address and per-slot stride of tensor `tensor`'s slot array in `layer`. */
DM_API int32_t dm_expert_cache_slot_memory(const dm_expert_cache *cache, int32_t layer,
                                           int32_t tensor, void **base, uint64_t *stride);
/* The acquire step of with_expert (src/expert.rs:138-164, src/glm52/expert.rs:157-181):
 * `cancelled` (may be NULL) is read before and after, as the reference does, and --
 * with the GLM rules -- once more before a miss's read, where a cancel leaves the slot
 * as it was. Returns the slot and whether it was a miss; the fill is queued, not
 * waited for. */
DM_API int32_t dm_expert_cache_acquire(dm_expert_cache *cache, int32_t layer, int32_t expert,
                                       const int32_t *cancelled, int32_t *slot, int32_t *miss);
/* Make `stream` wait for the slot's last fill / record that `stream`'s work so far
 * reads the slot (the next fill of the slot waits for it). */
DM_API int32_t dm_expert_cache_wait_slot(dm_expert_cache *cache, int32_t layer, int32_t slot,
                                         void *stream);
DM_API int32_t dm_expert_cache_release_slot(dm_expert_cache *cache, int32_t layer, int32_t slot,
                                            void *stream);
/* ExpertSlot::pinned (src/expert.rs:78-84): a pinned slot is never a victim (the GLM
 * rules have no pinning and ignore it). */
DM_API int32_t dm_expert_cache_set_pinned(dm_expert_cache *cache, int32_t layer, int32_t slot,
                                          int32_t pinned);
/* Expert held by a slot (-1 = empty). */
DM_API int32_t dm_expert_cache_slot_expert(const dm_expert_cache *cache, int32_t layer,
                                           int32_t slot, int32_t *expert);
/* Copy a slot's tensor bytes to the host after its fill (synchronous). */
DM_API int32_t dm_expert_cache_read_slot(dm_expert_cache *cache, int32_t layer, int32_t slot,
                                         int32_t tensor, void *destination, uint64_t length);
/* Counters (waits, bounded, for the fills in flight to time them). */
DM_API int32_t dm_expert_cache_get_stats(dm_expert_cache *cache, dm_expert_cache_stats *out);
/* Wait (bounded: DM_ERR_TIMEOUT) for every fill issued so far. */
DM_API int32_t dm_expert_cache_synchronize(dm_expert_cache *cache);

/* A MoE layer whose experts are cache layer `layer`'s slots: desc is as for
 * dm_moe_layer_create, except gate/up/down, which are taken from the cache (its
 * tensor sizes must match the layer's expert strides: gate_up + down for Gemma,
 * gate + up + down otherwise). The router and shared expert stay resident. */
DM_API int32_t dm_moe_layer_create_cached(dm_cuda_context *ctx, const dm_moe_desc *desc,
                                          dm_expert_cache *cache, int32_t layer,
                                          dm_moe_layer **out);
/* The routed block with out-of-core experts: router + top-k, then every (token,
 * expert) pair acquired in the reference's order (tokens in order, experts in
 * selection order, src/glm52/cpu.rs:755-772, src/gemma4/cpu.rs:559-611), misses
 * filled on the copy stream, the shared expert and resident experts computed first
 * and each missed expert as soon as its fill lands, then the combine. When a miss
 * would evict a slot that an earlier pair of the same call still has to read, the
 * pending pairs run first, so every pair sees its own expert -- the sequential
 * reference's semantics. The call waits (bounded) for the routed selection, which
 * the host bookkeeping needs; everything after it is queued on `stream`. */
DM_API int32_t dm_moe_forward_cached(dm_moe_layer *layer, const void *x, float *y,
                                     int32_t tokens, uint32_t *sel_idx, float *sel_weight,
                                     const int32_t *cancelled, void *stream);

#ifdef __cplusplus
}
#endif
#endif
