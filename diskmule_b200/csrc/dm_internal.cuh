// dm_internal.cuh -- host-side objects shared by the C-ABI translation units
// (dm_api.cu: contexts, buffers, layers; dm_cache.cu: expert residency).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "../../include/diskmule_cuda.h"
#include "dm_kernels.cuh"
#include "dm_tc.cuh"

struct dm_cuda_context;
struct dm_moe_layer;
struct dm_expert_cache;

namespace dmi {

// The detail message of the last failing call on this thread (dm_last_error_message).
extern thread_local char g_message[512];
int32_t fail(int32_t status, const char *fmt, ...);
int32_t cuda_fail(cudaError_t err, const char *what);

// Buffers, layers and caches hold a reference on their context.
void retain_context(dm_cuda_context *ctx);
void release_context(dm_cuda_context *ctx);

// Per-layer scratch of dm_moe_forward_cached: the routed selection, the pair rows in
// compute order and their metadata (device, plus a pinned host mirror).
struct CachedScratch {
  int capacity = 0;  // tokens
  void *device = nullptr;
  void *host = nullptr;  // pinned
  uint32_t *sel = nullptr;
  float *sel_w = nullptr, *logits = nullptr, *expert_in = nullptr;
  void *rows = nullptr;   // [R][H] input_type
  float *out = nullptr;   // [R][H]
  float *pair_out = nullptr;  // [R][H], row p = pair p, row T*k + t = shared of token t
  int32_t *meta = nullptr;    // [R] int4: expert id (slot), token, destination row, 0
  int32_t *ids = nullptr;     // [R] expert id of each row, as dm_moe_expert_rows reads it
  int32_t *status = nullptr;
  uint32_t *sel_h = nullptr;  // host mirrors
  int32_t *meta_h = nullptr;
  int32_t *status_h = nullptr;
  cudaEvent_t routed = nullptr;
};

// Expert caches (dm_cache.cu): cached layers hold a reference on their cache.
void cache_retain(dm_expert_cache *cache);
void cache_release(dm_expert_cache *cache);
int32_t cache_layer_view(const dm_expert_cache *cache, int layer, int *tensors, int *slots,
                         uint8_t *const **mem, const uint64_t **bytes);
bool cache_on_device(const dm_expert_cache *cache, int device);
void release_cached_scratch(CachedScratch &scratch);

// Layer scratch for `tokens` tokens (dm_api.cu), forward arguments over it, and the
// expert-kernel plans (GEMV or tcgen05) for the dispatch `a` describes.
int32_t ensure_layer_scratch(dm_moe_layer *L, int tokens);
dm::ForwardArgs fill_args(dm_moe_layer *L, const void *x, float *y, int32_t tokens);
struct Plans {
  dm::GemvPlan plan;
  dm::TcPlan tcp;
  const dm::GemvPlan *gp = nullptr;
  const dm::TcPlan *tp = nullptr;
};
void choose_plans(dm_moe_layer *L, dm::ForwardArgs &a, Plans &P);

}  // namespace dmi

#define DM_CUDA(call, what)                                        \
  do {                                                             \
    cudaError_t err__ = (call);                                    \
    if (err__ != cudaSuccess) return dmi::cuda_fail(err__, what);  \
  } while (0)

struct dm_cuda_context {
  int device = 0;
  // Buffers and layers hold a reference: dm_cuda_destroy frees the context once the
  // last of them is released, so a late free (a garbage collector) stays valid.
  int refs = 0;
  bool closed = false;
  cudaStream_t stream = nullptr;
  char name[256] = {0};
  // operator scratch (grown on demand)
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  int32_t *status = nullptr;

  int32_t ensure_scratch(size_t bytes) {
    if (bytes <= scratch_bytes) return DM_OK;
    if (scratch) cudaFree(scratch);
    scratch = nullptr;
    scratch_bytes = 0;
    size_t want = std::max(bytes, (size_t)1 << 20);
    cudaError_t err = cudaMalloc(&scratch, want);
    if (err != cudaSuccess)
      return dmi::fail(DM_ERR_ALLOCATION, "could not allocate a %zu-byte device buffer", want);
    scratch_bytes = want;
    return DM_OK;
  }
};

struct dm_buffer {
  dm_cuda_context *ctx = nullptr;
  void *device = nullptr;
  size_t length = 0;
  bool read_only = false;
};


struct dm_moe_layer {
  dm_cuda_context *ctx = nullptr;
  dm_moe_desc desc{};
  int E1 = 0;
  // Experts whose weights this layer holds: [first_expert, first_expert + local_experts)
  // of the desc.experts routed by the router (all of them unless created for expert
  // parallelism).
  int first_expert = 0, local_experts = 0;
  bool shared = false;
  void *router_t = nullptr;  // transposed router [H][E1]
  float *router_dup = nullptr;  // [H][router_dup_ld(E1)] f32 router for many tokens
  // GLM: the router is bf16 with every nonzero |w| in [2^-60, 2^60), so its products
  // with bf16 inputs are exact and the router chains may use fused steps
  int router_exact_products = 0;
  float *router_rows = nullptr; // [E1][H] f32 router rows for few tokens
  uint64_t gate_stride = 0, up_stride = 0, down_stride = 0;
  const uint8_t *up_base = nullptr;
  // scratch
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  int capacity = 0;
  dm::ForwardArgs args{};
  int last_tokens = 0;
  int last_launches = 0;
  int last_noalloc = 0;  // the last call was dm_moe_forward_noalloc
  // host-call staging
  void *io = nullptr;
  size_t io_bytes = 0;
  // pipelined host calls (dm_moe_forward_host_batches): two staging slots, a copy-in
  // and a copy-out stream, and a page-locked status word per batch
  void *pipe = nullptr;
  size_t pipe_bytes = 0;
  cudaStream_t pipe_in = nullptr, pipe_out = nullptr;
  cudaEvent_t pipe_ev[6] = {};
  int32_t *pipe_status = nullptr;
  int pipe_status_n = 0;
  // per-stage device timers (GenerationProfile analog)
  bool profiling = false;
  cudaEvent_t events[dm::kStageCount + 1] = {};
  // repacked copies of the 2-byte-aligned block formats, and their memory
  dm::GemvPlan plan{};
  std::vector<void *> owned;
  // tensor-core path: packed activations and TMA maps for 16/32/64-token tiles
  bool tc_ok = false;
  dm::TcPlan tc[3];
  dm::TcWeights tcw;  // tensor-core weight views (valid while tc_ok)
  // bf16 layers: run the down product on fp16 copies of the down weights (held in
  // `owned`) with single fp16 intermediates; off for cache layers, whose slots refill
  bool tc_f16_down = false;
  // CUDA graphs of repeated calls (keyed by buffers and token count)
  struct GraphEntry {
    const void *x;
    float *y;
    int tokens;
    uint32_t *sel_idx;
    float *sel_weight;
    int seen;
    cudaGraphExec_t exec;
    int launches;
    int failed = 0;
  };
  std::vector<GraphEntry> graphs;
  bool graphs_enabled = true;
  cudaStream_t capture = nullptr;
  // expert residency: a layer whose local experts are the slots of `cache` layer
  // `cache_layer` (dm_moe_layer_create_cached), with the forward's own scratch
  dm_expert_cache *cache = nullptr;
  int cache_layer = 0;
  dmi::CachedScratch cached;
  void drop_graphs() {
    for (auto &e : graphs)
      if (e.exec) cudaGraphExecDestroy(e.exec);
    graphs.clear();
  }
};

