// dm_kernels.cuh -- kernel argument blocks and launch helpers of the MoE path.
#pragma once

#include "dm_common.cuh"
#include "dm_gemv.cuh"

namespace dm {

enum Family { kGemma = DM_FAMILY_GEMMA4, kQwen = DM_FAMILY_QWEN35_MOE, kGlm = DM_FAMILY_GLM52 };

// Expert-parallel return map (dm_ep.cu): where the output row of received pair p goes.
// Pair p = (s * tmax + t) * k1 + j (rank s's token t, slot j; slot k is the shared
// expert) lands in rank s's output table at row t * k + j (j < k) or tokens[s] * k + t.
struct EpReturnMap {
  uint8_t *const *peer;     // [ranks] exchange-region bases
  const uint32_t *tokens;   // [ranks] token counts of the current forward
  size_t off_ret;           // byte offset of the output table in a region
  int tmax, k1, k;
};

// Everything a forward needs on the device, by value.
struct ForwardArgs {
  int family;
  int T, H, I, E, k;       // tokens, hidden, intermediate, routed experts, top-k
  int E1;                  // router columns: E (+1 for the Qwen shared gate vector)
  int shared;              // 1 if a shared expert runs for every token
  int n_groups, topk_groups, normalize;
  float routed_scale, epsilon, inv_sqrt_hidden;
  int input_bf16;          // x is bf16 (GLM) instead of f32
  const void *x;           // [T, H]
  float *y;                // [T, H]
  // router
  int router_bf16;
  const void *router_t;    // transposed router [H][E1]
  const float *bias;       // GLM correction bias [E]
  const float *router_scale, *routed_pre_norm, *expert_scale;
  const float *logit_bias; // optional [E], softmax families
  const float *router_dup; // [H][router_dup_ld] f32 router copy (many tokens), or null
  const float *router_rows;  // [E1][H] f32 router rows (few tokens)
  float *xT;               // [H][T rounded up to 32][2] transposed, duplicated router input
  uint8_t *x_tiny;         // [T/32 rounded up][H/32 rounded up]: 1 where a 32x32 tile of a bf16
                           // router input holds a nonzero |x| outside [2^-60, 2^60) (or null)
  int router_exact_products;  // GLM: bf16 router whose nonzero |w| all lie in [2^-60, 2^60)
  // experts
  int gate_type, up_type, down_type;
  const uint8_t *gate, *up, *down;
  uint64_t gate_stride, up_stride, down_stride;   // bytes per expert
  const uint8_t *sh_gate, *sh_up, *sh_down;
  // scratch
  float *router_in;        // Gemma [T, H]
  float *expert_in;        // Gemma [T, H] (routed_pre_norm applied)
  float *logits;           // [T, E1]
  uint32_t *sel_idx;       // [T, k]
  float *sel_w;            // [T, k]
  int32_t *counts;         // [E + 1]
  int32_t *offsets;        // [E + 2]
  int32_t *sorted;         // [T*k + T]
  int32_t *inverse;        // [T*k + T]
  int32_t *active;         // [E + 1] experts with tokens, ascending
  int32_t *n_active;       // [1]
  int rows_mode;           // sel_idx are explicit expert ids (id E = shared), k = 1
  int drop_invalid;        // rows mode: ids above E take no bucket and get no position
                           // (expert-parallel receivers: slots owned by other ranks)
  int chunk;               // tokens per work item
  int4 *items;             // [T*k + T + E + 1] work items: (expert, first token within the
                           // expert, first sorted position, tokens)
  int32_t *n_items;        // [1]
  int32_t *status;         // [1] device error word (0 = ok)
  float *h;                // [(T*k + T), I]
  float *ysorted;          // [(T*k + T), H]
  // expert-parallel receivers whose down product stores each output row straight into
  // its source rank's memory: ydest[pos] is that row (filled after the dispatch from
  // `ret`); null everywhere else
  float **ydest;
  EpReturnMap ret;
  // Work items of an expert with more than `chunk` tokens split its tokens evenly
  // (dispatch_kernel) instead of `chunk`-token items and a remainder.
  int balanced_items;
};

// Row stride (elements) of the transposed router [H][ld]: E1 rounded up to 8 so
// every 8-expert tile row is one aligned vector.
__host__ __device__ inline int router_ld(int E1) { return (E1 + 7) & ~7; }
// Row stride of the f32 router copy [H][ld] used for many tokens: E1 rounded up to the
// 64-expert tile.
__host__ __device__ inline int router_dup_ld(int E1) { return (E1 + 127) & ~127; }

enum DeviceStatus : int32_t {
  kStatusOk = 0,
  kStatusNonFiniteRouter = 1,
  kStatusNonFiniteNorm = 2,
  kStatusTimeout = 3,  // a bounded device wait ran out
};

// Forward stages, timed by optional events recorded at each stage's start.
enum Stage {
  kStagePrep = 0,
  kStageRouter,
  kStageTopk,
  kStageDispatch,
  kStageUp,
  kStageDown,
  kStageCombine,
  kStageCount
};

// launchers (dm_kernels.cu); each returns the number of kernels launched or -1.
// `ev`, when not null, holds kStageCount + 1 events recorded on `stream`.
// `gemv`, when not null, runs the expert products as the GEMV kernels of dm_gemv.cu;
// `tc`, when also given, runs them as the tcgen05 grouped GEMM of dm_tc.cu instead.
struct TcPlan;
// Stages run by launch_forward.
enum RunStages : int {
  kRunRoute = 1,     // Gemma prep, router logits, top-k
  kRunExperts = 2,   // dispatch, gate/up, down
  kRunCombine = 4,   // weighted combine into y
  kRunScatter = 8,   // rows mode: per-row outputs into y
  kRunIdentity = 16, // fill inverse with the identity (pair outputs given in pair order)
  kRunAll = kRunRoute | kRunExperts | kRunCombine,
};

int launch_forward(const ForwardArgs &a, cudaStream_t stream, cudaEvent_t *ev,
                   const GemvPlan *gemv, const TcPlan *tc = nullptr, int mode = kRunAll);
int launch_gemv(int kind, const uint8_t *w, int rows, int cols, const float *x, float *y,
                cudaStream_t stream);
// GLM-5.2 checkpoint encodings (int8 rows, grouped int4, fp8 e4m3 with 128 x 128 block
// scales) times x: one launch.
enum QuantEncoding { kQuantI8Row = 1, kQuantI4 = 2, kQuantF8 = 3 };
int launch_quant_gemv(int enc, const uint8_t *w, const float *scales, int rows, int cols,
                      int group, const float *x, float *y, cudaStream_t stream);
int launch_topk_softmax(const float *logits, int n, int k, uint32_t *idx, float *prob,
                        int32_t *status, cudaStream_t stream);
int launch_elementwise(int op, const float *a, const float *b, float *out, int n,
                       float eps, cudaStream_t stream);
// router [E][H] (+ the Qwen shared-gate row) -> [E1][H] f32 rows (layer set-up)
int launch_router_rows(const void *router, int bf16, int E, int H, const float *extra_col,
                       float *dst, cudaStream_t stream);
// [H][ld] router -> [H][router_dup_ld] f32 (layer set-up)
int launch_dup_router(const void *router_t, int bf16, int H, int E1, float *dst,
                      cudaStream_t stream);
// *flag = 1 if any nonzero |v| of n bf16 values lies outside [2^-60, 2^60) (or is not
// finite); the caller zeroes *flag first (layer set-up)
int launch_bf16_range_check(const uint16_t *v, size_t n, int32_t *flag, cudaStream_t stream);
int launch_transpose_router(const void *src, int src_bf16, int E, int H, const float *extra_col,
                            void *dst, cudaStream_t stream);

int launch_rms_norm(const float *x, const float *w, float *out, int n, float eps,
                    int32_t *status, cudaStream_t stream);

enum ElementwiseOp { kOpGeluMul = 0, kOpSiluMul = 1 };

}  // namespace dm
