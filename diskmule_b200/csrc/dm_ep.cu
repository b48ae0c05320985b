// dm_ep.cu -- expert parallelism over NVLink peer memory (dm_ep_* in
// include/diskmule_cuda.h).
//
// The reference runs every expert of a layer in one process (src/glm52/cpu.rs:711-778);
// here the experts of a layer are split over the GPUs of one box and the token rows
// travel between them as plain stores into the peers' memory (CUDA IPC mappings over
// NVLink / NVSwitch), signalled by per-rank epoch flags. One forward on rank r:
//
//   route      router + top-k of r's tokens (global expert ids)
//   send       one CTA per token: the k local expert ids of each slot (or 0xFF) go to
//              every rank's slot table, and the token row goes once to every rank that
//              owns one of its experts (and to r itself, for the shared expert); the
//              last CTA to finish publishes r's token count and its ready flag
//   wait       until every rank's ready flag holds this epoch (bounded)
//   plan       the received slots become the selection of a rows-mode forward over
//              world x max_tokens rows with k+1 slots (slot k = the shared expert of
//              r's own tokens); slots of other ranks' experts are dropped
//   experts    dispatch + grouped gate/up and down GEMMs on r's experts (dm_tc.cu)
//   return     each output row is stored into its source rank's pair-ordered output
//              table: on the bf16 tensor-core path by the down GEMM's own epilogue (a
//              destination table built right after the dispatch; the NVLink stores
//              overlap the GEMM), otherwise by a copy kernel after it; then r's done
//              flag is raised at every rank
//   wait       until every rank's done flag holds this epoch (bounded)
//   combine    selection-order weighted combine of r's returned rows + shared expert
//
// No host synchronisation and no collective library call happens inside a forward.
// Buffer reuse across forwards is safe without further handshakes: a rank sends the
// rows of forward e+1 only after its combine of forward e has seen every rank's done
// flag of e, which each rank raises only after its GEMMs of e have read their rows.
#include <cuda_runtime.h>

#include <cstring>

#include "dm_internal.cuh"

using dmi::cuda_fail;
using dmi::fail;

namespace {

constexpr int kMaxRanks = 32;
constexpr size_t kFlagBytes = 4096;
// u32 words of a rank's flag block
constexpr int kReady = 0;         // [kMaxRanks] epoch of the rows rank s sent here
constexpr int kDone = 32;         // [kMaxRanks] epoch of the outputs rank s returned here
constexpr int kTokens = 64;       // [kMaxRanks] token count of rank s's current forward
constexpr int kSendCount = 96;    // CTAs of this rank's send kernel that finished
constexpr int kReturnCount = 97;  // CTAs of this rank's return kernel that finished
constexpr uint8_t kNoSlot = 0xFF;
constexpr uint32_t kDrop = 0xFFFFFFFFu;
// about two seconds at the B200's clock: far beyond any skew between ranks that reach
// the same forward, short enough that a rank which never arrives is reported quickly
constexpr long long kWaitCycles = 4000000000ll;

size_t al(size_t v) { return (v + 255) & ~size_t(255); }

struct EpDev {
  uint8_t *const *peer;  // [world] exchange-region bases, this rank's own included
  int rank, world, tmax, H, k, k1, per;
  int xrow;              // bytes per token row
  size_t off_meta, off_x, off_ret;
  uint32_t epoch;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t *flags_of(const EpDev &e, int rank) {
  return reinterpret_cast<uint32_t *>(e.peer[rank]);
}

// The last CTA of a grid to finish raises `word` (ready or done) of this rank at every
// rank. Every CTA first makes its own stores visible system-wide.
__device__ __forceinline__ void signal_when_last(const EpDev &e, int counter, int word,
                                                 bool publish_tokens, uint32_t tokens) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  uint32_t *cnt = flags_of(e, e.rank) + counter;
  const uint32_t prev = atomicAdd(cnt, 1u);
  if (prev != gridDim.x - 1) return;
  __threadfence_system();
  atomicExch(cnt, 0u);  // the next forward's kernel starts after this one ends
  for (int d = 0; d < e.world; d++) {
    uint32_t *f = flags_of(e, d);
    if (publish_tokens) f[kTokens + e.rank] = tokens;
    st_release_sys(f + word + e.rank, e.epoch);
  }
}

// One CTA per token t < T (at least one CTA, so the flags are raised for T = 0).
__global__ void __launch_bounds__(256) ep_send_kernel(EpDev e, const uint8_t *rows, int T,
                                                      const uint32_t *sel) {
  __shared__ uint32_t s_sel[16];
  __shared__ uint32_t s_mask;
  const int t = blockIdx.x;
  if (t < T) {
    if (threadIdx.x < e.k) s_sel[threadIdx.x] = sel[(size_t)t * e.k + threadIdx.x];
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t m = 1u << e.rank;  // the shared expert runs where the token lives
      for (int j = 0; j < e.k; j++) m |= 1u << (s_sel[j] / (uint32_t)e.per);
      s_mask = m;
    }
    __syncthreads();
    // slot table: for every rank d, slot j holds the expert's id local to d or kNoSlot
    for (int i = threadIdx.x; i < e.world * e.k; i += blockDim.x) {
      const int d = i / e.k, j = i - d * e.k;
      const uint32_t id = s_sel[j], owner = id / (uint32_t)e.per;
      e.peer[d][e.off_meta + ((size_t)e.rank * e.tmax + t) * e.k + j] =
          owner == (uint32_t)d ? (uint8_t)(id - owner * e.per) : kNoSlot;
    }
    // the row, once per rank that needs it, in 16-byte pieces
    const uint32_t mask = s_mask;
    const uint4 *src = reinterpret_cast<const uint4 *>(rows + (size_t)t * e.xrow);
    const size_t dst_off = e.off_x + ((size_t)e.rank * e.tmax + t) * e.xrow;
    for (int c = threadIdx.x; c < e.xrow / 16; c += blockDim.x) {
      const uint4 v = src[c];
      for (int d = 0; d < e.world; d++)
        if (mask >> d & 1u) reinterpret_cast<uint4 *>(e.peer[d] + dst_off)[c] = v;
    }
  }
  signal_when_last(e, kSendCount, kReady, true, (uint32_t)T);
}

// One thread per rank: wait (bounded) until that rank's `word` flag here reaches epoch.
__global__ void ep_wait_kernel(EpDev e, int word, int32_t *status) {
  const int d = threadIdx.x;
  if (d >= e.world) return;
  const uint32_t *f = flags_of(e, e.rank) + word + d;
  const long long start = clock64();
  while ((int32_t)(ld_acquire_sys(f) - e.epoch) < 0) {
    if (clock64() - start > kWaitCycles) {
      atomicExch(status, dm::kStatusTimeout);
      return;
    }
    __nanosleep(200);
  }
}

// Received slots -> the selection of the rows-mode expert forward: row r = s * tmax + t
// (rank s's token t), slot j < k from the slot table, slot k the shared expert (local id
// `per`) of this rank's own tokens; everything else is dropped.
__global__ void ep_plan_kernel(EpDev e, uint32_t *recv_sel, const int32_t *status) {
  const uint8_t *own = e.peer[e.rank];
  const uint32_t *f = flags_of(e, e.rank);
  const bool bad = *status == dm::kStatusTimeout;
  const size_t n = (size_t)e.world * e.tmax * e.k1;
  for (size_t p = blockIdx.x * (size_t)blockDim.x + threadIdx.x; p < n;
       p += (size_t)gridDim.x * blockDim.x) {
    const size_t r = p / e.k1;
    const int j = (int)(p - r * e.k1);
    const int s = (int)(r / e.tmax), t = (int)(r - (size_t)s * e.tmax);
    uint32_t id = kDrop;
    if (!bad && t < (int)f[kTokens + s]) {
      if (j < e.k) {
        const uint8_t b = own[e.off_meta + r * e.k + j];
        if (b != kNoSlot) id = b;
      } else if (s == e.rank) {
        id = (uint32_t)e.per;
      }
    }
    recv_sel[p] = id;
  }
}

// The down product already stored every output row into its source rank's memory
// (ForwardArgs::ydest) and fenced: raise this rank's done flag at every rank.
__global__ void ep_signal_done_kernel(EpDev e) {
  const int d = threadIdx.x;
  if (d >= e.world) return;
  __threadfence_system();
  st_release_sys(flags_of(e, d) + kDone + e.rank, e.epoch);
}

// Warp per output row: row `pos` of the sorted outputs goes to its source rank's pair
// table (pair t*k + j, or T_s*k + t for the shared expert). The last CTA raises done.
__global__ void __launch_bounds__(256) ep_return_kernel(EpDev e, const int32_t *n_rows,
                                                        const int32_t *sorted,
                                                        const float *ysorted) {
  const uint32_t *f = flags_of(e, e.rank);
  const int count = *n_rows;
  const int lane = threadIdx.x & 31;
  const int warps = (int)(gridDim.x * blockDim.x) >> 5;
  for (int pos = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); pos < count; pos += warps) {
    const int p = sorted[pos];
    const int r = p / e.k1, j = p - r * e.k1;
    const int s = r / e.tmax, t = r - s * e.tmax;
    const size_t row = j < e.k ? (size_t)t * e.k + j : (size_t)f[kTokens + s] * e.k + t;
    float4 *dst = reinterpret_cast<float4 *>(e.peer[s] + e.off_ret + row * e.H * 4);
    const float4 *src = reinterpret_cast<const float4 *>(ysorted + (size_t)pos * e.H);
    for (int c = lane; c < e.H / 4; c += 32) dst[c] = src[c];
  }
  signal_when_last(e, kReturnCount, kDone, false, 0);
}

}  // namespace

struct dm_ep {
  dm_moe_layer *L = nullptr;
  int rank = 0, world = 1, tmax = 0, k = 0, k1 = 0, per = 0, xrow = 0;
  size_t off_meta = 0, off_x = 0, off_ret = 0, region_bytes = 0;
  uint8_t *region = nullptr;  // exchange region (flags | slot table | rows | outputs)
  uint8_t *peer[kMaxRanks] = {};
  bool peer_ipc[kMaxRanks] = {};
  bool connected = false;
  // local scratch: peer table, selection, received selection, status word
  void *local = nullptr;
  uint8_t **peer_dev = nullptr;
  uint32_t *sel = nullptr;
  float *sel_w = nullptr;
  uint32_t *recv_sel = nullptr;
  float **ydest = nullptr;  // per received pair: its output row in the source rank's memory
  int32_t *status = nullptr;
  uint32_t epoch = 0;
  int tokens = 0;
  int launches = 0;
  int n_sm = 148;
};

namespace {

EpDev dev_view(const dm_ep *ep) {
  EpDev e;
  e.peer = ep->peer_dev;
  e.rank = ep->rank;
  e.world = ep->world;
  e.tmax = ep->tmax;
  e.H = ep->L->desc.hidden;
  e.k = ep->k;
  e.k1 = ep->k1;
  e.per = ep->per;
  e.xrow = ep->xrow;
  e.off_meta = ep->off_meta;
  e.off_x = ep->off_x;
  e.off_ret = ep->off_ret;
  e.epoch = ep->epoch;
  return e;
}

int32_t check_ready(const dm_ep *ep) {
  if (!ep) return fail(DM_ERR_INVALID_ARGUMENT, "null expert-parallel handle");
  if (!ep->connected) return fail(DM_ERR_COMMUNICATOR, "dm_ep_connect_* has not run");
  return DM_OK;
}

}  // namespace

extern "C" {

int32_t dm_ep_create(dm_moe_layer *L, int32_t rank, int32_t world, int32_t max_tokens,
                     dm_ep **out) {
  if (!L || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  const dm_moe_desc &d = L->desc;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(DM_ERR_INVALID_ARGUMENT, "rank %d of %d ranks (at most %d)", rank, world, kMaxRanks);
  if (max_tokens < 1 || (int64_t)max_tokens * world > (1 << 20))
    return fail(DM_ERR_INVALID_ARGUMENT, "max_tokens must be 1..%d per rank", (1 << 20) / world);
  if (d.experts % world)
    return fail(DM_ERR_INVALID_ARGUMENT, "%d experts do not split over %d ranks", d.experts, world);
  const int per = d.experts / world;
  if (per > 255) return fail(DM_ERR_INVALID_ARGUMENT, "more than 255 experts per rank");
  if (d.top_k > 16) return fail(DM_ERR_INVALID_ARGUMENT, "top_k above 16");
  if (L->first_expert != rank * per || L->local_experts != per)
    return fail(DM_ERR_INVALID_ARGUMENT,
                "the layer holds experts %d..%d; rank %d of %d needs %d..%d", L->first_expert,
                L->first_expert + L->local_experts - 1, rank, world, rank * per, rank * per + per - 1);
  if (L->cache) return fail(DM_ERR_INVALID_ARGUMENT, "cache layers are not expert-parallel");
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  dm_ep *ep = new dm_ep();
  ep->L = L;
  ep->rank = rank;
  ep->world = world;
  ep->tmax = max_tokens;
  ep->k = d.top_k;
  ep->k1 = d.top_k + (L->shared ? 1 : 0);
  ep->per = per;
  // rows sent: the expert inputs (Gemma: normalised f32 rows; otherwise the token rows)
  ep->xrow = d.hidden * (d.family == DM_FAMILY_GEMMA4 ? 4 : (d.input_type == DM_BF16 ? 2 : 4));
  const size_t rows = (size_t)world * max_tokens;
  ep->off_meta = kFlagBytes;
  ep->off_x = al(ep->off_meta + rows * ep->k);
  ep->off_ret = al(ep->off_x + rows * ep->xrow);
  ep->region_bytes = al(ep->off_ret + (size_t)max_tokens * ep->k1 * d.hidden * 4);
  cudaDeviceGetAttribute(&ep->n_sm, cudaDevAttrMultiProcessorCount, L->ctx->device);
  auto cleanup = [&](int32_t rc) {
    if (ep->region) cudaFree(ep->region);
    if (ep->local) cudaFree(ep->local);
    delete ep;
    return rc;
  };
  if (cudaMalloc(&ep->region, ep->region_bytes) != cudaSuccess) {
    ep->region = nullptr;
    return cleanup(fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of exchange region",
                        ep->region_bytes));
  }
  const size_t local = al(kMaxRanks * sizeof(void *)) + 2 * al((size_t)max_tokens * ep->k * 4) +
                       al(rows * ep->k1 * 4) + al(rows * ep->k1 * sizeof(float *)) + al(4);
  if (cudaMalloc(&ep->local, local) != cudaSuccess) {
    ep->local = nullptr;
    return cleanup(fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of scratch", local));
  }
  dm::Arena a{(uint8_t *)ep->local, 0, local};
  ep->peer_dev = a.take<uint8_t *>(kMaxRanks);
  ep->sel = a.take<uint32_t>((size_t)max_tokens * ep->k);
  ep->sel_w = a.take<float>((size_t)max_tokens * ep->k);
  ep->recv_sel = a.take<uint32_t>(rows * ep->k1);
  ep->ydest = a.take<float *>(rows * ep->k1);
  ep->status = a.take<int32_t>(1);
  if (a.overflow) return cleanup(fail(DM_ERR_ALLOCATION, "scratch carve overflow"));
  // flags and counters start at zero (epoch 0 = nothing sent yet)
  if (cudaMemset(ep->region, 0, kFlagBytes) != cudaSuccess ||
      cudaMemset(ep->status, 0, 4) != cudaSuccess)
    return cleanup(cuda_fail(cudaGetLastError(), "exchange region set-up"));
  // the rows-mode forward over world x max_tokens received rows needs this much scratch
  int32_t rc = dmi::ensure_layer_scratch(L, (int)rows);
  if (rc != DM_OK) return cleanup(rc);
  if (cudaDeviceSynchronize() != cudaSuccess)
    return cleanup(cuda_fail(cudaGetLastError(), "exchange region set-up"));
  ep->peer[rank] = ep->region;
  *out = ep;
  return DM_OK;
}

int32_t dm_ep_ipc_handle(dm_ep *ep, void *handle) {
  if (!ep || !handle) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  DM_CUDA(cudaSetDevice(ep->L->ctx->device), "cudaSetDevice");
  cudaIpcMemHandle_t h;
  DM_CUDA(cudaIpcGetMemHandle(&h, ep->region), "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  return DM_OK;
}

static int32_t finish_connect(dm_ep *ep) {
  DM_CUDA(cudaMemcpy(ep->peer_dev, ep->peer, sizeof(ep->peer), cudaMemcpyHostToDevice),
          "peer table");
  ep->connected = true;
  return DM_OK;
}

int32_t dm_ep_connect_ipc(dm_ep *ep, const void *handles) {
  if (!ep || !handles) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (ep->connected) return fail(DM_ERR_INVALID_ARGUMENT, "already connected");
  DM_CUDA(cudaSetDevice(ep->L->ctx->device), "cudaSetDevice");
  const uint8_t *all = (const uint8_t *)handles;
  for (int d = 0; d < ep->world; d++) {
    if (d == ep->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, all + (size_t)d * sizeof(h), sizeof(h));
    void *p = nullptr;
    cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) {
      for (int q = 0; q < d; q++)
        if (ep->peer_ipc[q]) cudaIpcCloseMemHandle(ep->peer[q]);
      return cuda_fail(err, "cudaIpcOpenMemHandle of a peer's exchange region");
    }
    ep->peer[d] = (uint8_t *)p;
    ep->peer_ipc[d] = true;
  }
  return finish_connect(ep);
}

int32_t dm_ep_connect_local(dm_ep *ep, dm_ep *const *peers) {
  if (!ep || !peers) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (ep->connected) return fail(DM_ERR_INVALID_ARGUMENT, "already connected");
  for (int d = 0; d < ep->world; d++) {
    const dm_ep *q = peers[d];
    if (!q || q->world != ep->world || q->rank != d || q->tmax != ep->tmax ||
        q->region_bytes != ep->region_bytes)
      return fail(DM_ERR_INVALID_ARGUMENT, "peer %d does not match this expert-parallel group", d);
    if (q->L->ctx->device != ep->L->ctx->device) {
      cudaSetDevice(ep->L->ctx->device);
      cudaError_t err = cudaDeviceEnablePeerAccess(q->L->ctx->device, 0);
      if (err != cudaSuccess && err != cudaErrorPeerAccessAlreadyEnabled)
        return cuda_fail(err, "cudaDeviceEnablePeerAccess");
      cudaGetLastError();
    }
    ep->peer[d] = q->region;
  }
  DM_CUDA(cudaSetDevice(ep->L->ctx->device), "cudaSetDevice");
  return finish_connect(ep);
}

int32_t dm_ep_dispatch(dm_ep *ep, const void *x, int32_t tokens, void *stream) {
  int32_t rc = check_ready(ep);
  if (rc != DM_OK) return rc;
  if (!x && tokens > 0) return fail(DM_ERR_INVALID_ARGUMENT, "null input");
  if (tokens < 0 || tokens > ep->tmax)
    return fail(DM_ERR_INVALID_ARGUMENT, "%d tokens (this group takes 0..%d per rank)", tokens,
                ep->tmax);
  if ((uintptr_t)x & 15) return fail(DM_ERR_INVALID_ARGUMENT, "x must be 16-byte aligned");
  dm_moe_layer *L = ep->L;
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t s = (cudaStream_t)stream;
  ep->epoch++;
  ep->tokens = tokens;
  ep->launches = 0;
  DM_CUDA(cudaMemsetAsync(ep->status, 0, 4, s), "status reset");
  DM_CUDA(cudaMemsetAsync(L->args.status, 0, 4, s), "status reset");
  const uint8_t *rows = (const uint8_t *)x;
  if (tokens > 0) {
    dm::ForwardArgs a = dmi::fill_args(L, x, nullptr, tokens);
    a.sel_idx = ep->sel;
    a.sel_w = ep->sel_w;
    const int n = dm::launch_forward(a, s, nullptr, nullptr, nullptr, dm::kRunRoute);
    if (n < 0) return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "no router kernel for this layer");
    ep->launches += n;
    if (L->desc.family == DM_FAMILY_GEMMA4) rows = (const uint8_t *)a.expert_in;
  }
  ep_send_kernel<<<tokens > 0 ? tokens : 1, 256, 0, s>>>(dev_view(ep), rows, tokens, ep->sel);
  ep->launches++;
  DM_CUDA(cudaGetLastError(), "expert-parallel send");
  return DM_OK;
}

int32_t dm_ep_experts(dm_ep *ep, void *stream) {
  int32_t rc = check_ready(ep);
  if (rc != DM_OK) return rc;
  dm_moe_layer *L = ep->L;
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t s = (cudaStream_t)stream;
  const EpDev e = dev_view(ep);
  ep_wait_kernel<<<1, 32, 0, s>>>(e, kReady, ep->status);
  const size_t n = (size_t)ep->world * ep->tmax * ep->k1;
  ep_plan_kernel<<<(int)std::min<size_t>((n + 255) / 256, (size_t)ep->n_sm * 8), 256, 0, s>>>(
      e, ep->recv_sel, ep->status);
  const int T = ep->world * ep->tmax;
  dm::ForwardArgs a = dmi::fill_args(L, ep->region + ep->off_x, nullptr, T);
  a.k = ep->k1;
  a.E = ep->per;  // local ids; id `per` is the shared expert
  a.shared = 0;
  a.rows_mode = 1;
  a.drop_invalid = 1;
  a.sel_idx = ep->recv_sel;
  if (L->desc.family == DM_FAMILY_GEMMA4) a.expert_in = (float *)(ep->region + ep->off_x);
  dmi::Plans plans;
  dmi::choose_plans(L, a, plans);
  // On the bf16 tensor-core path with fp16 down weights the down GEMM's epilogue stores
  // each output row straight into its source rank's output table (the transfer overlaps
  // the GEMM); otherwise a return kernel copies the rows after it.
  const bool fused = plans.tp && plans.tp->bf16 && L->tcw.f16_down;
  if (fused) {
    a.ydest = ep->ydest;
    a.ret.peer = ep->peer_dev;
    a.ret.tokens = reinterpret_cast<const uint32_t *>(ep->region) + kTokens;
    a.ret.off_ret = ep->off_ret;
    a.ret.tmax = ep->tmax;
    a.ret.k1 = ep->k1;
    a.ret.k = ep->k;
  }
  const int m = dm::launch_forward(a, s, nullptr, plans.gp, plans.tp, dm::kRunExperts);
  if (m < 0) return fail(DM_ERR_UNSUPPORTED_TENSOR_TYPE, "no expert kernel for this format");
  if (fused)
    ep_signal_done_kernel<<<1, 32, 0, s>>>(e);
  else
    ep_return_kernel<<<ep->n_sm * 4, 256, 0, s>>>(e, a.offsets + a.E + 1, a.sorted, a.ysorted);
  ep->launches += m + 3;
  DM_CUDA(cudaGetLastError(), "expert-parallel experts");
  return DM_OK;
}

int32_t dm_ep_combine(dm_ep *ep, float *y, uint32_t *sel_idx, float *sel_weight, void *stream) {
  int32_t rc = check_ready(ep);
  if (rc != DM_OK) return rc;
  if (!y && ep->tokens > 0) return fail(DM_ERR_INVALID_ARGUMENT, "null output");
  if ((uintptr_t)y & 15) return fail(DM_ERR_INVALID_ARGUMENT, "y must be 16-byte aligned");
  dm_moe_layer *L = ep->L;
  DM_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t s = (cudaStream_t)stream;
  ep_wait_kernel<<<1, 32, 0, s>>>(dev_view(ep), kDone, ep->status);
  ep->launches++;
  const int T = ep->tokens;
  if (T > 0) {
    dm::ForwardArgs a = dmi::fill_args(L, nullptr, y, T);
    a.sel_idx = ep->sel;
    a.sel_w = ep->sel_w;
    a.ysorted = (float *)(ep->region + ep->off_ret);
    const int n = dm::launch_forward(a, s, nullptr, nullptr, nullptr,
                                     dm::kRunIdentity | dm::kRunCombine);
    if (n < 0) return fail(DM_ERR_COMMAND, "combine launch");
    ep->launches += n;
    if (sel_idx)
      DM_CUDA(cudaMemcpyAsync(sel_idx, ep->sel, (size_t)T * ep->k * 4, cudaMemcpyDeviceToDevice, s),
              "selection copy");
    if (sel_weight)
      DM_CUDA(cudaMemcpyAsync(sel_weight, ep->sel_w, (size_t)T * ep->k * 4,
                              cudaMemcpyDeviceToDevice, s), "weight copy");
  }
  DM_CUDA(cudaGetLastError(), "expert-parallel combine");
  L->last_launches = ep->launches;
  return DM_OK;
}

int32_t dm_ep_forward(dm_ep *ep, const void *x, float *y, int32_t tokens, uint32_t *sel_idx,
                      float *sel_weight, void *stream) {
  int32_t rc = dm_ep_dispatch(ep, x, tokens, stream);
  if (rc == DM_OK) rc = dm_ep_experts(ep, stream);
  if (rc == DM_OK) rc = dm_ep_combine(ep, y, sel_idx, sel_weight, stream);
  return rc;
}

int32_t dm_ep_status(dm_ep *ep, void *stream) {
  if (!ep) return fail(DM_ERR_INVALID_ARGUMENT, "null expert-parallel handle");
  DM_CUDA(cudaSetDevice(ep->L->ctx->device), "cudaSetDevice");
  int32_t st[2] = {0, 0};
  cudaStream_t s = (cudaStream_t)stream;
  DM_CUDA(cudaMemcpyAsync(&st[0], ep->status, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaMemcpyAsync(&st[1], ep->L->args.status, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaStreamSynchronize(s), "expert-parallel forward");
  if (st[0] == dm::kStatusTimeout)
    return fail(DM_ERR_TIMEOUT, "rank %d: a peer's rows or outputs did not arrive in time",
                ep->rank);
  if (st[1] == dm::kStatusNonFiniteRouter)
    return fail(DM_ERR_NON_FINITE, "router produced a non-finite score");
  if (st[1] == dm::kStatusTimeout)
    return fail(DM_ERR_TIMEOUT, "a bounded wait in the tensor-core GEMM ran out");
  if (st[1] == dm::kStatusNonFiniteNorm)
    return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");
  return DM_OK;
}

int32_t dm_ep_last_launch_count(const dm_ep *ep) { return ep ? ep->launches : 0; }

void dm_ep_destroy(dm_ep *ep) {
  if (!ep) return;
  cudaSetDevice(ep->L->ctx->device);
  cudaDeviceSynchronize();
  for (int d = 0; d < ep->world; d++)
    if (ep->peer_ipc[d]) cudaIpcCloseMemHandle(ep->peer[d]);
  if (ep->region) cudaFree(ep->region);
  if (ep->local) cudaFree(ep->local);
  cudaGetLastError();
  delete ep;
}

}  // extern "C"
