// dm_cache.cu -- out-of-core expert residency: HBM expert slots refilled from pinned
// host memory by copies on a side stream, with the reference's LRU bookkeeping
// (ExpertCache, src/expert.rs:64-229; Glm52ExpertCache, src/glm52/expert.rs:66-256),
// and the cached MoE forward built on it.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <new>
#include <thread>
#include <vector>

#include "dm_internal.cuh"

using dmi::cuda_fail;
using dmi::fail;

struct dm_expert_cache {
  dm_cuda_context *ctx = nullptr;  // null: host slots, memcpy fills
  int device = 0;
  int layers = 0, slots = 0;
  bool global_clock = false;
  std::vector<dm_expert_layout> layouts;
  struct Slot {
    int32_t expert = -1;
    uint64_t last_used = 0;
    bool pinned = false;
    bool filled = false;  // `fill` marks the slot's last fill
    bool read = false;    // `readers` marks the last work queued that reads the slot
    cudaStream_t waited = nullptr;  // a stream already ordered after the last fill
    bool waited_valid = false;
    cudaEvent_t fill = nullptr, readers = nullptr;
  };
  std::vector<Slot> table;       // [layer][slot]
  std::vector<uint64_t> clocks;  // per layer; entry 0 is the one clock of the GLM rules
  std::vector<uint8_t *> mem;    // [layer][4]: base of the tensor's [slots][bytes] array
  cudaStream_t copy = nullptr;
  dm_expert_read_fn reader = nullptr;
  void *reader_user = nullptr;
  // pinned staging for reader sources, double-buffered so a read overlaps a copy
  uint8_t *staging[2] = {nullptr, nullptr};
  uint64_t staging_bytes = 0;
  cudaEvent_t staging_free[2] = {nullptr, nullptr};
  bool staging_used[2] = {false, false};
  int staging_next = 0;
  struct Timing {
    cudaEvent_t start, end;
  };
  std::deque<Timing> timing;  // fills whose device time is not yet counted
  std::vector<Timing> spare;
  dm_expert_cache_stats stats{};
  int refs = 1;  // the creator's; each cached layer holds one more
  bool closed = false;

  Slot &at(int layer, int slot) { return table[(size_t)layer * slots + slot]; }
  uint64_t expert_bytes(int layer) const {
    uint64_t b = 0;
    for (int i = 0; i < layouts[layer].tensor_count; i++) b += layouts[layer].bytes[i];
    return b;
  }
  const uint8_t *source(int layer, int expert, int tensor) const {
    const dm_expert_layout &l = layouts[layer];
    if (l.expert_host)
      return l.expert_host[expert] ? (const uint8_t *)l.expert_host[expert] + l.offset[tensor]
                                   : nullptr;
    if (!l.host) return nullptr;
    return (const uint8_t *)l.host + l.offset[tensor] + (uint64_t)expert * l.bytes[tensor];
  }
};

namespace {

// Host waits are bounded: DISKMULE_CUDA_WAIT_TIMEOUT_MS (default two minutes; a
// 75 MB fill takes a few milliseconds over PCIe).
double wait_limit_seconds() {
  static double limit = [] {
    const char *env = getenv("DISKMULE_CUDA_WAIT_TIMEOUT_MS");
    double ms = env ? atof(env) : 0.0;
    return ms > 0.0 ? ms / 1000.0 : 120.0;
  }();
  return limit;
}

// Poll `ev` until it completes; a limit turns a stuck copy into DM_ERR_TIMEOUT.
int32_t wait_event(cudaEvent_t ev, const char *what) {
  const auto t0 = std::chrono::steady_clock::now();
  const double limit = wait_limit_seconds();
  for (int spins = 0;; spins++) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return DM_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit)
      return fail(DM_ERR_TIMEOUT, "%s did not complete within %.0f s", what, limit);
    if (spins > 200) std::this_thread::sleep_for(std::chrono::microseconds(20));
    else std::this_thread::yield();
  }
}

bool is_cancelled(const int32_t *flag) { return flag && __atomic_load_n(flag, __ATOMIC_RELAXED); }

// Count the device time of the fills that have finished (all of them with `wait`).
int32_t harvest(dm_expert_cache *C, bool wait) {
  while (!C->timing.empty()) {
    dm_expert_cache::Timing t = C->timing.front();
    if (wait) {
      int32_t rc = wait_event(t.end, "expert fill");
      if (rc != DM_OK) return rc;
    } else if (cudaEventQuery(t.end) != cudaSuccess) {
      break;
    }
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, t.start, t.end) == cudaSuccess)
      C->stats.io_wait_ns += (uint64_t)((double)ms * 1e6);
    C->timing.pop_front();
    C->spare.push_back(t);
  }
  return DM_OK;
}

int32_t ensure_staging(dm_expert_cache *C, uint64_t bytes) {
  if (bytes <= C->staging_bytes) return DM_OK;
  for (int b = 0; b < 2; b++) {
    if (C->staging_used[b]) {
      int32_t rc = wait_event(C->staging_free[b], "staging copy");
      if (rc != DM_OK) return rc;
      C->staging_used[b] = false;
    }
    if (C->staging[b]) {
      if (C->ctx) cudaFreeHost(C->staging[b]);
      else free(C->staging[b]);
      C->staging[b] = nullptr;
    }
  }
  C->staging_bytes = 0;
  for (int b = 0; b < 2; b++) {
    void *p = nullptr;
    if (C->ctx) {
      if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) p = nullptr;
    } else {
      p = malloc(bytes);
    }
    if (!p) return fail(DM_ERR_ALLOCATION, "could not allocate %llu bytes of pinned staging",
                        (unsigned long long)bytes);
    C->staging[b] = (uint8_t *)p;
  }
  C->staging_bytes = bytes;
  return DM_OK;
}

// Read expert `expert` of `layer` into `slot`. Every tensor is read before a slot
// byte changes, so a failed read leaves the slot as it was (src/expert.rs:207-214,
// src/glm52/expert.rs:223-233 return before the slot is updated). `cancelled`, when
// given, is checked between the reads and the first slot write: the GLM cache checks
// after its loads and drops them (src/glm52/expert.rs:229-231).
int32_t issue_fill(dm_expert_cache *C, int layer, int slot, int expert, const int32_t *cancelled) {
  const dm_expert_layout &l = C->layouts[layer];
  const uint64_t total = C->expert_bytes(layer);
  const uint8_t *src[4] = {nullptr, nullptr, nullptr, nullptr};
  int b = -1;
  if (C->reader) {
    int32_t rc = ensure_staging(C, total);
    if (rc != DM_OK) return rc;
    b = C->staging_next;
    C->staging_next ^= 1;
    if (C->staging_used[b]) {
      rc = wait_event(C->staging_free[b], "staging copy");
      if (rc != DM_OK) return rc;
      C->staging_used[b] = false;
    }
    uint64_t off = 0;
    for (int i = 0; i < l.tensor_count; i++) {
      const int64_t got = C->reader(C->reader_user, layer, expert, i, C->staging[b] + off, l.bytes[i]);
      if (got < 0)
        return fail(DM_ERR_IO, "reading tensor %d of expert %d in layer %d failed (errno %lld)", i,
                    expert, layer, (long long)-got);
      if ((uint64_t)got != l.bytes[i])
        return fail(DM_ERR_IO, "short read of tensor %d of expert %d in layer %d: %lld of %llu bytes",
                    i, expert, layer, (long long)got, (unsigned long long)l.bytes[i]);
      src[i] = C->staging[b] + off;
      off += l.bytes[i];
    }
  } else {
    for (int i = 0; i < l.tensor_count; i++) {
      src[i] = C->source(layer, expert, i);
      if (!src[i])
        return fail(DM_ERR_INVALID_ARGUMENT, "layer %d has no source for expert %d", layer, expert);
    }
  }
  if (is_cancelled(cancelled)) return fail(DM_ERR_CANCELLED, "GLM expert cache operation was cancelled");
  dm_expert_cache::Slot &s = C->at(layer, slot);
  if (!C->ctx) {
    for (int i = 0; i < l.tensor_count; i++)
      memcpy(C->mem[(size_t)layer * 4 + i] + (uint64_t)slot * l.bytes[i], src[i], l.bytes[i]);
  } else {
    cudaError_t err = cudaSuccess;
    if (s.read) err = cudaStreamWaitEvent(C->copy, s.readers, 0);
    dm_expert_cache::Timing t{};
    if (!C->spare.empty()) {
      t = C->spare.back();
      C->spare.pop_back();
    } else if (err == cudaSuccess) {
      err = cudaEventCreate(&t.start);
      if (err == cudaSuccess) err = cudaEventCreate(&t.end);
    }
    if (err == cudaSuccess) err = cudaEventRecord(t.start, C->copy);
    for (int i = 0; i < l.tensor_count && err == cudaSuccess; i++)
      err = cudaMemcpyAsync(C->mem[(size_t)layer * 4 + i] + (uint64_t)slot * l.bytes[i], src[i],
                            l.bytes[i], cudaMemcpyHostToDevice, C->copy);
    if (err == cudaSuccess) err = cudaEventRecord(t.end, C->copy);
    if (err == cudaSuccess && b >= 0) {
      err = cudaEventRecord(C->staging_free[b], C->copy);
      C->staging_used[b] = true;
    }
    if (err == cudaSuccess) err = cudaEventRecord(s.fill, C->copy);
    if (err != cudaSuccess) {
      // the slot's bytes may be partly overwritten: it no longer holds its expert
      if (C->global_clock && s.expert >= 0)
        C->stats.resident_bytes -= std::min(C->stats.resident_bytes, total);
      s.expert = -1;
      s.last_used = 0;
      if (t.start) C->spare.push_back(t);
      return cuda_fail(err, "expert fill");
    }
    C->timing.push_back(t);
    s.filled = true;
    s.waited_valid = false;
  }
  C->stats.h2d_bytes += total;
  C->stats.fills += 1;
  return DM_OK;
}

// ExpertCache::acquire (src/expert.rs:166-229) / Glm52ExpertCache::acquire
// (src/glm52/expert.rs:183-256) with the cancel checks of with_expert (src/expert.rs:
// 138-164, src/glm52/expert.rs:157-181). `before_fill(victim)` runs after the victim
// is chosen and before its bytes change: the cached forward uses it to queue the
// pending work that still reads the victim.
int32_t acquire(dm_expert_cache *C, int layer, int expert, const int32_t *cancelled, int *slot,
                int *miss, const std::function<int32_t(int)> &before_fill) {
  const char *cancel_msg = C->global_clock ? "GLM expert cache operation was cancelled"
                                           : "expert loading was cancelled";
  if (is_cancelled(cancelled)) return fail(DM_ERR_CANCELLED, "%s", cancel_msg);
  if (layer < 0 || layer >= C->layers)
    return fail(DM_ERR_INVALID_LAYER, "expert cache layer %d is outside its %d layers", layer,
                C->layers);
  if (expert < 0 || expert >= C->layouts[layer].expert_count)
    return fail(DM_ERR_INVALID_EXPERT, "expert %d is outside layer %d's %d experts", expert, layer,
                C->layouts[layer].expert_count);
  if (C->ctx) harvest(C, false);
  uint64_t &clock = C->clocks[C->global_clock ? 0 : layer];
  if (clock != UINT64_MAX) clock += 1;
  dm_expert_cache::Slot *row = &C->at(layer, 0);
  int found = -1;
  for (int i = 0; i < C->slots; i++)
    if (row[i].expert == expert) {
      found = i;
      break;
    }
  if (found >= 0) {
    row[found].last_used = clock;
    C->stats.hits += 1;
    *slot = found;
    *miss = 0;
  } else {
    C->stats.misses += 1;
    int victim = -1;
    for (int i = 0; i < C->slots; i++) {
      if (!C->global_clock && row[i].pinned) continue;
      if (victim < 0) {
        victim = i;
        continue;
      }
      const int occ_i = row[i].expert >= 0, occ_v = row[victim].expert >= 0;
      if (occ_i < occ_v || (occ_i == occ_v && row[i].last_used < row[victim].last_used)) victim = i;
    }
    if (victim < 0)
      return fail(DM_ERR_ALL_SLOTS_PINNED, "all expert slots in layer %d are pinned by in-flight work",
                  layer);
    const bool evicting = row[victim].expert >= 0;
    if (evicting) C->stats.evictions += 1;
    if (before_fill) {
      int32_t rc = before_fill(victim);
      if (rc != DM_OK) return rc;
    }
    int32_t rc = issue_fill(C, layer, victim, expert, C->global_clock ? cancelled : nullptr);
    if (rc != DM_OK) return rc;
    const uint64_t bytes = C->expert_bytes(layer);
    C->stats.reads += (uint64_t)C->layouts[layer].tensor_count;
    C->stats.bytes_read += bytes;
    if (C->global_clock)
      C->stats.resident_bytes =
          C->stats.resident_bytes - std::min(C->stats.resident_bytes, evicting ? bytes : 0) + bytes;
    row[victim].expert = expert;
    row[victim].last_used = clock;
    *slot = victim;
    *miss = 1;
  }
  if (is_cancelled(cancelled)) return fail(DM_ERR_CANCELLED, "%s", cancel_msg);
  return DM_OK;
}

void free_cache(dm_expert_cache *C) {
  if (C->ctx) {
    cudaSetDevice(C->device);
    if (C->copy) cudaStreamSynchronize(C->copy);
  }
  for (auto &s : C->table) {
    if (s.fill) cudaEventDestroy(s.fill);
    if (s.readers) cudaEventDestroy(s.readers);
  }
  for (auto &t : C->timing) {
    cudaEventDestroy(t.start);
    cudaEventDestroy(t.end);
  }
  for (auto &t : C->spare) {
    cudaEventDestroy(t.start);
    cudaEventDestroy(t.end);
  }
  for (uint8_t *p : C->mem) {
    if (!p) continue;
    if (C->ctx) cudaFree(p);
    else free(p);
  }
  for (int b = 0; b < 2; b++) {
    if (C->staging[b]) {
      if (C->ctx) cudaFreeHost(C->staging[b]);
      else free(C->staging[b]);
    }
    if (C->staging_free[b]) cudaEventDestroy(C->staging_free[b]);
  }
  if (C->copy) cudaStreamDestroy(C->copy);
  if (C->ctx) {
    cudaGetLastError();
    dmi::release_context(C->ctx);
  }
  delete C;
}

int32_t check_slot(const dm_expert_cache *C, int layer, int slot) {
  if (!C) return fail(DM_ERR_INVALID_ARGUMENT, "null cache");
  if (layer < 0 || layer >= C->layers)
    return fail(DM_ERR_INVALID_LAYER, "expert cache layer %d is outside its %d layers", layer,
                C->layers);
  if (slot < 0 || slot >= C->slots)
    return fail(DM_ERR_INVALID_ARGUMENT, "slot %d is outside the %d slots", slot, C->slots);
  return DM_OK;
}

}  // namespace

namespace dmi {

void cache_retain(dm_expert_cache *C) { C->refs++; }

void cache_release(dm_expert_cache *C) {
  if (--C->refs == 0) free_cache(C);
}

// Slot arrays and tensor sizes of one cache layer, for dm_moe_layer_create_cached.
int32_t cache_layer_view(const dm_expert_cache *C, int layer, int *tensors, int *slots,
                         uint8_t *const **mem, const uint64_t **bytes) {
  if (!C) return fail(DM_ERR_INVALID_ARGUMENT, "null cache");
  if (layer < 0 || layer >= C->layers)
    return fail(DM_ERR_INVALID_LAYER, "expert cache layer %d is outside its %d layers", layer,
                C->layers);
  *tensors = C->layouts[layer].tensor_count;
  *slots = C->slots;
  *mem = &C->mem[(size_t)layer * 4];
  *bytes = C->layouts[layer].bytes;
  return DM_OK;
}

bool cache_on_device(const dm_expert_cache *C, int device) { return C->ctx && C->device == device; }

void release_cached_scratch(CachedScratch &S) {
  if (S.device) cudaFree(S.device);
  if (S.host) cudaFreeHost(S.host);
  if (S.routed) cudaEventDestroy(S.routed);
  S = CachedScratch{};
}

}  // namespace dmi

extern "C" {

int32_t dm_cuda_host_alloc(dm_cuda_context *ctx, size_t length, void **out) {
  if (!ctx || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (length == 0) return fail(DM_ERR_ALLOCATION, "could not allocate 0 bytes of pinned memory");
  cudaSetDevice(ctx->device);
  if (cudaHostAlloc(out, length, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    *out = nullptr;
    return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of pinned host memory", length);
  }
  return DM_OK;
}

void dm_cuda_host_free(dm_cuda_context *ctx, void *host) {
  if (!ctx || !host) return;
  cudaSetDevice(ctx->device);
  cudaFreeHost(host);
  cudaGetLastError();
}

int32_t dm_cuda_host_register(dm_cuda_context *ctx, void *host, size_t length) {
  if (!ctx || !host || length == 0) return fail(DM_ERR_INVALID_ARGUMENT, "null or empty range");
  cudaSetDevice(ctx->device);
  DM_CUDA(cudaHostRegister(host, length, cudaHostRegisterPortable | cudaHostRegisterReadOnly),
          "cudaHostRegister");
  return DM_OK;
}

int32_t dm_cuda_host_unregister(dm_cuda_context *ctx, void *host) {
  if (!ctx || !host) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  cudaSetDevice(ctx->device);
  DM_CUDA(cudaHostUnregister(host), "cudaHostUnregister");
  return DM_OK;
}

int32_t dm_expert_cache_create(dm_cuda_context *ctx, const dm_expert_layout *layouts,
                               int32_t layers, int32_t slots_per_layer, int32_t global_clock,
                               dm_expert_cache **out) {
  if (!out) return fail(DM_ERR_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  if (slots_per_layer <= 0)
    return fail(DM_ERR_NO_SLOTS, "expert cache requires at least one slot per layer");
  if (!layouts || layers <= 0) return fail(DM_ERR_INVALID_ARGUMENT, "an expert cache needs layers");
  for (int l = 0; l < layers; l++) {
    const dm_expert_layout &x = layouts[l];
    if (x.expert_count <= 0 || x.tensor_count <= 0 || x.tensor_count > 4)
      return fail(DM_ERR_INVALID_ARGUMENT, "invalid expert cache layout: layer %d has %d experts, %d tensors",
                  l, x.expert_count, x.tensor_count);
    for (int i = 0; i < x.tensor_count; i++)
      if (x.bytes[i] == 0)
        return fail(DM_ERR_INVALID_ARGUMENT, "invalid expert cache layout: tensor %d of layer %d is empty",
                    i, l);
  }
  auto *C = new (std::nothrow) dm_expert_cache();
  if (!C) return fail(DM_ERR_ALLOCATION, "host allocation failed");
  C->ctx = ctx;
  C->layers = layers;
  C->slots = slots_per_layer;
  C->global_clock = global_clock != 0;
  C->layouts.assign(layouts, layouts + layers);
  C->table.resize((size_t)layers * slots_per_layer);
  C->clocks.assign(layers, 0);
  C->mem.assign((size_t)layers * 4, nullptr);
  if (ctx) {
    C->device = ctx->device;
    dmi::retain_context(ctx);
    cudaSetDevice(ctx->device);
  }
  auto bail = [&](int32_t rc) {
    free_cache(C);
    return rc;
  };
  // Sources read by DMA must be page-locked.
  if (ctx) {
    for (int l = 0; l < layers; l++) {
      const dm_expert_layout &x = layouts[l];
      for (int e = 0; e < (x.expert_host ? x.expert_count : 1); e++) {
        const void *p = x.expert_host ? x.expert_host[e] : x.host;
        if (!p) continue;
        cudaPointerAttributes attr{};
        if (cudaPointerGetAttributes(&attr, p) != cudaSuccess || attr.type != cudaMemoryTypeHost) {
          cudaGetLastError();
          return bail(fail(DM_ERR_INVALID_ARGUMENT,
                           "layer %d's expert source is not page-locked host memory "
                           "(use dm_cuda_host_alloc or dm_cuda_host_register)", l));
        }
      }
    }
  }
  uint64_t resident = 0;
  for (int l = 0; l < layers; l++) {
    for (int i = 0; i < layouts[l].tensor_count; i++) {
      const uint64_t bytes = (uint64_t)slots_per_layer * layouts[l].bytes[i];
      void *p = nullptr;
      if (ctx) {
        if (cudaMalloc(&p, bytes) != cudaSuccess) p = nullptr;
      } else {
        p = calloc(1, bytes);
      }
      if (!p) {
        cudaGetLastError();
        return bail(fail(DM_ERR_ALLOCATION, "could not allocate %llu bytes of expert slots",
                         (unsigned long long)bytes));
      }
      C->mem[(size_t)l * 4 + i] = (uint8_t *)p;
    }
    resident += (uint64_t)slots_per_layer * C->expert_bytes(l);
  }
  // The Metal cache allocates its slots up front (src/expert.rs:104-115); the GLM
  // cache counts bytes as experts load.
  C->stats.resident_bytes = C->global_clock ? 0 : resident;
  if (ctx) {
    cudaError_t err = cudaStreamCreateWithFlags(&C->copy, cudaStreamNonBlocking);
    for (auto &s : C->table) {
      if (err == cudaSuccess) err = cudaEventCreateWithFlags(&s.fill, cudaEventDisableTiming);
      if (err == cudaSuccess) err = cudaEventCreateWithFlags(&s.readers, cudaEventDisableTiming);
    }
    for (int b = 0; b < 2 && err == cudaSuccess; b++)
      err = cudaEventCreateWithFlags(&C->staging_free[b], cudaEventDisableTiming);
    if (err != cudaSuccess) return bail(cuda_fail(err, "expert cache set-up"));
  }
  *out = C;
  return DM_OK;
}

int32_t dm_expert_cache_set_reader(dm_expert_cache *C, dm_expert_read_fn read, void *user) {
  if (!C) return fail(DM_ERR_INVALID_ARGUMENT, "null cache");
  C->reader = read;
  C->reader_user = user;
  return DM_OK;
}

void dm_expert_cache_destroy(dm_expert_cache *C) {
  if (!C || C->closed) return;
  C->closed = true;
  dmi::cache_release(C);
}

int32_t dm_expert_cache_slots_per_layer(const dm_expert_cache *C) { return C ? C->slots : 0; }

int32_t dm_expert_cache_slot_memory(const dm_expert_cache *C, int32_t layer, int32_t tensor,
                                    void **base, uint64_t *stride) {
  if (!C || !base || !stride) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (layer < 0 || layer >= C->layers)
    return fail(DM_ERR_INVALID_LAYER, "expert cache layer %d is outside its %d layers", layer,
                C->layers);
  if (tensor < 0 || tensor >= C->layouts[layer].tensor_count)
    return fail(DM_ERR_INVALID_ARGUMENT, "tensor %d is outside layer %d's %d tensors", tensor, layer,
                C->layouts[layer].tensor_count);
  *base = C->mem[(size_t)layer * 4 + tensor];
  *stride = C->layouts[layer].bytes[tensor];
  return DM_OK;
}

int32_t dm_expert_cache_acquire(dm_expert_cache *C, int32_t layer, int32_t expert,
                                const int32_t *cancelled, int32_t *slot, int32_t *miss) {
  if (!C || !slot || !miss) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (C->ctx) cudaSetDevice(C->device);
  int s = -1, m = 0;
  int32_t rc = acquire(C, layer, expert, cancelled, &s, &m, nullptr);
  *slot = s;
  *miss = m;
  return rc;
}

int32_t dm_expert_cache_wait_slot(dm_expert_cache *C, int32_t layer, int32_t slot, void *stream) {
  int32_t rc = check_slot(C, layer, slot);
  if (rc != DM_OK || !C->ctx) return rc;
  dm_expert_cache::Slot &s = C->at(layer, slot);
  if (!s.filled) return DM_OK;
  cudaSetDevice(C->device);
  DM_CUDA(cudaStreamWaitEvent((cudaStream_t)stream, s.fill, 0), "wait for an expert fill");
  return DM_OK;
}

int32_t dm_expert_cache_release_slot(dm_expert_cache *C, int32_t layer, int32_t slot,
                                     void *stream) {
  int32_t rc = check_slot(C, layer, slot);
  if (rc != DM_OK || !C->ctx) return rc;
  cudaSetDevice(C->device);
  dm_expert_cache::Slot &s = C->at(layer, slot);
  DM_CUDA(cudaEventRecord(s.readers, (cudaStream_t)stream), "record an expert slot's readers");
  s.read = true;
  return DM_OK;
}

int32_t dm_expert_cache_set_pinned(dm_expert_cache *C, int32_t layer, int32_t slot,
                                   int32_t pinned) {
  int32_t rc = check_slot(C, layer, slot);
  if (rc != DM_OK) return rc;
  C->at(layer, slot).pinned = pinned != 0;
  return DM_OK;
}

int32_t dm_expert_cache_slot_expert(const dm_expert_cache *C, int32_t layer, int32_t slot,
                                    int32_t *expert) {
  int32_t rc = check_slot(C, layer, slot);
  if (rc != DM_OK) return rc;
  if (!expert) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  *expert = C->table[(size_t)layer * C->slots + slot].expert;
  return DM_OK;
}

int32_t dm_expert_cache_read_slot(dm_expert_cache *C, int32_t layer, int32_t slot, int32_t tensor,
                                  void *destination, uint64_t length) {
  int32_t rc = check_slot(C, layer, slot);
  if (rc != DM_OK) return rc;
  if (!destination) return fail(DM_ERR_INVALID_ARGUMENT, "null destination");
  if (tensor < 0 || tensor >= C->layouts[layer].tensor_count)
    return fail(DM_ERR_INVALID_ARGUMENT, "tensor %d is outside layer %d's tensors", tensor, layer);
  const uint64_t bytes = C->layouts[layer].bytes[tensor];
  if (length > bytes) return fail(DM_ERR_OUTPUT_LENGTH, "a slot tensor holds %llu bytes",
                                  (unsigned long long)bytes);
  const uint8_t *src = C->mem[(size_t)layer * 4 + tensor] + (uint64_t)slot * bytes;
  if (!C->ctx) {
    memcpy(destination, src, length);
    return DM_OK;
  }
  cudaSetDevice(C->device);
  dm_expert_cache::Slot &s = C->at(layer, slot);
  if (s.filled) {
    rc = wait_event(s.fill, "expert fill");
    if (rc != DM_OK) return rc;
  }
  DM_CUDA(cudaMemcpy(destination, src, length, cudaMemcpyDeviceToHost), "slot read");
  return DM_OK;
}

int32_t dm_expert_cache_get_stats(dm_expert_cache *C, dm_expert_cache_stats *out) {
  if (!C || !out) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (C->ctx) {
    cudaSetDevice(C->device);
    int32_t rc = harvest(C, true);
    if (rc != DM_OK) return rc;
  }
  *out = C->stats;
  return DM_OK;
}

int32_t dm_expert_cache_synchronize(dm_expert_cache *C) {
  if (!C) return fail(DM_ERR_INVALID_ARGUMENT, "null cache");
  if (!C->ctx) return DM_OK;
  cudaSetDevice(C->device);
  return harvest(C, true);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// the cached forward
// ---------------------------------------------------------------------------

namespace {

// rows[r] = src[meta[r].token] ([H] elements of `esize` bytes); ids[r] = meta[r].slot.
__global__ void gather_pair_rows_kernel(const uint8_t *__restrict__ src, int row_bytes,
                                        const int4 *__restrict__ meta, int count,
                                        uint8_t *__restrict__ rows, int32_t *__restrict__ ids) {
  const int r = blockIdx.x;
  if (r >= count) return;
  const int4 m = meta[r];
  if (threadIdx.x == 0) ids[r] = m.x;
  const uint4 *s = reinterpret_cast<const uint4 *>(src + (size_t)m.y * row_bytes);
  uint4 *d = reinterpret_cast<uint4 *>(rows + (size_t)r * row_bytes);
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d[i] = s[i];
}

// pair_out[meta[r].dest] = out[r] ([H] f32 rows).
__global__ void scatter_pair_rows_kernel(const float *__restrict__ out, int H,
                                         const int4 *__restrict__ meta, int count,
                                         float *__restrict__ pair_out) {
  const int r = blockIdx.x;
  if (r >= count) return;
  const int dst = meta[r].z;
  const float4 *s = reinterpret_cast<const float4 *>(out + (size_t)r * H);
  float4 *d = reinterpret_cast<float4 *>(pair_out + (size_t)dst * H);
  for (int i = threadIdx.x; i < H / 4; i += blockDim.x) d[i] = s[i];
}

int32_t ensure_cached_scratch(dm_moe_layer *L, int T) {
  dmi::CachedScratch &S = L->cached;
  if (T <= S.capacity) return DM_OK;
  const dm_moe_desc &d = L->desc;
  const size_t k = d.top_k, H = d.hidden, R = (size_t)T * k + (L->shared ? T : 0);
  const size_t xb = d.family == DM_FAMILY_GEMMA4 ? 4 : (d.input_type == DM_BF16 ? 2 : 4);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  size_t bytes = 2 * al((size_t)T * k * 4) + al((size_t)T * L->E1 * 4) +
                 (d.family == DM_FAMILY_GEMMA4 ? al((size_t)T * H * 4) : 0) + al(R * H * xb) +
                 2 * al(R * H * 4) + al(R * 16) + al(R * 4) + al(4);
  const size_t host_bytes = al((size_t)T * k * 4) + al(R * 16) + al(4);
  if (S.device) {
    cudaDeviceSynchronize();
    cudaFree(S.device);
    S.device = nullptr;
  }
  if (S.host) {
    cudaFreeHost(S.host);
    S.host = nullptr;
  }
  S.capacity = 0;
  if (cudaMalloc(&S.device, bytes) != cudaSuccess) {
    S.device = nullptr;
    return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of cached-forward scratch", bytes);
  }
  if (cudaHostAlloc(&S.host, host_bytes, cudaHostAllocDefault) != cudaSuccess) {
    S.host = nullptr;
    return fail(DM_ERR_ALLOCATION, "could not allocate %zu bytes of pinned scratch", host_bytes);
  }
  if (!S.routed && cudaEventCreateWithFlags(&S.routed, cudaEventDisableTiming) != cudaSuccess) {
    S.routed = nullptr;
    return fail(DM_ERR_COMMAND, "could not create an event");
  }
  dm::Arena a{(uint8_t *)S.device, 0, bytes};
  S.sel = a.take<uint32_t>((size_t)T * k);
  S.sel_w = a.take<float>((size_t)T * k);
  S.logits = a.take<float>((size_t)T * L->E1);
  S.expert_in = d.family == DM_FAMILY_GEMMA4 ? a.take<float>((size_t)T * H) : nullptr;
  S.rows = a.take<uint8_t>(R * H * xb);
  S.out = a.take<float>(R * H);
  S.pair_out = a.take<float>(R * H);
  S.meta = reinterpret_cast<int32_t *>(a.take<int4>(R));
  S.ids = a.take<int32_t>(R);
  S.status = a.take<int32_t>(1);
  dm::Arena h{(uint8_t *)S.host, 0, host_bytes};
  S.sel_h = h.take<uint32_t>((size_t)T * k);
  S.meta_h = reinterpret_cast<int32_t *>(h.take<int4>(R));
  S.status_h = h.take<int32_t>(1);
  if (a.overflow || h.overflow) return fail(DM_ERR_ALLOCATION, "cached scratch carve overflow");
  S.capacity = T;
  return DM_OK;
}

// Re-derive a slot's repacked copies (the split layouts of Q6_K / Q5_0 / Q8_0 that the
// GEMV reads) after the slot was refilled.
int refresh_slot(dm_moe_layer *L, int slot, cudaStream_t s) {
  const dm_moe_desc &d = L->desc;
  const uint64_t H = d.hidden, I = d.intermediate;
  const bool fused = d.family == DM_FAMILY_GEMMA4;
  int launches = 0;
  auto one = [&](int kind, const uint8_t *base, uint64_t stride, uint64_t rows, uint64_t cols,
                 const dm::SplitTensor &t) {
    if (!t.quant) return;
    launches++;
    int e = 0, b = 0;
    dm::block_layout(kind, &e, &b);
    const uint64_t per = rows * (cols / (uint64_t)e), g0 = (uint64_t)slot * per;
    const dm::SplitLayout sl = dm::split_layout(kind);
    dm::SplitTensor o;
    o.quant = t.quant + g0 * sl.quant_bytes;
    o.qh = t.qh ? t.qh + g0 * sl.qh_bytes : nullptr;
    o.d = t.d + g0;
    dm::launch_repack(kind, base + (uint64_t)slot * stride, per, o, s);
  };
  one(d.gate_type, (const uint8_t *)d.gate, L->gate_stride, fused ? 2 * I : I, H, L->plan.gate);
  if (!fused) one(d.up_type, (const uint8_t *)d.up, L->up_stride, I, H, L->plan.up);
  one(d.down_type, (const uint8_t *)d.down, L->down_stride, H, I, L->plan.down);
  return launches;
}

}  // namespace

extern "C" int32_t dm_moe_forward_cached(dm_moe_layer *L, const void *x, float *y, int32_t tokens,
                                         uint32_t *sel_idx, float *sel_weight,
                                         const int32_t *cancelled, void *stream) {
  if (!L || !x || !y) return fail(DM_ERR_INVALID_ARGUMENT, "null argument");
  if (!L->cache) return fail(DM_ERR_INVALID_ARGUMENT, "the layer was not created on an expert cache");
  if (tokens < 0) return fail(DM_ERR_INVALID_ARGUMENT, "negative token count");
  if (tokens == 0) return DM_OK;
  if (tokens > (1 << 20)) return fail(DM_ERR_OVERFLOW, "too many tokens in one call (limit 1048576)");
  if (((uintptr_t)y & 15) || ((uintptr_t)x & 15))
    return fail(DM_ERR_INVALID_ARGUMENT, "x and y must be 16-byte aligned device pointers");
  cudaSetDevice(L->ctx->device);
  dm_expert_cache *C = L->cache;
  const int li = L->cache_layer;
  const dm_moe_desc &d = L->desc;
  const int T = tokens, k = d.top_k, H = d.hidden;
  const bool gemma = d.family == DM_FAMILY_GEMMA4;
  const bool qwen_gate = d.family == DM_FAMILY_QWEN35_MOE && L->shared;
  int32_t rc = ensure_cached_scratch(L, T);
  if (rc != DM_OK) return rc;
  dmi::CachedScratch &S = L->cached;
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t *sel = sel_idx ? sel_idx : S.sel;
  float *w = sel_weight ? sel_weight : S.sel_w;

  // 1. router + top-k; the selection comes to the host for the bookkeeping
  rc = dm_moe_route(L, x, T, sel, w, gemma ? S.expert_in : nullptr, qwen_gate ? S.logits : nullptr,
                    stream);
  if (rc != DM_OK) return rc;
  int launches = L->last_launches;  // kernels of this call, for dm_moe_last_launch_count
  DM_CUDA(cudaMemcpyAsync(S.sel_h, sel, (size_t)T * k * 4, cudaMemcpyDeviceToHost, s), "selection copy");
  DM_CUDA(cudaMemcpyAsync(S.status_h, L->args.status, 4, cudaMemcpyDeviceToHost, s), "status copy");
  DM_CUDA(cudaEventRecord(S.routed, s), "event record");
  rc = wait_event(S.routed, "routed selection");
  if (rc != DM_OK) return rc;
  if (*S.status_h == dm::kStatusNonFiniteRouter)
    return fail(DM_ERR_NON_FINITE, "router produced a non-finite score");
  if (*S.status_h == dm::kStatusNonFiniteNorm)
    return fail(DM_ERR_NON_FINITE, "RMSNorm received a non-finite value");

  // 2. acquire every pair in the reference's order; queue compute in waves
  const int R = T * k + (L->shared ? T : 0);
  const int shared_id = C->slots;  // the layer's local id of the shared expert
  const uint8_t *src = gemma ? (const uint8_t *)S.expert_in : (const uint8_t *)x;
  const int row_bytes = H * (gemma ? 4 : (d.input_type == DM_BF16 ? 2 : 4));
  int4 *meta_h = reinterpret_cast<int4 *>(S.meta_h);
  int4 *meta_d = reinterpret_cast<int4 *>(S.meta);
  int cursor = 0;  // rows queued so far (all waves)
  struct Pending {
    int pair, slot;
  };
  std::vector<Pending> pending;            // pairs of the open wave, in order
  std::vector<int> fills;                  // slots filled in the open wave, in fill order
  std::vector<char> in_wave(C->slots, 0);  // slot read by a pair of the open wave
  std::vector<char> filled_in_wave(C->slots, 0);
  bool shared_done = !L->shared;

  auto run_group = [&](int first, int count) -> int32_t {
    if (count == 0) return DM_OK;
    int32_t r = dm_moe_expert_rows(L, (const uint8_t *)S.rows + (size_t)first * row_bytes,
                                   S.ids + first, count, S.out + (size_t)first * H, stream);
    launches += L->last_launches;
    return r;
  };
  // Queue the open wave: gather its rows, run the ready group (resident experts and the
  // shared expert) and then each filled slot's group after its fill, scatter.
  auto launch_wave = [&]() -> int32_t {
    const int first = cursor;
    int n = first;
    for (const Pending &p : pending)
      if (!filled_in_wave[p.slot])
        meta_h[n++] = make_int4(p.slot, p.pair / k, p.pair, 0);
    if (!shared_done)
      for (int t = 0; t < T; t++) meta_h[n++] = make_int4(shared_id, t, T * k + t, 0);
    const int ready_end = n;
    std::vector<int> group_end;
    for (int v : fills) {
      for (const Pending &p : pending)
        if (p.slot == v) meta_h[n++] = make_int4(p.slot, p.pair / k, p.pair, 0);
      group_end.push_back(n);
    }
    if (n == first) return DM_OK;
    const int count = n - first;
    DM_CUDA(cudaMemcpyAsync(meta_d + first, meta_h + first, (size_t)count * sizeof(int4),
                            cudaMemcpyHostToDevice, s), "pair metadata copy");
    gather_pair_rows_kernel<<<count, 128, 0, s>>>(src, row_bytes, meta_d + first, count,
                                                  (uint8_t *)S.rows + (size_t)first * row_bytes,
                                                  S.ids + first);
    DM_CUDA(cudaGetLastError(), "pair gather launch");
    launches++;
    // slots read by the ready group: order after their earlier fills on other streams
    for (const Pending &p : pending)
      if (!filled_in_wave[p.slot]) {
        dm_expert_cache::Slot &sl = C->at(li, p.slot);
        if (sl.filled && !(sl.waited_valid && sl.waited == s)) {
          DM_CUDA(cudaStreamWaitEvent(s, sl.fill, 0), "wait for an expert fill");
          sl.waited = s;
          sl.waited_valid = true;
        }
      }
    int32_t r = run_group(first, ready_end - first);
    if (r != DM_OK) return r;
    for (const Pending &p : pending)
      if (!filled_in_wave[p.slot]) {
        r = dm_expert_cache_release_slot(C, li, p.slot, stream);
        if (r != DM_OK) return r;
      }
    int start = ready_end;
    for (size_t g = 0; g < fills.size(); g++) {
      const int v = fills[g];
      dm_expert_cache::Slot &sl = C->at(li, v);
      DM_CUDA(cudaStreamWaitEvent(s, sl.fill, 0), "wait for an expert fill");
      sl.waited = s;
      sl.waited_valid = true;
      launches += refresh_slot(L, v, s);
      r = run_group(start, group_end[g] - start);
      if (r != DM_OK) return r;
      r = dm_expert_cache_release_slot(C, li, v, stream);
      if (r != DM_OK) return r;
      start = group_end[g];
    }
    scatter_pair_rows_kernel<<<count, 128, 0, s>>>(S.out + (size_t)first * H, H, meta_d + first,
                                                   count, S.pair_out);
    DM_CUDA(cudaGetLastError(), "pair scatter launch");
    launches++;
    cursor = n;
    shared_done = true;
    for (const Pending &p : pending) in_wave[p.slot] = 0;
    for (int v : fills) filled_in_wave[v] = 0;
    pending.clear();
    fills.clear();
    return DM_OK;
  };
  // A miss about to overwrite a slot that the open wave still reads closes the wave.
  auto before_fill = [&](int victim) -> int32_t {
    return in_wave[victim] ? launch_wave() : DM_OK;
  };

  for (int p = 0; p < T * k; p++) {
    int slot = -1, miss = 0;
    rc = acquire(C, li, (int)S.sel_h[p], cancelled, &slot, &miss, before_fill);
    if (rc != DM_OK) return rc;
    if (miss) {
      filled_in_wave[slot] = 1;
      fills.push_back(slot);
    }
    in_wave[slot] = 1;
    pending.push_back({p, slot});
  }
  rc = launch_wave();
  if (rc != DM_OK) return rc;

  // 3. combine in selection order (+ the shared expert)
  rc = dm_moe_combine_rows(L, T, sel, w, qwen_gate ? S.logits : nullptr, S.pair_out, y, stream);
  if (rc != DM_OK) return rc;
  L->last_launches = launches + L->last_launches;
  return DM_OK;
}
