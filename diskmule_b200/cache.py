"""Out-of-core expert residency over the C ABI.

`ExpertCache` mirrors ExpertCache (src/expert.rs:64-229) and, with
`global_clock=True`, Glm52ExpertCache (src/glm52/expert.rs:66-256): the same
`with_expert` / `stats` surface, LRU decisions and counters. Its slots live in HBM
and a miss is a copy from page-locked host memory on the cache's copy stream
(`PinnedHost`), or a host read through a callback (the reference's pread).
`CachedMoeLayer` is a MoE layer whose experts are one cache layer's slots
(dm_moe_layer_create_cached / dm_moe_forward_cached).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from ._native import check
from .moe import CudaContext, MoeLayer


class PinnedHost:
    """Page-locked host memory (dm_cuda_host_alloc), viewable as a numpy array."""

    def __init__(self, ctx: CudaContext, length: int):
        self.ctx = ctx
        self.length = int(length)
        p = C.c_void_p()
        check(N.lib().dm_cuda_host_alloc(ctx.handle, self.length, C.byref(p)))
        self.pointer = p.value

    def array(self, offset: int = 0, length: int | None = None) -> np.ndarray:
        n = self.length - offset if length is None else length
        buf = (C.c_uint8 * n).from_address(self.pointer + offset)
        return np.frombuffer(buf, dtype=np.uint8)

    def free(self):
        if self.pointer:
            N.lib().dm_cuda_host_free(self.ctx.handle, C.c_void_p(self.pointer))
            self.pointer = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Cancellation:
    """The shared cancel flag (the reference's `cancelled: &AtomicBool`)."""

    def __init__(self):
        self.flag = C.c_int32(0)

    def cancel(self):
        self.flag.value = 1

    def reset(self):
        self.flag.value = 0

    def __bool__(self):
        return bool(self.flag.value)


def layout(expert_count: int, tensor_bytes, host: int = 0, offsets=None, expert_host=None):
    """A dm_expert_layout: tensor i of expert e at `expert_host[e] + offsets[i]`, or at
    `host + offsets[i] + e * tensor_bytes[i]` (ExpertLayerLayout, src/expert.rs:44-51)."""
    lay = N.ExpertLayout()
    lay.expert_count = int(expert_count)
    lay.tensor_count = len(tensor_bytes)
    offsets = offsets or [0] * len(tensor_bytes)
    for i, b in enumerate(tensor_bytes):
        lay.bytes[i] = int(b)
        lay.offset[i] = int(offsets[i])
    lay.host = host or None
    keep = None
    if expert_host is not None:
        keep = (C.c_void_p * expert_count)(*[int(p) for p in expert_host])
        lay.expert_host = C.cast(keep, C.POINTER(C.c_void_p))
    return lay, keep


class ExpertCache:
    """dm_expert_cache. `ctx=None` keeps the slots in host memory (the same
    bookkeeping without a GPU)."""

    def __init__(self, ctx: CudaContext | None, layouts, slots_per_layer: int,
                 global_clock: bool = False):
        self.ctx = ctx
        self._keep = []
        arr = (N.ExpertLayout * len(layouts))()
        for i, item in enumerate(layouts):
            lay, keep = item if isinstance(item, tuple) else (item, None)
            arr[i] = lay
            self._keep.append(keep)
        self._layouts = arr
        h = C.c_void_p()
        check(N.lib().dm_expert_cache_create(ctx.handle if ctx else None, arr, len(layouts),
                                             int(slots_per_layer), int(global_clock), C.byref(h)))
        self._h = h
        self.global_clock = bool(global_clock)
        self._reader = None

    @property
    def handle(self):
        return self._h

    def slots_per_layer(self) -> int:
        return N.lib().dm_expert_cache_slots_per_layer(self._h)

    def set_reader(self, read):
        """Read misses through `read(layer, expert, tensor, length) -> bytes-like`
        (fewer bytes = a short read; an OSError = a failed read)."""

        def trampoline(_user, layer, expert, tensor, dst, length):
            try:
                data = read(layer, expert, tensor, int(length))
            except OSError as e:
                return -(e.errno or 5)
            n = min(len(data), int(length))
            C.memmove(dst, bytes(data[:n]), n)
            return n

        self._reader = N.READ_FN(trampoline)
        check(N.lib().dm_expert_cache_set_reader(self._h, self._reader, None))

    def acquire(self, layer: int, expert: int, cancelled: Cancellation | None = None):
        slot, miss = C.c_int32(), C.c_int32()
        check(N.lib().dm_expert_cache_acquire(self._h, layer, expert,
                                              C.byref(cancelled.flag) if cancelled is not None else None,
                                              C.byref(slot), C.byref(miss)))
        return slot.value, bool(miss.value)

    def with_expert(self, layer: int, expert: int, use, cancelled: Cancellation | None = None):
        """ExpertCache::with_expert (src/expert.rs:138-164): acquire, pin the slot while
        `use(slot)` runs, unpin."""
        slot, _ = self.acquire(layer, expert, cancelled)
        self.set_pinned(layer, slot, True)
        try:
            return use(slot)
        finally:
            self.set_pinned(layer, slot, False)

    def set_pinned(self, layer: int, slot: int, pinned: bool):
        check(N.lib().dm_expert_cache_set_pinned(self._h, layer, slot, int(pinned)))

    def slot_expert(self, layer: int, slot: int) -> int:
        e = C.c_int32()
        check(N.lib().dm_expert_cache_slot_expert(self._h, layer, slot, C.byref(e)))
        return e.value

    def slot_memory(self, layer: int, tensor: int) -> tuple[int, int]:
        base, stride = C.c_void_p(), C.c_uint64()
        check(N.lib().dm_expert_cache_slot_memory(self._h, layer, tensor, C.byref(base),
                                                  C.byref(stride)))
        return base.value or 0, stride.value

    def read_slot(self, layer: int, slot: int, tensor: int, length: int) -> np.ndarray:
        out = np.empty(length, dtype=np.uint8)
        check(N.lib().dm_expert_cache_read_slot(self._h, layer, slot, tensor,
                                                out.ctypes.data_as(C.c_void_p), length))
        return out

    def wait_slot(self, layer: int, slot: int, stream: int = 0):
        check(N.lib().dm_expert_cache_wait_slot(self._h, layer, slot,
                                                C.c_void_p(stream) if stream else None))

    def release_slot(self, layer: int, slot: int, stream: int = 0):
        check(N.lib().dm_expert_cache_release_slot(self._h, layer, slot,
                                                   C.c_void_p(stream) if stream else None))

    def stats(self) -> dict:
        s = N.ExpertCacheStats()
        check(N.lib().dm_expert_cache_get_stats(self._h, C.byref(s)))
        return {f: getattr(s, f) for f, _ in N.ExpertCacheStats._fields_}

    def synchronize(self):
        check(N.lib().dm_expert_cache_synchronize(self._h))

    def close(self):
        if self._h:
            N.lib().dm_expert_cache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CachedMoeLayer(MoeLayer):
    """A MoE layer whose experts are the slots of `cache` layer `layer`
    (dm_moe_layer_create_cached); `forward_cached` is the routed block with misses
    filled from the cache's source."""

    def __init__(self, ctx: CudaContext, desc: N.MoeDesc, cache: ExpertCache, layer: int,
                 keep_alive=()):
        self.ctx = ctx
        self.desc = desc
        self.cache = cache
        self.cache_layer = layer
        self._keep = list(keep_alive)
        h = C.c_void_p()
        check(N.lib().dm_moe_layer_create_cached(ctx.handle, C.byref(desc), cache.handle, layer,
                                                 C.byref(h)))
        self._h = h

    def forward_cached(self, x_ptr: int, y_ptr: int, tokens: int, sel_idx_ptr=None,
                       sel_w_ptr=None, cancelled: Cancellation | None = None, stream: int = 0):
        check(N.lib().dm_moe_forward_cached(self._h, C.c_void_p(x_ptr), C.c_void_p(y_ptr), tokens,
                                            C.c_void_p(sel_idx_ptr) if sel_idx_ptr else None,
                                            C.c_void_p(sel_w_ptr) if sel_w_ptr else None,
                                            C.byref(cancelled.flag) if cancelled is not None else None,
                                            C.c_void_p(stream) if stream else None))
