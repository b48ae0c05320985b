"""Expert residency bookkeeping on the CPU (dm_expert_cache with host slots).

The cache library call is the product; the checks are the reference's own cache tests
restated (src/expert.rs:266-325, src/glm52/expert.rs:555-595), the oracle's LRU
restatement (oracle/dm_oracle.c, dmo_lru_*) over random access sequences, and the
failure paths of a miss (failed / short read, cancel, all slots pinned) on the host.
"""
import ctypes as C
import errno

import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.cache import Cancellation, ExpertCache, layout
from oracle import oracle as O


def _status(excinfo):
    return excinfo.value.status


def reference_gemma_fixture():
    # the file of src/expert.rs:269-285: gate/up experts, then down experts
    data = np.array([1, 2, 3, 4, 5, 6, 7, 8, 11, 12, 13, 14, 15, 16, 17, 18], dtype=np.uint8)
    lay = layout(2, [4, 4], host=data.ctypes.data, offsets=[0, 8])
    return data, lay


def test_reference_gemma_cache_fixture():
    data, lay = reference_gemma_fixture()
    cache = ExpertCache(None, [lay], slots_per_layer=1)
    assert cache.slots_per_layer() == 1
    for _ in range(2):
        def use(slot):
            assert cache.read_slot(0, slot, 0, 4).tolist() == [1, 2, 3, 4]
            assert cache.read_slot(0, slot, 1, 4).tolist() == [11, 12, 13, 14]
        cache.with_expert(0, 0, use)

    def use1(slot):
        assert cache.read_slot(0, slot, 0, 4).tolist() == [5, 6, 7, 8]
        assert cache.read_slot(0, slot, 1, 4).tolist() == [15, 16, 17, 18]
    cache.with_expert(0, 1, use1)
    s = cache.stats()
    assert (s["hits"], s["misses"], s["evictions"], s["reads"], s["bytes_read"],
            s["resident_bytes"]) == (1, 2, 1, 4, 16, 8)
    assert s["h2d_bytes"] == 16 and s["fills"] == 2
    flag = Cancellation()
    flag.cancel()
    with pytest.raises(N.DmError) as e:
        cache.with_expert(0, 0, lambda slot: None, cancelled=flag)
    assert _status(e) == N.ERR_CANCELLED
    cache.close()


def test_reference_glm_cache_fixture():
    # src/glm52/expert.rs:555-595: layer 1 sparse, one slot, gate/up/down per expert
    rng = np.random.default_rng(1)
    blobs = [rng.integers(0, 256, 96, dtype=np.uint8) for _ in range(2)]
    lay_dense = layout(1, [32, 32, 32], expert_host=[blobs[0].ctypes.data])
    lay = layout(2, [32, 32, 32], offsets=[0, 32, 64], expert_host=[b.ctypes.data for b in blobs])
    cache = ExpertCache(None, [lay_dense, lay], slots_per_layer=1, global_clock=True)
    cancelled = Cancellation()
    for _ in range(2):
        slot, _ = cache.acquire(1, 0, cancelled)
        got = np.concatenate([cache.read_slot(1, slot, t, 32) for t in range(3)])
        assert np.array_equal(got, blobs[0])
    cache.acquire(1, 1, cancelled)
    s = cache.stats()
    assert (s["hits"], s["misses"], s["evictions"], s["reads"]) == (1, 2, 1, 6)
    assert s["bytes_read"] > 0 and s["resident_bytes"] > 0
    cancelled.cancel()
    with pytest.raises(N.DmError) as e:
        cache.acquire(1, 0, cancelled)
    assert _status(e) == N.ERR_CANCELLED


@pytest.mark.parametrize("global_clock", [0, 1])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_sequences_match_the_oracle_lru(global_clock, seed):
    rng = np.random.default_rng(seed)
    layers, experts, slots = 3, 12, 4
    sizes = [16, 8, 24] if global_clock else [16, 24]
    eb = sum(sizes)
    pools = [rng.integers(0, 256, experts * eb, dtype=np.uint8) for _ in range(layers)]
    offs = np.cumsum([0] + sizes[:-1]).tolist()
    lays = [layout(experts, sizes, offsets=[o * experts for o in offs], host=p.ctypes.data)
            for p in pools]
    cache = ExpertCache(None, lays, slots, global_clock=bool(global_clock))
    lru = O.Lru(layers, experts, slots, global_clock, eb, len(sizes))
    for step in range(400):
        layer = int(rng.integers(0, layers))
        expert = int(rng.integers(0, experts))
        if not global_clock and rng.random() < 0.1:
            slot = int(rng.integers(0, slots))
            pin = bool(rng.random() < 0.5)
            cache.set_pinned(layer, slot, pin)
            lru.set_pinned(layer, slot, pin)
            continue
        rc, slot_ref, miss_ref = lru.acquire(layer, expert)
        if rc == O.OK:
            slot, miss = cache.acquire(layer, expert)
            assert (slot, miss) == (slot_ref, miss_ref), step
            for t, (o, n) in enumerate(zip(offs, sizes)):
                want = pools[layer][o * experts + expert * n:o * experts + (expert + 1) * n]
                assert np.array_equal(cache.read_slot(layer, slot, t, n), want)
        else:
            assert rc == O.ERR_ALL_PINNED
            with pytest.raises(N.DmError) as e:
                cache.acquire(layer, expert)
            assert _status(e) == N.ERR_ALL_SLOTS_PINNED
    s, r = cache.stats(), lru.stats()
    for key in ("hits", "misses", "evictions", "reads", "bytes_read", "resident_bytes"):
        assert s[key] == r[key], key


def test_errors_before_any_state_change():
    data, lay = reference_gemma_fixture()
    with pytest.raises(N.DmError) as e:
        ExpertCache(None, [lay], slots_per_layer=0)
    assert _status(e) == N.ERR_NO_SLOTS
    cache = ExpertCache(None, [lay], slots_per_layer=2)
    with pytest.raises(N.DmError) as e:
        cache.acquire(1, 0)
    assert _status(e) == N.ERR_INVALID_LAYER
    with pytest.raises(N.DmError) as e:
        cache.acquire(0, 2)
    assert _status(e) == N.ERR_INVALID_EXPERT
    assert cache.stats()["misses"] == 0 and cache.stats()["hits"] == 0


def test_all_slots_pinned_with_the_pinning_rules_only():
    data, lay = reference_gemma_fixture()
    cache = ExpertCache(None, [lay], slots_per_layer=1)
    cache.acquire(0, 0)
    cache.set_pinned(0, 0, True)
    with pytest.raises(N.DmError) as e:
        cache.acquire(0, 1)
    assert _status(e) == N.ERR_ALL_SLOTS_PINNED
    assert cache.slot_expert(0, 0) == 0  # untouched
    s = cache.stats()
    # src/expert.rs:193-202 counts the miss before it finds no victim
    assert (s["misses"], s["evictions"], s["reads"]) == (2, 0, 2)
    # the GLM cache has no pinning: a pinned flag is ignored
    glm = ExpertCache(None, [lay], slots_per_layer=1, global_clock=True)
    glm.acquire(0, 0)
    glm.set_pinned(0, 0, True)
    assert glm.acquire(0, 1) == (0, True)


class Source:
    """A reader callback over a host pool that can fail, come up short or cancel."""

    def __init__(self, pool, sizes, experts):
        self.pool, self.sizes, self.experts = pool, sizes, experts
        self.offs = np.cumsum([0] + sizes[:-1]).tolist()
        self.fail_at = None  # (expert, tensor) -> OSError
        self.short_at = None
        self.cancel_at = None
        self.flag = None
        self.calls = 0

    def __call__(self, layer, expert, tensor, length):
        self.calls += 1
        if self.fail_at == (expert, tensor):
            raise OSError(errno.EIO, "injected read failure")
        o = self.offs[tensor] * self.experts + expert * self.sizes[tensor]
        data = self.pool[o:o + length].tobytes()
        if self.short_at == (expert, tensor):
            return data[:length // 2]
        if self.cancel_at == (expert, tensor):
            self.flag.cancel()
        return data


@pytest.mark.parametrize("global_clock", [False, True])
def test_reader_source_and_failed_or_short_reads_leave_the_slot(global_clock):
    rng = np.random.default_rng(4)
    sizes, experts = [12, 20], 3
    pool = rng.integers(0, 256, experts * sum(sizes), dtype=np.uint8)
    lay = layout(experts, sizes)
    cache = ExpertCache(None, [lay], slots_per_layer=1, global_clock=global_clock)
    src = Source(pool, sizes, experts)
    cache.set_reader(src)
    slot, miss = cache.acquire(0, 0)
    assert miss and src.calls == 2
    before = [cache.read_slot(0, 0, t, n) for t, n in enumerate(sizes)]
    for attr in ("fail_at", "short_at"):
        setattr(src, attr, (1, 1))
        with pytest.raises(N.DmError) as e:
            cache.acquire(0, 1)
        assert _status(e) == N.ERR_IO
        setattr(src, attr, None)
        # the slot still holds expert 0, byte for byte
        assert cache.slot_expert(0, 0) == 0
        assert all(np.array_equal(cache.read_slot(0, 0, t, n), b)
                   for t, (n, b) in enumerate(zip(sizes, before)))
    s = cache.stats()
    # misses and evictions counted before the read, reads and bytes only after it
    assert (s["misses"], s["evictions"], s["reads"], s["bytes_read"]) == (3, 2, 2, 32)
    assert cache.acquire(0, 0) == (0, False)


def test_cancel_during_a_read_follows_each_caches_rule():
    rng = np.random.default_rng(5)
    sizes, experts = [8, 8, 8], 3
    pool = rng.integers(0, 256, experts * 24, dtype=np.uint8)
    for global_clock in (False, True):
        cache = ExpertCache(None, [layout(experts, sizes)], 1, global_clock=global_clock)
        src = Source(pool, sizes, experts)
        flag = Cancellation()
        src.flag = flag
        cache.set_reader(src)
        cache.acquire(0, 0, flag)
        src.cancel_at = (1, 1)
        with pytest.raises(N.DmError) as e:
            cache.acquire(0, 1, flag)
        assert _status(e) == N.ERR_CANCELLED
        s = cache.stats()
        if global_clock:
            # Glm52ExpertCache drops the loaded expert: the slot keeps expert 0
            assert cache.slot_expert(0, 0) == 0
            assert (s["misses"], s["evictions"], s["reads"]) == (2, 1, 3)
        else:
            # ExpertCache::with_expert checks after acquire: the slot holds expert 1
            assert cache.slot_expert(0, 0) == 1
            assert (s["misses"], s["evictions"], s["reads"]) == (2, 1, 6)


def test_per_expert_blobs_may_alias():
    blob = np.arange(48, dtype=np.uint8)
    lay = layout(4, [16, 32], offsets=[0, 16], expert_host=[blob.ctypes.data] * 4)
    cache = ExpertCache(None, [lay], slots_per_layer=2)
    for e in range(4):
        slot, miss = cache.acquire(0, e)
        assert miss
        assert np.array_equal(cache.read_slot(0, slot, 1, 32), blob[16:])
    assert cache.stats()["evictions"] == 2
