"""Out-of-core expert residency on the GPU.

The cache's slot bytes and counters against the reference's own fixtures
(src/expert.rs:266-325) and the oracle's LRU; cached MoE layers (experts in pinned
host memory, a few HBM slots, misses copied on the cache's copy stream) against the
oracle block, including slot counts below top-k, where a later miss of the same call
evicts a slot that an earlier pair still reads; and a small GLM decode stack whose
greedy tokens must equal the oracle stack's.
"""
import numpy as np
import pytest
import torch

from diskmule_b200 import _native as N
from diskmule_b200.cache import Cancellation, ExpertCache, PinnedHost, layout
from diskmule_b200.moe import CudaContext
from diskmule_b200.stack import GlmStack
from oracle.stack import OracleStack
from diskmule_b200.synthetic import EXPERT_TENSORS, build_cached_layer
from oracle import oracle as O

from test_gpu_parity import as_f32, check, device_input, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def test_reference_fixture_on_the_device(ctx):
    src = PinnedHost(ctx, 16)
    src.array()[:] = [1, 2, 3, 4, 5, 6, 7, 8, 11, 12, 13, 14, 15, 16, 17, 18]
    cache = ExpertCache(ctx, [layout(2, [4, 4], host=src.pointer, offsets=[0, 8])], 1)
    try:
        for _ in range(2):
            slot, _ = cache.acquire(0, 0)
            assert cache.read_slot(0, slot, 0, 4).tolist() == [1, 2, 3, 4]
            assert cache.read_slot(0, slot, 1, 4).tolist() == [11, 12, 13, 14]
        slot, _ = cache.acquire(0, 1)
        assert cache.read_slot(0, slot, 0, 4).tolist() == [5, 6, 7, 8]
        assert cache.read_slot(0, slot, 1, 4).tolist() == [15, 16, 17, 18]
        s = cache.stats()
        assert (s["hits"], s["misses"], s["evictions"], s["reads"], s["bytes_read"],
                s["resident_bytes"]) == (1, 2, 1, 4, 16, 8)
        assert s["io_wait_ns"] > 0  # src/expert.rs:318: io_wait > 0
        flag = Cancellation()
        flag.cancel()
        with pytest.raises(N.DmError) as e:
            cache.acquire(0, 0, flag)
        assert e.value.status == N.ERR_CANCELLED
    finally:
        cache.close()
        src.free()


def test_pageable_source_is_refused(ctx):
    data = np.zeros(16, np.uint8)
    with pytest.raises(N.DmError) as e:
        ExpertCache(ctx, [layout(2, [4, 4], host=data.ctypes.data, offsets=[0, 8])], 1)
    assert e.value.status == N.ERR_INVALID_ARGUMENT


def lru_for(sl, slots):
    cfg = sl.cfg
    keys = EXPERT_TENSORS[cfg["family"]]
    eb = sum(sl.specs[k].expert_bytes for k in keys)
    return O.Lru(1, cfg["experts"], slots, int(sl.cache.global_clock), eb, len(keys))


CASES = [("glm52-small", 2, 1), ("glm52-small", 2, 9), ("glm52-small", 8, 33),
         ("glm52-small-flat", 1, 4), ("qwen35-small", 3, 5), ("qwen35-small", 16, 64),
         ("gemma4-small", 2, 7), ("gemma4-small", 12, 40)]


@pytest.mark.parametrize("name,slots,T", CASES)
def test_cached_layer_matches_the_oracle(ctx, name, slots, T):
    sl = build_cached_layer(ctx, name, seed=2, slots=slots)
    lru = lru_for(sl, slots)
    try:
        stream = torch.cuda.current_stream().cuda_stream
        for call, seed in enumerate((7, 8)):
            spec, raw = sl.inputs(T, seed=seed)
            x = torch.from_numpy(np.ascontiguousarray(device_input(spec, raw, T))).cuda()
            k = sl.cfg["top_k"]
            y = torch.empty((T, sl.cfg["hidden"]), dtype=torch.float32, device="cuda")
            sel = torch.empty((T, k), dtype=torch.int32, device="cuda")
            w = torch.empty((T, k), dtype=torch.float32, device="cuda")
            sl.layer.forward_cached(x.data_ptr(), y.data_ptr(), T, sel.data_ptr(), w.data_ptr(),
                                    stream=stream)
            torch.cuda.synchronize()
            y_ref, idx_ref, wt_ref = run_oracle(sl, as_f32(spec, raw, T))
            check(y.cpu().numpy(), sel.cpu().numpy().astype(np.uint32), w.cpu().numpy(), y_ref,
                  idx_ref, wt_ref)
            for e in idx_ref.ravel():
                rc, _, _ = lru.acquire(0, int(e))
                assert rc == O.OK
        s, r = sl.cache.stats(), lru.stats()
        for key in ("hits", "misses", "evictions", "reads", "bytes_read", "resident_bytes"):
            assert s[key] == r[key], (key, s, r)
        assert s["h2d_bytes"] == s["bytes_read"] and s["io_wait_ns"] > 0
    finally:
        sl.close()


def test_cancelled_forward_leaves_the_layer_usable(ctx):
    sl = build_cached_layer(ctx, "glm52-small", seed=2, slots=4)
    try:
        T = 3
        spec, raw = sl.inputs(T, seed=7)
        x = torch.from_numpy(np.ascontiguousarray(device_input(spec, raw, T))).cuda()
        y = torch.empty((T, sl.cfg["hidden"]), dtype=torch.float32, device="cuda")
        flag = Cancellation()
        flag.cancel()
        with pytest.raises(N.DmError) as e:
            sl.layer.forward_cached(x.data_ptr(), y.data_ptr(), T, cancelled=flag)
        assert e.value.status == N.ERR_CANCELLED
        flag.reset()
        sl.layer.forward_cached(x.data_ptr(), y.data_ptr(), T, cancelled=flag)
        torch.cuda.synchronize()
        y_ref, _, _ = run_oracle(sl, as_f32(spec, raw, T))
        rel = np.linalg.norm(y.cpu().numpy() - y_ref) / np.linalg.norm(y_ref)
        assert rel <= 1e-3
    finally:
        sl.close()


@pytest.mark.parametrize("slots,pool", [(2, None), (6, 40)])
def test_small_stack_greedy_tokens_match_the_oracle(ctx, slots, pool):
    st = GlmStack(ctx, "glm52-small", layers=3, slots=slots, vocab=512, pool_experts=pool, seed=5)
    try:
        steps = 12
        tokens = st.decode(first_token=17, steps=steps)
        assert st.status_bits() == 0
        ref = OracleStack(st, threads=4)
        ref_tokens = ref.decode(17, steps)
        assert tokens == ref_tokens
        # the cache saw the oracle's selections in order: one clock, per-layer slots
        lru = O.Lru(3, st.E, slots, 1, st.expert_bytes, 3)
        for step in ref.selections:
            for l, sel in enumerate(step):
                for e in sel:
                    assert lru.acquire(l, int(e))[0] == O.OK
        s, r = st.cache.stats(), lru.stats()
        for key in ("hits", "misses", "evictions", "reads", "bytes_read", "resident_bytes"):
            assert s[key] == r[key], (key, s, r)
        h = st.hidden()
        rel = np.linalg.norm(h - ref.last_hidden) / np.linalg.norm(ref.last_hidden)
        assert rel <= 1e-4, rel
    finally:
        st.close()
