"""The no-allocation forward against the allocating one and the oracle, through the C ABI.

Some callers of this library cannot call cudaMalloc while a layer runs: a runtime
that has already carved all device memory into its own pools (expert slot pools
sized to fill HBM), or a latency-critical stream that must not see cudaMalloc's
device-wide synchronisation. dm_moe_forward_noalloc serves them: it runs the same
kernels as dm_moe_forward with all per-call scratch taken from a fixed 8 MiB array
inside the library. These checks call both entry points on the same device buffers
and require the same results on two calls in a row (the array keeps the previous
call's contents and the outputs are filled with NaN before each call, so nothing
stale can pass), compare with the CPU oracle, and check the refusals: a call needing
more scratch than the array holds, and a layer that holds only some experts.

This file is collected last so that a stop-at-first-failure run has already run
every other test; it also passes when run alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import build_layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3        # layer-output tolerance used by the parity tests
REL_L2_TOKEN = 2e-3  # bound on any single token, as in the parity tests
WEIGHT_ATOL = 2e-7   # selection-weight tolerance used by the parity tests


def _close(y, ref):
    """The parity tests' output bar: relative L2 of the whole output within 1e-3 and of
    every token within 2e-3. (Above a few tokens per expert the allocating forward runs
    the tensor-core GEMM with fp16 operands while the no-allocation forward runs the
    CUDA-core GEMV, so the two differ by the tensor-core path's rounding.)"""
    d = (y - ref).astype(np.float64)
    r = ref.astype(np.float64)
    layer = np.linalg.norm(d) / np.linalg.norm(r)
    token = (np.linalg.norm(d, axis=-1) / np.maximum(np.linalg.norm(r, axis=-1), 1e-30)).max()
    return layer <= REL_L2 and token <= REL_L2_TOKEN, (float(layer), float(token))


def _as_f32(sl, raw, T):
    if sl.cfg["family"] == "glm52":
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(T, -1)
    return raw.view(np.float32).reshape(T, -1)


def _oracle(sl, x32, experts):
    """The oracle block with host weights generated for `experts` only (the others are
    never selected by these tokens)."""
    fn = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe, "glm52": O.glm_moe}[sl.cfg["family"]]
    rc, y, idx, wt = fn(sl.host_weights(experts), x32, threads=8)
    assert rc == O.OK
    return y, idx, wt


def _sentinel(buf):
    """Fill a device buffer with NaN bit patterns (0xFFFFFFFF is also an invalid index)."""
    buf.write(np.full(len(buf) // 4, 0xFFFFFFFF, np.uint32))


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def _largest_accepted(sl, x, y):
    """Largest token count the no-allocation forward accepts on this layer (bisection
    over the refusal, which happens before anything is launched)."""
    L = N.lib()
    lo, hi = 1, 4096
    while hi - lo > 1:
        mid = (lo + hi) // 2
        rc = L.dm_moe_forward_noalloc(sl.layer.handle, C.c_void_p(x.device_pointer),
                                      C.c_void_p(y.device_pointer), mid, None, None, None)
        if rc == N.OK:
            lo = mid
        else:
            assert rc == N.ERR_OVERFLOW
            hi = mid
    return lo


def _compare(ctx, sl, T, check_oracle=True):
    L = N.lib()
    H, k = sl.cfg["hidden"], sl.cfg["top_k"]
    _, raw = sl.inputs(T, seed=12)
    x = ctx.new_owned_buffer(raw.size)
    x.write(raw)
    out = {n: ctx.new_owned_buffer(T * H * 4 if n.startswith("y") else T * k * 4)
           for n in ("y_ref", "i_ref", "w_ref", "y", "i", "w")}
    p = {n: C.c_void_p(b.device_pointer) for n, b in out.items()}
    try:
        N.check(L.dm_moe_forward(sl.layer.handle, C.c_void_p(x.device_pointer), p["y_ref"], T,
                                 p["i_ref"], p["w_ref"], None))
        ctx.synchronize()
        y_ref = out["y_ref"].read().view(np.float32).reshape(T, H)
        i_ref = out["i_ref"].read().view(np.uint32).reshape(T, k)
        w_ref = out["w_ref"].read().view(np.float32).reshape(T, k)
        for _ in range(2):
            for n in ("y", "i", "w"):
                _sentinel(out[n])
            N.check(L.dm_moe_forward_noalloc(sl.layer.handle, C.c_void_p(x.device_pointer),
                                             p["y"], T, p["i"], p["w"], None))
            N.check(L.dm_moe_forward_noalloc_status(sl.layer.handle, None))
            y = out["y"].read().view(np.float32).reshape(T, H)
            i = out["i"].read().view(np.uint32).reshape(T, k)
            w = out["w"].read().view(np.float32).reshape(T, k)
            assert np.isfinite(y).all()
            assert np.array_equal(i, i_ref)
            assert np.max(np.abs(w - w_ref)) <= WEIGHT_ATOL
            ok, err = _close(y, y_ref)
            assert ok, err
        # the dispatch lists of a no-allocation call are not kept
        assert L.dm_moe_last_dispatch(sl.layer.handle, None, None, None, None) == \
            N.ERR_INVALID_ARGUMENT
        if check_oracle:
            y_o, i_o, w_o = _oracle(sl, _as_f32(sl, raw, T), sorted(set(i_ref.ravel().tolist())))
            assert np.array_equal(i, i_o)
            assert np.max(np.abs(w - w_o)) <= WEIGHT_ATOL
            ok, err = _close(y, y_o)
            assert ok, err
    finally:
        for b in out.values():
            b.free()
        x.free()


@pytest.mark.parametrize("name,T", [("qwen35-small", 3), ("qwen35-small", 17),
                                    ("gemma4-small", 5), ("glm52-small", 2), ("qwen35", 1)])
def test_noalloc_forward_matches_the_allocating_forward(ctx, name, T):
    sl = build_layer(ctx, name, seed=11)
    try:
        _compare(ctx, sl, T)
    finally:
        sl.close()


def test_noalloc_forward_at_its_largest_token_count(ctx):
    sl = build_layer(ctx, "qwen35-small", seed=11)
    try:
        H = sl.cfg["hidden"]
        x = ctx.new_owned_buffer(4096 * H * 4)
        y = ctx.new_owned_buffer(4096 * H * 4)
        x.write(np.zeros(4096 * H, np.float32))
        t_max = _largest_accepted(sl, x, y)
        ctx.synchronize()
        x.free()
        y.free()
        assert 17 < t_max < 4096
        _compare(ctx, sl, t_max, check_oracle=True)
    finally:
        sl.close()


def test_noalloc_forward_refuses_calls_beyond_its_scratch(ctx):
    L = N.lib()
    sl = build_layer(ctx, "qwen35-small", seed=11)
    try:
        buf = ctx.new_owned_buffer(1 << 16)
        ptr = C.c_void_p(buf.device_pointer)
        rc = L.dm_moe_forward_noalloc(sl.layer.handle, ptr, ptr, 4096, None, None, None)
        assert rc == N.ERR_OVERFLOW
        assert b"scratch" in L.dm_last_error_message()
        buf.free()
    finally:
        sl.close()


def test_noalloc_forward_refuses_a_layer_holding_some_experts(ctx):
    L = N.lib()
    sl = build_layer(ctx, "qwen35-small", seed=11, expert_range=(0, 16))
    try:
        buf = ctx.new_owned_buffer(1 << 16)
        ptr = C.c_void_p(buf.device_pointer)
        before = L.dm_moe_last_launch_count(sl.layer.handle)
        rc = L.dm_moe_forward_noalloc(sl.layer.handle, ptr, ptr, 2, None, None, None)
        assert rc == N.ERR_INVALID_ARGUMENT
        assert b"experts" in L.dm_last_error_message()
        assert L.dm_moe_last_launch_count(sl.layer.handle) == before
        buf.free()
    finally:
        sl.close()


def test_noalloc_status_reports_a_non_finite_router_input(ctx):
    L = N.lib()
    sl = build_layer(ctx, "qwen35-small", seed=11)
    try:
        H, T = sl.cfg["hidden"], 2
        xs = np.full((T, H), np.nan, np.float32)
        x = ctx.new_owned_buffer(xs.nbytes)
        x.write(xs)
        y = ctx.new_owned_buffer(xs.nbytes)
        N.check(L.dm_moe_forward_noalloc(sl.layer.handle, C.c_void_p(x.device_pointer),
                                         C.c_void_p(y.device_pointer), T, None, None, None))
        assert L.dm_moe_forward_noalloc_status(sl.layer.handle, None) == N.ERR_NON_FINITE
        # the next call starts from a cleared status word
        _, raw = sl.inputs(T, seed=12)
        x.write(raw)
        N.check(L.dm_moe_forward_noalloc(sl.layer.handle, C.c_void_p(x.device_pointer),
                                         C.c_void_p(y.device_pointer), T, None, None, None))
        N.check(L.dm_moe_forward_noalloc_status(sl.layer.handle, None))
        x.free()
        y.free()
    finally:
        sl.close()
