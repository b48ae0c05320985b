"""The no-allocation forward against the allocating one, through the C ABI.

Some callers of this library cannot call cudaMalloc while a layer runs: a runtime
that has already carved all device memory into its own pools (expert slot pools
sized to fill HBM), or a latency-critical stream that must not see cudaMalloc's
device-wide synchronisation. dm_moe_forward_noalloc serves them: it runs the same
kernels as dm_moe_forward with all per-call scratch taken from a fixed 8 MiB array
inside the library. These checks call both entry points on the same device buffers
and require the same results on two calls in a row (the array keeps the previous
call's contents, so the second call shows nothing stale leaks through), and that a
call needing more scratch than the array holds is refused.

This file is collected last so that a stop-at-first-failure run has already run
every other test; it also passes when run alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import build_layer

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3       # layer-output tolerance used by the parity tests
WEIGHT_ATOL = 2e-7  # selection-weight tolerance used by the parity tests


def _rel_l2(y, ref):
    num = np.linalg.norm((y - ref).astype(np.float64), axis=-1)
    den = np.linalg.norm(ref.astype(np.float64), axis=-1)
    return float((num / np.maximum(den, 1e-30)).max())


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


@pytest.mark.parametrize("name,T", [("qwen35-small", 3), ("gemma4-small", 5), ("glm52-small", 2),
                                    ("qwen35", 1)])
def test_noalloc_forward_matches_the_allocating_forward(ctx, name, T):
    L = N.lib()
    sl = build_layer(ctx, name, seed=11)
    try:
        H, k = sl.cfg["hidden"], sl.cfg["top_k"]
        _, raw = sl.inputs(T, seed=12)
        x = ctx.new_owned_buffer(raw.size)
        x.write(raw)
        out = {n: ctx.new_owned_buffer(T * H * 4 if n.startswith("y") else T * k * 4)
               for n in ("y_ref", "i_ref", "w_ref", "y", "i", "w")}
        p = {n: C.c_void_p(b.device_pointer) for n, b in out.items()}
        N.check(L.dm_moe_forward(sl.layer.handle, C.c_void_p(x.device_pointer), p["y_ref"], T,
                                 p["i_ref"], p["w_ref"], None))
        ctx.synchronize()
        y_ref = out["y_ref"].read().view(np.float32).reshape(T, H)
        i_ref = out["i_ref"].read().view(np.uint32).reshape(T, k)
        w_ref = out["w_ref"].read().view(np.float32).reshape(T, k)
        for _ in range(2):
            N.check(L.dm_moe_forward_noalloc(sl.layer.handle, C.c_void_p(x.device_pointer), p["y"],
                                             T, p["i"], p["w"], None))
            ctx.synchronize()
            y = out["y"].read().view(np.float32).reshape(T, H)
            i = out["i"].read().view(np.uint32).reshape(T, k)
            w = out["w"].read().view(np.float32).reshape(T, k)
            assert np.array_equal(i, i_ref)
            assert np.max(np.abs(w - w_ref)) <= WEIGHT_ATOL
            assert _rel_l2(y, y_ref) <= REL_L2
        for b in out.values():
            b.free()
        x.free()
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
