"""Bounded waits end in DM_ERR_TIMEOUT and leave the context usable.

Nothing here faults or hangs the GPU. The device-side case runs the same mbarrier
poll the tensor-core kernels use on a barrier nothing arrives on, limited to a few
million cycles; the host-side case holds the cache's copy stream behind a bounded
sleep kernel on a reader stream, so a slot fill cannot finish within a 200 ms host
limit. Each case then checks that the same context still computes correct results.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import build_layer

from test_gpu_parity import as_f32, check, device_input, run_oracle

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def forward_matches_the_oracle(ctx):
    sl = build_layer(ctx, "qwen35-small", seed=3)
    try:
        spec, raw = sl.inputs(5, seed=11)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, 5))
        check(y, idx, wt, *run_oracle(sl, as_f32(spec, raw, 5)))
    finally:
        sl.close()


def test_device_wait_gives_up_with_a_status(ctx):
    with pytest.raises(N.DmError) as e:
        N.check(N.lib().dm_selftest_device_wait(ctx.handle, 2_000_000))
    assert e.value.status == N.ERR_TIMEOUT and "gave up" in str(e.value)
    forward_matches_the_oracle(ctx)


def test_selftest_limit_is_checked(ctx):
    assert N.lib().dm_selftest_device_wait(ctx.handle, 0) == N.ERR_INVALID_ARGUMENT
    assert N.lib().dm_selftest_device_wait(None, 10) == N.ERR_INVALID_ARGUMENT


HOST_WAIT = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from diskmule_b200 import _native as N
from diskmule_b200.cache import ExpertCache, PinnedHost, layout
from diskmule_b200.moe import CudaContext

ctx = CudaContext(0)
src = PinnedHost(ctx, 32)
src.array()[:] = np.arange(32, dtype=np.uint8)
cache = ExpertCache(ctx, [layout(2, [16], host=src.pointer, offsets=[0])], 1)
slot, miss = cache.acquire(0, 0)
assert miss and cache.read_slot(0, slot, 0, 16).tolist() == list(range(16))
reader = torch.cuda.Stream()
with torch.cuda.stream(reader):
    torch.cuda._sleep(3_000_000_000)       # about 1.5 s at 2 GHz, then it ends
cache.release_slot(0, slot, reader.cuda_stream)
slot, miss = cache.acquire(0, 1)           # evicts expert 0: the fill waits for the reader
assert miss
try:
    cache.read_slot(0, slot, 0, 16)
    print("no timeout")
    sys.exit(1)
except N.DmError as e:
    assert e.status == N.ERR_TIMEOUT, e.status
reader.synchronize()
assert cache.read_slot(0, slot, 0, 16).tolist() == list(range(16, 32))
s = cache.stats()
assert (s["misses"], s["evictions"]) == (2, 1), s
cache.close()
src.free()
ctx.close()
print("ok")
"""


def test_cache_host_wait_gives_up_and_recovers():
    env = dict(os.environ, DISKMULE_CUDA_WAIT_TIMEOUT_MS="200")
    r = subprocess.run([sys.executable, "-c", HOST_WAIT, os.path.dirname(HERE)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
