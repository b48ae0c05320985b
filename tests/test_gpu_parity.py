"""GPU parity: the CUDA MoE path against the CPU oracle on identical seeded inputs.

Bar (north star): selected expert indices, their order and the dispatch lists are
bit-exact; selection weights within 2e-7 (the reference's own Metal top-k
tolerance, src/metal.rs:2242-2252); layer outputs within 1e-3 relative L2 per token.
"""
import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import build_layer, zipf_bias
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3        # relative L2 of the layer output
REL_L2_TOKEN = 2e-3  # sanity bound on any single token's relative L2
WEIGHT_ATOL = 2e-7


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def as_f32(spec, raw, T):
    if spec.kind == N.BF16:
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(T, -1)
    return raw.view(np.float32).reshape(T, -1)


def device_input(spec, raw, T):
    if spec.kind == N.BF16:
        return raw.view(np.uint16).reshape(T, -1)
    return raw.view(np.float32).reshape(T, -1)


def run_oracle(sl, x32, experts=None, threads=8):
    w = sl.host_weights(experts)
    fam = sl.cfg["family"]
    fn = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe, "glm52": O.glm_moe}[fam]
    rc, y, idx, wt = fn(w, x32, threads=threads)
    assert rc == O.OK
    return y, idx, wt


def rel_l2(y, ref):
    num = np.linalg.norm((y - ref).astype(np.float64), axis=-1)
    den = np.linalg.norm(ref.astype(np.float64), axis=-1)
    return num / np.maximum(den, 1e-30)


def check(y, idx, wt, y_ref, idx_ref, wt_ref):
    assert np.array_equal(idx, idx_ref), np.argwhere(idx != idx_ref)[:5]
    assert np.max(np.abs(wt - wt_ref)) <= WEIGHT_ATOL
    layer = float(np.linalg.norm((y - y_ref).astype(np.float64)) /
                  np.linalg.norm(y_ref.astype(np.float64)))
    token = rel_l2(y, y_ref)
    assert layer <= REL_L2, (layer, token.max())
    assert token.max() <= REL_L2_TOKEN, (layer, token.max())


def check_dispatch(sl, T, idx):
    counts, offsets, sorted_pairs, inverse = sl.layer.last_dispatch(T)
    rc, c2, o2, s2, i2 = O.dispatch(idx, sl.cfg["experts"])
    assert rc == O.OK
    assert np.array_equal(counts, c2)
    assert np.array_equal(offsets, o2)
    assert np.array_equal(sorted_pairs, s2)
    assert np.array_equal(inverse, i2)


SMALL = ["gemma4-small", "gemma4-small-q8", "qwen35-small", "qwen35-odd", "glm52-small",
         "glm52-small-flat"]


@pytest.mark.parametrize("name", SMALL)
@pytest.mark.parametrize("T", [1, 2, 3, 17, 130])
def test_small_layers_match_the_oracle(ctx, name, T):
    sl = build_layer(ctx, name, seed=2)
    try:
        spec, raw = sl.inputs(T, seed=7)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        y_ref, idx_ref, wt_ref = run_oracle(sl, as_f32(spec, raw, T))
        check(y, idx, wt, y_ref, idx_ref, wt_ref)
        check_dispatch(sl, T, idx)
    finally:
        sl.close()


@pytest.mark.parametrize("name", ["qwen35-small", "gemma4-small"])
@pytest.mark.parametrize("T", [1, 2, 5])
@pytest.mark.parametrize("mode", ["large", "small", "spike"])
def test_decode_inputs_of_extreme_magnitude_match_the_oracle(ctx, name, T, mode):
    # The Q4_K decode GEMV scales each token's 256-column block by a power of two and
    # splits it into f16 hi + lo halves: inputs far from 1 and a block whose values span
    # many binades must still match the oracle's f32 products.
    sl = build_layer(ctx, name, seed=4)
    try:
        spec, raw = sl.inputs(T, seed=11)
        x = as_f32(spec, raw, T).copy()
        if mode == "large":
            x *= np.float32(2.0 ** 40)
        elif mode == "small":
            x *= np.float32(2.0 ** -40)
        else:  # one column per 64 a thousand times larger than the rest
            x[:, ::64] *= np.float32(1000.0)
        y, idx, wt = sl.layer.forward_host(x)
        y_ref, idx_ref, wt_ref = run_oracle(sl, x)
        check(y, idx, wt, y_ref, idx_ref, wt_ref)
    finally:
        sl.close()


@pytest.mark.parametrize("name,T", [("gemma4", 1), ("gemma4", 8), ("qwen35", 1), ("qwen35", 8)])
def test_full_size_gguf_layers_match_the_oracle(ctx, name, T):
    sl = build_layer(ctx, name, seed=3)
    try:
        spec, raw = sl.inputs(T, seed=11)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        y_ref, idx_ref, wt_ref = run_oracle(sl, as_f32(spec, raw, T))
        check(y, idx, wt, y_ref, idx_ref, wt_ref)
        check_dispatch(sl, T, idx)
    finally:
        sl.close()


def test_full_size_glm_layer_matches_the_oracle(ctx):
    T = 2
    sl = build_layer(ctx, "glm52", seed=3)
    try:
        spec, raw = sl.inputs(T, seed=11)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        experts = sorted(set(idx.ravel().tolist()))
        y_ref, idx_ref, wt_ref = run_oracle(sl, as_f32(spec, raw, T), experts=experts)
        check(y, idx, wt, y_ref, idx_ref, wt_ref)
    finally:
        sl.close()


def test_full_size_glm_batch_on_tensor_cores(ctx):
    # 512 tokens x top-8 over 256 experts = 16 per expert: the bf16 tcgen05 path
    T, sub = 512, [0, 300, 511]
    sl = build_layer(ctx, "glm52", seed=6)
    try:
        spec, raw = sl.inputs(T, seed=19)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        experts = sorted(set(idx[sub].ravel().tolist()))
        x32 = as_f32(spec, raw, T)[sub]
        y_ref, idx_ref, wt_ref = run_oracle(sl, x32, experts=experts)
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
        check_dispatch(sl, T, idx)
        assert np.all(np.isfinite(y))
    finally:
        sl.close()


@pytest.mark.parametrize("name,T,sub", [("qwen35", 512, [0, 1, 255, 511]),
                                         ("gemma4", 128, [0, 63, 127])])
def test_full_batch_matches_the_oracle_on_a_token_subsample(ctx, name, T, sub):
    # tokens are independent in the reference, so a subsample is a full-size check
    sl = build_layer(ctx, name, seed=4)
    try:
        spec, raw = sl.inputs(T, seed=13)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        x32 = as_f32(spec, raw, T)[sub]
        y_ref, idx_ref, wt_ref = run_oracle(sl, x32)
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
        check_dispatch(sl, T, idx)
        assert np.all(np.isfinite(y))
    finally:
        sl.close()


def test_zipf_skewed_gemma_batch(ctx):
    T = 1024
    bias = zipf_bias(128, 1.1, 5)
    sl = build_layer(ctx, "gemma4", seed=5, logit_bias=bias)
    try:
        spec, raw = sl.inputs(T, seed=17)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        counts = np.bincount(idx.ravel(), minlength=128)
        assert counts.max() > 8 * T * 8 / 128  # heavily skewed
        sub = [0, 511, 1023]
        y_ref, idx_ref, wt_ref = run_oracle(sl, as_f32(spec, raw, T)[sub])
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
        check_dispatch(sl, T, idx)
    finally:
        sl.close()


def test_forward_is_deterministic(ctx):
    sl = build_layer(ctx, "qwen35-small", seed=9)
    try:
        spec, raw = sl.inputs(64, seed=1)
        x = device_input(spec, raw, 64)
        a = sl.layer.forward_host(x)
        b = sl.layer.forward_host(x)
        for u, v in zip(a, b):
            assert np.array_equal(u, v)
    finally:
        sl.close()


def test_non_finite_router_input_is_an_error(ctx):
    sl = build_layer(ctx, "qwen35-small", seed=9)
    try:
        spec, raw = sl.inputs(2, seed=1)
        x = device_input(spec, raw, 2).copy()
        x[1, 3] = np.inf
        with pytest.raises(N.DmError) as err:
            sl.layer.forward_host(x)
        assert err.value.status == N.ERR_NON_FINITE
    finally:
        sl.close()
