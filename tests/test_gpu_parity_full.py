"""GPU parity at the benchmark sizes, and routing on exact and one-ulp ties.

Configuration 3 (Gemma 4 shape, T=4096, Zipf-skewed router) and configuration 4
(GLM-5.2 shape, bf16, T=8192) run with the benchmark's own seeds. Every token's
selection and the whole dispatch are compared with the oracle (`oracle.route` runs
the reference's router and top-k without the expert weights); layer outputs are
compared on a token subsample (tokens are independent in the reference, so a
subsample at full size checks the full-size kernels).

Ties: the reference orders experts by `total_cmp` on the score and then by index
(src/cpu.rs:246-251, src/glm52/cpu.rs:742-747), so equal scores keep index order.
The tie tests give several experts the same router row (their logits are then equal
bit for bit on both sides) and, for GLM, bias values one unit in the last place of
the score apart.
"""
import os

import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import build_layer, zipf_bias
from oracle import oracle as O

from test_gpu_parity import as_f32, check, check_dispatch, device_input, run_oracle, WEIGHT_ATOL

pytestmark = pytest.mark.gpu

THREADS = max(1, min(os.cpu_count() or 1, 32))


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def check_routing(sl, x32, idx, wt, w=None):
    """Every token's selection against the oracle's router and top-k."""
    fam = sl.cfg["family"]
    if w is None:
        w = sl.host_weights(router_only=True)
    rc, idx_ref, wt_ref = O.route(fam, w, x32, threads=THREADS)
    assert rc == O.OK
    bad = np.argwhere(idx != idx_ref)
    assert bad.size == 0, (bad[:5], idx[bad[0][0]], idx_ref[bad[0][0]])
    assert np.max(np.abs(wt - wt_ref)) <= WEIGHT_ATOL


def test_configuration_3_gemma_zipf_t4096(ctx):
    T = 4096
    sl = build_layer(ctx, "gemma4", seed=1, logit_bias=zipf_bias(128, 1.1, 5))
    try:
        spec, raw = sl.inputs(T, seed=21)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        assert np.all(np.isfinite(y))
        x32 = as_f32(spec, raw, T)
        check_routing(sl, x32, idx, wt)
        check_dispatch(sl, T, idx)
        counts = np.bincount(idx.ravel(), minlength=128)
        assert counts.max() > 8 * T * 8 / 128  # the skew the configuration asks for
        # the subsample includes a token of the busiest and of the least busy used expert
        busiest = int(np.argmax(counts))
        used = np.flatnonzero(counts)
        quiet = int(used[np.argmin(counts[used])])
        sub = sorted({0, 1, 2047, 4095, int(np.argwhere(idx == busiest)[0][0]),
                      int(np.argwhere(idx == quiet)[0][0])})
        y_ref, idx_ref, wt_ref = run_oracle(sl, x32[sub], threads=THREADS)
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
    finally:
        sl.close()


def test_configuration_4_glm_t8192(ctx):
    T = 8192
    sl = build_layer(ctx, "glm52", seed=1)
    try:
        spec, raw = sl.inputs(T, seed=21)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        assert np.all(np.isfinite(y))
        x32 = as_f32(spec, raw, T)
        check_routing(sl, x32, idx, wt)
        check_dispatch(sl, T, idx)
        sub = [0, 4095, 8191]
        experts = sorted(set(idx[sub].ravel().tolist()))
        y_ref, idx_ref, wt_ref = run_oracle(sl, x32[sub], experts=experts, threads=THREADS)
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
    finally:
        sl.close()


# ---- ties ------------------------------------------------------------------------

def _scaled_rows(spec, raw, rows, src, factor):
    """Router bytes with `rows` replaced by row `src` times a power of two (exact)."""
    out = raw.copy()
    if spec.kind == N.F32:
        r = out.view(np.float32).reshape(spec.rows, spec.cols)
        r[rows] = r[src] * np.float32(factor)
    else:
        r = out.view(np.uint16).reshape(spec.rows, spec.cols)
        f = (r[src].astype(np.uint32) << 16).view(np.float32) * np.float32(factor)
        r[rows] = (f.view(np.uint32) >> 16).astype(np.uint16)
    return out


TIE_ROWS = {"qwen35-small": [2, 5, 9, 17, 30], "gemma4-small": [1, 4, 6, 11, 15],
            "glm52-small": [3, 5, 12, 13, 20], "glm52-small-flat": [2, 7, 8, 15]}
TIE_ROWS_FULL = {"qwen35": [2, 5, 9, 17, 300], "gemma4": [1, 4, 6, 11, 100]}


@pytest.mark.parametrize("name,T", [(n, t) for n in sorted(TIE_ROWS) for t in (5, 600)] +
                         [("qwen35", 600), ("gemma4", 600)])  # full routers: 128-expert tiles
def test_exact_and_one_ulp_ties_keep_the_reference_order(ctx, name, T):
    rows = TIE_ROWS[name] if name in TIE_ROWS else TIE_ROWS_FULL[name]
    src = rows[1]
    edited = {}

    def edit(sl):
        spec = sl.specs["router"]
        edited["router"] = _scaled_rows(spec, spec.host(), rows, src, 4.0)
        sl.buffers["router"].write(edited["router"])
        if "bias" in sl.specs:
            b = sl.specs["bias"].host().view(np.float32).copy()
            b[rows] = b[src]
            # one expert of the tie group one unit in the last place above the others in
            # the score's binade [0.5, 1): sigmoid(l) + b moves by exactly that unit
            b[rows[3]] = b[src] + np.float32(2.0 ** -24)
            edited["bias"] = b
            sl.buffers["bias"].write(b)

    sl = build_layer(ctx, name, seed=8, edit=edit)
    try:
        spec, raw = sl.inputs(T, seed=31)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        w = sl.host_weights()
        w["router"] = edited["router"].view(np.float32) if sl.specs["router"].kind == N.F32 \
            else edited["router"]
        if "bias" in edited:
            w["correction_bias"] = edited["bias"]
        x32 = as_f32(spec, raw, T)
        check_routing(sl, x32, idx, wt, w=w)
        check_dispatch(sl, T, idx)
        # the planted ties decided some selections
        in_group = np.isin(idx, rows).sum(axis=1)
        assert np.count_nonzero(in_group >= 2) > 0
        sub = [0, T // 2, T - 1] + [int(np.argmax(in_group))]
        sub = sorted(set(sub))
        rc, y_ref, idx_ref, wt_ref = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe,
                                      "glm52": O.glm_moe}[sl.cfg["family"]](w, x32[sub], threads=8)
        assert rc == O.OK
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
    finally:
        sl.close()


# ---- router kernel forms ---------------------------------------------------------

def test_qwen_many_tokens_take_the_wide_router(ctx):
    # 2048 tokens x 513 router rows: enough 32 x 128 tiles for the wide router kernel
    T = 2048
    sl = build_layer(ctx, "qwen35", seed=12)
    try:
        spec, raw = sl.inputs(T, seed=23)
        y, idx, wt = sl.layer.forward_host(device_input(spec, raw, T))
        x32 = as_f32(spec, raw, T)
        check_routing(sl, x32, idx, wt)
        check_dispatch(sl, T, idx)
        sub = [0, 1023, 2047]
        y_ref, idx_ref, wt_ref = run_oracle(sl, x32[sub], threads=THREADS)
        check(y[sub], idx[sub], wt[sub], y_ref, idx_ref, wt_ref)
    finally:
        sl.close()


def test_glm_input_outside_the_exact_product_range(ctx):
    # bf16 x bf16 router products are exact f32 values, so the GLM router chains may use
    # fused steps, unless a value leaves [2^-60, 2^60): tiles holding such values take the
    # two-rounding step. Plant subnormal, tiny and huge inputs in a few tokens.
    T = 4096
    sl = build_layer(ctx, "glm52", seed=2)
    try:
        spec, raw = sl.inputs(T, seed=29)
        x = raw.view(np.uint16).reshape(T, -1).copy()
        x[5, :] = 0x0001          # smallest bf16 subnormal, every column
        x[700, ::3] = 0x1F80      # 2^-64
        x[3001, 17] = 0x5E00      # 2^61
        x[3001, 18] = 0xDE00      # -2^61
        y, idx, wt = sl.layer.forward_host(x)
        assert np.all(np.isfinite(y))
        x32 = (x.astype(np.uint32) << 16).view(np.float32)
        check_routing(sl, x32, idx, wt)
        check_dispatch(sl, T, idx)
    finally:
        sl.close()
