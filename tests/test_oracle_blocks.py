"""The oracle's MoE blocks compose its pinned primitives as the reference does (CPU).

Each block is recomputed here from the primitive oracle calls (already pinned by
test_oracle_golden.py) following the reference source line by line.
"""
import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.synthetic import CONFIGS, input_spec, layer_specs, vectors
from oracle import oracle as O


class HostLayer:
    """host_weights() of a SyntheticLayer without a device."""

    def __init__(self, name, seed=1):
        from diskmule_b200.synthetic import SyntheticLayer
        cfg = dict(CONFIGS[name])
        self.sl = SyntheticLayer(name, cfg, seed, None, layer_specs(cfg, seed), vectors(cfg, seed))
        self.cfg = cfg

    def weights(self):
        return self.sl.host_weights()

    def x(self, T, seed=5):
        spec = input_spec(self.cfg, T, seed)
        raw = spec.host()
        if spec.kind == N.BF16:
            return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(T, -1)
        return raw.view(np.float32).reshape(T, -1)


def fma32(a, b, c):
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def test_gemma_block_composes_primitives():
    # src/gemma4/cpu.rs:559-611
    hl = HostLayer("gemma4-small")
    w = hl.weights()
    x = hl.x(3)
    rc, y, idx, prob = O.gemma_moe(w, x)
    assert rc == O.OK
    H, I, E, k = w["hidden"], w["intermediate"], w["experts"], w["top_k"]
    gu_row = O.row_byte_len(w["gate_up_type"], H)
    dn_row = O.row_byte_len(w["down_type"], I)
    for t in range(3):
        _, routed_in = O.rms_norm(x[t], w["routed_pre_norm"], 1e-6)
        _, router_in = O.rms_norm(x[t], None, 1e-6)
        inv_h = np.float32(1.0) / np.sqrt(np.float32(H))
        router_in = (router_in * (w["router_scale"] * inv_h).astype(np.float32)).astype(np.float32)
        _, logits = O.matvec(O.F32, E, H, w["router"].tobytes(), router_in)
        _, ei, ep = O.top_k_softmax(logits, k)
        assert ei.tolist() == idx[t].tolist() and ep.tolist() == prob[t].tolist()
        routed = np.zeros(H, np.float32)
        for e, p in zip(ei, ep):
            gu = w["gate_up"][e * 2 * I * gu_row:(e + 1) * 2 * I * gu_row]
            _, g = O.matvec(w["gate_up_type"], 2 * I, H, gu, routed_in)
            act = np.array([np.float32(O.gelu_tanh(a)) * b for a, b in zip(g[:I], g[I:])], np.float32)
            dn = w["down"][e * H * dn_row:(e + 1) * H * dn_row]
            _, out = O.matvec(w["down_type"], H, I, dn, act)
            scale = np.float32(p) * w["expert_scale"][e]
            routed = np.array([fma32(o, scale, r) for o, r in zip(out, routed)], np.float32)
        np.testing.assert_allclose(y[t], routed, rtol=1e-6, atol=1e-7)


def test_glm_block_composes_primitives():
    # src/glm52/cpu.rs:731-776 with the reference's flat routing (1 group)
    hl = HostLayer("glm52-small-flat")
    w = hl.weights()
    x = hl.x(2)
    rc, y, idx, wt = O.glm_moe(w, x)
    assert rc == O.OK
    H, I, E, k = w["hidden"], w["intermediate"], w["experts"], w["top_k"]
    eb = I * H * 2
    for t in range(2):
        _, logits = O.glm_matvec(O.BF16, E, H, w["router"], x[t])
        rc, ei, ew = O.glm_select(logits, w["correction_bias"], k)
        assert ei.tolist() == idx[t].tolist() and ew.tolist() == wt[t].tolist()
        out = np.zeros(H, np.float32)
        for e, we in zip(ei, ew):
            _, g = O.glm_matvec(O.BF16, I, H, w["gate"][e * eb:(e + 1) * eb], x[t])
            _, u = O.glm_matvec(O.BF16, I, H, w["up"][e * eb:(e + 1) * eb], x[t])
            h = np.array([np.float32(O.lib().dmo_glm_cached_silu(a)) * b for a, b in zip(g, u)], np.float32)
            _, o = O.glm_matvec(O.BF16, H, I, w["down"][e * eb:(e + 1) * eb], h)
            out = (out + (o * we).astype(np.float32) * np.float32(2.5)).astype(np.float32)
        _, g = O.glm_matvec(O.BF16, I, H, w["shared_gate"], x[t])
        _, u = O.glm_matvec(O.BF16, I, H, w["shared_up"], x[t])
        h = np.array([np.float32(O.lib().dmo_glm_silu(a)) * b for a, b in zip(g, u)], np.float32)
        _, o = O.glm_matvec(O.BF16, H, I, w["shared_down"], h)
        out = (out + o).astype(np.float32)
        np.testing.assert_array_equal(y[t], out)


def test_group_limit_restricts_selection_to_kept_groups():
    rng = np.random.default_rng(0)
    E, G, KG, k = 32, 4, 2, 4
    logits = rng.standard_normal(E).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    rc, idx, w = O.glm_select(logits, bias, k, G, KG)
    assert rc == O.OK
    sig = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
    ch = sig + bias
    per = E // G
    gscore = [np.sort(ch[g * per:(g + 1) * per])[-2:].sum() for g in range(G)]
    kept = set(np.argsort(-np.array(gscore), kind="stable")[:KG].tolist())
    assert all(int(i) // per in kept for i in idx)
    assert abs(float(w.sum()) - 1.0) < 1e-6
    # one group == the reference's ungrouped selection
    rc1, idx1, _ = O.glm_select(logits, bias, k, 1, 1)
    order = sorted(range(E), key=lambda e: (-np.float32(ch[e]), e))
    assert idx1.tolist() == order[:k]


def test_dispatch_is_a_stable_counting_sort():
    rng = np.random.default_rng(1)
    T, k, E = 50, 4, 9
    sel = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.uint32)
    rc, counts, offsets, sorted_pairs, inverse = O.dispatch(sel, E)
    assert rc == O.OK
    assert counts.tolist() == np.bincount(sel.ravel(), minlength=E).tolist()
    flat = sel.ravel()
    expect = sorted(range(T * k), key=lambda p: (flat[p], p))
    assert sorted_pairs.tolist() == expect
    assert all(sorted_pairs[inverse[p]] == p for p in range(T * k))
    assert offsets[-1] == T * k


@pytest.mark.parametrize("name", ["qwen35-small"])
def test_qwen_block_runs_and_is_deterministic(name):
    hl = HostLayer(name)
    w = hl.weights()
    x = hl.x(4)
    rc, y1, i1, p1 = O.qwen_moe(w, x, threads=4)
    rc2, y2, i2, p2 = O.qwen_moe(w, x, threads=1)
    assert rc == rc2 == O.OK
    assert np.array_equal(y1, y2) and np.array_equal(i1, i2)
    assert np.all(np.isfinite(y1)) and np.allclose(p1.sum(axis=1), 1.0, atol=1e-6)


@pytest.mark.parametrize("name", ["gemma4-small", "qwen35-small", "qwen35-odd", "glm52-small",
                                  "glm52-small-flat"])
def test_route_alone_selects_what_the_whole_block_selects(name):
    # oracle.route is the router + top-k of the block, run without any expert weights;
    # the full-size GPU parity tests compare every token's selection against it
    hl = HostLayer(name, seed=4)
    x = hl.x(40, seed=9)
    fam = hl.cfg["family"]
    block = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe, "glm52": O.glm_moe}[fam]
    rc, _, idx, wt = block(hl.weights(), x, threads=4)
    assert rc == O.OK
    rc, idx2, wt2 = O.route(fam, hl.sl.host_weights(router_only=True), x, threads=4)
    assert rc == O.OK
    assert np.array_equal(idx, idx2)
    assert np.array_equal(wt, wt2)
