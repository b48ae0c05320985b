"""Seeded synthetic tensors: determinism, slice independence and value ranges (CPU)."""
import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.synthetic import CONFIGS, TensorSpec, layer_specs, zipf_bias
from oracle import oracle as O


def test_same_seed_same_bytes_and_slices_match_the_whole():
    spec = TensorSpec("g", N.Q4_K, 8, 512, experts=4, seed=11)
    whole = spec.host()
    assert np.array_equal(whole, spec.host())
    for e in range(4):
        part = spec.host(e)
        assert np.array_equal(part, whole[e * spec.expert_bytes:(e + 1) * spec.expert_bytes])
    other = TensorSpec("g", N.Q4_K, 8, 512, experts=4, seed=12).host()
    assert not np.array_equal(whole, other)


@pytest.mark.parametrize("kind,offset", [(N.Q4_K, 0), (N.Q6_K, 208), (N.Q5_0, 0), (N.Q8_0, 0)])
def test_block_scales_are_f16_in_range(kind, offset):
    spec = TensorSpec("t", kind, 16, 256, seed=3)
    b = spec.host()
    bb = {N.Q4_K: 144, N.Q6_K: 210, N.Q5_0: 22, N.Q8_0: 34}[kind]
    blocks = b.reshape(-1, bb)
    d = np.array([O.f16_to_f32(int(x)) for x in blocks[:, offset:offset + 2].copy().view(np.uint16).ravel()])
    assert np.all(d >= 1e-3 * 0.999) and np.all(d <= 1e-2 * 1.001)
    if kind == N.Q4_K:
        dmin = np.array([O.f16_to_f32(int(x)) for x in blocks[:, 2:4].copy().view(np.uint16).ravel()])
        assert np.all(dmin >= 1e-3 * 0.999) and np.all(dmin <= 1e-2 * 1.001)


def test_dense_normal_moments():
    spec = TensorSpec("x", N.F32, 1, 200000, seed=5, sigma=1.0)
    v = spec.host().view(np.float32)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01
    bf = TensorSpec("w", N.BF16, 1, 100000, seed=5, sigma=0.02).host().view(np.uint16)
    f = (bf.astype(np.uint32) << 16).view(np.float32)
    assert abs(f.std() - 0.02) < 0.001


def test_config_shapes_match_the_benchmark_table():
    g = layer_specs(CONFIGS["gemma4"], 1)
    assert g["gate"].expert_bytes == 2_230_272          # 1408 rows x 1584 B
    assert g["down"].expert_bytes == 1_362_944          # Q5_0, 2816 rows x 484 B
    q = layer_specs(CONFIGS["qwen35"], 1)
    assert q["gate"].expert_bytes == 589_824 and q["down"].expert_bytes == 860_160
    m = layer_specs(CONFIGS["glm52"], 1)
    assert m["gate"].expert_bytes == 25_165_824


def test_zipf_bias_is_a_log_distribution():
    b = zipf_bias(128, 1.1, 3)
    assert np.isclose(np.exp(b.astype(np.float64)).sum(), 1.0, rtol=1e-5)
    assert b.max() > b.min() + 4


@pytest.mark.parametrize("name", ["glm52-small", "qwen35-small", "gemma4-small"])
def test_oracle_fill_equals_the_library_fill(name):
    """The CPU reference arm generates its inputs with the oracle library's copy of the
    generator (it never loads the CUDA library): the bytes must be the same."""
    from diskmule_b200.synthetic import input_spec
    cfg = CONFIGS[name]
    for key, spec in layer_specs(cfg, 4).items():
        assert np.array_equal(spec.host(), spec.host(fill=O.synth_fill)), key
        if spec.experts > 1:
            assert np.array_equal(spec.host(1), spec.host(1, O.synth_fill)), key
    x = input_spec(cfg, 7, 5)
    assert np.array_equal(x.host(), x.host(fill=O.synth_fill))
