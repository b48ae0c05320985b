"""GPU operators with the Metal backend's surface against the CPU oracle.

Mirrors src/metal.rs:2150-2279 (gemma_primitives_match_the_cpu_reference,
encoded_matvec_kernels_match_the_cpu_reference, mapped_matvec_reads_a_nonzero_file_
offset_without_copying) with the reference's tolerances.
"""
import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200._native import DmError
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import TensorSpec
from oracle import oracle as O
from tests.test_oracle_golden import metal_matvec_fixture

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def assert_close_relative(actual, expected):
    # src/metal.rs:2041-2050
    tol = np.maximum(5e-4, np.abs(expected) * 2e-5)
    assert np.all(np.abs(actual - expected) <= tol)


def test_device_name(ctx):
    assert "B200" in ctx.device_name() or ctx.device_name()


@pytest.mark.parametrize("kind", [O.F32, O.F16, O.Q5_0, O.Q8_0, O.Q4_K, O.Q6_K])
def test_encoded_matvec_kernels_match_the_cpu_reference(ctx, kind):
    rows = 3
    cols, enc = metal_matvec_fixture(kind, rows)
    x = np.array([((i * 11 % 53) - 26.0) * 0.0078125 for i in range(cols)], dtype=np.float32)
    rc, expected = O.matvec(kind, rows, cols, enc, x)
    assert rc == O.OK
    actual = ctx.matvec(kind, rows, cols, enc, x)
    assert_close_relative(actual, expected)


@pytest.mark.parametrize("kind,cols", [(N.Q4_K, 2816), (N.Q6_K, 512), (N.Q5_0, 704),
                                       (N.Q8_0, 704), (N.BF16, 6144), (N.F32, 300)])
def test_random_matvec_matches_oracle(ctx, kind, cols):
    rows = 257
    enc = TensorSpec("m", kind, rows, cols, seed=5).host()
    x = TensorSpec("x", N.F32, 1, cols, seed=6, sigma=1.0).host().view(np.float32)
    if kind == N.BF16:
        rc, expected = O.glm_matvec(O.BF16, rows, cols, enc, x)
    else:
        rc, expected = O.matvec(kind, rows, cols, enc, x)
    assert rc == O.OK
    actual = ctx.matvec(kind, rows, cols, enc, x)
    err = np.linalg.norm(actual - expected) / np.linalg.norm(expected)
    assert err < 1e-5


def test_mapped_matvec_reads_a_nonzero_offset(ctx):
    enc = np.array([1.0, 2.0, 3.0, 4.0], dtype=np.float32).view(np.uint8)
    data = np.concatenate([np.zeros(32, np.uint8), enc])
    buf = ctx.map_read_only(data)
    out = ctx.matvec_mapped(N.F32, 2, 2, buf, 32, enc.size, [0.5, -1.0])
    assert out.tolist() == [-1.5, -2.5]
    with pytest.raises(N.DmError) as e:
        ctx.matvec_mapped(N.F32, 2, 2, buf, 40, enc.size, [0.5, -1.0])
    assert e.value.status == N.ERR_MAPPED_RANGE


def test_matvec_validation_order(ctx):
    with pytest.raises(N.DmError) as e:
        ctx.matvec(N.F32, 2, 2, bytes(16), [1.0])
    assert e.value.status == N.ERR_INPUT_LENGTH
    with pytest.raises(N.DmError) as e:
        ctx.matvec(N.Q4_K, 1, 32, bytes(144), np.zeros(32))
    assert e.value.status == N.ERR_ELEMENT_COUNT
    with pytest.raises(N.DmError) as e:
        ctx.matvec(N.F32, 2, 2, bytes(12), [1.0, 2.0])
    assert e.value.status == N.ERR_BYTE_LENGTH
    with pytest.raises(N.DmError) as e:
        ctx.matvec(13, 1, 256, bytes(176), np.zeros(256))
    assert e.value.status == N.ERR_UNSUPPORTED_TENSOR_TYPE


def test_gemma_primitives_match_the_cpu_reference(ctx):
    # src/metal.rs:2164-2221
    x = np.array([((i % 31) - 15.0) * 0.071 for i in range(513)], dtype=np.float32)
    w = np.array([0.8 + (i % 13) * 0.025 for i in range(513)], dtype=np.float32)
    rc, expected = O.rms_norm(x, w, 1e-6)
    actual = ctx.rms_norm(x, w, 1e-6)
    assert np.array_equal(actual, expected)  # same chain: bit-exact (reference bar 2e-6)
    gate = x[:67]
    up = (np.float32(1.25) - gate * np.float32(0.2)).astype(np.float32)
    exp_gelu = np.array([np.float32(O.gelu_tanh(g)) * u for g, u in zip(gate, up)], np.float32)
    assert np.max(np.abs(ctx.gelu_mul(gate, up) - exp_gelu)) <= 2e-6
    lg = np.array([-80.0, -51.0, 37.0, 66.0, 90.0], np.float32)
    lu = np.array([2.0, -3.0, 4.0, -5.0, 6.0], np.float32)
    exp_large = np.array([np.float32(O.gelu_tanh(g)) * u for g, u in zip(lg, lu)], np.float32)
    assert np.max(np.abs(ctx.gelu_mul(lg, lu) - exp_large)) <= 2e-5
    exp_silu = np.array([np.float32(O.lib().dmo_glm_cached_silu(g)) * u for g, u in zip(lg, lu)], np.float32)
    assert np.max(np.abs(ctx.silu_mul(lg, lu) - exp_silu)) <= 2e-5
    logits = [-2.0, 7.5, 4.0, 7.5, 0.0, 7.49]
    rc, ei, ep = O.top_k_softmax(logits, 4)
    got = ctx.top_k_softmax(logits, 4)
    assert [i for i, _ in got] == ei.tolist()
    assert np.max(np.abs(np.array([p for _, p in got]) - ep)) <= 2e-7


def test_top_k_softmax_large_and_errors(ctx):
    rng = np.random.default_rng(3)
    lg = rng.standard_normal(5000).astype(np.float32)
    lg[17] = lg[4000] = lg.max() + 1  # a tie at the top: lower index first
    rc, ei, ep = O.top_k_softmax(lg, 10)
    got = ctx.top_k_softmax(lg, 10)
    assert [i for i, _ in got] == ei.tolist() and got[0][0] == 17
    with pytest.raises(N.DmError) as e:
        ctx.top_k_softmax([1.0, 2.0], 3)
    assert e.value.status == N.ERR_TOP_K
    with pytest.raises(N.DmError) as e:
        ctx.top_k_softmax([1.0, np.nan], 1)
    assert e.value.status == N.ERR_NON_FINITE


@pytest.mark.parametrize("kind", [N.Q4_K, N.Q6_K, N.Q5_0, N.Q8_0, N.BF16, N.F32, N.F16])
def test_synthetic_device_bytes_equal_host_bytes(ctx, kind):
    spec = TensorSpec("t", kind, 64, 512, experts=3, seed=77, sigma=0.5)
    buf = ctx.new_owned_buffer(spec.nbytes)
    spec.device_fill(buf.device_pointer)
    ctx.synchronize()
    assert np.array_equal(buf.read(), spec.host())


# ---------------------------------------------------------------------------
# GLM-5.2 checkpoint encodings (dm_cuda_matvec_safetensor)
# ---------------------------------------------------------------------------

def _glm_quant_case(kind, rows, cols, group, rng):
    if kind == "fp8":
        enc = rng.integers(0, 256, rows * cols, dtype=np.uint8)
        enc[(enc & 0x7F) == 0x7F] = 0x38  # no invalid codes
        scales = rng.uniform(0.5, 2.0, ((rows + 127) // 128) * ((cols + 127) // 128)).astype(np.float32)
    elif kind == "i8":
        enc = rng.integers(0, 256, rows * cols, dtype=np.uint8)
        scales = rng.uniform(1e-3, 1e-2, rows).astype(np.float32)
    else:
        enc = rng.integers(0, 256, rows * ((cols + 1) // 2), dtype=np.uint8)
        scales = rng.uniform(1e-3, 1e-2, rows * ((cols + group - 1) // group)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    return enc, scales, x


def test_safetensor_matvec_known_answers(ctx):
    w = np.full(129 * 130, 0x38, np.uint8)
    x = np.ones(130, np.float32)
    x[129] = 2.0
    y = ctx.matvec_safetensor(N.F8_E4M3, 129, 130, w, [2.0, 3.0, 5.0, 7.0], x)
    np.testing.assert_allclose(y[:128], 265.0, atol=1e-5, rtol=0)
    assert abs(y[128] - 661.0) < 1e-5
    i8 = np.array([-127, 0, 127, -2, 3, 4], np.int8).view(np.uint8)
    np.testing.assert_allclose(ctx.matvec_safetensor(N.U8_QUANT, 2, 3, i8, [0.1, 0.5], [1, 2, -1]),
                               [-25.4, 0.0], atol=1e-5)
    i4 = np.array([0x40, 0xC8, 0x0F, 0xA9, 0xCB, 0x0D], np.uint8)
    np.testing.assert_allclose(ctx.matvec_safetensor(N.U8_QUANT, 2, 5, i4, [0.5, 2.0], [1] * 5),
                               [-0.5, 30.0], atol=1e-5)
    with pytest.raises(DmError) as e:
        ctx.matvec_safetensor(N.U8_QUANT, 1, 256, np.zeros(196, np.uint8), [6.0], np.ones(256))
    assert e.value.status == N.ERR_BYTE_LENGTH


@pytest.mark.parametrize("kind,rows,cols,group", [
    ("i8", 300, 2048, 0), ("i4", 257, 6144, 32), ("i4", 64, 1000, 128), ("i4", 33, 515, 16),
    ("fp8", 384, 2048, 0), ("fp8", 129, 300, 0)])
def test_safetensor_matvec_matches_the_oracle(ctx, kind, rows, cols, group):
    rng = np.random.default_rng(rows * 7 + cols)
    enc, scales, x = _glm_quant_case(kind, rows, cols, group, rng)
    dtype = N.F8_E4M3 if kind == "fp8" else N.U8_QUANT
    y = ctx.matvec_safetensor(dtype, rows, cols, enc, scales, x)
    rc, y_ref = O.glm_quant_matvec(kind == "fp8", rows, cols, enc, scales, x, threads=8)
    assert rc == O.OK
    # per row: |error| within 1e-5 of the row's sum of |w * x| (reordered f32 sums)
    mag = np.zeros(rows)
    for r in range(rows):
        _, row = O.glm_quant_row(kind == "fp8", rows, cols, enc, scales, r)
        mag[r] = np.abs(row.astype(np.float64) * x).sum()
    assert np.all(np.abs(y.astype(np.float64) - y_ref) <= 1e-5 * mag + 1e-30)
