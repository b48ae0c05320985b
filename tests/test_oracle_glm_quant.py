"""The oracle's GLM-5.2 checkpoint encodings against the reference's known answers.

src/glm52/cpu.rs:1519-1547 (fp8 block scales), :1551-1601 (int8 rows, grouped int4, an
unresolvable U8 layout) and src/metal.rs:2315-2400 (fp8 matvec values 265 / 661).
"""
import numpy as np

from oracle import oracle as O


def test_fp8_applies_scales_per_128_by_128_block():
    w = np.full(129 * 130, 0x38, np.uint8)
    w[128 * 130 + 129] = 0xB8
    rc, row = O.glm_quant_row(True, 129, 130, w, [2.0, 3.0, 5.0, 7.0], 128)
    assert rc == O.OK
    assert row[0] == 5.0 and row[127] == 5.0 and row[128] == 7.0 and row[129] == -7.0


def test_fp8_matvec_matches_the_metal_fixture_values():
    w = np.full(129 * 130, 0x38, np.uint8)
    x = np.ones(130, np.float32)
    x[129] = 2.0
    rc, y = O.glm_quant_matvec(True, 129, 130, w, [2.0, 3.0, 5.0, 7.0], x)
    assert rc == O.OK
    np.testing.assert_allclose(y[:128], 265.0, rtol=0, atol=1e-5)
    assert abs(y[128] - 661.0) < 1e-5


def test_fp8_decoder_and_invalid_codes():
    assert O.f8_e4m3fn(0x38) == 1.0 and O.f8_e4m3fn(0xB8) == -1.0
    assert O.f8_e4m3fn(0x01) == 2.0 ** -9           # smallest subnormal
    assert O.f8_e4m3fn(0x7E) == 448.0                # largest finite
    assert O.f8_e4m3fn(0x7F) is None and O.f8_e4m3fn(0xFF) is None


def test_int8_rows_and_grouped_int4():
    i8 = np.array([-127, 0, 127, -2, 3, 4], np.int8).view(np.uint8)
    rc, y = O.glm_quant_matvec(False, 2, 3, i8, [0.1, 0.5], [1.0, 2.0, -1.0])
    assert rc == O.OK and np.array_equal(y, np.array([-25.4, 0.0], np.float32))
    rc, row = O.glm_quant_row(False, 2, 3, i8, [0.1, 0.5], 1)
    assert row.tolist() == [-1.0, 1.5, 2.0]
    i4 = np.array([0x40, 0xC8, 0x0F, 0xA9, 0xCB, 0x0D], np.uint8)
    rc, y = O.glm_quant_matvec(False, 2, 5, i4, [0.5, 2.0], [1.0] * 5)
    assert rc == O.OK and y.tolist() == [-0.5, 30.0]
    rc, row = O.glm_quant_row(False, 2, 5, i4, [0.5, 2.0], 0)
    assert row.tolist() == [-4.0, -2.0, 0.0, 2.0, 3.5]


def test_unresolvable_u8_layout_is_refused():
    assert O.glm_u8_encoding(1, 256, 196, 1) is None
    assert O.glm_u8_encoding(2, 300, 2 * 150, 2 * 2) == (2, 192)  # first group size that fits
