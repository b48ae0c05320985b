"""Pin the CPU oracle against the reference's own known-answer tests.

Each test restates one `#[test]` of the DiskMule Rust tree (cited by file:line)
and checks the C oracle produces the same values.
"""
import struct

import numpy as np
import pytest

from oracle import oracle as O


def f16le(bits):
    return struct.pack("<H", bits)


def test_decodes_f32_and_f16_values():
    # src/cpu.rs:671-688
    enc = struct.pack("<2f", 1.25, -2.5)
    rc, out = O.dequantize(O.F32, enc, 2)
    assert rc == O.OK and out.tolist() == [1.25, -2.5]
    enc = b"".join(f16le(b) for b in (0x3C00, 0xC000, 0x0001))
    rc, out = O.dequantize(O.F16, enc, 3)
    assert rc == O.OK and out.tolist() == [1.0, -2.0, 2.0 ** -24]


def test_decodes_q5_0_high_bits_and_nibbles():
    # src/cpu.rs:690-700
    block = bytearray(22)
    block[0:2] = f16le(0x4000)
    block[2:6] = b"\xff" * 4
    block[6:] = b"\x10" * 16
    rc, out = O.dequantize(O.Q5_0, bytes(block), 32)
    assert rc == O.OK
    assert out[:16].tolist() == [0.0] * 16
    assert out[16:].tolist() == [2.0] * 16


def test_decodes_q8_0_signed_values():
    # src/cpu.rs:702-714
    block = bytearray(34)
    block[0:2] = f16le(0x3800)
    for i in range(32):
        block[2 + i] = (i - 16) & 0xFF
    rc, out = O.dequantize(O.Q8_0, bytes(block), 32)
    assert rc == O.OK
    assert out.tolist() == [(i - 16.0) * 0.5 for i in range(32)]


def test_decodes_q4_k_group_scales_and_minima():
    # src/cpu.rs:716-731
    block = bytearray(144)
    block[0:2] = f16le(0x3800)
    block[2:4] = f16le(0x3400)
    block[4:8] = b"\x01" * 4
    block[8:12] = b"\x02" * 4
    block[12:16] = b"\x21" * 4
    block[16:] = b"\x30" * 128
    rc, out = O.dequantize(O.Q4_K, bytes(block), 256)
    assert rc == O.OK
    for g in range(4):
        assert out[64 * g:64 * g + 32].tolist() == [-0.5] * 32
        assert out[64 * g + 32:64 * g + 64].tolist() == [1.0] * 32


def test_unpacks_q4_k_high_scale_and_minimum_bits():
    # src/cpu.rs:733-740
    scales = bytearray(12)
    scales[0] = 0b1100_0000
    scales[4] = 0b1000_0000
    scales[8] = 0b1010_0001
    assert O.scale_min_q4_k(4, bytes(scales)) == (49, 42)


def test_decodes_q6_k_six_bit_groups():
    # src/cpu.rs:742-754
    block = bytearray(210)
    for i in range(16):
        block[192 + i] = i + 1
    block[208:210] = f16le(0x3800)
    rc, out = O.dequantize(O.Q6_K, bytes(block), 256)
    assert rc == O.OK
    for g in range(16):
        assert out[16 * g:16 * g + 16].tolist() == [-16.0 * (g + 1)] * 16


def test_matvec_uses_row_major_tensor_layout():
    # src/cpu.rs:756-765
    enc = struct.pack("<4f", 1.0, 2.0, 3.0, 4.0)
    rc, out = O.matvec(O.F32, 2, 2, enc, [0.5, -1.0])
    assert rc == O.OK and out.tolist() == [-1.5, -2.5]


def test_rejects_bad_lengths_and_unsupported_types():
    # src/cpu.rs:767-777
    rc, _ = O.dequantize(O.Q4_K, bytes(144), 32)
    assert rc == O.ERR_ELEMENT_COUNT
    rc, _ = O.dequantize(O.Q5_K, b"", 0)
    assert rc == O.ERR_UNSUPPORTED
    # matvec validation order (src/cpu.rs:354-383)
    rc, _ = O.matvec(O.F32, 2, 2, bytes(16), [1.0])
    assert rc == O.ERR_INPUT_LENGTH
    rc, _ = O.matvec(O.F32, 2, 2, bytes(16), [1.0, 2.0], out_len=3)
    assert rc == O.ERR_OUTPUT_LENGTH
    rc, _ = O.matvec(O.F32, 2, 2, bytes(12), [1.0, 2.0])
    assert rc == O.ERR_BYTE_LENGTH


def test_normalizes_weighted_and_unweighted_vectors():
    # src/cpu.rs:779-796
    x = np.array([3.0, 4.0], dtype=np.float32)
    rc, out = O.rms_norm(x, None, 1e-6)
    inv = np.float32(1.0) / np.sqrt(np.float32(12.5) + np.float32(1e-6))
    assert rc == O.OK
    assert out.tolist() == [np.float32(3.0) * inv, np.float32(4.0) * inv]
    rc, out = O.rms_norm(x, np.array([2.0, 0.5], dtype=np.float32), 1e-6)
    assert out.tolist() == [np.float32(6.0) * inv, np.float32(2.0) * inv]


def test_applies_gemma_gelu():
    # src/cpu.rs:798-807 (the gelu half; softcap is not on the MoE path)
    assert O.gelu_tanh(0.0) == 0.0
    assert abs(O.gelu_tanh(1.0) - 0.841192) < 1e-6


def test_softmax_and_top_k_are_stable_and_deterministic():
    # src/cpu.rs:820-834
    rc, p = O.softmax([1000.0, 999.0, float("-inf")])
    assert rc == O.OK
    assert abs(float(p.sum()) - 1.0) < 1e-6
    assert p[2] == 0.0
    rc, idx, prob = O.top_k_softmax([2.0, 3.0, 3.0, 0.0], 2)
    assert rc == O.OK
    assert idx.tolist() == [1, 2] and prob.tolist() == [0.5, 0.5]
    rc, i = O.argmax([1.0, 4.0, 4.0])
    assert rc == O.OK and i == 1
    rc, _, _ = O.top_k_softmax([1.0], 0)
    assert rc == O.ERR_TOPK


def test_top_k_rejects_non_finite_and_orders_negative_zero():
    # src/cpu.rs:240-252: non-finite logits are an error; total_cmp puts -0.0 below +0.0
    rc, _, _ = O.top_k_softmax([1.0, float("nan")], 1)
    assert rc == O.ERR_NONFINITE
    rc, idx, _ = O.top_k_softmax([-0.0, 0.0, -1.0], 2)
    assert rc == O.OK and idx.tolist() == [1, 0]


# ---- Metal parity fixtures (src/metal.rs:2052-2142), CPU side only ----------

def metal_matvec_fixture(kind, rows):
    """Byte patterns of src/metal.rs:2052-2142 (matvec_fixture)."""
    if kind == O.F32:
        cols = 64
        vals = [((i * 17) % 41) * 0.03125 - 0.625 for i in range(rows * cols)]
        return cols, struct.pack(f"<{len(vals)}f", *vals)
    if kind == O.F16:
        cols = 64
        pats = [0x3000, 0xB400, 0x3800, 0xBC00, 0x3C00, 0x4000]
        return cols, b"".join(f16le(pats[i % 6]) for i in range(rows * cols))
    enc = bytearray()
    if kind == O.Q5_0:
        for r in range(rows):
            for b in range(3):
                blk = bytearray(22)
                blk[0:2] = f16le(0x3400)
                for i in range(20):
                    blk[2 + i] = (i * 29 + r * 47 + b * 13 + 3) & 0xFF
                enc += blk
        return 96, bytes(enc)
    if kind == O.Q8_0:
        for r in range(rows):
            for b in range(3):
                blk = bytearray(34)
                blk[0:2] = f16le(0x3000)
                for i in range(32):
                    v = i * 7 - 101 + r * 11 + b * 17
                    blk[2 + i] = ((v + 0x8000) & 0xFF)  # i16 -> i8 -> u8 truncation
                enc += blk
        return 96, bytes(enc)
    if kind == O.Q4_K:
        for r in range(rows):
            for b in range(3):
                blk = bytearray(144)
                blk[0:2] = f16le(0x3000)
                blk[2:4] = f16le(0x2800)
                for i in range(140):
                    blk[4 + i] = (i * 19 + r * 31 + b * 43 + 5) & 0xFF
                enc += blk
        return 768, bytes(enc)
    if kind == O.Q6_K:
        for r in range(rows):
            for b in range(3):
                blk = bytearray(210)
                for i in range(192):
                    blk[i] = (i * 23 + r * 37 + b * 41 + 11) & 0xFF
                for i in range(16):
                    blk[192 + i] = (i * 5 - 37 + r * 3 + b * 7) & 0xFF
                blk[208:210] = f16le(0x2800)
                enc += blk
        return 768, bytes(enc)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", [O.F32, O.F16, O.Q5_0, O.Q8_0, O.Q4_K, O.Q6_K])
def test_metal_fixture_matvec_matches_f64_dot_of_dequantized_rows(kind):
    # The reference's Metal-vs-CPU fixture (src/metal.rs:2223-2245) with its
    # input pattern; the oracle's fma chain agrees with an f64 dot of its own
    # dequantized rows within assert_close_relative (src/metal.rs:2041-2050).
    rows = 3
    cols, enc = metal_matvec_fixture(kind, rows)
    x = np.array([((i * 11 % 53) - 26.0) * 0.0078125 for i in range(cols)], dtype=np.float32)
    rc, out = O.matvec(kind, rows, cols, enc, x)
    assert rc == O.OK
    rb = len(enc) // rows
    for r in range(rows):
        rc, w = O.dequantize(kind, enc[r * rb:(r + 1) * rb], cols)
        assert rc == O.OK
        exp = float(np.dot(w.astype(np.float64), x.astype(np.float64)))
        tol = max(5e-4, abs(exp) * 2e-5)
        assert abs(out[r] - exp) <= tol


def test_matvec_is_a_sequential_fma_chain():
    # src/cpu.rs:389-397: the row result is fold(0, |s,(w,x)| w.mul_add(x, s)).
    rng = np.random.default_rng(5)
    cols = 300
    w = rng.standard_normal(cols).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    rc, out = O.matvec(O.F32, 1, cols, w.tobytes(), x)
    s = np.float32(0.0)
    for a, b in zip(w.astype(np.float64), x.astype(np.float64)):
        s = np.float32(a * b + np.float64(s))  # exact product + one rounding == fmaf
    assert rc == O.OK and out[0] == s


# ---- expert residency counters ------------------------------------------------

def test_gemma_cache_counters_match_reference_fixture():
    # src/expert.rs:266-325: 2 experts, 1 slot, 4+4 byte slices.
    lru = O.Lru(layers=1, experts=2, slots=1, global_clock=0, expert_bytes=8, reads_per_miss=2)
    assert lru.acquire(0, 0)[0] == O.OK
    assert lru.acquire(0, 0)[0] == O.OK
    assert lru.acquire(0, 1)[0] == O.OK
    s = lru.stats()
    assert (s["hits"], s["misses"], s["evictions"], s["reads"], s["bytes_read"],
            s["resident_bytes"]) == (1, 2, 1, 4, 16, 8)


def test_glm_cache_counters_match_reference_fixture():
    # src/glm52/expert.rs:555-595: one slot, dense gate/up/down -> 3 reads per miss.
    lru = O.Lru(layers=2, experts=2, slots=1, global_clock=1, expert_bytes=96, reads_per_miss=3)
    for _ in range(2):
        assert lru.acquire(1, 0)[0] == O.OK
    assert lru.acquire(1, 1)[0] == O.OK
    s = lru.stats()
    assert (s["hits"], s["misses"], s["evictions"], s["reads"]) == (1, 2, 1, 6)
    assert s["bytes_read"] > 0 and s["resident_bytes"] > 0


def test_gemma_cache_skips_pinned_slots_and_reports_all_pinned():
    # src/expert.rs:195-202: pinned slots are not victims; none eligible -> AllSlotsPinned
    lru = O.Lru(layers=1, experts=4, slots=2, global_clock=0, expert_bytes=8, reads_per_miss=2)
    assert lru.acquire(0, 0)[1] == 0
    assert lru.acquire(0, 1)[1] == 1
    lru.set_pinned(0, 0, True)
    rc, slot, miss = lru.acquire(0, 2)
    assert rc == O.OK and slot == 1 and miss
    lru.set_pinned(0, 1, True)
    rc, _, _ = lru.acquire(0, 3)
    assert rc == O.ERR_ALL_PINNED
    rc, _, _ = lru.acquire(0, 9)
    assert rc == O.ERR_EXPERT
