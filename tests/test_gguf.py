"""GGUF index and expert slices (host code of the CUDA library; no GPU needed).

The fixtures are built the way the reference's own tests build theirs
(src/gguf.rs:1153-1191, :1429-1477) and every case restates one of those tests
(src/gguf.rs:1193-1426): the valid index, malformed and truncated metadata, invalid
alignment, tensor-size overflow, misaligned and out-of-bounds tensors, unknown types and
bad block shapes, truncated arrays, captured arrays, and bounded tensor reads. The error
texts are the reference's GgufError messages.
"""
import struct
import threading

import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200._native import DmError
from diskmule_b200.gguf import TensorSource, write_gguf

I32_T, U32_T, STRING_T, ARRAY_T = 5, 4, 8, 9


def put_u32(b, v):
    b += struct.pack("<I", v)


def put_u64(b, v):
    b += struct.pack("<Q", v)


def put_string(b, v):
    put_u64(b, len(v.encode()))
    b += v.encode()


def put_u32_metadata(b, key, v):
    put_string(b, key)
    put_u32(b, U32_T)
    put_u32(b, v)


def put_string_metadata(b, key, v):
    put_string(b, key)
    put_u32(b, STRING_T)
    put_string(b, v)


def pad_to(b, a):
    b += b"\0" * ((a - len(b) % a) % a)


def valid_fixture() -> bytearray:
    """One Q4_0 tensor [32, 1] of 18 bytes and four metadata entries."""
    b = bytearray(b"GGUF")
    put_u32(b, 3)
    put_u64(b, 1)
    put_u64(b, 4)
    put_string_metadata(b, "general.architecture", "gemma4")
    put_u32_metadata(b, "general.file_type", 15)
    put_u32_metadata(b, "general.alignment", 32)
    put_string_metadata(b, "general.name", "fixture")
    put_string(b, "weight")
    put_u32(b, 2)
    put_u64(b, 32)
    put_u64(b, 1)
    put_u32(b, 2)
    put_u64(b, 0)
    pad_to(b, 32)
    b += bytes(range(18))
    return b


def descriptor_start(b: bytes) -> int:
    """Byte offset of the tensor descriptor (the name length 6)."""
    return bytes(b).rindex(struct.pack("<Q", 6))


def parse_error(data) -> DmError:
    with pytest.raises(DmError) as e:
        TensorSource.parse(bytes(data))
    return e.value


def test_parses_valid_metadata_and_tensor_bounds():
    src = TensorSource.parse(bytes(valid_fixture()))
    assert src.version == 3 and src.alignment == 32
    assert src.architecture() == "gemma4"
    assert src.name() == "fixture"
    assert src.file_type() == 15
    ts = src.tensors
    assert len(ts) == 1
    assert ts[0].kind == 2  # Q4_0
    assert ts[0].dimensions == [32, 1]
    assert ts[0].byte_len == 18
    assert src.metadata_type("general.file_type") == (U32_T, 0, 1)


def test_rejects_malformed_and_truncated_metadata():
    bad_magic = valid_fixture()
    bad_magic[0] = ord("B")
    e = parse_error(bad_magic)
    assert e.status == N.ERR_FORMAT and "is not a GGUF file" in str(e)
    truncated = valid_fixture()[:28]
    e = parse_error(truncated)
    assert "GGUF is truncated at byte" in str(e)
    excessive = valid_fixture()
    excessive[16:24] = struct.pack("<Q", 2 ** 64 - 1)
    e = parse_error(excessive)
    assert str(e).startswith("metadata count") and "exceeds the inspection limit" in str(e)


def test_rejects_invalid_alignment():
    b = valid_fixture()
    key = b"general.alignment"
    pos = bytes(b).index(key) + len(key) + 4
    b[pos:pos + 4] = struct.pack("<I", 3)
    e = parse_error(b)
    assert "invalid general.alignment value 3" in str(e)


def test_rejects_tensor_math_overflow():
    b = valid_fixture()
    second = descriptor_start(b) + 8 + 6 + 4 + 8
    b[second:second + 8] = struct.pack("<Q", 2 ** 64 - 1)
    e = parse_error(b)
    assert e.status == N.ERR_OVERFLOW and "integer overflow" in str(e)


def test_rejects_misaligned_and_out_of_bounds_tensor_ranges():
    b = valid_fixture()
    off = descriptor_start(b) + 8 + 6 + 4 + 16 + 4
    mis = bytearray(b)
    mis[off:off + 8] = struct.pack("<Q", 1)
    assert "is not aligned to 32 bytes" in str(parse_error(mis))
    oob = bytearray(b)[:-1]
    assert "exceeds the" in str(parse_error(oob)) and "byte GGUF file" in str(parse_error(oob))


def test_rejects_unknown_tensor_types_and_bad_quantized_shapes():
    b = valid_fixture()
    d = descriptor_start(b)
    unknown = bytearray(b)
    unknown[d + 8 + 6 + 4 + 16:d + 8 + 6 + 4 + 20] = struct.pack("<I", 999)
    e = parse_error(unknown)
    assert e.status == N.ERR_UNSUPPORTED_TENSOR_TYPE and "type 999" in str(e)
    bad = bytearray(b)
    bad[d + 8 + 6 + 4:d + 8 + 6 + 4 + 8] = struct.pack("<Q", 31)
    assert "is not divisible by the 32-element block size for Q4_0" in str(parse_error(bad))


def test_rejects_truncated_array_values_without_allocating_the_array():
    b = bytearray(b"GGUF")
    put_u32(b, 3)
    put_u64(b, 0)
    put_u64(b, 1)
    put_string(b, "tokenizer.ggml.tokens")
    put_u32(b, ARRAY_T)
    put_u32(b, STRING_T)
    put_u64(b, 1)
    put_u64(b, 100)
    assert "GGUF is truncated" in str(parse_error(b))


def test_captures_only_requested_metadata_arrays():
    b = bytearray(b"GGUF")
    put_u32(b, 3)
    put_u64(b, 0)
    put_u64(b, 2)
    put_string(b, "tokenizer.ggml.tokens")
    put_u32(b, ARRAY_T)
    put_u32(b, STRING_T)
    put_u64(b, 2)
    put_string(b, "hello")
    put_string(b, " world")
    put_string(b, "tokenizer.ggml.token_type")
    put_u32(b, ARRAY_T)
    put_u32(b, I32_T)
    put_u64(b, 2)
    put_u32(b, 1)
    put_u32(b, 6)
    pad_to(b, 32)
    summary = TensorSource.parse(bytes(b))
    assert summary.metadata_type("tokenizer.ggml.tokens") == (ARRAY_T, STRING_T, 2)
    assert summary.metadata_array("tokenizer.ggml.tokens") is None
    captured = TensorSource.parse(bytes(b), capture_arrays=("tokenizer.ggml.tokens",
                                                            "tokenizer.ggml.token_type"))
    assert captured.metadata_array("tokenizer.ggml.tokens") == ["hello", " world"]
    assert captured.metadata_array("tokenizer.ggml.token_type").tolist() == [1, 6]


def test_tensor_source_reads_checked_ranges_concurrently(tmp_path):
    path = tmp_path / "fixture.gguf"
    path.write_bytes(bytes(valid_fixture()))
    src = TensorSource.open(str(path))
    assert src.path == str(path)
    assert src.tensor("weight").byte_len == 18
    assert src.tensor_bytes("weight").tolist() == list(range(18))
    assert src.tensor_bytes_by_index(1) is None
    errors = []

    def reader(offset, expected):
        try:
            assert src.read_tensor_at("weight", offset, len(expected)).tolist() == expected
        except Exception as e:  # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=reader, args=a) for a in ((0, [0, 1, 2, 3]),
                                                                  (10, [10, 11, 12, 13]))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors
    with pytest.raises(DmError) as e:
        src.read_tensor_at("missing", 0, 1)
    assert "was not found in the GGUF index" in str(e.value)
    with pytest.raises(DmError) as e:
        src.read_tensor_at("weight", 17, 2)
    assert "requested range 17..19 exceeds tensor" in str(e.value)
    src.close()


def test_missing_file_is_an_io_error(tmp_path):
    with pytest.raises(DmError) as e:
        TensorSource.open(str(tmp_path / "absent.gguf"))
    assert e.value.status == N.ERR_IO


def test_written_file_round_trips_and_expert_slices(tmp_path):
    """A Gemma-shaped expert layer written like a model file: the expert layout splits the
    fused tensors into equal per-expert slices at the tensors' absolute offsets
    (ExpertLayerLayout, bytes_per_expert), and a tensor whose bytes do not split over
    the experts is refused."""
    rng = np.random.default_rng(3)
    E, H, I = 4, 256, 64
    gu = rng.integers(0, 256, E * 2 * I * (H // 256) * 144, dtype=np.uint8)
    dn = rng.integers(0, 256, E * H * (I // 32) * 22, dtype=np.uint8)
    odd = rng.integers(0, 256, 3 * 18, dtype=np.uint8)
    path = tmp_path / "layer.gguf"
    write_gguf(str(path), {"general.architecture": (STRING_T, "gemma4")},
               [("blk.0.ffn_gate_up_exps.weight", [H, 2 * I, E], 12, gu.tobytes()),
                ("blk.0.ffn_down_exps.weight", [I, H, E], 6, dn.tobytes()),
                ("odd", [32, 3], 2, odd.tobytes())])
    src = TensorSource.open(str(path))
    lay = src.expert_layout("blk.0.ffn_gate_up_exps.weight", "blk.0.ffn_down_exps.weight", E)
    assert lay.gate_up_bytes * E == gu.size and lay.down_bytes * E == dn.size
    raw = path.read_bytes()
    for e in range(E):
        a = lay.gate_up_offset + e * lay.gate_up_bytes
        assert raw[a:a + lay.gate_up_bytes] == gu[e * lay.gate_up_bytes:(e + 1) * lay.gate_up_bytes].tobytes()
        b = lay.down_offset + e * lay.down_bytes
        assert raw[b:b + lay.down_bytes] == dn[e * lay.down_bytes:(e + 1) * lay.down_bytes].tobytes()
    with pytest.raises(DmError) as err:
        src.expert_layout("odd", "blk.0.ffn_down_exps.weight", 4)
    assert "is not divisible by 4 experts" in str(err.value)
    src.close()
