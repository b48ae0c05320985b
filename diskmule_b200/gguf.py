"""GGUF expert-slice loading over the C ABI (include/diskmule_gguf.h).

`TensorSource` mirrors the reference's reader of the same name (src/gguf.rs:610-723):
open a file, index it with the reference's limits and checks, look tensors up by name,
borrow their bytes from the read-only mapping, read bounded ranges. `ExpertLayerLayout`
is the per-expert byte layout the reference's expert cache uses (src/expert.rs:44-51).
`moe_layer_from_gguf` maps one layer's router and expert tensors into device memory and
builds the batched MoE layer over them, following the tensor names the reference loads
(src/gemma4.rs:346-406 for Gemma; the llama.cpp MoE names for separate gate / up / down
experts with a shared expert). `write_gguf` writes a version-3 file the way the
reference's own tests build their fixtures (src/gguf.rs:1429-1477).
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass

import numpy as np

from . import _native as N
from ._native import DmError, check


class TensorInfoC(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("type", C.c_int32), ("offset", C.c_uint64), ("absolute_offset", C.c_uint64),
                ("byte_len", C.c_uint64)]


class ExpertLayoutC(C.Structure):
    _fields_ = [("expert_count", C.c_int32), ("gate_up_offset", C.c_uint64),
                ("gate_up_bytes", C.c_uint64), ("down_offset", C.c_uint64),
                ("down_bytes", C.c_uint64)]


@dataclass
class TensorInfo:
    name: str
    dimensions: list
    kind: int
    offset: int
    absolute_offset: int
    byte_len: int


@dataclass
class ExpertLayerLayout:
    expert_count: int
    gate_up_offset: int
    gate_up_bytes: int
    down_offset: int
    down_bytes: int


class TensorSource:
    """An indexed GGUF file (TensorSource::open_with_arrays)."""

    def __init__(self, handle, path):
        self._h = handle
        self.path = path
        v, a, d, n = C.c_uint32(), C.c_uint32(), C.c_uint64(), C.c_uint64()
        check(N.lib().dm_gguf_header(self._h, C.byref(v), C.byref(a), C.byref(d), C.byref(n)))
        self.version, self.alignment = v.value, a.value
        self.data_offset, self.file_len = d.value, n.value

    @classmethod
    def open(cls, path: str, capture_arrays=()):
        h = C.c_void_p()
        keys = "\n".join(capture_arrays).encode() if capture_arrays else None
        check(N.lib().dm_gguf_open(str(path).encode(), keys, C.byref(h)))
        return cls(h, str(path))

    @classmethod
    def parse(cls, data: bytes, capture_arrays=()):
        """Index an in-memory image (GgufFile::read_from over a cursor)."""
        h = C.c_void_p()
        keys = "\n".join(capture_arrays).encode() if capture_arrays else None
        buf = (C.c_uint8 * len(data)).from_buffer_copy(data) if data else None
        check(N.lib().dm_gguf_parse(buf, len(data), keys, C.byref(h)))
        return cls(h, "<memory>")

    def __len__(self):
        return N.lib().dm_gguf_tensor_count(self._h)

    def _info(self, i: int) -> TensorInfo:
        t = TensorInfoC()
        check(N.lib().dm_gguf_tensor(self._h, i, C.byref(t)))
        return TensorInfo(t.name.decode(), list(t.dims[:t.n_dims]), t.type, t.offset,
                          t.absolute_offset, t.byte_len)

    @property
    def tensors(self):
        return [self._info(i) for i in range(len(self))]

    def index_of(self, name: str):
        i = C.c_int64()
        rc = N.lib().dm_gguf_find_tensor(self._h, name.encode(), C.byref(i))
        return None if rc != N.OK else i.value

    def tensor(self, name: str):
        i = self.index_of(name)
        return None if i is None else self._info(i)

    def tensor_bytes_by_index(self, i: int):
        if i < 0 or i >= len(self):
            return None
        p, n = C.c_void_p(), C.c_uint64()
        check(N.lib().dm_gguf_tensor_bytes(self._h, i, C.byref(p), C.byref(n)))
        if n.value == 0:
            return np.zeros(0, np.uint8)
        arr = np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p.value))
        arr.flags.writeable = False
        return arr  # a view of the read-only mapping, valid while the source is open

    def tensor_bytes(self, name: str):
        i = self.index_of(name)
        return None if i is None else self.tensor_bytes_by_index(i)

    def read_tensor_at(self, name: str, offset: int, length: int) -> np.ndarray:
        out = np.empty(length, np.uint8)
        check(N.lib().dm_gguf_read_tensor_at(self._h, name.encode(), offset,
                                             out.ctypes.data_as(C.c_void_p), length))
        return out

    # metadata
    def metadata_type(self, key: str):
        t, e, n = C.c_uint32(), C.c_uint32(), C.c_uint64()
        rc = N.lib().dm_gguf_metadata_type(self._h, key.encode(), C.byref(t), C.byref(e),
                                           C.byref(n))
        return None if rc != N.OK else (t.value, e.value, n.value)

    def metadata_int(self, key: str):
        v = C.c_uint64()
        rc = N.lib().dm_gguf_metadata_u64(self._h, key.encode(), C.byref(v))
        return None if rc != N.OK else v.value

    def metadata_float(self, key: str):
        v = C.c_double()
        rc = N.lib().dm_gguf_metadata_f64(self._h, key.encode(), C.byref(v))
        return None if rc != N.OK else v.value

    def metadata_string(self, key: str):
        t = self.metadata_type(key)
        if t is None or t[0] != 8:
            return None
        buf = C.create_string_buffer(t[2] + 1)
        check(N.lib().dm_gguf_metadata_string(self._h, key.encode(), buf, t[2] + 1))
        return buf.value.decode()

    def metadata_array(self, key: str):
        """A captured array's values (numbers as a numpy array, strings as a list)."""
        e, n, p = C.c_uint32(), C.c_uint64(), C.c_void_p()
        rc = N.lib().dm_gguf_metadata_array(self._h, key.encode(), C.byref(e), C.byref(n),
                                            C.byref(p))
        if rc != N.OK:
            return None
        if e.value == 8:
            ptrs = (C.c_char_p * n.value).from_address(p.value) if n.value else []
            return [s.decode() for s in ptrs]
        dtype = {0: np.uint8, 1: np.int8, 2: np.uint16, 3: np.int16, 4: np.uint32, 5: np.int32,
                 6: np.float32, 7: np.bool_, 10: np.uint64, 11: np.int64, 12: np.float64}[e.value]
        count = n.value * np.dtype(dtype).itemsize
        raw = bytes((C.c_uint8 * count).from_address(p.value)) if count else b""
        return np.frombuffer(raw, dtype=dtype).copy()

    def architecture(self):
        return self.metadata_string("general.architecture")

    def name(self):
        return self.metadata_string("general.name")

    def file_type(self):
        return self.metadata_int("general.file_type")

    def expert_layout(self, gate_up: str, down: str, expert_count: int) -> ExpertLayerLayout:
        out = ExpertLayoutC()
        check(N.lib().dm_gguf_expert_layout(self._h, gate_up.encode(), down.encode(),
                                            expert_count, C.byref(out)))
        return ExpertLayerLayout(out.expert_count, out.gate_up_offset, out.gate_up_bytes,
                                 out.down_offset, out.down_bytes)

    def close(self):
        if self._h:
            N.lib().dm_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# writing (fixtures)
# ---------------------------------------------------------------------------

U32, I32, F32, STRING, ARRAY = 4, 5, 6, 8, 9


def _string(v: str) -> bytes:
    b = v.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, metadata: dict, tensors: list, alignment: int = 32) -> None:
    """A GGUF v3 file: `metadata` maps keys to (type, value) with type U32 / I32 / F32 /
    STRING, or (ARRAY, element_type, values); `tensors` holds (name, dims, ggml_type,
    bytes) with dims in GGUF order (first = contiguous). Offsets are aligned."""
    meta = dict(metadata)
    meta.setdefault("general.alignment", (U32, alignment))
    out = bytearray(b"GGUF")
    out += struct.pack("<IQQ", 3, len(tensors), len(meta))
    for key, spec in meta.items():
        out += _string(key)
        t = spec[0]
        out += struct.pack("<I", t)
        if t == U32:
            out += struct.pack("<I", spec[1])
        elif t == I32:
            out += struct.pack("<i", spec[1])
        elif t == F32:
            out += struct.pack("<f", spec[1])
        elif t == STRING:
            out += _string(spec[1])
        elif t == ARRAY:
            et, values = spec[1], spec[2]
            out += struct.pack("<IQ", et, len(values))
            for v in values:
                out += _string(v) if et == STRING else struct.pack(
                    {U32: "<I", I32: "<i", F32: "<f"}[et], v)
        else:
            raise ValueError(f"metadata type {t}")
    offsets, off = [], 0
    for name, dims, kind, data in tensors:
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        off += len(data)
    for (name, dims, kind, data), o in zip(tensors, offsets):
        out += _string(name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", kind, o)
    out += b"\0" * ((-len(out)) % alignment)
    base = len(out)
    for (name, dims, kind, data), o in zip(tensors, offsets):
        out += b"\0" * (base + o - len(out))
        out += bytes(data)
    with open(path, "wb") as f:
        f.write(out)


# ---------------------------------------------------------------------------
# the MoE layer over a file's tensors
# ---------------------------------------------------------------------------

GEMMA_NAMES = {"router": "ffn_gate_inp.weight", "router_scale": "ffn_gate_inp.scale",
               "routed_pre_norm": "pre_ffw_norm_2.weight", "gate_up": "ffn_gate_up_exps.weight",
               "down": "ffn_down_exps.weight", "expert_scale": "ffn_down_exps.scale"}
SPLIT_NAMES = {"router": "ffn_gate_inp.weight", "gate": "ffn_gate_exps.weight",
               "up": "ffn_up_exps.weight", "down": "ffn_down_exps.weight",
               "shared_gate": "ffn_gate_shexp.weight", "shared_up": "ffn_up_shexp.weight",
               "shared_down": "ffn_down_shexp.weight",
               "shared_gate_vector": "ffn_gate_inp_shexp.weight",
               "correction_bias": "exp_probs_b.bias"}


class GgufMoeLayer:
    """A MoeLayer whose weights are the device copies of one GGUF layer's tensors."""

    def __init__(self, ctx, layer, buffers, layout, cfg):
        self.ctx, self.layer, self.buffers, self.layout, self.cfg = ctx, layer, buffers, layout, cfg

    def close(self):
        if self.layer is not None:
            self.layer.close()
            self.layer = None
        for b in self.buffers.values():
            b.free()
        self.buffers.clear()


def moe_layer_from_gguf(ctx, source: TensorSource, block: int, family: str, top_k: int,
                        epsilon: float = 1e-6, n_groups: int = 1, topk_groups: int = 1,
                        routed_scale: float = 1.0, normalize: bool = False) -> GgufMoeLayer:
    """Map layer `block`'s router and expert tensors (`blk.{block}.*`) into device memory
    and build the MoE layer over them. family: "gemma4" (fused gate_up experts, router
    and norm scales, per-expert down scale), "qwen35" (separate gate / up / down experts,
    sigmoid-gated shared expert) or "glm52" (separate experts, correction bias, shared
    expert). Expert tensors are copied to HBM once, in their file layout."""
    from .moe import MoeLayer
    names = GEMMA_NAMES if family == "gemma4" else SPLIT_NAMES
    pre = f"blk.{block}."
    info = {k: source.tensor(pre + v) for k, v in names.items()}
    for k in ("router", "down") + (("gate_up",) if family == "gemma4" else ("gate", "up")):
        if info[k] is None:
            raise DmError(N.ERR_FORMAT, f"tensor {pre + names[k]!r} was not found in the GGUF index")
    down = info["down"]
    I, H, E = down.dimensions[0], down.dimensions[1], down.dimensions[2]
    router = info["router"]
    if router.dimensions != [H, E]:
        raise DmError(N.ERR_FORMAT, f"router dimensions {router.dimensions} differ from [{H}, {E}]")
    buffers = {}

    def upload(key):
        t = info.get(key)
        if t is None:
            return None
        buf = ctx.map_read_only(source.tensor_bytes(t.name))
        buffers[key] = buf
        return buf.device_pointer

    d = N.MoeDesc()
    d.family = {"gemma4": N.FAMILY_GEMMA4, "qwen35": N.FAMILY_QWEN35_MOE,
                "glm52": N.FAMILY_GLM52}[family]
    d.hidden, d.intermediate, d.experts, d.top_k = H, I, E, top_k
    d.n_groups, d.topk_groups = n_groups, topk_groups
    d.normalize_topk = int(normalize)
    d.routed_scale = routed_scale
    d.epsilon = epsilon
    glm = family == "glm52"
    d.input_type = N.BF16 if glm else N.F32
    d.router_type = router.kind
    d.router = upload("router")
    d.down_type = down.kind
    d.down = upload("down")
    if family == "gemma4":
        gu = info["gate_up"]
        layout = source.expert_layout(gu.name, down.name, E)
        d.gate_type = d.up_type = gu.kind
        d.gate = upload("gate_up")
        d.up = None
        d.router_scale = upload("router_scale")
        d.routed_pre_norm = upload("routed_pre_norm")
        d.expert_scale = upload("expert_scale")
    else:
        layout = source.expert_layout(info["gate"].name, down.name, E)
        d.gate_type, d.up_type = info["gate"].kind, info["up"].kind
        d.gate = upload("gate")
        d.up = upload("up")
        if info.get("shared_gate") is not None:
            d.shared_intermediate = info["shared_gate"].dimensions[1]
            d.shared_gate = upload("shared_gate")
            d.shared_up = upload("shared_up")
            d.shared_down = upload("shared_down")
            d.shared_gate_vector = upload("shared_gate_vector")
        d.correction_bias = upload("correction_bias")
    ctx.synchronize()
    layer = MoeLayer(ctx, d)
    cfg = dict(family=family, hidden=H, intermediate=I, experts=E, top_k=top_k)
    return GgufMoeLayer(ctx, layer, buffers, layout, cfg)
