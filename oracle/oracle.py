"""ctypes view of the CPU oracle (oracle/libdm_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arm of bench.py, never by the diskmule_b200 package.
The oracle restates DiskMule's Rust CPU path in C; see dm_oracle.c for the
reference file:line each function follows.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdm_oracle.so")

F32, F16, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 6, 8, 12, 13, 14, 30

OK = 0
ERR_UNSUPPORTED = -1
ERR_ELEMENT_COUNT = -2
ERR_BYTE_LENGTH = -3
ERR_INPUT_LENGTH = -4
ERR_OUTPUT_LENGTH = -5
ERR_EMPTY = -6
ERR_NONFINITE = -7
ERR_TOPK = -8
ERR_PARAM = -9
ERR_EXPERT = -11
ERR_LAYER = -12
ERR_ALL_PINNED = -13


def build() -> str:
    """Compile the oracle with its Makefile if the library is missing or stale."""
    srcs = [os.path.join(HERE, f) for f in ("dm_oracle.c", "dm_oracle.h", "dm_oracle_synth.cpp")]
    if not os.path.exists(LIB_PATH) or any(os.path.getmtime(LIB_PATH) < os.path.getmtime(f)
                                           for f in srcs if os.path.exists(f)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        _declare(_lib)
    return _lib


P = C.c_void_p
SZ = C.c_size_t
I32 = C.c_int32


def _declare(L):
    L.dmo_f16_to_f32.argtypes = [C.c_uint16]
    L.dmo_f16_to_f32.restype = C.c_float
    L.dmo_bf16_to_f32.argtypes = [C.c_uint16]
    L.dmo_bf16_to_f32.restype = C.c_float
    L.dmo_row_byte_len.argtypes = [C.c_int, C.c_uint64, C.POINTER(C.c_uint64)]
    L.dmo_scale_min_q4_k.argtypes = [C.c_int, P, C.POINTER(C.c_uint8), C.POINTER(C.c_uint8)]
    L.dmo_dequantize.argtypes = [C.c_int, P, SZ, P, SZ]
    L.dmo_matvec.argtypes = [C.c_int, SZ, SZ, P, SZ, P, SZ, P, SZ, C.c_int]
    L.dmo_rms_norm.argtypes = [P, P, SZ, C.c_float, P]
    L.dmo_gelu_tanh.argtypes = [C.c_float]
    L.dmo_gelu_tanh.restype = C.c_float
    L.dmo_softmax_in_place.argtypes = [P, SZ]
    L.dmo_top_k_softmax.argtypes = [P, SZ, SZ, P, P]
    L.dmo_argmax.argtypes = [P, SZ, C.POINTER(C.c_size_t)]
    L.dmo_glm_rms_norm.argtypes = [P, P, SZ, C.c_float, P]
    L.dmo_glm_matvec.argtypes = [C.c_int, SZ, SZ, P, P, P, C.c_int]
    for name in ("dmo_glm_sigmoid", "dmo_glm_silu", "dmo_glm_cached_silu",
                 "dmo_qwen_sigmoid", "dmo_qwen_silu"):
        getattr(L, name).argtypes = [C.c_float]
        getattr(L, name).restype = C.c_float
    L.dmo_glm_select.argtypes = [P, P, SZ, SZ, SZ, SZ, C.c_int, P, P]
    L.dmo_dispatch.argtypes = [P, SZ, SZ, SZ, P, P, P, P]
    L.dmo_gemma_moe.argtypes = [P, P, SZ, P, P, P, C.c_int]
    L.dmo_qwen_moe.argtypes = [P, P, SZ, P, P, P, C.c_int]
    L.dmo_glm_moe.argtypes = [P, P, SZ, P, P, P, C.c_int]
    L.dmo_gemma_route.argtypes = [P, P, SZ, P, P, C.c_int]
    L.dmo_qwen_route.argtypes = [P, P, SZ, P, P, C.c_int]
    L.dmo_glm_route.argtypes = [P, P, SZ, P, P, C.c_int]
    L.dmo_lru_create.argtypes = [I32, I32, I32, I32, C.c_uint64, I32]
    L.dmo_lru_create.restype = P
    L.dmo_lru_destroy.argtypes = [P]
    L.dmo_lru_acquire.argtypes = [P, I32, I32, C.POINTER(I32), C.POINTER(I32)]
    L.dmo_lru_set_pinned.argtypes = [P, I32, I32, I32]
    L.dmo_lru_stats.argtypes = [P, P]
    L.dmo_gemma_ffn_block.argtypes = [P, P, P, SZ, P, P, P, C.c_int]
    L.dmo_f8_e4m3fn.argtypes = [C.c_uint8, C.POINTER(C.c_float)]
    L.dmo_glm_u8_encoding.argtypes = [SZ, SZ, SZ, SZ, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.dmo_glm_quant_matvec.argtypes = [C.c_int, SZ, SZ, P, SZ, P, SZ, P, P, C.c_int]
    L.dmo_glm_quant_row.argtypes = [C.c_int, SZ, SZ, P, SZ, P, SZ, SZ, P]
    L.dmo_synth_fill.argtypes = [I32, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                                 C.c_float, P]
    L.dmo_synth_fill.restype = I32


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def synth_fill(kind: int, seed: int, first_block: int, n_blocks: int, sigma: float,
               lo: float, hi: float, block_bytes: int) -> np.ndarray:
    """Bytes of blocks [first_block, first_block + n_blocks) of a seeded synthetic tensor
    (the generator of include/diskmule_synth.h, evaluated in this library)."""
    out = np.empty(n_blocks * block_bytes, dtype=np.uint8)
    rc = lib().dmo_synth_fill(kind, seed, first_block, n_blocks, sigma, lo, hi, _ptr(out))
    if rc != OK:
        raise ValueError(f"synthetic fill of kind {kind} failed ({rc})")
    return out


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a):
    return np.ascontiguousarray(np.frombuffer(bytes(a), dtype=np.uint8) if isinstance(a, (bytes, bytearray)) else a, dtype=np.uint8)


def f16_to_f32(bits: int) -> float:
    return lib().dmo_f16_to_f32(bits)


def row_byte_len(kind: int, elements: int):
    out = C.c_uint64()
    rc = lib().dmo_row_byte_len(kind, elements, C.byref(out))
    return None if rc != OK else out.value


def scale_min_q4_k(index: int, scales) -> tuple[int, int]:
    s = _u8(scales)
    a, b = C.c_uint8(), C.c_uint8()
    lib().dmo_scale_min_q4_k(index, _ptr(s), C.byref(a), C.byref(b))
    return a.value, b.value


def dequantize(kind: int, encoded, n: int):
    enc = _u8(encoded)
    out = np.zeros(n, dtype=np.float32)
    rc = lib().dmo_dequantize(kind, _ptr(enc), enc.size, _ptr(out), n)
    return rc, out


def matvec(kind: int, rows: int, columns: int, encoded, x, threads: int = 1, out_len=None):
    enc = _u8(encoded)
    x = _f32(x)
    n_out = rows if out_len is None else out_len
    out = np.zeros(n_out, dtype=np.float32)
    rc = lib().dmo_matvec(kind, rows, columns, _ptr(enc), enc.size, _ptr(x), x.size,
                          _ptr(out), n_out, threads)
    return rc, out


def rms_norm(x, weight, eps):
    x = _f32(x)
    w = None if weight is None else _f32(weight)
    out = np.zeros_like(x)
    rc = lib().dmo_rms_norm(_ptr(x), _ptr(w), x.size, eps, _ptr(out))
    return rc, out


def glm_rms_norm(x, weight, eps):
    """src/glm52/cpu.rs:912-924 (f64 mean square)."""
    x = _f32(x)
    w = _f32(weight)
    out = np.zeros_like(x)
    rc = lib().dmo_glm_rms_norm(_ptr(x), _ptr(w), x.size, eps, _ptr(out))
    return rc, out


def gelu_tanh(v: float) -> float:
    return lib().dmo_gelu_tanh(v)


def softmax(values):
    v = _f32(values).copy()
    rc = lib().dmo_softmax_in_place(_ptr(v), v.size)
    return rc, v


def top_k_softmax(logits, k: int):
    lg = _f32(logits)
    idx = np.zeros(max(k, 1), dtype=np.uint32)
    prob = np.zeros(max(k, 1), dtype=np.float32)
    rc = lib().dmo_top_k_softmax(_ptr(lg), lg.size, k, _ptr(idx), _ptr(prob))
    return rc, idx[:k], prob[:k]


def argmax(values):
    v = _f32(values)
    out = C.c_size_t()
    rc = lib().dmo_argmax(_ptr(v), v.size, C.byref(out))
    return rc, out.value


def glm_matvec(kind: int, rows: int, columns: int, encoded, x, threads: int = 1):
    enc = _u8(encoded)
    x = _f32(x)
    out = np.zeros(rows, dtype=np.float32)
    rc = lib().dmo_glm_matvec(kind, rows, columns, _ptr(enc), _ptr(x), _ptr(out), threads)
    return rc, out


def f8_e4m3fn(byte: int):
    v = C.c_float()
    rc = lib().dmo_f8_e4m3fn(byte, C.byref(v))
    return None if rc != OK else v.value


def glm_u8_encoding(rows, columns, encoded_bytes, scales):
    """(1, 0) int8 rows, (2, group) int4 grouped, or None (src/glm52/quant.rs)."""
    k, g = C.c_int(), C.c_int()
    rc = lib().dmo_glm_u8_encoding(rows, columns, encoded_bytes, scales, C.byref(k), C.byref(g))
    return None if rc != OK else (k.value, g.value)


def glm_quant_matvec(fp8: bool, rows: int, columns: int, encoded, scales, x, threads: int = 1):
    enc = _u8(encoded)
    sc = _f32(scales)
    xv = _f32(x)
    out = np.zeros(rows, np.float32)
    rc = lib().dmo_glm_quant_matvec(int(fp8), rows, columns, _ptr(enc), enc.size, _ptr(sc),
                                    sc.size, _ptr(xv), _ptr(out), threads)
    return rc, out


def glm_quant_row(fp8: bool, rows: int, columns: int, encoded, scales, r: int):
    enc = _u8(encoded)
    sc = _f32(scales)
    out = np.zeros(columns, np.float32)
    rc = lib().dmo_glm_quant_row(int(fp8), rows, columns, _ptr(enc), enc.size, _ptr(sc), sc.size,
                                 r, _ptr(out))
    return rc, out


def glm_select(logits, bias, k, n_groups=1, topk_groups=1, normalize=True):
    lg, b = _f32(logits), _f32(bias)
    idx = np.zeros(k, dtype=np.uint32)
    w = np.zeros(k, dtype=np.float32)
    rc = lib().dmo_glm_select(_ptr(lg), _ptr(b), lg.size, k, n_groups, topk_groups,
                              int(normalize), _ptr(idx), _ptr(w))
    return rc, idx, w


def dispatch(selected, experts: int):
    sel = np.ascontiguousarray(selected, dtype=np.uint32)
    T, k = sel.shape
    counts = np.zeros(experts, dtype=np.int32)
    offsets = np.zeros(experts + 1, dtype=np.int32)
    sorted_pairs = np.zeros(T * k, dtype=np.int32)
    inverse = np.zeros(T * k, dtype=np.int32)
    rc = lib().dmo_dispatch(_ptr(sel), T, k, experts, _ptr(counts), _ptr(offsets),
                            _ptr(sorted_pairs), _ptr(inverse))
    return rc, counts, offsets, sorted_pairs, inverse


class GemmaLayer(C.Structure):
    _fields_ = [("hidden", I32), ("intermediate", I32), ("experts", I32), ("top_k", I32),
                ("epsilon", C.c_float), ("router", P), ("router_scale", P),
                ("routed_pre_norm", P), ("gate_up_type", I32), ("gate_up", P),
                ("down_type", I32), ("down", P), ("expert_scale", P),
                ("router_logit_bias", P)]


class GemmaFfn(C.Structure):
    _fields_ = [("width", I32), ("gate_type", I32), ("up_type", I32), ("down_type", I32),
                ("gate", P), ("up", P), ("down", P), ("feed_forward_norm", P),
                ("shared_post_norm", P), ("routed_post_norm", P),
                ("post_feed_forward_norm", P), ("layer_output_scale", C.c_float)]


class QwenLayer(C.Structure):
    _fields_ = [("hidden", I32), ("intermediate", I32), ("experts", I32), ("top_k", I32),
                ("router", P), ("gate_type", I32), ("up_type", I32), ("down_type", I32),
                ("gate", P), ("up", P), ("down", P), ("shared_intermediate", I32),
                ("shared_gate", P), ("shared_up", P), ("shared_down", P),
                ("shared_gate_vector", P), ("router_logit_bias", P)]


class GlmLayer(C.Structure):
    _fields_ = [("hidden", I32), ("intermediate", I32), ("experts", I32), ("top_k", I32),
                ("n_groups", I32), ("topk_groups", I32), ("normalize", I32),
                ("routed_scale", C.c_float), ("weight_type", I32), ("router", P),
                ("correction_bias", P), ("gate", P), ("up", P), ("down", P),
                ("shared_intermediate", I32), ("shared_gate", P), ("shared_up", P),
                ("shared_down", P), ("expert_blobs", C.POINTER(P))]


def _gemma_layer(w: dict, H: int):
    return GemmaLayer(H, w["intermediate"], w["experts"], w["top_k"], w.get("epsilon", 1e-6),
                      _ptr(w["router"]), _ptr(w["router_scale"]), _ptr(w["routed_pre_norm"]),
                      w["gate_up_type"], _ptr(w.get("gate_up")), w["down_type"],
                      _ptr(w.get("down")), _ptr(w["expert_scale"]),
                      _ptr(w.get("router_logit_bias")))


def gemma_moe(w: dict, x, threads: int = 1):
    """Gemma-4 routed branch (src/gemma4/cpu.rs:559-611). `w` holds numpy arrays."""
    x = _f32(x)
    T, H = x.shape
    k = w["top_k"]
    layer = _gemma_layer(w, H)
    y = np.zeros((T, H), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.uint32)
    prob = np.zeros((T, k), dtype=np.float32)
    rc = lib().dmo_gemma_moe(C.byref(layer), _ptr(x), T, _ptr(y), _ptr(idx), _ptr(prob), threads)
    return rc, y, idx, prob


def gemma_ffn_block(w: dict, f: dict, x, threads: int = 1):
    """Gemma-4 feed-forward block (src/gemma4/cpu.rs:547-620): the routed branch of `w`
    (as gemma_moe) plus the shared FFN, norms, residual and layer scale of `f`."""
    x = _f32(x)
    T, H = x.shape
    k = w["top_k"]
    layer = _gemma_layer(w, H)
    norms = {n: _f32(f[n]) for n in ("feed_forward_norm", "shared_post_norm", "routed_post_norm",
                                     "post_feed_forward_norm")}
    ffn = GemmaFfn(f["width"], f["gate_type"], f["up_type"], f["down_type"], _ptr(f["gate"]),
                   _ptr(f["up"]), _ptr(f["down"]), _ptr(norms["feed_forward_norm"]),
                   _ptr(norms["shared_post_norm"]), _ptr(norms["routed_post_norm"]),
                   _ptr(norms["post_feed_forward_norm"]), f["layer_output_scale"])
    y = np.zeros((T, H), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.uint32)
    prob = np.zeros((T, k), dtype=np.float32)
    rc = lib().dmo_gemma_ffn_block(C.byref(ffn), C.byref(layer), _ptr(x), T, _ptr(y), _ptr(idx),
                                   _ptr(prob), threads)
    return rc, y, idx, prob


def _qwen_layer(w: dict, H: int):
    return QwenLayer(H, w["intermediate"], w["experts"], w["top_k"], _ptr(w["router"]),
                     w["gate_type"], w["up_type"], w["down_type"], _ptr(w.get("gate")),
                     _ptr(w.get("up")), _ptr(w.get("down")), w.get("shared_intermediate", 0),
                     _ptr(w.get("shared_gate")), _ptr(w.get("shared_up")),
                     _ptr(w.get("shared_down")), _ptr(w.get("shared_gate_vector")),
                     _ptr(w.get("router_logit_bias")))


def qwen_moe(w: dict, x, threads: int = 1):
    """Restated Qwen3.5-shaped MoE block (see dm_oracle.c for the definition)."""
    x = _f32(x)
    T, H = x.shape
    k = w["top_k"]
    layer = _qwen_layer(w, H)
    y = np.zeros((T, H), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.uint32)
    prob = np.zeros((T, k), dtype=np.float32)
    rc = lib().dmo_qwen_moe(C.byref(layer), _ptr(x), T, _ptr(y), _ptr(idx), _ptr(prob), threads)
    return rc, y, idx, prob


def _glm_layer(w: dict, H: int):
    return GlmLayer(H, w["intermediate"], w["experts"], w["top_k"], w.get("n_groups", 1),
                    w.get("topk_groups", 1), int(w.get("normalize", True)),
                    w.get("routed_scale", 1.0), w.get("weight_type", BF16), _ptr(w["router"]),
                    _ptr(w["correction_bias"]), _ptr(w.get("gate")), _ptr(w.get("up")),
                    _ptr(w.get("down")), w.get("shared_intermediate", 0),
                    _ptr(w.get("shared_gate")), _ptr(w.get("shared_up")),
                    _ptr(w.get("shared_down")))


def glm_moe(w: dict, x, threads: int = 1):
    """GLM-5.2 sparse feed-forward (src/glm52/cpu.rs:711-778)."""
    x = _f32(x)
    T, H = x.shape
    k = w["top_k"]
    layer = _glm_layer(w, H)
    blobs = w.get("expert_blobs")  # host addresses of per-expert gate|up|down blobs
    if blobs is not None:
        keep = (P * len(blobs))(*[int(b) for b in blobs])
        layer.expert_blobs = C.cast(keep, C.POINTER(P))
    y = np.zeros((T, H), dtype=np.float32)
    idx = np.zeros((T, k), dtype=np.uint32)
    wt = np.zeros((T, k), dtype=np.float32)
    rc = lib().dmo_glm_moe(C.byref(layer), _ptr(x), T, _ptr(y), _ptr(idx), _ptr(wt), threads)
    return rc, y, idx, wt


def route(family: str, w: dict, x, threads: int = 1):
    """The router and top-k of `family` ("gemma4", "qwen35", "glm52") alone, for every token
    of `x`: (rc, indices [T, k], weights [T, k]). Reads only the router tensors of `w`
    (src/gemma4/cpu.rs:562-576, src/cpu.rs:234-260, src/glm52/cpu.rs:731-754)."""
    x = _f32(x)
    T, H = x.shape
    k = w["top_k"]
    make, fn = {"gemma4": (_gemma_layer, lib().dmo_gemma_route),
                "qwen35": (_qwen_layer, lib().dmo_qwen_route),
                "glm52": (_glm_layer, lib().dmo_glm_route)}[family]
    layer = make(w, H)
    idx = np.zeros((T, k), dtype=np.uint32)
    wt = np.zeros((T, k), dtype=np.float32)
    rc = fn(C.byref(layer), _ptr(x), T, _ptr(idx), _ptr(wt), threads)
    return rc, idx, wt


class CacheStats(C.Structure):
    _fields_ = [("hits", C.c_uint64), ("misses", C.c_uint64), ("evictions", C.c_uint64),
                ("reads", C.c_uint64), ("bytes_read", C.c_uint64),
                ("resident_bytes", C.c_uint64)]


class Lru:
    """Restated expert LRU (src/expert.rs:166-229 / src/glm52/expert.rs:183-256)."""

    def __init__(self, layers, experts, slots, global_clock, expert_bytes, reads_per_miss):
        self.h = lib().dmo_lru_create(layers, experts, slots, global_clock, expert_bytes,
                                      reads_per_miss)

    def acquire(self, layer, expert):
        slot, miss = I32(), I32()
        rc = lib().dmo_lru_acquire(self.h, layer, expert, C.byref(slot), C.byref(miss))
        return rc, slot.value, bool(miss.value)

    def set_pinned(self, layer, slot, pinned):
        lib().dmo_lru_set_pinned(self.h, layer, slot, int(pinned))

    def stats(self):
        s = CacheStats()
        lib().dmo_lru_stats(self.h, C.byref(s))
        return {f: getattr(s, f) for f, _ in CacheStats._fields_}

    def __del__(self):
        if getattr(self, "h", None):
            lib().dmo_lru_destroy(self.h)
            self.h = None
