"""ctypes declarations of the C ABI (include/diskmule_cuda.h, include/diskmule_stack.h,
include/diskmule_selftest.h, include/diskmule_synth.h, include/diskmule_gguf.h).

The product path is the CUDA library `libdiskmule_cuda.so` built next to this file.
Nothing here falls back to a CPU implementation: if the library is missing the
import of `lib()` raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdiskmule_cuda.so")

# dm_status
OK = 0
ERR_NO_DEVICE = -1
ERR_ALLOCATION = -2
ERR_INVALID_ARGUMENT = -3
ERR_UNSUPPORTED_TENSOR_TYPE = -4
ERR_ELEMENT_COUNT = -5
ERR_BYTE_LENGTH = -6
ERR_INPUT_LENGTH = -7
ERR_OUTPUT_LENGTH = -8
ERR_EMPTY_INPUT = -9
ERR_NON_FINITE = -10
ERR_TOP_K = -11
ERR_MAPPED_RANGE = -12
ERR_OVERFLOW = -13
ERR_COMMAND = -14
ERR_INVALID_EXPERT = -15
ERR_INVALID_LAYER = -16
ERR_ALL_SLOTS_PINNED = -17
ERR_CANCELLED = -18
ERR_NO_SLOTS = -19
ERR_VECTOR_LENGTH = -20
ERR_POSITIVE_PARAMETER = -21
ERR_TIMEOUT = -22
ERR_NOT_BUILT = -23
ERR_COMMUNICATOR = -24
ERR_IO = -25
ERR_FORMAT = -26

# dm_tensor_type (GGML ids)
F32, F16, Q5_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 6, 8, 12, 14, 30
U8_QUANT, F8_E4M3 = 200, 201  # GLM-5.2 safetensors storage (dm_cuda_matvec_safetensor)
# dm_moe_family
FAMILY_GEMMA4, FAMILY_QWEN35_MOE, FAMILY_GLM52 = 1, 2, 3

P = C.c_void_p
SZ = C.c_size_t
I32 = C.c_int32


class MoeDesc(C.Structure):
    _fields_ = [
        ("family", I32),
        ("hidden", I32), ("intermediate", I32), ("experts", I32), ("top_k", I32),
        ("n_groups", I32), ("topk_groups", I32), ("normalize_topk", I32),
        ("routed_scale", C.c_float), ("epsilon", C.c_float),
        ("input_type", I32), ("router_type", I32), ("router", P),
        ("correction_bias", P), ("router_scale", P), ("routed_pre_norm", P),
        ("expert_scale", P),
        ("gate_type", I32), ("up_type", I32), ("down_type", I32),
        ("gate", P), ("up", P), ("down", P),
        ("shared_intermediate", I32),
        ("shared_gate", P), ("shared_up", P), ("shared_down", P),
        ("shared_gate_vector", P),
        ("router_logit_bias", P),
    ]


class ExpertLayout(C.Structure):
    """dm_expert_layout: one layer's experts in a host source."""
    _fields_ = [
        ("expert_count", I32), ("tensor_count", I32),
        ("bytes", C.c_uint64 * 4), ("offset", C.c_uint64 * 4),
        ("host", P), ("expert_host", C.POINTER(P)),
    ]


class ExpertCacheStats(C.Structure):
    """dm_expert_cache_stats (ExpertCacheStats, src/expert.rs:53-62)."""
    _fields_ = [
        ("hits", C.c_uint64), ("misses", C.c_uint64), ("evictions", C.c_uint64),
        ("reads", C.c_uint64), ("bytes_read", C.c_uint64), ("io_wait_ns", C.c_uint64),
        ("resident_bytes", C.c_uint64), ("h2d_bytes", C.c_uint64), ("fills", C.c_uint64),
    ]


# int64_t read(void *user, int32_t layer, int32_t expert, int32_t tensor, void *dst, uint64_t n)
READ_FN = C.CFUNCTYPE(C.c_int64, P, I32, I32, I32, P, C.c_uint64)

# Every symbol the headers declare, with its ctypes signature.
SIGNATURES = {
    "dm_status_string": ([I32], C.c_char_p),
    "dm_last_error_message": ([], C.c_char_p),
    "dm_cuda_create": ([I32, C.POINTER(P)], I32),
    "dm_cuda_destroy": ([P], None),
    "dm_cuda_device_name": ([P, C.c_char_p, SZ], I32),
    "dm_cuda_synchronize": ([P], I32),
    "dm_cuda_map_read_only": ([P, P, SZ, C.POINTER(P)], I32),
    "dm_cuda_new_owned_buffer": ([P, SZ, C.POINTER(P)], I32),
    "dm_buffer_write": ([P, SZ, P, SZ], I32),
    "dm_buffer_read": ([P, SZ, P, SZ], I32),
    "dm_buffer_length": ([P], SZ),
    "dm_buffer_device_pointer": ([P], P),
    "dm_buffer_free": ([P], None),
    "dm_cuda_matvec": ([P, I32, SZ, SZ, P, SZ, P, SZ, P, SZ], I32),
    "dm_cuda_matvec_mapped": ([P, I32, SZ, SZ, P, SZ, SZ, P, SZ, P, SZ], I32),
    "dm_cuda_matvec_safetensor": ([P, I32, SZ, SZ, P, SZ, P, SZ, P, SZ, P, SZ], I32),
    "dm_cuda_top_k_softmax": ([P, P, SZ, SZ, P, P], I32),
    "dm_cuda_gelu_mul": ([P, P, P, P, SZ], I32),
    "dm_cuda_silu_mul": ([P, P, P, P, SZ], I32),
    "dm_cuda_rms_norm": ([P, P, P, SZ, C.c_float, P], I32),
    "dm_moe_layer_create": ([P, C.POINTER(MoeDesc), C.POINTER(P)], I32),
    "dm_moe_layer_destroy": ([P], None),
    "dm_moe_forward": ([P, P, P, I32, P, P, P], I32),
    "dm_moe_forward_host": ([P, P, P, I32, P, P], I32),
    "dm_moe_forward_host_batches": ([P, I32, C.POINTER(P), C.POINTER(P), I32], I32),
    "dm_moe_last_dispatch": ([P, P, P, P, P], I32),
    "dm_moe_last_launch_count": ([P], I32),
    "dm_moe_forward_noalloc": ([P, P, P, I32, P, P, P], I32),
    "dm_moe_forward_noalloc_status": ([P, P], I32),
    "dm_moe_set_profiling": ([P, I32], I32),
    "dm_moe_stage_times": ([P, P, I32], I32),
    "dm_moe_stage_name": ([I32], C.c_char_p),
    "dm_moe_layer_create_ep": ([P, C.POINTER(MoeDesc), I32, I32, C.POINTER(P)], I32),
    "dm_moe_local_experts": ([P, C.POINTER(I32), C.POINTER(I32)], I32),
    "dm_moe_route": ([P, P, I32, P, P, P, P, P], I32),
    "dm_moe_expert_rows": ([P, P, P, I32, P, P], I32),
    "dm_moe_combine_rows": ([P, I32, P, P, P, P, P, P], I32),
    "dm_gemma_ffn_create": ([P, P, C.POINTER(P)], I32),
    "dm_gemma_ffn_forward": ([P, P, P, I32, P, P, P], I32),
    "dm_gemma_ffn_status": ([P, P], I32),
    "dm_gemma_ffn_destroy": ([P], None),
    "dm_ep_create": ([P, I32, I32, I32, C.POINTER(P)], I32),
    "dm_ep_ipc_handle": ([P, P], I32),
    "dm_ep_connect_ipc": ([P, P], I32),
    "dm_ep_connect_local": ([P, C.POINTER(P)], I32),
    "dm_ep_dispatch": ([P, P, I32, P], I32),
    "dm_ep_experts": ([P, P], I32),
    "dm_ep_combine": ([P, P, P, P, P], I32),
    "dm_ep_forward": ([P, P, P, I32, P, P, P], I32),
    "dm_ep_status": ([P, P], I32),
    "dm_ep_last_launch_count": ([P], I32),
    "dm_ep_destroy": ([P], None),
    "dm_cuda_host_alloc": ([P, SZ, C.POINTER(P)], I32),
    "dm_cuda_host_free": ([P, P], None),
    "dm_cuda_host_register": ([P, P, SZ], I32),
    "dm_cuda_host_unregister": ([P, P], I32),
    "dm_expert_cache_create": ([P, C.POINTER(ExpertLayout), I32, I32, I32, C.POINTER(P)], I32),
    "dm_expert_cache_set_reader": ([P, READ_FN, P], I32),
    "dm_expert_cache_destroy": ([P], None),
    "dm_expert_cache_slots_per_layer": ([P], I32),
    "dm_expert_cache_slot_memory": ([P, I32, I32, C.POINTER(P), C.POINTER(C.c_uint64)], I32),
    "dm_expert_cache_acquire": ([P, I32, I32, C.POINTER(I32), C.POINTER(I32), C.POINTER(I32)], I32),
    "dm_expert_cache_wait_slot": ([P, I32, I32, P], I32),
    "dm_expert_cache_release_slot": ([P, I32, I32, P], I32),
    "dm_expert_cache_set_pinned": ([P, I32, I32, I32], I32),
    "dm_expert_cache_slot_expert": ([P, I32, I32, C.POINTER(I32)], I32),
    "dm_expert_cache_read_slot": ([P, I32, I32, I32, P, C.c_uint64], I32),
    "dm_expert_cache_get_stats": ([P, C.POINTER(ExpertCacheStats)], I32),
    "dm_expert_cache_synchronize": ([P], I32),
    "dm_moe_layer_create_cached": ([P, C.POINTER(MoeDesc), P, I32, C.POINTER(P)], I32),
    "dm_moe_forward_cached": ([P, P, P, I32, P, P, C.POINTER(I32), P], I32),
    "dm_stack_embed": ([P, P, I32, I32, I32, P, P, P, P], I32),
    "dm_stack_add_rms_norm": ([P, P, P, P, I32, C.c_float, P, P, P], I32),
    "dm_stack_lm_head_argmax": ([P, P, I32, I32, I32, P, P, P, P, P], I32),
    "dm_selftest_device_wait": ([P, C.c_int64], I32),
    "dm_gguf_open": ([C.c_char_p, C.c_char_p, C.POINTER(P)], I32),
    "dm_gguf_parse": ([P, C.c_uint64, C.c_char_p, C.POINTER(P)], I32),
    "dm_gguf_close": ([P], None),
    "dm_gguf_header": ([P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                        C.POINTER(C.c_uint64)], I32),
    "dm_gguf_tensor_count": ([P], C.c_int64),
    "dm_gguf_find_tensor": ([P, C.c_char_p, C.POINTER(C.c_int64)], I32),
    "dm_gguf_tensor": ([P, C.c_int64, P], I32),
    "dm_gguf_tensor_bytes": ([P, C.c_int64, C.POINTER(P), C.POINTER(C.c_uint64)], I32),
    "dm_gguf_read_tensor_at": ([P, C.c_char_p, C.c_uint64, P, C.c_uint64], I32),
    "dm_gguf_metadata_type": ([P, C.c_char_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                               C.POINTER(C.c_uint64)], I32),
    "dm_gguf_metadata_u64": ([P, C.c_char_p, C.POINTER(C.c_uint64)], I32),
    "dm_gguf_metadata_f64": ([P, C.c_char_p, C.POINTER(C.c_double)], I32),
    "dm_gguf_metadata_string": ([P, C.c_char_p, C.c_char_p, C.c_uint64], I32),
    "dm_gguf_metadata_array": ([P, C.c_char_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                C.POINTER(P)], I32),
    "dm_gguf_expert_layout": ([P, C.c_char_p, C.c_char_p, I32, P], I32),
    "dm_synth_fill_host": ([I32, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                            C.c_float, P], I32),
    "dm_synth_fill_device": ([I32, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float,
                              C.c_float, P, P], I32),
}

_lib = None


def lib() -> C.CDLL:
    """Load the CUDA library (built by `diskmule_b200.build`); raise if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: run `python -m diskmule_b200.build` (there is no CPU "
                "fallback for this path)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


class DmError(RuntimeError):
    """A failed call: `status` is the dm_status code, the message its detail text."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


def check(status: int) -> None:
    if status != OK:
        L = lib()
        detail = L.dm_last_error_message().decode() or L.dm_status_string(status).decode()
        raise DmError(status, detail)
