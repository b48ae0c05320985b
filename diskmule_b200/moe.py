"""Host-side mirror of the reference's Metal backend surface, over the C ABI.

`CudaContext` mirrors `MetalContext` (src/metal.rs:179-1604): the same method
names, argument meaning and error behaviour (a `DmError` whose `status` names the
`MetalError` variant). `MoeLayer` is the batched routed-expert block that replaces
the per-token, per-expert loop of src/gemma4/cpu.rs:559-611 / src/glm52/cpu.rs:
711-778. Every call goes to libdiskmule_cuda.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from ._native import DmError, check


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, int):
        return C.c_void_p(a)
    return a.ctypes.data_as(C.c_void_p)


class Buffer:
    """A device buffer (MetalMappedBuffer / MetalOwnedBuffer, src/metal.rs:207-243)."""

    def __init__(self, handle, ctx):
        self._h = handle
        self._ctx = ctx

    @property
    def handle(self):
        return self._h

    def __len__(self):
        return N.lib().dm_buffer_length(self._h)

    @property
    def device_pointer(self) -> int:
        return N.lib().dm_buffer_device_pointer(self._h) or 0

    def write(self, data, offset: int = 0):
        a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        check(N.lib().dm_buffer_write(self._h, offset, _ptr(a), a.size))

    def read(self, length: int | None = None, offset: int = 0) -> np.ndarray:
        n = len(self) - offset if length is None else length
        out = np.empty(n, dtype=np.uint8)
        check(N.lib().dm_buffer_read(self._h, offset, _ptr(out), n))
        return out

    def free(self):
        if self._h:
            N.lib().dm_buffer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class CudaContext:
    """MetalContext's method surface on one B200 (src/metal.rs:291-1434)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(N.lib().dm_cuda_create(device, C.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def device_name(self) -> str:
        buf = C.create_string_buffer(256)
        check(N.lib().dm_cuda_device_name(self._h, buf, 256))
        return buf.value.decode()

    def synchronize(self):
        check(N.lib().dm_cuda_synchronize(self._h))

    def map_read_only(self, data) -> Buffer:
        a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        h = C.c_void_p()
        check(N.lib().dm_cuda_map_read_only(self._h, _ptr(a), a.size, C.byref(h)))
        return Buffer(h, self)

    def new_owned_buffer(self, length: int) -> Buffer:
        h = C.c_void_p()
        check(N.lib().dm_cuda_new_owned_buffer(self._h, length, C.byref(h)))
        return Buffer(h, self)

    def matvec(self, kind, rows, columns, encoded, input, output_len=None):
        enc = np.ascontiguousarray(np.frombuffer(encoded, np.uint8) if isinstance(encoded, (bytes, bytearray)) else encoded).view(np.uint8).reshape(-1)
        x = np.ascontiguousarray(input, dtype=np.float32)
        out = np.zeros(rows if output_len is None else output_len, dtype=np.float32)
        check(N.lib().dm_cuda_matvec(self._h, kind, rows, columns, _ptr(enc), enc.size,
                                      _ptr(x), x.size, _ptr(out), out.size))
        return out

    def matvec_mapped(self, kind, rows, columns, mapped: Buffer, offset, length, input,
                      output_len=None):
        x = np.ascontiguousarray(input, dtype=np.float32)
        out = np.zeros(rows if output_len is None else output_len, dtype=np.float32)
        check(N.lib().dm_cuda_matvec_mapped(self._h, kind, rows, columns, mapped.handle, offset,
                                             length, _ptr(x), x.size, _ptr(out), out.size))
        return out

    matvec_owned = matvec_mapped

    def matvec_safetensor(self, dtype, rows, columns, encoded, scales, input):
        """MetalContext::matvec_safetensor (src/metal.rs:883-992): F32 / F16 / BF16 rows,
        or the GLM-5.2 checkpoint storage N.U8_QUANT (int8 rows / grouped int4 with `.qs`
        scales) and N.F8_E4M3 (with 128 x 128 block `_scale_inv` scales)."""
        enc = np.ascontiguousarray(np.frombuffer(encoded, np.uint8) if isinstance(encoded, (bytes, bytearray)) else encoded).view(np.uint8).reshape(-1)
        sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        x = np.ascontiguousarray(input, dtype=np.float32)
        out = np.zeros(rows, dtype=np.float32)
        check(N.lib().dm_cuda_matvec_safetensor(self._h, dtype, rows, columns, _ptr(enc), enc.size,
                                                _ptr(sc), 0 if sc is None else sc.size, _ptr(x),
                                                x.size, _ptr(out), out.size))
        return out

    def top_k_softmax(self, logits, k):
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        idx = np.zeros(max(k, 1), dtype=np.uint32)
        prob = np.zeros(max(k, 1), dtype=np.float32)
        check(N.lib().dm_cuda_top_k_softmax(self._h, _ptr(lg), lg.size, k, _ptr(idx), _ptr(prob)))
        return [(int(i), float(p)) for i, p in zip(idx[:k], prob[:k])]

    def _binary(self, fn, gate, up):
        g = np.ascontiguousarray(gate, dtype=np.float32)
        u = np.ascontiguousarray(up, dtype=np.float32)
        if g.size != u.size:
            raise DmError(N.ERR_VECTOR_LENGTH, "up length differs from gate")
        out = np.zeros_like(g)
        check(fn(self._h, _ptr(g), _ptr(u), _ptr(out), g.size))
        return out

    def gelu_mul(self, gate, up):
        return self._binary(N.lib().dm_cuda_gelu_mul, gate, up)

    def silu_mul(self, gate, up):
        return self._binary(N.lib().dm_cuda_silu_mul, gate, up)

    def rms_norm(self, input, weight, epsilon):
        x = np.ascontiguousarray(input, dtype=np.float32)
        w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float32)
        if w is not None and w.size != x.size:
            raise DmError(N.ERR_VECTOR_LENGTH, "RMSNorm weight length differs from input")
        out = np.zeros_like(x)
        check(N.lib().dm_cuda_rms_norm(self._h, _ptr(x), _ptr(w), x.size, epsilon, _ptr(out)))
        return out

    def close(self):
        if self._h:
            N.lib().dm_cuda_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GemmaFfnDesc(C.Structure):
    _fields_ = [("width", C.c_int32), ("gate_type", C.c_int32), ("up_type", C.c_int32),
                ("down_type", C.c_int32), ("gate", C.c_void_p), ("up", C.c_void_p),
                ("down", C.c_void_p), ("feed_forward_norm", C.c_void_p),
                ("shared_post_norm", C.c_void_p), ("routed_post_norm", C.c_void_p),
                ("post_feed_forward_norm", C.c_void_p), ("layer_output_scale", C.c_float)]


class GemmaFfnBlock:
    """Gemma 4's whole feed-forward block (dm_gemma_ffn_*): the routed `layer` plus the
    dense shared FFN and the norms around it (src/gemma4/cpu.rs:547-620)."""

    def __init__(self, layer, desc: GemmaFfnDesc):
        self.layer, self.desc = layer, desc
        h = C.c_void_p()
        check(N.lib().dm_gemma_ffn_create(layer.handle, C.byref(desc), C.byref(h)))
        self._h = h

    def forward(self, x_ptr: int, hidden_ptr: int, tokens: int, sel_idx_ptr=0, sel_w_ptr=0,
                stream: int = 0):
        check(N.lib().dm_gemma_ffn_forward(self._h, C.c_void_p(x_ptr), C.c_void_p(hidden_ptr),
                                           tokens, C.c_void_p(sel_idx_ptr) if sel_idx_ptr else None,
                                           C.c_void_p(sel_w_ptr) if sel_w_ptr else None,
                                           C.c_void_p(stream) if stream else None))

    def status(self, stream: int = 0):
        check(N.lib().dm_gemma_ffn_status(self._h, C.c_void_p(stream) if stream else None))

    def close(self):
        if self._h:
            N.lib().dm_gemma_ffn_destroy(self._h)
            self._h = None


class MoeLayer:
    """The batched routed-expert block behind dm_moe_layer_create / dm_moe_forward.

    `desc` is a `_native.MoeDesc` whose weight fields hold device addresses.
    """

    def __init__(self, ctx: CudaContext, desc: N.MoeDesc, keep_alive=(), expert_range=None):
        """`expert_range=(first, count)`: a layer holding those experts only (the
        desc's expert weights are that range), for expert parallelism."""
        self.ctx = ctx
        self.desc = desc
        self._keep = list(keep_alive)
        h = C.c_void_p()
        if expert_range is None:
            check(N.lib().dm_moe_layer_create(ctx.handle, C.byref(desc), C.byref(h)))
        else:
            first, count = expert_range
            check(N.lib().dm_moe_layer_create_ep(ctx.handle, C.byref(desc), int(first), int(count),
                                                 C.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def forward(self, x_ptr: int, y_ptr: int, tokens: int, sel_idx_ptr=None, sel_w_ptr=None,
                stream: int = 0):
        """Stream-ordered forward on device pointers (dm_moe_forward)."""
        check(N.lib().dm_moe_forward(self._h, C.c_void_p(x_ptr), C.c_void_p(y_ptr), tokens,
                                      C.c_void_p(sel_idx_ptr) if sel_idx_ptr else None,
                                      C.c_void_p(sel_w_ptr) if sel_w_ptr else None,
                                      C.c_void_p(stream) if stream else None))

    def local_experts(self) -> tuple[int, int]:
        first, count = C.c_int32(), C.c_int32()
        check(N.lib().dm_moe_local_experts(self._h, C.byref(first), C.byref(count)))
        return first.value, count.value

    def route(self, x_ptr: int, tokens: int, sel_idx_ptr: int, sel_w_ptr: int,
              expert_in_ptr: int = 0, logits_ptr: int = 0, stream: int = 0):
        """Router + top-k only (dm_moe_route), device pointers."""
        check(N.lib().dm_moe_route(self._h, C.c_void_p(x_ptr), tokens, C.c_void_p(sel_idx_ptr),
                                    C.c_void_p(sel_w_ptr),
                                    C.c_void_p(expert_in_ptr) if expert_in_ptr else None,
                                    C.c_void_p(logits_ptr) if logits_ptr else None,
                                    C.c_void_p(stream) if stream else None))

    def expert_rows(self, rows_ptr: int, ids_ptr: int, count: int, out_ptr: int, stream: int = 0):
        """Unweighted expert outputs of rows on this layer's experts (dm_moe_expert_rows)."""
        check(N.lib().dm_moe_expert_rows(self._h, C.c_void_p(rows_ptr), C.c_void_p(ids_ptr),
                                          count, C.c_void_p(out_ptr),
                                          C.c_void_p(stream) if stream else None))

    def combine_rows(self, tokens: int, sel_idx_ptr: int, sel_w_ptr: int, pair_out_ptr: int,
                     y_ptr: int, logits_ptr: int = 0, stream: int = 0):
        """Weighted combine of per-pair outputs given in pair order (dm_moe_combine_rows)."""
        check(N.lib().dm_moe_combine_rows(self._h, tokens, C.c_void_p(sel_idx_ptr),
                                           C.c_void_p(sel_w_ptr),
                                           C.c_void_p(logits_ptr) if logits_ptr else None,
                                           C.c_void_p(pair_out_ptr), C.c_void_p(y_ptr),
                                           C.c_void_p(stream) if stream else None))

    def forward_host(self, x: np.ndarray, out=None):
        """Synchronous forward on host arrays (dm_moe_forward_host): (y, indices, weights).
        `out`, when given, is that triple preallocated (page-locked arrays make the
        copies direct DMA)."""
        x = np.ascontiguousarray(x)
        T = x.shape[0]
        H, k = self.desc.hidden, self.desc.top_k
        if out is not None:
            y, idx, w = out
            assert y.shape == (T, H) and y.dtype == np.float32 and y.flags.c_contiguous
            assert idx.shape == (T, k) and idx.dtype == np.uint32 and idx.flags.c_contiguous
            assert w.shape == (T, k) and w.dtype == np.float32 and w.flags.c_contiguous
        else:
            y = np.zeros((T, H), dtype=np.float32)
            idx = np.zeros((T, k), dtype=np.uint32)
            w = np.zeros((T, k), dtype=np.float32)
        check(N.lib().dm_moe_forward_host(self._h, _ptr(x), _ptr(y), T, _ptr(idx), _ptr(w)))
        return y, idx, w

    def forward_host_batches(self, xs, ys):
        """Pipelined forwards of equal-size host batches (dm_moe_forward_host_batches):
        xs[b] [T, hidden] (input type) -> ys[b] [T, hidden] f32, written in place."""
        n = len(xs)
        if n != len(ys):
            raise ValueError("xs and ys differ in length")
        if n == 0:
            return
        T = xs[0].shape[0]
        H = self.desc.hidden
        for a, b in zip(xs, ys):
            assert a.shape[0] == T and a.flags.c_contiguous
            assert b.shape == (T, H) and b.dtype == np.float32 and b.flags.c_contiguous
        xp = (C.c_void_p * n)(*[a.ctypes.data for a in xs])
        yp = (C.c_void_p * n)(*[b.ctypes.data for b in ys])
        check(N.lib().dm_moe_forward_host_batches(self._h, n, xp, yp, T))

    def last_dispatch(self, tokens: int):
        E, k = self.desc.experts, self.desc.top_k
        counts = np.zeros(E, np.int32)
        offsets = np.zeros(E + 1, np.int32)
        sorted_pairs = np.zeros(tokens * k, np.int32)
        inverse = np.zeros(tokens * k, np.int32)
        check(N.lib().dm_moe_last_dispatch(self._h, _ptr(counts), _ptr(offsets),
                                            _ptr(sorted_pairs), _ptr(inverse)))
        return counts, offsets, sorted_pairs, inverse

    def last_launch_count(self) -> int:
        return N.lib().dm_moe_last_launch_count(self._h)

    def set_profiling(self, enable: bool):
        check(N.lib().dm_moe_set_profiling(self._h, int(enable)))

    def stage_times(self) -> dict[str, float]:
        """Durations (ms) of the last forward's stages (needs set_profiling(True))."""
        buf = (C.c_float * 16)()
        n = N.lib().dm_moe_stage_times(self._h, buf, 16)
        if n < 0:
            check(n)
        return {N.lib().dm_moe_stage_name(i).decode(): float(buf[i]) for i in range(n)}

    def close(self):
        if self._h:
            N.lib().dm_moe_layer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
