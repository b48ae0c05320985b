"""A GLM-5.2-shaped decode stack with out-of-core experts.

`layers` sparse layers of one GLM shape, each `h += moe(rms_norm(h, norm_l))` -- the
feed-forward half of a GLM block in the reference's residual order
(src/glm52/cpu.rs:498-517; the attention half is not on this path) -- between a
synthetic bf16 embedding and output head with greedy argmax (src/glm52/cpu.rs:476-518).
Every layer's routed experts live in page-locked host memory as one blob per expert
(gate | up | down, bf16); each layer keeps `slots` of them in HBM through one expert
cache with the GLM rules (a single clock across layers, src/glm52/expert.rs:183-256),
so a decode step copies its misses over PCIe while resident experts compute. The
router, correction bias and shared expert of each layer stay in HBM.

Blob b holds the weights that `layer_specs(cfg, seed + l)` gives expert e, for
(l, e) = divmod(b, experts). With `pool_experts` below layers * experts, expert (l, e)
reads blob (l * experts + e) % pool_experts: the host pool then repeats weights, but
every miss still moves a whole expert over PCIe.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from ._native import check
from .cache import CachedMoeLayer, ExpertCache, PinnedHost, layout
from .moe import CudaContext
from .synthetic import CONFIGS, FAMILIES, TensorSpec, layer_specs


def _vector(seed: int, n: int) -> np.ndarray:
    """RMSNorm weights: U[0.5, 1.5), seeded."""
    return np.random.default_rng(seed).uniform(0.5, 1.5, n).astype(np.float32)


class GlmStack:
    def __init__(self, ctx: CudaContext, name: str = "glm52", layers: int = 8, slots: int = 8,
                 vocab: int = 32768, pool_experts: int | None = None, seed: int = 11,
                 epsilon: float = 1e-5, fill_batch: int = 16):
        cfg = dict(CONFIGS[name])
        assert cfg["family"] == "glm52"
        self.ctx, self.cfg, self.name = ctx, cfg, name
        self.n_layers, self.slots, self.vocab, self.seed = layers, slots, vocab, seed
        self.epsilon = float(epsilon)
        H, I, E = cfg["hidden"], cfg["intermediate"], cfg["experts"]
        self.H, self.I, self.E = H, I, E
        self.tensor_bytes = I * H * 2
        self.expert_bytes = 3 * self.tensor_bytes
        self.pool_experts = min(pool_experts or layers * E, layers * E)
        self.specs = [layer_specs(cfg, seed + l) for l in range(layers)]
        self._buffers = []
        self._fill_pool(fill_batch)
        # resident per-layer tensors
        self.layer_buf = []
        for l in range(layers):
            bufs = {}
            for key in ("router", "bias", "shared_gate", "shared_up", "shared_down"):
                spec = self.specs[l][key]
                bufs[key] = self._device(spec.nbytes)
                spec.device_fill(bufs[key].device_pointer)
            self.layer_buf.append(bufs)
        self.norms = [_vector(seed * 131 + l, H) for l in range(layers)]
        self.out_norm = _vector(seed * 131 + 997, H)
        self.norm_buf = [ctx.map_read_only(v) for v in self.norms]
        self.out_norm_buf = ctx.map_read_only(self.out_norm)
        self.embed_spec = TensorSpec("embed", N.BF16, vocab, H, 1, seed * 1009 + 501, 1.0)
        self.head_spec = TensorSpec("head", N.BF16, vocab, H, 1, seed * 1009 + 502, 0.02)
        self.embed = self._device(self.embed_spec.nbytes)
        self.embed_spec.device_fill(self.embed.device_pointer)
        self.head = self._device(self.head_spec.nbytes)
        self.head_spec.device_fill(self.head.device_pointer)
        # expert cache over the pool
        lays = []
        for l in range(layers):
            blobs = [self.blob_pointer(l, e) for e in range(E)]
            lays.append(layout(E, [self.tensor_bytes] * 3,
                               offsets=[0, self.tensor_bytes, 2 * self.tensor_bytes],
                               expert_host=blobs))
        self.cache = ExpertCache(ctx, lays, slots, global_clock=True)
        self.layers = []
        for l in range(layers):
            self.layers.append(CachedMoeLayer(ctx, self._desc(l), self.cache, l))
        # step state
        self.h = self._device(H * 4)
        self.n = self._device(H * 4)
        self.y = self._device(H * 4)
        self.logits = self._device(vocab * 4)
        self.status = self._device(256)
        self.token_ring = self._device(4 * 2)
        check(N.lib().dm_buffer_write(self.status.handle, 0,
                                      np.zeros(64, np.uint8).ctypes.data_as(C.c_void_p), 64))
        ctx.synchronize()

    # ---- construction -------------------------------------------------------
    def _device(self, nbytes: int):
        b = self.ctx.new_owned_buffer(nbytes)
        self._buffers.append(b)
        return b

    def blob_index(self, layer: int, expert: int) -> int:
        return (layer * self.E + expert) % self.pool_experts

    def blob_pointer(self, layer: int, expert: int) -> int:
        return self.pool.pointer + self.blob_index(layer, expert) * self.expert_bytes

    def _fill_pool(self, batch: int):
        """Generate blob b's gate, up, down on the device in batches and copy them into
        page-locked host memory."""
        P, eb, tb = self.pool_experts, self.expert_bytes, self.tensor_bytes
        self.pool = PinnedHost(self.ctx, P * eb)
        batch = max(1, min(batch, P))
        staging = self.ctx.new_owned_buffer(batch * eb)
        base = staging.device_pointer
        try:
            for b0 in range(0, P, batch):
                n = min(batch, P - b0)
                for j in range(n):
                    l, e = divmod(b0 + j, self.E)
                    for t, key in enumerate(("gate", "up", "down")):
                        self.specs[l][key].device_fill(base + j * eb + t * tb, expert=e)
                check(N.lib().dm_buffer_read(staging.handle, 0,
                                             C.c_void_p(self.pool.pointer + b0 * eb), n * eb))
        finally:
            staging.free()

    def _desc(self, l: int) -> N.MoeDesc:
        cfg, b = self.cfg, self.layer_buf[l]
        d = N.MoeDesc()
        d.family = FAMILIES["glm52"]
        d.hidden, d.intermediate, d.experts, d.top_k = self.H, self.I, self.E, cfg["top_k"]
        d.n_groups, d.topk_groups = cfg["n_groups"], cfg["topk_groups"]
        d.normalize_topk = int(cfg["normalize"])
        d.routed_scale = cfg["routed_scale"]
        d.epsilon = 1e-6
        d.input_type = N.F32  # the normalised hidden state
        d.router_type = N.BF16
        d.router = b["router"].device_pointer
        d.correction_bias = b["bias"].device_pointer
        d.gate_type = d.up_type = d.down_type = N.BF16
        d.shared_intermediate = self.I
        d.shared_gate = b["shared_gate"].device_pointer
        d.shared_up = b["shared_up"].device_pointer
        d.shared_down = b["shared_down"].device_pointer
        return d

    # ---- decode -------------------------------------------------------------
    def step(self, token_ptr: int, next_ptr: int, stream: int = 0, cancelled=None):
        """One greedy step: *next_ptr = argmax(head(norm(stack(embed(*token_ptr)))))."""
        L = N.lib()
        s = C.c_void_p(stream) if stream else None
        ctx = self.ctx.handle
        st = C.c_void_p(self.status.device_pointer)
        h, n, y = (C.c_void_p(b.device_pointer) for b in (self.h, self.n, self.y))
        check(L.dm_stack_embed(ctx, C.c_void_p(self.embed.device_pointer), N.BF16, self.vocab,
                               self.H, C.c_void_p(token_ptr), h, st, s))
        check(L.dm_stack_add_rms_norm(ctx, h, None, C.c_void_p(self.norm_buf[0].device_pointer),
                                      self.H, self.epsilon, n, st, s))
        for l, layer in enumerate(self.layers):
            layer.forward_cached(self.n.device_pointer, self.y.device_pointer, 1,
                                 cancelled=cancelled, stream=stream)
            w = self.norm_buf[l + 1] if l + 1 < self.n_layers else self.out_norm_buf
            check(L.dm_stack_add_rms_norm(ctx, h, y, C.c_void_p(w.device_pointer), self.H,
                                          self.epsilon, n, st, s))
        check(L.dm_stack_lm_head_argmax(ctx, C.c_void_p(self.head.device_pointer), N.BF16,
                                        self.vocab, self.H, n,
                                        C.c_void_p(self.logits.device_pointer),
                                        C.c_void_p(next_ptr), st, s))

    def decode(self, first_token: int, steps: int, stream: int = 0, host_tokens=None):
        """Greedy decode; returns the `steps` generated tokens. Each step's token is
        read back to the host (the step's result)."""
        ring = self.token_ring.device_pointer
        tok = np.array([first_token], dtype=np.int32)
        check(N.lib().dm_buffer_write(self.token_ring.handle, 0,
                                      tok.ctypes.data_as(C.c_void_p), 4))
        out = []
        for i in range(steps):
            cur, nxt = ring + 4 * (i & 1), ring + 4 * ((i + 1) & 1)
            self.step(cur, nxt, stream)
            check(N.lib().dm_buffer_read(self.token_ring.handle, 4 * ((i + 1) & 1),
                                         tok.ctypes.data_as(C.c_void_p), 4))
            out.append(int(tok[0]))
        return out

    def status_bits(self) -> int:
        v = np.zeros(1, np.int32)
        check(N.lib().dm_buffer_read(self.status.handle, 0, v.ctypes.data_as(C.c_void_p), 4))
        return int(v[0])

    def hidden(self) -> np.ndarray:
        return self.h.read().view(np.float32).copy()

    # ---- the oracle's view of the same weights ---------------------------------
    def host_layer(self, l: int) -> dict:
        """Oracle inputs for layer l (src/glm52/cpu.rs:711-778), expert weights read
        from the host pool blobs."""
        cfg, sp = self.cfg, self.specs[l]
        return dict(hidden=self.H, intermediate=self.I, experts=self.E, top_k=cfg["top_k"],
                    n_groups=cfg["n_groups"], topk_groups=cfg["topk_groups"],
                    normalize=cfg["normalize"], routed_scale=cfg["routed_scale"],
                    weight_type=N.BF16, router=sp["router"].host(),
                    correction_bias=sp["bias"].host().view(np.float32),
                    shared_intermediate=self.I, shared_gate=sp["shared_gate"].host(),
                    shared_up=sp["shared_up"].host(), shared_down=sp["shared_down"].host(),
                    expert_blobs=[self.blob_pointer(l, e) for e in range(self.E)])

    def embed_row(self, token: int) -> np.ndarray:
        row = self.embed_spec.host()[token * self.H * 2:(token + 1) * self.H * 2]
        return (row.view(np.uint16).astype(np.uint32) << 16).view(np.float32)

    def close(self):
        for layer in getattr(self, "layers", []):
            layer.close()
        self.layers = []
        if getattr(self, "cache", None) is not None:
            self.cache.close()
            self.cache = None
        for b in self._buffers:
            b.free()
        self._buffers = []
        for b in getattr(self, "norm_buf", []) + [getattr(self, "out_norm_buf", None)]:
            if b is not None:
                b.free()
        self.norm_buf = []
        self.out_norm_buf = None
        if getattr(self, "pool", None) is not None:
            self.pool.free()
            self.pool = None
