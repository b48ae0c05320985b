"""Seeded synthetic MoE layers with the shapes of the benchmark configurations.

No checkpoints are available, so every weight is generated: block b of a tensor is
a pure function of (seed, b) (include/diskmule_synth.h), written straight into HBM
by a kernel or into host memory by the same code on the CPU, bit for bit equal.
Shapes and value distributions follow the benchmark configurations:

  gemma4  hidden 2816, 128 experts, top-8, intermediate 704, fused Q4_K gate_up,
          Q5_0 down (Q4_K cannot encode K = 704), router f32 N(0, 0.02)
  qwen35  hidden 2048, 512 experts, top-10, intermediate 512, Q4_K gate/up, Q6_K down,
          shared expert + sigmoid gate vector f32 N(0, 0.02)
  glm52   hidden 6144, 256 experts, top-8, intermediate 2048, bf16 N(0, 0.02), shared
          expert, correction bias f32 N(0, 0.01), 8 groups / 4 kept, routed scale 2.5
Block formats: f16 d (and dmin) uniform in [1e-3, 1e-2], all other bytes uniform.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _native as N
from .moe import CudaContext, MoeLayer

FAMILIES = {"gemma4": N.FAMILY_GEMMA4, "qwen35": N.FAMILY_QWEN35_MOE, "glm52": N.FAMILY_GLM52}

CONFIGS = {
    "gemma4": dict(family="gemma4", hidden=2816, intermediate=704, experts=128, top_k=8,
                   gate_type=N.Q4_K, down_type=N.Q5_0, epsilon=1e-6),
    "qwen35": dict(family="qwen35", hidden=2048, intermediate=512, experts=512, top_k=10,
                   gate_type=N.Q4_K, down_type=N.Q6_K, shared=True),
    "glm52": dict(family="glm52", hidden=6144, intermediate=2048, experts=256, top_k=8,
                  gate_type=N.BF16, down_type=N.BF16, shared=True, n_groups=8, topk_groups=4,
                  routed_scale=2.5, normalize=True),
    # reduced shapes of the same families for fast parity sweeps
    "gemma4-small": dict(family="gemma4", hidden=512, intermediate=128, experts=16, top_k=4,
                         gate_type=N.Q4_K, down_type=N.Q5_0, epsilon=1e-6),
    "gemma4-small-q8": dict(family="gemma4", hidden=512, intermediate=128, experts=16, top_k=4,
                            gate_type=N.Q4_K, down_type=N.Q8_0, epsilon=1e-6),
    "qwen35-small": dict(family="qwen35", hidden=512, intermediate=256, experts=32, top_k=4,
                         gate_type=N.Q4_K, down_type=N.Q6_K, shared=True),
    # 40 experts, top-10: the last top-k warp holds fewer valid experts than k
    "qwen35-odd": dict(family="qwen35", hidden=256, intermediate=256, experts=40, top_k=10,
                       gate_type=N.Q4_K, down_type=N.Q6_K, shared=True),
    "glm52-small": dict(family="glm52", hidden=256, intermediate=128, experts=32, top_k=4,
                        gate_type=N.BF16, down_type=N.BF16, shared=True, n_groups=4,
                        topk_groups=2, routed_scale=2.5, normalize=True),
    # the GLM shapes with 32 experts (2.4 GB): at T=1024 each expert gets the ~256 tokens
    # it gets at T=8192 with 256 experts, so its GEMM tiles match config 4's (profiling)
    "glm52-e32": dict(family="glm52", hidden=6144, intermediate=2048, experts=32, top_k=8,
                      gate_type=N.BF16, down_type=N.BF16, shared=True, n_groups=8,
                      topk_groups=4, routed_scale=2.5, normalize=True),
    "glm52-small-flat": dict(family="glm52", hidden=256, intermediate=128, experts=16, top_k=2,
                             gate_type=N.BF16, down_type=N.BF16, shared=True, n_groups=1,
                             topk_groups=1, routed_scale=2.5, normalize=True),
}

SCALE_LO, SCALE_HI = 1e-3, 1e-2
_BLOCK = {N.F32: (1, 4), N.F16: (1, 2), N.BF16: (1, 2), N.Q5_0: (32, 22), N.Q8_0: (32, 34),
          N.Q4_K: (256, 144), N.Q6_K: (256, 210)}


@dataclass
class TensorSpec:
    name: str
    kind: int
    rows: int
    cols: int
    experts: int = 1
    seed: int = 0
    sigma: float = 0.02

    @property
    def blocks_per_row(self) -> int:
        e, _ = _BLOCK[self.kind]
        assert self.cols % e == 0, (self.name, self.cols)
        return self.cols // e

    @property
    def row_bytes(self) -> int:
        return self.blocks_per_row * _BLOCK[self.kind][1]

    @property
    def expert_bytes(self) -> int:
        return self.rows * self.row_bytes

    @property
    def nbytes(self) -> int:
        return self.experts * self.expert_bytes

    def _range(self, expert: int | None, count: int = 1):
        per = self.rows * self.blocks_per_row
        return (0, per * self.experts) if expert is None else (expert * per, per * count)

    def host(self, expert: int | None = None, fill=None) -> np.ndarray:
        """Bytes of the whole tensor, or of one expert's slice, generated on the CPU.
        `fill(kind, seed, first_block, n_blocks, sigma, lo, hi, block_bytes)` replaces
        the library's host fill (the CPU reference arm passes the oracle's, so that it
        never loads the CUDA library); both evaluate the same generator."""
        first, n = self._range(expert)
        if fill is not None:
            return fill(self.kind, self.seed, first, n, self.sigma, SCALE_LO, SCALE_HI,
                        _BLOCK[self.kind][1])
        out = np.empty(n * _BLOCK[self.kind][1], dtype=np.uint8)
        N.check(N.lib().dm_synth_fill_host(self.kind, self.seed, first, n, self.sigma,
                                           SCALE_LO, SCALE_HI, out.ctypes.data_as(C.c_void_p)))
        return out

    def device_fill(self, ptr: int, expert: int | None = None, stream: int = 0, count: int = 1):
        """Device bytes of the whole tensor, or of experts expert..expert+count-1."""
        first, n = self._range(expert, count)
        N.check(N.lib().dm_synth_fill_device(self.kind, self.seed, first, n, self.sigma,
                                             SCALE_LO, SCALE_HI, C.c_void_p(ptr),
                                             C.c_void_p(stream) if stream else None))


def layer_specs(cfg: dict, seed: int) -> dict[str, TensorSpec]:
    H, I, E = cfg["hidden"], cfg["intermediate"], cfg["experts"]
    fam = cfg["family"]
    s = lambda i: seed * 1009 + i  # noqa: E731
    specs = {}
    if fam == "gemma4":
        specs["router"] = TensorSpec("router", N.F32, E, H, 1, s(1), 0.02)
        specs["gate"] = TensorSpec("gate_up", cfg["gate_type"], 2 * I, H, E, s(2))
        specs["down"] = TensorSpec("down", cfg["down_type"], H, I, E, s(3))
    elif fam == "qwen35":
        specs["router"] = TensorSpec("router", N.F32, E, H, 1, s(1), 0.02)
        specs["gate"] = TensorSpec("gate", cfg["gate_type"], I, H, E, s(2))
        specs["up"] = TensorSpec("up", cfg["gate_type"], I, H, E, s(3))
        specs["down"] = TensorSpec("down", cfg["down_type"], H, I, E, s(4))
        if cfg.get("shared"):
            specs["shared_gate"] = TensorSpec("shared_gate", cfg["gate_type"], I, H, 1, s(5))
            specs["shared_up"] = TensorSpec("shared_up", cfg["gate_type"], I, H, 1, s(6))
            specs["shared_down"] = TensorSpec("shared_down", cfg["down_type"], H, I, 1, s(7))
            specs["shared_gate_vector"] = TensorSpec("shared_gate_vector", N.F32, 1, H, 1, s(8), 0.02)
    else:
        specs["router"] = TensorSpec("router", N.BF16, E, H, 1, s(1), 0.02)
        specs["bias"] = TensorSpec("correction_bias", N.F32, 1, E, 1, s(9), 0.01)
        specs["gate"] = TensorSpec("gate", N.BF16, I, H, E, s(2), 0.02)
        specs["up"] = TensorSpec("up", N.BF16, I, H, E, s(3), 0.02)
        specs["down"] = TensorSpec("down", N.BF16, H, I, E, s(4), 0.02)
        if cfg.get("shared"):
            specs["shared_gate"] = TensorSpec("shared_gate", N.BF16, I, H, 1, s(5), 0.02)
            specs["shared_up"] = TensorSpec("shared_up", N.BF16, I, H, 1, s(6), 0.02)
            specs["shared_down"] = TensorSpec("shared_down", N.BF16, H, I, 1, s(7), 0.02)
    return specs


def vectors(cfg: dict, seed: int) -> dict[str, np.ndarray]:
    """Small per-feature vectors (Gemma norm scales, expert scales): U[0.5, 1.5)."""
    rng = np.random.default_rng(seed * 7919 + 17)
    out = {}
    if cfg["family"] == "gemma4":
        out["router_scale"] = rng.uniform(0.5, 1.5, cfg["hidden"]).astype(np.float32)
        out["routed_pre_norm"] = rng.uniform(0.5, 1.5, cfg["hidden"]).astype(np.float32)
        out["expert_scale"] = rng.uniform(0.5, 1.5, cfg["experts"]).astype(np.float32)
    return out


def zipf_bias(experts: int, s: float, seed: int) -> np.ndarray:
    """log of Zipf(s) weights over a seeded permutation of the experts (skewed routing)."""
    rng = np.random.default_rng(seed * 31 + 7)
    ranks = rng.permutation(experts) + 1
    z = 1.0 / ranks.astype(np.float64) ** s
    z /= z.sum()
    return np.log(z).astype(np.float32)


def input_spec(cfg: dict, tokens: int, seed: int) -> TensorSpec:
    kind = N.BF16 if cfg["family"] == "glm52" else N.F32
    return TensorSpec("x", kind, tokens, cfg["hidden"], 1, seed * 1009 + 99, 1.0)


@dataclass
class SyntheticLayer:
    """A device-resident synthetic layer plus the means to rebuild its bytes on the host."""

    name: str
    cfg: dict
    seed: int
    ctx: CudaContext
    specs: dict
    vecs: dict
    buffers: dict = field(default_factory=dict)
    layer: MoeLayer | None = None
    logit_bias: np.ndarray | None = None

    def ptr(self, key: str) -> int:
        return self.buffers[key].device_pointer if key in self.buffers else 0

    def host_weights(self, experts=None, fill=None, router_only=False) -> dict:
        """Oracle inputs: full tensors (or the listed experts, others zero). `fill` as in
        `TensorSpec.host`. `router_only` leaves out every expert and shared-expert tensor
        (for `oracle.route`, which reads the router alone)."""
        cfg = self.cfg
        w = dict(hidden=cfg["hidden"], intermediate=cfg["intermediate"], experts=cfg["experts"],
                 top_k=cfg["top_k"], epsilon=cfg.get("epsilon", 1e-6))
        for key, spec in self.specs.items():
            if router_only and key not in ("router", "bias"):
                continue
            if experts is None or spec.experts == 1:
                w[key] = spec.host(fill=fill)
            else:
                full = np.zeros(spec.nbytes, dtype=np.uint8)
                for e in experts:
                    full[e * spec.expert_bytes:(e + 1) * spec.expert_bytes] = spec.host(e, fill)
                w[key] = full
        for key in ("router", "shared_gate_vector"):
            if key in w and self.specs[key].kind == N.F32:
                w[key] = w[key].view(np.float32)
        if "bias" in w:
            w["correction_bias"] = w.pop("bias").view(np.float32)
        w.update(self.vecs)
        if self.logit_bias is not None:
            w["router_logit_bias"] = self.logit_bias
        fam = cfg["family"]
        if fam == "gemma4":
            w["gate_up_type"], w["gate_up"] = cfg["gate_type"], w.pop("gate", None)
            w["down_type"] = cfg["down_type"]
        elif fam == "qwen35":
            w["gate_type"] = w["up_type"] = cfg["gate_type"]
            w["down_type"] = cfg["down_type"]
            if cfg.get("shared"):
                w["shared_intermediate"] = cfg["intermediate"]
        else:
            w["weight_type"] = N.BF16
            w["n_groups"], w["topk_groups"] = cfg["n_groups"], cfg["topk_groups"]
            w["routed_scale"], w["normalize"] = cfg["routed_scale"], cfg["normalize"]
            if cfg.get("shared"):
                w["shared_intermediate"] = cfg["intermediate"]
        return w

    def inputs(self, tokens: int, seed: int, fill=None) -> tuple[TensorSpec, np.ndarray]:
        spec = input_spec(self.cfg, tokens, seed)
        return spec, spec.host(fill=fill)

    def close(self):
        if self.layer is not None:
            self.layer.close()
            self.layer = None
        for b in self.buffers.values():
            b.free()
        self.buffers.clear()
        if getattr(self, "cache", None) is not None:
            self.cache.close()
            self.cache = None
        if getattr(self, "pool", None) is not None:
            self.pool.free()
            self.pool = None


def _desc(sl: SyntheticLayer) -> N.MoeDesc:
    """The layer descriptor over `sl`'s device buffers."""
    cfg = sl.cfg
    d = N.MoeDesc()
    d.family = FAMILIES[cfg["family"]]
    d.hidden, d.intermediate, d.experts, d.top_k = (cfg["hidden"], cfg["intermediate"],
                                                    cfg["experts"], cfg["top_k"])
    d.n_groups = cfg.get("n_groups", 1)
    d.topk_groups = cfg.get("topk_groups", 1)
    d.normalize_topk = int(cfg.get("normalize", False))
    d.routed_scale = cfg.get("routed_scale", 1.0)
    d.epsilon = cfg.get("epsilon", 1e-6)
    glm = cfg["family"] == "glm52"
    d.input_type = N.BF16 if glm else N.F32
    d.router_type = N.BF16 if glm else N.F32
    d.router = sl.ptr("router")
    d.correction_bias = sl.ptr("bias") or None
    d.router_scale = sl.ptr("router_scale") or None
    d.routed_pre_norm = sl.ptr("routed_pre_norm") or None
    d.expert_scale = sl.ptr("expert_scale") or None
    d.gate_type = cfg["gate_type"]
    d.up_type = cfg["gate_type"]
    d.down_type = cfg["down_type"]
    d.gate = sl.ptr("gate")
    d.up = sl.ptr("up") or None
    d.down = sl.ptr("down")
    if cfg.get("shared"):
        d.shared_intermediate = cfg["intermediate"]
        d.shared_gate = sl.ptr("shared_gate")
        d.shared_up = sl.ptr("shared_up")
        d.shared_down = sl.ptr("shared_down")
        d.shared_gate_vector = sl.ptr("shared_gate_vector") or None
    d.router_logit_bias = sl.ptr("router_logit_bias") or None
    return d


def build_layer(ctx: CudaContext, name: str, seed: int = 1, logit_bias=None,
                expert_range=None, edit=None) -> SyntheticLayer:
    """A device-resident synthetic layer. `expert_range=(first, count)` builds a shard
    holding only those experts' weights (the same bytes as in the whole layer) for
    expert parallelism; the router and shared expert stay whole. `edit(sl)` runs after
    the device buffers are filled and before the layer is created, so it may overwrite
    their bytes (through `sl.buffers[key].write`)."""
    cfg = dict(CONFIGS[name])
    specs = layer_specs(cfg, seed)
    vecs = vectors(cfg, seed)
    sl = SyntheticLayer(name, cfg, seed, ctx, specs, vecs)
    for key, spec in specs.items():
        if expert_range is not None and spec.experts > 1:
            first, count = expert_range
            buf = ctx.new_owned_buffer(count * spec.expert_bytes)
            spec.device_fill(buf.device_pointer, expert=first, count=count)
        else:
            buf = ctx.new_owned_buffer(spec.nbytes)
            spec.device_fill(buf.device_pointer)
        sl.buffers[key] = buf
    for key, v in vecs.items():
        sl.buffers[key] = ctx.map_read_only(v)
    if logit_bias is not None:
        sl.logit_bias = np.ascontiguousarray(logit_bias, dtype=np.float32)
        sl.buffers["router_logit_bias"] = ctx.map_read_only(sl.logit_bias)
    ctx.synchronize()
    if edit is not None:
        edit(sl)
        ctx.synchronize()
    d = _desc(sl)
    sl.layer = MoeLayer(ctx, d, expert_range=expert_range)
    return sl


GEMMA_FFN_WIDTH = {"gemma4": 2112, "gemma4-small": 192, "gemma4-small-q8": 192}


@dataclass
class SyntheticGemmaBlock:
    """A synthetic Gemma 4 feed-forward block: a routed layer plus the dense shared FFN
    (Q4_K gate / up [W][H], Q5_0 down [H][W]; Gemma-4-26B's feed_forward_length is 2112),
    the four norm vectors U[0.5, 1.5) and a layer output scale."""

    sl: SyntheticLayer
    width: int
    specs: dict
    norms: dict
    layer_scale: float
    buffers: dict = field(default_factory=dict)
    block: object = None

    def host_ffn(self) -> dict:
        """Oracle inputs of the shared FFN and norms (oracle.gemma_ffn_block's `f`)."""
        f = dict(width=self.width, gate_type=self.specs["gate"].kind,
                 up_type=self.specs["up"].kind, down_type=self.specs["down"].kind,
                 gate=self.specs["gate"].host(), up=self.specs["up"].host(),
                 down=self.specs["down"].host(), layer_output_scale=self.layer_scale)
        f.update(self.norms)
        return f

    def close(self):
        if self.block is not None:
            self.block.close()
            self.block = None
        for b in self.buffers.values():
            b.free()
        self.buffers.clear()
        self.sl.close()


def build_gemma_block(ctx: CudaContext, name: str = "gemma4", seed: int = 1,
                      logit_bias=None) -> SyntheticGemmaBlock:
    from .moe import GemmaFfnBlock, GemmaFfnDesc
    cfg = CONFIGS[name]
    H, W = cfg["hidden"], GEMMA_FFN_WIDTH[name]
    sl = build_layer(ctx, name, seed, logit_bias=logit_bias)
    s = lambda i: seed * 1009 + 50 + i  # noqa: E731
    specs = {"gate": TensorSpec("ffn_gate", cfg["gate_type"], W, H, 1, s(1)),
             "up": TensorSpec("ffn_up", cfg["gate_type"], W, H, 1, s(2)),
             "down": TensorSpec("ffn_down", cfg["down_type"], H, W, 1, s(3))}
    rng = np.random.default_rng(seed * 7919 + 23)
    norms = {n: rng.uniform(0.5, 1.5, H).astype(np.float32)
             for n in ("feed_forward_norm", "shared_post_norm", "routed_post_norm",
                       "post_feed_forward_norm")}
    gb = SyntheticGemmaBlock(sl, W, specs, norms, float(rng.uniform(0.5, 1.5)))
    for key, spec in specs.items():
        buf = ctx.new_owned_buffer(spec.nbytes)
        spec.device_fill(buf.device_pointer)
        gb.buffers[key] = buf
    for key, v in norms.items():
        gb.buffers[key] = ctx.map_read_only(v)
    ctx.synchronize()
    d = GemmaFfnDesc()
    d.width = W
    d.gate_type = d.up_type = cfg["gate_type"]
    d.down_type = cfg["down_type"]
    d.gate, d.up, d.down = (gb.buffers[k].device_pointer for k in ("gate", "up", "down"))
    for key in norms:
        setattr(d, key, gb.buffers[key].device_pointer)
    d.layer_output_scale = gb.layer_scale
    gb.block = GemmaFfnBlock(sl.layer, d)
    return gb


EXPERT_TENSORS = {"gemma4": ("gate", "down"), "qwen35": ("gate", "up", "down"),
                  "glm52": ("gate", "up", "down")}


def build_cached_layer(ctx: CudaContext, name: str, seed: int = 1, slots: int = 8,
                       global_clock: bool | None = None, logit_bias=None,
                       input_type: int | None = None) -> SyntheticLayer:
    """A synthetic layer whose experts are out of core: the expert tensors sit in
    page-locked host memory in the reference's layout ([experts][rows][blocks] per
    tensor, tensors one after another), and the layer holds `slots` of them in HBM
    through an expert cache (GLM rules for the GLM family unless `global_clock` says
    otherwise). The router, shared expert and vectors are device-resident as in
    `build_layer`; `sl.cache` is the cache and `sl.pool` the host source."""
    from .cache import CachedMoeLayer, ExpertCache, PinnedHost, layout
    cfg = dict(CONFIGS[name])
    specs = layer_specs(cfg, seed)
    vecs = vectors(cfg, seed)
    sl = SyntheticLayer(name, cfg, seed, ctx, specs, vecs)
    keys = EXPERT_TENSORS[cfg["family"]]
    E = cfg["experts"]
    sizes = [specs[k].expert_bytes for k in keys]
    pool = PinnedHost(ctx, E * sum(sizes))
    offsets, off = [], 0
    for k, n in zip(keys, sizes):
        pool.array(off, E * n)[:] = specs[k].host()
        offsets.append(off)
        off += E * n
    if global_clock is None:
        global_clock = cfg["family"] == "glm52"
    sl.cache = ExpertCache(ctx, [layout(E, sizes, host=pool.pointer, offsets=offsets)], slots,
                           global_clock=global_clock)
    sl.pool = pool
    for key, spec in specs.items():
        if key in keys:
            continue
        buf = ctx.new_owned_buffer(spec.nbytes)
        spec.device_fill(buf.device_pointer)
        sl.buffers[key] = buf
    for key, v in vecs.items():
        sl.buffers[key] = ctx.map_read_only(v)
    if logit_bias is not None:
        sl.logit_bias = np.ascontiguousarray(logit_bias, dtype=np.float32)
        sl.buffers["router_logit_bias"] = ctx.map_read_only(sl.logit_bias)
    ctx.synchronize()
    d = _desc(sl)
    if input_type is not None:
        d.input_type = input_type
    sl.layer = CachedMoeLayer(ctx, d, sl.cache, 0)
    return sl
