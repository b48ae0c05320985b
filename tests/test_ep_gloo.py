"""Expert parallelism host logic on CPU: two gloo ranks, each holding half the experts.

The EP driver (diskmule_b200/ep.py) runs with a backend whose compute steps are the
oracle's GLM restatement (src/glm52/cpu.rs:711-778: router, sigmoid top-k, expert MLP,
selection-order combine); the sharded result must equal the single-process oracle
block bit for bit, because every expert output and the combine order are identical.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from diskmule_b200 import _native as N
from diskmule_b200.ep import ExpertParallel, Routed, exchange_plan
from diskmule_b200.synthetic import CONFIGS, input_spec, layer_specs
from oracle import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bf16_rows(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return raw.view(np.uint16).reshape(rows, cols)


class OracleGlmBackend:
    """GLM block steps computed by the oracle for experts [first, first + count)."""

    def __init__(self, cfg, specs, first, count):
        self.cfg, self.first, self.count = cfg, first, count
        H, I = cfg["hidden"], cfg["intermediate"]
        self.H, self.I = H, I
        self.router = specs["router"].host()
        self.bias = specs["bias"].host().view(np.float32)
        self.gate = [specs["gate"].host(e) for e in range(first, first + count)]
        self.up = [specs["up"].host(e) for e in range(first, first + count)]
        self.down = [specs["down"].host(e) for e in range(first, first + count)]
        self.sh = (specs["shared_gate"].host(), specs["shared_up"].host(), specs["shared_down"].host())
        self.has_shared = True

    def local_experts(self):
        return self.first, self.count

    def route(self, x: torch.Tensor) -> Routed:
        cfg = self.cfg
        xs = x.numpy().astype(np.float32)
        T, k = xs.shape[0], cfg["top_k"]
        idx = np.zeros((T, k), np.int32)
        w = np.zeros((T, k), np.float32)
        for t in range(T):
            rc, lg = O.glm_matvec(N.BF16, cfg["experts"], self.H, self.router, xs[t])
            assert rc == O.OK
            rc, i, ww = O.glm_select(lg, self.bias, k, cfg["n_groups"], cfg["topk_groups"],
                                     cfg["normalize"])
            assert rc == O.OK
            idx[t], w[t] = i, ww
        return Routed(torch.from_numpy(idx), torch.from_numpy(w))

    def rows(self, x, routed):
        return x

    def _mlp(self, gate, up, down, x, act):
        _, g = O.glm_matvec(N.BF16, self.I, self.H, gate, x)
        _, u = O.glm_matvec(N.BF16, self.I, self.H, up, x)
        h = np.array([act(float(v)) for v in g], dtype=np.float32) * u
        _, out = O.glm_matvec(N.BF16, self.H, self.I, down, h)
        return out

    def expert_rows(self, rows: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        L = O.lib()
        xs = rows.numpy().astype(np.float32)
        out = np.zeros((xs.shape[0], self.H), np.float32)
        for r in range(xs.shape[0]):
            e = int(ids[r])
            if e == self.count:
                out[r] = self._mlp(*self.sh, xs[r], L.dmo_glm_silu)
            else:
                out[r] = self._mlp(self.gate[e], self.up[e], self.down[e], xs[r],
                                   L.dmo_glm_cached_silu)
        return torch.from_numpy(out)

    def combine(self, routed: Routed, pair_out: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        T, k = routed.sel_idx.shape
        po = pair_out.numpy()
        w = routed.sel_w.numpy()
        scale = np.float32(cfg["routed_scale"])
        y = np.zeros((T, self.H), np.float32)
        for t in range(T):
            for j in range(k):  # selection order, w*x*scale then add (src/glm52/cpu.rs:769-771)
                y[t] = y[t] + po[t * k + j] * w[t, j] * scale
            y[t] = y[t] + po[T * k + t]
        return torch.from_numpy(y)


def _rank_main(rank, world, port, name, tokens, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = dict(CONFIGS[name])
        specs = layer_specs(cfg, seed=3)
        E = cfg["experts"]
        per = E // world
        backend = OracleGlmBackend(cfg, specs, rank * per, per)
        raw = input_spec(cfg, tokens, 5).host()
        x = _bf16_rows(raw, tokens, cfg["hidden"])
        x32 = (x.astype(np.uint32) << 16).view(np.float32)
        mine = np.array_split(np.arange(tokens), world)[rank]
        ep = ExpertParallel(backend, E, cfg["top_k"])
        y = ep.forward(torch.from_numpy(x32[mine].copy()))
        result[rank] = (mine, y.numpy())
    finally:
        dist.destroy_process_group()


def _single_process(name, tokens):
    cfg = dict(CONFIGS[name])
    specs = layer_specs(cfg, seed=3)
    raw = input_spec(cfg, tokens, 5).host()
    x32 = (_bf16_rows(raw, tokens, cfg["hidden"]).astype(np.uint32) << 16).view(np.float32)
    w = dict(hidden=cfg["hidden"], intermediate=cfg["intermediate"], experts=cfg["experts"],
             top_k=cfg["top_k"], weight_type=N.BF16, n_groups=cfg["n_groups"],
             topk_groups=cfg["topk_groups"], routed_scale=cfg["routed_scale"],
             normalize=cfg["normalize"], shared_intermediate=cfg["intermediate"])
    for key, spec in specs.items():
        w[key] = spec.host()
    w["correction_bias"] = w.pop("bias").view(np.float32)
    rc, y, idx, wt = O.glm_moe(w, x32)
    assert rc == O.OK
    return y


def test_exchange_plan_groups_pairs_by_owner():
    sel = torch.tensor([[5, 0], [3, 7], [4, 1]])
    order, counts, local = exchange_plan(sel, experts=8, world=2)
    # owners: 5->1, 0->0, 3->0, 7->1, 4->1, 1->0; stable by pair index within an owner
    assert order.tolist() == [1, 2, 5, 0, 3, 4]
    assert counts.tolist() == [3, 3]
    assert local.tolist() == [0, 3, 1, 1, 3, 0]


@pytest.mark.parametrize("name,tokens", [("glm52-small", 6)])
def test_two_rank_expert_parallel_equals_single_process(name, tokens):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, name, tokens, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    y_ref = _single_process(name, tokens)
    for r in range(2):
        mine, y = result[r]
        assert np.array_equal(y, y_ref[mine]), np.abs(y - y_ref[mine]).max()
