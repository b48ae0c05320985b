"""Expert parallelism on the GPU.

Single GPU: two shard layers (each half the experts) composed by hand — route, ship
rows to the owning shard, expert products, combine — must match the oracle exactly in
the selections and within the 1e-3 relative-L2 bar in the outputs, like the whole
layer. Two GPUs (skipped with fewer): the NCCL driver of diskmule_b200/ep.py.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from diskmule_b200.ep import exchange_plan
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import CONFIGS, build_layer, input_spec
from oracle import oracle as O

from test_gpu_parity import check, device_input, as_f32, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


@pytest.mark.parametrize("name,T", [("glm52-small", 40), ("glm52-small", 300),
                                     ("qwen35-small", 64), ("gemma4-small", 64)])
def test_two_shards_on_one_gpu_match_the_oracle(ctx, name, T):
    cfg = CONFIGS[name]
    E, k, H = cfg["experts"], cfg["top_k"], cfg["hidden"]
    per = E // 2
    shards = [build_layer(ctx, name, seed=2, expert_range=(r * per, per)) for r in range(2)]
    full = build_layer(ctx, name, seed=2)
    try:
        spec, raw = full.inputs(T, seed=7)
        xh = device_input(spec, raw, T)
        x = torch.from_numpy(np.ascontiguousarray(xh)).cuda()
        stream = torch.cuda.current_stream().cuda_stream
        shared = bool(cfg.get("shared"))
        cols = E + (1 if cfg["family"] == "qwen35" and shared else 0)
        sel = torch.empty((T, k), dtype=torch.int32, device="cuda")
        w = torch.empty((T, k), dtype=torch.float32, device="cuda")
        ein = torch.empty((T, H), dtype=torch.float32, device="cuda") if cfg["family"] == "gemma4" else None
        logits = torch.empty((T, cols), dtype=torch.float32, device="cuda")
        s0 = shards[0].layer
        s0.route(x.data_ptr(), T, sel.data_ptr(), w.data_ptr(), ein.data_ptr() if ein is not None else 0,
                 logits.data_ptr(), stream)
        rows = ein if ein is not None else x
        order, counts, local = exchange_plan(sel.cpu(), E, 2)
        tok = torch.div(order, k, rounding_mode="floor").cuda()
        back = torch.empty((T * k, H), dtype=torch.float32, device="cuda")
        start = 0
        for r, n in enumerate(counts.tolist()):
            if n == 0:
                continue
            sl_rows = rows.index_select(0, tok[start:start + n]).contiguous()
            ids = local[start:start + n].cuda()
            out = torch.empty((n, H), dtype=torch.float32, device="cuda")
            shards[r].layer.expert_rows(sl_rows.data_ptr(), ids.data_ptr(), n, out.data_ptr(), stream)
            back[start:start + n] = out
            start += n
        pair_out = torch.empty((T * k + (T if shared else 0), H), dtype=torch.float32, device="cuda")
        pair_out.index_copy_(0, order.cuda(), back)
        if shared:
            ids = torch.full((T,), per, dtype=torch.int32, device="cuda")
            sh = torch.empty((T, H), dtype=torch.float32, device="cuda")
            s0.expert_rows(rows.contiguous().data_ptr(), ids.data_ptr(), T, sh.data_ptr(), stream)
            pair_out[T * k:] = sh
        y = torch.empty((T, H), dtype=torch.float32, device="cuda")
        s0.combine_rows(T, sel.data_ptr(), w.data_ptr(), pair_out.data_ptr(), y.data_ptr(),
                        logits.data_ptr(), stream)
        torch.cuda.synchronize()
        y_ref, idx_ref, wt_ref = run_oracle(full, as_f32(spec, raw, T))
        check(y.cpu().numpy(), sel.cpu().numpy().astype(np.uint32), w.cpu().numpy(), y_ref,
              idx_ref, wt_ref)
    finally:
        for s in shards:
            s.close()
        full.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, name, T, out):
    import torch.distributed as dist
    from diskmule_b200.ep import ExpertParallel, cuda_backend_for
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        cfg = CONFIGS[name]
        per = cfg["experts"] // world
        ctx = CudaContext(rank)
        sl = build_layer(ctx, name, seed=2, expert_range=(rank * per, per))
        spec = input_spec(cfg, T, 7)
        raw = spec.host()
        xh = raw.view(np.uint16).reshape(T, -1)
        mine = np.array_split(np.arange(T), world)[rank]
        x = torch.from_numpy(np.ascontiguousarray(xh[mine]).view(np.int16)).cuda().view(torch.bfloat16)
        ep = ExpertParallel(cuda_backend_for(sl), cfg["experts"], cfg["top_k"])
        y = ep.forward(x)
        torch.cuda.synchronize()
        out[rank] = (mine, y.cpu().numpy())
        sl.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_expert_parallel_matches_the_oracle():
    import torch.multiprocessing as mp
    name, T = "glm52-small", 64
    mpc = mp.get_context("spawn")
    out = mpc.Manager().dict()
    port = _free_port()
    procs = [mpc.Process(target=_nccl_rank, args=(r, 2, port, name, T, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ctx = CudaContext(0)
    full = build_layer(ctx, name, seed=2)
    try:
        spec, raw = full.inputs(T, seed=7)
        y_ref, idx_ref, wt_ref = run_oracle(full, as_f32(spec, raw, T))
        y = np.zeros_like(y_ref)
        for r in range(2):
            mine, yr = out[r]
            y[mine] = yr
        layer = float(np.linalg.norm((y - y_ref).astype(np.float64)) / np.linalg.norm(y_ref))
        assert layer <= 1e-3, layer
    finally:
        full.close()
        ctx.close()


# ---------------------------------------------------------------------------
# peer-memory data plane (dm_ep_*)
# ---------------------------------------------------------------------------

def _peer_group(ctx, name, world, tmax, seed=2):
    from diskmule_b200.ep import PeerExpertParallel
    cfg = CONFIGS[name]
    per = cfg["experts"] // world
    shards = [build_layer(ctx, name, seed=seed, expert_range=(r * per, per)) for r in range(world)]
    eps = [PeerExpertParallel(s.layer, r, world, tmax) for r, s in enumerate(shards)]
    PeerExpertParallel.connect_local(eps)
    return shards, eps


def _peer_forward(eps, xs, ks):
    """One forward of every rank, phase by phase in one stream (ranks on one GPU)."""
    T_all = [x.shape[0] for x in xs]
    for ep, x in zip(eps, xs):
        ep.dispatch(x)
    for ep in eps:
        ep.experts()
    out = []
    for ep, T in zip(eps, T_all):
        y = torch.empty((T, ep.hidden), dtype=torch.float32, device="cuda")
        i = torch.empty((T, ks), dtype=torch.int32, device="cuda")
        w = torch.empty((T, ks), dtype=torch.float32, device="cuda")
        ep.combine(y, i, w)
        out.append((y, i, w))
    torch.cuda.synchronize()
    for ep in eps:
        ep.status()
    return [(y.cpu().numpy(), i.cpu().numpy().view(np.uint32), w.cpu().numpy()) for y, i, w in out]


@pytest.mark.parametrize("name,world,splits", [
    ("glm52-small", 2, (32, 32)),
    ("glm52-small", 4, (80, 75, 0, 100)),      # a rank without tokens
    ("glm52-small-flat", 2, (300, 212)),
    ("qwen35-small", 2, (48, 16)),
    ("gemma4-small", 2, (40, 24)),
])
def test_peer_ranks_on_one_gpu_match_the_oracle(ctx, name, world, splits):
    cfg = CONFIGS[name]
    k = cfg["top_k"]
    tmax = max(splits)
    shards, eps = _peer_group(ctx, name, world, tmax)
    full = build_layer(ctx, name, seed=2)
    try:
        for rep, seed in enumerate((7, 8)):  # two forwards: epochs advance, buffers reused
            T = sum(splits)
            spec, raw = full.inputs(T, seed=seed)
            xh = device_input(spec, raw, T)
            bounds = np.cumsum((0,) + tuple(splits))
            xs = [torch.from_numpy(np.ascontiguousarray(xh[a:b])).cuda() for a, b in
                  zip(bounds[:-1], bounds[1:])]
            if spec.kind == 30:
                xs = [x.view(torch.bfloat16) if x.dtype == torch.int16 else x for x in xs]
            res = _peer_forward(eps, xs, k)
            y = np.concatenate([r[0] for r in res])
            idx = np.concatenate([r[1] for r in res])
            wt = np.concatenate([r[2] for r in res])
            y_ref, idx_ref, wt_ref = run_oracle(full, as_f32(spec, raw, T))
            check(y, idx, wt, y_ref, idx_ref, wt_ref)
    finally:
        for ep in eps:
            ep.close()
        for s in shards:
            s.close()
        full.close()


def test_peer_wait_for_a_missing_rank_times_out(ctx):
    """Rank 1 never sends: rank 0's bounded waits give up (about two seconds each), the
    forward reports DM_ERR_TIMEOUT and the context keeps working."""
    from diskmule_b200._native import DmError, ERR_TIMEOUT
    name = "glm52-small"
    shards, eps = _peer_group(ctx, name, 2, 16)
    try:
        spec, raw = shards[0].inputs(16, seed=3)
        x = torch.from_numpy(np.ascontiguousarray(device_input(spec, raw, 16))).cuda()
        eps[0].dispatch(x.view(torch.bfloat16))
        eps[0].experts()
        eps[0].combine()
        torch.cuda.synchronize()
        with pytest.raises(DmError) as err:
            eps[0].status()
        assert err.value.status == ERR_TIMEOUT
    finally:
        for ep in eps:
            ep.close()
        for s in shards:
            s.close()
    full = build_layer(ctx, name, seed=2)
    try:
        spec, raw = full.inputs(8, seed=4)
        y, idx, wt = full.layer.forward_host(device_input(spec, raw, 8))
        y_ref, idx_ref, wt_ref = run_oracle(full, as_f32(spec, raw, 8))
        check(y, idx, wt, y_ref, idx_ref, wt_ref)
    finally:
        full.close()


def _peer_rank(rank, world, port, name, splits, out):
    import torch.distributed as dist
    from diskmule_b200.ep import PeerExpertParallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    # the handle exchange only: gloo on the host, no collective on the data path
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = CONFIGS[name]
        per = cfg["experts"] // world
        ctx = CudaContext(rank)
        sl = build_layer(ctx, name, seed=2, expert_range=(rank * per, per))
        ep = PeerExpertParallel(sl.layer, rank, world, max(splits))
        ep.connect_ipc()
        results = []
        for seed in (7, 8, 9):
            T = sum(splits)
            raw = input_spec(cfg, T, seed).host()
            xh = raw.view(np.uint16).reshape(T, -1)
            a = sum(splits[:rank])
            x = torch.from_numpy(np.ascontiguousarray(xh[a:a + splits[rank]]).view(np.int16)).cuda()
            y = ep.forward(x.view(torch.bfloat16))
            torch.cuda.synchronize()
            ep.status()
            results.append(y.cpu().numpy())
        out[rank] = results
        dist.barrier()  # no rank unmaps or frees while another still works
        ep.close()
        dist.barrier()
        sl.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_expert_parallel_on_two_gpus_matches_the_oracle():
    import torch.multiprocessing as mp
    name, splits = "glm52-small", (40, 24)
    mpc = mp.get_context("spawn")
    out = mpc.Manager().dict()
    port = _free_port()
    procs = [mpc.Process(target=_peer_rank, args=(r, 2, port, name, splits, out))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ctx = CudaContext(0)
    full = build_layer(ctx, name, seed=2)
    try:
        T = sum(splits)
        for i, seed in enumerate((7, 8, 9)):
            spec, raw = full.inputs(T, seed=seed)
            y_ref, _, _ = run_oracle(full, as_f32(spec, raw, T))
            y = np.concatenate([out[0][i], out[1][i]])
            layer = float(np.linalg.norm((y - y_ref).astype(np.float64)) / np.linalg.norm(y_ref))
            assert layer <= 1e-3, (i, layer)
    finally:
        full.close()
        ctx.close()
