"""Expert parallelism: experts sharded over the ranks of a process group.

Two data planes share the same split of the block:

* `PeerExpertParallel` (the default): the library's own kernels move the token rows
  and the expert outputs by direct stores into the other GPUs' memory over NVLink
  (CUDA IPC mappings of each rank's exchange region) with device-side epoch flags, so
  one forward has no host synchronisation and no collective-library call
  (dm_ep_* in include/diskmule_cuda.h).
* `ExpertParallel`: the collective baseline, torch.distributed all_to_all_single
  (NCCL on GPUs, gloo on CPU in the tests), described below.

Rank g holds experts [g*E/n, (g+1)*E/n) of every layer plus the replicated router and
shared expert, and routes its own T/n tokens. One forward (the GLM block of
src/glm52/cpu.rs:711-778 split across GPUs):

  1. route the local tokens (router + top-k, global expert ids);
  2. order the (token, slot) pairs by owning rank (stable, so pair order is kept per
     rank) and exchange the per-rank pair counts (all-to-all);
  3. all-to-all the token rows and the expert ids local to the receiver;
  4. run the received rows through the local experts (unweighted outputs);
  5. all-to-all the outputs back and put them in pair order;
  6. run the shared expert on the local tokens and combine in selection order.

The collectives are torch.distributed all_to_all_single (NCCL over NVLink on GPUs,
gloo on CPU in the tests); the compute steps are a backend's. `CudaBackend` runs them
through the C ABI (dm_moe_route / dm_moe_expert_rows / dm_moe_combine_rows).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from ._native import check


def exchange_plan(sel_idx: torch.Tensor, experts: int, world: int):
    """Destination rank of every pair, the pair order grouped by destination and the
    per-destination counts. Pairs are p = t*k + j in row-major order of sel_idx."""
    flat = sel_idx.reshape(-1).long()
    per = experts // world
    dest = torch.div(flat, per, rounding_mode="floor")
    order = torch.argsort(dest, stable=True)
    counts = torch.bincount(dest, minlength=world)
    local_ids = (flat - dest * per)[order].to(torch.int32)
    return order, counts, local_ids


def all_to_all(send: torch.Tensor, send_counts: list[int], recv_counts: list[int], group=None):
    """Variable-size all-to-all along dim 0 (2-byte integer rows travel as bf16 bits:
    NCCL has no 16-bit integer type)."""
    wire = send.view(torch.bfloat16) if send.dtype in (torch.uint16, torch.int16) else send
    recv = wire.new_empty((sum(recv_counts),) + tuple(wire.shape[1:]))
    dist.all_to_all_single(recv, wire.contiguous(), recv_counts, send_counts, group=group)
    return recv.view(send.dtype) if wire is not send else recv


class ExpertParallel:
    """EP forward over `backend` (route, rows, expert_rows, combine, local_experts)."""

    def __init__(self, backend, experts: int, top_k: int, group=None):
        self.backend = backend
        self.experts = experts
        self.top_k = top_k
        self.group = group
        self.world = dist.get_world_size(group)
        if experts % self.world:
            raise ValueError(f"{experts} experts do not split over {self.world} ranks")

    def forward(self, x: torch.Tensor, marks=None) -> torch.Tensor:
        """One expert-parallel forward of this rank's tokens x [T, H]. `marks`, when
        given, is called with a stage name at every stage boundary (profiling)."""
        b, k = self.backend, self.top_k
        mark = marks or (lambda name: None)
        T = x.shape[0]
        mark("route")
        routed = b.route(x)
        mark("exchange")
        order, counts, local_ids = exchange_plan(routed.sel_idx, self.experts, self.world)
        counts_dev = counts.to(x.device)
        recv_counts_dev = torch.empty_like(counts_dev)
        dist.all_to_all_single(recv_counts_dev, counts_dev, group=self.group)
        send_counts = counts.tolist()
        recv_counts = recv_counts_dev.cpu().tolist()
        rows = b.rows(x, routed)                       # [T, H] rows the experts consume
        send_rows = rows.index_select(0, torch.div(order, k, rounding_mode="floor").to(rows.device))
        recv_rows = all_to_all(send_rows, send_counts, recv_counts, self.group)
        recv_ids = all_to_all(local_ids.to(x.device), send_counts, recv_counts, self.group)
        mark("experts")
        out = b.expert_rows(recv_rows, recv_ids)       # [R, H] f32
        self.last_rows = int(recv_rows.shape[0]) + (T if b.has_shared else 0)
        P = T * k
        shared = b.has_shared
        pair_out = out.new_empty((P + (T if shared else 0), out.shape[1]))
        if shared:
            _, local = b.local_experts()
            ids = torch.full((T,), local, dtype=torch.int32, device=x.device)
            pair_out[P:] = b.expert_rows(rows, ids)
        mark("return")
        back = all_to_all(out, recv_counts, send_counts, self.group)
        pair_out[:P].index_copy_(0, order.to(back.device), back)
        mark("combine")
        y = b.combine(routed, pair_out)
        mark("end")
        self.last_routed = routed
        return y

    def last_selection(self, n: int):
        """Selected expert ids and weights of the first n tokens of the last forward."""
        r = self.last_routed
        return (r.sel_idx[:n].cpu().numpy().view(np.uint32), r.sel_w[:n].cpu().numpy())

    def profile_step(self, x: torch.Tensor):
        """One forward with CUDA events at its stage boundaries: (kernel launches of the
        step counted by the backend, {stage: ms})."""
        ev = {}
        names = []
        stream = torch.cuda.current_stream()

        def mark(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            ev[name] = e
            names.append(name)

        self.backend.launches = 0
        self.forward(x, marks=mark)
        torch.cuda.synchronize()
        stage = {a: ev[a].elapsed_time(ev[b]) for a, b in zip(names, names[1:])}
        return self.backend.launches, stage

    def forward_host_stream(self, x_host: torch.Tensor, y_host, steps: int):
        """`steps` forwards of the page-locked host rows x_host, each output copied back
        into y_host[i % len(y_host)]: the input copy of step i+1 runs on a side stream
        while step i computes, and the output copy of step i on another."""
        dev = torch.device("cuda", torch.cuda.current_device())
        cs = torch.cuda.current_stream()
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        bufs = [torch.empty_like(x_host, device=dev) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        with torch.cuda.stream(s_in):
            bufs[0].copy_(x_host, non_blocking=True)
            ready[0].record(s_in)
        for i in range(steps):
            j = i & 1
            if i + 1 < steps:
                with torch.cuda.stream(s_in):
                    if i >= 1:
                        s_in.wait_event(done[1 - j])
                    bufs[1 - j].copy_(x_host, non_blocking=True)
                    ready[1 - j].record(s_in)
            cs.wait_event(ready[j])
            y = self.forward(bufs[j])
            done[j].record(cs)
            s_out.wait_stream(cs)
            with torch.cuda.stream(s_out):
                y_host[i % len(y_host)].copy_(y, non_blocking=True)
                y.record_stream(s_out)
        torch.cuda.synchronize()


class Routed:
    """The result of a backend's route step."""

    def __init__(self, sel_idx, sel_w, expert_in=None, logits=None):
        self.sel_idx, self.sel_w, self.expert_in, self.logits = sel_idx, sel_w, expert_in, logits


class CudaBackend:
    """The EP compute steps on a `MoeLayer` built for this rank's expert range."""

    def __init__(self, layer, family: str, hidden: int, top_k: int, router_columns: int,
                 shared: bool):
        self.layer = layer
        self.family = family
        self.hidden = hidden
        self.top_k = top_k
        self.router_columns = router_columns
        self.has_shared = shared
        self.launches = 0  # kernels launched through this backend (a count for benchmarks)

    def _stream(self) -> int:
        return torch.cuda.current_stream().cuda_stream

    def local_experts(self):
        return self.layer.local_experts()

    def route(self, x: torch.Tensor) -> Routed:
        T = x.shape[0]
        sel_idx = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        sel_w = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        expert_in = (torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
                     if self.family == "gemma4" else None)
        logits = (torch.empty((T, self.router_columns), dtype=torch.float32, device=x.device)
                  if self.family == "qwen35" and self.has_shared else None)
        self.layer.route(x.data_ptr(), T, sel_idx.data_ptr(), sel_w.data_ptr(),
                         expert_in.data_ptr() if expert_in is not None else 0,
                         logits.data_ptr() if logits is not None else 0, self._stream())
        self.launches += self.layer.last_launch_count()
        return Routed(sel_idx, sel_w, expert_in, logits)

    def rows(self, x: torch.Tensor, routed: Routed) -> torch.Tensor:
        return routed.expert_in if routed.expert_in is not None else x

    def expert_rows(self, rows: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        out = torch.empty((rows.shape[0], self.hidden), dtype=torch.float32, device=rows.device)
        if rows.shape[0]:
            self.layer.expert_rows(rows.contiguous().data_ptr(), ids.contiguous().data_ptr(),
                                   rows.shape[0], out.data_ptr(), self._stream())
            self.launches += self.layer.last_launch_count()
        return out

    def combine(self, routed: Routed, pair_out: torch.Tensor) -> torch.Tensor:
        T = routed.sel_idx.shape[0]
        y = torch.empty((T, self.hidden), dtype=torch.float32, device=pair_out.device)
        self.layer.combine_rows(T, routed.sel_idx.data_ptr(), routed.sel_w.data_ptr(),
                                pair_out.contiguous().data_ptr(), y.data_ptr(),
                                routed.logits.data_ptr() if routed.logits is not None else 0,
                                self._stream())
        self.launches += self.layer.last_launch_count()
        return y


def cuda_backend_for(sl) -> CudaBackend:
    """Backend over a `synthetic.SyntheticLayer` built with an expert range."""
    cfg = sl.cfg
    shared = bool(cfg.get("shared"))
    columns = cfg["experts"] + (1 if cfg["family"] == "qwen35" and shared else 0)
    return CudaBackend(sl.layer, cfg["family"], cfg["hidden"], cfg["top_k"], columns, shared)


class PeerExpertParallel:
    """Expert parallelism over NVLink peer memory (dm_ep_*): rank `rank` of `world` holds
    the experts of `layer` (a shard built for [rank*E/world, (rank+1)*E/world)) and
    runs up to `max_tokens` tokens per forward. Call `connect_ipc` on every rank (one
    process per GPU), or `connect_local` once with every rank of one process, before
    the first forward."""

    HANDLE_BYTES = 64

    def __init__(self, layer, rank: int, world: int, max_tokens: int):
        self.layer = layer
        self.rank, self.world, self.max_tokens = rank, world, max_tokens
        self.hidden = layer.desc.hidden
        self.top_k = layer.desc.top_k
        h = C.c_void_p()
        check(N.lib().dm_ep_create(layer.handle, rank, world, max_tokens, C.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def ipc_handle(self) -> bytes:
        buf = (C.c_uint8 * self.HANDLE_BYTES)()
        check(N.lib().dm_ep_ipc_handle(self._h, buf))
        return bytes(buf)

    def connect_ipc(self, group=None):
        """Exchange exchange-region handles with every rank of `group` and map them."""
        handles = [None] * self.world
        dist.all_gather_object(handles, self.ipc_handle(), group=group)
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(N.lib().dm_ep_connect_ipc(self._h, buf))
        dist.barrier(group=group)  # every rank mapped before anyone sends

    @staticmethod
    def connect_local(ranks):
        """Connect the ranks of one process (one GPU or several)."""
        arr = (C.c_void_p * len(ranks))(*[r.handle.value for r in ranks])
        for r in ranks:
            check(N.lib().dm_ep_connect_local(r.handle, arr))

    @staticmethod
    def _stream(stream):
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream
        return C.c_void_p(stream) if stream else None

    def dispatch(self, x: torch.Tensor, stream=None):
        self.tokens = x.shape[0]
        check(N.lib().dm_ep_dispatch(self._h, C.c_void_p(x.data_ptr()), self.tokens,
                                     self._stream(stream)))

    def experts(self, stream=None):
        check(N.lib().dm_ep_experts(self._h, self._stream(stream)))

    def combine(self, y=None, sel_idx=None, sel_w=None, stream=None) -> torch.Tensor:
        if y is None:
            y = torch.empty((self.tokens, self.hidden), dtype=torch.float32, device="cuda")
        ptr = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        check(N.lib().dm_ep_combine(self._h, ptr(y), ptr(sel_idx), ptr(sel_w),
                                    self._stream(stream)))
        return y

    def forward(self, x: torch.Tensor, y=None, sel_idx=None, sel_w=None,
                stream=None) -> torch.Tensor:
        """One expert-parallel forward of this rank's tokens x [T, H] (device)."""
        T = x.shape[0]
        if y is None:
            y = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
        ptr = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        self.tokens = T
        check(N.lib().dm_ep_forward(self._h, ptr(x), ptr(y), T, ptr(sel_idx), ptr(sel_w),
                                    self._stream(stream)))
        return y

    def status(self, stream=None):
        check(N.lib().dm_ep_status(self._h, self._stream(stream)))

    def last_launch_count(self) -> int:
        return N.lib().dm_ep_last_launch_count(self._h)

    def close(self):
        if self._h:
            N.lib().dm_ep_destroy(self._h)
            self._h = None
