"""Distributed SpMM: the dist_spmm_node pipeline (src/dist_spmm_node.cu:20-444) per rank.

One process per GPU. ``torch.distributed`` carries the host collectives the reference
does with MPI (Gather/Bcast of the HSDMA demand matrix, Allgather(v) of the needed sets,
the IPC handle exchange, Allreduce of the timings); the data path is the native library:
copy-engine bulk copies and NVLink gather kernels from the peers' B buffers (CUDA IPC)
overlapped with the sm_100a SpMM kernels.

``build_local_group`` builds all ranks inside one process (ranks may share a GPU), which
is how the multi-rank path is exercised on a single GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field, replace

import numpy as np

from ._lib import P, c_f32, c_i32, c_i64, c_vp, call, dsp_rank_desc, dsp_rank_stats, lib
from .matrix import Csr
from . import planner


# ---------------------------------------------------------------------------- plan

@dataclass
class GlobalPlan:
    """Everything every rank must agree on after the setup collectives."""
    T: int
    cpt: int
    remap: np.ndarray        # int32 [T]
    n_col: np.ndarray        # int32 [T] merged (node union) sizes
    offsets: np.ndarray      # int64 [T+1]
    merged: np.ndarray       # int32 flat merged needed lists (tile-local, ascending)
    hsdma_ms: float = 0.0
    demand: np.ndarray | None = None  # P x T pre-merge n_col lists


def global_plan(tilings: list, task_dist: int, n_rolls: int) -> GlobalPlan:
    """Allocation (src/dist_spmm_node.cu:134-168) and node merge (:174-181) from every
    rank's tiling (what the Gather / Allgatherv of the reference deliver)."""
    import time
    demand = np.stack([t.n_col for t in tilings]).astype(np.int32)
    t0 = time.perf_counter()
    remap = planner.allocate(task_dist, demand, n_rolls)
    hs = (time.perf_counter() - t0) * 1e3 if task_dist == 2 else 0.0
    cols = np.concatenate([t.needed for t in tilings]) if tilings else np.zeros(0, np.int32)
    n, off, merged = planner.merge_needed(demand, cols)
    return GlobalPlan(demand.shape[1], tilings[0].cpt, remap, n, off, merged, hs, demand)


# ---------------------------------------------------------------------------- rank

FETCH_ENGINES = {"lsu": 0, "tma": 1}  # DSP_FETCH_LSU / DSP_FETCH_TMA
PIPELINES = {"auto": 0, "rows": 1, "split": 2, "groups": 3}  # DSP_PIPELINE_*


class Rank:
    """A dsp_rank: one GPU's segments, B / C buffers, fetch plan and streams."""

    def __init__(self, local: Csr, rank: int, world: int, device: int, dims: int, M: int, m_lb: int,
                 plan: GlobalPlan, n_slice: np.ndarray, sparse: np.ndarray, n_streams: int = 4,
                 fetch_engine: str = "lsu", pipeline: str = "auto", groups: int = 0):
        self.rank, self.world, self.device, self.dims, self.M = rank, world, device, dims, M
        self.m_local = local.num_rows
        self.m_lb = m_lb
        self.T, self.cpt, self.remap = plan.T, plan.cpt, np.array(plan.remap, np.int32)
        self._keep = [local, plan, np.ascontiguousarray(n_slice, np.int32), np.ascontiguousarray(sparse, np.uint8)]
        c = local.to_c()
        self._keep.append(c)
        d = dsp_rank_desc()
        d.rank, d.world, d.device, d.dims, d.T, d.n_streams = rank, world, device, dims, plan.T, n_streams
        d.cpt, d.M, d.m_lb = plan.cpt, M, m_lb
        d.local = ctypes.pointer(c)
        d.remap = np.ascontiguousarray(plan.remap, np.int32).ctypes.data_as(P(c_i32))
        d.sparse = self._keep[3].ctypes.data_as(P(ctypes.c_uint8))
        merged = plan.merged if plan.merged.size else np.zeros(1, np.int32)
        self._keep.append(merged)
        d.needed_offsets = plan.offsets.ctypes.data_as(P(c_i64))
        d.needed_cols = merged.ctypes.data_as(P(c_i32))
        d.n_slice = self._keep[2].ctypes.data_as(P(c_i32))
        d.fetch_engine = FETCH_ENGINES[fetch_engine]
        d.pipeline = PIPELINES[pipeline]
        d.groups = groups
        h = c_vp()
        call("dsp_rank_create", ctypes.byref(d), ctypes.byref(h))
        self._h = h

    # buffers
    def b_ptr(self) -> int:
        p = c_vp()
        call("dsp_rank_b_ptr", self._h, ctypes.byref(p))
        return int(p.value or 0)

    def c_ptr(self) -> int:
        p = c_vp()
        call("dsp_rank_c_ptr", self._h, ctypes.byref(p))
        return int(p.value or 0)

    def ipc_handle(self) -> bytes:
        buf = (ctypes.c_uint8 * 64)()
        call("dsp_rank_ipc_handle", self._h, buf)
        return bytes(buf)

    def open_peer(self, peer: int, handle: bytes) -> None:
        buf = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
        call("dsp_rank_open_peer", self._h, peer, buf)

    def set_peer(self, peer: int, ptr: int, device: int) -> None:
        call("dsp_rank_set_peer", self._h, peer, ptr, device)

    # data movement and compute
    def fill_b(self, seed: int, stream: int = 0) -> None:
        call("dsp_rank_fill_b", self._h, seed, stream)

    def poison_remote(self, stream: int = 0) -> None:
        """NaN-fill every B row this rank does not own (unfetched rows then poison C)."""
        call("dsp_rank_poison_remote", self._h, stream)

    def upload_b(self, B_host: np.ndarray, stream: int = 0) -> None:
        assert B_host.dtype == np.float32 and B_host.flags.c_contiguous and B_host.shape == (self.M, self.dims)
        call("dsp_rank_upload_b", self._h, B_host.ctypes.data, stream)

    def upload_b_ptr(self, host_ptr: int, stream: int = 0) -> None:
        call("dsp_rank_upload_b", self._h, host_ptr, stream)

    def upload_b_owned_ptr(self, host_ptr: int, stream: int = 0) -> None:
        """Owned tiles only, back to back in ascending tile order (owned_rows x dims)."""
        call("dsp_rank_upload_b_owned", self._h, host_ptr, stream)

    def owned_tiles(self) -> list:
        """(first row, rows) of every owned tile, ascending: the layout of upload_b_owned."""
        out = []
        for t in range(self.T):
            if self.remap[t] == self.rank:
                row0 = t * self.cpt
                n = min(self.cpt, self.M - row0)
                if n > 0:
                    out.append((row0, n))
        return out

    def step(self, stream: int = 0) -> None:
        call("dsp_rank_step", self._h, stream)

    def check_error(self) -> None:
        """Raise DspError(DSP_ERR_TIMEOUT) if a fetch wait of an earlier step gave up."""
        call("dsp_rank_check_error", self._h)

    def download_c(self, C_host: np.ndarray, stream: int = 0) -> None:
        assert C_host.dtype == np.float32 and C_host.flags.c_contiguous and C_host.shape == (self.m_local, self.dims)
        call("dsp_rank_download_c", self._h, C_host.ctypes.data, stream)

    def download_c_ptr(self, host_ptr: int, stream: int = 0) -> None:
        call("dsp_rank_download_c", self._h, host_ptr, stream)

    def last_compute_ms(self) -> float:
        ms = c_f32()
        call("dsp_rank_last_compute_ms", self._h, ctypes.byref(ms))
        return float(ms.value)

    def timeline(self) -> list:
        """Last step: per entry k, (fetch_begin, fetch_end of ring position k, seg_begin,
        seg_end of phase or row group k) in ms from the step start (None where nothing ran)."""
        n = self.stats()["timeline_len"]
        buf = (c_f32 * (4 * n))()
        call("dsp_rank_last_timeline", self._h, buf, 4 * n)
        out = []
        for k in range(n):
            out.append(tuple(None if buf[4 * k + i] < 0 else round(float(buf[4 * k + i]), 4) for i in range(4)))
        return out

    def stats(self) -> dict:
        s = dsp_rank_stats()
        call("dsp_rank_stats_get", self._h, ctypes.byref(s))
        return {k: (round(float(getattr(s, k)), 4) if t is ctypes.c_float else int(getattr(s, k)))
                for k, t in dsp_rank_stats._fields_}

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dsp_rank_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


FETCH_SCOPES = ("node", "rank")


def fetch_view(plan: GlobalPlan, tiling, scope: str = "node") -> GlobalPlan:
    """The needed lists a rank fetches from: the node-merged union of every rank's lists
    ("node", the reference's double_level_comm_node_processing, src/utils.h:439-547), or
    only this rank's own lists ("rank": fewer NVLink bytes when the ranks' needs differ;
    the selector then sees this rank's own list sizes)."""
    if scope == "node":
        return plan
    if scope == "rank":
        return replace(plan, n_col=np.ascontiguousarray(tiling.n_col, np.int32),
                       offsets=np.ascontiguousarray(tiling.offsets, np.int64),
                       merged=np.ascontiguousarray(tiling.needed, np.int32))
    raise ValueError(f"fetch scope {scope!r}: expected one of {FETCH_SCOPES}")


def make_rank(local: Csr, rank: int, world: int, device: int, dims: int, M: int, m_lb: int, tiling,
              plan: GlobalPlan, comm_type: int, platform: str = "h100", n_streams: int = 4,
              fetch_engine: str = "lsu", fetch_scope: str = "node", pipeline: str = "auto",
              groups: int = 0) -> Rank:
    """Selector (CommMan_hp ctor, src/comm_man.h:341-410) + rank construction."""
    view = fetch_view(plan, tiling, fetch_scope)
    sparse = planner.comm_select(comm_type, dims, view.n_col, tiling.n_slice, platform)
    r = Rank(local, rank, world, device, dims, M, m_lb, view, tiling.n_slice, sparse, n_streams, fetch_engine,
             pipeline, groups)
    r.sparse = sparse
    r.n_slice = tiling.n_slice
    r.n_col = view.n_col
    return r


# ---------------------------------------------------------------------------- in-process group

@dataclass
class LocalGroup:
    ranks: list
    plan: GlobalPlan
    bounds: list
    tilings: list
    dims: int
    M: int
    nnz: int
    traffic_intra: int = 0
    sparse: list = field(default_factory=list)

    def step(self, streams=None) -> None:
        for i, r in enumerate(self.ranks):
            r.step(0 if streams is None else streams[i])

    def close(self) -> None:
        for r in self.ranks:
            r.close()


def build_local_group(g: Csr, world: int, devices, dims: int, n_rolls: int = 4, task_dist: int = 2,
                      comm_type: int = 2, platform: str = "h100", n_streams: int = 4,
                      fetch_engine: str = "lsu", partition: str = "rows",
                      fetch_scope: str = "node", pipeline: str = "auto", groups: int = 0) -> LocalGroup:
    """All `world` ranks of the pipeline in this process; devices[p] is rank p's GPU
    (ranks may share one). Peers read each other's B directly (same device, or peer
    access between devices)."""
    M = g.num_rows
    T = world * n_rolls
    bounds = [planner.bounds(g, world, p, partition) for p in range(world)]
    locals_ = [planner.partition(g, lb, ub) for lb, ub in bounds]
    tilings = [planner.tile(loc, T) for loc in locals_]
    plan = global_plan(tilings, task_dist, n_rolls)
    ranks = [make_rank(locals_[p], p, world, devices[p], dims, M, bounds[p][0], tilings[p], plan, comm_type,
                       platform, n_streams, fetch_engine, fetch_scope, pipeline, groups) for p in range(world)]
    for p in range(world):
        for q in range(world):
            if p != q:
                ranks[p].set_peer(q, ranks[q].b_ptr(), devices[q])
    traffic = sum(planner.traffic_intra(p, plan.remap, ranks[p].sparse, ranks[p].n_col, tilings[p].n_slice, dims)
                  for p in range(world))
    return LocalGroup(ranks, plan, bounds, tilings, dims, M, g.nnz, traffic, [r.sparse for r in ranks])


# ---------------------------------------------------------------------------- torch.distributed

class TorchComm:
    """Host collectives over a torch.distributed process group (NCCL or gloo)."""

    def __init__(self, group=None):
        import torch
        import torch.distributed as dist
        self.dist = dist
        self.torch = torch
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        backend = dist.get_backend(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")

    def allgather_i32(self, arr: np.ndarray) -> list:
        """Variable-length all-gather of int32 arrays (Allgather + Allgatherv)."""
        torch = self.torch
        a = torch.from_numpy(np.ascontiguousarray(arr, np.int32).reshape(-1)).to(self.device)
        n = torch.tensor([a.numel()], dtype=torch.int64, device=self.device)
        sizes = [torch.zeros_like(n) for _ in range(self.world)]
        self.dist.all_gather(sizes, n, group=self.group)
        sizes = [int(s.item()) for s in sizes]
        cap = max(max(sizes), 1)
        pad = torch.zeros(cap, dtype=torch.int32, device=self.device)
        pad[: a.numel()] = a
        outs = [torch.zeros(cap, dtype=torch.int32, device=self.device) for _ in range(self.world)]
        self.dist.all_gather(outs, pad, group=self.group)
        return [o[:s].cpu().numpy() for o, s in zip(outs, sizes)]

    def allgather_bytes(self, b: bytes) -> list:
        arr = np.frombuffer(b, np.uint8).astype(np.int32)
        return [bytes(x.astype(np.uint8)) for x in self.allgather_i32(arr)]

    def allreduce_max(self, x: float) -> float:
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def allreduce_sum_i64(self, x: int) -> int:
        t = self.torch.tensor([x], dtype=self.torch.int64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
        return int(t.item())

    def barrier(self) -> None:
        if self.device.type == "cuda":
            self.dist.barrier(group=self.group, device_ids=[self.device.index])
        else:
            self.dist.barrier(group=self.group)


def distributed_plan(comm, local: Csr, n_rolls: int, task_dist: int, device_setup: bool = False):
    """This rank's tiling plus the agreed global plan, via host collectives: every rank
    contributes its demand row and needed lists; the allocation is computed from the
    gathered demand (identically on every rank, which equals the reference's root
    compute + broadcast).

    device_setup (NCCL groups): tile on the GPU from a column-presence byte map and form
    the node union as an all-reduce MAX of the ranks' maps instead of all-gathering the
    lists; same plan."""
    T = comm.world * n_rolls
    if device_setup:
        return _distributed_plan_device(comm, local, n_rolls, task_dist)
    mine = planner.tile(local, T)
    n_cols = comm.allgather_i32(mine.n_col)
    needed = comm.allgather_i32(mine.needed)

    class _T:  # tiling of another rank as far as the plan needs it
        def __init__(self, n_col, needed_, cpt):
            self.n_col, self.needed, self.cpt = n_col, needed_, cpt

    tilings = [_T(n_cols[p], needed[p], mine.cpt) for p in range(comm.world)]
    plan = global_plan(tilings, task_dist, n_rolls)
    return mine, plan


def _distributed_plan_device(comm, local: Csr, n_rolls: int, task_dist: int):
    import time

    torch = comm.torch
    if comm.device.type != "cuda":
        raise RuntimeError("device_setup needs an NCCL process group (CUDA tensors)")
    T = comm.world * n_rolls
    M = local.num_cols
    d_cols = torch.from_numpy(np.ascontiguousarray(local.indices, np.int64)).to(comm.device)
    stream = torch.cuda.current_stream(comm.device).cuda_stream
    present = planner.col_presence(d_cols, M, stream)
    mine = planner.tile_device(d_cols, M, T, present, stream)
    demand = np.stack(comm.allgather_i32(mine.n_col)).astype(np.int32)
    comm.dist.all_reduce(present, op=comm.dist.ReduceOp.MAX, group=comm.group)  # node union
    n, off, merged = planner.needed_from_presence(present, M, T, stream)
    t0 = time.perf_counter()
    remap = planner.allocate(task_dist, demand, n_rolls)
    hs = (time.perf_counter() - t0) * 1e3 if task_dist == 2 else 0.0
    return mine, GlobalPlan(T, mine.cpt, remap, n, off, merged, hs, demand)


def connect_peers(comm, rank: Rank) -> None:
    """Exchange CUDA IPC handles of every rank's B and open the peers' buffers."""
    handles = comm.allgather_bytes(rank.ipc_handle())
    for q, h in enumerate(handles):
        if q != comm.rank:
            rank.open_peer(q, h)
