"""Multi-GPU request dispatch for the paged-KV denoise path: one process per GPU, requests sharded.

Requests (and LingBot episodes) are independent: each rank owns one pool on its own GPU, the block
tables and KV of the requests it was given, and runs their whole denoise loop locally. Nothing
crosses GPUs on the data path. The only traffic is control traffic around it:

  * rank 0 holds the request table (id, prefix length, valid prefix, input seed) and scatters each
    rank its share of descriptors (`scatter_requests`);
  * after the loop, rank 0 gathers per-request results (`gather_results`), and the step time is
    reduced as the maximum over ranks (`max_over_ranks`).

Assignment (`assign_requests`) is either the plain `i mod n` rule or length-aware greedy
balancing: requests sorted by decreasing prefix length (ties by id), each placed on the rank with
the least total keys so far (ties to the lowest rank). Attention cost per request is linear in its
key count, so equal key totals mean equal per-rank time. This is the partitioning of the reference
server's request loop (serving/vla-server.cpp:240-523, one request at a time on one device) spread
over N devices. Every function works on any torch.distributed backend; the tests run it on `gloo`
ranks on the CPU, and the bench on NCCL.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np


@dataclass(frozen=True)
class RequestDesc:
    """One request of the denoise path: what a rank needs to build and run it."""

    req_id: int
    prefix_len: int  # cached prefix tokens (rows in the pool)
    prefix_valid: int  # keys visible to the suffix (<= prefix_len; the rest is padding)
    seed: int  # seed of the request's synthetic inputs


def assign_requests(prefix_lens: Sequence[int], world: int, policy: str = "balanced") -> List[List[int]]:
    """Request indices per rank. `balanced` equalises total keys; `modulo` is i -> i mod world.

    Each rank's list is in increasing request order, so a rank's results come back in a fixed,
    reproducible order."""
    if world < 1:
        raise ValueError("world must be >= 1")
    n = len(prefix_lens)
    if policy == "modulo":
        return [list(range(r, n, world)) for r in range(world)]
    if policy != "balanced":
        raise ValueError(f"unknown policy {policy!r}")
    order = sorted(range(n), key=lambda i: (-int(prefix_lens[i]), i))
    load = [0] * world
    count = [0] * world
    per = (n + world - 1) // world  # no rank takes more than ceil(n / world) requests
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min((r for r in range(world) if count[r] < per), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += int(prefix_lens[i])
        count[r] += 1
    return [sorted(x) for x in out]


def make_requests(n: int, lo: int, hi: int, seed: int, padded: bool = False) -> List[RequestDesc]:
    """Seeded request table: prefix lengths U[lo, hi]; with `padded`, 768 image tokens + U[20, 48]
    valid text tokens are visible and the rest of the prefix is padding."""
    rng = np.random.default_rng(seed)
    plen = rng.integers(lo, hi + 1, size=n)
    pvalid = (768 + rng.integers(20, 49, size=n)) if padded else plen
    return [RequestDesc(i, int(plen[i]), int(min(pvalid[i], plen[i])), int(seed * 1000003 + i)) for i in range(n)]


def _dist():
    import torch.distributed as dist

    return dist if dist.is_available() and dist.is_initialized() else None


def scatter_requests(all_reqs: Optional[List[RequestDesc]], world: int, rank: int,
                     policy: str = "balanced") -> List[RequestDesc]:
    """Rank 0 passes the whole table (others pass None); every rank returns its own share."""
    dist = _dist()
    if world == 1 or dist is None:
        assert all_reqs is not None
        return list(all_reqs)
    shares = None
    if rank == 0:
        assert all_reqs is not None
        idx = assign_requests([r.prefix_len for r in all_reqs], world, policy)
        shares = [[asdict(all_reqs[i]) for i in ix] for ix in idx]
    out: List[Optional[list]] = [None]
    dist.scatter_object_list(out, shares, src=0)
    return [RequestDesc(**d) for d in out[0]]


def gather_results(local: Dict[int, np.ndarray], world: int, rank: int) -> Optional[Dict[int, np.ndarray]]:
    """Per-request results (req_id -> array) from every rank, merged on rank 0 (None elsewhere)."""
    dist = _dist()
    if world == 1 or dist is None:
        return dict(local)
    objs = [None] * world if rank == 0 else None
    dist.gather_object(local, objs, dst=0)
    if rank != 0:
        return None
    merged: Dict[int, np.ndarray] = {}
    for part in objs:
        for k, v in part.items():
            if k in merged:
                raise RuntimeError(f"request {k} returned by two ranks")
            merged[k] = v
    return merged


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar (step time) over all ranks."""
    dist = _dist()
    if dist is None or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(local, world: int, rank: int):
    """Rank 0 receives every rank's device result tensor (all the same shape) over the process
    group's backend -- NCCL on GPUs -- stacked as [world, ...]; other ranks get None."""
    dist = _dist()
    if world == 1 or dist is None:
        return local[None]
    import torch

    out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device) if rank == 0 else None
    dist.gather(local, gather_list=list(out.unbind(0)) if rank == 0 else None, dst=0)
    return out


def local_cpus_of_gpu(device_index: int) -> Optional[List[int]]:
    """Host CPUs attached to the GPU's NUMA node (from its PCI device's local_cpulist), or None
    where that cannot be read."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            bus = pynvml.nvmlDeviceGetPciInfo(pynvml.nvmlDeviceGetHandleByIndex(device_index)).busId
        finally:
            pynvml.nvmlShutdown()
        if isinstance(bus, bytes):
            bus = bus.decode()
        # NVML reports an 8-hex-digit domain ("00000000:1B:00.0"); sysfs uses 4 and lower case
        dom, rest = bus.split(":", 1)
        path = f"/sys/bus/pci/devices/{int(dom, 16):04x}:{rest.lower()}/local_cpulist"
        with open(path) as f:
            spec = f.read().strip()
    except Exception:
        return None
    cpus: List[int] = []
    for part in spec.split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.extend(range(int(a), int(b) + 1))
        elif part:
            cpus.append(int(part))
    return cpus or None


def bind_to_gpu_numa_node(device_index: int) -> Optional[List[int]]:
    """Restrict this process to the CPUs of its GPU's NUMA node, so that pinned host buffers
    allocated afterwards are local to the GPU's PCIe root; returns the CPU list (None: unchanged).
    CUDA_VISIBLE_DEVICES remapping is respected by NVML index only when it is unset or an identity
    list; otherwise nothing is changed."""
    import os

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if not all(x.isdigit() for x in ids) or device_index >= len(ids):
            return None
        device_index = int(ids[device_index])
    cpus = local_cpus_of_gpu(device_index)
    if not cpus:
        return None
    try:
        allowed = os.sched_getaffinity(0)
        keep = [c for c in cpus if c in allowed]
        if not keep:
            return None
        os.sched_setaffinity(0, keep)
        return keep
    except (AttributeError, OSError):
        return None
