"""Sharding of independent compression windows over the GPUs of one box.

redukt compresses independent windows (files or fixed-size chunks); each window's decode step
only reads its own recurrent state, so the path partitions without any exchange: window i goes
to rank i mod G, one process per GPU (the plugin is a process-global singleton,
plugins/redukt-gpu-cuda/mamba_cuda.cu:180), and every rank writes its own outputs.  The only
cross-rank operations are outside the data path: a barrier and a max over ranks of the elapsed
time, and an optional gather of per-window results for reporting.
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence


def windows_for_rank(n_windows: int, rank: int, world: int) -> List[int]:
    """Window indices owned by `rank`: i mod world == rank, ascending."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return list(range(rank, n_windows, world))


def rank_env() -> Dict[str, int]:
    return {"rank": int(os.environ.get("RANK", "0")), "world": int(os.environ.get("WORLD_SIZE", "1")),
            "local": int(os.environ.get("LOCAL_RANK", "0"))}


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank scalar (e.g. elapsed seconds) over the process group; identity alone."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_results(local: Dict[int, object], dist=None) -> Dict[int, object]:
    """Merge every rank's {window index: result} on all ranks (for reporting, not the data path)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return dict(local)
    parts: List[Optional[Dict[int, object]]] = [None] * dist.get_world_size()
    dist.all_gather_object(parts, local)
    merged: Dict[int, object] = {}
    for p in parts:
        for k, v in (p or {}).items():
            if k in merged:
                raise RuntimeError(f"window {k} processed by two ranks")
            merged[k] = v
    return merged


def check_partition(n_windows: int, world: int, owned: Sequence[Sequence[int]]) -> None:
    seen = sorted(i for part in owned for i in part)
    if seen != list(range(n_windows)):
        raise RuntimeError("windows are not partitioned exactly once over the ranks")
