"""Multi-GPU plumbing: one process per GPU, torch.distributed for the host side.

Every config except long-context decode shards into independent work with no
data-path collective (by sequence, by KV head or by layer).  Long-context
decode splits the key range across GPUs; each GPU reduces its range to
per-head (m, l, o) partials on-device, the partials (a few KB) are
all-gathered over NCCL into local buffers and merged by the log-sum-exp
kernel.  No GPU ever loads another GPU's memory.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional, Sequence

import torch
import torch.distributed as dist


def shard_by_length(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Longest-first greedy: each sequence goes to the rank with the least
    total keys so far (ties -> lowest rank).  Returns per-rank index lists,
    each sorted ascending.  Deterministic for given lengths."""
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda j: (-lengths[j], j)):
        r = min(range(world), key=lambda x: (load[x], x))
        out[r].append(i)
        load[r] += lengths[i]
    return [sorted(x) for x in out]


def split_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [begin, end) share of n items for rank (sizes differ by <= 1)."""
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def env_rank() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str = "nccl", timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialises the process group from torchrun's environment (no-op for 1 rank)."""
    rank, world, local = env_rank()
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local


def allgather_merge_partials(ml: torch.Tensor, o: torch.Tensor, out: torch.Tensor, n_heads: int, head_dim: int,
                             gate: Optional[torch.Tensor] = None, group=None) -> None:
    """Split-KV merge across ranks: all-gather this rank's (m, l) [n_heads, 2]
    and o [n_heads, head_dim] partials, then merge them on this GPU with the
    library's log-sum-exp kernel.  Every rank ends with the full output."""
    from . import attn

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        attn.merge_partials(out, ml, o, 1, n_heads, head_dim, gate)
        return
    payload = torch.cat([ml.reshape(-1), o.reshape(-1)])
    gathered = torch.empty(world * payload.numel(), dtype=payload.dtype, device=payload.device)
    dist.all_gather_into_tensor(gathered, payload, group=group)
    g = gathered.view(world, -1)
    n_ml = n_heads * 2
    all_ml = g[:, :n_ml].contiguous()
    all_o = g[:, n_ml:].contiguous()
    attn.merge_partials(out, all_ml, all_o, world, n_heads, head_dim, gate)
