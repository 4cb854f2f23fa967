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


def causal_row_split(S: int, world: int, rank: int, quant: int = 128) -> tuple[int, int]:
    """Query rows [r0, r1) of an S-token causal prefill for rank, with about
    equal causal work (row r attends r+1 keys, so the boundaries sit at
    S*sqrt(k/world)), rounded to multiples of `quant` (the kernel's row tile)."""
    import math

    def cut(k: int) -> int:
        if k <= 0:
            return 0
        if k >= world:
            return S
        return min(S, int(round(S * math.sqrt(k / world) / quant)) * quant)

    return cut(rank), cut(rank + 1)


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


def gather_partials(ml: torch.Tensor, o: torch.Tensor, n_heads: int, head_dim: int,
                    group=None) -> tuple[torch.Tensor, torch.Tensor, int]:
    """All-gathers every rank's (m, l) [n_heads, 2] and o [n_heads, head_dim]
    partials into local buffers: returns ([world, n_heads, 2], [world, n_heads,
    head_dim], world).  One collective of n_heads*(2+head_dim) floats per rank."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return ml.reshape(1, n_heads, 2), o.reshape(1, n_heads, head_dim), 1
    payload = torch.cat([ml.reshape(-1), o.reshape(-1)])
    parts = [torch.empty_like(payload) for _ in range(world)]
    dist.all_gather(parts, payload, group=group)
    g = torch.stack(parts)
    n_ml = n_heads * 2
    return (g[:, :n_ml].reshape(world, n_heads, 2).contiguous(),
            g[:, n_ml:].reshape(world, n_heads, head_dim).contiguous(), world)


def allgather_merge_partials(ml: torch.Tensor, o: torch.Tensor, out: torch.Tensor, n_heads: int, head_dim: int,
                             gate: Optional[torch.Tensor] = None, group=None) -> None:
    """Split-KV merge across ranks: gather every rank's partials (above), then
    merge them on this GPU with the library's log-sum-exp kernel.  Every rank
    ends with the full output.  Ranks with an empty key range send l = 0 and
    are skipped by the merge."""
    from . import attn

    all_ml, all_o, world = gather_partials(ml, o, n_heads, head_dim, group)
    attn.merge_partials(out, all_ml, all_o, world, n_heads, head_dim, gate)
