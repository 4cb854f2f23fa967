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


def kv_head_shard(n_heads: int, n_kv_heads: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """Attention split by KV head: rank keeps whole GQA groups, query heads
    [h0, h1) and KV heads [g0, g1), so it needs no collective.  The shard is
    addressed by pointer offsets alone (q/out + h0*head_dim, K/V + g0*head_dim,
    the row strides q_stride and kv_dim unchanged)."""
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    per = n_kv_heads // world
    g0, g1 = rank * per, (rank + 1) * per
    group = n_heads // n_kv_heads
    return g0 * group, g1 * group, g0, g1


def gdn_vhead_shard(n_vheads: int, num_k_heads: int, world: int, rank: int) -> tuple[int, int, int]:
    """GDN split by value head: rank owns v-heads [v0, v1) (state, v, gate,
    beta, z, out for those heads) and reads the q/k heads h % num_k_heads they
    map to.  Returns (v0, v1, k_off): with the q/k base pointers advanced by
    k_off heads, the kernel's own mapping (local head) % num_k_heads lands on
    the right q/k head for every local head."""
    if n_vheads % world:
        raise ValueError(f"{n_vheads} v-heads do not split over {world} ranks")
    per = n_vheads // world
    v0, v1 = rank * per, (rank + 1) * per
    if v0 % num_k_heads == 0:
        return v0, v1, 0
    if per <= num_k_heads and v0 % num_k_heads + per <= num_k_heads:
        return v0, v1, v0 % num_k_heads
    raise ValueError(f"v-head shard [{v0}, {v1}) wraps the {num_k_heads} k-heads")


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


class PartialExchange:
    """Preallocated split-KV exchange for repeated decode steps.

    This rank's partials live in one payload buffer: `ml` [n_heads, 2] (m, l)
    followed by `o` [n_heads, head_dim], both views that decode_partial writes
    in place.  run() all-gathers the payload into [world, payload] with ONE
    NCCL all-gather (straight into its final layout, no host-side copies) and
    merges the packed parts on this GPU with the log-sum-exp kernel.  Every
    call issues the same collective in the same order, so a whole step
    (partial decode + exchange + merge) can be captured in one CUDA graph."""

    def __init__(self, n_heads: int, head_dim: int, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.n_heads, self.head_dim = n_heads, head_dim
        n = n_heads * (2 + head_dim)
        self.payload = torch.zeros(n, dtype=torch.float32, device=device)
        self.ml = self.payload[:n_heads * 2].view(n_heads, 2)
        self.o = self.payload[n_heads * 2:].view(n_heads, head_dim)
        self.parts = torch.zeros(self.world * n, dtype=torch.float32, device=device)

    def gather(self) -> tuple[torch.Tensor, torch.Tensor]:
        """All ranks' partials as ([world, n_heads, 2], [world, n_heads, head_dim]) tensors."""
        if self.world > 1:
            dist.all_gather_into_tensor(self.parts, self.payload, group=self.group)
        else:
            self.parts.copy_(self.payload)
        p = self.parts.view(self.world, -1)
        H = self.n_heads
        return p[:, :H * 2].reshape(self.world, H, 2), p[:, H * 2:].reshape(self.world, H, self.head_dim)

    def run(self, out: torch.Tensor, gate: Optional[torch.Tensor] = None) -> None:
        from . import attn

        if self.world > 1:
            dist.all_gather_into_tensor(self.parts, self.payload, group=self.group)
            attn.merge_partials_packed(out, self.parts, self.world, self.n_heads, self.head_dim, gate)
        else:
            attn.merge_partials_packed(out, self.payload, 1, self.n_heads, self.head_dim, gate)


class PeerExchange:
    """Split-KV exchange over peer memory: the one-kernel alternative to
    PartialExchange's NCCL all-gather.

    Every rank owns a receive area (library cudaMalloc) and maps all peers'
    areas through CUDA IPC; the 64-byte handles travel over the process
    group (all_gather_object).  run() launches yattn_exchange_merge: this
    rank's (ml, o) go into every rank's area over NVLink (stores only), each
    rank waits for all parts in its own memory and merges them.  The epoch
    that pairs the ranks' calls lives on the device, so a step including
    run() can be captured in a CUDA graph.  Every rank must make the same
    sequence of run() calls; close() (collective) unmaps and frees."""

    def __init__(self, n_heads: int, head_dim: int, device, group=None):
        import ctypes as C

        from ._lib import call, lib

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_heads, self.head_dim = n_heads, head_dim
        n = n_heads * (2 + head_dim)
        self.payload = torch.zeros(n, dtype=torch.float32, device=device)
        self.ml = self.payload[:n_heads * 2].view(n_heads, 2)
        self.o = self.payload[n_heads * 2:].view(n_heads, head_dim)
        area = C.c_void_p()
        call("yattn_exchange_area_alloc", self.world, n_heads, head_dim, C.byref(area))
        self.area = area.value
        handle = (C.c_uint8 * 64)()
        call("yattn_ipc_handle", self.area, handle)
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, bytes(handle), group=group)
        else:
            handles = [bytes(handle)]
        self.peers = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.peers.append(self.area)
                continue
            ptr = C.c_void_p()
            call("yattn_ipc_open", (C.c_uint8 * 64).from_buffer_copy(hb), C.byref(ptr))
            self.peers.append(ptr.value)
        self._areas = (C.c_void_p * self.world)(*self.peers)
        self._lib = lib

    def run(self, out: torch.Tensor, gate: Optional[torch.Tensor] = None, wait_limit_ns: int = 0) -> None:
        """wait_limit_ns bounds the wait for the peers' parts (0: the library's 2 s).  On
        timeout out is NaN and yattn_device_status reads 401; the areas' epochs are then
        out of step, so the exchange must be rebuilt before the next call."""
        from ._lib import call

        call("yattn_exchange_merge", self.payload.data_ptr(), self.payload.data_ptr() + self.n_heads * 2 * 4,
             self._areas, self.world, self.rank, self.n_heads, self.head_dim, out.data_ptr(),
             gate.data_ptr() if gate is not None else None, wait_limit_ns, torch.cuda.current_stream().cuda_stream)

    def decode(self, out: torch.Tensor, q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor, k_begin: int,
               k_end: int, n_kv_heads: int, kv_dim: int, gate: Optional[torch.Tensor] = None,
               wait_limit_ns: int = 0) -> None:
        """One step of the split decode in two launches (yattn_decode_exchange): this rank's keys
        [k_begin, k_end) reduced on its GPU, merged and exchanged with every rank in one kernel."""
        from ._lib import call

        call("yattn_decode_exchange", q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(), k_begin, k_end,
             self.n_heads, n_kv_heads, self.head_dim, kv_dim, self._areas, self.world, self.rank, out.data_ptr(),
             gate.data_ptr() if gate is not None else None, wait_limit_ns, None, 0,
             torch.cuda.current_stream().cuda_stream)

    def close(self) -> None:
        """Collective: every rank's pushes are done before any area is unmapped or freed."""
        from ._lib import call

        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for r, ptr in enumerate(self.peers):
            if r != self.rank:
                call("yattn_ipc_close", ptr)
        if self.world > 1:
            dist.barrier(group=self.group)
        call("yattn_exchange_area_free", self.area)
        self.peers = []
