"""Host-side multi-GPU logic on CPU: sharding rules, and the split-KV partial
exchange run as two gloo ranks (the log-sum-exp merge itself is the library's
GPU kernel; here a numpy restatement of it checks the exchanged payload)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from yllm_b200 import dist as ydist


def test_shard_by_length_balances_and_covers():
    from yllm_b200.configs import CFG3

    lens = CFG3.ctx()
    for world in (1, 2, 4, 8):
        shards = ydist.shard_by_length(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lens)))
        loads = [sum(lens[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lens)
        assert shards == ydist.shard_by_length(lens, world)   # deterministic


@pytest.mark.parametrize("n,world", [(131072, 8), (7, 3), (1, 4), (64, 8)])
def test_split_range_covers(n, world):
    prev = 0
    sizes = []
    for r in range(world):
        a, b = ydist.split_range(n, world, r)
        assert a == prev
        prev = b
        sizes.append(b - a)
    assert prev == n and max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("S,world", [(2048, 1), (2048, 2), (2048, 4), (2048, 8), (4096, 8), (300, 4)])
def test_causal_row_split(S, world):
    cuts = [ydist.causal_row_split(S, world, r) for r in range(world)]
    assert cuts[0][0] == 0 and cuts[-1][1] == S
    for (a, b), (c, d) in zip(cuts, cuts[1:]):
        assert b == c
    work = [sum(r + 1 for r in range(a, b)) for a, b in cuts]
    if S >= 128 * world * 2:
        assert max(work) <= 1.6 * (S * (S + 1) / 2) / world


def lse_merge(ml, o):
    """numpy restatement of the merge kernel: ml [P, H, 2] (m in log2 units), o [P, H, D]."""
    m, l = ml[..., 0], ml[..., 1]
    live = l > 0
    M = np.where(live, m, -np.inf).max(axis=0)
    w = np.where(live, np.exp2(m - M[None]), 0.0)
    return (w[..., None] * o).sum(0) / (w * l).sum(0)[:, None]


def _partials(scores, v):
    """(m, l, o) of one key range: scores [H, T] already in log2 units."""
    m = scores.max(axis=1)
    p = np.exp2(scores - m[:, None])
    return np.stack([m, p.sum(1)], axis=1), p @ v


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    rng = np.random.default_rng(0)
    H, D, T = 4, 16, 1000
    scores = rng.standard_normal((H, T)) * 3
    v = rng.standard_normal((T, D))
    a, b = ydist.split_range(T, world, rank)
    ml, o = _partials(scores[:, a:b], v[a:b])
    all_ml, all_o, w = ydist.gather_partials(torch.from_numpy(ml), torch.from_numpy(o), H, D)
    merged = lse_merge(all_ml.numpy(), all_o.numpy())
    full_ml, full_o = _partials(scores, v)
    ret[rank] = float(np.max(np.abs(merged - full_o / full_ml[:, 1:2])))
    dist.destroy_process_group()


def test_split_kv_exchange_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert ret[0] < 1e-12 and ret[1] < 1e-12


def _exchange_worker(rank, world, port, ret):
    """PartialExchange: preallocated buffers, two steps with new partials each."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    H, D, T = 4, 16, 999
    ex = ydist.PartialExchange(H, D, device="cpu")
    worst = 0.0
    for step in range(2):
        rng = np.random.default_rng(step)
        scores = rng.standard_normal((H, T)) * 3
        v = rng.standard_normal((T, D))
        a, b = ydist.split_range(T, world, rank)
        ml, o = _partials(scores[:, a:b], v[a:b])
        ex.ml.copy_(torch.from_numpy(ml))
        ex.o.copy_(torch.from_numpy(o))
        all_ml, all_o = ex.gather()
        assert all_ml.shape == (world, H, 2) and all_o.shape == (world, H, D)
        merged = lse_merge(all_ml.double().numpy(), all_o.double().numpy())
        full_ml, full_o = _partials(scores, v)
        ref = full_o / full_ml[:, 1:2]
        worst = max(worst, float(np.max(np.abs(merged - ref) / np.maximum(np.abs(ref), 1e-3))))
    ret[rank] = worst
    dist.destroy_process_group()


def test_partial_exchange_three_gloo_ranks():
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 3, port, ret)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert all(ret[r] < 1e-4 for r in range(3)), dict(ret)


def _leaver(rank, world, port, ret):
    """Rank 1 leaves between steps; rank 0's next exchange ends in an error
    after the process-group timeout instead of waiting forever."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    ml = torch.zeros(2, 2)
    o = torch.zeros(2, 4)
    ydist.gather_partials(ml, o, 2, 4)   # step 1: both ranks
    if rank == 1:
        ret[1] = "left"
        os._exit(0)
    try:
        ydist.gather_partials(ml, o, 2, 4)   # step 2: the peer is gone
        ret[0] = "no error"
    except Exception as e:  # noqa: BLE001 -- any collective error is the expected outcome
        ret[0] = "error: " + type(e).__name__
    os._exit(0)


def test_exchange_fails_cleanly_when_a_rank_leaves():
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert ret.get(1) == "left"
    assert str(ret.get(0, "")).startswith("error"), ret.get(0)
