"""Split-KV exchange over peer memory (yattn_exchange_merge), on one GPU and on
two.  Long-context decode splits one query's keys over the GPUs; each GPU's
(m, l, o) partial is stored into every GPU's receive area and each GPU merges
all parts (log-sum-exp) -- compared here with the whole-range decode and the
CPU oracle (engine.c:1074-1096).  Tolerance: per element 2e-3 * max(|ref|,
f * rms(ref)), f from oracle.noise_floor (1e-3 or the fp32 noise it measures)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle

pytestmark = pytest.mark.gpu

H, KV, HD = 32, 8, 128


def _case(seed, T):
    rng = np.random.default_rng(seed)
    kd = KV * HD
    q = rng.standard_normal(H * HD).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    return q, k, v, kd


def _to_dev(dev, q, k, v):
    tq = torch.from_numpy(q).to(dev)
    tk = torch.from_numpy(k.view(np.int16)).to(dev).view(torch.uint16)
    tv = torch.from_numpy(v.view(np.int16)).to(dev).view(torch.uint16)
    return tq, tk, tv


def test_exchange_single_rank_repeats_and_graph_replays():
    """world = 1: the push lands in the rank's own area; the device epoch
    advances on every launch, so eager calls and graph replays all merge."""
    from yllm_b200 import attn
    from yllm_b200.dist import PeerExchange

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    T = 9000
    q, k, v, kd = _case(11, T)
    tq, tk, tv = _to_dev(dev, q, k, v)
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, HD, kd)
    ex = PeerExchange(H, HD, device=dev)
    try:
        outs = []
        for _ in range(3):
            out = torch.full((H * HD,), float("nan"), device=dev)
            attn.decode_partial(ex.ml, ex.o, tq, tk, tv, 0, T, H, KV, HD, kd)
            ex.run(out)
            outs.append(out)
        torch.cuda.synchronize()
        exact = oracle.exact_decode(q, k, v, T - 1, H, KV, HD, kd)
        for out in outs:
            oracle.assert_close(out.cpu().numpy(), want, what="exchange world 1", exact=exact)
        out_g = torch.full((H * HD,), float("nan"), device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            attn.decode_partial(ex.ml, ex.o, tq, tk, tv, 0, T, H, KV, HD, kd)
            ex.run(out_g)
        for _ in range(3):
            out_g.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            oracle.assert_close(out_g.cpu().numpy(), want, what="exchange world 1, graph replay", exact=exact)
        del g
        assert attn.device_status() == 0
    finally:
        ex.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, T, ret):
    import torch.distributed as dist

    from yllm_b200 import attn
    from yllm_b200.dist import PeerExchange, split_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    q, k, v, kd = _case(12, T)
    tq, tk, tv = _to_dev(dev, q, k, v)
    full = torch.zeros(H * HD, device=dev)
    attn.attn_decode(full, tq, tk, tv, T - 1, H, KV, HD, kd)
    torch.cuda.synchronize()
    floor = oracle.noise_floor(full.cpu().numpy(), oracle.exact_decode(q, k, v, T - 1, H, KV, HD, kd))
    ex = PeerExchange(H, HD, device=dev)
    worst = 0.0
    k0, k1 = split_range(T, world, rank)
    for it in range(8):   # alternating the two-call form and the fused one, on the same areas and epochs
        out = torch.full((H * HD,), float("nan"), device=dev)
        if it % 2 == 0:
            attn.decode_partial(ex.ml, ex.o, tq, tk, tv, k0, k1, H, KV, HD, kd)
            ex.run(out)
        else:
            ex.decode(out, tq, tk, tv, k0, k1, KV, kd)
        torch.cuda.synchronize()
        worst = max(worst, oracle.rel_err(out.cpu().numpy(), full.cpu().numpy(), floor))
    ret[rank] = (worst, attn.device_status())
    ex.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_exchange_two_ranks_matches_whole_range():
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 20001, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    for r in range(2):
        err, status = ret[r]
        assert status == 0 and err <= oracle.REL_TOL, (r, err, status)


def test_exchange_all_shards_empty_gives_zero():
    """Every rank's part has l == 0 (no keys in any shard): the merge writes 0
    (or 0 times the gate), not 0/0."""
    from yllm_b200 import attn
    from yllm_b200.dist import PeerExchange

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    ex = PeerExchange(H, HD, device=dev)
    try:
        gate = torch.randn(H * HD, device=dev)
        for g in (None, gate):
            ex.ml[:, 0] = float("-inf")
            ex.ml[:, 1] = 0.0
            ex.o.fill_(1.0)
            out = torch.full((H * HD,), float("nan"), device=dev)
            ex.run(out, g)
            torch.cuda.synchronize()
            assert torch.count_nonzero(out).item() == 0, "empty shards must merge to 0"
        assert attn.device_status() == 0
    finally:
        ex.close()


def test_exchange_wait_runs_out_and_reports_401():
    """A bounded device wait that runs out, on one GPU and without a fault:
    a world-2 exchange whose second rank's area is a second buffer on this
    same GPU that no kernel ever publishes to.  With a 10 ms wait limit the
    call returns, yattn_device_status reads 401 (exchange timeout) and the
    output is NaN; after the status is cleared a fresh exchange works."""
    import ctypes as C

    from yllm_b200 import attn
    from yllm_b200._lib import call
    from yllm_b200.dist import PeerExchange

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    assert attn.device_status(clear=True) == 0
    areas = []
    try:
        for _ in range(2):
            a = C.c_void_p()
            call("yattn_exchange_area_alloc", 2, H, HD, C.byref(a))
            areas.append(a.value)
        arr = (C.c_void_p * 2)(*areas)
        payload = torch.zeros(H * (2 + HD), device=dev)
        payload[: H * 2].view(H, 2)[:, 1] = 1.0
        out = torch.zeros(H * HD, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        call("yattn_exchange_merge", payload.data_ptr(), payload.data_ptr() + H * 2 * 4, arr, 2, 0, H, HD,
             out.data_ptr(), None, 10_000_000, stream)
        t1.record()
        torch.cuda.synchronize()
        waited_ms = t0.elapsed_time(t1)
        assert attn.device_status(clear=True) == 401
        assert torch.isnan(out).all(), "a timed-out merge must leave NaN, not a stale result"
        assert 5.0 <= waited_ms < 1000.0, waited_ms   # the 10 ms bound, not the 2 s default
        assert attn.device_status() == 0
    finally:
        torch.cuda.synchronize()
        for a in areas:
            call("yattn_exchange_area_free", a)
    # the context is still usable: a fresh world-1 exchange merges correctly
    T = 3000
    q, k, v, kd = _case(13, T)
    tq, tk, tv = _to_dev(dev, q, k, v)
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, HD, kd)
    ex = PeerExchange(H, HD, device=dev)
    try:
        out = torch.full((H * HD,), float("nan"), device=dev)
        attn.decode_partial(ex.ml, ex.o, tq, tk, tv, 0, T, H, KV, HD, kd)
        ex.run(out)
        torch.cuda.synchronize()
        oracle.assert_close(out.cpu().numpy(), want, what="exchange after a timeout",
                            exact=oracle.exact_decode(q, k, v, T - 1, H, KV, HD, kd))
        assert attn.device_status() == 0
    finally:
        ex.close()


@pytest.mark.parametrize("T,gated", [(50, False), (3000, True), (40000, False)])
def test_fused_decode_exchange_world1(T, gated):
    """yattn_decode_exchange at world 1: the partial decode and the merge +
    exchange kernel (one split, and many) against the oracle, eagerly and in
    graph replays."""
    from yllm_b200 import attn
    from yllm_b200.dist import PeerExchange

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    q, k, v, kd = _case(21 + T, T)
    tq, tk, tv = _to_dev(dev, q, k, v)
    gate = np.random.default_rng(T).standard_normal(H * HD).astype(np.float32) if gated else None
    tg = torch.from_numpy(gate).to(dev) if gated else None
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, HD, kd, gate=gate)
    exact = oracle.exact_decode(q, k, v, T - 1, H, KV, HD, kd, gate=gate)
    ex = PeerExchange(H, HD, device=dev)
    try:
        for _ in range(2):
            out = torch.full((H * HD,), float("nan"), device=dev)
            ex.decode(out, tq, tk, tv, 0, T, KV, kd, gate=tg)
            torch.cuda.synchronize()
            oracle.assert_close(out.cpu().numpy(), want, what=f"fused decode exchange T{T}", exact=exact)
        out_g = torch.full((H * HD,), float("nan"), device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ex.decode(out_g, tq, tk, tv, 0, T, KV, kd, gate=tg)
        for _ in range(3):
            out_g.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            oracle.assert_close(out_g.cpu().numpy(), want, what=f"fused decode exchange T{T}, graph", exact=exact)
        del g
        assert attn.device_status() == 0
    finally:
        ex.close()


def test_fused_decode_exchange_empty_shard_world1():
    """A rank with no keys (k_begin == k_end) still takes part: at world 1 every head is 0."""
    from yllm_b200 import attn
    from yllm_b200.dist import PeerExchange

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    q, k, v, kd = _case(5, 64)
    tq, tk, tv = _to_dev(dev, q, k, v)
    ex = PeerExchange(H, HD, device=dev)
    try:
        out = torch.full((H * HD,), float("nan"), device=dev)
        ex.decode(out, tq, tk, tv, 10, 10, KV, kd)
        torch.cuda.synchronize()
        assert torch.count_nonzero(out).item() == 0
        assert attn.device_status() == 0
    finally:
        ex.close()
