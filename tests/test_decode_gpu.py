"""GPU parity of the decode path against the CPU oracle (engine.c:1074-1096).

Tolerance: per element |gpu - cpu| <= 2e-3 * max(|cpu|, f * rms(cpu))
(oracle.assert_close), f = 1e-3 unless the CPU's own fp32 rounding, measured
against a float64 evaluation of the same inputs (oracle.exact_decode), needs a
higher floor (oracle.noise_floor).  Seeded-input plumbing is checked bit for bit.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    import yllm_b200.attn  # noqa: F401  (loads the CUDA library)

    return torch.device("cuda:0")


def _u16(t):
    return t.cpu().numpy().view(np.uint16)


# ------------------------------------------------------------- plumbing

def test_fixture_bits_match_oracle(dev):
    from yllm_b200 import fixtures
    from yllm_b200.configs import CFG1, CFG2, CFG3, CFG5_GATED_DECODE

    for cfg, layer, seq in [(CFG1, 0, 0), (CFG1, 23, 0), (CFG3, 5, 17), (CFG5_GATED_DECODE, 0, 3)]:
        d = fixtures.decode_inputs(cfg, layers=[layer], seqs=[seq], device=dev)
        o = oracle.decode_fixture(cfg, layer, seq)
        assert np.array_equal(_u16(d.k_view(0, 0)), o["k"]), (cfg.name, "k")
        assert np.array_equal(_u16(d.v_view(0, 0)), o["v"]), (cfg.name, "v")
        assert np.array_equal(d.q[0, 0].cpu().numpy().view(np.uint32), o["q"].view(np.uint32)), (cfg.name, "q")
        if cfg.gated:
            assert np.array_equal(d.gate[0, 0].cpu().numpy().view(np.uint32), o["gate"].view(np.uint32))
    p = fixtures.prefill_inputs(CFG2, device=dev)
    o = oracle.prefill_fixture(CFG2)
    assert np.array_equal(p.q.cpu().numpy().view(np.uint32), o["q"].view(np.uint32))
    assert np.array_equal(_u16(p.k), o["k"]) and np.array_equal(_u16(p.v), o["v"])


def test_gdn_fixture_bits_match_oracle(dev):
    from yllm_b200 import fixtures

    lib = oracle.load()
    n = 4096 * 32
    g = torch.empty(n, device=dev)
    b = torch.empty(n, device=dev)
    fixtures.gen_gdn_gates(g, b, 11, 12)
    gc = np.empty(n, np.float32)
    bc = np.empty(n, np.float32)
    lib.orc_gdn_gates(11, 12, 0, n, gc, bc)
    assert np.array_equal(g.cpu().numpy().view(np.uint32), gc.view(np.uint32))
    assert np.array_equal(b.cpu().numpy().view(np.uint32), bc.view(np.uint32))
    rows, H, D = 64, 16, 128
    qk = torch.empty(rows * H * D, device=dev)
    fixtures.gen_gdn_qk(qk, 21, rows, H, D, 1e-6, first_row=100)
    qc = np.empty(rows * H * D, np.float32)
    lib.orc_gdn_qk(21, 100, rows, H, D, 1e-6, qc)
    assert np.array_equal(qk.cpu().numpy().view(np.uint32), qc.view(np.uint32))


def test_checksum_matches_oracle(dev):
    from yllm_b200 import fixtures

    x = torch.randint(0, 65535, (3 * 65536 + 40,), dtype=torch.int32, device=dev)
    assert fixtures.checksum(x) == oracle.checksum(x.cpu().numpy())


def test_store_kv_rounds_like_engine(dev):
    from yllm_b200 import attn

    lib = oracle.load()
    hi = np.arange(0, 65536, 7, dtype=np.uint64) << np.uint64(16)
    lows = np.array([0, 1, 0x0FFF, 0x1000, 0x1001, 0x1FFF, 0x2000, 0xFFFF], dtype=np.uint64)
    f = (hi[:, None] | lows[None, :]).ravel().astype(np.uint32).view(np.float32)
    kv_dim = 128
    n = f.size // kv_dim * kv_dim
    f = f[:n]
    k = torch.from_numpy(f.copy()).to(dev)
    v = torch.from_numpy(f[::-1].copy()).to(dev)
    rows = n // kv_dim
    kc = torch.zeros((rows + 3) * kv_dim, dtype=torch.uint16, device=dev)
    vc = torch.zeros_like(kc)
    attn.store_kv(kc, vc, k, v, 3, kv_dim)
    torch.cuda.synchronize()
    assert np.array_equal(_u16(kc)[3 * kv_dim:], oracle.f32_to_f16(f, lib=lib))
    assert np.array_equal(_u16(vc)[3 * kv_dim:], oracle.f32_to_f16(f[::-1].copy(), lib=lib))
    assert not _u16(kc)[:3 * kv_dim].any()
    # drop-in single-row form
    attn.cuda_k_store_kv(kc, vc, k[:kv_dim], v[:kv_dim], 0, kv_dim)
    torch.cuda.synchronize()
    assert np.array_equal(_u16(kc)[:kv_dim], oracle.f32_to_f16(f[:kv_dim], lib=lib))


# ------------------------------------------------------------- decode parity

def _rand_case(dev, H, KV, hd, T, seed, kv_extra=0):
    rng = np.random.default_rng(seed)
    kd = KV * hd + kv_extra
    q = rng.standard_normal(H * hd).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    tq = torch.from_numpy(q).to(dev)
    tk = torch.from_numpy(k.view(np.int16)).to(dev).view(torch.uint16)
    tv = torch.from_numpy(v.view(np.int16)).to(dev).view(torch.uint16)
    return q, k, v, kd, tq, tk, tv


@pytest.mark.parametrize("H,KV,hd,T", [
    (14, 2, 64, 512), (14, 2, 64, 1), (14, 2, 64, 2), (32, 8, 128, 1000), (32, 8, 128, 33),
    (16, 2, 256, 700), (16, 16, 128, 65), (32, 4, 64, 300), (14, 4, 128, 129), (8, 1, 128, 4000),
    (3, 3, 64, 31), (24, 4, 256, 96),
])
def test_decode_matches_oracle(dev, H, KV, hd, T):
    from yllm_b200 import attn

    q, k, v, kd, tq, tk, tv = _rand_case(dev, H, KV, hd, T, seed=H * 1000 + T)
    out = torch.zeros(H * hd, device=dev)
    attn.attn_decode(out, tq, tk, tv, T - 1, H, KV, hd, kd)
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, hd, kd)
    exact = oracle.exact_decode(q, k, v, T - 1, H, KV, hd, kd)
    torch.cuda.synchronize()
    oracle.assert_close(out.cpu().numpy(), want, what=f"decode H{H} KV{KV} hd{hd} T{T}", exact=exact)
    # the drop-in entry point gives the same bits
    out2 = torch.zeros_like(out)
    attn.cuda_k_attn_decode(out2, tq, tk, tv, T - 1, H, KV, hd, kd)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    assert attn.device_status() == 0


def test_decode_padded_kv_rows(dev):
    """kv_dim larger than n_kv*head_dim (row padding) is honoured."""
    from yllm_b200 import attn

    H, KV, hd, T = 8, 2, 128, 300
    q, k, v, kd, tq, tk, tv = _rand_case(dev, H, KV, hd, T, seed=3, kv_extra=64)
    out = torch.zeros(H * hd, device=dev)
    attn.attn_decode(out, tq, tk, tv, T - 1, H, KV, hd, kd)
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, hd, kd)
    torch.cuda.synchronize()
    oracle.assert_close(out.cpu().numpy(), want, what="padded rows",
                        exact=oracle.exact_decode(q, k, v, T - 1, H, KV, hd, kd))


def test_decode_config1_all_layers(dev):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG1 as c

    d = fixtures.decode_inputs(c, device=dev)
    for layer in range(c.layers):
        attn.cuda_k_attn_decode(d.out[layer, 0], d.q[layer, 0], d.k_view(layer, 0), d.v_view(layer, 0),
                                d.ctx[0] - 1, c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim)
    torch.cuda.synchronize()
    for layer in range(c.layers):
        f = oracle.decode_fixture(c, layer, 0)
        want = oracle.attn_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim)
        exact = oracle.exact_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim)
        oracle.assert_close(d.out[layer, 0].cpu().numpy(), want, what=f"config1 layer {layer}", exact=exact)


def _pool(d):
    return (d.kv_pool.data_ptr(), d.kv_pool.numel() * d.kv_pool.element_size())


@pytest.mark.parametrize("pooled", [False, True])
def test_decode_config3_batched_plan(dev, pooled):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG3 as c

    ctx = c.ctx()
    # 16 of the 64 sequences (the shortest, the longest, and an even spread) x 4 of the 32 layers
    seqs = sorted(set([int(np.argmin(ctx)), int(np.argmax(ctx))] + list(range(0, 64, 4))))[:16]
    layers = [0, 9, 22, 31]
    d = fixtures.decode_inputs(c, layers=layers, seqs=seqs, device=dev)
    plan = attn.DecodePlan.build([x - 1 for x in d.ctx], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim,
                                 pool=_pool(d) if pooled else None)
    for li in range(len(layers)):
        items = attn.make_items([(d.q[li, si], d.out[li, si], d.k_ptr(li, si), d.v_ptr(li, si), None,
                                  d.ctx[si] - 1) for si in range(len(seqs))])
        plan.run(items)
    torch.cuda.synchronize()
    for li, layer in enumerate(layers):
        for si, s in enumerate(seqs):
            f = oracle.decode_fixture(c, layer, s)
            want = oracle.attn_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim,
                                      c.kv_dim)
            exact = oracle.exact_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim,
                                        c.kv_dim)
            oracle.assert_close(d.out[li, si].cpu().numpy(), want, what=f"config3 layer {layer} seq {s}",
                                exact=exact)
    assert attn.device_status() == 0


def test_decode_config4_long_context(dev):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG4 as c

    d = fixtures.decode_inputs(c, device=dev)
    attn.attn_decode(d.out[0, 0], d.q[0, 0], d.k_view(0, 0), d.v_view(0, 0), d.ctx[0] - 1, c.n_heads,
                     c.n_kv_heads, c.head_dim, c.kv_dim)
    torch.cuda.synchronize()
    f = oracle.decode_fixture(c, 0, 0)
    want = oracle.attn_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim)
    exact = oracle.exact_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim)
    oracle.assert_close(d.out[0, 0].cpu().numpy(), want, what="config4", exact=exact)


@pytest.mark.parametrize("pooled", [False, True])
def test_gated_decode_qwen35(dev, pooled):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GATED_DECODE as c

    seqs = list(range(c.n_seqs))   # all 32 sequences of the batch
    d = fixtures.decode_inputs(c, seqs=seqs, device=dev)
    plan = attn.DecodePlan.build([x - 1 for x in d.ctx], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim,
                                 pool=_pool(d) if pooled else None)
    items = attn.make_items([(d.q[0, si], d.out[0, si], d.k_ptr(0, si), d.v_ptr(0, si), d.gate[0, si],
                              d.ctx[si] - 1) for si in range(len(seqs))])
    plan.run(items)
    torch.cuda.synchronize()
    for si, s in enumerate(seqs):
        f = oracle.decode_fixture(c, 0, s)
        want = oracle.attn_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim,
                                  gate=f["gate"])
        exact = oracle.exact_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim,
                                    c.kv_dim, gate=f["gate"])
        oracle.assert_close(d.out[0, si].cpu().numpy(), want, what=f"gated decode seq {s}", exact=exact)


@pytest.mark.parametrize("H,KV,hd,ctxs", [
    (32, 8, 128, [1, 17, 128, 129, 2000, 5000]), (14, 2, 64, [512, 1, 300, 3000]),
    (16, 2, 256, [4096, 63, 64, 65]), (8, 1, 128, [9000, 5]), (24, 3, 64, [777, 1200]),
])
def test_pooled_batched_decode_ragged(dev, H, KV, hd, ctxs):
    """yattn_decode_run_pooled: items' K and V at arbitrary row offsets of one
    pool (tensor-copy kernels, one kv head per CTA) against the oracle."""
    from yllm_b200 import attn

    rng = np.random.default_rng(H * 7 + hd + len(ctxs))
    kd = KV * hd
    offs, rows = [], 3                      # leading rows belong to nobody
    for c in ctxs:
        offs.append(rows)
        rows += 2 * c + 5                   # K rows, V rows, a gap
    pool_np = oracle.f32_to_f16(rng.standard_normal(rows * kd).astype(np.float32)).reshape(rows, kd)
    pool = torch.from_numpy(pool_np.view(np.int16)).to(dev).view(torch.uint16)
    base = pool.data_ptr()
    qs = [rng.standard_normal(H * hd).astype(np.float32) for _ in ctxs]
    tq = [torch.from_numpy(q).to(dev) for q in qs]
    outs = [torch.full((H * hd,), float("nan"), device=dev) for _ in ctxs]
    plan = attn.DecodePlan.build([c - 1 for c in ctxs], H, KV, hd, kd, pool=(base, pool.numel() * 2))
    items = attn.make_items([(tq[i], outs[i], base + offs[i] * kd * 2, base + (offs[i] + c) * kd * 2, None, c - 1)
                             for i, c in enumerate(ctxs)])
    plan.run(items)
    torch.cuda.synchronize()
    for i, c in enumerate(ctxs):
        k = np.ascontiguousarray(pool_np[offs[i]:offs[i] + c]).reshape(-1)
        v = np.ascontiguousarray(pool_np[offs[i] + c:offs[i] + 2 * c]).reshape(-1)
        want = oracle.attn_decode(qs[i], k, v, c - 1, H, KV, hd, kd)
        oracle.assert_close(outs[i].cpu().numpy(), want, what=f"pooled H{H} KV{KV} hd{hd} ctx{c}",
                            exact=oracle.exact_decode(qs[i], k, v, c - 1, H, KV, hd, kd))
    assert attn.device_status() == 0


def test_split_partials_merge_to_full(dev):
    """decode_partial over disjoint key shards + merge_partials == whole-range decode."""
    from yllm_b200 import attn

    H, KV, hd, T = 32, 8, 128, 5000
    q, k, v, kd, tq, tk, tv = _rand_case(dev, H, KV, hd, T, seed=77)
    bounds = [0, 1, 1200, 1201, 3333, T]
    n = len(bounds) - 1
    ml = torch.zeros(n, H, 2, device=dev)
    o = torch.zeros(n, H, hd, device=dev)
    for i in range(n):
        attn.decode_partial(ml[i], o[i], tq, tk, tv, bounds[i], bounds[i + 1], H, KV, hd, kd)
    out = torch.zeros(H * hd, device=dev)
    attn.merge_partials(out, ml, o, n, H, hd)
    torch.cuda.synchronize()
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, hd, kd)
    oracle.assert_close(out.cpu().numpy(), want, what="split merge",
                        exact=oracle.exact_decode(q, k, v, T - 1, H, KV, hd, kd))
    # an empty shard (l = 0) is ignored by the merge
    ml2 = torch.cat([ml, torch.zeros(1, H, 2, device=dev)])
    o2 = torch.cat([o, torch.zeros(1, H, hd, device=dev)])
    out2 = torch.zeros_like(out)
    attn.merge_partials(out2, ml2, o2, n + 1, H, hd)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_packed_exchange_payload_merge(dev):
    """The multi-GPU exchange layout: each shard's partials written into a
    PartialExchange payload, the payloads laid end to end (what one
    all-gather produces) and merged by merge_partials_packed."""
    from yllm_b200 import attn
    from yllm_b200.dist import PartialExchange

    H, KV, hd, T = 32, 8, 128, 9000
    q, k, v, kd, tq, tk, tv = _rand_case(dev, H, KV, hd, T, seed=78)
    bounds = [0, 2250, 4500, 6750, T]
    exs = [PartialExchange(H, hd, device=dev) for _ in range(4)]
    for i, ex in enumerate(exs):
        attn.decode_partial(ex.ml, ex.o, tq, tk, tv, bounds[i], bounds[i + 1], H, KV, hd, kd)
    parts = torch.cat([ex.payload for ex in exs])
    out = torch.zeros(H * hd, device=dev)
    attn.merge_partials_packed(out, parts, 4, H, hd)
    torch.cuda.synchronize()
    want = oracle.attn_decode(q, k, v, T - 1, H, KV, hd, kd)
    oracle.assert_close(out.cpu().numpy(), want, what="packed exchange merge",
                        exact=oracle.exact_decode(q, k, v, T - 1, H, KV, hd, kd))


def test_repeated_runs_are_deterministic_and_reuse_workspace(dev):
    from yllm_b200 import attn

    H, KV, hd, T = 32, 8, 128, 20000
    q, k, v, kd, tq, tk, tv = _rand_case(dev, H, KV, hd, T, seed=5)
    outs = []
    for _ in range(3):
        out = torch.zeros(H * hd, device=dev)
        attn.attn_decode(out, tq, tk, tv, T - 1, H, KV, hd, kd)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_dropin_reports_misaligned_pointer(dev):
    from yllm_b200 import _lib, attn

    H, KV, hd, T = 8, 2, 64, 10
    q, k, v, kd, tq, tk, tv = _rand_case(dev, H, KV, hd, T, seed=1)
    out = torch.zeros(H * hd, device=dev)
    with pytest.raises(_lib.YattnError, match="aligned"):
        _lib.call_void("cuda_k_attn_decode", out.data_ptr(), tq.data_ptr(), tk.data_ptr() + 2, tv.data_ptr(),
                       T - 2, H, KV, hd, kd)


@pytest.mark.parametrize("kind,H,KV,hd,n_dims,theta,ctxs,gated,ctas", [
    (0, 32, 8, 128, 128, 500000.0, [1, 17, 64, 65, 700, 1500, 4096], False, 0),   # Llama-3-8B heads, llama pairs
    (1, 14, 2, 64, 64, 1000000.0, [512, 1, 300, 3000], False, 0),                 # Qwen2.5-0.5B heads, qwen pairs
    (2, 16, 2, 256, 64, 10000000.0, [4096, 63, 64, 65], True, 0),                 # qwen35 gated attention, M-RoPE
    # few CTAs: each runs many units of many tiles back to back, so the RoPE warp runs whole units
    # ahead of the ring (its q slots and arrives must still land in their tiles' phases)
    (0, 32, 8, 128, 128, 500000.0, [1, 17, 64, 65, 700, 1500, 4096], False, 3),
    (1, 14, 2, 64, 64, 1000000.0, [512, 1, 300, 3000, 2047], False, 2),
    (2, 16, 2, 256, 64, 10000000.0, [4096, 63, 64, 65, 1000], True, 2),
])
def test_fused_rope_store_decode(dev, kind, H, KV, hd, n_dims, theta, ctxs, gated, ctas):
    """yattn_decode_run_pooled_rope: the decode step's RoPE + KV store (engine.c:1052-1072; M-RoPE 921-934)
    fused into the attention launch.  Against the same step as two launches (yattn_rope_store_kv, then
    yattn_decode_run_pooled): the pool after the step (every cache row, the new ones included) is identical
    and the outputs agree; against the oracle, the new K rows are within one fp16 ulp of the reference's
    rope + f32_to_f16 (V bit-exact) and the outputs pass the parity bar.  q is left unrotated."""
    from yllm_b200 import attn

    rng = np.random.default_rng(kind * 31 + hd + len(ctxs))
    kd = KV * hd
    offs, rows = [], 3
    for c in ctxs:
        offs.append(rows)
        rows += 2 * c + 5
    hist = oracle.f32_to_f16(rng.standard_normal(rows * kd).astype(np.float32)).reshape(rows, kd)
    pool_a = torch.from_numpy(hist.view(np.int16)).to(dev).view(torch.uint16)
    pool_b = pool_a.clone()
    q = [rng.standard_normal(H * hd).astype(np.float32) for _ in ctxs]
    kn = [rng.standard_normal(kd).astype(np.float32) for _ in ctxs]
    vn = [rng.standard_normal(kd).astype(np.float32) for _ in ctxs]
    gates = [rng.standard_normal(H * hd).astype(np.float32) if gated else None for _ in ctxs]
    t = lambda x: torch.from_numpy(x).to(dev) if x is not None else None
    tk, tv, tg = [t(x) for x in kn], [t(x) for x in vn], [t(x) for x in gates]
    qa, qb = [t(x) for x in q], [t(x) for x in q]
    outa = [torch.full((H * hd,), float("nan"), device=dev) for _ in ctxs]
    outb = [torch.full((H * hd,), float("nan"), device=dev) for _ in ctxs]
    pos = [c - 1 for c in ctxs]
    kbase = lambda pool, i: pool.data_ptr() + offs[i] * kd * 2
    vbase = lambda pool, i: pool.data_ptr() + (offs[i] + ctxs[i]) * kd * 2
    # two launches: RoPE + store, then the pooled decode
    ritems = attn.make_rope_items([(qa[i], tk[i], tv[i], kbase(pool_a, i), vbase(pool_a, i), pos[i])
                                   for i in range(len(ctxs))])
    attn.rope_store_kv(ritems, len(ctxs), H, KV, hd, kd, kind, theta, n_rope_dims=n_dims)
    plan_a = attn.DecodePlan.build(pos, H, KV, hd, kd, pool=(pool_a.data_ptr(), pool_a.numel() * 2))
    plan_a.run(attn.make_items([(qa[i], outa[i], kbase(pool_a, i), vbase(pool_a, i), tg[i], pos[i])
                                for i in range(len(ctxs))]))
    # one launch
    plan_b = attn.DecodePlan.build(pos, H, KV, hd, kd, target_ctas=ctas, pool=(pool_b.data_ptr(), pool_b.numel() * 2))
    items_b = attn.make_items([(qb[i], outb[i], kbase(pool_b, i), vbase(pool_b, i), tg[i], pos[i])
                               for i in range(len(ctxs))])
    rows_b = attn.make_new_rows([(tk[i], tv[i]) for i in range(len(ctxs))])
    for _ in range(2):   # a repeat rewrites the same rows with the same values
        plan_b.run_rope(items_b, rows_b, kind, theta, n_rope_dims=n_dims)
    torch.cuda.synchronize()
    assert attn.device_status() == 0
    assert torch.equal(pool_a, pool_b), "fused store differs from the RoPE store kernel"
    for i in range(len(ctxs)):
        assert torch.equal(qb[i].cpu(), torch.from_numpy(q[i])), "q must be left unrotated"
    lib = oracle.load("ref") if oracle.has_ref() else oracle.load("port")
    pool_np = pool_b.cpu().numpy().view(np.uint16).reshape(rows, kd)
    for i, c in enumerate(ctxs):
        # the new rows against the reference's rope + f32_to_f16
        qr, kr = q[i].copy(), kn[i].copy()
        kc = np.zeros((c) * kd, np.uint16)
        vc = np.zeros((c) * kd, np.uint16)
        lib.orc_rope_store(qr, kr, vn[i].copy(), kc, vc, H, KV, hd, kd, kind, n_dims, pos[i], theta)
        krow = pool_np[offs[i] + pos[i]]
        vrow = pool_np[offs[i] + c + pos[i]]
        assert np.array_equal(vrow, vc[pos[i] * kd:]), f"V row of seq {i}"
        dk = np.abs(krow.astype(np.int32) - kc[pos[i] * kd:].astype(np.int32))
        assert dk.max() <= 1 and (dk != 0).sum() <= max(1, kd // 100), f"K row of seq {i}"
        # the outputs: the two paths, and the engine's attention over the stored cache with the reference's q
        k_i = np.ascontiguousarray(pool_np[offs[i]:offs[i] + c]).reshape(-1)
        v_i = np.ascontiguousarray(pool_np[offs[i] + c:offs[i] + 2 * c]).reshape(-1)
        want = oracle.attn_decode(qr, k_i, v_i, pos[i], H, KV, hd, kd, gate=gates[i])
        exact = oracle.exact_decode(qr, k_i, v_i, pos[i], H, KV, hd, kd, gate=gates[i])
        got_b = outb[i].cpu().numpy()
        oracle.assert_close(got_b, outa[i].cpu().numpy(), what=f"fused vs two launches, kind {kind} ctx {c}",
                            exact=exact)
        oracle.assert_close(got_b, want, what=f"fused RoPE store decode vs oracle, kind {kind} ctx {c}", exact=exact)
