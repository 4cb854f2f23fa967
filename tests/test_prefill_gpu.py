"""GPU parity of the tcgen05 prefill path against the CPU oracle (engine.c:533-563).

Tolerance: per element |gpu - cpu| <= 2e-3 * max(|cpu|, f * rms(cpu)), f = 1e-3
unless the CPU's own fp32 rounding against a float64 evaluation of the same
inputs (oracle.exact_prefill) needs more (oracle.noise_floor).  q is either
plain fp32, as the engine passes its projections (cuda_fwd.c:220), for the
default kernel (q split into fp16 hi + lo), or fp16-exact (config 2's fixture),
for which both the default kernel and the hi-only kernel a caller selects with
YATTN_PREFILL_Q_F16 are checked.  P is held as fp16 hi + lo, accumulation fp32.
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
    import yllm_b200.attn  # noqa: F401

    return torch.device("cuda:0")


def _case(dev, H, KV, hd, P0, B, seed, kv_extra=0, q_extra=0, gated=False, fp32_q=False, scale=0.5):
    rng = np.random.default_rng(seed)
    kd = KV * hd + kv_extra
    qs = H * hd + q_extra
    lib = oracle.load()
    q = (rng.standard_normal((B, qs)) * scale).astype(np.float32)
    if not fp32_q:
        q = oracle.f16_to_f32(oracle.f32_to_f16(q, lib=lib), lib=lib).reshape(B, qs)   # fp16-exact q
    n = P0 + B
    k = oracle.f32_to_f16((rng.standard_normal(n * kd) * scale).astype(np.float32), lib=lib)
    v = oracle.f32_to_f16((rng.standard_normal(n * kd) * 0.5).astype(np.float32), lib=lib)
    gate = rng.standard_normal((B, qs)).astype(np.float32) if gated else None
    t = lambda a: torch.from_numpy(a).to(dev)
    tk = t(k.view(np.int16)).view(torch.uint16)
    tv = t(v.view(np.int16)).view(torch.uint16)
    return dict(q=q, k=k, v=v, kd=kd, qs=qs, gate=gate, tq=t(q), tk=tk, tv=tv,
                tg=t(gate) if gated else None)


@pytest.mark.parametrize("H,KV,hd,P0,B", [
    (16, 8, 128, 0, 200), (16, 8, 128, 37, 100), (16, 8, 128, 0, 1), (16, 8, 128, 5, 129),
    (14, 2, 64, 0, 300), (32, 8, 64, 300, 64), (16, 2, 256, 0, 200), (8, 1, 256, 130, 70),
    (12, 4, 128, 0, 256), (4, 4, 128, 1000, 40),
])
def test_prefill_matches_oracle(dev, H, KV, hd, P0, B):
    from yllm_b200 import attn

    c = _case(dev, H, KV, hd, P0, B, seed=H + hd + P0 + B)
    want = oracle.attn_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"])
    exact = oracle.exact_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"])
    for q_f16 in (False, True):   # the default kernel and the hi-only one (q here is fp16-exact)
        out = torch.zeros(B, c["qs"], device=dev)
        attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], P0, B, H, KV, hd, c["kd"], c["qs"], q_f16=q_f16)
        torch.cuda.synchronize()
        oracle.assert_close(out.cpu().numpy()[:, :H * hd], want[:, :H * hd],
                            what=f"prefill H{H} KV{KV} hd{hd} P0{P0} B{B} q_f16={q_f16}", exact=exact[:, :H * hd])
        assert attn.device_status() == 0


def test_prefill_strides_and_dropin(dev):
    """q_stride > n_heads*head_dim (the engine passes hidden) and padded kv rows."""
    from yllm_b200 import attn

    H, KV, hd, P0, B = 8, 2, 128, 17, 150
    c = _case(dev, H, KV, hd, P0, B, seed=11, kv_extra=128, q_extra=64)
    out = torch.full((B, c["qs"]), 7.0, device=dev)
    attn.cuda_k_attn_prefill(out, c["tq"], c["tk"], c["tv"], P0, B, H, KV, hd, c["kd"], c["qs"])
    torch.cuda.synchronize()
    want = oracle.attn_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"])
    exact = oracle.exact_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"])
    got = out.cpu().numpy()
    oracle.assert_close(got[:, :H * hd], want[:, :H * hd], what="strided prefill", exact=exact[:, :H * hd])
    assert np.all(got[:, H * hd:] == 7.0), "columns past n_heads*head_dim must be untouched"


def test_prefill_gated(dev):
    from yllm_b200 import attn

    H, KV, hd, P0, B = 16, 2, 256, 0, 300
    c = _case(dev, H, KV, hd, P0, B, seed=5, gated=True)
    out = torch.zeros(B, c["qs"], device=dev)
    attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], P0, B, H, KV, hd, c["kd"], c["qs"], gate=c["tg"])
    want = oracle.attn_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"], gate=c["gate"])
    exact = oracle.exact_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"], gate=c["gate"])
    torch.cuda.synchronize()
    oracle.assert_close(out.cpu().numpy(), want, what="gated prefill", exact=exact)


def test_prefill_config2_full(dev):
    """Qwen3-0.6B shape, 2048 tokens, one call."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG2 as c

    p = fixtures.prefill_inputs(c, device=dev)
    f = oracle.prefill_fixture(c)
    want = oracle.attn_prefill(f["q"], f["k"], f["v"], 0, c.seq_len, c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim,
                               c.n_heads * c.head_dim)
    exact = oracle.exact_prefill(f["q"], f["k"], f["v"], 0, c.seq_len, c.n_heads, c.n_kv_heads, c.head_dim,
                                 c.kv_dim, c.n_heads * c.head_dim)
    for q_f16 in (True, False):   # the config's q is fp16: the hi-only kernel (the bench's) and the default one
        p.out.zero_()
        attn.attn_prefill(p.out, p.q, p.k, p.v, 0, c.seq_len, c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim,
                          c.n_heads * c.head_dim, q_f16=q_f16)
        torch.cuda.synchronize()
        oracle.assert_close(p.out.cpu().numpy(), want, what=f"config2 prefill q_f16={q_f16}", exact=exact)
    assert attn.device_status() == 0


def test_prefill_config5_gated_full(dev):
    """BASELINE config 5 gated attention prefill (4096 tokens, hd 256), every
    row of the one GPU call against the oracle's whole-sequence prefill; and the
    engine's chunked form (the last 64 tokens, keys 0..4095) gives those rows."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GATED_PREFILL as c

    S, H, hd = c.seq_len, c.n_heads, c.head_dim
    p = fixtures.prefill_inputs(c, device=dev)
    f = oracle.prefill_fixture(c)
    want = oracle.attn_prefill(f["q"], f["k"], f["v"], 0, S, H, c.n_kv_heads, hd, c.kv_dim, H * hd, gate=f["gate"])
    exact = oracle.exact_prefill(f["q"], f["k"], f["v"], 0, S, H, c.n_kv_heads, hd, c.kv_dim, H * hd,
                                 gate=f["gate"])
    for q_f16 in (False, True):   # the config's q is fp16: the default kernel and the hi-only one
        p.out.zero_()
        attn.attn_prefill(p.out, p.q, p.k, p.v, 0, S, H, c.n_kv_heads, hd, c.kv_dim, H * hd, gate=p.gate,
                          q_f16=q_f16)
        torch.cuda.synchronize()
        got = p.out.cpu().numpy()
        oracle.assert_close(got, want, what=f"config5 gated prefill (all 4096 rows) q_f16={q_f16}", exact=exact)
    assert attn.device_status() == 0
    B = 64
    chunk = oracle.attn_prefill(f["q"][S - B:], f["k"], f["v"], S - B, B, H, c.n_kv_heads, hd, c.kv_dim, H * hd,
                                gate=f["gate"][S - B:])
    oracle.assert_close(got[S - B:], chunk, what="config5 gated prefill (last chunk)", exact=exact[S - B:])


@pytest.mark.parametrize("scale", [0.5, 2.0, 4.0])
def test_prefill_fp32_q_config2_shape(dev, scale):
    """q as the engine passes it: plain fp32 (not fp16-exact), q and k drawn
    from N(0,1)*scale, at config 2's shape (16/8 heads, hd 128, 2048 tokens,
    full output).  Scale 4 gives score standard deviations near 16, sharply
    peaked rows, where a rounding of q to fp16 alone moves the scores by
    several 1e-3."""
    from yllm_b200 import attn

    H, KV, hd, B = 16, 8, 128, 2048
    c = _case(dev, H, KV, hd, 0, B, seed=int(scale * 10) + 1, fp32_q=True, scale=scale)
    out = torch.zeros(B, c["qs"], device=dev)
    attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], 0, B, H, KV, hd, c["kd"], c["qs"])
    want = oracle.attn_prefill(c["q"], c["k"], c["v"], 0, B, H, KV, hd, c["kd"], c["qs"])
    exact = oracle.exact_prefill(c["q"], c["k"], c["v"], 0, B, H, KV, hd, c["kd"], c["qs"])
    torch.cuda.synchronize()
    oracle.assert_close(out.cpu().numpy(), want, what=f"fp32 q prefill scale {scale}", exact=exact)
    assert attn.device_status() == 0


@pytest.mark.parametrize("H,KV,hd,P0,B,gated", [
    (16, 2, 256, 0, 1000, True), (14, 2, 64, 100, 300, False), (8, 1, 256, 130, 70, False),
])
def test_prefill_fp32_q_other_head_dims(dev, H, KV, hd, P0, B, gated):
    """fp32 q at head_dim 256 (the qwen35 gated shape) and 64."""
    from yllm_b200 import attn

    c = _case(dev, H, KV, hd, P0, B, seed=hd + B, gated=gated, fp32_q=True, scale=2.0)
    out = torch.zeros(B, c["qs"], device=dev)
    attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], P0, B, H, KV, hd, c["kd"], c["qs"], gate=c["tg"])
    want = oracle.attn_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"], gate=c["gate"])
    exact = oracle.exact_prefill(c["q"], c["k"], c["v"], P0, B, H, KV, hd, c["kd"], c["qs"], gate=c["gate"])
    torch.cuda.synchronize()
    oracle.assert_close(out.cpu().numpy(), want, what=f"fp32 q prefill H{H} hd{hd} gated={gated}", exact=exact)
    assert attn.device_status() == 0


def test_prefill_q_f16_flag_checks_its_claim(dev):
    """YATTN_PREFILL_Q_F16 promises fp16-exact q.  A call whose first query tile
    keeps that promise and whose second breaks it reports device status 202
    (the broken tile runs on q's hi plane alone); the same q without the flag
    matches the oracle."""
    from yllm_b200 import attn

    H, KV, hd, B = 8, 2, 128, 256
    c = _case(dev, H, KV, hd, 0, B, seed=99, fp32_q=True, scale=2.0)
    q = c["q"].copy()
    q[:128] = oracle.f16_to_f32(oracle.f32_to_f16(q[:128])).reshape(128, -1)
    tq = torch.from_numpy(q).to(dev)
    out = torch.zeros(B, c["qs"], device=dev)
    assert attn.device_status() == 0
    attn.attn_prefill(out, tq, c["tk"], c["tv"], 0, B, H, KV, hd, c["kd"], c["qs"], q_f16=True)
    torch.cuda.synchronize()
    assert attn.device_status() == 202
    assert attn.device_status() == 0
    attn.attn_prefill(out, tq, c["tk"], c["tv"], 0, B, H, KV, hd, c["kd"], c["qs"])
    want = oracle.attn_prefill(q, c["k"], c["v"], 0, B, H, KV, hd, c["kd"], c["qs"])
    exact = oracle.exact_prefill(q, c["k"], c["v"], 0, B, H, KV, hd, c["kd"], c["qs"])
    torch.cuda.synchronize()
    oracle.assert_close(out.cpu().numpy(), want, what="half fp16-exact, half fp32 q", exact=exact)
    assert attn.device_status() == 0


def test_prefill_last_row_equals_decode(dev):
    """The last prefill row and a decode at the same position (two kernels) both match the oracle's decode
    of that row."""
    from yllm_b200 import attn

    H, KV, hd, B = 32, 8, 128, 777
    c = _case(dev, H, KV, hd, 0, B, seed=3)
    out = torch.zeros(B, c["qs"], device=dev)
    attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], 0, B, H, KV, hd, c["kd"], c["qs"])
    dec = torch.zeros(H * hd, device=dev)
    attn.attn_decode(dec, c["tq"][B - 1].contiguous(), c["tk"], c["tv"], B - 1, H, KV, hd, c["kd"])
    torch.cuda.synchronize()
    want = oracle.attn_decode(c["q"][B - 1], c["k"], c["v"], B - 1, H, KV, hd, c["kd"])
    exact = oracle.exact_decode(c["q"][B - 1], c["k"], c["v"], B - 1, H, KV, hd, c["kd"])
    oracle.assert_close(out[B - 1].cpu().numpy(), want, what="prefill last row vs oracle decode", exact=exact)
    oracle.assert_close(dec.cpu().numpy(), want, what="decode vs oracle decode", exact=exact)


def test_prefill_rejects_bad_geometry(dev):
    from yllm_b200 import _lib, attn

    c = _case(dev, 8, 2, 128, 0, 10, seed=1)
    out = torch.zeros(10, c["qs"], device=dev)
    with pytest.raises(_lib.YattnError, match="head_dim"):
        attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], 0, 10, 8, 2, 96, c["kd"], c["qs"])
    with pytest.raises(_lib.YattnError, match="q_stride"):
        attn.attn_prefill(out, c["tq"], c["tk"], c["tv"], 0, 10, 8, 2, 128, c["kd"], 1022)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_prefill_kv_head_shards_match_whole(dev, world):
    """Split by KV head (each rank keeps whole GQA groups, no collective): the
    shards, addressed by pointer offsets with the row strides unchanged,
    reproduce the unsharded call bit for bit."""
    from yllm_b200 import attn
    from yllm_b200.dist import kv_head_shard

    H, KV, hd, P0, B = 16, 8, 128, 64, 300
    c = _case(dev, H, KV, hd, P0, B, seed=world)
    whole = torch.zeros(B, c["qs"], device=dev)
    attn.attn_prefill(whole, c["tq"], c["tk"], c["tv"], P0, B, H, KV, hd, c["kd"], c["qs"])
    parts = torch.full((B, c["qs"]), float("nan"), device=dev)
    for r in range(world):
        h0, h1, g0, g1 = kv_head_shard(H, KV, world, r)
        attn.attn_prefill(parts.view(-1)[h0 * hd:], c["tq"].view(-1)[h0 * hd:], c["tk"].view(-1)[g0 * hd:],
                          c["tv"].view(-1)[g0 * hd:], P0, B, h1 - h0, g1 - g0, hd, c["kd"], c["qs"])
    torch.cuda.synchronize()
    assert torch.equal(parts, whole)
