"""GPU parity of the Gated DeltaNet kernels against the CPU oracle
(gdn_state_update, matvec.c:975-1004; rmsnorm_gated, matvec.c:1007-1021;
token-by-token prefill, engine.c:723-734).  Tolerance on outputs and on the
final fp32 state: per element |gpu - cpu| <= 2e-3 * max(|cpu|, f * rms(cpu)),
f = 1e-3 unless the CPU's own fp32 rounding against a float64 run of the same
recurrence (oracle.exact_gdn) needs more (oracle.noise_floor)."""
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


def _np(t):
    return t.detach().cpu().numpy().ravel()


def test_gdn_fixture_bits(dev):
    from yllm_b200 import fixtures
    from yllm_b200.configs import CFG5_GDN as c

    g = fixtures.gdn_inputs(c, 4, 3, seeded_state=True, device=dev)
    o = oracle.gdn_fixture(c, 4, 3, seeded_state=True)
    for name in ("S", "q", "k", "v", "z", "gate", "beta", "norm_w"):
        assert np.array_equal(_np(getattr(g, name)).view(np.uint32), o[name].view(np.uint32)), name


@pytest.mark.parametrize("epilogue", [False, True])
def test_gdn_decode_batch32(dev, epilogue):
    """BASELINE config 5b: 32 sequences, one token each, seeded state."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    n = c.batch
    g = fixtures.gdn_inputs(c, n, 1, seeded_state=True, device=dev)
    attn.gdn_decode(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, n, c.num_k_heads, c.head_dim, c.n_v_heads,
                    c.head_dim, norm_w=g.norm_w if epilogue else None, z=g.z if epilogue else None, eps=c.eps)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, n, 1, seeded_state=True)
    S_want, out_want = oracle.gdn_run(fx, c, n, 1, epilogue)
    S_ex, out_ex = oracle.exact_gdn(fx, c, n, 1, epilogue)
    oracle.assert_close(_np(g.out), out_want, what="gdn decode out", exact=out_ex)
    oracle.assert_close(_np(g.S), S_want, what="gdn decode state", exact=S_ex)


def test_gdn_dropin_matches_reference_signature(dev):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    g = fixtures.gdn_inputs(c, 1, 1, seeded_state=True, device=dev)
    attn.cuda_k_gdn_state_update(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, c.num_k_heads, c.head_dim, c.n_v_heads,
                                 c.head_dim)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, 1, 1, seeded_state=True)
    S_want, out_want = oracle.gdn_run(fx, c, 1, 1, False)
    S_ex, out_ex = oracle.exact_gdn(fx, c, 1, 1, False)
    oracle.assert_close(_np(g.out), out_want, what="drop-in out", exact=out_ex)
    oracle.assert_close(_np(g.S), S_want, what="drop-in state", exact=S_ex)


@pytest.mark.parametrize("n_seqs,T,seeded,epilogue", [(1, 37, True, True), (3, 100, False, False),
                                                      (2, 1, True, False)])
def test_gdn_prefill_small(dev, n_seqs, T, seeded, epilogue):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    g = fixtures.gdn_inputs(c, n_seqs, T, seeded_state=seeded, device=dev)
    attn.gdn_prefill(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, n_seqs, T, c.num_k_heads, c.head_dim, c.n_v_heads,
                     c.head_dim, norm_w=g.norm_w if epilogue else None, z=g.z if epilogue else None, eps=c.eps)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, n_seqs, T, seeded_state=seeded)
    S_want, out_want = oracle.gdn_run(fx, c, n_seqs, T, epilogue)
    S_ex, out_ex = oracle.exact_gdn(fx, c, n_seqs, T, epilogue)
    oracle.assert_close(_np(g.out), out_want, what=f"gdn prefill out {n_seqs}x{T}", exact=out_ex)
    oracle.assert_close(_np(g.S), S_want, what=f"gdn prefill state {n_seqs}x{T}", exact=S_ex)


def test_gdn_prefill_config5a_full(dev):
    """BASELINE config 5a: 4096 tokens from a zero state, 16 k-heads / 32 v-heads."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    T = c.tokens
    g = fixtures.gdn_inputs(c, 1, T, seeded_state=False, device=dev)
    attn.gdn_prefill(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, 1, T, c.num_k_heads, c.head_dim, c.n_v_heads,
                     c.head_dim, norm_w=g.norm_w, z=g.z, eps=c.eps)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, 1, T, seeded_state=False)
    S_want, out_want = oracle.gdn_run(fx, c, 1, T, True)
    S_ex, out_ex = oracle.exact_gdn(fx, c, 1, T, True)
    oracle.assert_close(_np(g.out), out_want, what="gdn 4096-token prefill out", exact=out_ex)
    oracle.assert_close(_np(g.S), S_want, what="gdn 4096-token prefill state", exact=S_ex)


@pytest.mark.parametrize("n_seqs,T,seeded", [(1, 63, True), (1, 64, True), (2, 65, True), (1, 200, False),
                                              (3, 129, True)])
def test_gdn_chunked_matches_recurrent_kernel(dev, n_seqs, T, seeded):
    """The chunked tensor-core prefill (64-token chunks, ragged last chunk,
    several sequences) and the token-by-token GPU kernel, which follows the
    reference's operation order, both against the oracle."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    D, NK, NV = c.head_dim, c.num_k_heads, c.n_v_heads
    a = fixtures.gdn_inputs(c, n_seqs, T, seeded_state=seeded, device=dev)
    b = fixtures.gdn_inputs(c, n_seqs, T, seeded_state=seeded, device=dev)
    attn.gdn_prefill(a.S, a.out, a.q, a.k, a.v, a.gate, a.beta, n_seqs, T, NK, D, NV, D, norm_w=a.norm_w, z=a.z,
                     eps=c.eps)
    attn.gdn_prefill_recurrent(b.S, b.out, b.q, b.k, b.v, b.gate, b.beta, n_seqs, T, NK, D, NV, D, norm_w=b.norm_w,
                               z=b.z, eps=c.eps)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, n_seqs, T, seeded_state=seeded)
    S_want, out_want = oracle.gdn_run(fx, c, n_seqs, T, True)
    S_ex, out_ex = oracle.exact_gdn(fx, c, n_seqs, T, True)
    for name, g_ in (("chunked", a), ("recurrent", b)):
        oracle.assert_close(_np(g_.out), out_want, what=f"{name} out {n_seqs}x{T}", exact=out_ex)
        oracle.assert_close(_np(g_.S), S_want, what=f"{name} state {n_seqs}x{T}", exact=S_ex)
    assert attn.device_status() == 0


def test_gdn_prefill_equals_decode_steps(dev):
    """T prefill tokens and T single-token decodes (two kernels, same recurrence) both match the oracle."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    T = 20
    a = fixtures.gdn_inputs(c, 1, T, seeded_state=True, device=dev)
    b = fixtures.gdn_inputs(c, 1, T, seeded_state=True, device=dev)
    D, NK, NV = c.head_dim, c.num_k_heads, c.n_v_heads
    attn.gdn_prefill(a.S, a.out, a.q, a.k, a.v, a.gate, a.beta, 1, T, NK, D, NV, D)
    for t in range(T):
        attn.gdn_decode(b.S, b.out[t], b.q[t], b.k[t], b.v[t], b.gate[t], b.beta[t], 1, NK, D, NV, D)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, 1, T, seeded_state=True)
    S_want, out_want = oracle.gdn_run(fx, c, 1, T, False)
    S_ex, out_ex = oracle.exact_gdn(fx, c, 1, T, False)
    for name, g_ in (("prefill", a), ("decode steps", b)):
        oracle.assert_close(_np(g_.out), out_want, what=f"gdn {name} out", exact=out_ex)
        oracle.assert_close(_np(g_.S), S_want, what=f"gdn {name} state", exact=S_ex)


def test_gdn_rejects_unsupported(dev):
    from yllm_b200 import _lib, attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    g = fixtures.gdn_inputs(c, 1, 1, seeded_state=False, device=dev)
    with pytest.raises(_lib.YattnError, match="head dims"):
        attn.gdn_decode(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, 1, 16, 64, 32, 64)
    with pytest.raises(_lib.YattnError, match="together"):
        attn.gdn_decode(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, 1, 16, 128, 32, 128, norm_w=g.norm_w)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gdn_prefill_vhead_shards_match_whole(dev, world):
    """Split by value head (no collective): each rank holds its heads' state,
    v, z, gate, beta and output densely and reads q/k through the k-head
    offset; the shards reproduce the unsharded call bit for bit."""
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c
    from yllm_b200.dist import gdn_vhead_shard

    D, NK, NV, T = c.head_dim, c.num_k_heads, c.n_v_heads, 48
    g = fixtures.gdn_inputs(c, 1, T, seeded_state=True, device=dev)
    S_whole = g.S.clone()
    attn.gdn_prefill(S_whole, g.out, g.q, g.k, g.v, g.gate, g.beta, 1, T, NK, D, NV, D, norm_w=g.norm_w, z=g.z,
                     eps=c.eps)
    for r in range(world):
        v0, v1, koff = gdn_vhead_shard(NV, NK, world, r)
        n = v1 - v0
        S = g.S[:, v0:v1].contiguous()
        out = torch.full((T, n * D), float("nan"), device=dev)
        attn.gdn_prefill(S, out, g.q.view(-1)[koff * D:], g.k.view(-1)[koff * D:],
                         g.v[:, v0 * D:v1 * D].contiguous(), g.gate[:, v0:v1].contiguous(),
                         g.beta[:, v0:v1].contiguous(), 1, T, NK, D, n, D, norm_w=g.norm_w,
                         z=g.z[:, v0 * D:v1 * D].contiguous(), eps=c.eps)
        torch.cuda.synchronize()
        assert torch.equal(out, g.out[:, v0 * D:v1 * D]), f"rank {r} output"
        assert torch.equal(S, S_whole[:, v0:v1]), f"rank {r} state"


def _ref_lib():
    return oracle.load("ref") if oracle.has_ref() else oracle.load("port")


@pytest.mark.parametrize("n_seqs,T,nk,hk,nv,hv,kw", [
    (32, 1, 16, 128, 32, 128, 4),     # config 5b decode step: the qwen35 GDN layer shape
    (2, 100, 2, 128, 4, 128, 4),      # a prefill chunk with a ragged last tile
    (3, 2, 2, 64, 6, 64, 4),          # fewer tokens than taps: the delay line keeps old rows
    (1, 33, 1, 256, 2, 128, 3),       # wide k heads, three taps
])
def test_gdn_inputs_matches_reference(dev, n_seqs, T, nk, hk, nv, hv, kw):
    """yattn_gdn_inputs against engine.c:785-821 run token by token (oracle/_ref's conv1d_update and
    l2norm_inplace).  Relative error <= 1e-5 (device expf / log1pf); the delay line is moved bit for bit."""
    from yllm_b200 import attn
    from test_oracle import _gdn_inputs_case, run_gdn_inputs

    rng = np.random.default_rng(1000 + T)
    c = _gdn_inputs_case(rng, n_seqs, T, nk, hk, nv, hv, kw)
    want = run_gdn_inputs(_ref_lib(), c, n_seqs, T, nk, hk, nv, hv, kw)
    t = {n: torch.from_numpy(np.ascontiguousarray(x)).to(dev) for n, x in c.items()}
    q = torch.zeros(n_seqs, T, nk * hk, device=dev)
    k = torch.zeros_like(q)
    v = torch.zeros(n_seqs, T, nv * hv, device=dev)
    gate = torch.zeros(n_seqs, T, nv, device=dev)
    beta = torch.zeros_like(gate)
    attn.gdn_inputs(t["qkv"], t["state"], t["w"], t["alpha"], t["beta_in"], t["dt"], t["a"], q, k, v, gate, beta,
                    n_seqs, T, kw, nk, hk, nv, hv, eps=1e-6)
    torch.cuda.synchronize()
    assert attn.device_status() == 0
    for name, got, ref in zip(("q", "k", "v", "gate", "beta"), (q, k, v, gate, beta), want[:5]):
        e = oracle.rel_err(_np(got), ref.ravel())
        assert e <= 1e-5, f"{name}: relative error {e:.2e}"
    assert np.array_equal(_np(t["state"]), want[5].ravel()), "delay line"
    assert np.array_equal(_np(t["qkv"]), c["qkv"].ravel()), "qkv must not be modified"


def test_gdn_layer_decode_from_projections(dev):
    """A qwen35 GDN layer step on the GPU from its projections: yattn_gdn_inputs, then yattn_gdn_decode with
    the rmsnorm_gated epilogue, against the oracle doing the same per token (engine.c:785-852)."""
    from yllm_b200 import attn
    from test_oracle import _gdn_inputs_case, run_gdn_inputs

    n_seqs, T, nk, hk, nv, hv, kw = 4, 3, 16, 128, 32, 128, 4
    lib = _ref_lib()
    rng = np.random.default_rng(77)
    c = _gdn_inputs_case(rng, n_seqs, T, nk, hk, nv, hv, kw)
    S0 = (0.05 * rng.standard_normal((n_seqs, nv, hv, hk))).astype(np.float32)
    z = rng.standard_normal((n_seqs, T, nv * hv)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(hv)).astype(np.float32)
    qr, kr, vr, gr, br, _ = run_gdn_inputs(lib, c, n_seqs, T, nk, hk, nv, hv, kw)
    S_ref = S0.copy()
    out_ref = np.zeros((n_seqs, T, nv * hv), np.float32)
    for s in range(n_seqs):
        for t_ in range(T):
            o = np.zeros(nv * hv, np.float32)
            Ss = np.ascontiguousarray(S_ref[s])
            lib.orc_gdn_step(Ss, o, qr[s, t_], kr[s, t_], vr[s, t_], gr[s, t_], br[s, t_], nk, hk, nv, hv,
                             norm_w.ctypes.data, np.ascontiguousarray(z[s, t_]).ctypes.data, 1e-6)
            S_ref[s] = Ss
            out_ref[s, t_] = o
    t = {n: torch.from_numpy(np.ascontiguousarray(x)).to(dev) for n, x in c.items()}
    S = torch.from_numpy(S0).to(dev)
    zt = torch.from_numpy(z).to(dev)
    nw = torch.from_numpy(norm_w).to(dev)
    out = torch.zeros(n_seqs, T, nv * hv, device=dev)
    q = torch.zeros(n_seqs, 1, nk * hk, device=dev)
    k = torch.zeros_like(q)
    v = torch.zeros(n_seqs, 1, nv * hv, device=dev)
    gate = torch.zeros(n_seqs, 1, nv, device=dev)
    beta = torch.zeros_like(gate)
    for t_ in range(T):   # one decode step per token: projections of token t_ of every sequence
        sl = {n: t[n][:, t_:t_ + 1].contiguous() for n in ("qkv", "alpha", "beta_in")}
        attn.gdn_inputs(sl["qkv"], t["state"], t["w"], sl["alpha"], sl["beta_in"], t["dt"], t["a"], q, k, v, gate,
                        beta, n_seqs, 1, kw, nk, hk, nv, hv)
        o = torch.zeros(n_seqs, nv * hv, device=dev)
        attn.gdn_decode(S, o, q, k, v, gate, beta, n_seqs, nk, hk, nv, hv, norm_w=nw,
                        z=zt[:, t_].contiguous(), eps=1e-6)
        out[:, t_] = o
    torch.cuda.synchronize()
    assert attn.device_status() == 0
    from types import SimpleNamespace
    fx = dict(S=S0, q=qr, k=kr, v=vr, z=z, gate=gr, beta=br, norm_w=norm_w)
    S_ex, out_ex = oracle.exact_gdn(fx, SimpleNamespace(head_dim=hk, num_k_heads=nk, n_v_heads=nv, eps=1e-6),
                                    n_seqs, T, True)
    oracle.assert_close(_np(out), out_ref.ravel(), what="GDN layer output", exact=out_ex)
    oracle.assert_close(_np(S), S_ref.ravel(), what="GDN state", exact=S_ex)
