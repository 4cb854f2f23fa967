"""GPU parity of the Gated DeltaNet kernels against the CPU oracle
(gdn_state_update, matvec.c:975-1004; rmsnorm_gated, matvec.c:1007-1021;
token-by-token prefill, engine.c:723-734).  Tolerance oracle.REL_TOL (2e-3,
relative to max(|cpu|, rms(cpu))) on outputs and on the final fp32 state."""
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
    oracle.assert_close(_np(g.out), out_want, what="gdn decode out")
    oracle.assert_close(_np(g.S), S_want, what="gdn decode state")


def test_gdn_dropin_matches_reference_signature(dev):
    from yllm_b200 import attn, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    g = fixtures.gdn_inputs(c, 1, 1, seeded_state=True, device=dev)
    attn.cuda_k_gdn_state_update(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, c.num_k_heads, c.head_dim, c.n_v_heads,
                                 c.head_dim)
    torch.cuda.synchronize()
    fx = oracle.gdn_fixture(c, 1, 1, seeded_state=True)
    S_want, out_want = oracle.gdn_run(fx, c, 1, 1, False)
    oracle.assert_close(_np(g.out), out_want, what="drop-in out")
    oracle.assert_close(_np(g.S), S_want, what="drop-in state")


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
    oracle.assert_close(_np(g.out), out_want, what=f"gdn prefill out {n_seqs}x{T}")
    oracle.assert_close(_np(g.S), S_want, what=f"gdn prefill state {n_seqs}x{T}")


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
    oracle.assert_close(_np(g.out), out_want, what="gdn 4096-token prefill out")
    oracle.assert_close(_np(g.S), S_want, what="gdn 4096-token prefill state")


@pytest.mark.parametrize("n_seqs,T,seeded", [(1, 63, True), (1, 64, True), (2, 65, True), (1, 200, False),
                                              (3, 129, True)])
def test_gdn_chunked_matches_recurrent_kernel(dev, n_seqs, T, seeded):
    """The chunked tensor-core prefill (64-token chunks, ragged last chunk,
    several sequences) against the token-by-token GPU kernel, which follows
    the reference's operation order."""
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
    oracle.assert_close(_np(a.out), _np(b.out), what=f"chunked vs recurrent out {n_seqs}x{T}")
    oracle.assert_close(_np(a.S), _np(b.S), what=f"chunked vs recurrent state {n_seqs}x{T}")
    assert attn.device_status() == 0


def test_gdn_prefill_equals_decode_steps(dev):
    """T prefill tokens == T single-token decodes (two kernels, same recurrence)."""
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
    oracle.assert_close(_np(a.out), _np(b.out), what="prefill vs decode out")
    oracle.assert_close(_np(a.S), _np(b.S), what="prefill vs decode state")


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
