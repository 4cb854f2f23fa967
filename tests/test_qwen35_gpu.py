"""One decode step of a qwen35 hybrid block on the GPU, as one sequence of
library calls, from the layer inputs to the attention output (engine.c:760-960):

  GDN layer:        yattn_gdn_inputs (gates, conv1d delay line + silu, q/k l2norm;
                    engine.c:785-821) -> yattn_gdn_decode with the rmsnorm_gated
                    epilogue (matvec.c:975-1021; engine.c:831-852) -> the fp16
                    output projection (yattn_gemv_f16, matvec.c:111-122)
  gated attention:  fp16 projections of q, gate, k, v (engine.c:899-905) ->
                    QK-norm + M-RoPE + fp16 KV store in one launch
                    (yattn_rope_store_kv with YattnQkNorm; engine.c:915-934) ->
                    the gated decode over each sequence's cache (the batched plan
                    with a gate per item; engine.c:935-960)

The block's hidden-state rmsnorms and residual adds (engine.c:775, 871, 898) are
the engine's, outside this library, and are left out.  Every stage is checked
against the oracle run on the GPU's own input to that stage (the reference
build's functions where it travelled with the tree), so a rounding difference
upstream -- one fp16 ulp in a stored K row -- does not compound into the next
stage's check: the test shows the calls compose (layouts, strides, gate rows,
cache rows) and each stage keeps its own parity bar.  Shapes: config 5's
qwen3.5 layers (GDN 16 k / 32 v heads x 128; attention 16 q / 2 kv heads x 256,
M-RoPE on 64 dims), hidden 1024, four sequences at positions up to 4095."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

HID = 1024
NK, HK, NV, HV, KW = 16, 128, 32, 128, 4               # GDN layer
H, KVH, HD, NROT, THETA = 16, 2, 256, 64, 10000000.0   # gated attention layer
EPS = 1e-6


def _lib():
    return oracle.load("ref") if oracle.has_ref() else oracle.load("port")


def _np(t):
    return t.detach().cpu().numpy()


def _f16w(rng, out, inn, scale):
    return oracle.f32_to_f16((scale * rng.standard_normal(out * inn)).astype(np.float32)).reshape(out, inn)


def test_qwen35_block_decode_step():
    from yllm_b200 import attn
    from test_oracle import _gdn_inputs_case, run_gdn_inputs

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = _lib()
    rng = np.random.default_rng(35)
    positions = [100, 777, 2047, 4095]
    B = len(positions)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    tw = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)

    # ---------------- GDN layer ----------------
    c = _gdn_inputs_case(rng, B, 1, NK, HK, NV, HV, KW)
    S0 = (0.05 * rng.standard_normal((B, NV, HV, HK))).astype(np.float32)
    z = rng.standard_normal((B, NV * HV)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(HV)).astype(np.float32)
    w_o = _f16w(rng, HID, NV * HV, 0.02)
    g = {n: t(x) for n, x in c.items()}
    q = torch.zeros(B, 1, NK * HK, device=dev)
    k = torch.zeros_like(q)
    v = torch.zeros(B, 1, NV * HV, device=dev)
    gate = torch.zeros(B, 1, NV, device=dev)
    beta = torch.zeros_like(gate)
    S = t(S0)
    o_gdn = torch.zeros(B, NV * HV, device=dev)
    h1 = torch.zeros(B, HID, device=dev)
    attn.gdn_inputs(g["qkv"], g["state"], g["w"], g["alpha"], g["beta_in"], g["dt"], g["a"], q, k, v, gate, beta,
                    B, 1, KW, NK, HK, NV, HV, eps=EPS)
    attn.gdn_decode(S, o_gdn, q, k, v, gate, beta, B, NK, HK, NV, HV, norm_w=t(norm_w), z=t(z), eps=EPS)
    attn.gemv_f16(h1, tw(w_o), o_gdn, HID, NV * HV, B)

    # ---------------- gated attention layer ----------------
    w_q, w_g = _f16w(rng, H * HD, HID, 0.05), _f16w(rng, H * HD, HID, 0.05)
    w_k, w_v = _f16w(rng, KVH * HD, HID, 0.05), _f16w(rng, KVH * HD, HID, 0.05)
    qn_w = (1 + 0.2 * rng.standard_normal((2, HD))).astype(np.float32)
    kd = KVH * HD
    caches = []
    for p in positions:   # history rows 0..p-1; row p is written by the store below
        kc = np.zeros((p + 1) * kd, np.uint16)
        vc = np.zeros((p + 1) * kd, np.uint16)
        kc[: p * kd] = oracle.f32_to_f16(rng.standard_normal(p * kd).astype(np.float32))
        vc[: p * kd] = oracle.f32_to_f16(rng.standard_normal(p * kd).astype(np.float32))
        caches.append((kc, vc))
    tk_c = [tw(kc) for kc, _ in caches]
    tv_c = [tw(vc) for _, vc in caches]
    aq, ag = torch.zeros(B, H * HD, device=dev), torch.zeros(B, H * HD, device=dev)
    ak, av = torch.zeros(B, kd, device=dev), torch.zeros(B, kd, device=dev)
    for y, w in ((aq, w_q), (ag, w_g), (ak, w_k), (av, w_v)):
        attn.gemv_f16(y, tw(w), h1, w.shape[0], HID, B)
    torch.cuda.synchronize()
    aq_pre, ak_pre, av_pre = _np(aq).copy(), _np(ak).copy(), _np(av).copy()   # the store's inputs, for the oracle
    qnw = t(qn_w)
    items = attn.make_rope_items([(aq[i], ak[i], av[i], tk_c[i], tv_c[i], positions[i]) for i in range(B)])
    attn.rope_store_kv(items, B, H, KVH, HD, kd, attn.ROPE_MROPE, THETA, n_rope_dims=NROT,
                       norm=attn.qk_norm(qnw[0], qnw[1], EPS))
    out = torch.full((B, H * HD), float("nan"), device=dev)
    plan = attn.DecodePlan.build(positions, H, KVH, HD, kd)
    ditems = attn.make_items([(aq[i], out[i], tk_c[i], tv_c[i], ag[i], positions[i]) for i in range(B)])
    plan.run(ditems)
    torch.cuda.synchronize()
    assert attn.device_status() == 0

    # ---------------- stage checks, each on the GPU's input to that stage ----------------
    qr, kr, vr, gr, br, st = run_gdn_inputs(lib, c, B, 1, NK, HK, NV, HV, KW)
    for name, got, want in (("q", q, qr), ("k", k, kr), ("v", v, vr), ("gate", gate, gr), ("beta", beta, br)):
        e = oracle.rel_err(_np(got).ravel(), want.ravel())
        assert e <= 1e-5, f"gdn inputs {name}: relative error {e:.2e}"
    assert np.array_equal(_np(g["state"]), st), "conv delay line"

    qg, kg, vg, gg, bg = (_np(x).reshape(B, -1) for x in (q, k, v, gate, beta))
    S_ref = S0.copy()
    o_ref = np.zeros((B, NV * HV), np.float32)
    for s in range(B):
        Ss = np.ascontiguousarray(S_ref[s])
        lib.orc_gdn_step(Ss, o_ref[s], qg[s], kg[s], vg[s], gg[s], bg[s], NK, HK, NV, HV, norm_w.ctypes.data,
                         np.ascontiguousarray(z[s]).ctypes.data, EPS)
        S_ref[s] = Ss
    fx = dict(S=S0, q=qg, k=kg, v=vg, z=z, gate=gg, beta=bg, norm_w=norm_w)
    S_ex, o_ex = oracle.exact_gdn(fx, SimpleNamespace(head_dim=HK, num_k_heads=NK, n_v_heads=NV, eps=EPS), B, 1, True)
    oracle.assert_close(_np(o_gdn).ravel(), o_ref.ravel(), what="qwen35 block: GDN output", exact=o_ex)
    oracle.assert_close(_np(S).ravel(), S_ref.ravel(), what="qwen35 block: GDN state", exact=S_ex)

    def gemv_check(y, w, x, what):
        want = np.zeros((B, w.shape[0]), np.float32)
        lib.orc_gemv_f16(want, np.ascontiguousarray(w.ravel()), np.ascontiguousarray(x), w.shape[0], w.shape[1], B)
        exact = x.astype(np.float64) @ w.view(np.float16).astype(np.float64).T
        oracle.assert_close(y, want, tol=2e-5, what=f"qwen35 block: {what}", exact=exact)

    gemv_check(_np(h1), w_o, _np(o_gdn), "GDN output projection")
    h1n = _np(h1)
    gemv_check(aq_pre, w_q, h1n, "q projection")
    gemv_check(_np(ag), w_g, h1n, "gate projection")
    gemv_check(ak_pre, w_k, h1n, "k projection")
    gemv_check(av_pre, w_v, h1n, "v projection")

    q_rot = _np(aq)
    for s, p in enumerate(positions):
        qi, ki = aq_pre[s].copy(), ak_pre[s].copy()
        kc_ref = caches[s][0].copy()
        vc_ref = caches[s][1].copy()
        lib.orc_qknorm_rope_store(qi, ki, av_pre[s].copy(), kc_ref, vc_ref, H, KVH, HD, kd, attn.ROPE_MROPE, NROT, p,
                                  THETA, qn_w[0].ctypes.data, qn_w[1].ctypes.data, 0, EPS)
        e = oracle.rope_err(q_rot[s], qi, attn.ROPE_MROPE, HD, NROT)
        assert e <= 1e-5, f"QK-norm + M-RoPE q, seq {s}: relative error {e:.2e}"
        kg_c = _np(tk_c[s]).view(np.uint16)
        vg_c = _np(tv_c[s]).view(np.uint16)
        assert np.array_equal(vg_c, vc_ref), f"V row at {p}"
        dk = np.abs(kg_c.astype(np.int32) - kc_ref.astype(np.int32))
        assert dk.max() <= 1 and (dk != 0).sum() <= max(1, kd // 100), f"K row at {p}"
        # gated attention over the GPU's own cache (history + the row it stored)
        want = oracle.attn_decode(q_rot[s], kg_c, vg_c, p, H, KVH, HD, kd, gate=_np(ag)[s])
        exact = oracle.exact_decode(q_rot[s], kg_c, vg_c, p, H, KVH, HD, kd, gate=_np(ag)[s])
        oracle.assert_close(_np(out)[s], want, what=f"qwen35 block: gated attention, pos {p}", exact=exact)
