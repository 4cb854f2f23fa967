"""Fused RoPE + KV store (yattn_rope_store_kv) against the reference's own
rope_inplace / rope_inplace_qwen / rope_inplace_mrope (matvec.c:890-939, from
the oracle's reference build when present) and the engine's f32_to_f16
(platform.c:340-379).  q is compared in fp32; the cache rows in fp16 bits,
where the device's sinf/cosf may move a value by one fp16 ulp (the only
difference the kernel allows itself; every other operation follows the
reference's fp32 order).

q's bar: per element |gpu - cpu| <= 1e-5 * max(|pair|, 1e-3 * rms(cpu)), where
|pair| is the norm of the element's rotation pair.  A rotation keeps that norm,
and a few-ulp difference in sin/cos moves both outputs by a few ulps of it;
measured against the output element alone, any cancellation in a*c - b*s
would inflate the relative error without any change in the arithmetic."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _ref_lib():
    # the reference build where it travelled with the tree, else the port (bit-equal on the CPU)
    return oracle.load("ref") if oracle.has_ref() else oracle.load("port")


@pytest.mark.parametrize("kind,H,KV,hd,n_dims,theta", [
    (0, 32, 8, 128, 128, 500000.0),      # LLaMA pairs (2j, 2j+1), Llama-3-8B heads
    (1, 14, 2, 64, 64, 1000000.0),       # Qwen half-split pairs, Qwen2.5-0.5B heads
    (2, 16, 2, 256, 64, 10000000.0),     # qwen35 M-RoPE: first 64 of 256 dims
])
def test_rope_store_matches_reference(dev, kind, H, KV, hd, n_dims, theta):
    from yllm_b200 import attn

    lib = _ref_lib()
    rng = np.random.default_rng(kind * 100 + hd)
    kd = KV * hd
    positions = [0, 1, 7, 511, 4095, 8191, 65537, 131071]
    rows = max(positions) + 2
    n = len(positions)
    q = rng.standard_normal((n, H * hd)).astype(np.float32)
    k = rng.standard_normal((n, kd)).astype(np.float32)
    v = rng.standard_normal((n, kd)).astype(np.float32)
    sentinel = 0x7BCD
    kc = torch.full((rows * kd,), sentinel, dtype=torch.int16, device=dev)
    vc = torch.full((rows * kd,), sentinel, dtype=torch.int16, device=dev)
    tq = torch.from_numpy(q).to(dev)
    tk = torch.from_numpy(k).to(dev)
    tv = torch.from_numpy(v).to(dev)
    items = attn.make_rope_items([(tq[i], tk[i], tv[i], kc, vc, positions[i]) for i in range(n)], device=dev)
    attn.rope_store_kv(items, n, H, KV, hd, kd, kind, theta, n_rope_dims=n_dims)
    torch.cuda.synchronize()
    assert attn.device_status() == 0

    # reference: engine.c:1052-1072 / 921-934 for each item, into a host copy of the cache
    q_ref, k_ref = q.copy(), k.copy()
    kc_ref = np.full(rows * kd, sentinel, np.uint16)
    vc_ref = np.full(rows * kd, sentinel, np.uint16)
    for i, pos in enumerate(positions):
        qi, ki = np.ascontiguousarray(q_ref[i]), np.ascontiguousarray(k_ref[i])
        lib.orc_rope_store(qi, ki, np.ascontiguousarray(v[i]), kc_ref, vc_ref, H, KV, hd, kd, kind, n_dims, pos,
                           theta)
        q_ref[i], k_ref[i] = qi, ki
    q_gpu = tq.cpu().numpy()
    e = oracle.rope_err(q_gpu, q_ref, kind, hd, n_dims)
    assert e <= 1e-5, f"q after RoPE: relative error {e:.2e}"

    kc_np = kc.cpu().numpy().view(np.uint16).reshape(rows, kd)
    vc_np = vc.cpu().numpy().view(np.uint16).reshape(rows, kd)
    kc_ref = kc_ref.reshape(rows, kd)
    vc_ref = vc_ref.reshape(rows, kd)
    assert np.array_equal(vc_np, vc_ref), "V rows differ from the engine's rounding"
    dk = np.abs(kc_np.astype(np.int32) - kc_ref.astype(np.int32))
    assert dk.max() <= 1, f"K rows off by {dk.max()} fp16 ulps"
    assert (dk != 0).mean() <= 0.01, f"{(dk != 0).mean():.3%} of K values differ by one ulp"
    # every other row is untouched
    written = np.zeros(rows, dtype=bool)
    written[positions] = True
    assert np.all(kc_np[~written] == sentinel) and np.all(vc_np[~written] == sentinel)


@pytest.mark.parametrize("kind,H,KV,hd,n_dims,theta,q_pad", [
    (1, 16, 8, 128, 128, 1000000.0, 0),     # Qwen3-0.6B prefill chunk
    (0, 32, 8, 128, 128, 500000.0, 64),     # llama, q rows with a wider stride
    (2, 16, 2, 256, 64, 10000000.0, 0),     # qwen35 gated attention layer
])
def test_rope_store_batch_matches_reference(dev, kind, H, KV, hd, n_dims, theta, q_pad):
    """yattn_rope_store_kv_batch: B consecutive tokens from pos_start, each row against orc_rope_store."""
    from yllm_b200 import attn

    lib = _ref_lib()
    rng = np.random.default_rng(7 + kind)
    kd = KV * hd
    B, pos_start = 300, 1700
    qs = H * hd + q_pad
    rows = pos_start + B + 5
    q = rng.standard_normal((B, qs)).astype(np.float32)
    k = rng.standard_normal((B, kd)).astype(np.float32)
    v = rng.standard_normal((B, kd)).astype(np.float32)
    sentinel = 0x1234
    kc = torch.full((rows * kd,), sentinel, dtype=torch.int16, device=dev)
    vc = torch.full((rows * kd,), sentinel, dtype=torch.int16, device=dev)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    attn.rope_store_kv_batch(tq, tk, tv, kc, vc, pos_start, B, H, KV, hd, kd, kind, theta, n_rope_dims=n_dims,
                             q_stride=qs)
    torch.cuda.synchronize()
    assert attn.device_status() == 0

    q_ref, k_ref = q.copy(), k.copy()
    kc_ref = np.full(rows * kd, sentinel, np.uint16)
    vc_ref = np.full(rows * kd, sentinel, np.uint16)
    for b in range(B):
        qi, ki = np.ascontiguousarray(q_ref[b, :H * hd]), np.ascontiguousarray(k_ref[b])
        lib.orc_rope_store(qi, ki, np.ascontiguousarray(v[b]), kc_ref, vc_ref, H, KV, hd, kd, kind, n_dims,
                           pos_start + b, theta)
        q_ref[b, :H * hd], k_ref[b] = qi, ki
    q_gpu = tq.cpu().numpy()
    assert np.array_equal(q_gpu[:, H * hd:], q[:, H * hd:]), "padding columns of q were touched"
    e = oracle.rope_err(q_gpu[:, :H * hd], q_ref[:, :H * hd], kind, hd, n_dims)
    assert e <= 1e-5, f"q after RoPE: relative error {e:.2e}"
    kc_np = kc.cpu().numpy().view(np.uint16)
    vc_np = vc.cpu().numpy().view(np.uint16)
    assert np.array_equal(vc_np, vc_ref), "V rows differ from the engine's rounding"
    dk = np.abs(kc_np.astype(np.int32) - kc_ref.astype(np.int32))
    assert dk.max() <= 1, f"K rows off by {dk.max()} fp16 ulps"
    assert (dk != 0).mean() <= 0.01


def _norm_weights(rng, hd, f16):
    w = (1.0 + 0.3 * rng.standard_normal((2, hd))).astype(np.float32)
    if f16:
        w = oracle.f32_to_f16(w).reshape(2, hd)
    return w


@pytest.mark.parametrize("kind,H,KV,hd,n_dims,theta,f16", [
    (1, 16, 8, 128, 128, 1000000.0, False),   # Qwen3-0.6B: QK-norm then the qwen half-split rotation
    (1, 16, 8, 128, 128, 1000000.0, True),    # the same with fp16 norm weights
    (2, 16, 2, 256, 64, 10000000.0, False),   # qwen35 gated attention: QK-norm then M-RoPE on 64 of 256 dims
    (2, 16, 2, 256, 64, 10000000.0, True),
])
def test_qknorm_rope_store_matches_reference(dev, kind, H, KV, hd, n_dims, theta, f16):
    """QK-norm (rmsnorm of every q and k head with the layer's weights, engine.c:915-919 / 1036-1045) fused
    into the RoPE store, against the reference's rmsnorm + rope + f32_to_f16 per item (oracle/_ref)."""
    from yllm_b200 import attn

    lib = _ref_lib()
    rng = np.random.default_rng(31 * hd + kind + f16)
    kd = KV * hd
    positions = [0, 3, 511, 4095, 70000]
    rows = max(positions) + 1
    n = len(positions)
    q = (3.0 * rng.standard_normal((n, H * hd))).astype(np.float32)   # unnormalised projections
    k = (3.0 * rng.standard_normal((n, kd))).astype(np.float32)
    v = rng.standard_normal((n, kd)).astype(np.float32)
    w = _norm_weights(rng, hd, f16)
    eps = 1e-6
    kc = torch.zeros(rows * kd, dtype=torch.int16, device=dev)
    vc = torch.zeros_like(kc)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    wt = torch.from_numpy(w.view(np.int16) if f16 else w).to(dev)
    items = attn.make_rope_items([(tq[i], tk[i], tv[i], kc, vc, positions[i]) for i in range(n)], device=dev)
    attn.rope_store_kv(items, n, H, KV, hd, kd, kind, theta, n_rope_dims=n_dims,
                       norm=attn.qk_norm(wt[0], wt[1], eps))
    torch.cuda.synchronize()
    assert attn.device_status() == 0
    assert torch.equal(tk, torch.from_numpy(k).to(dev)), "k must not be modified"
    q_ref, k_ref = q.copy(), k.copy()
    kc_ref = np.zeros(rows * kd, np.uint16)
    vc_ref = np.zeros(rows * kd, np.uint16)
    wq, wk = np.ascontiguousarray(w[0]), np.ascontiguousarray(w[1])
    for i, pos in enumerate(positions):
        qi, ki = np.ascontiguousarray(q_ref[i]), np.ascontiguousarray(k_ref[i])
        lib.orc_qknorm_rope_store(qi, ki, np.ascontiguousarray(v[i]), kc_ref, vc_ref, H, KV, hd, kd, kind, n_dims,
                                  pos, theta, wq.ctypes.data, wk.ctypes.data, 1 if f16 else 0, eps)
        q_ref[i] = qi
    e = oracle.rope_err(tq.cpu().numpy(), q_ref, kind, hd, n_dims)
    assert e <= 1e-5, f"q after QK-norm + RoPE: relative error {e:.2e}"
    kc_np = kc.cpu().numpy().view(np.uint16)
    vc_np = vc.cpu().numpy().view(np.uint16)
    assert np.array_equal(vc_np, vc_ref), "V rows differ from the engine's rounding"
    dk = np.abs(kc_np.astype(np.int32) - kc_ref.astype(np.int32))
    assert dk.max() <= 1, f"K rows off by {dk.max()} fp16 ulps"
    assert (dk != 0).sum() <= max(1, 0.01 * n * kd), f"{(dk != 0).sum()} K values differ by one ulp"


def test_qknorm_rope_store_batch_matches_reference(dev):
    """The batch form (a prefill chunk of consecutive tokens) with QK-norm, qwen35 shape."""
    from yllm_b200 import attn

    lib = _ref_lib()
    kind, H, KV, hd, n_dims, theta, eps = 2, 16, 2, 256, 64, 10000000.0, 1e-6
    rng = np.random.default_rng(5)
    kd = KV * hd
    B, pos_start = 200, 4000
    rows = pos_start + B
    q = (2.0 * rng.standard_normal((B, H * hd))).astype(np.float32)
    k = (2.0 * rng.standard_normal((B, kd))).astype(np.float32)
    v = rng.standard_normal((B, kd)).astype(np.float32)
    w = _norm_weights(rng, hd, False)
    kc = torch.zeros(rows * kd, dtype=torch.int16, device=dev)
    vc = torch.zeros_like(kc)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    wt = torch.from_numpy(w).to(dev)
    attn.rope_store_kv_batch(tq, tk, tv, kc, vc, pos_start, B, H, KV, hd, kd, kind, theta, n_rope_dims=n_dims,
                             norm=attn.qk_norm(wt[0], wt[1], eps))
    torch.cuda.synchronize()
    assert attn.device_status() == 0
    q_ref, k_ref = q.copy(), k.copy()
    kc_ref = np.zeros(rows * kd, np.uint16)
    vc_ref = np.zeros(rows * kd, np.uint16)
    for b in range(B):
        qi, ki = np.ascontiguousarray(q_ref[b]), np.ascontiguousarray(k_ref[b])
        lib.orc_qknorm_rope_store(qi, ki, np.ascontiguousarray(v[b]), kc_ref, vc_ref, H, KV, hd, kd, kind, n_dims,
                                  pos_start + b, theta, w[0].ctypes.data, w[1].ctypes.data, 0, eps)
        q_ref[b] = qi
    e = oracle.rope_err(tq.cpu().numpy(), q_ref, kind, hd, n_dims)
    assert e <= 1e-5, f"q after QK-norm + RoPE: relative error {e:.2e}"
    assert np.array_equal(vc.cpu().numpy().view(np.uint16), vc_ref)
    dk = np.abs(kc.cpu().numpy().view(np.uint16).astype(np.int32) - kc_ref.astype(np.int32))
    assert dk.max() <= 1 and (dk != 0).mean() <= 0.01
