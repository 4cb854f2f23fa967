"""Our attention beside the reference's own CUDA attention kernels.

The reference's inference/cuda/cuda_kernels.cu is compiled unmodified for
sm_100a into oracle/_ref/libref_cuda.so.  Its cuda_k_attn_decode /
cuda_k_attn_prefill (cuda_kernels.cu:543-655: one block per query head,
one key per step) and ours get identical device inputs: the outputs must
agree within the parity tolerance (per element 2e-3 * max(|ref|, f * rms(ref)),
f = 1e-3 unless the reference kernel's own fp32 rounding against a float64
evaluation needs more), and ours must be faster.  Run with -s to see the
timings.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_gpu():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    if not oracle.has_ref_gpu():
        pytest.skip("oracle/_ref/libref_cuda.so not built (reference sources absent)")
    return oracle.load_ref_gpu()


def _kv(rng, rows, kd, dev):
    k = oracle.f32_to_f16(rng.standard_normal(rows * kd).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal(rows * kd).astype(np.float32))
    return (torch.from_numpy(k.view(np.int16)).to(dev).view(torch.uint16),
            torch.from_numpy(v.view(np.int16)).to(dev).view(torch.uint16))


def _time(fn, reps):
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / reps   # us per call


@pytest.mark.parametrize("H,KV,hd,T", [(14, 2, 64, 512),      # config 1 shape
                                       (32, 8, 128, 4096),    # one config-3 sequence
                                       (16, 2, 256, 4096)])   # qwen35 gated-attention shape, no gate
def test_decode_against_reference_cuda(ref_gpu, H, KV, hd, T):
    from yllm_b200 import attn

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(T + hd)
    kd = KV * hd
    qn = rng.standard_normal(H * hd).astype(np.float32)
    q = torch.from_numpy(qn).to(dev)
    k, v = _kv(rng, T, kd, dev)
    out_ref = torch.zeros(H * hd, device=dev)
    out = torch.zeros(H * hd, device=dev)
    run_ref = lambda: ref_gpu.cuda_k_attn_decode(out_ref.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                 T - 1, H, KV, hd, kd)
    run_ours = lambda: attn.attn_decode(out, q, k, v, T - 1, H, KV, hd, kd)
    t_ref = _time(run_ref, 3)
    t_ours = _time(run_ours, 20)
    exact = oracle.exact_decode(qn, k.cpu().numpy().view(np.uint16), v.cpu().numpy().view(np.uint16), T - 1, H, KV,
                                hd, kd)
    oracle.assert_close(out.cpu().numpy(), out_ref.cpu().numpy(), what=f"decode vs reference CUDA H{H} hd{hd} T{T}",
                        exact=exact)
    print(f"\ndecode H={H} KV={KV} hd={hd} T={T}: reference CUDA {t_ref:.1f} us, ours {t_ours:.1f} us, "
          f"{t_ref / t_ours:.1f}x")
    assert t_ours < t_ref / 2


def test_prefill_chunk_against_reference_cuda(ref_gpu):
    """The engine's batched prefill calls the kernel on chunks of at most 64 tokens (engine.c:622-654): the last
    64-token chunk of config 2 (Qwen3-0.6B shape, 2048 tokens)."""
    from yllm_b200 import attn

    dev = torch.device("cuda:0")
    H, KV, hd, S, B = 16, 8, 128, 2048, 64
    p0 = S - B
    kd = KV * hd
    rng = np.random.default_rng(2)
    qn = (0.5 * rng.standard_normal(B * H * hd)).astype(np.float32)   # plain fp32, as the engine passes it
    q = torch.from_numpy(qn).to(dev)
    k, v = _kv(rng, S, kd, dev)
    out_ref = torch.zeros(B * H * hd, device=dev)
    out = torch.zeros(B * H * hd, device=dev)
    run_ref = lambda: ref_gpu.cuda_k_attn_prefill(out_ref.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                  p0, B, H, KV, hd, kd, H * hd)
    run_ours = lambda: attn.attn_prefill(out, q, k, v, p0, B, H, KV, hd, kd, H * hd)
    t_ref = _time(run_ref, 3)
    t_ours = _time(run_ours, 20)
    exact = oracle.exact_prefill(qn, k.cpu().numpy().view(np.uint16), v.cpu().numpy().view(np.uint16), p0, B, H, KV,
                                 hd, kd, H * hd)
    oracle.assert_close(out.cpu().numpy().reshape(B, H * hd), out_ref.cpu().numpy().reshape(B, H * hd),
                        what="prefill chunk vs reference CUDA", exact=exact)
    print(f"\nprefill chunk B={B} at pos {p0}: reference CUDA {t_ref:.1f} us, ours {t_ours:.1f} us, "
          f"{t_ref / t_ours:.1f}x")
    assert t_ours < t_ref / 2


def test_gemv_against_reference_cuda(ref_gpu):
    """One 14336 x 4096 matrix (Llama-3-8B gate/up): the reference's cuda_k_gemv_q4k (one CTA per output row,
    cuda_kernels.cu:161-199) and its cuda_k_gemv_f16 on cuBLAS (x rounded to fp16, cuda_kernels.cu:53-87) beside
    ours.  Q4_K within 2e-5 (both fp32); fp16 within the parity tolerance (the reference rounds x)."""
    import ctypes as C

    from yllm_b200 import attn

    dev = torch.device("cuda:0")
    out, inn = 14336, 4096
    rng = np.random.default_rng(11)
    nb = inn // 256
    w4 = rng.integers(0, 256, (out, nb, 144), dtype=np.uint8)
    w4[:, :, 0:2] = (rng.uniform(0.5, 2, (out, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(out, nb, 2)
    w4[:, :, 2:4] = (rng.uniform(0.5, 2, (out, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(out, nb, 2)
    tw4 = torch.from_numpy(w4.reshape(-1)).to(dev)
    tw16 = torch.from_numpy((0.02 * rng.standard_normal((out, inn))).astype(np.float16).view(np.int16)).to(dev)
    xn = rng.standard_normal(inn).astype(np.float32)
    x = torch.from_numpy(xn).to(dev)
    xf16 = torch.empty(inn, dtype=torch.int16, device=dev)
    from test_gemv_gpu import q4k_dequant_f64
    exact = {"q4k": q4k_dequant_f64(w4.reshape(-1), out, inn) @ xn.astype(np.float64),
             "f16": tw16.cpu().numpy().view(np.float16).astype(np.float64) @ xn.astype(np.float64)}
    y_ref, y = torch.zeros(out, device=dev), torch.zeros(out, device=dev)
    err = C.create_string_buffer(256)
    handle = C.c_void_p()
    assert ref_gpu.cuda_k_cublas_create(C.byref(handle), err, 256) == 0, err.value
    try:
        for name, ours, theirs, tol in (
                ("q4k", lambda: attn.gemv_q4k(y, tw4, x, out, inn, 1),
                 lambda: ref_gpu.cuda_k_gemv_q4k(y_ref.data_ptr(), tw4.data_ptr(), x.data_ptr(), out, inn, err, 256),
                 2e-5),
                ("f16", lambda: attn.gemv_f16(y, tw16, x, out, inn, 1),
                 lambda: ref_gpu.cuda_k_gemv_f16(handle, y_ref.data_ptr(), tw16.data_ptr(), x.data_ptr(),
                                                 xf16.data_ptr(), out, inn, err, 256),
                 oracle.REL_TOL)):
            t_ref = _time(theirs, 20)
            t_ours = _time(ours, 20)
            oracle.assert_close(y.cpu().numpy(), y_ref.cpu().numpy(), tol=tol, what=f"gemv {name} vs reference",
                                exact=exact[name])
            print(f"\ngemv {name} {out}x{inn}: reference CUDA {t_ref:.1f} us, ours {t_ours:.1f} us, "
                  f"{t_ref / t_ours:.2f}x")
    finally:
        ref_gpu.cuda_k_cublas_destroy(handle)


def test_rope_store_against_reference_cuda(ref_gpu):
    """One layer of config 3's decode step (64 sequences, Llama-3-8B heads): the reference's CUDA block makes three
    launches per sequence (cuda_k_rope_llama_heads on q and on k, cuda_k_store_kv; cuda_fwd.c:136-147), ours one
    launch for all.  q within 1e-5; cache rows within one fp16 ulp (the reference's store rounds to nearest even, the
    engine's CPU store half-up; nvcc contracts the reference's rotation into FMAs)."""
    from yllm_b200 import attn
    from yllm_b200.configs import CFG3

    dev = torch.device("cuda:0")
    H, KV, hd, theta = 32, 8, 128, 500000.0
    kd = KV * hd
    ctx = CFG3.ctx()
    n = len(ctx)
    offs = np.cumsum([0] + ctx[:-1])
    rows = int(sum(ctx))
    rng = np.random.default_rng(3)
    q0 = torch.from_numpy(rng.standard_normal((n, H * hd)).astype(np.float32)).to(dev)
    k0 = torch.from_numpy(rng.standard_normal((n, kd)).astype(np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((n, kd)).astype(np.float32)).to(dev)
    caches = {name: (torch.zeros(rows * kd, dtype=torch.int16, device=dev),
                     torch.zeros(rows * kd, dtype=torch.int16, device=dev)) for name in ("ref", "ours")}
    q_ref, k_ref, q, k = q0.clone(), k0.clone(), q0.clone(), k0.clone()
    kc_r, vc_r = caches["ref"]
    kc_o, vc_o = caches["ours"]

    def run_ref():
        for i in range(n):
            pos = ctx[i] - 1
            ref_gpu.cuda_k_rope_llama_heads(q_ref[i].data_ptr(), H, hd, pos, theta)
            ref_gpu.cuda_k_rope_llama_heads(k_ref[i].data_ptr(), KV, hd, pos, theta)
            ref_gpu.cuda_k_store_kv(kc_r.data_ptr() + 2 * int(offs[i]) * kd, vc_r.data_ptr() + 2 * int(offs[i]) * kd,
                                    k_ref[i].data_ptr(), v[i].data_ptr(), pos, kd)

    items = attn.make_rope_items([(q[i], k[i], v[i], kc_o.data_ptr() + 2 * int(offs[i]) * kd,
                                   vc_o.data_ptr() + 2 * int(offs[i]) * kd, ctx[i] - 1) for i in range(n)])
    run_ours = lambda: attn.rope_store_kv(items, n, H, KV, hd, kd, attn.ROPE_LLAMA, theta)
    run_ref()
    run_ours()
    torch.cuda.synchronize()
    e = oracle.rope_err(q.cpu().numpy(), q_ref.cpu().numpy(), 0, hd, hd)
    assert e <= 1e-5, f"rope q vs reference CUDA: relative error {e:.2e}"
    for (a, b) in ((kc_o, kc_r), (vc_o, vc_r)):
        d = (a.cpu().numpy().view(np.uint16).astype(np.int32) - b.cpu().numpy().view(np.uint16).astype(np.int32))
        assert np.abs(d).max() <= 1
    # timing: each side repeats its work on already-rotated data (the cost does not depend on the values)
    t_ref = _time(run_ref, 3)
    t_ours = _time(run_ours, 20)
    print(f"\nrope + KV store, 64 sequences: reference CUDA {t_ref:.1f} us ({3 * n} launches), ours {t_ours:.1f} us "
          f"(1 launch), {t_ref / t_ours:.1f}x")
    assert t_ours < t_ref / 2
