"""The allocation-free decode entry point, yattn_attn_decode_noalloc.

It serves callers that cannot call cudaMalloc while decoding (a fixed device
memory budget, or an allocator that must not be re-entered from the decode
thread): its split-KV scratch is a static device array inside the library.
Each case is checked against the allocating entry point and against the CPU
oracle (engine.c:1074-1096 restated), on two calls in a row, and the device
status word must stay 0.  A misaligned gate is rejected on the device (status
103, read through yattn_device_status) without any access through it.
This file is collected last so a failure here leaves every other test run.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _noalloc(out, q, k, v, gate, pos, H, KV, hd, kd, stream):
    from yllm_b200._lib import call

    call("yattn_attn_decode_noalloc", out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
         gate.data_ptr() if gate is not None else None, pos, H, KV, hd, kd, stream)


def _case(dev, H, KV, hd, T, seed, gated=False):
    rng = np.random.default_rng(seed)
    kd = KV * hd
    qn = rng.standard_normal(H * hd).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    gn = rng.standard_normal(H * hd).astype(np.float32) if gated else None
    q = torch.from_numpy(qn).to(dev)
    tk = torch.from_numpy(k.view(np.int16)).to(dev).view(torch.uint16)
    tv = torch.from_numpy(v.view(np.int16)).to(dev).view(torch.uint16)
    gate = torch.from_numpy(gn).to(dev) if gated else None
    want = oracle.attn_decode(qn, k, v, T - 1, H, KV, hd, kd, gate=gn)
    exact = oracle.exact_decode(qn, k, v, T - 1, H, KV, hd, kd, gate=gn)
    return q, tk, tv, gate, kd, (want, exact)


@pytest.mark.parametrize("H,KV,hd,T,gated", [
    (32, 8, 128, 20000, False),   # many splits: scratch partials + merge counters in use
    (14, 2, 64, 512, False),      # Qwen2.5-0.5B decode shape
    (16, 2, 256, 3000, True),     # qwen35 gated attention
    (8, 2, 128, 20, False),       # one split: no partials
])
def test_noalloc_decode_matches_allocating_entry(H, KV, hd, T, gated):
    from yllm_b200 import attn

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    attn.device_status(clear=True)   # start from a clean status word
    q, k, v, gate, kd, want_cpu = _case(dev, H, KV, hd, T, seed=H + T, gated=gated)
    stream = torch.cuda.current_stream().cuda_stream
    ref = torch.zeros(H * hd, device=dev)
    attn.attn_decode(ref, q, k, v, T - 1, H, KV, hd, kd, gate=gate)
    outs = []
    for _ in range(2):   # the second call reuses the static scratch left by the first
        out = torch.full((H * hd,), float("nan"), device=dev)
        _noalloc(out, q, k, v, gate, T - 1, H, KV, hd, kd, stream)
        outs.append(out)
    torch.cuda.synchronize()
    want = ref.cpu().numpy()
    for out in outs:
        got = out.cpu().numpy()
        oracle.assert_close(got, want, what=f"noalloc vs yattn_attn_decode H{H} KV{KV} hd{hd} T{T}",
                            exact=want_cpu[1])
        oracle.assert_close(got, want_cpu[0], what=f"noalloc vs CPU oracle H{H} KV{KV} hd{hd} T{T}",
                            exact=want_cpu[1])
    assert attn.device_status() == 0


def test_noalloc_scratch_covers_every_geometry():
    """The plan keeps a query's split partials to about one wave of CTAs, so the
    4 MiB static scratch (minus its 256-byte header) holds them for every
    supported geometry -- head_dim up to 256, up to 8 query heads per kv head,
    any context length; the entry still rejects a larger need with -1.  The
    longest case also runs against the allocating entry."""
    from yllm_b200._lib import lib

    worst = 0
    for hd in (64, 128, 256):
        for kv in (1, 2, 4, 8, 16, 64):
            for T in (1, 1000, 32768, 1 << 20, 1 << 22):
                need = lib.yattn_decode_partial_workspace_bytes(T, 8 * kv, kv, hd)
                worst = max(worst, need)
    assert 0 < worst <= (4 << 20) - 256, worst

    from yllm_b200 import attn

    dev = torch.device("cuda:0")
    H, KV, hd, T = 64, 8, 256, 40000
    q, k, v, gate, kd, _ = _case(dev, H, KV, hd, T, seed=5)
    ref = torch.zeros(H * hd, device=dev)
    attn.attn_decode(ref, q, k, v, T - 1, H, KV, hd, kd)
    out = torch.full((H * hd,), float("nan"), device=dev)
    _noalloc(out, q, k, v, None, T - 1, H, KV, hd, kd, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_noalloc_device_failure_reaches_device_status():
    """A gate that is not 16-byte aligned is rejected on the device: the
    decode stops with status 103, which yattn_device_status reports (and
    clears); the next call with a good gate runs clean."""
    from yllm_b200 import attn

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    attn.device_status(clear=True)
    H, KV, hd, T = 16, 2, 256, 700
    q, k, v, gate, kd, want_cpu = _case(dev, H, KV, hd, T, seed=9, gated=True)
    stream = torch.cuda.current_stream().cuda_stream
    bad = torch.zeros(H * hd + 4, device=dev)
    bad[1:1 + H * hd].copy_(gate)
    out = torch.zeros(H * hd, device=dev)
    _noalloc(out, q, k, v, bad[1:], T - 1, H, KV, hd, kd, stream)   # 4 bytes off a 16-byte boundary
    torch.cuda.synchronize()
    assert attn.device_status(clear=True) == 103
    assert attn.device_status() == 0
    _noalloc(out, q, k, v, gate, T - 1, H, KV, hd, kd, stream)
    torch.cuda.synchronize()
    assert attn.device_status() == 0
    oracle.assert_close(out.cpu().numpy(), want_cpu[0], what="noalloc after a rejected call", exact=want_cpu[1])


def test_noalloc_rejects_wrapping_position():
    """pos = 2^32 - 1 would make the key range [0, pos + 1) wrap to empty: a
    host-side error, as yattn_attn_decode gives."""
    from yllm_b200._lib import YattnError

    dev = torch.device("cuda:0")
    q, k, v, gate, kd, _ = _case(dev, 8, 2, 128, 16, seed=3)
    out = torch.zeros(8 * 128, device=dev)
    with pytest.raises(YattnError, match="empty key range"):
        _noalloc(out, q, k, v, None, 0xFFFFFFFF, 8, 2, 128, kd, torch.cuda.current_stream().cuda_stream)
