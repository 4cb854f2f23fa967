"""GPU parity of the linear-layer glue (yattn_gemv_q4k / _f16 and the
cuda_k_gemv_* / cuda_k_gemm_* drop-ins) against the oracle: Q4_K weights
dequantised by the reference's q4k_block (matvec.c:40-59) and summed in fp32
(the arithmetic of cuda_kernels.cu:142-159); fp16 rows through the engine's
matmul (matvec.c:111-122).  The GPU sums in another order: per element
|gpu - cpu| <= 2e-5 * max(|cpu|, f * rms(cpu)), f = 1e-3 unless the CPU's own
fp32 summation, measured against a float64 product of the same dequantised
weights, needs more (oracle.noise_floor)."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
TOL = 2e-5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _ref_lib():
    return oracle.load("ref") if oracle.has_ref() else oracle.load("port")


def q4k_weights(rng, out, in_):
    """Random Q4_K rows: d, dmin small fp16, random 6-bit scales/mins and nibbles."""
    nb = in_ // 256
    blk = rng.integers(0, 256, (out, nb, 144), dtype=np.uint8)
    d = (rng.uniform(0.5, 2.0, (out, nb)) * 1e-3).astype(np.float16)
    dmin = (rng.uniform(0.5, 2.0, (out, nb)) * 1e-3).astype(np.float16)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(out, nb, 2)
    blk[:, :, 2:4] = dmin.view(np.uint8).reshape(out, nb, 2)
    return np.ascontiguousarray(blk.reshape(-1))


def q4k_dequant_f64(w, out, in_):
    """The published Q4_K block layout decoded in float64 for every block at once:
    [out, in_] weights d*sc*n - dmin*m (the decode of matvec.c:26-59)."""
    blk = np.asarray(w, np.uint8).reshape(out * (in_ // 256), 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float64)
    dmin = blk[:, 2:4].copy().view(np.float16).astype(np.float64)
    q = blk[:, 4:16].astype(np.int64)
    y = np.empty((blk.shape[0], 256))
    for g in range(8):
        if g < 4:
            sc, mn = q[:, g] & 63, q[:, g + 4] & 63
        else:
            sc = (q[:, g + 4] & 0xF) | ((q[:, g - 4] >> 6) << 4)
            mn = (q[:, g + 4] >> 4) | ((q[:, g] >> 6) << 4)
        nib = blk[:, 16 + (g // 2) * 32: 16 + (g // 2) * 32 + 32].astype(np.int64)
        nib = (nib >> 4) if g & 1 else (nib & 0xF)
        y[:, g * 32:(g + 1) * 32] = d * sc[:, None] * nib - (dmin[:, 0] * mn)[:, None]
    return y.reshape(out, in_)


@pytest.mark.parametrize("out,in_,B", [(4096, 4096, 1), (1000, 512, 3), (14336, 4096, 4), (96, 2048, 9),
                                      # one token: the tensor-core kernel at every k-slice count (rows of 56,
                                      # 2 and 1 blocks), a ragged last 16-row tile, and a 72-block row
                                      (4096, 14336, 1), (1000, 512, 1), (37, 256, 1), (64, 18432, 1),
                                      # tall matrices take 32-row tiles (ragged last tile in the second)
                                      (14336, 4096, 1), (9500, 4096, 1)])
def test_gemv_q4k_matches_reference(dev, out, in_, B):
    from yllm_b200 import attn

    rng = np.random.default_rng(out + in_ + B)
    w = q4k_weights(rng, out, in_)
    x = rng.standard_normal((B, in_)).astype(np.float32)
    want = np.zeros((B, out), np.float32)
    _ref_lib().orc_gemv_q4k(want, w, x, out, in_, B)
    tw, tx = torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev)
    y = torch.zeros(B, out, device=dev)
    attn.gemv_q4k(y, tw, tx, out, in_, B)
    torch.cuda.synchronize()
    exact = x.astype(np.float64) @ q4k_dequant_f64(w, out, in_).T
    oracle.assert_close(y.cpu().numpy(), want, tol=TOL, what=f"q4k gemv {out}x{in_} B{B}", exact=exact)


@pytest.mark.parametrize("out,in_,B", [(4096, 4096, 1), (1000, 1003, 2), (11008, 4096, 4), (64, 4096, 6)])
def test_gemv_f16_matches_engine_matmul(dev, out, in_, B):
    from yllm_b200 import attn

    rng = np.random.default_rng(out * 3 + in_ + B)
    w = (0.02 * rng.standard_normal((out, in_))).astype(np.float16).view(np.uint16).reshape(-1)
    x = rng.standard_normal((B, in_)).astype(np.float32)
    want = np.zeros((B, out), np.float32)
    _ref_lib().orc_gemv_f16(want, np.ascontiguousarray(w), x, out, in_, B)
    tw = torch.from_numpy(w.view(np.int16)).to(dev)
    tx = torch.from_numpy(x).to(dev)
    y = torch.zeros(B, out, device=dev)
    attn.gemv_f16(y, tw, tx, out, in_, B)
    torch.cuda.synchronize()
    exact = x.astype(np.float64) @ w.view(np.float16).reshape(out, in_).astype(np.float64).T
    oracle.assert_close(y.cpu().numpy(), want, tol=TOL, what=f"f16 gemv {out}x{in_} B{B}", exact=exact)


def test_gemv_dropins_match(dev):
    """The reference-named entry points give the same bits as the yattn_ calls they wrap."""
    from yllm_b200 import attn
    from yllm_b200._lib import lib

    rng = np.random.default_rng(5)
    out, in_, B = 512, 1024, 3
    w4 = torch.from_numpy(q4k_weights(rng, out, in_)).to(dev)
    w16 = torch.from_numpy((0.02 * rng.standard_normal((out, in_))).astype(np.float16).view(np.int16)).to(dev)
    x = torch.from_numpy(rng.standard_normal((B, in_)).astype(np.float32)).to(dev)
    err = C.create_string_buffer(256)
    for name_v, name_m, w, fn, extra in (("cuda_k_gemv_q4k", "cuda_k_gemm_q4k", w4, attn.gemv_q4k, ()),
                                         ("cuda_k_gemv_f16", "cuda_k_gemm_f16", w16, attn.gemv_f16, (None,))):
        ya, yb, yc, y1 = (torch.zeros(B, out, device=dev) for _ in range(4))
        fn(ya, w, x, out, in_, B)
        fn(y1, w, x, out, in_, 1)   # one token takes the single-token kernel, as the GEMV drop-in does
        pre = extra
        args_v = (*pre, yb.data_ptr(), w.data_ptr(), x.data_ptr(), *(() if not pre else (None,)), out, in_)
        assert getattr(lib, name_v)(*args_v, err, 256) == 0, err.value
        args_m = (*pre, yc.data_ptr(), w.data_ptr(), x.data_ptr(), *(() if not pre else (None,)), out, in_, B)
        assert getattr(lib, name_m)(*args_m, err, 256) == 0, err.value
        torch.cuda.synchronize()
        assert torch.equal(yb[0], y1[0]) and torch.equal(yc, ya), name_v


@pytest.mark.parametrize("outs,in_", [((4096, 1024, 1024), 4096), ((14336, 14336), 4096), ((37, 1000, 16, 999), 512),
                                      ((100,), 256), ((64, 48), 2048)])
def test_gemv_q4k_multi_matches_single_and_reference(dev, outs, in_):
    """One launch over matrices that share x (q/k/v, gate/up): every output equals the single-matrix call bit for
    bit, and the oracle within the GEMV tolerance."""
    from yllm_b200 import attn

    rng = np.random.default_rng(sum(outs) + in_)
    ws = [q4k_weights(rng, o, in_) for o in outs]
    x = rng.standard_normal(in_).astype(np.float32)
    tx = torch.from_numpy(x).to(dev)
    tws = [torch.from_numpy(w).to(dev) for w in ws]
    ys = [torch.full((o,), float("nan"), device=dev) for o in outs]
    ones = [torch.zeros(o, device=dev) for o in outs]
    attn.gemv_q4k_multi(ys, tws, outs, tx, in_)
    for y1, tw, o in zip(ones, tws, outs):
        attn.gemv_q4k(y1, tw, tx, o, in_, 1)
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(ys[i], ones[i]), f"matrix {i} ({o} x {in_}) differs from the single call"
        want = np.zeros(o, np.float32)
        _ref_lib().orc_gemv_q4k(want, ws[i], x, o, in_, 1)
        exact = q4k_dequant_f64(ws[i], o, in_) @ x.astype(np.float64)
        oracle.assert_close(ys[i].cpu().numpy(), want, tol=TOL, what=f"q4k multi {i}: {o}x{in_}", exact=exact)


def test_gemv_q4k_multi_rejects_bad_args(dev):
    from yllm_b200 import attn

    x = torch.zeros(256, device=dev)
    w = torch.zeros(144 * 4, dtype=torch.uint8, device=dev)
    y = torch.zeros(4, device=dev)
    with pytest.raises(ValueError):
        attn.gemv_q4k_multi([y] * 5, [w] * 5, [4] * 5, x, 256)   # more than four matrices
    with pytest.raises(RuntimeError):
        attn.gemv_q4k_multi([y], [w], [4], x, 100)               # in not a multiple of 256
