"""ctypes wrapper of the CPU oracle (oracle/liboracle.so, oracle/_ref/libyattn_ref.so).

Test infrastructure: used by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline only.  The fixture builders here restate yllm_b200/fixtures.py on the
CPU so both sides consume identical bytes.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"
PORT_SO = ORACLE_DIR / "liboracle.so"
REF_SO = ORACLE_DIR / "_ref" / "libyattn_ref.so"
REF_GPU_SO = ORACLE_DIR / "_ref" / "libref_cuda.so"   # the reference's own cuda_kernels.cu, built for sm_100a
# the reference source tree (present where the oracle's reference build is made; absent on GPU boxes):
# $YATTN_REF_TREE, else a checkout named `reference` beside this repository
REF_TREE = Path(os.environ["YATTN_REF_TREE"]) if os.environ.get("YATTN_REF_TREE") else ROOT.parent / "reference"

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
u32, u64, sz, dbl, flt, vp = C.c_uint32, C.c_uint64, C.c_size_t, C.c_double, C.c_float, C.c_void_p

_PROTOS = {
    "orc_build_kind": (C.c_int, []),
    "orc_max_threads": (C.c_int, []),
    "orc_set_threads": (None, [C.c_int]),
    "orc_f16_to_f32": (flt, [C.c_uint16]),
    "orc_f32_to_f16": (C.c_uint16, [flt]),
    "orc_softmax": (None, [f32p, u32]),
    "orc_rope_inplace": (None, [f32p, u32, u32, flt]),
    "orc_rope_inplace_qwen": (None, [f32p, u32, u32, flt]),
    "orc_rope_inplace_mrope": (None, [f32p, u32, u32, u32, flt]),
    "orc_l2norm_inplace": (None, [f32p, u32, flt]),
    "orc_gdn_state_update": (None, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, u32, u32, u32, u32]),
    "orc_rmsnorm_gated_f32": (None, [f32p, f32p, f32p, f32p, u32, flt]),
    "orc_f32_to_f16_buf": (None, [f32p, u16p, sz]),
    "orc_conv1d_update": (None, [f32p, f32p, f32p, u32, u32]),
    "orc_gdn_inputs": (None, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, u32, u32, u32,
                              u32, u32, u32, u32, u32, flt]),
    "orc_sess_kv_save": (C.c_int, [u16p, u32, u32, u32, u32, C.c_char_p]),
    "orc_sess_kv_load": (C.c_int, [u16p, u32, u32, u32, C.c_char_p, C.POINTER(u32)]),
    "orc_q4k_block": (None, [f32p, u8p]),
    "orc_matmul_f16": (None, [f32p, f32p, u16p, u32, u32]),
    "orc_matmul_q4k": (None, [f32p, f32p, u8p, u32, u32]),
    "orc_gemv_q4k": (None, [f32p, u8p, f32p, u32, u32, u32]),
    "orc_gemv_f16": (None, [f32p, u16p, f32p, u32, u32, u32]),
    "orc_rope_store": (None, [f32p, f32p, f32p, u16p, u16p, u32, u32, u32, u32, C.c_int, u32, u32, flt]),
    "orc_rmsnorm": (None, [f32p, f32p, vp, u32, flt, C.c_int]),
    "orc_qknorm_rope_store": (None, [f32p, f32p, f32p, u16p, u16p, u32, u32, u32, u32, C.c_int, u32, u32, flt, vp, vp,
                                     C.c_int, flt]),
    "orc_f16_to_f32_buf": (None, [u16p, f32p, sz]),
    "orc_attn_decode": (None, [f32p, f32p, u16p, u16p, u32, u32, u32, u32, u32]),
    "orc_attn_prefill": (None, [f32p, f32p, u16p, u16p, u32, u32, u32, u32, u32, u32, u32]),
    "orc_attn_decode_gated": (None, [f32p, f32p, f32p, u16p, u16p, u32, u32, u32, u32, u32]),
    "orc_attn_prefill_gated": (None, [f32p, f32p, f32p, u16p, u16p, u32, u32, u32, u32, u32, u32, u32]),
    "orc_gdn_step": (None, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, u32, u32, u32, u32, vp, vp, flt]),
    "orc_gdn_prefill": (None, [f32p, f32p, f32p, f32p, f32p, f32p, f32p, u32, u32, u32, u32, u32, vp, vp, flt]),
    "orc_det_log": (dbl, [dbl]),
    "orc_det_exp": (dbl, [dbl]),
    "orc_det_sincos": (None, [dbl, C.POINTER(dbl), C.POINTER(dbl)]),
    "orc_stream_draw": (u64, [u64, u64]),
    "orc_normal_d": (dbl, [u64, u64]),
    "orc_fill_normal": (None, [u64, u64, sz, dbl, f32p]),
    "orc_rope_rows": (None, [f32p, sz, u32, u32, u32, dbl]),
    "orc_round_f16": (None, [f32p, sz, u16p]),
    "orc_round_f16_inplace": (None, [f32p, sz]),
    "orc_round_bf16_inplace": (None, [f32p, sz]),
    "orc_gdn_gates": (None, [u64, u64, u64, sz, f32p, f32p]),
    "orc_gdn_qk": (None, [u64, u64, sz, u32, u32, flt, f32p]),
    "orc_ctx_len": (u32, [u64, u32, u32, u32]),
    "orc_checksum64": (u64, [vp, sz]),
}

_cache: dict = {}


def ensure_built() -> None:
    """Builds the oracle (and, where the reference tree exists, oracle/_ref)."""
    if PORT_SO.exists() and ((REF_SO.exists() and REF_GPU_SO.exists()) or not REF_TREE.exists()):
        return
    subprocess.run(["make", "-C", str(ORACLE_DIR)], check=True, capture_output=True)


def load(kind: str = "port") -> C.CDLL:
    """kind='port' (restated helpers) or 'ref' (reference matvec.c/platform.c linked)."""
    if kind in _cache:
        return _cache[kind]
    ensure_built()
    path = PORT_SO if kind == "port" else REF_SO
    if not path.exists():
        raise FileNotFoundError(f"{path} not built")
    lib = C.CDLL(str(path))
    for name, (res, args) in _PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _cache[kind] = lib
    return lib


def load_ref_gpu() -> C.CDLL:
    """The reference's CUDA kernels (inference/cuda/cuda_kernels.cu, unmodified): its attention entry points take
    device pointers and launch on the legacy default stream (cuda_kernels.h:55-63)."""
    if "ref_gpu" in _cache:
        return _cache["ref_gpu"]
    ensure_built()
    if not REF_GPU_SO.exists():
        raise FileNotFoundError(f"{REF_GPU_SO} not built")
    lib = C.CDLL(str(REF_GPU_SO))
    lib.cuda_k_attn_decode.restype = None
    lib.cuda_k_attn_decode.argtypes = [vp] * 4 + [u32] * 5
    lib.cuda_k_attn_prefill.restype = None
    lib.cuda_k_attn_prefill.argtypes = [vp] * 4 + [u32] * 7
    lib.cuda_k_gemv_q4k.restype = C.c_int
    lib.cuda_k_gemv_q4k.argtypes = [vp, vp, vp, u32, u32, C.c_char_p, sz]
    lib.cuda_k_gemv_f16.restype = C.c_int
    lib.cuda_k_gemv_f16.argtypes = [vp, vp, vp, vp, vp, u32, u32, C.c_char_p, sz]
    lib.cuda_k_cublas_create.restype = C.c_int
    lib.cuda_k_cublas_create.argtypes = [C.POINTER(vp), C.c_char_p, sz]
    lib.cuda_k_cublas_destroy.restype = None
    lib.cuda_k_cublas_destroy.argtypes = [vp]
    lib.cuda_k_rope_llama_heads.restype = None
    lib.cuda_k_rope_llama_heads.argtypes = [vp, u32, u32, u32, flt]
    lib.cuda_k_store_kv.restype = None
    lib.cuda_k_store_kv.argtypes = [vp, vp, vp, vp, u32, u32]
    _cache["ref_gpu"] = lib
    return lib


def has_ref_gpu() -> bool:
    try:
        load_ref_gpu()
        return True
    except (FileNotFoundError, OSError, subprocess.CalledProcessError):
        return False


def has_ref() -> bool:
    try:
        load("ref")
        return True
    except (FileNotFoundError, OSError, subprocess.CalledProcessError):
        return False


# ------------------------------------------------------------ fixture rows

GEN_F32, GEN_F16, GEN_F32_F16, GEN_F32_BF16 = 0, 1, 2, 3


def gen_rows(kind: int, n_rows: int, n_heads: int, hd: int, seed: int, first_row: int = 0, scale: float = 1.0,
             rope: bool = False, pos0: int = 0, theta: float = 1e6, lib=None) -> np.ndarray:
    """CPU restatement of yattn_gen_rows (dense rows, no stride)."""
    lib = lib or load()
    row = n_heads * hd
    x = np.empty(n_rows * row, dtype=np.float32)
    lib.orc_fill_normal(seed, first_row * row, x.size, float(scale), x)
    if rope:
        lib.orc_rope_rows(x, n_rows, n_heads, hd, pos0, float(theta))
    if kind == GEN_F16:
        out = np.empty(x.size, dtype=np.uint16)
        lib.orc_round_f16(x, x.size, out)
        return out.reshape(n_rows, row)
    if kind == GEN_F32_F16:
        lib.orc_round_f16_inplace(x, x.size)
    elif kind == GEN_F32_BF16:
        lib.orc_round_bf16_inplace(x, x.size)
    return x.reshape(n_rows, row)


def decode_fixture(cfg, layer: int, seq: int, lib=None) -> dict:
    """One (layer, seq) decode query of a DecodeCfg, as the GPU builds it."""
    from yllm_b200.configs import seed_of

    c = cfg.ctx()[seq]
    hd, H = cfg.head_dim, cfg.n_heads
    k = gen_rows(GEN_F16, c, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "k", layer, seq), rope=cfg.rope,
                 theta=cfg.theta, lib=lib)
    v = gen_rows(GEN_F16, c, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "v", layer, seq), lib=lib)
    qk = GEN_F32_BF16 if cfg.q_kind == "bf16" else GEN_F32
    q = gen_rows(qk, 1, H, hd, seed_of(cfg.cfg, "q", layer, seq), rope=cfg.rope, pos0=c - 1, theta=cfg.theta,
                 lib=lib)[0]
    gate = None
    if cfg.gated:
        gate = gen_rows(GEN_F32_BF16, 1, H, hd, seed_of(cfg.cfg, "gate", layer, seq), lib=lib)[0]
    return {"q": q, "k": k, "v": v, "gate": gate, "pos": c - 1}


def prefill_fixture(cfg, seq_len: Optional[int] = None, lib=None) -> dict:
    from yllm_b200.configs import seed_of

    S = seq_len or cfg.seq_len
    H, hd = cfg.n_heads, cfg.head_dim
    q = gen_rows(GEN_F32_F16, S, H, hd, seed_of(cfg.cfg, "q"), scale=cfg.scale, rope=cfg.rope, theta=cfg.theta,
                 lib=lib)
    k = gen_rows(GEN_F16, S, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "k"), scale=cfg.scale, rope=cfg.rope,
                 theta=cfg.theta, lib=lib)
    v = gen_rows(GEN_F16, S, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "v"), scale=cfg.scale, lib=lib)
    gate = None
    if cfg.gated:
        gate = gen_rows(GEN_F32_BF16, S, H, hd, seed_of(cfg.cfg, "gate"), lib=lib)
    return {"q": q, "k": k, "v": v, "gate": gate}


def gdn_fixture(cfg, n_seqs: int, T: int, seeded_state: bool, lib=None) -> dict:
    """CPU restatement of yllm_b200.fixtures.gdn_inputs (same bits)."""
    from yllm_b200.configs import seed_of

    lib = lib or load()
    D, NK, NV, c = cfg.head_dim, cfg.num_k_heads, cfg.n_v_heads, cfg.cfg
    rows = n_seqs * T
    S = np.zeros(n_seqs * NV * D * D, dtype=np.float32)
    if seeded_state:
        S = gen_rows(GEN_F32, n_seqs * NV * D, 1, D, seed_of(c, "state"), scale=cfg.state_scale, lib=lib).ravel()
    q = np.empty(rows * NK * D, np.float32)
    k = np.empty(rows * NK * D, np.float32)
    lib.orc_gdn_qk(seed_of(c, "gdn_q"), 0, rows, NK, D, cfg.eps, q)
    lib.orc_gdn_qk(seed_of(c, "gdn_k"), 0, rows, NK, D, cfg.eps, k)
    v = gen_rows(GEN_F32_BF16, rows, NV, D, seed_of(c, "gdn_v"), lib=lib).ravel()
    z = gen_rows(GEN_F32_BF16, rows, NV, D, seed_of(c, "z"), lib=lib).ravel()
    gate = np.empty(rows * NV, np.float32)
    beta = np.empty(rows * NV, np.float32)
    lib.orc_gdn_gates(seed_of(c, "gdn_a"), seed_of(c, "gdn_b"), 0, rows * NV, gate, beta)
    w = gen_rows(GEN_F32, 1, 1, D, seed_of(c, "norm_w"), scale=0.1, lib=lib).ravel()
    w = (w + np.float32(1.0)).astype(np.float32)
    return dict(S=S, q=q, k=k, v=v, z=z, gate=gate, beta=beta, norm_w=w)


def gdn_run(fx: dict, cfg, n_seqs: int, T: int, epilogue: bool, lib=None) -> tuple:
    """engine.c:723-734 + 826-852: token-by-token gdn_state_update (+ rmsnorm_gated)
    per sequence.  Returns (final state, outputs [n_seqs*T, n_vheads*128])."""
    lib = lib or load()
    D, NK, NV = cfg.head_dim, cfg.num_k_heads, cfg.n_v_heads
    S = fx["S"].copy()
    out = np.zeros(n_seqs * T * NV * D, np.float32)
    per_state = NV * D * D
    for s in range(n_seqs):
        Ss = S[s * per_state:(s + 1) * per_state]   # view: updated in place
        r0 = s * T
        sl = lambda a, width: np.ascontiguousarray(a[r0 * width:(r0 + T) * width])
        os_ = np.zeros(T * NV * D, np.float32)
        zs = sl(fx["z"], NV * D)
        w = fx["norm_w"]
        lib.orc_gdn_prefill(Ss, os_, sl(fx["q"], NK * D), sl(fx["k"], NK * D), sl(fx["v"], NV * D),
                            sl(fx["gate"], NV), sl(fx["beta"], NV), T, NK, D, NV, D,
                            w.ctypes.data if epilogue else None, zs.ctypes.data if epilogue else None, cfg.eps)
        out[r0 * NV * D:(r0 + T) * NV * D] = os_
    return S, out


# ------------------------------------------------------------ attention

def attn_decode(q, k, v, pos, n_heads, n_kv, hd, kv_dim, gate=None, lib=None) -> np.ndarray:
    lib = lib or load()
    out = np.zeros(n_heads * hd, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.uint16).ravel()
    v = np.ascontiguousarray(v, dtype=np.uint16).ravel()
    if gate is None:
        lib.orc_attn_decode(out, q, k, v, pos, n_heads, n_kv, hd, kv_dim)
    else:
        lib.orc_attn_decode_gated(out, q, np.ascontiguousarray(gate, dtype=np.float32), k, v, pos, n_heads, n_kv,
                                  hd, kv_dim)
    return out


def attn_prefill(q, k, v, pos_start, B, n_heads, n_kv, hd, kv_dim, q_stride, gate=None, lib=None) -> np.ndarray:
    lib = lib or load()
    out = np.zeros((B, q_stride), dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.float32).ravel()
    k = np.ascontiguousarray(k, dtype=np.uint16).ravel()
    v = np.ascontiguousarray(v, dtype=np.uint16).ravel()
    o = out.ravel()
    if gate is None:
        lib.orc_attn_prefill(o, q, k, v, pos_start, B, n_heads, n_kv, hd, kv_dim, q_stride)
    else:
        lib.orc_attn_prefill_gated(o, q, np.ascontiguousarray(gate, dtype=np.float32).ravel(), k, v, pos_start, B,
                                   n_heads, n_kv, hd, kv_dim, q_stride)
    return out


def f32_to_f16(x: np.ndarray, lib=None) -> np.ndarray:
    lib = lib or load()
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size, dtype=np.uint16)
    lib.orc_f32_to_f16_buf(x, out, x.size)
    return out


def f16_to_f32(h: np.ndarray, lib=None) -> np.ndarray:
    lib = lib or load()
    h = np.ascontiguousarray(h, dtype=np.uint16).ravel()
    out = np.empty(h.size, dtype=np.float32)
    lib.orc_f16_to_f32_buf(h, out, h.size)
    return out


def checksum(a: np.ndarray, lib=None) -> int:
    lib = lib or load()
    a = np.ascontiguousarray(a)
    return int(lib.orc_checksum64(a.ctypes.data, a.nbytes))


# ------------------------------------------------------------ tolerance

REL_TOL = 2e-3      # the north star's 2e-3 relative bar
RMS_FLOOR = 1e-3    # the per-element floor of the parity metric, in units of rms(cpu)

# (what, error, floor) of every assert_close in this process; the GPU test run
# writes it out (tests/conftest.py) so the achieved margins are on record.
PARITY_LOG: list = []


def rel_err(gpu: np.ndarray, cpu: np.ndarray, floor: float = RMS_FLOOR) -> float:
    """max_i |gpu_i - cpu_i| / max(|cpu_i|, floor * rms(cpu)).

    With the default floor this is the parity metric the work is held to:
    per element |gpu - cpu| <= 2e-3 * max(|cpu|, 1e-3 * rms(cpu))."""
    gpu = np.asarray(gpu, dtype=np.float64)
    cpu = np.asarray(cpu, dtype=np.float64)
    if not cpu.size:
        return 0.0
    rms = float(np.sqrt(np.mean(cpu * cpu)))
    den = np.maximum(np.abs(cpu), max(floor * rms, 1e-300))
    return float(np.max(np.abs(gpu - cpu) / den))


# The GPU kernels multiply fp32 values as fp16 hi + lo pairs (q and p in
# decode, q and P in prefill, every contraction of the chunked GDN): 22
# significant bits, unit roundoff 2^-22 against fp32's 2^-24.  Their rounding
# noise can therefore reach 4 times the CPU's, and a GPU-CPU difference
# carries both: 1 + 4 = 5.  PARITY_LOG records the measured ratio
# max|gpu - exact| / max|cpu - exact| of every check beside it.
NOISE_MARGIN = 5.0


def noise_floor(cpu: np.ndarray, exact: np.ndarray, margin: float = NOISE_MARGIN, tol: float = REL_TOL) -> float:
    """The rms floor that the CPU result's own rounding requires.

    `exact` is the same computation in float64.  The fp32 CPU result differs
    from it by up to e = max|cpu - exact|.  The returned floor is the smallest
    one at which a GPU-CPU difference of margin * e passes the bar `tol` on
    every element, and never below RMS_FLOOR: on short reductions this is
    RMS_FLOOR itself, on long ones (many keys, thousands of recurrent steps)
    the fp32 summation noise near zero outputs sets it."""
    cpu = np.asarray(cpu, dtype=np.float64)
    exact = np.asarray(exact, dtype=np.float64)
    rms = float(np.sqrt(np.mean(cpu * cpu))) if cpu.size else 0.0
    if rms == 0.0:
        return RMS_FLOOR
    e = float(np.max(np.abs(cpu - exact)))
    return max(RMS_FLOOR, margin * e / (tol * rms))


def assert_close(gpu: np.ndarray, cpu: np.ndarray, tol: float = REL_TOL, what: str = "",
                 exact: Optional[np.ndarray] = None, floor: Optional[float] = None) -> float:
    """Asserts the parity metric rel_err(gpu, cpu, floor) <= tol.  The floor is
    RMS_FLOOR unless `exact` (the float64 evaluation) is given, in which case
    it is noise_floor(cpu, exact)."""
    gpu = np.asarray(gpu)
    assert np.all(np.isfinite(gpu)), f"{what}: non-finite GPU output"
    if floor is None:
        floor = RMS_FLOOR if exact is None else noise_floor(cpu, exact, tol=tol)
    e = rel_err(gpu, cpu, floor)
    rec = {"what": what, "err": e, "floor": floor, "tol": tol, "err_at_1e-3": rel_err(gpu, cpu, RMS_FLOOR)}
    if exact is not None:   # how much noisier than the CPU the GPU result is, against float64
        g = np.asarray(gpu, np.float64).ravel()
        c = np.asarray(cpu, np.float64).ravel()
        x = np.asarray(exact, np.float64).ravel()
        ce = float(np.max(np.abs(c - x)))
        rec["noise_ratio"] = float(np.max(np.abs(g - x))) / ce if ce > 0 else None
    PARITY_LOG.append(rec)
    assert e <= tol, f"{what}: relative error {e:.3e} > {tol:.1e} (rms floor {floor:.2e})"
    return e


# ------------------------------------------------------------ RoPE

def rope_pair_norm(x, kind, hd, n_dims):
    """Per element: the norm of its rotation pair (llama 2j/2j+1, qwen j/j+hd/2,
    M-RoPE j/j+n/2 within the first n dims; unrotated dims: the element)."""
    x = np.asarray(x, np.float64)
    heads = x.reshape(-1, hd)
    mate = np.arange(hd)
    if kind == 0:
        mate = mate ^ 1
    elif kind == 1:
        mate = (mate + hd // 2) % hd
    else:
        half = n_dims // 2
        m = np.arange(n_dims)
        mate[:n_dims] = np.where(m < half, m + half, m - half)
    return np.sqrt(heads * heads + heads[:, mate] ** 2).reshape(x.shape)


def rope_err(gpu, ref, kind, hd, n_dims):
    """max |gpu - ref| / max(|pair|, 1e-3 * rms(ref)): the error of rotated q
    measured against the norm of each element's rotation pair, which a
    rotation keeps (a few-ulp sin/cos difference moves both outputs by a few
    ulps of it; the output element alone can be a cancellation)."""
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    den = np.maximum(rope_pair_norm(ref, kind, hd, n_dims), 1e-3 * rms)
    return float(np.max(np.abs(np.asarray(gpu, np.float64) - ref) / den))


# ------------------------------------------------- float64 evaluations
#
# The same attention and recurrence as the engine (engine.c:1074-1096, 533-563,
# 935-960; matvec.c:975-1021), evaluated in float64 from the same input bits.
# They are not the parity target (the fp32 oracle is); they measure how far the
# fp32 oracle itself sits from the exact value, which sets noise_floor.

def _heads_of(g, H, KV):
    return [h for h in range(H) if h * KV // H == g]


def exact_decode(q, k, v, pos, n_heads, n_kv, hd, kv_dim, gate=None) -> np.ndarray:
    kf = f16_to_f32(np.asarray(k, np.uint16).ravel()[: (pos + 1) * kv_dim]).astype(np.float64).reshape(-1, kv_dim)
    vf = f16_to_f32(np.asarray(v, np.uint16).ravel()[: (pos + 1) * kv_dim]).astype(np.float64).reshape(-1, kv_dim)
    q64 = np.asarray(q, np.float64).reshape(n_heads, hd)
    out = np.empty((n_heads, hd))
    for g in range(n_kv):
        hs = _heads_of(g, n_heads, n_kv)
        if not hs:
            continue
        s = (q64[hs] @ kf[:, g * hd:(g + 1) * hd].T) / np.sqrt(hd)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[hs] = p @ vf[:, g * hd:(g + 1) * hd]
    out = out.ravel()
    if gate is not None:
        out = out / (1.0 + np.exp(-np.asarray(gate, np.float64).ravel()))
    return out


def exact_prefill(q, k, v, pos_start, B, n_heads, n_kv, hd, kv_dim, q_stride, gate=None,
                  rows: Optional[slice] = None) -> np.ndarray:
    """float64 causal prefill, [B, q_stride] (columns past n_heads*hd are 0)."""
    n = pos_start + B
    kf = f16_to_f32(np.asarray(k, np.uint16).ravel()[: n * kv_dim]).astype(np.float64).reshape(n, kv_dim)
    vf = f16_to_f32(np.asarray(v, np.uint16).ravel()[: n * kv_dim]).astype(np.float64).reshape(n, kv_dim)
    q64 = np.asarray(q, np.float64).reshape(B, q_stride)
    out = np.zeros((B, q_stride))
    pos = pos_start + np.arange(B)
    for h in range(n_heads):
        g = h * n_kv // n_heads
        Kg, Vg = kf[:, g * hd:(g + 1) * hd], vf[:, g * hd:(g + 1) * hd]
        for r0 in range(0, B, 512):
            r1 = min(B, r0 + 512)
            s = (q64[r0:r1, h * hd:(h + 1) * hd] @ Kg.T) / np.sqrt(hd)
            s[np.arange(n)[None, :] > pos[r0:r1, None]] = -np.inf
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            out[r0:r1, h * hd:(h + 1) * hd] = p @ Vg
    if gate is not None:
        g64 = np.asarray(gate, np.float64).reshape(B, q_stride)
        out[:, : n_heads * hd] /= 1.0 + np.exp(-g64[:, : n_heads * hd])
    return out


def exact_gdn(fx: dict, cfg, n_seqs: int, T: int, epilogue: bool) -> tuple:
    """float64 form of gdn_run: (final state, outputs)."""
    D, NK, NV = cfg.head_dim, cfg.num_k_heads, cfg.n_v_heads
    S_all = np.asarray(fx["S"], np.float64).reshape(n_seqs, NV, D, D).copy()
    q = np.asarray(fx["q"], np.float64).reshape(n_seqs, T, NK, D)
    k = np.asarray(fx["k"], np.float64).reshape(n_seqs, T, NK, D)
    v = np.asarray(fx["v"], np.float64).reshape(n_seqs, T, NV, D)
    z = np.asarray(fx["z"], np.float64).reshape(n_seqs, T, NV, D)
    gate = np.asarray(fx["gate"], np.float64).reshape(n_seqs, T, NV)
    beta = np.asarray(fx["beta"], np.float64).reshape(n_seqs, T, NV)
    w = np.asarray(fx["norm_w"], np.float64)
    kh = np.arange(NV) % NK
    out = np.empty((n_seqs, T, NV, D))
    scale = 1.0 / np.sqrt(D)
    for s in range(n_seqs):
        S = S_all[s]                                   # [NV, D(v row j), D(k index i)]
        for t in range(T):
            kt, qt = k[s, t, kh], q[s, t, kh]           # [NV, D]
            S *= np.exp(gate[s, t])[:, None, None]
            dot = np.einsum("hji,hi->hj", S, kt)
            delta = (v[s, t] - dot) * beta[s, t][:, None]
            S += delta[:, :, None] * kt[:, None, :]
            o = np.einsum("hji,hi->hj", S, qt) * scale
            if epilogue:
                zz = z[s, t]
                inv = 1.0 / np.sqrt(np.mean(o * o, axis=1, keepdims=True) + cfg.eps)
                o = o * w[None, :] * inv * (zz / (1.0 + np.exp(-zz)))
            out[s, t] = o
    return S_all.ravel(), out.ravel()
