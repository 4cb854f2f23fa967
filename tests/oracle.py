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
# the reference source tree (present where the oracle's reference build is made; absent on GPU boxes)
REF_TREE = Path(os.environ.get("YATTN_REF_TREE", "/root/reference"))

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

REL_TOL = 2e-3


def rel_err(gpu: np.ndarray, cpu: np.ndarray) -> float:
    """max |gpu - cpu| / max(|cpu|, rms(cpu)): the relative error the parity
    bar (2e-3) is stated in.  The rms floor keeps near-zero outputs (where the
    CPU's own fp32 summation order already differs from any other order by
    more than 2e-3 relative) from dominating."""
    gpu = np.asarray(gpu, dtype=np.float64)
    cpu = np.asarray(cpu, dtype=np.float64)
    rms = float(np.sqrt(np.mean(cpu * cpu))) if cpu.size else 0.0
    den = np.maximum(np.abs(cpu), rms if rms > 0 else 1e-30)
    return float(np.max(np.abs(gpu - cpu) / den)) if cpu.size else 0.0


def assert_close(gpu: np.ndarray, cpu: np.ndarray, tol: float = REL_TOL, what: str = "") -> float:
    assert np.all(np.isfinite(gpu)), f"{what}: non-finite GPU output"
    e = rel_err(gpu, cpu)
    assert e <= tol, f"{what}: relative error {e:.3e} > {tol:.1e}"
    return e
