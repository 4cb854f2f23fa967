"""Regenerates the golden fixtures under tests/golden/.

  reference_kat.json  known answers transcribed from the reference's own unit
                      tests (tests/test_matvec.c): f16 conversion 32-55,
                      rope_inplace 213-228, softmax 231-239.
  golden_ref.npz      outputs of oracle/_ref/libyattn_ref.so -- the reference's
                      matvec.c / platform.c compiled unmodified under the
                      restated engine.c loops -- on small seeded cases, so the
                      port can be pinned on a machine without the reference tree.
  golden_glue.npz     the same for the rows around the attention path (RoPE +
                      KV store, GDN layer inputs, Q4_K / fp16 matmul, the
                      session KV file), plus the reference's own Q4_K decode
                      golden vector (tests/ref_data.h K4_RAW / K4_REF, checked
                      by its test_matvec.c:57-69 to 1e-6), parsed from that file.

Run from the repo root (needs the reference tree to build oracle/_ref):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

import oracle  # noqa: E402


def kat() -> dict:
    s = math.exp(1) + math.exp(2) + math.exp(3)
    return {
        "source": "reference tests/test_matvec.c",
        "f16_to_f32": [  # test_matvec.c:34-44 (hex input, expected value, tolerance)
            ["0x0000", 0.0, 1e-9], ["0x8000", -0.0, 1e-9], ["0x3c00", 1.0, 1e-9], ["0xbc00", -1.0, 1e-9],
            ["0x0001", 5.960464477539063e-8, 1e-12], ["0x8001", -5.960464477539063e-8, 1e-12],
            ["0x03f7", 6.049871444702148e-5, 1e-12], ["0x83f7", -6.049871444702148e-5, 1e-12],
            ["0x0400", 6.103515625e-5, 1e-12], ["0x7c00", "inf", 0], ["0xfc00", "-inf", 0],
        ],
        "f16_round_trip": ["0x0000", "0x3c00", "0xbc00", "0x0400", "0x7bff", "0x03ff", "0x8003", "0x3555",
                           "0xc555", "0x03f7"],  # test_matvec.c:46-54
        "rope_inplace": [  # test_matvec.c:213-228: (v, d, pos, theta, expected prefix, tol)
            [[1.0, 0.0, 0.0, 1.0], 4, 0, 10000.0, [1.0, 0.0, 0.0, 1.0], 1e-6],
            [[1.0, 0.0, 0.0, 1.0], 4, 1, 10000.0, [math.cos(1.0), math.sin(1.0)], 1e-5],
        ],
        "softmax": [  # test_matvec.c:231-239
            [[1.0, 2.0, 3.0], [math.exp(1) / s, math.exp(2) / s, math.exp(3) / s], 1e-6],
        ],
    }


def golden(lib) -> dict:
    rng = np.random.default_rng(20261201)
    g = {}
    # helpers
    bits = rng.integers(0, 2**32, 40000, dtype=np.uint64).astype(np.uint32)
    f = bits.view(np.float32)
    g["f32_bits"] = bits
    g["f32_to_f16"] = oracle.f32_to_f16(f, lib=lib)
    h = np.arange(65536, dtype=np.uint16)
    g["f16_to_f32_all"] = oracle.f16_to_f32(h, lib=lib)
    x = rng.standard_normal(1000).astype(np.float32) * 4
    sm = x.copy()
    lib.orc_softmax(sm, sm.size)
    g["softmax_in"], g["softmax_out"] = x, sm
    for name in ("rope_inplace", "rope_inplace_qwen"):
        v = rng.standard_normal(128).astype(np.float32)
        w = v.copy()
        getattr(lib, "orc_" + name)(w, 128, 777, 1e6)
        g[name + "_in"], g[name + "_out"] = v, w
    v = rng.standard_normal(256).astype(np.float32)
    w = v.copy()
    lib.orc_rope_inplace_mrope(w, 256, 64, 1234, 1e7)
    g["rope_mrope_in"], g["rope_mrope_out"] = v, w
    v = rng.standard_normal(128).astype(np.float32)
    w = v.copy()
    lib.orc_l2norm_inplace(w, 128, 1e-6)
    g["l2norm_in"], g["l2norm_out"] = v, w
    # decode (Qwen2.5 shape, short context), prefill (Qwen3 shape, short), gated (hd 256)
    for tag, (H, KV, hd, T) in {"dec": (14, 2, 64, 97), "gdec": (16, 2, 256, 33)}.items():
        kd = KV * hd
        q = rng.standard_normal(H * hd).astype(np.float32)
        k = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32), lib=lib)
        vv = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32), lib=lib)
        gate = rng.standard_normal(H * hd).astype(np.float32) if tag == "gdec" else None
        out = oracle.attn_decode(q, k, vv, T - 1, H, KV, hd, kd, gate=gate, lib=lib)
        g[tag + "_q"], g[tag + "_k"], g[tag + "_v"], g[tag + "_out"] = q, k, vv, out
        g[tag + "_geom"] = np.array([H, KV, hd, T], dtype=np.int64)
        if gate is not None:
            g[tag + "_gate"] = gate
    H, KV, hd, S, P0 = 16, 8, 128, 40, 9
    kd = KV * hd
    q = rng.standard_normal((S, H * hd)).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal((P0 + S) * kd).astype(np.float32), lib=lib)
    vv = oracle.f32_to_f16(rng.standard_normal((P0 + S) * kd).astype(np.float32), lib=lib)
    out = oracle.attn_prefill(q, k, vv, P0, S, H, KV, hd, kd, H * hd, lib=lib)
    g["pre_q"], g["pre_k"], g["pre_v"], g["pre_out"] = q, k, vv, out
    g["pre_geom"] = np.array([H, KV, hd, S, P0], dtype=np.int64)
    # GDN: 4 tokens, 4 k-heads, 8 v-heads, 32/32, with the rmsnorm_gated epilogue
    T, NK, NV, D = 4, 4, 8, 32
    S0 = (rng.standard_normal(NV * D * D) * 0.1).astype(np.float32)
    qg = rng.standard_normal((T, NK * D)).astype(np.float32)
    kg = rng.standard_normal((T, NK * D)).astype(np.float32)
    for t in range(T):
        for hh in range(NK):
            lib.orc_l2norm_inplace(qg[t, hh * D:(hh + 1) * D], D, 1e-6)
            lib.orc_l2norm_inplace(kg[t, hh * D:(hh + 1) * D], D, 1e-6)
    vg = rng.standard_normal((T, NV * D)).astype(np.float32)
    gt = (-np.log1p(np.exp(rng.standard_normal((T, NV))))).astype(np.float32)
    bt = (1 / (1 + np.exp(-rng.standard_normal((T, NV))))).astype(np.float32)
    z = rng.standard_normal((T, NV * D)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    S = S0.copy()
    og = np.zeros((T, NV * D), dtype=np.float32)
    lib.orc_gdn_prefill(S, og.ravel(), np.ascontiguousarray(qg.ravel()), np.ascontiguousarray(kg.ravel()),
                        np.ascontiguousarray(vg.ravel()), np.ascontiguousarray(gt.ravel()),
                        np.ascontiguousarray(bt.ravel()), T, NK, D, NV, D, w.ctypes.data, z.ctypes.data, 1e-6)
    for key, val in dict(S0=S0, q=qg, k=kg, v=vg, gate=gt, beta=bt, z=z, w=w, S1=S, out=og).items():
        g["gdn_" + key] = val
    g["gdn_geom"] = np.array([T, NK, NV, D], dtype=np.int64)
    return g


def ref_q4k_golden(ref_tree: Path) -> dict:
    """K4_RAW (two 144-byte Q4_K blocks) and K4_REF (their 512 decoded values) from the reference's
    tests/ref_data.h, parsed from the C initialisers."""
    import re

    text = (ref_tree / "tests" / "ref_data.h").read_text()

    def array(name):
        m = re.search(r"%s\[\]\s*=\s*\{(.*?)\};" % name, text, re.S)
        return [t.strip() for t in m.group(1).replace("\n", " ").split(",") if t.strip()]

    raw = np.array([int(t, 16) for t in array("K4_RAW")], dtype=np.uint8)
    ref = np.array([float(t.rstrip("fF")) for t in array("K4_REF")], dtype=np.float32)
    assert raw.size == 288 and ref.size == 512, (raw.size, ref.size)
    return {"q4k_raw": raw, "q4k_ref": ref}


def glue(lib) -> dict:
    rng = np.random.default_rng(20261202)
    g = {}
    # RoPE + KV store, one token of each kind (engine.c:1052-1072, 921-934)
    for kind, (H, KV, hd, nd, theta, pos) in {0: (8, 2, 128, 128, 5e5, 4095), 1: (4, 2, 64, 64, 1e6, 37),
                                              2: (4, 2, 256, 64, 1e7, 70000)}.items():
        kd = KV * hd
        q = rng.standard_normal(H * hd).astype(np.float32)
        k = rng.standard_normal(kd).astype(np.float32)
        v = rng.standard_normal(kd).astype(np.float32)
        qo, ko = q.copy(), k.copy()
        kc = np.zeros((pos + 1) * kd, np.uint16)
        vc = np.zeros((pos + 1) * kd, np.uint16)
        lib.orc_rope_store(qo, ko, v, kc, vc, H, KV, hd, kd, kind, nd, pos, theta)
        tag = f"rope{kind}_"
        g[tag + "in"] = np.concatenate([q, k, v])
        g[tag + "q"], g[tag + "krow"], g[tag + "vrow"] = qo, kc[pos * kd:], vc[pos * kd:]
        g[tag + "geom"] = np.array([H, KV, hd, nd, pos], dtype=np.int64)
        g[tag + "theta"] = np.array([theta], dtype=np.float32)
    # GDN layer inputs, 2 sequences x 5 tokens (engine.c:785-821)
    n_seqs, T, nk, hk, nv, hv, kw = 2, 5, 2, 32, 4, 32, 4
    cc = 2 * nk * hk + nv * hv
    case = dict(qkv=rng.standard_normal((n_seqs, T, cc)).astype(np.float32),
                state=rng.standard_normal((n_seqs, kw, cc)).astype(np.float32),
                w=(0.5 * rng.standard_normal((cc, kw))).astype(np.float32),
                alpha=rng.standard_normal((n_seqs, T, nv)).astype(np.float32),
                beta_in=rng.standard_normal((n_seqs, T, nv)).astype(np.float32),
                dt=rng.standard_normal(nv).astype(np.float32),
                a=-np.abs(rng.standard_normal(nv)).astype(np.float32))
    q = np.zeros((n_seqs, T, nk * hk), np.float32)
    k = np.zeros_like(q)
    v = np.zeros((n_seqs, T, nv * hv), np.float32)
    gate = np.zeros((n_seqs, T, nv), np.float32)
    beta = np.zeros_like(gate)
    st = case["state"].copy()
    lib.orc_gdn_inputs(case["qkv"], st, case["w"], case["alpha"], case["beta_in"], case["dt"], case["a"], q, k, v,
                       gate, beta, n_seqs, T, cc, kw, nk, hk, nv, hv, 1e-6)
    for key, val in case.items():
        g["gdni_" + key] = val
    for key, val in dict(q=q, k=k, v=v, gate=gate, beta=beta, state_out=st).items():
        g["gdni_out_" + key] = val
    g["gdni_geom"] = np.array([n_seqs, T, nk, hk, nv, hv, kw], dtype=np.int64)
    # linear layers: fp32 Q4_K dequant-dot and the engine's fp16 matmul, 2 tokens
    out, inn, B = 24, 512, 2
    nb = inn // 256
    w4 = rng.integers(0, 256, (out, nb, 144), dtype=np.uint8)
    w4[:, :, 0:2] = (rng.uniform(0.5, 2, (out, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(out, nb, 2)
    w4[:, :, 2:4] = (rng.uniform(0.5, 2, (out, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(out, nb, 2)
    w4 = np.ascontiguousarray(w4.reshape(-1))
    w16 = (0.02 * rng.standard_normal((out, inn))).astype(np.float16).view(np.uint16).reshape(-1)
    x = rng.standard_normal((B, inn)).astype(np.float32)
    y4 = np.zeros((B, out), np.float32)
    y16 = np.zeros((B, out), np.float32)
    lib.orc_gemv_q4k(y4, w4, x, out, inn, B)
    lib.orc_gemv_f16(y16, np.ascontiguousarray(w16), x, out, inn, B)
    g.update(lin_w4=w4, lin_w16=w16, lin_x=x, lin_y4=y4, lin_y16=y16,
             lin_geom=np.array([out, inn, B], dtype=np.int64))
    # session KV file bytes (cache.c:174-195): 2 blocks, kv_dim 16, max_seq 8, pos 5
    nb_, kd_, ms_, pos_ = 2, 16, 8, 5
    blob = rng.integers(0, 1 << 16, (2 * nb_ + 1) * ms_ * kd_, dtype=np.uint16)
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "s.kv"
        assert lib.orc_sess_kv_save(blob, nb_, kd_, ms_, pos_, str(path).encode()) == 0
        g["sess_file"] = np.frombuffer(path.read_bytes(), dtype=np.uint8).copy()
    g["sess_blob"] = blob
    g["sess_geom"] = np.array([nb_, kd_, ms_, pos_], dtype=np.int64)
    return g


def main() -> None:
    (HERE / "reference_kat.json").write_text(json.dumps(kat(), indent=1) + "\n")
    lib = oracle.load("ref")
    np.savez_compressed(HERE / "golden_ref.npz", **golden(lib))
    ref_tree = Path(oracle.REF_TREE)
    np.savez_compressed(HERE / "golden_glue.npz", **glue(lib), **ref_q4k_golden(ref_tree))
    print("wrote", HERE / "reference_kat.json", HERE / "golden_ref.npz", HERE / "golden_glue.npz")


if __name__ == "__main__":
    main()
