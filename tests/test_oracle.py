"""Pins the CPU oracle: reference known answers, reference-build golden vectors,
port == reference bit for bit, and the deterministic input generator."""
import ctypes as C
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLD / "golden_ref.npz"))


def test_reference_known_answers(orc):
    kat = json.loads((GOLD / "reference_kat.json").read_text())
    for hx, want, tol in kat["f16_to_f32"]:
        got = orc.orc_f16_to_f32(int(hx, 16))
        if isinstance(want, str):
            assert math.isinf(got) and (got < 0) == want.startswith("-"), hx
        else:
            assert abs(got - want) <= tol, (hx, got, want)   # CHECK_NEAR semantics
    for hx in kat["f16_round_trip"]:
        h = int(hx, 16)
        assert orc.orc_f32_to_f16(orc.orc_f16_to_f32(h)) == h, hx
    for v, d, pos, theta, want, tol in kat["rope_inplace"]:
        x = np.array(v, dtype=np.float32)
        orc.orc_rope_inplace(x, d, pos, theta)
        assert np.all(np.abs(x[:len(want)] - np.array(want)) <= tol)
    for v, want, tol in kat["softmax"]:
        x = np.array(v, dtype=np.float32)
        orc.orc_softmax(x, x.size)
        assert np.all(np.abs(x - np.array(want)) <= tol)
        assert abs(float(x.sum()) - 1.0) <= tol


def test_port_matches_reference_golden_helpers(orc, gold):
    f = gold["f32_bits"].view(np.float32)
    assert np.array_equal(oracle.f32_to_f16(f, lib=orc), gold["f32_to_f16"])
    h = np.arange(65536, dtype=np.uint16)
    got = oracle.f16_to_f32(h, lib=orc)
    want = gold["f16_to_f32_all"]
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    x = gold["softmax_in"].copy()
    orc.orc_softmax(x, x.size)
    assert np.array_equal(x, gold["softmax_out"])
    for name in ("rope_inplace", "rope_inplace_qwen"):
        x = gold[name + "_in"].copy()
        getattr(orc, "orc_" + name)(x, 128, 777, 1e6)
        assert np.array_equal(x, gold[name + "_out"]), name
    x = gold["rope_mrope_in"].copy()
    orc.orc_rope_inplace_mrope(x, 256, 64, 1234, 1e7)
    assert np.array_equal(x, gold["rope_mrope_out"])
    x = gold["l2norm_in"].copy()
    orc.orc_l2norm_inplace(x, 128, 1e-6)
    assert np.array_equal(x, gold["l2norm_out"])


def test_port_matches_reference_golden_attention(orc, gold):
    for tag in ("dec", "gdec"):
        H, KV, hd, T = (int(v) for v in gold[tag + "_geom"])
        gate = gold.get(tag + "_gate")
        out = oracle.attn_decode(gold[tag + "_q"], gold[tag + "_k"], gold[tag + "_v"], T - 1, H, KV, hd, KV * hd,
                                 gate=gate, lib=orc)
        assert np.array_equal(out, gold[tag + "_out"]), tag
    H, KV, hd, S, P0 = (int(v) for v in gold["pre_geom"])
    out = oracle.attn_prefill(gold["pre_q"], gold["pre_k"], gold["pre_v"], P0, S, H, KV, hd, KV * hd, H * hd,
                              lib=orc)
    assert np.array_equal(out, gold["pre_out"])


def test_port_matches_reference_golden_gdn(orc, gold):
    T, NK, NV, D = (int(v) for v in gold["gdn_geom"])
    S = gold["gdn_S0"].copy()
    out = np.zeros((T, NV * D), dtype=np.float32)
    w, z = gold["gdn_w"], gold["gdn_z"]
    orc.orc_gdn_prefill(S, out.ravel(), gold["gdn_q"].ravel(), gold["gdn_k"].ravel(), gold["gdn_v"].ravel(),
                        gold["gdn_gate"].ravel(), gold["gdn_beta"].ravel(), T, NK, D, NV, D, w.ctypes.data,
                        z.ctypes.data, 1e-6)
    assert np.array_equal(S, gold["gdn_S1"])
    assert np.array_equal(out, gold["gdn_out"])


def test_port_equals_reference_build_live(orc, orc_ref):
    """Where the reference tree is present, compare the two builds directly."""
    assert orc.orc_build_kind() == 0 and orc_ref.orc_build_kind() == 1
    hi = np.arange(65536, dtype=np.uint64) << np.uint64(16)
    lows = np.array([0, 1, 0x0FFF, 0x1000, 0x1001, 0x1FFF, 0x2000, 0x7FFF, 0x8000, 0xFFFF, 0x2FFF, 0x3000],
                    dtype=np.uint64)
    f = (hi[:, None] | lows[None, :]).ravel().astype(np.uint32).view(np.float32)
    assert np.array_equal(oracle.f32_to_f16(f, lib=orc), oracle.f32_to_f16(f, lib=orc_ref))
    rng = np.random.default_rng(5)
    H, KV, hd, T = 32, 8, 128, 300
    kd = KV * hd
    q = rng.standard_normal(H * hd).astype(np.float32)
    k = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    v = oracle.f32_to_f16(rng.standard_normal(T * kd).astype(np.float32))
    a = oracle.attn_decode(q, k, v, T - 1, H, KV, hd, kd, lib=orc)
    b = oracle.attn_decode(q, k, v, T - 1, H, KV, hd, kd, lib=orc_ref)
    assert np.array_equal(a, b)
    # GDN, full qwen3.5 head geometry, a few steps
    NK, NV, D, steps = 16, 32, 128, 3
    Sa = (rng.standard_normal(NV * D * D) * 0.1).astype(np.float32)
    Sb = Sa.copy()
    for _ in range(steps):
        qg = rng.standard_normal(NK * D).astype(np.float32)
        kg = rng.standard_normal(NK * D).astype(np.float32)
        for hh in range(NK):
            orc.orc_l2norm_inplace(qg[hh * D:(hh + 1) * D], D, 1e-6)
            orc.orc_l2norm_inplace(kg[hh * D:(hh + 1) * D], D, 1e-6)
        vg = rng.standard_normal(NV * D).astype(np.float32)
        gt = rng.uniform(-3, 0, NV).astype(np.float32)
        bt = rng.uniform(0, 1, NV).astype(np.float32)
        oa = np.zeros(NV * D, np.float32)
        ob = np.zeros(NV * D, np.float32)
        orc.orc_gdn_step(Sa, oa, qg, kg, vg, gt, bt, NK, D, NV, D, None, None, 1e-6)
        orc_ref.orc_gdn_step(Sb, ob, qg, kg, vg, gt, bt, NK, D, NV, D, None, None, 1e-6)
        assert np.array_equal(oa, ob) and np.array_equal(Sa, Sb)


def test_rope_store_port_equals_reference_build(orc, orc_ref):
    """orc_rope_store (engine.c:1052-1072, 921-934) on both builds: same q, k and cache bits, every kind."""
    rng = np.random.default_rng(11)
    for kind, H, KV, hd, nd, theta in ((0, 32, 8, 128, 128, 5e5), (1, 14, 2, 64, 64, 1e6), (2, 16, 2, 256, 64, 1e7)):
        kd = KV * hd
        for pos in (0, 3, 4095, 131071):
            q = rng.standard_normal(H * hd).astype(np.float32)
            k = rng.standard_normal(kd).astype(np.float32)
            v = rng.standard_normal(kd).astype(np.float32)
            outs = []
            for lib in (orc, orc_ref):
                qq, kk = q.copy(), k.copy()
                kc = np.zeros((pos + 1) * kd, np.uint16)
                vc = np.zeros((pos + 1) * kd, np.uint16)
                lib.orc_rope_store(qq, kk, v, kc, vc, H, KV, hd, kd, kind, nd, pos, theta)
                outs.append((qq, kk, kc[pos * kd:], vc[pos * kd:]))
            for a, b in zip(*outs):
                assert np.array_equal(a, b), (kind, pos)
            if kind == 2:   # dims past n_dims pass through unrotated
                assert np.array_equal(outs[0][1].reshape(KV, hd)[:, nd:], k.reshape(KV, hd)[:, nd:])


def _gdn_inputs_case(rng, n_seqs, T, nk, hk, nv, hv, kw):
    C_ = 2 * nk * hk + nv * hv
    return dict(qkv=rng.standard_normal((n_seqs, T, C_)).astype(np.float32),
                state=rng.standard_normal((n_seqs, kw, C_)).astype(np.float32),
                w=(0.5 * rng.standard_normal((C_, kw))).astype(np.float32),
                alpha=rng.standard_normal((n_seqs, T, nv)).astype(np.float32),
                beta_in=rng.standard_normal((n_seqs, T, nv)).astype(np.float32),
                dt=rng.standard_normal(nv).astype(np.float32),
                a=-np.abs(rng.standard_normal(nv)).astype(np.float32))


def run_gdn_inputs(lib, c, n_seqs, T, nk, hk, nv, hv, kw, eps=1e-6):
    q = np.zeros((n_seqs, T, nk * hk), np.float32)
    k = np.zeros_like(q)
    v = np.zeros((n_seqs, T, nv * hv), np.float32)
    gate = np.zeros((n_seqs, T, nv), np.float32)
    beta = np.zeros_like(gate)
    st = c["state"].copy()
    lib.orc_gdn_inputs(c["qkv"], st, c["w"], c["alpha"], c["beta_in"], c["dt"], c["a"], q, k, v, gate, beta,
                       n_seqs, T, 2 * nk * hk + nv * hv, kw, nk, hk, nv, hv, eps)
    return q, k, v, gate, beta, st


def test_gdn_inputs_port_equals_reference_build(orc, orc_ref):
    """orc_gdn_inputs (engine.c:785-821 per token) with the port's conv1d_update / l2norm against the
    reference's matvec.c: same bits, including the delay line left behind."""
    rng = np.random.default_rng(21)
    for n_seqs, T, nk, hk, nv, hv, kw in ((2, 7, 2, 64, 4, 64, 4), (1, 3, 2, 128, 2, 128, 4), (1, 5, 1, 64, 2, 64, 2)):
        c = _gdn_inputs_case(rng, n_seqs, T, nk, hk, nv, hv, kw)
        a = run_gdn_inputs(orc, c, n_seqs, T, nk, hk, nv, hv, kw)
        b = run_gdn_inputs(orc_ref, c, n_seqs, T, nk, hk, nv, hv, kw)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)
        q = a[0].reshape(n_seqs * T * nk, hk)
        assert np.allclose(np.linalg.norm(q, axis=1), 1.0, atol=1e-5)   # l2-normalised heads


def test_sess_kv_port_equals_reference_build(orc, orc_ref, tmp_path):
    """The session KV file (cache.c:174-247): the restated writer makes the reference's bytes, and both
    loaders read either file back into the same regions, refusing a different geometry."""
    rng = np.random.default_rng(3)
    nb, kd, max_seq = 3, 64, 40
    blob = rng.integers(0, 1 << 16, (2 * nb + 1) * max_seq * kd, dtype=np.uint16)
    for pos in (0, 1, 17, max_seq):
        fa, fb = tmp_path / f"a{pos}.kv", tmp_path / f"b{pos}.kv"
        assert orc.orc_sess_kv_save(blob, nb, kd, max_seq, pos, str(fa).encode()) == 0
        assert orc_ref.orc_sess_kv_save(blob, nb, kd, max_seq, pos, str(fb).encode()) == 0
        assert fa.read_bytes() == fb.read_bytes()
        assert len(fa.read_bytes()) == 24 + 2 * nb * pos * kd * 2
        for lib in (orc, orc_ref):
            back = np.zeros_like(blob)
            p = C.c_uint32(99)
            assert lib.orc_sess_kv_load(back, nb, kd, max_seq, str(fa).encode(), C.byref(p)) == 0
            assert p.value == pos
            want = np.zeros_like(blob).reshape(2 * nb + 1, max_seq, kd)
            src = blob.reshape(2 * nb + 1, max_seq, kd)
            want[1:, :pos] = src[1:, :pos]
            assert np.array_equal(back.reshape(want.shape), want)
            assert lib.orc_sess_kv_load(back, nb + 1, kd, max_seq, str(fa).encode(), C.byref(p)) == -1
            assert lib.orc_sess_kv_load(back, nb, kd, max_seq + 1, str(fa).encode(), C.byref(p)) == -1


def _q4k_decode_numpy(blk):
    """An independent numpy decoder of one 144-byte Q4_K block (the published GGML layout)."""
    d = float(np.frombuffer(blk[0:2].tobytes(), np.float16)[0])
    dmin = float(np.frombuffer(blk[2:4].tobytes(), np.float16)[0])
    q = blk[4:16].astype(np.int64)
    out = np.zeros(256, np.float64)
    for g in range(8):
        if g < 4:
            sc, mn = q[g] & 63, q[g + 4] & 63
        else:
            sc = (q[g + 4] & 0xF) | ((q[g - 4] >> 6) << 4)
            mn = (q[g + 4] >> 4) | ((q[g] >> 6) << 4)
        nib = blk[16 + (g // 2) * 32: 16 + (g // 2) * 32 + 32].astype(np.int64)
        nib = (nib >> 4) if g & 1 else (nib & 0xF)
        out[g * 32:(g + 1) * 32] = d * sc * nib - dmin * mn
    return out


def test_q4k_and_f16_matmul_port_equals_reference(orc, orc_ref):
    """q4k_block against an independent decoder; the fp32 Q4_K dot and the engine's fp16 matmul bit for bit
    between the port and the reference build."""
    rng = np.random.default_rng(9)
    out, in_, B = 37, 512, 2
    nb = in_ // 256
    w = rng.integers(0, 256, (out, nb, 144), dtype=np.uint8)
    w[:, :, 0:2] = (rng.uniform(0.5, 2, (out, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(out, nb, 2)
    w[:, :, 2:4] = (rng.uniform(0.5, 2, (out, nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(out, nb, 2)
    w = np.ascontiguousarray(w.reshape(-1))
    for lib in (orc, orc_ref):
        y = np.zeros(256, np.float32)
        lib.orc_q4k_block(y, np.ascontiguousarray(w[:144]))
        assert np.allclose(y, _q4k_decode_numpy(w[:144]), rtol=1e-6, atol=1e-9)
    x = rng.standard_normal((B, in_)).astype(np.float32)
    ya, yb = np.zeros((B, out), np.float32), np.zeros((B, out), np.float32)
    orc.orc_gemv_q4k(ya, w, x, out, in_, B)
    orc_ref.orc_gemv_q4k(yb, w, x, out, in_, B)
    assert np.array_equal(ya, yb)
    w16 = (0.02 * rng.standard_normal((out, in_))).astype(np.float16).view(np.uint16).reshape(-1)
    orc.orc_gemv_f16(ya, np.ascontiguousarray(w16), x, out, in_, B)
    orc_ref.orc_gemv_f16(yb, np.ascontiguousarray(w16), x, out, in_, B)
    assert np.array_equal(ya, yb)


@pytest.fixture(scope="module")
def glue():
    return dict(np.load(GOLD / "golden_glue.npz"))


def test_q4k_block_matches_reference_golden_vector(orc, glue):
    """The reference's own Q4_K decode golden (tests/ref_data.h, two blocks of a real model row; its
    test_matvec.c:57-69 checks q4k_block against it to 1e-6): the port and, where built, the reference build."""
    import oracle

    libs = [orc] + ([oracle.load("ref")] if oracle.has_ref() else [])
    for lib in libs:
        out = np.zeros(512, np.float32)
        for b in range(2):
            y = np.zeros(256, np.float32)
            lib.orc_q4k_block(y, np.ascontiguousarray(glue["q4k_raw"][b * 144:(b + 1) * 144]))
            out[b * 256:(b + 1) * 256] = y
        assert np.max(np.abs(out - glue["q4k_ref"])) <= 1e-6


def test_port_matches_reference_golden_glue(orc, glue):
    """The port reproduces the reference build's outputs bit for bit on the rows around the attention path:
    RoPE + KV store, GDN layer inputs, the Q4_K / fp16 matmuls and the session KV file."""
    for kind in (0, 1, 2):
        t = f"rope{kind}_"
        H, KV, hd, nd, pos = (int(x) for x in glue[t + "geom"])
        kd = KV * hd
        inp = glue[t + "in"]
        q, k, v = inp[:H * hd].copy(), inp[H * hd:H * hd + kd].copy(), inp[H * hd + kd:].copy()
        kc = np.zeros((pos + 1) * kd, np.uint16)
        vc = np.zeros((pos + 1) * kd, np.uint16)
        orc.orc_rope_store(q, k, v, kc, vc, H, KV, hd, kd, kind, nd, pos, float(glue[t + "theta"][0]))
        assert np.array_equal(q, glue[t + "q"]) and np.array_equal(kc[pos * kd:], glue[t + "krow"])
        assert np.array_equal(vc[pos * kd:], glue[t + "vrow"])
    n_seqs, T, nk, hk, nv, hv, kw = (int(x) for x in glue["gdni_geom"])
    cc = 2 * nk * hk + nv * hv
    outs = dict(q=np.zeros((n_seqs, T, nk * hk), np.float32), k=np.zeros((n_seqs, T, nk * hk), np.float32),
                v=np.zeros((n_seqs, T, nv * hv), np.float32), gate=np.zeros((n_seqs, T, nv), np.float32),
                beta=np.zeros((n_seqs, T, nv), np.float32))
    st = glue["gdni_state"].copy()
    orc.orc_gdn_inputs(glue["gdni_qkv"], st, glue["gdni_w"], glue["gdni_alpha"], glue["gdni_beta_in"],
                       glue["gdni_dt"], glue["gdni_a"], outs["q"], outs["k"], outs["v"], outs["gate"], outs["beta"],
                       n_seqs, T, cc, kw, nk, hk, nv, hv, 1e-6)
    for key, val in outs.items():
        assert np.array_equal(val, glue["gdni_out_" + key]), key
    assert np.array_equal(st, glue["gdni_out_state_out"])
    out, inn, B = (int(x) for x in glue["lin_geom"])
    y = np.zeros((B, out), np.float32)
    orc.orc_gemv_q4k(y, glue["lin_w4"], glue["lin_x"], out, inn, B)
    assert np.array_equal(y, glue["lin_y4"])
    orc.orc_gemv_f16(y, glue["lin_w16"], glue["lin_x"], out, inn, B)
    assert np.array_equal(y, glue["lin_y16"])


def test_port_session_file_matches_reference_golden(orc, glue, tmp_path):
    nb, kd, ms, pos = (int(x) for x in glue["sess_geom"])
    path = tmp_path / "s.kv"
    assert orc.orc_sess_kv_save(glue["sess_blob"], nb, kd, ms, pos, str(path).encode()) == 0
    assert path.read_bytes() == glue["sess_file"].tobytes()


def test_per_head_gdn_call_equals_all_heads_call(orc):
    """orc_gdn_step splits the reference call per head; same bits as one call."""
    rng = np.random.default_rng(9)
    NK, NV, D = 4, 8, 32
    S1 = (rng.standard_normal(NV * D * D) * 0.1).astype(np.float32)
    S2 = S1.copy()
    q = rng.standard_normal(NK * D).astype(np.float32)
    k = rng.standard_normal(NK * D).astype(np.float32)
    v = rng.standard_normal(NV * D).astype(np.float32)
    g = rng.uniform(-2, 0, NV).astype(np.float32)
    b = rng.uniform(0, 1, NV).astype(np.float32)
    o1 = np.zeros(NV * D, np.float32)
    o2 = np.zeros(NV * D, np.float32)
    orc.orc_gdn_state_update(S1, o1, q, k, v, g, b, NK, D, NV, D)
    orc.orc_gdn_step(S2, o2, q, k, v, g, b, NK, D, NV, D, None, None, 1e-6)
    assert np.array_equal(o1, o2) and np.array_equal(S1, S2)


def test_det_math_accuracy(orc):
    rng = np.random.default_rng(1)
    for x in rng.uniform(1e-7, 1, 2000):
        assert abs(orc.orc_det_log(x) - math.log(x)) < 4e-15
    for x in rng.uniform(-40, 40, 2000):
        assert abs(orc.orc_det_exp(x) / math.exp(x) - 1) < 4e-16
    s, c = C.c_double(), C.c_double()
    for x in rng.uniform(-3e5, 3e5, 2000):
        orc.orc_det_sincos(x, C.byref(s), C.byref(c))
        assert abs(s.value - math.sin(x)) < 1e-10 and abs(c.value - math.cos(x)) < 1e-10


def test_normal_stream_statistics(orc):
    x = np.empty(400000, dtype=np.float32)
    orc.orc_fill_normal(12345, 0, x.size, 1.0, x)
    assert abs(float(x.mean())) < 0.01
    assert abs(float(x.std()) - 1.0) < 0.01
    kurt = float(((x - x.mean()) ** 4).mean() / x.var() ** 2)
    assert abs(kurt - 3.0) < 0.05
    # draws are the reference's splitmix64 (yrng) sequence
    st = C.c_uint64(777)
    lib_yrng = orc.orc_yrng if hasattr(orc, "orc_yrng") else None
    if lib_yrng is not None:
        lib_yrng.restype = C.c_uint64
        lib_yrng.argtypes = [C.POINTER(C.c_uint64)]
        for kk in range(5):
            assert lib_yrng(C.byref(st)) == orc.orc_stream_draw(777, kk)


def test_fixture_rope_matches_reference_rope(orc, orc_ref):
    """The generator's double-precision rotation agrees with the engine's float
    rope_inplace_qwen (matvec.c:907-921) to float accuracy."""
    H, hd, pos = 2, 128, 511
    rows = oracle.gen_rows(oracle.GEN_F32, 1, H, hd, 99, rope=False, lib=orc)[0]
    rot = oracle.gen_rows(oracle.GEN_F32, 1, H, hd, 99, rope=True, pos0=pos, theta=1e6, lib=orc)[0]
    ref = rows.copy()
    for h in range(H):
        orc_ref.orc_rope_inplace_qwen(ref[h * hd:(h + 1) * hd], hd, pos, 1e6)
    assert np.max(np.abs(rot - ref)) < 2e-4 * max(1.0, float(np.max(np.abs(ref))))


def test_config_seeds_and_ctx(orc):
    from yllm_b200.configs import CFG3, ctx_lengths, seed_of, splitmix_draw

    seed = seed_of(3, "ctx")
    for i in range(64):
        assert splitmix_draw(seed, i) == orc.orc_stream_draw(seed, i)
    lens = ctx_lengths(64, 1024, 8192, seed)
    assert lens == [orc.orc_ctx_len(seed, i, 1024, 8192) for i in range(64)]
    assert CFG3.ctx() == lens and min(lens) >= 1024 and max(lens) <= 8192
