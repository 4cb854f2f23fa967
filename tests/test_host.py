"""Host-side checks of the C ABI library that need no GPU."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "yllm_attn_sm100.h"


def declared_functions() -> list:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "defined")))


def test_library_exports_every_declared_symbol():
    from yllm_b200 import _lib

    names = declared_functions()
    assert "cuda_k_attn_decode" in names and "yattn_decode_run" in names
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for n in names:
        assert hasattr(_lib.lib, n)


def test_struct_layout_matches_header(tmp_path):
    from yllm_b200._lib import YattnDecodeItem, YattnDecodeWork

    src = tmp_path / "s.c"
    src.write_text('#include "yllm_attn_sm100.h"\n#include <stdio.h>\n#include <stddef.h>\n'
                   'int main(void){printf("%zu %zu %zu %zu\\n", sizeof(YattnDecodeItem), sizeof(YattnDecodeWork),'
                   ' offsetof(YattnDecodeItem,pos), offsetof(YattnDecodeWork,part_base));return 0;}\n')
    exe = tmp_path / "s"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    a, b, c, d = (int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split())
    assert a == C.sizeof(YattnDecodeItem) and b == C.sizeof(YattnDecodeWork)
    assert c == YattnDecodeItem.pos.offset and d == YattnDecodeWork.part_base.offset


def test_rope_item_layout_matches_header(tmp_path):
    from yllm_b200._lib import YattnRopeItem

    src = tmp_path / "r.c"
    src.write_text('#include "yllm_attn_sm100.h"\n#include <stdio.h>\n#include <stddef.h>\n'
                   'int main(void){printf("%zu %zu %zu\\n", sizeof(YattnRopeItem), offsetof(YattnRopeItem,vcache),'
                   ' offsetof(YattnRopeItem,pos));return 0;}\n')
    exe = tmp_path / "r"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    a, b, c = (int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split())
    assert a == C.sizeof(YattnRopeItem) and b == YattnRopeItem.vcache.offset and c == YattnRopeItem.pos.offset


def heads_per_cta(n_kv, hd):
    """The library's kv-head grouping: largest of 8/4/2/1 (4 at head_dim 256) dividing n_kv."""
    cap = 4 if hd >= 256 else 8
    hc = cap
    while hc > 1 and n_kv % hc:
        hc //= 2
    return hc


def _plan(pos, n_kv, hd=128, split=0, target=592):
    from yllm_b200._lib import YattnDecodeWork, lib

    pos = np.asarray(pos, dtype=np.uint32)
    cap = 200000
    work = (YattnDecodeWork * cap)()
    nw, npart, ng = C.c_uint32(), C.c_uint32(), C.c_uint32()
    err = C.create_string_buffer(256)
    rc = lib.yattn_decode_plan(pos.ctypes.data_as(C.POINTER(C.c_uint32)), pos.size, n_kv, hd, split, target,
                               work, cap, C.byref(nw), C.byref(npart), C.byref(ng), err, 256)
    assert rc == 0, err.value
    return [work[i] for i in range(nw.value)], npart.value, ng.value


@pytest.mark.parametrize("pos,n_kv,hd,split", [
    ([511], 2, 64, 0), ([0], 8, 128, 0), ([131071], 8, 128, 0), ([4095] * 32, 2, 256, 0),
    ([1023, 8191, 5000, 1, 77], 8, 128, 0), ([300, 301, 5], 4, 128, 64), ([700, 9], 6, 128, 128),
    ([1000], 8, 256, 0), ([2000, 5], 3, 64, 0),
])
def test_decode_plan_covers_every_key_once(pos, n_kv, hd, split):
    hc = heads_per_cta(n_kv, hd)
    work, n_parts, n_groups = _plan(pos, n_kv, hd, split)
    seen = {}
    parts, groups = [], set()
    for w in work:
        assert w.kv_head % hc == 0
        key = (w.item, w.kv_head)
        assert 0 <= w.t_begin < w.t_end <= pos[w.item] + 1
        seen.setdefault(key, []).append((w.t_begin, w.t_end, w.split, w.n_splits))
        if w.n_splits > 1:
            for h in range(hc):   # one partial slot per (kv head of the group, split)
                parts.append(w.part_base + h * w.n_splits + w.split)
            groups.add(w.group)
    for i, p in enumerate(pos):
        for kg in range(n_kv // hc):
            segs = sorted(seen[(i, kg * hc)])
            assert segs[0][0] == 0 and segs[-1][1] == p + 1
            for a, b in zip(segs, segs[1:]):
                assert a[1] == b[0]
            assert sorted(s[2] for s in segs) == list(range(len(segs)))
            assert all(s[3] == len(segs) for s in segs)
    assert sorted(parts) == list(range(n_parts)) and groups == set(range(n_groups))
    ctas = [w.cta for w in work]
    assert ctas == sorted(ctas)          # units grouped by the CTA that streams them
    if split:                            # uniform splits: one unit per CTA, longest first
        lens = [w.t_end - w.t_begin for w in work]
        assert lens == sorted(lens, reverse=True) and ctas == list(range(len(work)))


@pytest.mark.parametrize("target", [148, 37])
def test_balanced_plan_evens_out_ctas(target):
    """Automatic splits: units are grouped by CTA in increasing order, the plan
    fits one wave, no CTA carries more than ~10 % over an equal share of keys
    (each further unit charged 192 keys), no (item, head group) has more than
    32 splits, and split numbering matches the range order."""
    from yllm_b200.configs import CFG3 as c

    pos = [x - 1 for x in c.ctx()]
    hc = heads_per_cta(c.n_kv_heads, c.head_dim)
    work, _, _ = _plan(pos, c.n_kv_heads, c.head_dim, 0, target)
    ctas = [w.cta for w in work]
    assert ctas == sorted(ctas) and ctas[0] == 0 and set(ctas) == set(range(ctas[-1] + 1))
    load, units = {}, {}
    for w in work:
        load[w.cta] = load.get(w.cta, 0) + (w.t_end - w.t_begin)
        units[w.cta] = units.get(w.cta, 0) + 1
    total = sum(p + 1 for p in pos) * (c.n_kv_heads // hc)
    share = total / target
    charged = [load[k] + 192 * (units[k] - 1) for k in load]  # each further unit costs ~192 keys
    assert max(charged) <= 1.1 * share + 128
    assert len(load) <= target                               # one wave
    by_range = {}
    for w in work:
        by_range.setdefault((w.item, w.kv_head), []).append(w)
    for segs in by_range.values():
        assert len(segs) <= 32
        assert [w.split for w in segs] == list(range(len(segs)))
        assert all(w.n_splits == len(segs) for w in segs)
        assert all(w.t_end - w.t_begin >= 128 or len(segs) == 1 for w in segs)


@pytest.mark.parametrize("pooled", [False, True])
def test_balanced_plan_cta_numbers_dense(pooled):
    """Every CTA number 0..n-1 carries at least one unit (the run launches one
    CTA per unit, so a gap would leave units unrun), for ragged random batches."""
    from yllm_b200._lib import YattnDecodeWork, lib

    rng = np.random.default_rng(7)
    fn = lib.yattn_decode_plan_pooled if pooled else lib.yattn_decode_plan
    for trial in range(300):
        n = int(rng.integers(1, 40))
        pos = rng.integers(0, int(rng.choice([300, 5000, 40000])), size=n).astype(np.uint32)
        n_kv, hd = [(8, 128), (2, 256), (2, 64), (4, 128), (1, 128)][trial % 5]
        target = int(rng.choice([148, 37, 296]))
        cap = 200000
        work = (YattnDecodeWork * cap)()
        nw, npart, ng = C.c_uint32(), C.c_uint32(), C.c_uint32()
        err = C.create_string_buffer(256)
        rc = fn(pos.ctypes.data_as(C.POINTER(C.c_uint32)), n, n_kv, hd, 0, target, work, cap, C.byref(nw),
                C.byref(npart), C.byref(ng), err, 256)
        assert rc == 0, err.value
        ctas = [work[i].cta for i in range(nw.value)]
        assert ctas == sorted(ctas) and set(ctas) == set(range(ctas[-1] + 1)), (trial, n, n_kv, hd, target)
        assert ctas[-1] + 1 <= nw.value                      # one CTA per unit is launched
        if int(pos.astype(np.int64).sum()) >= 256 * target:   # enough work: one wave
            assert ctas[-1] + 1 <= target


def test_plan_rejects_bad_args():
    from yllm_b200._lib import YattnDecodeWork, lib

    err = C.create_string_buffer(256)
    nw, npart, ng = C.c_uint32(), C.c_uint32(), C.c_uint32()
    pos = (C.c_uint32 * 1)(10)
    work = (YattnDecodeWork * 1)()
    rc = lib.yattn_decode_plan(pos, 1, 0, 128, 0, 1, work, 1, C.byref(nw), C.byref(npart), C.byref(ng), err, 256)
    assert rc == -1 and b"bad arguments" in err.value
    rc = lib.yattn_decode_plan(pos, 1, 8, 96, 0, 1, work, 1, C.byref(nw), C.byref(npart), C.byref(ng), err, 256)
    assert rc == -1 and b"head_dim 96" in err.value
    pos = (C.c_uint32 * 1)(100000)
    rc = lib.yattn_decode_plan(pos, 1, 8, 128, 64, 1, work, 1, C.byref(nw), C.byref(npart), C.byref(ng), err, 256)
    assert rc == -1 and b"work_cap" in err.value and nw.value > 1


def test_error_paths_before_any_device_work():
    from yllm_b200._lib import YattnError, call, call_void, lib

    with pytest.raises(YattnError, match="head_dim 96"):
        call("yattn_attn_decode", 0, 0, 0, 0, None, 10, 8, 2, 96, 192, None)
    with pytest.raises(YattnError, match="query heads per kv head"):
        call("yattn_decode_run", 1, 1, 1, 0, 0, 64, 2, 128, 256, None, 0, None)
    with pytest.raises(YattnError, match="kv_dim"):
        call("yattn_attn_decode", 0, 0, 0, 0, None, 10, 8, 2, 128, 100, None)
    with pytest.raises(YattnError, match="head_dim 96"):
        call_void("cuda_k_attn_decode", 0, 0, 0, 0, 10, 8, 2, 96, 192)
    lib.yattn_clear_error()
    assert lib.yattn_last_error() == b""
    assert lib.yattn_version() >= 10000


def test_workspace_size_formula():
    from yllm_b200._lib import lib

    # counters (256-aligned) + (m,l) (256-aligned) + o
    n = lib.yattn_decode_workspace_bytes(10, 3, 32, 8, 128)
    assert n == 256 + 512 + 10 * 4 * 128 * 4
    assert lib.yattn_decode_workspace_bytes(0, 0, 32, 8, 128) == 0


def test_rope_store_rejects_bad_arguments():
    """yattn_rope_store_kv checks its geometry and rope kind on the host, before any launch."""
    import ctypes as C

    from yllm_b200._lib import lib

    err = C.create_string_buffer(256)
    fake = C.c_void_p(0x1000)   # never dereferenced: every case fails before a launch
    assert lib.yattn_rope_store_kv(fake, 0, 32, 8, 128, 1024, 0, 0, 1e4, None, None, err, 256) == 0   # nothing to do
    assert lib.yattn_rope_store_kv(fake, 4, 32, 8, 128, 1024, 3, 0, 1e4, None, None, err, 256) == -1
    assert b"rope_kind" in err.value
    assert lib.yattn_rope_store_kv(fake, 4, 32, 8, 127, 1024, 0, 0, 1e4, None, None, err, 256) == -1
    assert b"geometry" in err.value
    assert lib.yattn_rope_store_kv(fake, 4, 16, 2, 256, 512, 2, 300, 1e4, None, None, err, 256) == -1
    assert b"rotated dims" in err.value
    assert lib.yattn_rope_store_kv(None, 4, 32, 8, 128, 1024, 0, 0, 1e4, None, None, err, 256) == -1
    # the batch form
    assert lib.yattn_rope_store_kv_batch(fake, fake, fake, fake, fake, 0, 0, 4096, 32, 8, 128, 1024, 0, 0, 1e4,
                                         None, None, err, 256) == 0
    assert lib.yattn_rope_store_kv_batch(fake, fake, fake, fake, fake, 0, 8, 4000, 32, 8, 128, 1024, 0, 0, 1e4,
                                         None, None, err, 256) == -1
    assert b"q_stride" in err.value
    assert lib.yattn_rope_store_kv_batch(fake, None, fake, fake, fake, 0, 8, 4096, 32, 8, 128, 1024, 0, 0, 1e4,
                                         None, None, err, 256) == -1
    # QK-norm needs both weight vectors, aligned to their element size
    from yllm_b200._lib import YattnQkNorm

    half = YattnQkNorm(0x1000, None, 0, 1e-6)
    assert lib.yattn_rope_store_kv(fake, 4, 16, 8, 128, 1024, 1, 0, 1e6, C.byref(half), None, err, 256) == -1
    assert b"both" in err.value
    odd = YattnQkNorm(0x1002, 0x2000, 0, 1e-6)
    assert lib.yattn_rope_store_kv(fake, 4, 16, 8, 128, 1024, 1, 0, 1e6, C.byref(odd), None, err, 256) == -1
    assert b"aligned" in err.value
    assert lib.yattn_rope_store_kv_batch(fake, fake, fake, fake, fake, 0xFFFFFFF0, 64, 4096, 32, 8, 128, 1024, 0, 0,
                                         1e4, None, None, err, 256) == -1
    assert b"overflow" in err.value


def test_gdn_inputs_rejects_bad_arguments():
    """yattn_gdn_inputs checks the channel split and the taps on the host, before any launch."""
    import ctypes as C

    from yllm_b200._lib import lib

    err = C.create_string_buffer(256)
    f = C.c_void_p(0x1000)   # never dereferenced
    ptrs = [f] * 12
    assert lib.yattn_gdn_inputs(*ptrs, 0, 1, 8192, 4, 16, 128, 32, 128, 1e-6, None, err, 256) == 0   # no work
    assert lib.yattn_gdn_inputs(*ptrs, 1, 1, 10000, 4, 16, 128, 32, 128, 1e-6, None, err, 256) == -1
    assert b"conv_chan" in err.value
    assert lib.yattn_gdn_inputs(*ptrs, 1, 1, 8192, 9, 16, 128, 32, 128, 1e-6, None, err, 256) == -1
    assert b"kwidth" in err.value
    assert lib.yattn_gdn_inputs(*ptrs, 1, 1, 2 * 512 + 512, 4, 1, 512, 1, 512, 1e-6, None, err, 256) == -1
    bad = list(ptrs)
    bad[3] = None
    assert lib.yattn_gdn_inputs(*bad, 1, 1, 8192, 4, 16, 128, 32, 128, 1e-6, None, err, 256) == -1
    assert b"null" in err.value


def test_sess_kv_checks_before_touching_the_device(tmp_path):
    """The session KV calls check their arguments and the file header on the host before any device copy
    (a fake device pointer is never dereferenced)."""
    import ctypes as C
    import struct

    from yllm_b200._lib import lib

    err = C.create_string_buffer(256)
    fake = C.c_void_p(0x1000)
    p = C.c_uint32(7)
    path = tmp_path / "x.kv"
    path.write_bytes(b"YLLMSKV0" + struct.pack("<4I", 2, 128, 16, 5))
    assert lib.yattn_sess_kv_load(fake, 3, 128, 16, str(path).encode(), C.byref(p), None, err, 256) == -1
    assert b"n_blocks=2" in err.value and p.value == 7
    assert lib.yattn_sess_kv_load(fake, 2, 256, 16, str(path).encode(), C.byref(p), None, err, 256) == -1
    assert lib.yattn_sess_kv_load(fake, 2, 128, 17, str(path).encode(), C.byref(p), None, err, 256) == -1
    path.write_bytes(b"YLLMSKV0" + struct.pack("<4I", 2, 128, 16, 17))    # pos > max_seq
    assert lib.yattn_sess_kv_load(fake, 2, 128, 16, str(path).encode(), C.byref(p), None, err, 256) == -1
    path.write_bytes(b"YLLMSESS" + struct.pack("<4I", 2, 128, 16, 5))    # the token file's magic
    assert lib.yattn_sess_kv_load(fake, 2, 128, 16, str(path).encode(), C.byref(p), None, err, 256) == -1
    assert b"not a session KV file" in err.value
    assert lib.yattn_sess_kv_load(fake, 2, 128, 16, str(tmp_path / "missing").encode(), C.byref(p), None, err,
                                  256) == -1
    assert lib.yattn_sess_kv_save(fake, 2, 128, 16, 17, str(path).encode(), None, err, 256) == -1
    assert b"pos 17 > max_seq 16" in err.value
    assert lib.yattn_sess_kv_save(None, 2, 128, 16, 5, str(path).encode(), None, err, 256) == -1


def test_gemv_checks_arguments():
    """The linear-layer calls reject a Q4_K row that is not whole blocks and unaligned Q4_K operands on the host."""
    import ctypes as C

    from yllm_b200._lib import lib

    err = C.create_string_buffer(256)
    f = C.c_void_p(0x1000)
    assert lib.yattn_gemv_q4k(f, f, f, 64, 300, 1, None, err, 256) == -1
    assert b"multiple of 256" in err.value
    assert lib.yattn_gemv_q4k(f, C.c_void_p(0x1004), f, 64, 256, 1, None, err, 256) == -1
    assert b"aligned" in err.value
    assert lib.cuda_k_gemv_q4k(f, f, f, 0, 256, err, 256) == -1
    assert lib.cuda_k_gemm_f16(None, f, f, f, None, 64, 64, 0, err, 256) == -1
    assert lib.yattn_gemv_f16(None, f, f, 64, 64, 1, None, err, 256) == -1


def _plan_ctas(ctx, n_kv, hd, target=148):
    import ctypes as C

    from yllm_b200._lib import YattnDecodeWork, lib

    pos = (C.c_uint32 * len(ctx))(*[c - 1 for c in ctx])
    cap = 8192
    w = (YattnDecodeWork * cap)()
    nw, npp, ng = C.c_uint32(), C.c_uint32(), C.c_uint32()
    err = C.create_string_buffer(256)
    assert lib.yattn_decode_plan_pooled(pos, len(ctx), n_kv, hd, 0, target, w, cap, C.byref(nw), C.byref(npp),
                                        C.byref(ng), err, 256) == 0, err.value
    ctas = {}
    for i in range(nw.value):
        ctas.setdefault(w[i].cta, []).append((w[i].item, w[i].kv_head, w[i].t_begin, w[i].t_end))
    return ctas


def test_decode_plan_cuts():
    """The balanced plan covers every key of every (item, kv head) once; equal ranges fewer than the CTAs take the
    equal cut (one unit per CTA), ragged ones the balanced cut within the CTA budget."""
    from yllm_b200.configs import CFG3, CFG5_GATED_DECODE

    for cfg, expect_uniform in ((CFG5_GATED_DECODE, True), (CFG3, False)):
        ctx = cfg.ctx()
        ctas = _plan_ctas(ctx, cfg.n_kv_heads, cfg.head_dim)
        assert len(ctas) <= 148
        cover = {}
        for units in ctas.values():
            for item, kvh, b, e in units:
                cover.setdefault((item, kvh), []).append((b, e))
        for (item, kvh), spans in cover.items():
            spans.sort()
            assert spans[0][0] == 0 and spans[-1][1] == ctx[item]
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:])), "gap or overlap"
        one_unit = all(len(u) == 1 for u in ctas.values())
        assert one_unit == expect_uniform, cfg.name
    # config 5c: 32 x 4096 keys over 2 kv heads -> 2 pieces of 2048 per range on 128 CTAs
    ctas = _plan_ctas(CFG5_GATED_DECODE.ctx(), 2, 256)
    assert len(ctas) == 128 and all(u[0][3] - u[0][2] == 2048 for u in ctas.values())
