"""ctypes binding of libyllm_attn_sm100.so (the C ABI in include/yllm_attn_sm100.h).

Importing this module loads the in-tree shared library.  There is no fallback:
if the library is missing the import fails with instructions to build it.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libyllm_attn_sm100.so"

if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing: build the CUDA library first "
        "(python -m yllm_b200.build, or __graft_entry__.build())"
    )

lib = C.CDLL(str(LIB_PATH))

u16p = C.POINTER(C.c_uint16)
f32p = C.POINTER(C.c_float)
vp = C.c_void_p
u32 = C.c_uint32
u64 = C.c_uint64
sz = C.c_size_t
cp = C.c_char_p


class YattnDecodeItem(C.Structure):
    _fields_ = [
        ("q", vp),
        ("out", vp),
        ("k", vp),
        ("v", vp),
        ("gate", vp),
        ("pos", u32),
        ("reserved", u32),
    ]


class YattnRopeItem(C.Structure):
    _fields_ = [
        ("q", vp),
        ("k", vp),
        ("v", vp),
        ("kcache", vp),
        ("vcache", vp),
        ("pos", u32),
        ("reserved", u32),
    ]


class YattnDecodeNewRow(C.Structure):
    _fields_ = [
        ("k", vp),
        ("v", vp),
    ]


class YattnQkNorm(C.Structure):
    _fields_ = [
        ("q_w", vp),
        ("k_w", vp),
        ("w_f16", C.c_int),
        ("eps", C.c_float),
    ]


class YattnDecodeWork(C.Structure):
    _fields_ = [
        ("item", u32),
        ("kv_head", C.c_uint16),
        ("n_splits", C.c_uint16),
        ("split", u32),
        ("t_begin", u32),
        ("t_end", u32),
        ("part_base", u32),
        ("group", u32),
        ("cta", u32),
    ]


def _proto(name, restype, argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = argtypes
    return fn


E = [cp, sz]  # (err, errlen) tail

PROTOS = {
    "yattn_version": (C.c_int, []),
    "yattn_last_error": (cp, []),
    "yattn_clear_error": (None, []),
    "yattn_device_status": (C.c_int, [C.POINTER(C.c_int), C.c_int, *E]),
    "cuda_k_attn_decode": (None, [vp, vp, vp, vp, u32, u32, u32, u32, u32]),
    "cuda_k_attn_prefill": (None, [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32]),
    "yattn_attn_prefill": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, u32, vp, *E]),
    "cuda_k_store_kv": (None, [vp, vp, vp, vp, u32, u32]),
    "cuda_k_store_kv_batch": (None, [vp, vp, vp, vp, u32, u32, u32]),
    "yattn_decode_plan": (
        C.c_int,
        [C.POINTER(u32), u32, u32, u32, u32, u32, C.POINTER(YattnDecodeWork), u32,
         C.POINTER(u32), C.POINTER(u32), C.POINTER(u32), *E],
    ),
    "yattn_decode_plan_pooled": (
        C.c_int,
        [C.POINTER(u32), u32, u32, u32, u32, u32, C.POINTER(YattnDecodeWork), u32,
         C.POINTER(u32), C.POINTER(u32), C.POINTER(u32), *E],
    ),
    "yattn_decode_run_pooled": (
        C.c_int, [vp, vp, u32, u32, u32, u32, u32, u32, u32, vp, sz, vp, sz, vp, *E]),
    "yattn_decode_workspace_bytes": (sz, [u32, u32, u32, u32, u32]),
    "yattn_decode_workspace_init": (C.c_int, [vp, sz, vp, *E]),
    "yattn_decode_run": (C.c_int, [vp, vp, u32, u32, u32, u32, u32, u32, u32, vp, sz, vp, *E]),
    "yattn_decode_partial_workspace_bytes": (sz, [u32, u32, u32, u32]),
    "yattn_decode_partial": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, sz, vp, *E]),
    "yattn_merge_partials": (C.c_int, [vp, vp, vp, u32, u32, u32, vp, vp, *E]),
    "yattn_merge_partials_packed": (C.c_int, [vp, vp, u32, u32, u32, vp, vp, *E]),
    "yattn_exchange_area_bytes": (sz, [u32, u32, u32]),
    "yattn_exchange_area_alloc": (C.c_int, [u32, u32, u32, C.POINTER(vp), *E]),
    "yattn_exchange_area_free": (C.c_int, [vp, *E]),
    "yattn_ipc_handle": (C.c_int, [vp, vp, *E]),
    "yattn_ipc_open": (C.c_int, [vp, C.POINTER(vp), *E]),
    "yattn_ipc_close": (C.c_int, [vp, *E]),
    "yattn_exchange_merge": (C.c_int, [vp, vp, vp, u32, u32, u32, u32, vp, vp, u64, vp, *E]),
    "yattn_attn_decode": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, *E]),
    "yattn_decode_run_pooled_rope": (C.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, vp, sz, C.c_int, u32,
                                               C.c_float, vp, sz, vp, *E]),
    "yattn_decode_exchange": (C.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, u32, u32, vp, vp, u64, vp, sz,
                                        vp, *E]),
    "yattn_attn_decode_noalloc": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, *E]),
    "yattn_reserve": (C.c_int, [sz, *E]),
    "yattn_store_kv": (C.c_int, [vp, vp, vp, vp, u32, u32, u32, vp, *E]),
    "yattn_rope_store_kv": (C.c_int, [vp, u32, u32, u32, u32, u32, C.c_int, u32, C.c_float, vp, vp, *E]),
    "yattn_gdn_inputs": (C.c_int, [vp] * 12 + [u32] * 8 + [C.c_float, vp, *E]),
    "yattn_sess_kv_save": (C.c_int, [vp, u32, u32, u32, u32, C.c_char_p, vp, *E]),
    "yattn_sess_kv_load": (C.c_int, [vp, u32, u32, u32, C.c_char_p, C.POINTER(u32), vp, *E]),
    "yattn_gemv_q4k": (C.c_int, [vp, vp, vp, u32, u32, u32, vp, *E]),
    "yattn_gemv_q4k_multi": (C.c_int, [u32, vp, vp, vp, vp, u32, vp, *E]),
    "yattn_gemv_f16": (C.c_int, [vp, vp, vp, u32, u32, u32, vp, *E]),
    "cuda_k_gemv_q4k": (C.c_int, [vp, vp, vp, u32, u32, *E]),
    "cuda_k_gemm_q4k": (C.c_int, [vp, vp, vp, u32, u32, u32, *E]),
    "cuda_k_gemv_f16": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, *E]),
    "cuda_k_gemm_f16": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, *E]),
    "yattn_rope_store_kv_batch": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, C.c_int, u32,
                                            C.c_float, vp, vp, *E]),
    "cuda_k_gdn_state_update": (None, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32]),
    "yattn_gdn_decode": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, vp, C.c_float, vp, *E]),
    "yattn_gdn_prefill": (
        C.c_int, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp, C.c_float, vp, *E]),
    "yattn_gdn_prefill_recurrent": (
        C.c_int, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp, C.c_float, vp, *E]),
    "yattn_gen_rows": (
        C.c_int,
        [vp, C.c_int, sz, sz, u32, u32, u64, u64, C.c_double, C.c_int, u32, C.c_double, vp, *E],
    ),
    "yattn_gen_gdn_gates": (C.c_int, [vp, vp, u64, u64, u64, sz, vp, *E]),
    "yattn_gen_gdn_qk": (C.c_int, [vp, u64, u64, sz, u32, u32, C.c_float, vp, *E]),
    "yattn_checksum": (C.c_int, [vp, sz, C.POINTER(u64), vp, *E]),
}

for _name, (_res, _args) in PROTOS.items():
    _proto(_name, _res, _args)


class YattnError(RuntimeError):
    """A C-ABI entry point returned -1 (or left yattn_last_error set)."""


def call(name: str, *args) -> None:
    """Calls an error-returning yattn_* entry point and raises on -1."""
    err = C.create_string_buffer(512)
    rc = getattr(lib, name)(*args, err, C.sizeof(err))
    if rc != 0:
        raise YattnError(f"{name}: {err.value.decode(errors='replace')}")


def call_void(name: str, *args) -> None:
    """Calls a void drop-in entry point and raises if it recorded an error."""
    lib.yattn_clear_error()
    getattr(lib, name)(*args)
    msg = lib.yattn_last_error()
    if msg:
        raise YattnError(f"{name}: {msg.decode(errors='replace')}")
