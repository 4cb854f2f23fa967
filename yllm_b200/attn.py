"""Host-side mirror of the engine's attention entry points on torch tensors.

Each function forwards to the C ABI (include/yllm_attn_sm100.h) with the
tensors' device pointers and the current torch stream.  Names and argument
meaning follow the reference's CUDA launchers (inference/cuda/cuda_kernels.h):
cuda_k_attn_decode, cuda_k_attn_prefill, cuda_k_store_kv(_batch), plus the
batched / split-KV / gated / GDN entry points the engine lacks today.
Nothing here computes attention on the host: every path launches the CUDA
library, and a missing library fails at import.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import (YattnDecodeItem, YattnDecodeNewRow, YattnDecodeWork, YattnQkNorm, YattnRopeItem, call,
                   call_void, lib)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _kv_tensor(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda or t.dtype not in (torch.uint16, torch.float16, torch.int16):
        raise ValueError(f"{name} must be a CUDA fp16-bits tensor (uint16/float16/int16)")


# ----------------------------------------------------------------- drop-ins

def cuda_k_attn_decode(att_out: torch.Tensor, q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor,
                       pos: int, n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int) -> None:
    """Same contract as the reference launcher (cuda_kernels.h:55-58), legacy default stream."""
    _need(att_out, torch.float32, "att_out")
    _need(q, torch.float32, "q")
    _kv_tensor(kcache, "kcache")
    _kv_tensor(vcache, "vcache")
    call_void("cuda_k_attn_decode", att_out.data_ptr(), q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(),
              pos, n_heads, n_kv_heads, head_dim, kv_dim)


def cuda_k_attn_prefill(att_out: torch.Tensor, q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor,
                        pos_start: int, B: int, n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int,
                        q_stride: int) -> None:
    """Same contract as the reference launcher (cuda_kernels.h:60-63), legacy default stream."""
    _need(att_out, torch.float32, "att_out")
    _need(q, torch.float32, "q")
    _kv_tensor(kcache, "kcache")
    _kv_tensor(vcache, "vcache")
    call_void("cuda_k_attn_prefill", att_out.data_ptr(), q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(),
              pos_start, B, n_heads, n_kv_heads, head_dim, kv_dim, q_stride)


PREFILL_Q_F16 = 1   # YATTN_PREFILL_Q_F16: every q value is an fp16 value


def attn_prefill(att_out: torch.Tensor, q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor,
                 pos_start: int, B: int, n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int, q_stride: int,
                 gate: Optional[torch.Tensor] = None, q_f16: bool = False, stream=None) -> None:
    """Causal prefill of B tokens at pos_start (keys 0..pos_start+b), optional qwen35 gate.  q_f16=True
    promises that every q value is exactly an fp16 value (the kernel then skips q's lo plane; it checks the
    promise and reports a broken one as device status 202)."""
    _need(att_out, torch.float32, "att_out")
    _need(q, torch.float32, "q")
    if gate is not None:
        _need(gate, torch.float32, "gate")
    call("yattn_attn_prefill", att_out.data_ptr(), q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(), _ptr(gate),
         pos_start, B, n_heads, n_kv_heads, head_dim, kv_dim, q_stride, PREFILL_Q_F16 if q_f16 else 0,
         _stream(stream))


def cuda_k_store_kv(kcache: torch.Tensor, vcache: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos: int,
                    kv_dim: int) -> None:
    call_void("cuda_k_store_kv", kcache.data_ptr(), vcache.data_ptr(), k.data_ptr(), v.data_ptr(), pos, kv_dim)


def cuda_k_store_kv_batch(kcache: torch.Tensor, vcache: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          pos_start: int, B: int, kv_dim: int) -> None:
    call_void("cuda_k_store_kv_batch", kcache.data_ptr(), vcache.data_ptr(), k.data_ptr(), v.data_ptr(),
              pos_start, B, kv_dim)


# ------------------------------------------------------- error-returning API

def attn_decode(att_out: torch.Tensor, q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor, pos: int,
                n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int, gate: Optional[torch.Tensor] = None,
                stream=None) -> None:
    """One decode query (keys 0..pos) of one layer; optional qwen35 sigmoid gate."""
    _need(att_out, torch.float32, "att_out")
    _need(q, torch.float32, "q")
    if gate is not None:
        _need(gate, torch.float32, "gate")
    call("yattn_attn_decode", att_out.data_ptr(), q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(), _ptr(gate),
         pos, n_heads, n_kv_heads, head_dim, kv_dim, _stream(stream))


def store_kv(kcache: torch.Tensor, vcache: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos_start: int,
             kv_dim: int, stream=None) -> None:
    """fp32 rows -> fp16 cache rows pos_start.. with the engine's f32_to_f16 rounding."""
    _need(k, torch.float32, "k")
    _need(v, torch.float32, "v")
    B = k.numel() // kv_dim
    call("yattn_store_kv", kcache.data_ptr(), vcache.data_ptr(), k.data_ptr(), v.data_ptr(), pos_start, B, kv_dim,
         _stream(stream))


@dataclass
class DecodePlan:
    """A split schedule for a batch of decode queries (one per item).

    The schedule depends only on the query positions, so one plan serves every
    layer of a decode step: run() takes a device array of items per call.
    """

    n_items: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    kv_dim: int
    work: torch.Tensor        # device bytes of YattnDecodeWork[n_work]
    n_work: int
    n_parts: int
    n_groups: int
    workspace: Optional[torch.Tensor]
    pool: Optional[tuple] = None      # (base pointer, bytes): run through the pooled tensor-copy kernels

    @staticmethod
    def build(positions: Sequence[int], n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int,
              split_tokens: int = 0, target_ctas: int = 0, device=None,
              pool: Optional[tuple] = None) -> "DecodePlan":
        """pool = (base, bytes) of one allocation holding every item's K and V rows
        (row stride kv_dim): the plan and runs use the pooled variants."""
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.uint32))
        n = int(pos.size)
        cap = max(1, n * n_kv_heads * 64)
        while True:
            work = (YattnDecodeWork * cap)()
            n_work, n_parts, n_groups = C.c_uint32(), C.c_uint32(), C.c_uint32()
            err = C.create_string_buffer(512)
            plan_fn = lib.yattn_decode_plan_pooled if pool is not None else lib.yattn_decode_plan
            rc = plan_fn(pos.ctypes.data_as(C.POINTER(C.c_uint32)), n, n_kv_heads, head_dim,
                         split_tokens, target_ctas, work, cap, C.byref(n_work), C.byref(n_parts),
                         C.byref(n_groups), err, 512)
            if rc == 0:
                break
            if n_work.value > cap:
                cap = n_work.value
                continue
            raise _lib.YattnError("yattn_decode_plan: " + err.value.decode())
        nbytes = n_work.value * C.sizeof(YattnDecodeWork)
        host = torch.frombuffer(bytearray(C.string_at(work, nbytes)), dtype=torch.uint8)
        dev = host.to(device or "cuda")
        ws_bytes = lib.yattn_decode_workspace_bytes(n_parts.value, n_groups.value, n_heads, n_kv_heads, head_dim)
        ws = None
        if ws_bytes:
            ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device or "cuda")
        return DecodePlan(n, n_heads, n_kv_heads, head_dim, kv_dim, dev, n_work.value, n_parts.value,
                          n_groups.value, ws, tuple(pool) if pool is not None else None)

    def run_rope(self, items_dev: torch.Tensor, rows_dev: torch.Tensor, rope_kind: int, theta: float,
                 n_rope_dims: int = 0, stream=None) -> None:
        """run() with the step's RoPE + KV store fused in (yattn_decode_run_pooled_rope): items' q unrotated,
        rows_dev (make_new_rows) the new tokens' k and v; pooled plans only."""
        if self.pool is None:
            raise ValueError("the fused RoPE store runs on a pooled plan")
        ws_ptr = self.workspace.data_ptr() if self.workspace is not None else None
        ws_len = self.workspace.numel() if self.workspace is not None else 0
        call("yattn_decode_run_pooled_rope", items_dev.data_ptr(), rows_dev.data_ptr(), self.work.data_ptr(),
             self.n_work, self.n_parts, self.n_groups, self.n_heads, self.n_kv_heads, self.head_dim, self.kv_dim,
             self.pool[0], self.pool[1], rope_kind, n_rope_dims, theta, ws_ptr, ws_len, _stream(stream))

    def run(self, items_dev: torch.Tensor, stream=None) -> None:
        ws_ptr = self.workspace.data_ptr() if self.workspace is not None else None
        ws_len = self.workspace.numel() if self.workspace is not None else 0
        if self.pool is not None:
            call("yattn_decode_run_pooled", items_dev.data_ptr(), self.work.data_ptr(), self.n_work, self.n_parts,
                 self.n_groups, self.n_heads, self.n_kv_heads, self.head_dim, self.kv_dim, self.pool[0],
                 self.pool[1], ws_ptr, ws_len, _stream(stream))
        else:
            call("yattn_decode_run", items_dev.data_ptr(), self.work.data_ptr(), self.n_work, self.n_parts,
                 self.n_groups, self.n_heads, self.n_kv_heads, self.head_dim, self.kv_dim, ws_ptr, ws_len,
                 _stream(stream))


def make_items(entries: Sequence[tuple], device=None) -> torch.Tensor:
    """Device array of YattnDecodeItem from (q, out, k, v, gate_or_None, pos) tuples of tensors."""
    arr = (YattnDecodeItem * len(entries))()
    for i, (q, out, k, v, gate, pos) in enumerate(entries):
        arr[i].q = q.data_ptr()
        arr[i].out = out.data_ptr()
        arr[i].k = k.data_ptr() if isinstance(k, torch.Tensor) else int(k)
        arr[i].v = v.data_ptr() if isinstance(v, torch.Tensor) else int(v)
        arr[i].gate = gate.data_ptr() if gate is not None else 0
        arr[i].pos = int(pos)
    raw = bytearray(C.string_at(arr, C.sizeof(arr)))
    return torch.frombuffer(raw, dtype=torch.uint8).to(device or "cuda")


ROPE_LLAMA, ROPE_QWEN, ROPE_MROPE = 0, 1, 2


def make_new_rows(entries: Sequence[tuple], device=None) -> torch.Tensor:
    """Device array of YattnDecodeNewRow from (k, v) tensors: each item's new token (fp32, n_kv_heads*head_dim)."""
    arr = (YattnDecodeNewRow * len(entries))()
    for i, (k, v) in enumerate(entries):
        _need(k, torch.float32, "k")
        _need(v, torch.float32, "v")
        arr[i].k = k.data_ptr()
        arr[i].v = v.data_ptr()
    raw = bytearray(C.string_at(arr, C.sizeof(arr)))
    return torch.frombuffer(raw, dtype=torch.uint8).to(device or "cuda")


def make_rope_items(entries: Sequence[tuple], device=None) -> torch.Tensor:
    """Device array of YattnRopeItem from (q, k, v, kcache, vcache, pos) tuples; kcache / vcache are
    tensors or raw device addresses of the layer's cache bases."""
    arr = (YattnRopeItem * len(entries))()
    for i, (q, k, v, kc, vc, pos) in enumerate(entries):
        arr[i].q = q.data_ptr()
        arr[i].k = k.data_ptr()
        arr[i].v = v.data_ptr()
        arr[i].kcache = kc.data_ptr() if isinstance(kc, torch.Tensor) else int(kc)
        arr[i].vcache = vc.data_ptr() if isinstance(vc, torch.Tensor) else int(vc)
        arr[i].pos = int(pos)
    raw = bytearray(C.string_at(arr, C.sizeof(arr)))
    return torch.frombuffer(raw, dtype=torch.uint8).to(device or "cuda")


def qk_norm(q_w: torch.Tensor, k_w: torch.Tensor, eps: float):
    """The QK-norm argument of rope_store_kv(_batch): the layer's q and k rmsnorm weights (head_dim values, fp32,
    or fp16 as int16/uint16/float16 tensors) and eps (engine.c:915-919, 1036-1045)."""
    f16 = q_w.dtype in (torch.int16, torch.uint16, torch.float16)
    if f16 != (k_w.dtype in (torch.int16, torch.uint16, torch.float16)):
        raise ValueError("q and k norm weights must have the same dtype")
    if not f16:
        _need(q_w, torch.float32, "q_w")
        _need(k_w, torch.float32, "k_w")
    return YattnQkNorm(q_w.data_ptr(), k_w.data_ptr(), 1 if f16 else 0, float(eps))


def _norm_arg(norm):
    return None if norm is None else C.byref(norm)


def rope_store_kv(items: torch.Tensor, n_items: int, n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int,
                  rope_kind: int, theta: float, n_rope_dims: int = 0, norm=None, stream=None) -> None:
    """One decode step's RoPE of q (in place) and k, and the fp16 store of k and v at each item's position
    (engine.c:1052-1072 / cuda_fwd.c:136-147 for every item, one launch).  norm (qk_norm(...)) applies the
    per-head QK-norm first."""
    call("yattn_rope_store_kv", items.data_ptr(), n_items, n_heads, n_kv_heads, head_dim, kv_dim, rope_kind,
         n_rope_dims, theta, _norm_arg(norm), _stream(stream))


def rope_store_kv_batch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kcache: torch.Tensor,
                        vcache: torch.Tensor, pos_start: int, B: int, n_heads: int, n_kv_heads: int, head_dim: int,
                        kv_dim: int, rope_kind: int, theta: float, n_rope_dims: int = 0, q_stride: int = 0,
                        norm=None, stream=None) -> None:
    """RoPE + KV store of B consecutive tokens (rows of q, k, v) at positions pos_start.. (the batched prefill's
    cuda_fwd.c:207-218 in one launch).  q is rotated in place; norm as in rope_store_kv."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _need(t, torch.float32, name)
    call("yattn_rope_store_kv_batch", q.data_ptr(), k.data_ptr(), v.data_ptr(), kcache.data_ptr(), vcache.data_ptr(),
         pos_start, B, q_stride or n_heads * head_dim, n_heads, n_kv_heads, head_dim, kv_dim, rope_kind, n_rope_dims,
         theta, _norm_arg(norm), _stream(stream))


def decode_partial(ml: torch.Tensor, o: torch.Tensor, q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor,
                   t_begin: int, t_end: int, n_heads: int, n_kv_heads: int, head_dim: int, kv_dim: int,
                   stream=None) -> None:
    """Unmerged (m, l, o) over keys [t_begin, t_end): m in log2 units (score*log2 e)."""
    call("yattn_decode_partial", ml.data_ptr(), o.data_ptr(), q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(),
         t_begin, t_end, n_heads, n_kv_heads, head_dim, kv_dim, None, 0, _stream(stream))


def merge_partials(out: torch.Tensor, ml: torch.Tensor, o: torch.Tensor, n_parts: int, n_heads: int,
                   head_dim: int, gate: Optional[torch.Tensor] = None, stream=None) -> None:
    """Log-sum-exp merge of [n_parts][n_heads] partials into out[n_heads*head_dim]."""
    call("yattn_merge_partials", out.data_ptr(), ml.data_ptr(), o.data_ptr(), n_parts, n_heads, head_dim,
         _ptr(gate), _stream(stream))


def merge_partials_packed(out: torch.Tensor, parts: torch.Tensor, n_parts: int, n_heads: int, head_dim: int,
                          gate: Optional[torch.Tensor] = None, stream=None) -> None:
    """Log-sum-exp merge of packed parts [n_parts][n_heads*2 (m, l) + n_heads*head_dim (o)]."""
    call("yattn_merge_partials_packed", out.data_ptr(), parts.data_ptr(), n_parts, n_heads, head_dim, _ptr(gate),
         _stream(stream))


def cuda_k_gdn_state_update(S: torch.Tensor, out: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            gate: torch.Tensor, beta: torch.Tensor, num_k_heads: int, hk: int, n_vheads: int,
                            hv: int) -> None:
    """gdn_state_update (matvec.h:35-37) on device tensors, legacy default stream."""
    call_void("cuda_k_gdn_state_update", S.data_ptr(), out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
              gate.data_ptr(), beta.data_ptr(), num_k_heads, hk, n_vheads, hv)


def gdn_decode(S, out, q, k, v, gate, beta, n_seqs: int, num_k_heads: int, hk: int, n_vheads: int, hv: int,
               norm_w: Optional[torch.Tensor] = None, z: Optional[torch.Tensor] = None, eps: float = 1e-6,
               stream=None) -> None:
    """One GDN token for each of n_seqs sequences (state updated in place)."""
    for name, t in (("S", S), ("out", out), ("q", q), ("k", k), ("v", v), ("gate", gate), ("beta", beta)):
        _need(t, torch.float32, name)
    call("yattn_gdn_decode", S.data_ptr(), out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
         gate.data_ptr(), beta.data_ptr(), n_seqs, num_k_heads, hk, n_vheads, hv, _ptr(norm_w), _ptr(z), float(eps),
         _stream(stream))


def gdn_inputs(qkv, conv_state, conv_w, alpha, beta_in, ssm_dt, ssm_a, q, k, v, gate, beta, n_seqs: int, T: int,
               kwidth: int, num_k_heads: int, hk: int, n_vheads: int, hv: int, eps: float = 1e-6,
               stream=None) -> None:
    """The GDN layer's inputs for T tokens of n_seqs sequences (engine.c:785-821): gates, conv1d + silu, q/k/v
    split with l2-normalised q and k heads; conv_state updated in place."""
    for name, t in (("qkv", qkv), ("conv_state", conv_state), ("conv_w", conv_w), ("alpha", alpha),
                    ("beta_in", beta_in), ("ssm_dt", ssm_dt), ("ssm_a", ssm_a), ("q", q), ("k", k), ("v", v),
                    ("gate", gate), ("beta", beta)):
        _need(t, torch.float32, name)
    conv_chan = 2 * num_k_heads * hk + n_vheads * hv
    call("yattn_gdn_inputs", qkv.data_ptr(), conv_state.data_ptr(), conv_w.data_ptr(), alpha.data_ptr(),
         beta_in.data_ptr(), ssm_dt.data_ptr(), ssm_a.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
         gate.data_ptr(), beta.data_ptr(), n_seqs, T, conv_chan, kwidth, num_k_heads, hk, n_vheads, hv, float(eps),
         _stream(stream))


def gdn_prefill(S, out, q, k, v, gate, beta, n_seqs: int, T: int, num_k_heads: int, hk: int, n_vheads: int,
                hv: int, norm_w: Optional[torch.Tensor] = None, z: Optional[torch.Tensor] = None,
                eps: float = 1e-6, stream=None) -> None:
    """T GDN tokens per sequence in order (state updated in place)."""
    for name, t in (("S", S), ("out", out), ("q", q), ("k", k), ("v", v), ("gate", gate), ("beta", beta)):
        _need(t, torch.float32, name)
    call("yattn_gdn_prefill", S.data_ptr(), out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
         gate.data_ptr(), beta.data_ptr(), n_seqs, T, num_k_heads, hk, n_vheads, hv, _ptr(norm_w), _ptr(z),
         float(eps), _stream(stream))


def gdn_prefill_recurrent(S, out, q, k, v, gate, beta, n_seqs: int, T: int, num_k_heads: int, hk: int,
                          n_vheads: int, hv: int, norm_w: Optional[torch.Tensor] = None,
                          z: Optional[torch.Tensor] = None, eps: float = 1e-6, stream=None) -> None:
    """gdn_prefill token by token in the reference's operation order (GPU cross-check)."""
    for name, t in (("S", S), ("out", out), ("q", q), ("k", k), ("v", v), ("gate", gate), ("beta", beta)):
        _need(t, torch.float32, name)
    call("yattn_gdn_prefill_recurrent", S.data_ptr(), out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
         gate.data_ptr(), beta.data_ptr(), n_seqs, T, num_k_heads, hk, n_vheads, hv, _ptr(norm_w), _ptr(z),
         float(eps), _stream(stream))


def gemv_q4k(y: torch.Tensor, w: torch.Tensor, x: torch.Tensor, out: int, in_: int, B: int = 1,
             stream=None) -> None:
    """y[B][out] = Q4_K W[out][in] . x[B][in] (cuda_kernels.cu:161-249 semantics, fp32 x)."""
    _need(y, torch.float32, "y")
    _need(x, torch.float32, "x")
    if w.dtype != torch.uint8 or not w.is_cuda or w.numel() < out * (in_ // 256) * 144:
        raise ValueError("w must be a CUDA uint8 tensor of out * in/256 Q4_K blocks")
    call("yattn_gemv_q4k", y.data_ptr(), w.data_ptr(), x.data_ptr(), out, in_, B, _stream(stream))


def gemv_q4k_multi(ys, ws, outs, x: torch.Tensor, in_: int, stream=None) -> None:
    """One token through up to four Q4_K matrices that read the same x, in one launch: ys[i][:outs[i]] =
    W_i . x, each bit-identical to gemv_q4k(ys[i], ws[i], x, outs[i], in_) (the engine's q/k/v or gate/up
    calls of cuda_fwd.c:94-168 fused)."""
    n = len(ws)
    if not (1 <= n <= 4) or len(ys) != n or len(outs) != n:
        raise ValueError("gemv_q4k_multi: 1 to 4 matrices, with as many outputs and row counts")
    _need(x, torch.float32, "x")
    for y, w, o in zip(ys, ws, outs):
        _need(y, torch.float32, "y")
        if w.dtype != torch.uint8 or not w.is_cuda or w.numel() < o * (in_ // 256) * 144:
            raise ValueError("w must be a CUDA uint8 tensor of out * in/256 Q4_K blocks")
    yp = (C.c_void_p * n)(*[y.data_ptr() for y in ys])
    wp = (C.c_void_p * n)(*[w.data_ptr() for w in ws])
    op = (C.c_uint32 * n)(*[int(o) for o in outs])
    call("yattn_gemv_q4k_multi", n, yp, wp, op, x.data_ptr(), in_, _stream(stream))


def gemv_f16(y: torch.Tensor, w: torch.Tensor, x: torch.Tensor, out: int, in_: int, B: int = 1,
             stream=None) -> None:
    """y[B][out] = fp16 W[out][in] . x[B][in] in fp32 (matvec.c:111-122 per token)."""
    _need(y, torch.float32, "y")
    _need(x, torch.float32, "x")
    if w.element_size() != 2 or not w.is_cuda or w.numel() < out * in_:
        raise ValueError("w must be a CUDA 16-bit tensor of out * in fp16 weights")
    call("yattn_gemv_f16", y.data_ptr(), w.data_ptr(), x.data_ptr(), out, in_, B, _stream(stream))


def sess_kv_save(kv: torch.Tensor, n_blocks: int, kv_dim: int, max_seq: int, pos: int, path: str,
                 stream=None) -> None:
    """Writes the first pos rows of every block's K and V regions of the device blob kv
    ([2*n_blocks+1][max_seq][kv_dim] fp16) as the engine's session KV file (cache.c:174-195)."""
    if kv.numel() * kv.element_size() < (2 * n_blocks + 1) * max_seq * kv_dim * 2:
        raise ValueError("kv is smaller than the (2*n_blocks+1)-region blob")
    call("yattn_sess_kv_save", kv.data_ptr(), n_blocks, kv_dim, max_seq, pos, os.fsencode(path), _stream(stream))


def sess_kv_load(kv: torch.Tensor, n_blocks: int, kv_dim: int, max_seq: int, path: str, stream=None) -> int:
    """Reads an engine session KV file into the device blob kv; returns the file's pos (cache.c:219-247)."""
    if kv.numel() * kv.element_size() < (2 * n_blocks + 1) * max_seq * kv_dim * 2:
        raise ValueError("kv is smaller than the (2*n_blocks+1)-region blob")
    p = C.c_uint32(0)
    call("yattn_sess_kv_load", kv.data_ptr(), n_blocks, kv_dim, max_seq, os.fsencode(path), C.byref(p),
         _stream(stream))
    return p.value


def device_status(clear: bool = True) -> int:
    st = C.c_int(0)
    call("yattn_device_status", C.byref(st), 1 if clear else 0)
    return st.value


def reserve(nbytes: int) -> None:
    call("yattn_reserve", nbytes)


def version() -> int:
    return lib.yattn_version()
