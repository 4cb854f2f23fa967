"""Seeded workload inputs generated directly in HBM by the library's fixture kernels.

Layouts follow the engine: K/V caches are fp16 bits (torch.uint16) rows of
kv_dim; q/out are fp32 with heads contiguous.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ._lib import call
from .attn import _stream
from .configs import DecodeCfg, GdnCfg, PrefillCfg, seed_of

GEN_F32, GEN_F16, GEN_F32_F16, GEN_F32_BF16 = 0, 1, 2, 3


def gen_rows(dst: torch.Tensor, kind: int, row_stride: int, n_rows: int, n_heads: int, head_dim: int, seed: int,
             first_row: int = 0, scale: float = 1.0, rope: bool = False, pos0: int = 0, theta: float = 1e6,
             stream=None) -> None:
    call("yattn_gen_rows", dst.data_ptr(), kind, row_stride, n_rows, n_heads, head_dim, seed, first_row,
         float(scale), 1 if rope else 0, pos0, float(theta), _stream(stream))


def gen_gdn_gates(gate: torch.Tensor, beta: torch.Tensor, seed_a: int, seed_b: int, first: int = 0,
                  stream=None) -> None:
    call("yattn_gen_gdn_gates", gate.data_ptr(), beta.data_ptr(), seed_a, seed_b, first, gate.numel(),
         _stream(stream))


def gen_gdn_qk(dst: torch.Tensor, seed: int, n_rows: int, n_heads: int, head_dim: int, eps: float,
               first_row: int = 0, stream=None) -> None:
    call("yattn_gen_gdn_qk", dst.data_ptr(), seed, first_row, n_rows, n_heads, head_dim, float(eps),
         _stream(stream))


def checksum(t: torch.Tensor, stream=None) -> int:
    import ctypes as C

    out = C.c_uint64(0)
    call("yattn_checksum", t.data_ptr(), t.numel() * t.element_size(), C.byref(out), _stream(stream))
    return out.value


@dataclass
class DecodeInputs:
    cfg: DecodeCfg
    ctx: list
    q: torch.Tensor          # [layers, n_seqs, n_heads*hd] f32
    out: torch.Tensor        # same shape
    gate: Optional[torch.Tensor]
    kv_pool: torch.Tensor    # uint16, per sequence one engine blob [2*n_layers][ctx_i][kv_dim]
    seq_off: list            # element offset of each sequence's blob in kv_pool
    n_layers: int            # layers actually built (K regions 0..n-1, V regions n..2n-1)

    def k_ptr(self, layer: int, seq: int) -> int:
        c = self.ctx[seq]
        return self.kv_pool.data_ptr() + 2 * (self.seq_off[seq] + layer * c * self.cfg.kv_dim)

    def v_ptr(self, layer: int, seq: int) -> int:
        c = self.ctx[seq]
        return self.kv_pool.data_ptr() + 2 * (self.seq_off[seq] + (self.n_layers + layer) * c * self.cfg.kv_dim)

    def k_view(self, layer: int, seq: int) -> torch.Tensor:
        c, kd = self.ctx[seq], self.cfg.kv_dim
        o = self.seq_off[seq] + layer * c * kd
        return self.kv_pool[o:o + c * kd].view(c, kd)

    def v_view(self, layer: int, seq: int) -> torch.Tensor:
        c, kd = self.ctx[seq], self.cfg.kv_dim
        o = self.seq_off[seq] + (self.n_layers + layer) * c * kd
        return self.kv_pool[o:o + c * kd].view(c, kd)


def decode_inputs(cfg: DecodeCfg, layers: Optional[list] = None, seqs: Optional[list] = None,
                  device="cuda") -> DecodeInputs:
    """Builds the config's KV caches and queries.  layers/seqs pick a subset
    (seed numbering keeps the full config's indices)."""
    layers = list(range(cfg.layers)) if layers is None else list(layers)
    seqs = list(range(cfg.n_seqs)) if seqs is None else list(seqs)
    ctx = [cfg.ctx_of(s) for s in seqs]
    L, kd, H, hd = len(layers), cfg.kv_dim, cfg.n_heads, cfg.head_dim
    offs, tot = [], 0
    for c in ctx:
        offs.append(tot)
        tot += 2 * L * c * kd
    pool = torch.empty(tot, dtype=torch.uint16, device=device)
    q = torch.empty(L, len(seqs), H * hd, dtype=torch.float32, device=device)
    gate = torch.empty_like(q) if cfg.gated else None
    qkind = GEN_F32_BF16 if cfg.q_kind == "bf16" else GEN_F32
    for li, l in enumerate(layers):
        for si, s in enumerate(seqs):
            c = ctx[si]
            kbase = pool[offs[si] + li * c * kd:]
            vbase = pool[offs[si] + (L + li) * c * kd:]
            gen_rows(kbase, GEN_F16, kd, c, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "k", l, s), rope=cfg.rope,
                     theta=cfg.theta)
            gen_rows(vbase, GEN_F16, kd, c, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "v", l, s))
            gen_rows(q[li, si], qkind, H * hd, 1, H, hd, seed_of(cfg.cfg, "q", l, s), rope=cfg.rope, pos0=c - 1,
                     theta=cfg.theta)
            if gate is not None:
                gen_rows(gate[li, si], GEN_F32_BF16, H * hd, 1, H, hd, seed_of(cfg.cfg, "gate", l, s))
    out = torch.zeros_like(q)
    return DecodeInputs(cfg, ctx, q, out, gate, pool, offs, L)


@dataclass
class GdnInputs:
    cfg: GdnCfg
    n_seqs: int
    T: int
    S: torch.Tensor       # [n_seqs, n_vheads, 128, 128] f32
    q: torch.Tensor       # [n_seqs*T, num_k_heads*128]
    k: torch.Tensor
    v: torch.Tensor       # [n_seqs*T, n_vheads*128]
    gate: torch.Tensor    # [n_seqs*T, n_vheads]
    beta: torch.Tensor
    z: torch.Tensor       # [n_seqs*T, n_vheads*128]
    norm_w: torch.Tensor  # [128]
    out: torch.Tensor


def gdn_inputs(cfg: GdnCfg, n_seqs: int, T: int, seeded_state: bool, device="cuda") -> GdnInputs:
    """GDN token inputs for n_seqs sequences of T tokens (rows seq*T + t):
    q,k = l2norm(bf16(N(0,1))), v,z = bf16(N(0,1)), gate = -softplus(N(0,1)),
    beta = sigmoid(N(0,1)), norm weight 1 + 0.1 N(0,1); state zero or N(0,1)*state_scale."""
    D, NK, NV = cfg.head_dim, cfg.num_k_heads, cfg.n_v_heads
    rows = n_seqs * T
    c = cfg.cfg
    S = torch.zeros(n_seqs, NV, D, D, dtype=torch.float32, device=device)
    if seeded_state:
        gen_rows(S, GEN_F32, D, n_seqs * NV * D, 1, D, seed_of(c, "state"), scale=cfg.state_scale)
    q = torch.empty(rows, NK * D, dtype=torch.float32, device=device)
    k = torch.empty_like(q)
    gen_gdn_qk(q, seed_of(c, "gdn_q"), rows, NK, D, cfg.eps)
    gen_gdn_qk(k, seed_of(c, "gdn_k"), rows, NK, D, cfg.eps)
    v = torch.empty(rows, NV * D, dtype=torch.float32, device=device)
    gen_rows(v, GEN_F32_BF16, NV * D, rows, NV, D, seed_of(c, "gdn_v"))
    z = torch.empty_like(v)
    gen_rows(z, GEN_F32_BF16, NV * D, rows, NV, D, seed_of(c, "z"))
    gate = torch.empty(rows, NV, dtype=torch.float32, device=device)
    beta = torch.empty_like(gate)
    gen_gdn_gates(gate, beta, seed_of(c, "gdn_a"), seed_of(c, "gdn_b"))
    w = torch.empty(D, dtype=torch.float32, device=device)
    gen_rows(w, GEN_F32, D, 1, 1, D, seed_of(c, "norm_w"), scale=0.1)
    w += 1.0
    out = torch.zeros_like(v)
    return GdnInputs(cfg, n_seqs, T, S, q, k, v, gate, beta, z, w, out)


@dataclass
class PrefillInputs:
    cfg: PrefillCfg
    q: torch.Tensor       # [S, n_heads*hd] f32 (fp16-exact values)
    k: torch.Tensor       # [S, kv_dim] uint16
    v: torch.Tensor       # [S, kv_dim] uint16
    gate: Optional[torch.Tensor]
    out: torch.Tensor


def prefill_inputs(cfg: PrefillCfg, seq_len: Optional[int] = None, device="cuda") -> PrefillInputs:
    S = seq_len or cfg.seq_len
    H, hd, kd = cfg.n_heads, cfg.head_dim, cfg.kv_dim
    q = torch.empty(S, H * hd, dtype=torch.float32, device=device)
    k = torch.empty(S, kd, dtype=torch.uint16, device=device)
    v = torch.empty(S, kd, dtype=torch.uint16, device=device)
    gen_rows(q, GEN_F32_F16, H * hd, S, H, hd, seed_of(cfg.cfg, "q"), scale=cfg.scale, rope=cfg.rope,
             theta=cfg.theta)
    gen_rows(k, GEN_F16, kd, S, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "k"), scale=cfg.scale, rope=cfg.rope,
             theta=cfg.theta)
    gen_rows(v, GEN_F16, kd, S, cfg.n_kv_heads, hd, seed_of(cfg.cfg, "v"), scale=cfg.scale)
    gate = None
    if cfg.gated:
        gate = torch.empty(S, H * hd, dtype=torch.float32, device=device)
        gen_rows(gate, GEN_F32_BF16, H * hd, S, H, hd, seed_of(cfg.cfg, "gate"))
    out = torch.zeros(S, H * hd, dtype=torch.float32, device=device)
    return PrefillInputs(cfg, q, k, v, gate, out)
