"""The five attention workloads (shapes, seeds) the path is measured and checked on.

Seeds: every tensor of every config has its own splitmix64 stream
seed_of(config, tensor, layer, seq); value i of a tensor is draw i of that
stream (Box-Muller, see yllm_b200/csrc/fixture.cu).  The same numbers are
produced on the GPU (fixture kernels) and by the test oracle on the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass

MASK64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15

TENSOR = {
    "q": 1, "k": 2, "v": 3, "gate": 4, "gdn_a": 5, "gdn_b": 6, "z": 7, "norm_w": 8,
    "state": 9, "ctx": 10, "gdn_q": 11, "gdn_k": 12, "gdn_v": 13,
}


def seed_of(cfg: int, tensor: str, layer: int = 0, seq: int = 0) -> int:
    return (0x5941 << 48) ^ (cfg << 40) ^ (TENSOR[tensor] << 32) ^ ((layer & 0xFFFF) << 16) ^ (seq & 0xFFFF)


def splitmix_draw(seed: int, k: int) -> int:
    """k-th (0-based) yrng() output of stream `seed` (platform.c:405-417)."""
    if seed == 0:
        seed = GOLDEN
    z = (seed + (k + 1) * GOLDEN) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def ctx_lengths(n: int, lo: int, hi: int, seed: int) -> list[int]:
    """Ragged context lengths, uniform in [lo, hi]."""
    return [lo + splitmix_draw(seed, i) % (hi - lo + 1) for i in range(n)]


@dataclass(frozen=True)
class DecodeCfg:
    cfg: int
    name: str
    n_heads: int
    n_kv_heads: int
    head_dim: int
    layers: int
    n_seqs: int
    ctx_lo: int
    ctx_hi: int
    rope: bool = False
    theta: float = 1e6
    gated: bool = False
    q_kind: str = "f32"   # f32 | bf16

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def ctx(self) -> list[int]:
        if self.ctx_lo == self.ctx_hi:
            return [self.ctx_lo] * self.n_seqs
        return ctx_lengths(self.n_seqs, self.ctx_lo, self.ctx_hi, seed_of(self.cfg, "ctx"))

    def ctx_of(self, seq: int) -> int:
        """Context length of sequence `seq`: ctx()[seq % n_seqs].  A job of N
        batches (one per GPU under weak scaling) repeats the config's lengths,
        so every GPU's share has the config's work; the KV/q bytes still differ
        per sequence (their seeds use the full sequence id)."""
        if self.ctx_lo == self.ctx_hi:
            return self.ctx_lo
        i = seq % self.n_seqs
        return self.ctx_lo + splitmix_draw(seed_of(self.cfg, "ctx"), i) % (self.ctx_hi - self.ctx_lo + 1)

    def kv_bytes_per_step(self) -> int:
        """K+V bytes one decode step reads (all layers, all sequences)."""
        return sum(self.ctx()) * self.kv_dim * 2 * 2 * self.layers

    def qo_bytes_per_step(self) -> int:
        return self.layers * self.n_seqs * self.n_heads * self.head_dim * 4 * 2


@dataclass(frozen=True)
class PrefillCfg:
    cfg: int
    name: str
    n_heads: int
    n_kv_heads: int
    head_dim: int
    seq_len: int
    scale: float = 1.0
    rope: bool = True
    theta: float = 1e6
    gated: bool = False

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def causal_flops(self) -> float:
        s = self.seq_len
        return 4.0 * self.head_dim * self.n_heads * s * (s + 1) / 2


@dataclass(frozen=True)
class GdnCfg:
    cfg: int
    name: str
    num_k_heads: int
    n_v_heads: int
    head_dim: int
    tokens: int
    chunk: int
    batch: int
    eps: float = 1e-6
    state_scale: float = 0.1


# the engine's CPU decode today (Qwen2.5-0.5B shape)
CFG1 = DecodeCfg(1, "qwen2.5-0.5b-decode-ctx512", 14, 2, 64, 24, 1, 512, 512, rope=True)
# causal batched prefill (Qwen3-0.6B shape), test_prefill_batch path
CFG2 = PrefillCfg(2, "qwen3-0.6b-prefill-s2048", 16, 8, 128, 2048, scale=0.5, rope=True)
# batched ragged decode (Llama-3-8B attention shape), sharded by sequence
CFG3 = DecodeCfg(3, "llama3-8b-batched-decode-64seq", 32, 8, 128, 32, 64, 1024, 8192)
# long-context single-sequence decode, split-KV across GPUs
CFG4 = DecodeCfg(4, "long-ctx-decode-131072", 32, 8, 128, 1, 1, 131072, 131072)
# qwen3.5 hybrid -- GDN and gated full attention
CFG5_GDN = GdnCfg(5, "qwen3.5-gdn", 16, 32, 128, 4096, 64, 32)
CFG5_GATED_DECODE = DecodeCfg(6, "qwen3.5-gated-decode-b32-ctx4096", 16, 2, 256, 1, 32, 4096, 4096,
                              gated=True, q_kind="bf16")
CFG5_GATED_PREFILL = PrefillCfg(7, "qwen3.5-gated-prefill-4096", 16, 2, 256, 4096, scale=1.0, rope=False,
                                gated=True)
