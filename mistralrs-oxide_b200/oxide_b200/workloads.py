"""Seeded synthetic workloads at Mistral-7B shapes and their algorithmic bytes.

Shapes, distributions and seeds of the five benchmark configurations:

  C1  RMSNorm f32: x [2048, 4096] ~ N(0,1), w [4096] ~ U(0.5,1.5), eps 1e-5 (seed 0)
  C2  residual add a+b, a,b [8192, 4096] ~ N(0,1); row-broadcast multiply by
      s [4096] ~ U(0.5,1.5); SwiGLU silu(gate)*up, gate,up [8192, 14336] ~ N(0,1) (seed 1)
  C3  scale+mask+softmax f32 over decode scores [8 x 32 heads x 1 x 32768],
      raw = z*sqrt(128) (scale 1/sqrt(128)), keys >= len_b masked,
      len_b ~ U[1024, 32768]; row argmax over logits [64, 32000] ~ N(0,1) (seed 2)
  C4  RoPE bf16: q [4096, 32, 128], k [4096, 8, 128] ~ N(0,1), positions
      0..4095, theta 1e6, f32 tables (seed 3)
  C5  the non-GEMM op chain of one Mistral-7B decoder layer in bf16 at
      64 seqs x 2048 tokens (hidden 4096, intermediate 14336, 32 q / 8 kv heads,
      head_dim 128, vocab 32000), seed 4

Host inputs come from numpy's PCG64 (``np.random.default_rng(seed)``) as f32
and are rounded to bf16 (nearest-even) where a config is bf16.  C5's ~30 G
elements are generated on the device instead (numpy would take minutes),
one sequence block at a time, each block from its own seeded torch CUDA
generator, so any range of sequences is reproducible on its own; GEMM
outputs the chain consumes are seeded N(0,1) tensors of the GEMM's output
shape (the GEMMs are not part of this path).  Algorithmic bytes count each
input read once and each output written once; masked softmax keys that are
never read are not counted.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

HIDDEN, INTER, NQ, NKV, HEAD_DIM, VOCAB = 4096, 14336, 32, 8, 128, 32000

F32, BF16 = 4, 2


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


# ---- C1 -----------------------------------------------------------------------
@dataclass
class C1:
    rows: int = 2048
    cols: int = HIDDEN
    eps: float = 1e-5
    seed: int = 0

    def inputs(self):
        rng = np.random.default_rng(self.seed)
        x = rng.standard_normal((self.rows, self.cols), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, self.cols).astype(np.float32)
        return x, w

    def bytes(self) -> int:
        return 2 * self.rows * self.cols * F32 + self.cols * F32


# ---- C2 -----------------------------------------------------------------------
@dataclass
class C2:
    rows: int = 8192
    cols: int = HIDDEN
    inter: int = INTER
    seed: int = 1

    def inputs(self):
        rng = np.random.default_rng(self.seed)
        a = rng.standard_normal((self.rows, self.cols), dtype=np.float32)
        b = rng.standard_normal((self.rows, self.cols), dtype=np.float32)
        s = rng.uniform(0.5, 1.5, self.cols).astype(np.float32)
        gate = rng.standard_normal((self.rows, self.inter), dtype=np.float32)
        up = rng.standard_normal((self.rows, self.inter), dtype=np.float32)
        return a, b, s, gate, up

    def bytes_add(self) -> int:
        return 3 * self.rows * self.cols * F32

    def bytes_mul(self) -> int:
        return 2 * self.rows * self.cols * F32 + self.cols * F32

    def bytes_silu_mul(self) -> int:
        return 3 * self.rows * self.inter * F32

    def bytes(self) -> int:
        """One step: h = a + b; y = h * s; o = silu(gate) * up."""
        return self.bytes_add() + self.bytes_mul() + self.bytes_silu_mul()


# ---- C3 -----------------------------------------------------------------------
@dataclass
class C3:
    batch: int = 8
    heads: int = NQ
    keys: int = 32768
    head_dim: int = HEAD_DIM
    logit_rows: int = 64
    vocab: int = VOCAB
    seed: int = 2

    @property
    def scale(self) -> float:
        return float(np.float32(1.0) / np.sqrt(np.float32(self.head_dim)))

    def inputs(self):
        rng = np.random.default_rng(self.seed)
        z = rng.standard_normal((self.batch, self.heads, 1, self.keys), dtype=np.float32)
        scores = (z * np.float32(math.sqrt(self.head_dim))).astype(np.float32)
        lens = rng.integers(1024, self.keys, size=self.batch, endpoint=True).astype(np.int32)
        logits = rng.standard_normal((self.logit_rows, self.vocab), dtype=np.float32)
        return scores, lens, logits

    def bytes_softmax(self, lens) -> int:
        """Unmasked keys read once, every probability written, lens read."""
        read = int(np.sum(np.minimum(lens, self.keys))) * self.heads * F32
        return read + self.batch * self.heads * self.keys * F32 + self.batch * 4

    def bytes_softmax_full(self) -> int:
        return 2 * self.batch * self.heads * self.keys * F32 + self.batch * 4

    def bytes_argmax(self) -> int:
        return self.logit_rows * self.vocab * F32 + self.logit_rows * 4


# ---- C4 -----------------------------------------------------------------------
@dataclass
class C4:
    tokens: int = 4096
    q_heads: int = NQ
    k_heads: int = NKV
    head_dim: int = HEAD_DIM
    theta: float = 1e6
    seed: int = 3

    def inputs(self):
        rng = np.random.default_rng(self.seed)
        q = f32_to_bf16_bits(rng.standard_normal((self.tokens, self.q_heads, self.head_dim),
                                                  dtype=np.float32))
        k = f32_to_bf16_bits(rng.standard_normal((self.tokens, self.k_heads, self.head_dim),
                                                  dtype=np.float32))
        return q, k

    def bytes(self) -> int:
        qk = self.tokens * (self.q_heads + self.k_heads) * self.head_dim * BF16
        tables = 2 * self.tokens * (self.head_dim // 2) * F32
        return 2 * qk + tables


# ---- C5 -----------------------------------------------------------------------
@dataclass
class C5:
    seqs: int = 64
    seq_len: int = 2048
    hidden: int = HIDDEN
    inter: int = INTER
    q_heads: int = NQ
    k_heads: int = NKV
    head_dim: int = HEAD_DIM
    vocab: int = VOCAB
    theta: float = 1e6
    eps: float = 1e-5
    seed: int = 4

    @property
    def rows(self) -> int:
        return self.seqs * self.seq_len

    def step_bytes(self) -> dict:
        """Algorithmic bytes of each op of one chain step (bf16 tensors)."""
        R, H, I = self.rows, self.hidden, self.inter
        T = self.seq_len
        s_rows = self.seqs * self.q_heads * T
        # causal: query i of a sequence reads keys 0..i
        causal_reads = self.seqs * self.q_heads * (T * (T + 1) // 2)
        return {
            "add_rms_norm": 4 * R * H * BF16 + H * BF16,
            "rope": 2 * R * (self.q_heads + self.k_heads) * self.head_dim * BF16
                    + 2 * T * (self.head_dim // 2) * F32,
            "softmax": causal_reads * BF16 + s_rows * T * BF16,
            "silu_mul": 3 * R * I * BF16,
            "add": 3 * R * H * BF16,
            "rms_norm": 2 * R * H * BF16 + H * BF16,
            "argmax": R * self.vocab * BF16 + R * 4,
            "sumsq": R * H * BF16 + 8,
        }

    def bytes(self) -> int:
        return sum(self.step_bytes().values())

    # Tensors of the chain, in generation order; each is produced one
    # sequence block at a time so that any sequence range is reproducible.
    TENSORS = ("x", "r", "q", "k", "scores", "gate", "up", "mlp", "logits")

    def block_shape(self, name: str, seqs: int) -> tuple:
        t = seqs * self.seq_len
        return {"x": (t, self.hidden), "r": (t, self.hidden), "mlp": (t, self.hidden),
                "q": (t, self.q_heads, self.head_dim), "k": (t, self.k_heads, self.head_dim),
                "scores": (seqs * self.q_heads * self.seq_len, self.seq_len),
                "gate": (t, self.inter), "up": (t, self.inter), "logits": (t, self.vocab)}[name]

    def block_seed(self, name: str, seq: int) -> int:
        """Seed of tensor `name`'s block for sequence `seq` (seed 4 of the config
        in the high bits): the chain's inputs for a range of sequences do not
        depend on how the 64 sequences are split across ranks."""
        return (self.seed << 40) | (self.TENSORS.index(name) << 20) | seq

    def device_inputs(self, seq_lo: int, seq_hi: int, device) -> dict:
        """bf16 N(0,1) inputs of sequences [seq_lo, seq_hi) on `device`, plus
        the norm weight w = 1.  Each sequence's block of each tensor comes from
        its own seeded torch generator, so the rows of sequence s are the same
        whether generated alone, in a rank's shard or in the whole batch."""
        import torch

        n = seq_hi - seq_lo
        if not 0 <= seq_lo <= seq_hi <= self.seqs:
            raise ValueError(f"sequence range [{seq_lo}, {seq_hi}) outside [0, {self.seqs})")
        out = {}
        g = torch.Generator(device=device)
        for name in self.TENSORS:
            t = torch.empty(self.block_shape(name, n), dtype=torch.bfloat16, device=device)
            per = t.shape[0] // max(n, 1)
            for i in range(n):
                g.manual_seed(self.block_seed(name, seq_lo + i))
                blk = t[i * per:(i + 1) * per]
                torch.randn(blk.shape, generator=g, out=blk)
            out[name] = t
        out["w"] = torch.ones(self.hidden, dtype=torch.bfloat16, device=device)
        return out
