"""numpy front end of the CPU oracle (oxide_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.  It
may be imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs,
never by the product package.  PARITY UNPINNED by reference outputs (the Rust
reference cannot be built); pinned by known-answer tests and an independent
numpy restatement (tests/test_oracle_kat.py, tests/test_oracle_numpy.py).

bf16 arrays are numpy uint16 holding raw bf16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_DIR, "liboxide_oracle.so")

ADD, SUB, MUL, DIV = 0, 1, 2, 3
RED_SUM, RED_MAX, RED_SUMSQ = 0, 1, 2

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", _DIR], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        h = C.CDLL(LIB_PATH)
        u64, i32, f32, vp = C.c_uint64, C.c_int, C.c_float, C.c_void_p
        sig = {
            "orc_binary_f32": [i32, vp, u64, vp, u64, vp, u64, i32],
            "orc_binary_bf16": [i32, vp, u64, vp, u64, vp, u64, i32],
            "orc_scale_f32": [vp, vp, f32, u64, i32],
            "orc_scale_bf16": [vp, vp, f32, u64, i32],
            "orc_silu_f32": [vp, vp, u64, i32],
            "orc_silu_bf16": [vp, vp, u64, i32],
            "orc_silu_mul_f32": [vp, vp, vp, u64, i32],
            "orc_silu_mul_bf16": [vp, vp, vp, u64, i32],
            "orc_rms_norm_f32": [vp, vp, vp, u64, u64, f32, i32],
            "orc_rms_norm_bf16": [vp, vp, vp, u64, u64, f32, i32],
            "orc_add_rms_norm_f32": [vp, vp, vp, vp, vp, u64, u64, f32, i32],
            "orc_add_rms_norm_bf16": [vp, vp, vp, vp, vp, u64, u64, f32, i32],
            "orc_softmax_f32": [vp, vp, u64, u64, u64, i32],
            "orc_softmax_bf16": [vp, vp, u64, u64, u64, i32],
            "orc_scale_mask_softmax_f32": [vp, vp, u64, u64, f32, vp, u64, vp, u64, u64, i32],
            "orc_scale_mask_softmax_bf16": [vp, vp, u64, u64, f32, vp, u64, vp, u64, u64, i32],
            "orc_rope_table_f32": [f32, u64, u64, vp, vp],
            "orc_rope_f32": [vp, vp, u64, u64, u64, i32, vp, vp, vp, i32],
            "orc_rope_bf16": [vp, vp, u64, u64, u64, i32, vp, vp, vp, i32],
            "orc_argmax_rows_f32": [vp, u64, u64, vp, i32],
            "orc_argmax_rows_bf16": [vp, u64, u64, vp, i32],
            "orc_reduce_rows_f32": [i32, vp, u64, u64, vp, i32],
            "orc_reduce_rows_bf16": [i32, vp, u64, u64, vp, i32],
            "orc_unary_f32": [i32, vp, vp, u64, f32, f32, i32],
            "orc_unary_bf16": [i32, vp, vp, u64, f32, f32, i32],
            "orc_layer_norm_f32": [vp, vp, vp, vp, u64, u64, f32, i32],
            "orc_layer_norm_bf16": [vp, vp, vp, vp, u64, u64, f32, i32],
            "orc_repeat_kv": [vp, vp, u64, u64, u64, u64, u64, u64],
            "orc_decode_attention_f32": [vp, vp, vp, vp, vp, u64, u64, u64, u64, u64, f32, i32],
            "orc_decode_attention_bf16": [vp, vp, vp, vp, vp, u64, u64, u64, u64, u64, f32, i32],
            "orc_decode_weights_f32": [vp, u64, i32, vp],
            "orc_decode_weights_bf16": [vp, u64, i32, vp],
            "orc_softmax_temperature_f32": [vp, u64, u64, f32, vp, i32],
            "orc_softmax_temperature_bf16": [vp, u64, u64, f32, vp, i32],
            "orc_sample_f32": [vp, u64, u64, f32, u64, f32, vp, vp, vp, i32],
            "orc_sample_bf16": [vp, u64, u64, f32, u64, f32, vp, vp, vp, i32],
        }
        for name, args in sig.items():
            fn = getattr(h, name)
            fn.argtypes = args
            fn.restype = None
        for name in ("orc_reduce_f32", "orc_reduce_bf16"):
            fn = getattr(h, name)
            fn.argtypes = [i32, vp, u64, i32]
            fn.restype = C.c_double
        h.orc_reduce_seq_f32.argtypes = [i32, vp, u64]
        h.orc_reduce_seq_f32.restype = C.c_float
        h.orc_max_threads.restype = i32
        h.orc_decode_f16_bits_f32.argtypes = [C.c_uint16]
        h.orc_decode_f16_bits_f32.restype = C.c_float
        h.orc_sample_probs.argtypes = [vp, u64, u64, f32, f32]
        h.orc_sample_probs.restype = C.c_uint32
        h.orc_kv_append.argtypes = [vp, vp, vp, vp, u64, u64, u64, u64, u64, u64, u64]
        h.orc_kv_append.restype = i32
        h.orc_f32_to_bf16.argtypes = [C.c_float]
        h.orc_f32_to_bf16.restype = C.c_uint16
        _lib = h
    return _lib


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ---- helpers ------------------------------------------------------------------
def _p(a):
    return None if a is None else a.ctypes.data


def _sfx(a: np.ndarray) -> str:
    if a.dtype == np.float32:
        return "f32"
    if a.dtype == np.uint16:
        return "bf16"
    raise TypeError(f"oracle arrays are float32 or uint16 (bf16 bits), got {a.dtype}")


def _c(a):
    return None if a is None else np.ascontiguousarray(a)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (numpy; NaN -> quiet NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- ops ----------------------------------------------------------------------
def binary(op, a, b, n=None, threads=1, out=None):
    a, b = _c(a), _c(b)
    n = max(a.size, b.size) if n is None else n
    out = np.empty(n, dtype=a.dtype) if out is None else out
    getattr(lib(), f"orc_binary_{_sfx(a)}")(op, _p(a), a.size, _p(b), b.size, _p(out), n, threads)
    return out


def scale(x, s, threads=1):
    x = _c(x)
    out = np.empty_like(x)
    getattr(lib(), f"orc_scale_{_sfx(x)}")(_p(x), _p(out), float(s), x.size, threads)
    return out


def silu(x, threads=1):
    x = _c(x)
    out = np.empty_like(x)
    getattr(lib(), f"orc_silu_{_sfx(x)}")(_p(x), _p(out), x.size, threads)
    return out


def silu_mul(g, u, threads=1, out=None):
    g, u = _c(g), _c(u)
    out = np.empty_like(g) if out is None else out
    getattr(lib(), f"orc_silu_mul_{_sfx(g)}")(_p(g), _p(u), _p(out), g.size, threads)
    return out


# unary op codes (oxide_unop in include/oxide_ops.h)
RELU, GELU, GELU_QUICK, SIGMOID, TANH, EXP, LOG, SQRT, POW, CLAMP, NEG, ABS = range(12)


def unary(op, x, a=0.0, b=0.0, threads=1):
    """src/ops/activation.rs / src/ops/math.rs unary ops; a = exponent (pow) or
    min (clamp), b = max (clamp)."""
    x = _c(x)
    out = np.empty_like(x)
    getattr(lib(), f"orc_unary_{_sfx(x)}")(op, _p(x), _p(out), x.size, float(a), float(b), threads)
    return out


def layer_norm(x, w, b, eps, threads=1):
    """src/ops/norm.rs:53-117 over the last dim of x."""
    x, w, b = _c(x), _c(w), _c(b)
    cols = w.size
    out = np.empty_like(x)
    getattr(lib(), f"orc_layer_norm_{_sfx(x)}")(_p(x), _p(w), _p(b), _p(out), x.size // cols, cols,
                                                float(eps), threads)
    return out


def repeat_kv(x, n_rep):
    """src/ops/attention.rs:161-201: x [b, h, s, d] -> [b, h * n_rep, s, d]."""
    x = _c(x)
    b, h, s, d = x.shape
    out = np.empty((b, h * n_rep, s, d), dtype=x.dtype)
    lib().orc_repeat_kv(_p(x), _p(out), b, h, s, d, n_rep, x.itemsize)
    return out


def kv_append(kc, vc, k, v, cur):
    """src/cache/kv_cache.rs:55-85 (in place); returns False on overflow."""
    b, h, m, d = kc.shape
    k, v = _c(k), _c(v)
    return lib().orc_kv_append(_p(kc), _p(vc), _p(k), _p(v), b, h, m, d, cur, k.shape[2], kc.itemsize) == 0


def decode_attention(q, kc, vc, lens=None, scale=None, threads=1):
    """src/ops/attention.rs:41-87 for one query token: q [b, hq, d], caches
    [b, hkv, max_seq, d], lens [b] int32 (None: every position)."""
    q, kc, vc = _c(q), _c(kc), _c(vc)
    b, hq, d = q.shape
    hkv, m = kc.shape[1], kc.shape[2]
    if scale is None:
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    lp = None if lens is None else _c(np.asarray(lens, np.int32))
    out = np.empty_like(q)
    getattr(lib(), f"orc_decode_attention_{_sfx(q)}")(_p(q), _p(kc), _p(vc), None if lp is None else _p(lp),
                                                      _p(out), b, hq, hkv, m, d, float(scale), threads)
    return out


SAMPLE_INVALID = 0xFFFFFFFF
WDT_F32, WDT_F16, WDT_BF16 = 0, 1, 2


def decode_weights(raw, dtype_code, out_bf16=False):
    """src/loading/safetensors.rs:48-82 element decode of little-endian bytes
    (a numpy uint8 array) -> f32 values (or bf16 bits with out_bf16)."""
    raw = _c(np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw)
    n = raw.size // (4 if dtype_code == WDT_F32 else 2)
    if out_bf16:
        out = np.empty(n, np.uint16)
        lib().orc_decode_weights_bf16(_p(raw), n, int(dtype_code), _p(out))
    else:
        out = np.empty(n, np.float32)
        lib().orc_decode_weights_f32(_p(raw), n, int(dtype_code), _p(out))
    return out


def softmax_with_temperature(logits, temperature, threads=1):
    """src/tokenizer.rs:166-180 on each row of logits [rows, vocab] (f32 or
    bf16 bits); returns f32 probabilities."""
    x = _c(logits)
    vocab = x.shape[-1]
    out = np.empty(x.shape, np.float32)
    getattr(lib(), f"orc_softmax_temperature_{_sfx(x)}")(_p(x), x.size // max(vocab, 1), vocab,
                                                          float(temperature), _p(out), threads)
    return out


def sample_probs(probs, top_k, top_p, u):
    """sample_top_p / sample_top_k (src/tokenizer.rs:182-232) on one row of
    probabilities with the uniform draw u."""
    p = _c(np.asarray(probs, np.float32))
    return int(lib().orc_sample_probs(_p(p), p.size, int(top_k), float(top_p), float(u)))


def sample(logits, temperature, top_k, top_p, uniforms, threads=1):
    """sample_next_token (src/pipeline.rs:181-205) per row of logits
    [rows, vocab]; returns (tokens uint32 [rows], probs f32 [rows, vocab])."""
    x = _c(logits)
    vocab = x.shape[-1]
    rows = x.size // max(vocab, 1)
    u = _c(np.asarray(uniforms, np.float32).reshape(rows))
    tok = np.empty(rows, np.uint32)
    probs = np.empty((rows, vocab), np.float32)
    getattr(lib(), f"orc_sample_{_sfx(x)}")(_p(x), rows, vocab, float(temperature), int(top_k), float(top_p),
                                             _p(u), _p(tok), _p(probs), threads)
    return tok, probs


def rms_norm(x, w, eps, threads=1, out=None):
    x, w = _c(x), _c(w)
    cols = w.size
    out = np.empty_like(x) if out is None else out
    getattr(lib(), f"orc_rms_norm_{_sfx(x)}")(_p(x), _p(w), _p(out), x.size // cols, cols,
                                              float(eps), threads)
    return out


def add_rms_norm(x, r, w, eps, threads=1, h=None, y=None):
    x, r, w = _c(x), _c(r), _c(w)
    cols = w.size
    h = np.empty_like(x) if h is None else h
    y = np.empty_like(x) if y is None else y
    getattr(lib(), f"orc_add_rms_norm_{_sfx(x)}")(_p(x), _p(r), _p(w), _p(h), _p(y),
                                                  x.size // cols, cols, float(eps), threads)
    return h, y


def softmax(x, outer, dim, inner, threads=1):
    x = _c(x)
    out = np.empty_like(x)
    getattr(lib(), f"orc_softmax_{_sfx(x)}")(_p(x), _p(out), outer, dim, inner, threads)
    return out


def scale_mask_softmax(x, cols, scale, mask=None, lens=None, rows_per_len=1, causal_q_len=0,
                       threads=1, out=None):
    x = _c(x)
    mask = None if mask is None else _c(np.asarray(mask, dtype=np.float32))
    lens = None if lens is None else _c(np.asarray(lens, dtype=np.int32))
    out = np.empty_like(x) if out is None else out
    getattr(lib(), f"orc_scale_mask_softmax_{_sfx(x)}")(
        _p(x), _p(out), x.size // cols, cols, float(scale), _p(mask),
        0 if mask is None else mask.size, _p(lens), rows_per_len, causal_q_len, threads)
    return out


def rope_table(theta, head_dim, max_pos):
    half = head_dim // 2
    cos = np.empty((max_pos, half), dtype=np.float32)
    sin = np.empty((max_pos, half), dtype=np.float32)
    lib().orc_rope_table_f32(float(theta), head_dim, max_pos, _p(cos), _p(sin))
    return cos, sin


def rope(x, tokens, heads, head_dim, layout, cos, sin, positions=None, threads=1, out=None):
    x = _c(x)
    cos, sin = _c(cos), _c(sin)
    positions = None if positions is None else _c(np.asarray(positions, dtype=np.int32))
    out = np.empty_like(x) if out is None else out
    getattr(lib(), f"orc_rope_{_sfx(x)}")(_p(x), _p(out), tokens, heads, head_dim, layout,
                                          _p(cos), _p(sin), _p(positions), threads)
    return out


def argmax_rows(x, cols, threads=1, out=None):
    x = _c(x)
    rows = x.size // cols
    idx = np.empty(rows, dtype=np.uint32) if out is None else out
    getattr(lib(), f"orc_argmax_rows_{_sfx(x)}")(_p(x), rows, cols, _p(idx), threads)
    return idx


def reduce_rows(op, x, cols, threads=1):
    x = _c(x)
    rows = x.size // cols
    out = np.empty(rows, dtype=np.float32)
    getattr(lib(), f"orc_reduce_rows_{_sfx(x)}")(op, _p(x), rows, cols, _p(out), threads)
    return out


def reduce(op, x, threads=1) -> float:
    x = _c(x)
    return float(getattr(lib(), f"orc_reduce_{_sfx(x)}")(op, _p(x), x.size, threads))


def reduce_seq_f32(op, x) -> float:
    x = _c(np.asarray(x, dtype=np.float32))
    return float(lib().orc_reduce_seq_f32(op, _p(x), x.size))
