"""Host-buffer ops: the library's pipelined oxide_pipe_* entry points on numpy
arrays.

A :class:`Pipe` owns device staging buffers on one GPU (allocated once by
``oxide_pipe_create``).  Each op uploads its host inputs chunk by chunk, runs
the same kernels as :mod:`oxide_b200.ops` on each chunk and downloads the
result while the next chunk uploads, so the results are bit-identical to the
device-tensor ops.  Arrays are C-contiguous numpy arrays: ``float32`` for the
f32 forms, ``uint16`` holding bf16 bit patterns for the bf16 forms.  The
copies overlap only when the host memory is page-locked (numpy views of
pinned torch tensors, ``torch.empty(..., pin_memory=True).numpy()``).

In deferred mode (``with pipe.deferred():``) the calls return once their work
is enqueued, so one op's uploads overlap the previous op's downloads; the
block's exit waits for everything, and host arrays must stay alive and
outputs unread until then.

Each method follows one reference call: ``add``/``mul_rowbcast`` the
broadcasting binary ops (src/ops/matmul.rs:74-108), ``silu_mul`` the MLP gate
(src/layers/attention.rs:144-145), ``rms_norm``/``add_rms_norm`` the transformer block's
norms (src/layers/transformer.rs:64-67), ``scale_mask_softmax`` the attention
scores (src/ops/attention.rs:41-79), ``argmax_rows`` greedy sampling and
``rope_bf16`` apply_rotary_emb (src/ops/attention.rs:96-159).
"""
from __future__ import annotations

import contextlib
import ctypes as C

import numpy as np

from ._lib import ADD, DIV, MUL, SUB, call

_BINARY = {"add": ADD, "sub": SUB, "mul": MUL, "div": DIV}


def _arr(name: str, a, dtype) -> np.ndarray:
    if not isinstance(a, np.ndarray):
        raise TypeError(f"{name}: expected a numpy array, got {type(a).__name__}")
    if a.dtype != dtype:
        raise TypeError(f"{name}: expected dtype {np.dtype(dtype)}, got {a.dtype}")
    if not a.flags.c_contiguous:
        raise ValueError(f"{name}: must be C-contiguous")
    return a


def _out(name: str, out, shape, dtype) -> np.ndarray:
    if out is None:
        return np.empty(shape, dtype)
    _arr(name, out, dtype)
    if out.shape != tuple(shape):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {out.shape}")
    if not out.flags.writeable:
        raise ValueError(f"{name}: must be writeable")
    return out


def _rows_cols(name: str, a: np.ndarray) -> tuple[int, int]:
    if a.ndim < 1 or a.shape[-1] == 0:
        raise ValueError(f"{name}: needs a non-empty last dimension")
    cols = a.shape[-1]
    return a.size // cols, cols


def _p(a) -> int | None:
    return None if a is None else a.ctypes.data


class Pipe:
    """Pipelined host-buffer ops on GPU ``device``: ``chunk_bytes`` per staged
    chunk, ``depth`` chunks in flight."""

    def __init__(self, device: int = 0, chunk_bytes: int = 16 << 20, depth: int = 4):
        self._h = C.c_void_p()
        call("oxide_pipe_create", int(device), int(chunk_bytes), int(depth), C.byref(self._h))
        self._keep: list = []  # host arrays referenced by work enqueued in deferred mode
        self._deferred = False

    @property
    def handle(self) -> C.c_void_p:
        if not self._h:
            raise ValueError("pipe is closed")
        return self._h

    def close(self) -> None:
        if self._h:
            call("oxide_pipe_destroy", self._h)
            self._h = C.c_void_p()
            self._keep.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- deferred mode ---------------------------------------------------------------
    def sync(self) -> None:
        """Wait for every enqueued op; outputs are then readable."""
        call("oxide_pipe_sync", self.handle)
        self._keep.clear()

    @contextlib.contextmanager
    def deferred(self):
        """Ops inside the block overlap one another; the exit waits for all."""
        call("oxide_pipe_defer", self.handle, 1)
        self._deferred = True
        try:
            yield self
        finally:
            self._deferred = False
            call("oxide_pipe_defer", self.handle, 0)
            self._keep.clear()

    def _run(self, name: str, arrays, *args):
        call(name, self.handle, *args)
        if self._deferred:
            self._keep.extend(a for a in arrays if a is not None)

    # -- ops ----------------------------------------------------------------------------
    def binary(self, op: str, a, b, out=None) -> np.ndarray:
        """out = a (op) b, f32; b has a's size or a size dividing it (broadcast
        over a's trailing elements, one value per column for a row vector)."""
        if op not in _BINARY:
            raise ValueError(f"binary: op must be one of {sorted(_BINARY)}")
        a = _arr("a", a, np.float32)
        b = _arr("b", b, np.float32)
        out = _out("out", out, a.shape, np.float32)
        self._run("oxide_pipe_binary_f32", (a, b, out), _BINARY[op], a.ctypes.data, a.size, b.ctypes.data, b.size,
                  out.ctypes.data, out.size)
        return out

    def add(self, a, b, out=None) -> np.ndarray:
        return self.binary("add", a, b, out)

    def mul_rowbcast(self, a, s, out=None) -> np.ndarray:
        """out[r, c] = a[r, c] * s[c]."""
        a = _arr("a", a, np.float32)
        if s.shape != (a.shape[-1],):
            raise ValueError(f"mul_rowbcast: s must have shape ({a.shape[-1]},), got {s.shape}")
        return self.binary("mul", a, s, out)

    def add_mul_rowbcast(self, a, b, s, h=None, y=None) -> tuple[np.ndarray, np.ndarray]:
        """h = a + b and y = h * s[col], one upload of a, b and s."""
        a = _arr("a", a, np.float32)
        b = _arr("b", b, np.float32)
        s = _arr("s", s, np.float32)
        rows, cols = _rows_cols("a", a)
        if b.shape != a.shape or s.shape != (cols,):
            raise ValueError("add_mul_rowbcast: b must match a and s must be one value per column")
        h = _out("h", h, a.shape, np.float32)
        y = _out("y", y, a.shape, np.float32)
        self._run("oxide_pipe_add_mul_rowbcast_f32", (a, b, s, h, y), a.ctypes.data, b.ctypes.data, s.ctypes.data,
                  h.ctypes.data, y.ctypes.data, rows, cols)
        return h, y

    def silu_mul(self, gate, up, out=None) -> np.ndarray:
        """out = silu(gate) * up, f32."""
        gate = _arr("gate", gate, np.float32)
        up = _arr("up", up, np.float32)
        if up.shape != gate.shape:
            raise ValueError("silu_mul: gate and up must have the same shape")
        out = _out("out", out, gate.shape, np.float32)
        self._run("oxide_pipe_silu_mul_f32", (gate, up, out), gate.ctypes.data, up.ctypes.data, out.ctypes.data,
                  gate.size)
        return out

    def rms_norm(self, x, w, eps: float, out=None) -> np.ndarray:
        """RMSNorm of each row of x (f32) with weight w [cols]."""
        x = _arr("x", x, np.float32)
        w = _arr("w", w, np.float32)
        rows, cols = _rows_cols("x", x)
        if w.shape != (cols,):
            raise ValueError(f"rms_norm: w must have shape ({cols},)")
        out = _out("out", out, x.shape, np.float32)
        self._run("oxide_pipe_rms_norm_f32", (x, w, out), x.ctypes.data, w.ctypes.data, out.ctypes.data, rows, cols,
                  float(eps))
        return out

    def add_rms_norm(self, x, r, w, eps: float, h=None, y=None) -> tuple[np.ndarray, np.ndarray]:
        """h = x + r and y = rms_norm(h) * w; f32, or bf16 as uint16 arrays."""
        dt = np.uint16 if isinstance(x, np.ndarray) and x.dtype == np.uint16 else np.float32
        x = _arr("x", x, dt)
        r = _arr("r", r, dt)
        w = _arr("w", w, dt)
        rows, cols = _rows_cols("x", x)
        if r.shape != x.shape or w.shape != (cols,):
            raise ValueError("add_rms_norm: r must match x and w must be one value per column")
        h = _out("h", h, x.shape, dt)
        y = _out("y", y, x.shape, dt)
        name = "oxide_pipe_add_rms_norm_f32" if dt == np.float32 else "oxide_pipe_add_rms_norm_bf16"
        self._run(name, (x, r, w, h, y), x.ctypes.data, r.ctypes.data, w.ctypes.data, h.ctypes.data, y.ctypes.data,
                  rows, cols, float(eps))
        return h, y

    def scale_mask_softmax(self, x, scale: float, mask=None, lens=None, rows_per_len: int = 1,
                           causal_q_len: int = 0, out=None) -> np.ndarray:
        """softmax(x * scale + mask) per row (f32).  mask: f32 added cyclically
        (its length divides the element count); lens: int32 key counts, one
        per rows_per_len rows (keys past a row's count get probability 0);
        causal_q_len > 0: causal mask for blocks of that many query rows."""
        x = _arr("x", x, np.float32)
        rows, cols = _rows_cols("x", x)
        if mask is not None:
            mask = _arr("mask", mask, np.float32)
        if lens is not None:
            lens = _arr("lens", lens, np.int32)
            if rows_per_len <= 0 or lens.size * rows_per_len != rows:
                raise ValueError("scale_mask_softmax: lens needs one count per rows_per_len rows")
        out = _out("out", out, x.shape, np.float32)
        self._run("oxide_pipe_scale_mask_softmax_f32", (x, out, mask, lens), x.ctypes.data, out.ctypes.data, rows,
                  cols, float(scale), _p(mask), 0 if mask is None else mask.size, _p(lens),
                  rows_per_len if lens is not None else 0, int(causal_q_len))
        return out

    def argmax_rows(self, x, out=None) -> np.ndarray:
        """Index of the first maximum of each row (f32), as uint32."""
        x = _arr("x", x, np.float32)
        rows, cols = _rows_cols("x", x)
        out = _out("idx", out, (rows,), np.uint32)
        self._run("oxide_pipe_argmax_rows_f32", (x, out), x.ctypes.data, rows, cols, out.ctypes.data)
        return out

    def rope_bf16(self, q, cos, sin, k=None, positions=None, q_out=None, k_out=None):
        """Rotary embedding of q [tokens, q_heads, head_dim] (and k
        [tokens, k_heads, head_dim]) in bf16 (uint16 arrays), with cos/sin
        tables [table_rows, head_dim/2] f32 indexed by positions (int32, one per
        token; None: position = token index).  Outputs may be the inputs."""
        q = _arr("q", q, np.uint16)
        if q.ndim != 3:
            raise ValueError("rope_bf16: q must be [tokens, heads, head_dim]")
        tokens, qh, d = q.shape
        cos = _arr("cos", cos, np.float32)
        sin = _arr("sin", sin, np.float32)
        if cos.ndim != 2 or cos.shape[1] * 2 != d or sin.shape != cos.shape:
            raise ValueError("rope_bf16: cos and sin must be [table_rows, head_dim / 2]")
        kh = 0
        if k is not None:
            k = _arr("k", k, np.uint16)
            if k.ndim != 3 or k.shape[0] != tokens or k.shape[2] != d:
                raise ValueError("rope_bf16: k must be [tokens, k_heads, head_dim]")
            kh = k.shape[1]
            k_out = _out("k_out", k_out, k.shape, np.uint16)
        if positions is not None:
            positions = _arr("positions", positions, np.int32)
            if positions.shape != (tokens,):
                raise ValueError("rope_bf16: positions needs one entry per token")
        q_out = _out("q_out", q_out, q.shape, np.uint16)
        self._run("oxide_pipe_rope_bf16", (q, q_out, k, k_out, cos, sin, positions), q.ctypes.data,
                  q_out.ctypes.data, qh, _p(k), _p(k_out), kh, cos.ctypes.data, sin.ctypes.data, cos.shape[0],
                  _p(positions), tokens, d)
        return (q_out, k_out) if k is not None else q_out
