"""Tensor-level ops over the C ABI, named after mistralrs-oxide's ``src/ops``.

Each function mirrors a reference free function (``fn(&Tensor, ...) ->
OxideResult<Tensor>``): inputs are borrowed, a new output is allocated and
returned, and invalid shapes raise (``OxideError`` with status
OXIDE_ERR_INVALID_ARG, like ``OxideError::InvalidArgument``).  Tensors must be
contiguous CUDA tensors of dtype float32 or bfloat16; work runs on the current
torch CUDA stream.  PyTorch only supplies device memory and the stream: every
op is one call into liboxide_b200.so.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import ADD, DIV, MUL, RED_MAX, RED_SUM, RED_SUMSQ, SUB, OxideError, call

_SFX = {torch.float32: "f32", torch.bfloat16: "bf16"}


def _sfx(t: torch.Tensor) -> str:
    if t.dtype not in _SFX:
        raise OxideError(_lib.ERR_UNSUPPORTED, "oxide", f"dtype {t.dtype} is not float32/bfloat16")
    return _SFX[t.dtype]


def _check(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise OxideError(_lib.ERR_INVALID_ARG, "oxide", "tensor is not on a CUDA device")
        if not t.is_contiguous():
            raise OxideError(_lib.ERR_INVALID_ARG, "oxide", "tensor is not contiguous")


def _need(cond: bool, op: str, msg: str) -> None:
    if not cond:
        raise OxideError(_lib.ERR_INVALID_ARG, op, msg)


def _same_dtype(op: str, ref: torch.Tensor, **named: Optional[torch.Tensor]) -> None:
    """Every named operand has ref's dtype: the kernels size their reads by
    the input's element type, so a narrower operand would be over-read."""
    for name, t in named.items():
        if t is not None:
            _need(t.dtype == ref.dtype, op, f"{name} dtype {t.dtype} differs from the input's {ref.dtype}")


def _out_like(op: str, ref: torch.Tensor, **named: Optional[torch.Tensor]) -> None:
    """A caller-given output holds exactly ref's element count in ref's dtype."""
    for name, t in named.items():
        if t is not None:
            _need(t.dtype == ref.dtype and t.numel() == ref.numel(), op,
                  f"{name} must be {ref.dtype} with {ref.numel()} elements, got {t.dtype} with {t.numel()}")


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def broadcast_shape(a: Sequence[int], b: Sequence[int]) -> list[int]:
    """Output shape of a binary op; src/ops/matmul.rs:160-177."""
    out = []
    for i in range(max(len(a), len(b))):
        da = a[len(a) - 1 - i] if i < len(a) else 1
        db = b[len(b) - 1 - i] if i < len(b) else 1
        if da != db and da != 1 and db != 1:
            raise OxideError(_lib.ERR_INVALID_ARG, "broadcast",
                             f"shape mismatch {list(a)} and {list(b)}")
        out.append(max(da, db))
    return out[::-1]


def binary(op: int, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """out[i] = a[i % a.numel()] op b[i % b.numel()] (src/ops/matmul.rs:136-158)."""
    _check(a, b)
    if a.dtype != b.dtype:
        raise OxideError(_lib.ERR_INVALID_ARG, "binary", "operand dtypes differ")
    out = torch.empty(broadcast_shape(a.shape, b.shape), dtype=a.dtype, device=a.device)
    call(f"oxide_binary_{_sfx(a)}", op, _p(a), a.numel(), _p(b), b.numel(), _p(out), out.numel(),
         _stream())
    return out


def add(a, b):  # src/ops/matmul.rs:74
    return binary(ADD, a, b)


def sub(a, b):  # src/ops/matmul.rs:110
    return binary(SUB, a, b)


def mul(a, b):  # src/ops/matmul.rs:97
    return binary(MUL, a, b)


def div(a, b):  # src/ops/matmul.rs:123
    return binary(DIV, a, b)


def mul_rowbcast(x: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """x[rows, cols] * s[cols] (ops::mul with a trailing-dim broadcast)."""
    cols = s.numel()
    _same_dtype("mul_rowbcast", x, s=s)
    _need(x.dim() >= 1 and cols >= 1 and x.shape[-1] == cols, "mul_rowbcast",
          f"broadcast operand of {cols} elements doesn't match the last dim of {list(x.shape)}")
    _check(x, s)
    out = torch.empty_like(x)
    call(f"oxide_mul_rowbcast_{_sfx(x)}", _p(x), _p(s), _p(out), x.numel() // cols, cols, _stream())
    return out


def add_mul_rowbcast(a: torch.Tensor, b: torch.Tensor, s: torch.Tensor,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(a + b)[rows, cols] * s[cols] in one pass: ops::add then ops::mul with a
    trailing-dim broadcast (src/ops/matmul.rs:74-108), the sum rounded to a's
    dtype first and not stored.  out may be a or b (in place), not s."""
    if b.shape != a.shape or b.dtype != a.dtype or s.dtype != a.dtype:
        raise OxideError(_lib.ERR_INVALID_ARG, "add_mul_rowbcast", "operands must share shape and dtype")
    cols = s.numel()
    if a.dim() < 1 or a.shape[-1] != cols:
        raise OxideError(_lib.ERR_INVALID_ARG, "add_mul_rowbcast",
                         f"broadcast operand of {cols} elements doesn't match the last dim of {list(a.shape)}")
    _out_like("add_mul_rowbcast", a, out=out)
    _need(out is None or out.data_ptr() != s.data_ptr(), "add_mul_rowbcast", "out must not alias s")
    _check(a, b, s, out)
    out = torch.empty_like(a) if out is None else out
    call(f"oxide_add_mul_rowbcast_{_sfx(a)}", _p(a), _p(b), _p(s), _p(out), a.numel() // cols, cols, _stream())
    return out


def scale(x: torch.Tensor, s: float) -> torch.Tensor:
    """x * s (KernelManager::launch_scale, src/cuda_backend/kernels.rs:159)."""
    _check(x)
    out = torch.empty_like(x)
    call(f"oxide_scale_{_sfx(x)}", _p(x), _p(out), float(s), x.numel(), _stream())
    return out


def silu(x: torch.Tensor) -> torch.Tensor:
    """src/ops/activation.rs:21-37."""
    _check(x)
    out = torch.empty_like(x)
    call(f"oxide_silu_{_sfx(x)}", _p(x), _p(out), x.numel(), _stream())
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mul(silu(gate), up) in one pass (src/layers/attention.rs:144-145)."""
    if gate.shape != up.shape:
        raise OxideError(_lib.ERR_INVALID_ARG, "silu_mul", "gate and up shapes differ")
    _same_dtype("silu_mul", gate, up=up)
    _out_like("silu_mul", gate, out=out)
    _check(gate, up, out)
    out = torch.empty_like(gate) if out is None else out
    call(f"oxide_silu_mul_{_sfx(gate)}", _p(gate), _p(up), _p(out), gate.numel(), _stream())
    return out


def unary(op: int, x: torch.Tensor, a: float = 0.0, b: float = 0.0,
          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = op(x) elementwise (oxide_unop: src/ops/activation.rs, src/ops/math.rs)."""
    _out_like("unary", x, out=out)
    _check(x, out)
    out = torch.empty_like(x) if out is None else out
    call(f"oxide_unary_{_sfx(x)}", op, _p(x), _p(out), x.numel(), float(a), float(b), _stream())
    return out


def relu(x):  # src/ops/activation.rs:4-19
    return unary(_lib.RELU, x)


def gelu(x):  # src/ops/activation.rs:39-56 (tanh approximation)
    return unary(_lib.GELU, x)


def gelu_quick(x):  # src/ops/activation.rs:58-74
    return unary(_lib.GELU_QUICK, x)


def sigmoid(x):  # src/ops/activation.rs:126-140
    return unary(_lib.SIGMOID, x)


def tanh(x):  # src/ops/activation.rs:142-156
    return unary(_lib.TANH, x)


def exp(x):  # src/ops/math.rs:4-19
    return unary(_lib.EXP, x)


def log(x):  # src/ops/math.rs:21-36 (natural log)
    return unary(_lib.LOG, x)


def sqrt(x):  # src/ops/math.rs:38-53
    return unary(_lib.SQRT, x)


def pow(x, n: float):  # src/ops/math.rs:55-70
    return unary(_lib.POW, x, n)


def clamp(x, lo: float, hi: float):  # src/ops/math.rs:72-87
    return unary(_lib.CLAMP, x, lo, hi)


def neg(x):  # src/ops/math.rs:89-104
    return unary(_lib.NEG, x)


def abs(x):  # src/ops/math.rs:106-121
    return unary(_lib.ABS, x)


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """src/ops/norm.rs:53-117."""
    _same_dtype("layer_norm", x, weight=w, bias=b)
    _out_like("layer_norm", x, out=out)
    _check(x, w, b, out)
    if x.dim() < 1:
        raise OxideError(_lib.ERR_INVALID_ARG, "layer_norm", "layer_norm requires at least 1D tensor")
    cols = x.shape[-1]
    if w.dim() != 1 or w.shape[0] != cols:
        raise OxideError(_lib.ERR_INVALID_ARG, "layer_norm",
                         f"layer_norm weight shape {list(w.shape)} doesn't match input last dim {cols}")
    if b.dim() != 1 or b.shape[0] != cols:
        raise OxideError(_lib.ERR_INVALID_ARG, "layer_norm",
                         f"layer_norm bias shape {list(b.shape)} doesn't match input last dim {cols}")
    out = torch.empty_like(x) if out is None else out
    call(f"oxide_layer_norm_{_sfx(x)}", _p(x), _p(w), _p(b), _p(out), x.numel() // cols, cols,
         float(eps), _stream())
    return out


def add_layer_norm(x: torch.Tensor, r: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """layer_norm(x + r): the fused add + layer_norm of src/kernels/normalization.rs:123-167
    (the sum rounded to x's dtype first, not stored)."""
    if r.shape != x.shape or r.dtype != x.dtype:
        raise OxideError(_lib.ERR_INVALID_ARG, "add_layer_norm", "residual must match the input's shape and dtype")
    _same_dtype("add_layer_norm", x, weight=w, bias=b)
    _out_like("add_layer_norm", x, out=out)
    _check(x, r, w, b, out)
    if x.dim() < 1:
        raise OxideError(_lib.ERR_INVALID_ARG, "add_layer_norm", "layer_norm requires at least 1D tensor")
    cols = x.shape[-1]
    if w.dim() != 1 or w.shape[0] != cols:
        raise OxideError(_lib.ERR_INVALID_ARG, "add_layer_norm",
                         f"layer_norm weight shape {list(w.shape)} doesn't match input last dim {cols}")
    if b.dim() != 1 or b.shape[0] != cols:
        raise OxideError(_lib.ERR_INVALID_ARG, "add_layer_norm",
                         f"layer_norm bias shape {list(b.shape)} doesn't match input last dim {cols}")
    out = torch.empty_like(x) if out is None else out
    call(f"oxide_add_layer_norm_{_sfx(x)}", _p(x), _p(r), _p(w), _p(b), _p(out), x.numel() // cols, cols,
         float(eps), _stream())
    return out


def _norm_check(x: torch.Tensor, w: torch.Tensor) -> int:
    if x.dim() < 1:
        raise OxideError(_lib.ERR_INVALID_ARG, "rms_norm", "rms_norm requires at least 1D tensor")
    if w.dim() != 1 or w.shape[0] != x.shape[-1]:
        raise OxideError(_lib.ERR_INVALID_ARG, "rms_norm",
                         f"rms_norm weight shape {list(w.shape)} doesn't match input last dim {x.shape[-1]}")
    _same_dtype("rms_norm", x, weight=w)
    return x.shape[-1]


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """src/ops/norm.rs:4-51."""
    cols = _norm_check(x, w)
    _out_like("rms_norm", x, out=out)
    _check(x, w, out)
    out = torch.empty_like(x) if out is None else out
    call(f"oxide_rms_norm_{_sfx(x)}", _p(x), _p(w), _p(out), x.numel() // cols, cols, float(eps),
         _stream())
    return out


def add_rms_norm(x: torch.Tensor, r: torch.Tensor, w: torch.Tensor, eps: float,
                 h: Optional[torch.Tensor] = None, y: Optional[torch.Tensor] = None):
    """(h, y) with h = x + r and y = rms_norm(h) (src/layers/transformer.rs:64-67)."""
    cols = _norm_check(x, w)
    _need(r.shape == x.shape and r.dtype == x.dtype, "add_rms_norm",
          "residual must match the input's shape and dtype")
    _out_like("add_rms_norm", x, h=h, y=y)
    _need(h is None or y is None or h.data_ptr() != y.data_ptr(), "add_rms_norm", "h and y must not alias")
    _check(x, r, w, h, y)
    h = torch.empty_like(x) if h is None else h
    y = torch.empty_like(x) if y is None else y
    call(f"oxide_add_rms_norm_{_sfx(x)}", _p(x), _p(r), _p(w), _p(h), _p(y), x.numel() // cols, cols,
         float(eps), _stream())
    return h, y


def softmax(x: torch.Tensor, dim: int) -> torch.Tensor:
    """softmax along `dim` (src/ops/activation.rs:76-124)."""
    _check(x)
    if dim >= x.dim() or dim < 0:
        raise OxideError(_lib.ERR_INVALID_ARG, "softmax",
                         f"softmax dim {dim} out of range for rank {x.dim()}")
    outer = 1
    for d in x.shape[:dim]:
        outer *= d
    inner = 1
    for d in x.shape[dim + 1:]:
        inner *= d
    out = torch.empty_like(x)
    call(f"oxide_softmax_{_sfx(x)}", _p(x), _p(out), outer, x.shape[dim], inner, _stream())
    return out


def scale_mask_softmax(x: torch.Tensor, scale: float, mask: Optional[torch.Tensor] = None,
                       lens: Optional[torch.Tensor] = None, rows_per_len: int = 1,
                       causal_q_len: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(x * scale + mask) over the last dim (src/ops/attention.rs:41,60,63-79).

    ``mask`` (f32) is added as mask[j % mask.numel()]; ``lens`` (int32, one per
    group of ``rows_per_len`` rows) and ``causal_q_len`` cut each row's valid
    length; keys beyond it are 0."""
    if mask is not None and mask.dtype != torch.float32:
        raise OxideError(_lib.ERR_INVALID_ARG, "scale_mask_softmax", "mask must be float32")
    if lens is not None and lens.dtype != torch.int32:
        raise OxideError(_lib.ERR_INVALID_ARG, "scale_mask_softmax", "lens must be int32")
    _need(x.dim() >= 1, "scale_mask_softmax", "scores need at least one dim")
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    if lens is not None:
        _need(rows_per_len >= 1 and lens.numel() >= -(-rows // rows_per_len), "scale_mask_softmax",
              f"lens needs one entry per {rows_per_len} rows ({-(-rows // max(1, rows_per_len))}), "
              f"got {lens.numel()}")
    _out_like("scale_mask_softmax", x, out=out)
    _check(x, mask, lens, out)
    out = torch.empty_like(x) if out is None else out
    call(f"oxide_scale_mask_softmax_{_sfx(x)}", _p(x), _p(out), x.numel() // cols, cols,
         float(scale), _p(mask), 0 if mask is None else mask.numel(), _p(lens), rows_per_len,
         causal_q_len, _stream())
    return out


def rope_table(theta: float, head_dim: int, max_pos: int):
    """(cos, sin) f32 tables [max_pos, head_dim/2] (src/models/mistral.rs:91-115), on the host."""
    half = head_dim // 2
    cos = torch.empty((max_pos, half), dtype=torch.float32)
    sin = torch.empty((max_pos, half), dtype=torch.float32)
    call("oxide_rope_table_host_f32", float(theta), head_dim, max_pos, cos.data_ptr(), sin.data_ptr())
    return cos, sin


def rope(q: torch.Tensor, k: Optional[torch.Tensor], cos: torch.Tensor, sin: torch.Tensor,
         positions: Optional[torch.Tensor] = None, layout: str = "token",
         q_out: Optional[torch.Tensor] = None, k_out: Optional[torch.Tensor] = None):
    """Rotate-half RoPE of q (and k) in one launch (src/ops/attention.rs:139-155).

    layout "token": [tokens, heads, head_dim]; "head": [heads, tokens, head_dim]
    (any leading dims fold into heads).  Pass q_out=q / k_out=k for in-place."""
    _same_dtype("rope", q, k=k)
    _out_like("rope", q, q_out=q_out)
    if k is not None:
        _out_like("rope", k, k_out=k_out)
    _need(cos.dtype == torch.float32 and sin.dtype == torch.float32, "rope", "cos/sin tables must be float32")
    _check(q, k, cos, sin, positions, q_out, k_out)
    head_dim = q.shape[-1]
    if layout == "token":
        tokens, qh = q.shape[0], q.numel() // (q.shape[0] * head_dim)
        kh = 0 if k is None else k.numel() // (k.shape[0] * head_dim)
        lay = 0
    elif layout == "head":
        tokens = q.shape[-2]
        qh = q.numel() // (tokens * head_dim)
        kh = 0 if k is None else k.numel() // (tokens * head_dim)
        lay = 1
    else:
        raise OxideError(_lib.ERR_INVALID_ARG, "rope", f"unknown layout {layout!r}")
    if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] != head_dim // 2:
        raise OxideError(_lib.ERR_INVALID_ARG, "rope",
                         f"cos/sin shape {list(cos.shape)} doesn't match [*, {head_dim // 2}]")
    if positions is not None and positions.dtype != torch.int32:
        raise OxideError(_lib.ERR_INVALID_ARG, "rope", "positions must be int32")
    _need(positions is None or positions.numel() >= tokens, "rope",
          f"positions needs {tokens} entries, got {0 if positions is None else positions.numel()}")
    q_out = torch.empty_like(q) if q_out is None else q_out
    if k is not None:
        k_out = torch.empty_like(k) if k_out is None else k_out
    call(f"oxide_rope_{_sfx(q)}", _p(q), _p(q_out), qh, _p(k), _p(k_out) if k is not None else None,
         kh, _p(cos), _p(sin), cos.shape[0], _p(positions), tokens, head_dim, lay, _stream())
    return (q_out, k_out) if k is not None else q_out


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """src/ops/attention.rs:96-159: x [..., seq_len, head_dim], cos/sin [seq_len, half]."""
    if x.dim() < 3:
        raise OxideError(_lib.ERR_INVALID_ARG, "apply_rotary_emb",
                         "apply_rotary_emb requires at least 3D tensor")
    seq_len, head_dim = x.shape[-2], x.shape[-1]
    if list(cos.shape) != [seq_len, head_dim // 2] or list(sin.shape) != [seq_len, head_dim // 2]:
        raise OxideError(_lib.ERR_INVALID_ARG, "apply_rotary_emb",
                         f"cos shape {list(cos.shape)} doesn't match expected {[seq_len, head_dim // 2]}")
    return rope(x, None, cos, sin, layout="head")


def argmax(x: torch.Tensor) -> torch.Tensor:
    """Row argmax over the last dim -> int32 indices (lowest index on ties)."""
    _check(x)
    cols = x.shape[-1]
    idx = torch.empty(x.shape[:-1], dtype=torch.int32, device=x.device)
    call(f"oxide_argmax_rows_{_sfx(x)}", _p(x), x.numel() // cols, cols, _p(idx), _stream())
    return idx


def reduce_rows(x: torch.Tensor, op: int) -> torch.Tensor:
    """Per-row sum / max / sum of squares over the last dim -> f32."""
    _check(x)
    cols = x.shape[-1]
    out = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    call(f"oxide_reduce_rows_{_sfx(x)}", op, _p(x), x.numel() // cols, cols, _p(out), _stream())
    return out


def workspace_bytes(n: int) -> int:
    return int(_lib.lib().oxide_reduce_workspace_bytes(n))


def reduce(x: torch.Tensor, op: int, workspace: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Whole-tensor sum / max / sum of squares -> f64 scalar tensor on the device."""
    n = x.numel()
    _need(workspace is None or workspace.numel() * workspace.element_size() >= workspace_bytes(n), "reduce",
          f"workspace must hold {workspace_bytes(n)} bytes")
    _need(out is None or (out.dtype == torch.float64 and out.numel() == 1), "reduce",
          "out must be one float64 element")
    _check(x, workspace, out)
    if workspace is None:
        workspace = torch.empty(workspace_bytes(n), dtype=torch.uint8, device=x.device)
    out = torch.empty((), dtype=torch.float64, device=x.device) if out is None else out
    call(f"oxide_reduce_{_sfx(x)}", op, _p(x), n, _p(out), _p(workspace),
         workspace.numel() * workspace.element_size(), _stream())
    return out


def reduce_sum(x):
    return reduce(x, RED_SUM)


def reduce_max(x):
    return reduce(x, RED_MAX)


def reduce_sumsq(x):
    return reduce(x, RED_SUMSQ)


def repeat_kv(x: torch.Tensor, n_rep: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """src/ops/attention.rs:161-201: x [batch, kv_heads, seq, head_dim] ->
    [batch, kv_heads * n_rep, seq, head_dim] (head h * n_rep + r = head h)."""
    if x.dim() < 4:
        raise OxideError(_lib.ERR_INVALID_ARG, "repeat_kv",
                         "repeat_kv requires 4D tensor (batch, heads, seq_len, head_dim)")
    _need(int(n_rep) >= 1, "repeat_kv", "n_rep must be >= 1")
    _need(out is None or (out.dtype == x.dtype and out.numel() == x.numel() * int(n_rep)), "repeat_kv",
          f"out must be {x.dtype} with {x.numel() * int(n_rep)} elements")
    _check(x, out)
    b, h, s, d = x.shape[0], x.shape[1], x.shape[2], x.numel() // (x.shape[0] * x.shape[1] * x.shape[2])
    shape = list(x.shape)
    shape[1] *= n_rep
    out = torch.empty(shape, dtype=x.dtype, device=x.device) if out is None else out
    call(f"oxide_repeat_kv_{_sfx(x)}", _p(x), _p(out), b, h, s, d, int(n_rep), _stream())
    return out


class KvCache:
    """Per-layer key/value caches [batch, kv_heads, max_seq_len, head_dim] on
    the device, mirroring src/cache/kv_cache.rs (KVCache::new / update / get /
    clear / is_full / get_cache_size).  update() appends with one kernel
    (oxide_kv_cache_append_*) at the layer's own length: the reference keeps a
    single counter advanced by every layer's update, which would place layer
    1's tokens after layer 0's; here each layer tracks its own length and
    current_seq_len() is layer 0's."""

    def __init__(self, num_layers: int, batch_size: int, num_kv_heads: int, head_dim: int,
                 max_seq_len: int, dtype=torch.float32, device="cuda"):
        if dtype not in _SFX:
            raise OxideError(_lib.ERR_UNSUPPORTED, "KvCache", f"dtype {dtype} is not float32/bfloat16")
        shape = (batch_size, num_kv_heads, max_seq_len, head_dim)
        self.k_cache = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v_cache = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self._len = [0] * num_layers
        self.max_seq_len, self.num_layers = max_seq_len, num_layers
        self.num_kv_heads, self.head_dim, self.batch_size = num_kv_heads, head_dim, batch_size

    def _layer(self, layer_idx: int) -> None:
        if not 0 <= layer_idx < self.num_layers:
            raise OxideError(_lib.ERR_INVALID_ARG, "KvCache",
                             f"Layer index {layer_idx} out of range for {self.num_layers} layers")

    def update(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """kv_cache.rs:55-85: append key/value [batch, kv_heads, new_len, head_dim]."""
        self._layer(layer_idx)
        _check(key, value)
        kc, vc = self.k_cache[layer_idx], self.v_cache[layer_idx]
        if key.shape != value.shape or key.shape[:2] != kc.shape[:2] or key.shape[3] != kc.shape[3] \
                or key.dtype != kc.dtype or value.dtype != kc.dtype:
            raise OxideError(_lib.ERR_INVALID_ARG, "KvCache",
                             f"key/value {list(key.shape)} do not match the cache {list(kc.shape)}")
        cur, new = self._len[layer_idx], key.shape[2]
        if cur + new > self.max_seq_len:
            raise OxideError(_lib.ERR_INVALID_ARG, "KvCache",
                             f"KV cache overflow: {cur + new} > {self.max_seq_len}")
        call(f"oxide_kv_cache_append_{_sfx(kc)}", _p(kc), _p(vc), _p(key), _p(value), self.batch_size,
             self.num_kv_heads, self.max_seq_len, self.head_dim, cur, new, _stream())
        self._len[layer_idx] = cur + new

    def get(self, layer_idx: int, seq_len: Optional[int] = None):
        """kv_cache.rs:87-110: views [batch, kv_heads, seq_len, head_dim] of the
        first seq_len positions (default: the layer's length), None if 0."""
        self._layer(layer_idx)
        n = self._len[layer_idx] if seq_len is None else seq_len
        if n == 0:
            return None
        return self.k_cache[layer_idx][:, :, :n], self.v_cache[layer_idx][:, :, :n]

    def current_seq_len(self) -> int:
        return self._len[0]

    def clear(self) -> None:
        self._len = [0] * self.num_layers

    def is_full(self) -> bool:
        return self._len[0] >= self.max_seq_len

    def get_cache_size(self) -> int:
        """Bytes held by all layers' k and v caches (kv_cache.rs:128-133)."""
        es = self.k_cache[0].element_size() if self.k_cache else 4
        return 2 * self.batch_size * self.num_kv_heads * self.max_seq_len * self.head_dim * es * self.num_layers


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     lens: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                     workspace: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query token per (batch, head) against KV caches: the attention of
    src/ops/attention.rs:41-87 with q_len = 1, keys j < lens[b] (int32; None:
    every position), query head h reading kv head h // (q_heads // kv_heads).
    q [batch, q_heads, head_dim]; caches [batch, kv_heads, max_seq, head_dim].
    scale defaults to the reference's (head_dim as f32).sqrt().recip()."""
    if q.dim() != 3 or k_cache.dim() != 4 or k_cache.shape != v_cache.shape or \
            k_cache.shape[0] != q.shape[0] or k_cache.shape[3] != q.shape[2]:
        raise OxideError(_lib.ERR_INVALID_ARG, "decode_attention",
                         f"q {list(q.shape)} and caches {list(k_cache.shape)} do not match")
    if lens is not None and lens.dtype != torch.int32:
        raise OxideError(_lib.ERR_INVALID_ARG, "decode_attention", "lens must be int32")
    _same_dtype("decode_attention", q, k_cache=k_cache, v_cache=v_cache)
    _out_like("decode_attention", q, out=out)
    b, hq, d = q.shape
    hkv, m = k_cache.shape[1], k_cache.shape[2]
    _need(lens is None or lens.numel() >= b, "decode_attention", f"lens needs {b} entries")
    need = int(_lib.lib().oxide_decode_attention_workspace_bytes(b, hq, m, d))
    _need(workspace is None or workspace.numel() * workspace.element_size() >= need, "decode_attention",
          f"workspace must hold {need} bytes")
    _check(q, k_cache, v_cache, lens, workspace, out)
    if scale is None:
        scale = float(torch.tensor(float(d), dtype=torch.float32).sqrt().reciprocal())
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    call(f"oxide_decode_attention_{_sfx(q)}", _p(q), _p(k_cache), _p(v_cache), _p(lens), _p(out), b, hq, hkv,
         m, d, float(scale), _p(workspace), workspace.numel() * workspace.element_size(), _stream())
    return out


# ---- token sampling (src/tokenizer.rs:166-232, src/pipeline.rs:181-205) ----
SAMPLE_INVALID = -1  # OXIDE_SAMPLE_INVALID seen through an int32 tensor


def softmax_with_temperature(logits: torch.Tensor, temperature: float,
                             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """src/tokenizer.rs:166-180 over the last dim -> f32 probabilities."""
    _need(out is None or (out.dtype == torch.float32 and out.numel() == logits.numel()),
          "softmax_with_temperature", f"out must be float32 with {logits.numel()} elements")
    _check(logits, out)
    vocab = logits.shape[-1]
    if out is None:
        out = torch.empty(logits.shape, dtype=torch.float32, device=logits.device)
    call(f"oxide_softmax_with_temperature_{_sfx(logits)}", _p(logits), _p(out),
         math.prod(logits.shape[:-1]), vocab, float(temperature), _stream())
    return out


def sample_next_token(logits: torch.Tensor, uniforms: torch.Tensor, temperature: float = 1.0,
                      top_k: int = 50, top_p: float = 1.0,
                      probs_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """sample_next_token (src/pipeline.rs:181-205) for every row of logits
    [..., vocab]: softmax_with_temperature, then sample_top_p when top_p < 1,
    else sample_top_k, with uniforms[row] (f32 in [0, 1), on the device) as
    the reference's fastrand::f32() draw.  Returns int32 token ids;
    SAMPLE_INVALID (-1) marks a row whose probabilities hold a NaN (the
    reference's sort panics there).  The defaults are InferenceParams::default's
    (src/tokenizer.rs:153-162)."""
    _check(logits, uniforms, probs_out)
    vocab = logits.shape[-1]
    rows = math.prod(logits.shape[:-1])
    if probs_out is not None and (probs_out.dtype != torch.float32 or probs_out.numel() != rows * vocab):
        raise ValueError("probs_out must be f32 with the logits' element count")
    if uniforms.dtype != torch.float32 or uniforms.numel() != rows:
        raise ValueError(f"uniforms must be f32 with one value per row ({rows})")
    tokens = torch.empty(logits.shape[:-1], dtype=torch.int32, device=logits.device)
    call(f"oxide_sample_{_sfx(logits)}", _p(logits), rows, vocab, float(temperature), int(top_k),
         float(top_p), _p(uniforms), _p(tokens), _p(probs_out), _stream())
    return tokens
