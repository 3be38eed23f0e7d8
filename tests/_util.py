"""Helpers shared by the GPU parity tests: numpy <-> torch moves (bf16 as raw
uint16 bits on the numpy side) and ulp distances."""
import numpy as np
import torch


def to_dev(a: np.ndarray, dev="cuda") -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.contiguous().cpu().numpy()


def misaligned_copy(a: np.ndarray, dev="cuda") -> torch.Tensor:
    """Device copy of `a` whose data pointer is one element past a 16-byte boundary."""
    t = to_dev(a, dev).reshape(-1)
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=dev)
    view = buf[1:]
    view.copy_(t)
    assert view.data_ptr() % 16 != 0
    return view.view(a.shape)


def _ordered(bits: np.ndarray, width: int) -> np.ndarray:
    b = bits.astype(np.int64)
    sign = 1 << (width - 1)
    return np.where(b & sign, -(b & (sign - 1)), b)


def ulp_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    ua = np.ascontiguousarray(a, np.float32).view(np.uint32)
    ub = np.ascontiguousarray(b, np.float32).view(np.uint32)
    return np.abs(_ordered(ua, 32) - _ordered(ub, 32))


def ulp_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.abs(_ordered(np.asarray(a, np.uint16), 16) - _ordered(np.asarray(b, np.uint16), 16))


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def assert_bits_equal(got: np.ndarray, ref: np.ndarray):
    got, ref = np.ascontiguousarray(got), np.ascontiguousarray(ref)
    assert got.shape == ref.shape or got.size == ref.size
    g = got.reshape(-1).view(np.uint16 if got.dtype == np.uint16 else np.uint32)
    r = ref.reshape(-1).view(np.uint16 if ref.dtype == np.uint16 else np.uint32)
    bad = np.nonzero(g != r)[0]
    assert bad.size == 0, f"{bad.size} of {g.size} differ; first at {bad[:5]}"


def assert_close_rel(got: np.ndarray, ref: np.ndarray, rel: float):
    """|got - ref| <= rel * |ref| elementwise (f32 results), NaN positions equal."""
    got = np.asarray(got, np.float32).reshape(-1)
    ref = np.asarray(ref, np.float32).reshape(-1)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    m = ~np.isnan(ref)
    err = np.abs(got[m].astype(np.float64) - ref[m].astype(np.float64))
    lim = rel * np.abs(ref[m].astype(np.float64)) + 1e-38
    worst = np.max(err / lim) if err.size else 0.0
    assert worst <= 1.0, f"max error {worst:.3g}x the {rel} relative tolerance"


def assert_parity_rel(got: np.ndarray, ref: np.ndarray, exact: np.ndarray, rel: float):
    """Parity for f32 results whose reference accumulates long sums
    sequentially in f32: the reference itself is off the exact value by
    |ref - exact| (a sequential f32 sum of n terms drifts by ~sqrt(n) ulps),
    so the kernel must be within `rel` of the exact value and within
    rel + that drift of the reference."""
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    exact = np.asarray(exact, np.float64).reshape(-1)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    m = ~np.isnan(ref)
    g, r, e = got[m], ref[m], exact[m]
    lim = rel * np.abs(e) + 1e-38
    acc = np.max(np.abs(g - e) / lim, initial=0.0)
    assert acc <= 1.0, f"kernel error vs exact is {acc:.3g}x the {rel} relative tolerance"
    par = np.max(np.abs(g - r) / (lim + np.abs(r - e)), initial=0.0)
    assert par <= 1.0, f"kernel vs reference exceeds rel + reference drift ({par:.3g}x)"


def softmax_exact(s: np.ndarray, lens=None) -> np.ndarray:
    """Softmax of f32 score rows with exp and the sum in f64; keys at or
    beyond lens[row] are 0 (rows with length 0 are all 0)."""
    s = np.asarray(s, np.float64)
    rows, cols = s.shape
    out = np.zeros_like(s)
    for r in range(rows):
        n = cols if lens is None else int(lens[r])
        if n <= 0:
            continue
        v = s[r, :n]
        e = np.exp(v - np.max(v))
        out[r, :n] = e / np.sum(e)
    return out


def rms_norm_exact(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float64)
    rms = np.sqrt(np.sum(x * x, axis=-1, keepdims=True) / x.shape[-1] + np.float64(np.float32(eps)))
    return x / rms * np.asarray(w, np.float64)


def assert_ulp(got: np.ndarray, ref: np.ndarray, max_ulp: int):
    d = ulp_bf16(got, ref) if got.dtype == np.uint16 else ulp_f32(got, ref)
    assert d.max(initial=0) <= max_ulp, f"max {d.max()} ulp (> {max_ulp}) at {np.argmax(d)}"


SAMPLE_INVALID = 0xFFFFFFFF


def sample_exact(p, top_k, top_p, u):
    """The reference's selection (sample_top_p / sample_top_k,
    src/tokenizer.rs:182-232) in exact (f64) arithmetic on one row of f32
    probabilities.  Returns (token, margin): margin is the distance, relative
    to the row's total, between a deciding threshold (top_p for the prefix, r
    for the walk) and the nearest running sum -- a result computed with
    rounded sums can differ only when the margin is within that rounding."""
    p = np.asarray(p, np.float32).ravel()
    n = p.size
    if n == 0:
        return 0, np.inf
    if n >= 2 and np.isnan(p).any():
        return SAMPLE_INVALID, np.inf
    order = np.argsort(-p.astype(np.float64), kind="stable")
    c = np.cumsum(p[order].astype(np.float64))
    scale = max(float(c[-1]), 1e-300)
    margin = np.inf
    if np.float32(top_p) < np.float32(1.0):
        tp = float(np.float32(top_p))
        i = int(np.searchsorted(c, tp, side="left"))
        keep = n if i >= n else i + 1
        near = [c[j] for j in (i - 1, i) if 0 <= j < n]
        margin = min(margin, min(abs(tp - x) for x in near) / scale)
    else:
        keep = min(int(top_k), n)
    if keep == 0:
        return 0, margin
    total = float(c[keep - 1])
    r = min(float(np.float32(np.float32(u) * np.float32(total))), total)
    j = min(int(np.searchsorted(c[:keep], r, side="left")), keep - 1)
    near = [c[x] for x in (j - 1, j) if 0 <= x < keep]
    margin = min(margin, min(abs(r - x) for x in near) / scale)
    return int(order[j]), margin


def in_drift_band(tok, ref, p_ref):
    """The two tokens are at most one sorted position apart, or the mass
    strictly between them lies within the rounding drift of the reference's
    sequential f32 running sums (n 2^-24 of the total, doubled for the kept
    prefix's total and the walk, and doubled again for the other side)."""
    p_ref = np.asarray(p_ref, np.float32)
    n = p_ref.size
    order = np.argsort(-p_ref.astype(np.float64), kind="stable")
    pos = np.empty(n, np.int64)
    pos[order] = np.arange(n)
    c = np.cumsum(p_ref[order].astype(np.float64))
    lo, hi = sorted((int(pos[tok]), int(pos[ref])))
    return hi - lo <= 1 or c[hi - 1] - c[lo] <= 4 * n * 2.0 ** -24 * c[-1]


F32_REL = 1e-5
BF16_ULP = 1
# The f32 SiLU kernels take e^-x from exp_rn_f32, correctly rounded on every
# float; the reference's glibc expf is not on 4.0e-5 of all floats and on
# 6.3e-4 of N(0,1)-distributed ones (1 ulp off there).  Where the two
# exponentials agree every later step rounds the same, so the result must be
# the reference's bits; elsewhere the 1-ulp difference passes through the
# rounded steps of x * (1 / (1 + e)) * up: within 2^-21 relative (measured
# over every float: up to 5 ulp where 1 + e is a rounding tie (e >= 2^24),
# more where 1 / (1 + e) is subnormal).
SILU_F32_REL = 2.0 ** -21


def assert_silu_f32_parity(got, ref, x, orc, threads=None):
    """f32 silu / silu*up (x = the gate) against the oracle: bit-exact at
    every element whose e^-x the reference's expf rounds correctly -- apart
    from e^-x within 2^-40 (relative) of a rounding boundary between two
    floats, where the float64 exp used as the judge here cannot tell which
    side of the boundary e^-x lies -- elsewhere within SILU_F32_REL, NaN
    exactly where the oracle has NaN."""
    u32 = np.uint32
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    got = np.ascontiguousarray(got, np.float32).reshape(-1)
    ref = np.ascontiguousarray(ref, np.float32).reshape(-1)
    nx = (-x).astype(np.float32)
    e_lib = orc.unary(orc.EXP, nx, threads=threads or orc.max_threads())
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        e64 = np.exp(nx.astype(np.float64))
        e_cr = e64.astype(np.float32)
        # the rounding boundary on e64's side of its nearest float
        up = e64 >= e_cr.astype(np.float64)
        nb = np.where(up, np.nextafter(e_cr, np.float32(np.inf)), np.nextafter(e_cr, np.float32(0)))
        mid = (e_cr.astype(np.float64) + nb.astype(np.float64)) * 0.5
        hard = np.abs(e64 - mid) <= 2.0 ** -40 * np.abs(e64)
    lib_cr = ((e_lib.view(u32) == e_cr.view(u32)) | (np.isnan(e_lib) & np.isnan(e_cr))) & ~hard
    gn, rn = np.isnan(got), np.isnan(ref)
    assert np.array_equal(gn, rn), "NaN positions differ"
    same = (got.view(u32) == ref.view(u32)) | (gn & rn)
    bad = np.nonzero(lib_cr & ~same)[0]
    assert bad.size == 0, f"{bad.size} results differ where the reference's exp is correctly rounded (first {bad[:5]})"
    ok = ~gn & ~same
    g64, r64 = got[ok].astype(np.float64), ref[ok].astype(np.float64)
    rel = np.abs(g64 - r64) <= SILU_F32_REL * np.abs(r64) + 2.0 ** -140
    assert rel.all(), f"{np.count_nonzero(~rel)} results beyond 2^-21 relative"
    return int(np.count_nonzero(~same)), int(np.count_nonzero(~lib_cr))


def smax_close(got, ref, x, cols, dtype, scale=1.0, mask=None, lens=None, rows_per_len=1,
               causal_q=0):
    """f32: parity within 1e-5 relative of the exact softmax of the same f32
    scores (plus the reference's own sequential-sum drift); bf16: 1 ulp."""
    if dtype == "bf16":
        assert_ulp(got, ref, BF16_ULP)
        return
    s = (np.asarray(x, np.float32).reshape(-1, cols) * np.float32(scale)).astype(np.float32)
    if mask is not None:
        s = (s + np.asarray(mask, np.float32)[np.arange(cols) % mask.size]).astype(np.float32)
    rows = s.shape[0]
    n = np.full(rows, cols, np.int64)
    if lens is not None:
        n = np.minimum(n, np.maximum(np.asarray(lens, np.int64)[np.arange(rows) // rows_per_len], 0))
    if causal_q:
        n = np.minimum(n, np.arange(rows) % causal_q + 1 + cols - causal_q)
    assert_parity_rel(got, ref, softmax_exact(s, n), F32_REL)
