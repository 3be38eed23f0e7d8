"""Parity of the remaining elementwise ops of the reference (relu, gelu,
gelu_quick, sigmoid, tanh, exp, log, sqrt, pow, clamp, neg, abs) and of
layer_norm against the CPU oracle, through the C ABI.

Bars (stated per op): bit-exact where the op is one IEEE operation or a
selection (relu, neg, abs, clamp, sqrt); within a few ulp where CUDA's
expf / logf / tanhf / powf replace glibc's (each within 2 ulp of the exact
value; the reference's chain then rounds the same steps); gelu additionally
allows 2^-22 |x| absolute where 1 + tanh(..) cancels for x << 0.  bf16 results
are within one bf16 ulp (gelu: or the same absolute slack).  layer_norm: within
1e-5 of the exact (f64) value relative to |normalized * w| + |b| +
|w| * mean|x| / sd (the last term: the conditioning of x - mean) and to the
reference within that plus the reference's own sequential-sum drift.
"""
import numpy as np
import pytest

from _util import assert_bits_equal, bf16_to_f32, misaligned_copy, to_dev, to_np, ulp_bf16, ulp_f32

F = np.float32

ULP_BAR = {  # op -> max ulp of the f32 result vs the oracle
    "relu": 0, "neg": 0, "abs": 0, "clamp": 0, "sqrt": 0,
    "exp": 4, "log": 4, "tanh": 4, "pow": 8, "sigmoid": 8, "gelu_quick": 8, "gelu": 8,
}


def _inputs(op, n, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * 4).astype(F)
    if op in ("log", "sqrt", "pow"):
        x = np.abs(x) + F(1e-3)
    specials = np.array([0.0, 1.0, -1.0, 0.5, 30.0, -30.0, 100.0, -100.0, np.inf, -np.inf, np.nan],
                        F)
    if op in ("log", "sqrt", "pow"):
        specials = np.array([0.0, 1.0, 0.5, 2.0, 1e-30, 1e30, np.inf, -1.0, np.nan], F)
    x[: specials.size] = specials
    return x


def _params(op):
    return {"pow": (1.7, 0.0), "clamp": (-1.5, 2.5)}.get(op, (0.0, 0.0))


def _same_nan_and_zero(got, ref):
    gn, rn = np.isnan(got), np.isnan(ref)
    assert np.array_equal(gn, rn), "NaN positions differ"
    m = ~gn & ~((got == 0) & (ref == 0))  # +0 and -0 both accepted where the reference gives a zero
    return m


@pytest.mark.gpu
@pytest.mark.parametrize("op", list(ULP_BAR))
def test_unary_f32_matches_oracle(cuda, orc, op):
    from oxide_b200 import _lib, ops

    code = getattr(_lib, op.upper())
    x = _inputs(op, 100003, 500 + code)  # odd length: vector body + scalar tail
    a, b = _params(op)
    got = to_np(ops.unary(code, to_dev(x), a, b))
    ref = orc.unary(code, x, a, b)
    m = _same_nan_and_zero(got, ref)
    d = ulp_f32(got[m], ref[m])
    if op == "gelu":  # 1 + tanh(v) cancels for x << 0
        slack = np.abs(got[m].astype(np.float64) - ref[m]) <= 2.0 ** -22 * np.abs(x[m].astype(np.float64))
        d = np.where(slack, 0, d)
    assert d.max(initial=0) <= ULP_BAR[op], f"{op}: max {d.max()} ulp"
    # unaligned pointers take the scalar kernel: same results
    got2 = to_np(ops.unary(code, misaligned_copy(x), a, b))
    m2 = _same_nan_and_zero(got2, got)
    assert np.array_equal(got2[m2].view(np.uint32), got[m2].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("op", list(ULP_BAR))
def test_unary_bf16_matches_oracle(cuda, orc, op):
    from oxide_b200 import _lib, ops

    code = getattr(_lib, op.upper())
    x = orc.f32_to_bf16(_inputs(op, 4099, 600 + code))
    a, b = _params(op)
    got = to_np(ops.unary(code, to_dev(x), a, b))
    ref = orc.unary(code, x, a, b)
    gf, rf = bf16_to_f32(got), bf16_to_f32(ref)
    m = _same_nan_and_zero(gf, rf)
    d = ulp_bf16(got[m], ref[m])
    if op == "gelu":
        xf = bf16_to_f32(x)[m].astype(np.float64)
        d = np.where(np.abs(gf[m].astype(np.float64) - rf[m]) <= 2.0 ** -22 * np.abs(xf), 0, d)
    assert d.max(initial=0) <= (0 if ULP_BAR[op] == 0 else 1), f"{op}: max {d.max()} bf16 ulp"


@pytest.mark.gpu
def test_named_activation_entry_points_match_unary(cuda):
    import torch

    from oxide_b200 import _lib

    x = torch.randn(5000, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    for name, code in (("relu", _lib.RELU), ("gelu", _lib.GELU), ("sigmoid", _lib.SIGMOID),
                       ("tanh", _lib.TANH)):
        a = torch.empty_like(x)
        b = torch.empty_like(x)
        _lib.call(f"oxide_{name}_f32", x.data_ptr(), a.data_ptr(), x.numel(), st)
        _lib.call("oxide_unary_f32", code, x.data_ptr(), b.data_ptr(), x.numel(), 0.0, 0.0, st)
        assert torch.equal(a, b), name


@pytest.mark.gpu
def test_unary_argument_errors(cuda):
    import torch

    from oxide_b200 import _lib

    x = torch.zeros(16, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    assert _lib.raw("oxide_unary_f32", _lib.CLAMP, x.data_ptr(), x.data_ptr(), 16, 2.0, 1.0,
                    st) == _lib.ERR_INVALID_ARG
    assert "min <= max" in _lib.last_error()
    assert _lib.raw("oxide_unary_f32", 99, x.data_ptr(), x.data_ptr(), 16, 0.0, 0.0,
                    st) == _lib.ERR_INVALID_ARG
    assert _lib.raw("oxide_unary_f32", _lib.EXP, None, None, 0, 0.0, 0.0, st) == _lib.OK


def _ln_scale(x, w, b):
    """The exact (f64) layer_norm and the magnitude its f32 result is measured
    against: |n * w| + |b|, plus |w| * mean(|x|) / sd -- the deviation x - mean
    is formed from an f32 row mean whose rounding is relative to the row's
    values, not to the deviation, so where x is close to the mean the f32
    result (the reference's as much as the kernel's) carries that much."""
    x = x.astype(np.float64)
    mean = x.mean(axis=1, keepdims=True)
    sd = np.sqrt(((x - mean) ** 2).mean(axis=1, keepdims=True) + np.float64(F(1e-5)))
    nrm = (x - mean) / sd
    wd = w.astype(np.float64)
    exact = nrm * wd + b.astype(np.float64)
    cond = np.abs(wd) * np.abs(x).mean(axis=1, keepdims=True) / sd
    return exact, np.abs(nrm * wd) + np.abs(b.astype(np.float64)) + cond


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(3, 1), (8, 33), (16, 768), (4, 4096), (3, 5000), (2, 20000),
                                       # many rows: rows near their mean (x - mean conditioning)
                                       (20000, 256), (5000, 4096)])
def test_layer_norm_matches_oracle(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    rng = np.random.default_rng(rows * 7919 + cols)
    x = (rng.standard_normal((rows, cols)) * 3 + 1).astype(F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    b = rng.uniform(-0.5, 0.5, cols).astype(F)
    if dtype == "bf16":
        x, w, b = orc.f32_to_bf16(x), orc.f32_to_bf16(w), orc.f32_to_bf16(b)
    got = to_np(ops.layer_norm(to_dev(x), to_dev(w), to_dev(b), 1e-5))
    ref = orc.layer_norm(x, w, b, 1e-5)
    xf = bf16_to_f32(x) if dtype == "bf16" else x
    wf = bf16_to_f32(w) if dtype == "bf16" else w
    bf = bf16_to_f32(b) if dtype == "bf16" else b
    exact, scale = _ln_scale(xf, wf, bf)
    if dtype == "f32":
        g = got.astype(np.float64)
        lim = 1e-5 * scale + 1e-30
        assert np.all(np.abs(g - exact) <= lim), "kernel vs exact"
        assert np.all(np.abs(g - ref) <= lim + np.abs(ref - exact)), "kernel vs reference + its drift"
    else:
        d = ulp_bf16(got, ref)
        gd = np.abs(bf16_to_f32(got).astype(np.float64) - bf16_to_f32(ref))
        ok = (d <= 1) | (gd <= 2.0 ** -8 * scale)  # cancellation in w * n + b
        assert ok.all(), f"max {d.max()} bf16 ulp"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(8, 33), (16, 768), (64, 4096), (2, 20000), (5000, 1024),
                                       (4096, 4096)])
def test_add_layer_norm_matches_oracle_and_unfused(cuda, orc, dtype, rows, cols):
    """layer_norm(x + r) (the reference's fused-add intent): against the
    oracle's add then layer_norm, within the layer_norm bar; bit-equal to the
    device's own add followed by layer_norm (the sum is rounded to the I/O type
    first); in place over x."""
    from oxide_b200 import ops

    rng = np.random.default_rng(rows * 104729 + cols)
    x = (rng.standard_normal((rows, cols)) * 2 + 0.5).astype(F)
    r = rng.standard_normal((rows, cols)).astype(F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    b = rng.uniform(-0.5, 0.5, cols).astype(F)
    if dtype == "bf16":
        x, r, w, b = (orc.f32_to_bf16(a) for a in (x, r, w, b))
    tx, tr, tw, tb = to_dev(x), to_dev(r), to_dev(w), to_dev(b)
    got = to_np(ops.add_layer_norm(tx, tr, tw, tb, 1e-5))
    h = orc.binary(orc.ADD, x.reshape(-1), r.reshape(-1)).reshape(rows, cols)
    ref = orc.layer_norm(h, w, b, 1e-5)
    f = (lambda a: bf16_to_f32(a)) if dtype == "bf16" else (lambda a: a)
    exact, scale = _ln_scale(f(h), f(w), f(b))
    if dtype == "f32":
        g = got.astype(np.float64)
        lim = 1e-5 * scale + 1e-30
        assert np.all(np.abs(g - exact) <= lim), "kernel vs exact"
        assert np.all(np.abs(g - ref) <= lim + np.abs(ref - exact)), "kernel vs reference + its drift"
    else:
        d = ulp_bf16(got, ref)
        gd = np.abs(bf16_to_f32(got).astype(np.float64) - bf16_to_f32(ref))
        assert np.all((d <= 1) | (gd <= 2.0 ** -8 * scale))
    unfused = to_np(ops.layer_norm(ops.add(tx, tr), tw, tb, 1e-5))
    assert_bits_equal(got, unfused)
    ops.add_layer_norm(tx, tr, tw, tb, 1e-5, out=tx)
    assert_bits_equal(to_np(tx), got)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_add_layer_norm_misaligned_residual(cuda, orc, dtype):
    """x aligned, r one element off a 16-byte boundary: the row kernel's vector
    path needs both, so this alone sends the call to the element kernel (which
    sums in another order); within the same bar of the oracle as the vector
    path."""
    from oxide_b200 import ops

    rows, cols = 96, 4096
    rng = np.random.default_rng(77)
    x = rng.standard_normal((rows, cols)).astype(F)
    r = rng.standard_normal((rows, cols)).astype(F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    b = rng.uniform(-0.5, 0.5, cols).astype(F)
    if dtype == "bf16":
        x, r, w, b = (orc.f32_to_bf16(a) for a in (x, r, w, b))
    got = to_np(ops.add_layer_norm(to_dev(x), misaligned_copy(r), to_dev(w), to_dev(b), 1e-5))
    h = orc.binary(orc.ADD, x.reshape(-1), r.reshape(-1)).reshape(rows, cols)
    ref = orc.layer_norm(h, w, b, 1e-5)
    f = (lambda a: bf16_to_f32(a)) if dtype == "bf16" else (lambda a: a)
    exact, scale = _ln_scale(f(h), f(w), f(b))
    if dtype == "f32":
        g = got.astype(np.float64)
        lim = 1e-5 * scale + 1e-30
        assert np.all(np.abs(g - exact) <= lim), "kernel vs exact"
        assert np.all(np.abs(g - ref) <= lim + np.abs(ref - exact)), "kernel vs reference + its drift"
    else:
        d = ulp_bf16(got, ref)
        gd = np.abs(bf16_to_f32(got).astype(np.float64) - bf16_to_f32(ref))
        assert np.all((d <= 1) | (gd <= 2.0 ** -8 * scale))


@pytest.mark.gpu
def test_add_layer_norm_argument_errors(cuda):
    import torch

    from oxide_b200 import OxideError, _lib, ops

    x = torch.ones(4, 64, device=cuda)
    w, b = torch.ones(64, device=cuda), torch.zeros(64, device=cuda)
    with pytest.raises(OxideError, match="residual"):
        ops.add_layer_norm(x, x[:, :32].contiguous(), w, b, 1e-5)
    st = torch.cuda.current_stream().cuda_stream
    assert _lib.raw("oxide_add_layer_norm_f32", x.data_ptr(), None, w.data_ptr(), b.data_ptr(),
                    x.data_ptr(), 4, 64, 1e-5, st) == _lib.ERR_INVALID_ARG
    assert "null pointer" in _lib.last_error()


@pytest.mark.gpu
def test_layer_norm_constant_rows_and_shape_errors(cuda, orc):
    import torch

    from oxide_b200 import OxideError, ops

    x = torch.full((5, 768), 2.5, device=cuda)
    w = torch.rand(768, device=cuda) + 0.5
    b = torch.rand(768, device=cuda) - 0.5
    y = ops.layer_norm(x, w, b, 1e-5)
    assert torch.equal(y, b.expand_as(y))  # mean exact, deviations 0, 0 * w + b = b
    with pytest.raises(OxideError, match="bias shape"):
        ops.layer_norm(x, w, b[:10], 1e-5)
    with pytest.raises(OxideError, match="weight shape"):
        ops.layer_norm(x, w[:10], b, 1e-5)


# ---------------------------------------------------------------- KV cache / repeat_kv
@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("b,h,s,d,rep", [(2, 8, 37, 128, 4), (1, 1, 1, 8, 1), (3, 2, 5, 6, 3)])
def test_repeat_kv_bit_exact(cuda, orc, dtype, b, h, s, d, rep):
    from oxide_b200 import ops

    x = np.random.default_rng(b * 100 + d).standard_normal((b, h, s, d)).astype(F)
    if dtype == "bf16":
        x = orc.f32_to_bf16(x)
    got = to_np(ops.repeat_kv(to_dev(x), rep))
    assert got.shape == (b, h * rep, s, d)
    assert np.array_equal(got, orc.repeat_kv(x, rep))


@pytest.mark.gpu
def test_repeat_kv_unaligned_and_errors(cuda, orc):
    from oxide_b200 import OxideError, ops

    x = np.random.default_rng(9).standard_normal((2, 4, 9, 16)).astype(F)
    got = to_np(ops.repeat_kv(misaligned_copy(x), 2))  # scalar kernel
    assert np.array_equal(got, orc.repeat_kv(x, 2))
    with pytest.raises(OxideError, match="4D"):
        ops.repeat_kv(to_dev(x[0]), 2)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kv_cache_decode_appends_equal_prefill(cuda, orc, dtype):
    """A prefill of 7 tokens followed by 5 single-token decode steps leaves the
    cache equal to the oracle's appends and to one 12-token prefill."""
    import torch

    from oxide_b200 import OxideError, ops

    B, H, D, M = 2, 8, 128, 16
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    rng = np.random.default_rng(11)
    ks = rng.standard_normal((B, H, 12, D)).astype(F)
    vs = rng.standard_normal((B, H, 12, D)).astype(F)
    if dtype == "bf16":
        ks, vs = orc.f32_to_bf16(ks), orc.f32_to_bf16(vs)
    cache = ops.KvCache(2, B, H, D, M, dtype=tdt)
    cache.update(0, to_dev(np.ascontiguousarray(ks[:, :, :7])), to_dev(np.ascontiguousarray(vs[:, :, :7])))
    for t in range(7, 12):
        cache.update(0, to_dev(np.ascontiguousarray(ks[:, :, t:t + 1])),
                     to_dev(np.ascontiguousarray(vs[:, :, t:t + 1])))
    assert cache.current_seq_len() == 12 and not cache.is_full()
    kc = np.zeros((B, H, M, D), ks.dtype)
    vc = np.zeros_like(kc)
    assert orc.kv_append(kc, vc, ks, vs, 0)
    assert np.array_equal(to_np(cache.k_cache[0]), kc) and np.array_equal(to_np(cache.v_cache[0]), vc)
    k, v = cache.get(0)
    assert k.shape == (B, H, 12, D) and np.array_equal(to_np(k.contiguous()), ks)
    assert cache.get(1) is None  # layer 1 untouched
    with pytest.raises(OxideError, match="KV cache overflow: 17 > 16"):
        cache.update(0, to_dev(np.ascontiguousarray(ks[:, :, :5])), to_dev(np.ascontiguousarray(vs[:, :, :5])))
    with pytest.raises(OxideError, match="Layer index 2 out of range"):
        cache.update(2, to_dev(ks), to_dev(vs))
    assert cache.get_cache_size() == 2 * B * H * M * D * (4 if dtype == "f32" else 2) * 2
    cache.clear()
    assert cache.current_seq_len() == 0


@pytest.mark.gpu
def test_kv_append_abi_overflow_writes_nothing(cuda):
    import torch

    from oxide_b200 import _lib

    kc = torch.zeros(1, 1, 4, 8, device=cuda)
    vc = torch.zeros_like(kc)
    k = torch.ones(1, 1, 3, 8, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    rc = _lib.raw("oxide_kv_cache_append_f32", kc.data_ptr(), vc.data_ptr(), k.data_ptr(), k.data_ptr(),
                  1, 1, 4, 8, 2, 3, st)
    assert rc == _lib.ERR_INVALID_ARG and "overflow" in _lib.last_error()
    torch.cuda.synchronize()
    assert not kc.any() and not vc.any()


# ---------------------------------------------------------------- decode attention
def _attn_exact(q, kc, vc, lens, scale):
    q, kc, vc = (np.asarray(a, np.float64) for a in (q, kc, vc))
    b, hq, d = q.shape
    hkv = kc.shape[1]
    rep = hq // hkv
    out = np.zeros((b, hq, d))
    mag = np.zeros((b, hq, d))
    for bi in range(b):
        n = kc.shape[2] if lens is None else max(0, min(int(lens[bi]), kc.shape[2]))
        for h in range(hq):
            if n == 0:
                continue
            k, v = kc[bi, h // rep, :n], vc[bi, h // rep, :n]
            s = (k @ q[bi, h]) * np.float64(scale)
            p = np.exp(s - s.max())
            p /= p.sum()
            out[bi, h] = p @ v
            mag[bi, h] = p @ np.abs(v)
    return out, mag


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("b,hq,hkv,m,d,lens", [
    (2, 8, 2, 300, 128, [300, 77]),      # rep 4 (Mistral), a partial tile
    (3, 4, 4, 1000, 128, [1000, 1, 0]),   # rep 1, a single key, an empty sequence
    (1, 16, 2, 4500, 128, [4321]),        # rep 8, many splits
    (2, 6, 3, 129, 128, None),            # rep 2, no lengths
    (2, 4, 2, 50, 64, [50, 33]),          # head_dim 64: the generic kernel
    # many short sequences (some empty): with more units than CTAs each CTA of
    # the balanced bf16 schedule covers several (sequence, kv head) groups
    (200, 32, 8, 128, 128, [int(x) for x in np.random.default_rng(7).integers(0, 129, 200)]),
])
def test_decode_attention_matches_oracle(cuda, orc, dtype, b, hq, hkv, m, d, lens):
    from oxide_b200 import ops

    rng = np.random.default_rng(b * 1000 + m)
    q = rng.standard_normal((b, hq, d)).astype(F)
    kc = rng.standard_normal((b, hkv, m, d)).astype(F)
    vc = rng.standard_normal((b, hkv, m, d)).astype(F)
    if dtype == "bf16":
        q, kc, vc = orc.f32_to_bf16(q), orc.f32_to_bf16(kc), orc.f32_to_bf16(vc)
    lz = None if lens is None else np.array(lens, np.int32)
    got = to_np(ops.decode_attention(to_dev(q), to_dev(kc), to_dev(vc),
                                     None if lz is None else to_dev(lz)))
    ref = orc.decode_attention(q, kc, vc, lz)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    f = (lambda a: bf16_to_f32(a)) if dtype == "bf16" else (lambda a: a)
    exact, mag = _attn_exact(f(q), f(kc), f(vc), lz, scale)
    g = f(got).astype(np.float64)
    r = f(ref).astype(np.float64)
    if dtype == "f32":
        lim = 1e-5 * mag + 1e-7
        assert np.all(np.abs(g - exact) <= lim), "kernel vs exact"
        assert np.all(np.abs(g - r) <= lim + np.abs(r - exact)), "kernel vs reference + its drift"
    else:
        # within 1 bf16 ulp of the exact value, or 2^-14 sum p|v| where the
        # output cancels; against the reference within that plus its own error
        d_ex = ulp_bf16(got, orc.f32_to_bf16(np.asarray(exact, np.float32)).reshape(got.shape))
        ok = (d_ex <= 1) | (np.abs(g - exact) <= 2.0 ** -14 * mag + 1e-30)
        assert ok.all(), f"{np.count_nonzero(~ok)} outputs off the exact value (max {d_ex.max()} bf16 ulp)"
        d_ulp = ulp_bf16(got, ref)
        ok = (d_ulp <= 1) | (np.abs(g - r) <= 2.0 ** -14 * mag + np.abs(r - exact) + 1e-30)
        assert ok.all(), f"max {d_ulp.max()} bf16 ulp from the reference"
    if lz is not None:
        for bi, n in enumerate(lz):
            if n == 0:
                assert np.all(g[bi] == 0)


@pytest.mark.gpu
def test_decode_attention_equals_repeat_kv_then_softmax(cuda):
    """The GQA head map equals materialising repeat_kv and attending per head."""
    import torch

    from oxide_b200 import ops

    g = torch.Generator(device=cuda).manual_seed(5)
    q = torch.randn(2, 8, 128, device=cuda, generator=g)
    kc = torch.randn(2, 2, 200, 128, device=cuda, generator=g)
    vc = torch.randn(2, 2, 200, 128, device=cuda, generator=g)
    lens = torch.tensor([200, 150], dtype=torch.int32, device=cuda)
    got = ops.decode_attention(q, kc, vc, lens)
    k4, v4 = ops.repeat_kv(kc, 4), ops.repeat_kv(vc, 4)
    want = torch.empty_like(got)
    for bi, n in enumerate((200, 150)):
        s = torch.einsum("hd,hjd->hj", q[bi].double(), k4[bi, :, :n].double()) / np.sqrt(128.0)
        want[bi] = torch.einsum("hj,hjd->hd", torch.softmax(s, -1), v4[bi, :, :n].double()).float()
    assert torch.allclose(got, want, rtol=1e-4, atol=1e-5)
