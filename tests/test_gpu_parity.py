"""CUDA kernels vs the CPU oracle on seeded inputs, through the C ABI.

Tolerances (stated by the parity contract):
  * add / sub / mul / div / scale / row-broadcast mul, RoPE, argmax indices,
    row max: bit-exact (RoPE uses no transcendental on the device: the tables
    are inputs, so its IEEE arithmetic matches exactly);
  * SiLU and SiLU*mul f32: bit-exact wherever the reference's expf (glibc) is
    correctly rounded, within 2^-21 relative elsewhere (assert_silu_f32_parity);
  * RMSNorm, softmax, sums (f32): within 1e-5 relative of the exact (f64)
    value, and of the reference within 1e-5 plus the reference's own
    sequential-f32-sum drift from exact (which alone reaches ~3e-5 relative
    for 32768-key softmax rows);
  * every bf16 result: <= 1 bf16 ulp.
"""
import numpy as np
import pytest
import torch

from _util import (assert_bits_equal, assert_close_rel, assert_parity_rel, assert_ulp, bf16_to_f32,
                   misaligned_copy, rms_norm_exact, smax_close, softmax_exact, to_dev, to_np, ulp_f32)

pytestmark = pytest.mark.gpu

from _util import BF16_ULP, F32_REL, assert_silu_f32_parity  # noqa: E402

F = np.float32


def rand(shape, seed, dtype="f32", scale=1.0, orc=None):
    x = (np.random.default_rng(seed).standard_normal(shape, dtype=F) * F(scale)).astype(F)
    return x if dtype == "f32" else orc.f32_to_bf16(x).reshape(shape)


def close(got, ref, dtype, rel=F32_REL):
    if dtype == "bf16":
        assert_ulp(got, ref, BF16_ULP)
    else:
        assert_close_rel(got, ref, rel)


# ---------------------------------------------------------------- binary ops
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("na,nb,n", [
    (4096 * 16, 4096 * 16, 4096 * 16),  # full, vector path
    (1001, 1001, 1001),                 # vector path + scalar tail
    (8192 * 3, 4096, 8192 * 3),         # row broadcast of b
    (512, 512 * 6, 512 * 6),            # broadcast of a
    (40, 24, 120),                      # both indexed modulo
    (6, 10, 30),                        # modulo lengths not vector multiples -> scalar
    (1, 1, 1),
])
def test_binary(cuda, orc, dtype, op, na, nb, n):
    from oxide_b200 import ops

    a = rand(na, 1, dtype, orc=orc)
    b = rand(nb, 2, dtype, orc=orc)
    if op == 3:
        b = (np.abs(bf16_to_f32(b) if dtype == "bf16" else b) + F(0.5)).astype(F)
        b = b if dtype == "f32" else orc.f32_to_bf16(b)
    ref = orc.binary(op, a, b, n)
    out = torch.empty(n, dtype=torch.float32 if dtype == "f32" else torch.bfloat16, device=cuda)
    from oxide_b200._lib import call

    ta, tb = to_dev(a), to_dev(b)  # keep both alive across the call
    call(f"oxide_binary_{dtype}", op, ta.data_ptr(), na, tb.data_ptr(), nb, out.data_ptr(), n, None)
    torch.cuda.synchronize()
    assert_bits_equal(to_np(out), ref)
    if nb < na == n:
        # tensor-level API with reference broadcasting: [rows, cols] op [cols]
        got = ops.binary(op, to_dev(a).view(n // nb, nb), to_dev(b))
        assert_bits_equal(to_np(got).reshape(-1), ref)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_binary_misaligned_pointers(cuda, orc, dtype):
    from oxide_b200._lib import call

    n = 4099
    a, b = rand(n, 3, dtype, orc=orc), rand(n, 4, dtype, orc=orc)
    ta, tb = misaligned_copy(a), misaligned_copy(b)
    out = misaligned_copy(np.zeros_like(a))
    call(f"oxide_binary_{dtype}", 0, ta.data_ptr(), n, tb.data_ptr(), n, out.data_ptr(), n, None)
    torch.cuda.synchronize()
    assert_bits_equal(to_np(out), orc.binary(0, a, b, n))


def test_named_binary_wrappers(cuda, orc):
    from oxide_b200._lib import call

    rows, cols = 300, 4096
    a, b = rand((rows, cols), 5), rand((rows, cols), 6)
    s = np.random.default_rng(7).uniform(0.5, 1.5, cols).astype(F)
    ta, tb, ts = to_dev(a), to_dev(b), to_dev(s)
    out = torch.empty_like(ta)
    for name, op in (("oxide_add_f32", 0), ("oxide_sub_f32", 1), ("oxide_div_f32", 3)):
        call(name, ta.data_ptr(), tb.data_ptr(), out.data_ptr(), a.size, None)
        torch.cuda.synchronize()
        assert_bits_equal(to_np(out), orc.binary(op, a, b))
    call("oxide_mul_rowbcast_f32", ta.data_ptr(), ts.data_ptr(), out.data_ptr(), rows, cols, None)
    torch.cuda.synchronize()
    assert_bits_equal(to_np(out), orc.binary(2, a, s, a.size))
    ab, bb, sb = orc.f32_to_bf16(a), orc.f32_to_bf16(b), orc.f32_to_bf16(s)
    tab, tbb, tsb = to_dev(ab), to_dev(bb), to_dev(sb)
    outb = torch.empty_like(tab)
    call("oxide_add_bf16", tab.data_ptr(), tbb.data_ptr(), outb.data_ptr(), a.size, None)
    torch.cuda.synchronize()
    assert_bits_equal(to_np(outb), orc.binary(0, ab, bb))
    call("oxide_mul_rowbcast_bf16", tab.data_ptr(), tsb.data_ptr(), outb.data_ptr(), rows, cols, None)
    torch.cuda.synchronize()
    assert_bits_equal(to_np(outb), orc.binary(2, ab, sb, a.size))


def test_in_place_add(cuda, orc):
    from oxide_b200._lib import call

    a, b = rand(1 << 20, 8), rand(1 << 20, 9)
    ta, tb = to_dev(a), to_dev(b)
    call("oxide_add_f32", ta.data_ptr(), tb.data_ptr(), ta.data_ptr(), a.size, None)
    torch.cuda.synchronize()
    assert_bits_equal(to_np(ta), orc.binary(0, a, b))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_scale(cuda, orc, dtype):
    from oxide_b200 import ops

    x = rand(12345, 10, dtype, orc=orc)
    got = ops.scale(to_dev(x), 0.0883883)
    assert_bits_equal(to_np(got), orc.scale(x, 0.0883883))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(64, 4096), (7, 33), (3, 8), (1, 100000)])
def test_add_mul_rowbcast_bit_exact(cuda, orc, dtype, rows, cols):
    """(a + b) * s[col] in one pass: bit-equal to the oracle's add then
    row-broadcast mul and to the device's own two ops; cols = 33 takes the
    element kernel; in place over a."""
    from oxide_b200 import ops

    a, b = rand((rows, cols), 60, dtype, orc=orc), rand((rows, cols), 61, dtype, orc=orc)
    sv = np.random.default_rng(62).uniform(0.5, 1.5, cols).astype(F)
    if dtype == "bf16":
        sv = orc.f32_to_bf16(sv)
    ta, tb, ts = to_dev(a), to_dev(b), to_dev(sv)
    got = to_np(ops.add_mul_rowbcast(ta, tb, ts))
    h = orc.binary(orc.ADD, a.reshape(-1), b.reshape(-1))
    ref = orc.binary(orc.MUL, h, sv).reshape(rows, cols)
    assert_bits_equal(got, ref)
    assert_bits_equal(got, to_np(ops.mul_rowbcast(ops.add(ta, tb), ts)))
    ops.add_mul_rowbcast(ta, tb, ts, out=ta)
    assert_bits_equal(to_np(ta), got)
    ta = to_dev(a)
    ops.add_mul_rowbcast(ta, tb, ts, out=tb)  # in place over b
    assert_bits_equal(to_np(tb), got)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("which", ["b", "s", "out"])
def test_add_mul_rowbcast_one_misaligned_operand(cuda, orc, dtype, which):
    """One operand one element off a 16-byte boundary while the others are
    aligned: the entry point must take the element kernel for that alone."""
    from oxide_b200 import ops

    rows, cols = 48, 4096
    a, b = rand((rows, cols), 63, dtype, orc=orc), rand((rows, cols), 64, dtype, orc=orc)
    sv = np.random.default_rng(65).uniform(0.5, 1.5, cols).astype(F)
    if dtype == "bf16":
        sv = orc.f32_to_bf16(sv)
    ta = to_dev(a)
    tb = misaligned_copy(b) if which == "b" else to_dev(b)
    ts = misaligned_copy(sv) if which == "s" else to_dev(sv)
    out = misaligned_copy(np.zeros_like(a)) if which == "out" else None
    got = to_np(ops.add_mul_rowbcast(ta, tb, ts, out=out))
    ref = orc.binary(orc.MUL, orc.binary(orc.ADD, a.reshape(-1), b.reshape(-1)), sv).reshape(rows, cols)
    assert_bits_equal(got, ref)


# ---------------------------------------------------------------- activations
@pytest.mark.parametrize("n", [1, 7, 4096, 1 << 20, (1 << 20) + 3])
def test_silu_mul_f32(cuda, orc, n):
    from oxide_b200 import ops

    g, u = rand(n, 11, scale=4.0), rand(n, 12)
    got = to_np(ops.silu_mul(to_dev(g), to_dev(u)))
    assert_silu_f32_parity(got, orc.silu_mul(g, u), g, orc)
    got = ops.silu(to_dev(g))
    assert_silu_f32_parity(to_np(got), orc.silu(g), g, orc)


@pytest.mark.parametrize("n", [9, 1 << 20])
def test_silu_mul_bf16(cuda, orc, n):
    from oxide_b200 import ops

    g, u = rand(n, 13, "bf16", 4.0, orc), rand(n, 14, "bf16", orc=orc)
    got = ops.silu_mul(to_dev(g), to_dev(u))
    assert_ulp(to_np(got), orc.silu_mul(g, u), BF16_ULP)
    assert_ulp(to_np(ops.silu(to_dev(g))), orc.silu(g), BF16_ULP)


def test_silu_mul_bf16_subnormal_and_special(cuda, orc):
    """bf16 silu * up where the product is a bf16 subnormal (gates near -90,
    small up values), and NaN / +-inf / +-0 operands: within 1 bf16 ulp of the
    reference (the packed product rounds once where the reference's f32
    multiply rounds a subnormal product twice), NaN where the reference has
    NaN."""
    from oxide_b200 import ops
    from _util import ulp_bf16

    rng = np.random.default_rng(17)
    n = 1 << 16
    g = rng.uniform(-100.0, -80.0, n).astype(F)
    u = (rng.uniform(1e-3, 1.0, n) * rng.choice([-1.0, 1.0], n)).astype(F)
    special = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1.0, -1.0, 3.0], F)
    g[:64] = np.repeat(special, 8)
    u[:64] = np.tile(special, 8)
    gb, ub = orc.f32_to_bf16(g), orc.f32_to_bf16(u)
    got = to_np(ops.silu_mul(to_dev(gb), to_dev(ub)))
    ref = orc.silu_mul(gb, ub)
    gn, rn = np.isnan(bf16_to_f32(got)), np.isnan(bf16_to_f32(ref))
    assert np.array_equal(gn, rn)
    assert ulp_bf16(got[~gn], ref[~rn]).max(initial=0) <= BF16_ULP
    mag = np.abs(bf16_to_f32(got))
    assert np.count_nonzero((mag > 0) & (mag < np.float32(2.0 ** -126))) > 100  # subnormals exercised


def test_silu_extremes(cuda, orc):
    from oxide_b200 import ops

    x = np.array([0.0, -0.0, -100.0, 100.0, -88.0, 88.0, 1e-30, -1e-30], dtype=F)
    got = to_np(ops.silu(to_dev(x)))
    assert_silu_f32_parity(got, orc.silu(x), x, orc)


def test_silu_f32_every_float(cuda, orc):
    """oxide_silu_f32 over every f32 bit pattern against the oracle's silu
    (glibc expf, as the reference's f32::exp): the reference's bits wherever
    its expf is correctly rounded, within 2^-21 relative elsewhere, NaN
    exactly where the oracle has NaN."""
    from oxide_b200._lib import call

    chunk = 1 << 28
    threads = orc.max_threads()
    out = torch.empty(chunk, dtype=torch.float32, device=cuda)
    differ = libmiss = 0
    for c in range((1 << 32) // chunk):
        x = np.arange(c * chunk, (c + 1) * chunk, dtype=np.uint32).view(np.float32)
        tx = torch.from_numpy(x).to(cuda)
        call("oxide_silu_f32", tx.data_ptr(), out.data_ptr(), chunk, None)
        got = out.cpu().numpy()
        d, m = assert_silu_f32_parity(got, orc.silu(x, threads=threads), x, orc, threads)
        differ, libmiss = differ + d, libmiss + m
        del tx
    assert differ <= libmiss  # differences only where the reference's exp misrounds


def _silu_host_lib():
    """tests/cpp/silu_host.cu built as a shared library (nvcc, host code only)."""
    import ctypes
    import os
    import subprocess

    from conftest import PKG, ROOT

    src = os.path.join(ROOT, "tests", "cpp", "silu_host.cu")
    so = os.path.join(ROOT, "tests", "cpp", "_build", "libsilu_host.so")
    hdr = os.path.join(PKG, "csrc", "oxide_common.cuh")
    if not os.path.exists(so) or os.path.getmtime(so) < max(os.path.getmtime(src), os.path.getmtime(hdr)):
        os.makedirs(os.path.dirname(so), exist_ok=True)
        subprocess.run(["/usr/local/cuda/bin/nvcc", "-O2", "-std=c++17", "-x", "cu", "-shared",
                        "-gencode", "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "include"),
                        "-I", os.path.join(PKG, "csrc"), "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off",
                        "-o", so, src, "-lgomp"], check=True, timeout=600)
    lib = ctypes.CDLL(so)
    lib.silu_bits_host.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p]
    lib.silu_bits_host.restype = None
    return lib


def test_silu_f32_device_bits_equal_host_build(cuda):
    """The f32 SiLU kernels (the vector path: the paired f32 exponential, its
    rounding test and the fix-ups of undecided elements; silu * up with up = 1;
    and the scalar path of a misaligned view) against the host build of the
    same arithmetic, bit for bit, on every 16th f32 bit pattern: the device
    must compute exactly the operations written."""
    from oxide_b200 import ops

    lib = _silu_host_lib()
    stride, n = 16, 1 << 24
    ones = torch.ones(n, dtype=torch.float32, device=cuda)
    for c in range((1 << 32) // (stride * n)):
        first = c * stride * n
        host = np.empty(n, dtype=F)
        lib.silu_bits_host(first, stride, n, host.ctypes.data)
        x = (first + np.arange(n, dtype=np.uint64) * stride).astype(np.uint32).view(F)
        tx = torch.from_numpy(x).to(cuda)
        outs = [to_np(ops.silu(tx)), to_np(ops.silu_mul(tx, ones))]
        if c == 0:
            buf = torch.empty(n + 1, dtype=torch.float32, device=cuda)
            buf[1:].copy_(tx)
            outs.append(to_np(ops.silu(buf[1:])))  # 4-byte offset: the scalar kernel
        nan = np.isnan(host)
        for got in outs:
            assert np.array_equal(np.isnan(got), nan)
            bad = np.nonzero(got[~nan].view(np.uint32) != host[~nan].view(np.uint32))[0]
            assert bad.size == 0, f"{bad.size} differ from the host build, e.g. x = {x[~nan][bad[:4]]}"


def test_fused_silu_mul_equals_unfused(cuda, orc):
    """silu then mul (two kernels) == the fused kernel, bit for bit, both dtypes
    (bf16 products away from the subnormal range, where the fused kernel's
    single rounding can differ by one ulp from the f32 multiply's two)."""
    from oxide_b200 import ops

    for dtype in ("f32", "bf16"):
        g, u = rand(1 << 18, 15, dtype, 3.0, orc), rand(1 << 18, 16, dtype, orc=orc)
        tg, tu = to_dev(g), to_dev(u)
        fused = to_np(ops.silu_mul(tg, tu))
        unfused = to_np(ops.mul(ops.silu(tg), tu))
        assert_bits_equal(fused, unfused)


# ---------------------------------------------------------------- RMSNorm
NORM_SHAPES = [(1, 1), (3, 17), (7, 128), (64, 4096), (33, 5000), (2, 65536), (2, 70000)]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", NORM_SHAPES)
def test_rms_norm(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    x = rand((rows, cols), 20 + cols, dtype, orc=orc)
    w = np.random.default_rng(21).uniform(0.5, 1.5, cols).astype(F)
    w = w if dtype == "f32" else orc.f32_to_bf16(w)
    got = ops.rms_norm(to_dev(x), to_dev(w), 1e-5)
    ref = orc.rms_norm(x, w, 1e-5)
    if dtype == "f32":
        assert_parity_rel(to_np(got), ref, rms_norm_exact(x, w, 1e-5), F32_REL)
    else:
        assert_ulp(to_np(got), ref, BF16_ULP)


def test_rms_norm_misaligned(cuda, orc):
    from oxide_b200 import ops

    x = rand((5, 256), 22)
    w = np.random.default_rng(23).uniform(0.5, 1.5, 256).astype(F)
    tx = misaligned_copy(x)
    got = ops.rms_norm(tx, to_dev(w), 1e-6)
    assert_close_rel(to_np(got), orc.rms_norm(x, w, 1e-6), F32_REL)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(3, 17), (128, 4096), (2, 70000)])
def test_add_rms_norm(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    x = rand((rows, cols), 24, dtype, orc=orc)
    r = rand((rows, cols), 25, dtype, orc=orc)
    w = np.ones(cols, F) if dtype == "f32" else orc.f32_to_bf16(np.ones(cols, F))
    h, y = ops.add_rms_norm(to_dev(x), to_dev(r), to_dev(w), 1e-5)
    rh, ry = orc.add_rms_norm(x, r, w, 1e-5)
    assert_bits_equal(to_np(h), rh)
    close(to_np(y), ry, dtype)
    # the fused kernel equals add followed by rms_norm on the device: h bit for
    # bit; y too in bf16, where both kernels hold 32 elements per thread and
    # so reduce in the same order (the fused f32 kernel holds 16, so its sum
    # of squares may round differently: within tolerance of the reference)
    h2 = ops.add(to_dev(x), to_dev(r))
    y2 = ops.rms_norm(h2, to_dev(w), 1e-5)
    assert_bits_equal(to_np(h), to_np(h2))
    if dtype == "bf16":
        assert_bits_equal(to_np(y), to_np(y2))


def test_add_rms_norm_in_place_residual(cuda, orc):
    from oxide_b200 import ops

    x, r = rand((64, 4096), 26, "bf16", orc=orc), rand((64, 4096), 27, "bf16", orc=orc)
    w = orc.f32_to_bf16(np.random.default_rng(28).uniform(0.5, 1.5, 4096).astype(F))
    tx = to_dev(x)
    h, y = ops.add_rms_norm(tx, to_dev(r), to_dev(w), 1e-5, h=tx)
    rh, ry = orc.add_rms_norm(x, r, w, 1e-5)
    assert_bits_equal(to_np(tx), rh)
    assert_ulp(to_np(y), ry, BF16_ULP)


# ---------------------------------------------------------------- softmax
SMAX_SHAPES = [(5, 1), (8, 33), (16, 128), (4, 2048), (4, 4096), (6, 6000), (3, 32768),
               (2, 100000), (1, 200000)]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", SMAX_SHAPES)
def test_softmax_rows(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    x = rand((rows, cols), 30 + cols, dtype, 3.0, orc)
    got = ops.softmax(to_dev(x), 1)
    smax_close(to_np(got), orc.softmax(x, rows, cols, 1), x, cols, dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_softmax_inner_dim(cuda, orc, dtype):
    from oxide_b200 import ops

    x = rand((3, 50, 7), 31, dtype, 2.0, orc)
    got = ops.softmax(to_dev(x), 1)
    close(to_np(got), orc.softmax(x, 3, 50, 7).reshape(3, 50, 7), dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_masked_softmax_lens(cuda, orc, dtype):
    """C3 shape family: [batch x heads x 1 x keys] with per-batch KV lengths."""
    from oxide_b200 import ops

    batch, heads, keys = 4, 8, 32768
    x = rand((batch, heads, 1, keys), 32, dtype, float(np.sqrt(128.0)), orc)
    lens = np.array([1024, 32768, 5000, 0], dtype=np.int32)  # includes a fully masked batch
    scale = float(F(1.0) / np.sqrt(F(128)))
    got = ops.scale_mask_softmax(to_dev(x), scale, lens=to_dev(lens), rows_per_len=heads)
    ref = orc.scale_mask_softmax(x, keys, scale, lens=lens, rows_per_len=heads)
    smax_close(to_np(got), ref, x, keys, dtype, scale, lens=lens, rows_per_len=heads)
    g = to_np(got).reshape(batch * heads, keys)
    if dtype == "f32":
        assert np.all(g[-heads:] == 0)  # len 0 -> zeros
        assert np.all(g[:heads, 1024:] == 0)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_additive_mask_softmax(cuda, orc, dtype):
    from oxide_b200 import ops

    rows, cols = 12, 1000
    x = rand((rows, cols), 33, dtype, 5.0, orc)
    mask = np.where(np.random.default_rng(34).random(cols) < 0.3, -np.inf, 0.25).astype(F)
    got = ops.scale_mask_softmax(to_dev(x), 0.125, mask=to_dev(mask))
    smax_close(to_np(got), orc.scale_mask_softmax(x, cols, 0.125, mask=mask), x, cols, dtype,
               0.125, mask=mask)
    # a short mask repeats (mask[j % mask_len])
    short = np.array([0.0, -1.0, -np.inf], F)
    got = ops.scale_mask_softmax(to_dev(x), 0.125, mask=to_dev(short))
    smax_close(to_np(got), orc.scale_mask_softmax(x, cols, 0.125, mask=short), x, cols, dtype,
               0.125, mask=short)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_long_row_softmax_masked_prefix_nan_and_inf(cuda, orc, dtype):
    """Rows longer than a CTA's register tile (streamed in slices): an
    additive mask whose first 5000 keys are -inf (slices that see only -inf
    add nothing), a NaN key and a +inf key (their rows are all NaN, like the
    reference's), a row of -inf scores (NaN), and lengths that end inside a
    slice."""
    from oxide_b200 import ops

    rows, cols = 8, 20000
    x = rand((rows, cols), 37, dtype, 4.0, orc)
    nan, inf, ninf = (0x7FC0, 0x7F80, 0xFF80) if dtype == "bf16" else (np.nan, np.inf, -np.inf)
    x[1, 12345] = nan
    x[2, 7] = inf
    x[3, :] = ninf
    mask = np.full(cols, 0.5, F)
    mask[:5000] = -np.inf
    got = ops.scale_mask_softmax(to_dev(x), 0.125, mask=to_dev(mask))
    ref = orc.scale_mask_softmax(x, cols, 0.125, mask=mask)
    if dtype == "bf16":
        from _util import ulp_bf16

        gn, rn = np.isnan(bf16_to_f32(to_np(got))), np.isnan(bf16_to_f32(ref))
        assert np.array_equal(gn, rn)
        assert ulp_bf16(to_np(got)[~gn], ref[~rn]).max(initial=0) <= BF16_ULP
    else:
        smax_close(to_np(got), ref, x, cols, dtype, 0.125, mask=mask)
    lens = np.array([20000, 5001, 4999, 1], np.int32)
    got = ops.scale_mask_softmax(to_dev(x), 0.125, lens=to_dev(lens), rows_per_len=2)
    ref = orc.scale_mask_softmax(x, cols, 0.125, lens=lens, rows_per_len=2)
    if dtype == "bf16":
        gn, rn = np.isnan(bf16_to_f32(to_np(got))), np.isnan(bf16_to_f32(ref))
        assert np.array_equal(gn, rn)
        assert ulp_bf16(to_np(got)[~gn], ref[~rn]).max(initial=0) <= BF16_ULP
    else:
        smax_close(to_np(got), ref, x, cols, dtype, 0.125, lens=lens, rows_per_len=2)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("q_len,cols", [(256, 256), (64, 300), (2048, 2048)])
def test_causal_softmax(cuda, orc, dtype, q_len, cols):
    """C5 shape family: [seqs x heads x q_len x keys] with a causal mask."""
    from oxide_b200 import ops

    rows = 2 * q_len
    x = rand((rows, cols), 35 + cols, dtype, 4.0, orc)
    got = ops.scale_mask_softmax(to_dev(x), 0.0883883, causal_q_len=q_len)
    smax_close(to_np(got), orc.scale_mask_softmax(x, cols, 0.0883883, causal_q_len=q_len), x,
               cols, dtype, 0.0883883, causal_q=q_len)


@pytest.mark.parametrize("cols", [8, 40, 256, 264, 1024, 2048])
def test_bf16_softmax_short_rows_edge_cases(cuda, orc, cols):
    """bf16 rows of whole 8-key vectors up to 2048 keys: scores spread so wide
    that exp underflows to subnormals and zero, ragged lengths (0, 1, partial
    vectors, full), and rows with NaN, +inf and all -inf keys."""
    from oxide_b200 import ops
    from _util import bf16_to_f32, ulp_bf16

    rows = 64
    x = rand((rows, cols), 40 + cols, "bf16", 30.0, orc)
    x[5, 3 % cols] = 0x7FC0          # NaN key: the row is NaN
    x[6, 7 % cols] = 0x7F80          # +inf key: NaN like the reference (inf - inf)
    x[7, :] = 0xFF80                 # all -inf: NaN like the reference
    lens = np.random.default_rng(cols).integers(0, cols + 1, rows // 2).astype(np.int32)
    lens[:4] = [0, cols, 1, max(cols - 3, 1)]
    for kw in ({"lens": lens, "rows_per_len": 2}, {"causal_q_len": min(cols, 16)}, {}):
        dev_kw = {k: (to_dev(v) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}
        got = to_np(ops.scale_mask_softmax(to_dev(x), 1.0, **dev_kw))
        ref = orc.scale_mask_softmax(x, cols, 1.0, **kw)
        gn, rn = np.isnan(bf16_to_f32(got)), np.isnan(bf16_to_f32(ref))
        assert np.array_equal(gn, rn), kw
        d = ulp_bf16(got[~gn], ref[~rn])
        assert d.max(initial=0) <= BF16_ULP, (kw, d.max())


def test_softmax_rows_sum_to_one_and_deterministic(cuda, orc):
    from oxide_b200 import ops

    x = to_dev(rand((256, 32768), 36, scale=11.3))
    p1 = ops.softmax(x, 1)
    p2 = ops.softmax(x, 1)
    assert torch.equal(p1, p2)
    assert torch.allclose(p1.double().sum(1), torch.ones(256, dtype=torch.float64, device=cuda),
                          atol=1e-5)


def test_all_neg_inf_additive_mask_is_nan_like_reference(cuda, orc):
    from oxide_b200 import ops

    x = to_dev(np.zeros((2, 64), F))
    got = to_np(ops.scale_mask_softmax(x, 1.0, mask=to_dev(np.full(64, -np.inf, F))))
    assert np.all(np.isnan(got))


# ---------------------------------------------------------------- RoPE
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("layout", ["token", "head"])
def test_rope(cuda, orc, dtype, layout):
    from oxide_b200 import ops

    tokens, qh, kh, d = 300, 8, 2, 128
    cos, sin = orc.rope_table(1e6, d, 512)
    shape_q = (tokens, qh, d) if layout == "token" else (qh, tokens, d)
    shape_k = (tokens, kh, d) if layout == "token" else (kh, tokens, d)
    q, k = rand(shape_q, 40, dtype, orc=orc), rand(shape_k, 41, dtype, orc=orc)
    pos = np.random.default_rng(42).integers(0, 512, tokens).astype(np.int32)
    tq, tk = ops.rope(to_dev(q), to_dev(k), to_dev(cos), to_dev(sin), to_dev(pos), layout)
    lay = 0 if layout == "token" else 1
    assert_bits_equal(to_np(tq), orc.rope(q, tokens, qh, d, lay, cos, sin, pos))
    assert_bits_equal(to_np(tk), orc.rope(k, tokens, kh, d, lay, cos, sin, pos))


def test_rope_in_place_no_positions_no_k(cuda, orc):
    from oxide_b200 import ops

    tokens, h, d = 64, 4, 64
    cos, sin = orc.rope_table(1e4, d, tokens)
    q = rand((tokens, h, d), 43, "bf16", orc=orc)
    tq = to_dev(q)
    ops.rope(tq, None, to_dev(cos), to_dev(sin), q_out=tq)
    assert_bits_equal(to_np(tq), orc.rope(q, tokens, h, d, 0, cos, sin))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_rope_vector_path_ragged_group_many_heads_bad_position(cuda, orc, dtype):
    """The vector kernel with an odd token count (a token group cut short),
    more (head, chunk) items per token than threads (the item loop), q and k
    rotated in place, and one position beyond the table (that token NaN)."""
    from oxide_b200 import ops

    tokens, qh, kh, d = 301, 64, 16, 128
    cos, sin = orc.rope_table(1e6, d, 400)
    q, k = rand((tokens, qh, d), 46, dtype, orc=orc), rand((tokens, kh, d), 47, dtype, orc=orc)
    pos = np.random.default_rng(48).integers(0, 400, tokens).astype(np.int32)
    pos[tokens - 1] = 400
    tq, tk = to_dev(q), to_dev(k)
    ops.rope(tq, tk, to_dev(cos), to_dev(sin), to_dev(pos), q_out=tq, k_out=tk)
    okpos = np.where(pos == 400, 0, pos)
    for got, x, h in ((to_np(tq), q, qh), (to_np(tk), k, kh)):
        ref = orc.rope(x, tokens, h, d, 0, cos, sin, okpos)
        gf = bf16_to_f32(got) if dtype == "bf16" else got
        assert np.all(np.isnan(gf[tokens - 1]))
        assert_bits_equal(got[: tokens - 1], ref[: tokens - 1])


def test_apply_rotary_emb_reference_layout(cuda, orc):
    """ops::apply_rotary_emb: x [batch, heads, seq, d] with tables [seq, half]."""
    from oxide_b200 import ops

    b, h, s, d = 2, 3, 40, 32
    cos, sin = orc.rope_table(1e4, d, s)
    x = rand((b, h, s, d), 44)
    got = ops.apply_rotary_emb(to_dev(x), to_dev(cos), to_dev(sin))
    assert_bits_equal(to_np(got), orc.rope(x, s, b * h, d, 1, cos, sin))


def test_rope_unaligned_head_dim_and_bad_position(cuda, orc):
    from oxide_b200 import ops

    tokens, h, d = 10, 3, 6  # half = 3: scalar kernel
    cos, sin = orc.rope_table(1e4, d, 16)
    q = rand((tokens, h, d), 45)
    pos = np.arange(tokens, dtype=np.int32)
    pos[4] = 99  # beyond the table -> NaN for that token, no out-of-bounds read
    got = to_np(ops.rope(to_dev(q), None, to_dev(cos), to_dev(sin), to_dev(pos)))
    ref = orc.rope(q, tokens, h, d, 0, cos, sin, np.where(pos == 99, 0, pos))
    assert np.all(np.isnan(got[4]))
    keep = np.arange(tokens) != 4
    assert_bits_equal(got[keep], ref[keep])


# ---------------------------------------------------------------- argmax
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(64, 32000), (1000, 100), (3, 7), (1, 1), (2, 300001)])
def test_argmax(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    x = rand((rows, cols), 50 + cols, dtype, orc=orc)
    got = ops.argmax(to_dev(x))
    assert np.array_equal(to_np(got).astype(np.uint32), orc.argmax_rows(x, cols))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("cols", [4096, 32000, 40000])  # 256-thread CTAs / clusters, one 1024-thread CTA per row
def test_argmax_ties_nan_signed_zero(cuda, orc, dtype, cols):
    from oxide_b200 import ops

    x = np.random.default_rng(51).standard_normal((6, cols), dtype=F)
    x[0, [5, 77, cols - 96]] = 50.0                 # tie, the last one in another CTA's part
    x[1] = -0.0
    x[1, 9] = 0.0                                    # -0 == +0 -> index 0
    x[2] = np.nan
    x[2, 1234] = -np.inf                             # NaN below everything
    x[3] = np.nan                                    # all NaN -> 0
    x[4, cols - 1] = np.inf
    x[5] = -np.inf
    if dtype == "bf16":
        x = orc.f32_to_bf16(x).reshape(x.shape)
    got = to_np(ops.argmax(to_dev(x))).astype(np.uint32)
    assert np.array_equal(got, orc.argmax_rows(x, cols))
    assert got.tolist()[:5] == [5, 0, 1234, 0, cols - 1]


def test_argmax_misaligned(cuda, orc):
    from oxide_b200 import ops

    x = rand((5, 1000), 52)
    got = ops.argmax(misaligned_copy(x))
    assert np.array_equal(to_np(got).astype(np.uint32), orc.argmax_rows(x, 1000))


# ---------------------------------------------------------------- reductions
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(1, 1), (17, 333), (64, 4096), (4, 100000)])
def test_reduce_rows(cuda, orc, dtype, rows, cols):
    from oxide_b200 import ops

    x = rand((rows, cols), 60 + cols, dtype, orc=orc)
    xf = (x if dtype == "f32" else bf16_to_f32(x).reshape(rows, cols)).astype(np.float64)
    scale = np.sum(np.abs(xf), axis=1) + 1e-30  # sums of signed terms: relative to sum |x|
    for op in (0, 1, 2):
        got = to_np(ops.reduce_rows(to_dev(x), op)).astype(np.float64)
        ref = orc.reduce_rows(op, x, cols).astype(np.float64)
        if op == 1:
            assert_bits_equal(got.astype(F), ref.astype(F))
            continue
        exact = np.sum(xf, axis=1) if op == 0 else np.sum(xf * xf, axis=1)
        lim = F32_REL * (scale if op == 0 else exact)
        # within 1e-5 of the exact sum, and of the reference's sequential f32
        # sum up to that sum's own drift from exact
        assert np.all(np.abs(got - exact) <= lim)
        assert np.all(np.abs(got - ref) <= lim + np.abs(ref - exact))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("n", [1, 12345, 1 << 20, 10_000_003])
def test_reduce_global(cuda, orc, dtype, n):
    from oxide_b200 import ops

    x = rand(n, 70 + n % 97, dtype, orc=orc)
    tx = to_dev(x)
    absum = float(np.sum(np.abs((x if dtype == "f32" else bf16_to_f32(x)).astype(np.float64))))
    for op in (0, 1, 2):
        got = float(ops.reduce(tx, op).item())
        ref = orc.reduce(op, x)
        if op == 1:
            assert got == ref
        elif op == 0:
            assert abs(got - ref) <= F32_REL * absum
        else:
            assert abs(got - ref) <= F32_REL * abs(ref)
    # deterministic: the same bits on a second run
    a = ops.reduce(tx, 2)
    b = ops.reduce(tx, 2)
    assert a.item() == b.item()


def test_reduce_global_misaligned_and_empty(cuda, orc):
    from oxide_b200 import ops

    x = rand(100001, 80)
    got = float(ops.reduce(misaligned_copy(x), 2).item())
    assert abs(got - orc.reduce(2, x)) <= F32_REL * orc.reduce(2, x)
    e = torch.empty(0, dtype=torch.float32, device=cuda)
    assert float(ops.reduce(e, 0).item()) == 0.0
    assert float(ops.reduce(e, 1).item()) == float("-inf")


# ---------------------------------------------------------------- status on the GPU path
def test_injected_failure_does_not_launch(cuda, orc):
    from oxide_b200 import _lib, ops

    x = to_dev(rand((4, 64), 90))
    w = to_dev(np.ones(64, F))
    out = torch.full_like(x, 7.0)
    _lib.lib().oxide_debug_fail_next(b"oxide_rms_norm_f32")
    with pytest.raises(_lib.OxideError) as e:
        ops.rms_norm(x, w, 1e-5, out=out)
    assert e.value.status == _lib.ERR_INJECTED
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing ran
    ops.rms_norm(x, w, 1e-5, out=out)  # next call runs normally
    torch.cuda.synchronize()
    assert not torch.all(out == 7.0)


# ---------------------------------------------------------------- row-shared division
def test_rowdiv_matches_ieee_division(cuda):
    """RowDiv (RN reciprocal + two FMA residual corrections) returns the IEEE
    quotient: random numerators/divisors over the ranges RMSNorm and softmax
    use, adversarial divisors (all-ones significands, powers of two, values
    near 1), the fallback ranges (0, subnormal, huge, inf, NaN)."""
    from oxide_b200._lib import call

    rng = np.random.default_rng(123)
    a = np.concatenate([
        rng.standard_normal(1 << 20).astype(F) * F(3),                       # RMSNorm numerators
        rng.random(1 << 20).astype(F),                                        # softmax e in [0, 1)
        np.exp(rng.uniform(-80, 0, 1 << 18)).astype(F),                       # small e
        (rng.integers(1, 1 << 24, 1 << 16) * F(2.0) ** rng.integers(-40, 40, 1 << 16)).astype(F),
        np.array([0.0, -0.0, 1e-40, -1e-40, 2.0 ** -61, 2.0 ** 61, np.inf, -np.inf, np.nan,
                  3.4e38, 1.0, 1.0 - 2 ** -24], dtype=F),
    ]).astype(F)
    ones = (np.array([0x3F7FFFFF, 0x3FFFFFFF, 0x407FFFFF, 0x4F7FFFFF], dtype=np.uint32)).view(F)
    b = np.concatenate([
        np.exp(rng.uniform(-5.8, 6.0, 200)).astype(F),   # rms in [sqrt(eps)..], sums up to ~400
        rng.uniform(1.0, 32768.0, 200).astype(F),          # softmax sums
        ones, np.array([1.0, 2.0, 0.5, 1.0 + 2 ** -23, 2.0 - 2 ** -22, 3.0, 7.0, 1e-3], F),
        np.array([0.0, 1e-40, 2.0 ** 70, np.inf, np.nan], F),
    ]).astype(F)
    # every subnormal numerator, both signs, against divisors across the range
    sub = np.arange(1, 1 << 23, dtype=np.uint32)
    a2 = np.concatenate([sub, sub | 0x80000000]).view(F)
    b2 = np.concatenate([np.exp(rng.uniform(-41.0, 41.0, 48)).astype(F), ones,
                         np.array([1.0, 3.0, 0.75, 2.0 ** -60, 2.0 ** 60], F)]).astype(F)
    for aa, bb in ((a, b), (a2, b2)):
        ta, tb = to_dev(aa), to_dev(bb)
        out = torch.tensor([0, -1], dtype=torch.int64, device=cuda)  # {0, UINT64_MAX}
        call("oxide_selftest_rowdiv", ta.data_ptr(), aa.size, tb.data_ptr(), bb.size,
             out.data_ptr(), None)
        torch.cuda.synchronize()
        count, first = out.cpu().tolist()
        assert count == 0, \
            f"{count} mismatches; first pair a={aa[first // bb.size]!r} b={bb[first % bb.size]!r}"
