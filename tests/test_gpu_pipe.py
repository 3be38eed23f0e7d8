"""Host-buffer pipeline (oxide_pipe_*): results equal the oracle (and the
device-buffer entry points) for pageable and page-locked host memory, across
many chunks and a ragged last chunk."""
import ctypes as C

import numpy as np
import pytest
import torch

from _util import assert_bits_equal, assert_parity_rel, assert_silu_f32_parity, assert_ulp, rms_norm_exact

pytestmark = pytest.mark.gpu
F = np.float32


@pytest.fixture()
def pipe(cuda):
    from oxide_b200._lib import call, lib

    h = C.c_void_p()
    call("oxide_pipe_create", 0, 1 << 20, 3, C.byref(h))  # 1 MiB chunks: many chunks
    yield h
    lib().oxide_pipe_destroy(h)


def host(a, pinned):
    if not pinned:
        return np.ascontiguousarray(a)
    t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    return t.numpy()  # a numpy view of page-locked memory (t kept alive by the view)


@pytest.mark.parametrize("pinned", [False, True])
def test_pipe_binary_and_broadcast(pipe, orc, pinned):
    from oxide_b200._lib import call

    rng = np.random.default_rng(1)
    n = 3 * (1 << 20) + 4096 * 3  # ragged last chunk
    a = host(rng.standard_normal(n, dtype=F), pinned)
    b = host(rng.standard_normal(n, dtype=F), pinned)
    out = host(np.zeros(n, F), pinned)
    call("oxide_pipe_binary_f32", pipe, 0, a.ctypes.data, n, b.ctypes.data, n, out.ctypes.data, n)
    assert_bits_equal(out, orc.binary(0, a, b))
    s = host(rng.uniform(0.5, 1.5, 4096).astype(F), pinned)
    call("oxide_pipe_binary_f32", pipe, 2, a.ctypes.data, n, s.ctypes.data, 4096, out.ctypes.data, n)
    assert_bits_equal(out, orc.binary(2, a, s, n))


@pytest.mark.parametrize("pinned", [False, True])
def test_pipe_silu_mul(pipe, orc, pinned):
    from oxide_b200._lib import call

    rng = np.random.default_rng(2)
    n = 5 * (1 << 18) + 3
    g = host(rng.standard_normal(n, dtype=F) * F(4), pinned)
    u = host(rng.standard_normal(n, dtype=F), pinned)
    out = host(np.zeros(n, F), pinned)
    call("oxide_pipe_silu_mul_f32", pipe, g.ctypes.data, u.ctypes.data, out.ctypes.data, n)
    # identical to the device-buffer entry point
    from oxide_b200 import ops

    dev = ops.silu_mul(torch.from_numpy(np.array(g)).cuda(), torch.from_numpy(np.array(u)).cuda())
    assert_bits_equal(out, dev.cpu().numpy())
    assert_silu_f32_parity(out, orc.silu_mul(g, u), g, orc)


def test_pipe_rms_norm(pipe, orc):
    from oxide_b200._lib import call

    rng = np.random.default_rng(3)
    rows, cols = 300, 4096
    x = rng.standard_normal((rows, cols), dtype=F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    out = np.zeros_like(x)
    call("oxide_pipe_rms_norm_f32", pipe, x.ctypes.data, w.ctypes.data, out.ctypes.data, rows,
         cols, 1e-5)
    assert_parity_rel(out, orc.rms_norm(x, w, 1e-5), rms_norm_exact(x, w, 1e-5), 1e-5)


def test_pipe_rejects_bad_arguments(pipe, olib):
    lib = olib.lib()
    buf = np.zeros(16, F)
    p = buf.ctypes.data
    assert lib.oxide_pipe_binary_f32(pipe, 0, p, 3, p, 16, p, 16) == olib.ERR_INVALID_ARG
    assert lib.oxide_pipe_binary_f32(None, 0, p, 16, p, 16, p, 16) == olib.ERR_INVALID_ARG
    # a row larger than the 1 MiB chunk
    assert lib.oxide_pipe_rms_norm_f32(pipe, p, p, p, 1, 1 << 20, 1e-5) == olib.ERR_UNSUPPORTED


def test_pipe_add_mul_rowbcast_h_and_y(pipe, orc):
    """h = a + b and y = h * s from one upload: both equal the oracle's add then
    row-broadcast mul bit for bit, over many chunks and a ragged last one."""
    from oxide_b200._lib import call

    rng = np.random.default_rng(4)
    rows, cols = 200, 4096  # 16 rows per 1 MiB chunk: 13 chunks
    a, b = rng.standard_normal((rows, cols), dtype=F), rng.standard_normal((rows, cols), dtype=F)
    s = rng.uniform(0.5, 1.5, cols).astype(F)
    h, y = np.zeros_like(a), np.zeros_like(a)
    call("oxide_pipe_add_mul_rowbcast_f32", pipe, a.ctypes.data, b.ctypes.data, s.ctypes.data, h.ctypes.data,
         y.ctypes.data, rows, cols)
    rh = orc.binary(0, a, b)
    assert_bits_equal(h, rh)
    assert_bits_equal(y, orc.binary(2, rh, s, rh.size))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_pipe_add_rms_norm(pipe, orc, dtype):
    from oxide_b200 import ops
    from oxide_b200._lib import call
    from _util import to_dev, to_np

    rng = np.random.default_rng(5)
    rows, cols = 150, 4096
    x, r = rng.standard_normal((rows, cols), dtype=F), rng.standard_normal((rows, cols), dtype=F)
    w = rng.uniform(0.5, 1.5, cols).astype(F)
    if dtype == "bf16":
        x, r, w = orc.f32_to_bf16(x).reshape(rows, cols), orc.f32_to_bf16(r).reshape(rows, cols), orc.f32_to_bf16(w)
    h, y = np.zeros_like(x), np.zeros_like(x)
    call(f"oxide_pipe_add_rms_norm_{dtype}", pipe, x.ctypes.data, r.ctypes.data, w.ctypes.data, h.ctypes.data,
         y.ctypes.data, rows, cols, 1e-5)
    dh, dy = ops.add_rms_norm(to_dev(x), to_dev(r), to_dev(w), 1e-5)
    assert_bits_equal(h, to_np(dh))
    assert_bits_equal(y, to_np(dy))
    rh, ry = orc.add_rms_norm(x, r, w, 1e-5)
    assert_bits_equal(h, rh)
    if dtype == "bf16":
        assert_ulp(y, ry, 1)


@pytest.mark.parametrize("mode", ["lens", "mask", "causal"])
def test_pipe_scale_mask_softmax(pipe, orc, mode):
    """The host form uploads only each group's valid keys with lens; results
    equal the device entry point on the same rows and the oracle's bar."""
    from oxide_b200 import ops
    from oxide_b200._lib import call
    from _util import smax_close, to_dev, to_np

    rng = np.random.default_rng(6)
    rows, cols = 96, 8192  # 32 rows per 1 MiB chunk
    x = (rng.standard_normal((rows, cols), dtype=F) * F(3)).astype(F)
    kw, args = {}, [None, 0, None, 1, 0]
    if mode == "lens":
        lens = np.array([8192, 1, 0, 5000, 4097, 12, 8191, 333], np.int32)  # 12 rows per sequence
        kw, args = {"lens": lens, "rows_per_len": 12}, [None, 0, lens.ctypes.data, 12, 0]
    elif mode == "mask":
        mask = np.where(rng.random(cols) < 0.2, -np.inf, 0.5).astype(F)
        kw, args = {"mask": mask}, [mask.ctypes.data, cols, None, 1, 0]
    else:
        kw, args = {"causal_q_len": 16}, [None, 0, None, 1, 16]
    out = np.full_like(x, np.nan)
    call("oxide_pipe_scale_mask_softmax_f32", pipe, x.ctypes.data, out.ctypes.data, rows, cols, 0.125, *args)
    dev_kw = {k: (to_dev(v) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}
    assert_bits_equal(out, to_np(ops.scale_mask_softmax(to_dev(x), 0.125, **dev_kw)))
    ref = orc.scale_mask_softmax(x, cols, 0.125, **kw)
    smax_close(out, ref, x, cols, "f32", 0.125, mask=kw.get("mask"), lens=kw.get("lens"),
               rows_per_len=kw.get("rows_per_len", 1), causal_q=kw.get("causal_q_len", 0))


def test_pipe_argmax(pipe, orc):
    from oxide_b200._lib import call

    rng = np.random.default_rng(7)
    rows, cols = 100, 32000  # 8 rows per chunk
    x = rng.standard_normal((rows, cols), dtype=F)
    x[3, 100:105] = 50.0  # tie: lowest index wins
    idx = np.zeros(rows, np.uint32)
    call("oxide_pipe_argmax_rows_f32", pipe, x.ctypes.data, rows, cols, idx.ctypes.data)
    assert np.array_equal(idx, orc.argmax_rows(x, cols))
    assert idx[3] == 100


@pytest.mark.parametrize("with_pos", [False, True])
def test_pipe_rope_bf16(pipe, orc, with_pos):
    """q and k over many token chunks; without positions the tables are
    offset per chunk, with positions they are read per token."""
    from oxide_b200._lib import call

    rng = np.random.default_rng(8)
    tokens, qh, kh, d = 600, 32, 8, 128  # 128 tokens per 1 MiB chunk: 5 chunks
    q = orc.f32_to_bf16(rng.standard_normal((tokens, qh, d), dtype=F)).reshape(tokens, qh, d)
    k = orc.f32_to_bf16(rng.standard_normal((tokens, kh, d), dtype=F)).reshape(tokens, kh, d)
    cos, sin = orc.rope_table(1e6, d, 1024)
    pos = rng.integers(0, 1024, tokens).astype(np.int32) if with_pos else None
    qo, ko = np.zeros_like(q), np.zeros_like(k)
    call("oxide_pipe_rope_bf16", pipe, q.ctypes.data, qo.ctypes.data, qh, k.ctypes.data, ko.ctypes.data, kh,
         cos.ctypes.data, sin.ctypes.data, 1024, None if pos is None else pos.ctypes.data, tokens, d)
    assert_bits_equal(qo, orc.rope(q, tokens, qh, d, 0, cos, sin, pos))
    assert_bits_equal(ko, orc.rope(k, tokens, kh, d, 0, cos, sin, pos))


def test_pipe_deferred_ops_overlap_and_keep_their_broadcasts(pipe, orc):
    """Deferred mode: ops return once enqueued and share the streams; each
    op's broadcast operand (a different norm weight per op) must not be
    overwritten while the op before still reads its own."""
    from oxide_b200._lib import call

    rng = np.random.default_rng(9)
    rows, cols = 256, 4096
    xs = [rng.standard_normal((rows, cols), dtype=F) for _ in range(3)]
    ws = [rng.uniform(0.5, 1.5, cols).astype(F) for _ in range(3)]
    outs = [np.zeros_like(x) for x in xs]
    g = rng.standard_normal(rows * cols, dtype=F)
    u = rng.standard_normal(rows * cols, dtype=F)
    o = np.zeros_like(g)
    call("oxide_pipe_defer", pipe, 1)
    for x, w, out in zip(xs, ws, outs):
        call("oxide_pipe_rms_norm_f32", pipe, x.ctypes.data, w.ctypes.data, out.ctypes.data, rows, cols, 1e-5)
        call("oxide_pipe_silu_mul_f32", pipe, g.ctypes.data, u.ctypes.data, o.ctypes.data, g.size)
    call("oxide_pipe_sync", pipe)
    call("oxide_pipe_defer", pipe, 0)
    for x, w, out in zip(xs, ws, outs):
        assert_parity_rel(out, orc.rms_norm(x, w, 1e-5), rms_norm_exact(x, w, 1e-5), 1e-5)
    assert_silu_f32_parity(o, orc.silu_mul(g, u), g, orc)


def test_pipe_new_forms_reject_bad_arguments(pipe, olib):
    lib = olib.lib()
    buf = np.zeros(64, F)
    p = buf.ctypes.data
    # lens groups of 64 rows of 8192 keys (2 MiB) exceed the 1 MiB chunk
    lens = np.array([1], np.int32)
    assert lib.oxide_pipe_scale_mask_softmax_f32(pipe, p, p, 64, 8192, 1.0, None, 0, lens.ctypes.data, 64, 0) \
        == olib.ERR_UNSUPPORTED
    assert lib.oxide_pipe_scale_mask_softmax_f32(pipe, p, p, 4, 16, 1.0, None, 0, lens.ctypes.data, 0, 0) \
        == olib.ERR_INVALID_ARG
    # no positions and fewer table rows than tokens
    assert lib.oxide_pipe_rope_bf16(pipe, p, p, 1, None, None, 0, p, p, 2, None, 4, 8) == olib.ERR_INVALID_ARG
    assert lib.oxide_pipe_add_mul_rowbcast_f32(pipe, p, None, p, p, p, 1, 16) == olib.ERR_INVALID_ARG
    assert lib.oxide_pipe_sync(None) == olib.ERR_INVALID_ARG


def test_pipe_class_equals_device_ops(cuda, orc):
    """oxide_b200.pipe.Pipe: every method bit-identical to the device-tensor op
    of oxide_b200.ops on the same inputs, in immediate and deferred mode."""
    from oxide_b200 import ops
    from oxide_b200.pipe import Pipe

    rng = np.random.default_rng(21)
    rows, cols = 300, 1024
    a, b, g, u = (rng.standard_normal((rows, cols), dtype=F) for _ in range(4))
    s = rng.uniform(0.5, 1.5, cols).astype(F)
    d = lambda x: torch.from_numpy(x).cuda()  # noqa: E731
    h = lambda t: t.cpu().numpy()  # noqa: E731
    with Pipe(0, chunk_bytes=1 << 18, depth=3) as p:
        hh, yy = p.add_mul_rowbcast(a, b, s)
        assert_bits_equal(hh, h(ops.add(d(a), d(b))))
        assert_bits_equal(yy, h(ops.mul_rowbcast(d(hh), d(s))))
        with p.deferred():
            sm = p.silu_mul(g, u)
            rn = p.rms_norm(a, s, 1e-5)
            hx, yx = p.add_rms_norm(a, b, s, 1e-5)
            am = p.argmax_rows(g)
            sx = p.scale_mask_softmax(a, 0.125, lens=rng.integers(0, cols + 1, rows // 4).astype(np.int32),
                                      rows_per_len=4)
        assert_bits_equal(sm, h(ops.silu_mul(d(g), d(u))))
        assert_bits_equal(rn, h(ops.rms_norm(d(a), d(s), 1e-5)))
        hd, yd = ops.add_rms_norm(d(a), d(b), d(s), 1e-5)
        assert_bits_equal(hx, h(hd))
        assert_bits_equal(yx, h(yd))
        assert np.array_equal(am, orc.argmax_rows(g, cols))
        assert np.all(np.isfinite(sx)) and np.allclose(sx.sum(axis=1)[sx.sum(axis=1) > 0], 1, atol=1e-5)
