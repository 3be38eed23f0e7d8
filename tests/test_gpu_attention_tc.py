"""Decode attention on the tcgen05 / TMA kernel (bf16, head_dim 128): against
the exact (f64) attention of src/ops/attention.rs:41-87 with q_len = 1 and
against the split-K mma.sync kernel, at the C3 decode shape and at the edges
of its tile division -- sequences of 0, 1, 127, 128, 129 keys, fewer tiles
than CTAs, many short sequences, every rep, and caches holding NaN past each
sequence's length (never read as values: those keys are masked and their
value rows cleared before the product).

Bar: within 1 bf16 ulp of the exact value rounded to bf16, or within
2^-14 * sum_j p_j |v_j| where the output cancels (P enters the product with
16 significant bits, the scores are exact bf16 products in f32)."""
import numpy as np
import pytest

from _util import bf16_to_f32, to_dev, to_np, ulp_bf16

pytestmark = pytest.mark.gpu
F = np.float32


def _exact(q, kc, vc, lens, scale):
    q, kc, vc = (np.asarray(a, np.float64) for a in (q, kc, vc))
    b, hq, d = q.shape
    rep = hq // kc.shape[1]
    out = np.zeros((b, hq, d))
    mag = np.zeros((b, hq, d))
    for bi in range(b):
        n = kc.shape[2] if lens is None else max(0, min(int(lens[bi]), kc.shape[2]))
        if n == 0:
            continue
        for kh in range(kc.shape[1]):
            k, v = kc[bi, kh, :n], vc[bi, kh, :n]
            qs = q[bi, kh * rep:(kh + 1) * rep]
            s = (qs @ k.T) * np.float64(scale)
            p = np.exp(s - s.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            out[bi, kh * rep:(kh + 1) * rep] = p @ v
            mag[bi, kh * rep:(kh + 1) * rep] = p @ np.abs(v)
    return out, mag


def _attend(q, kc, vc, lens, path):
    import torch

    from oxide_b200 import _lib, ops

    _lib.lib().oxide_debug_decode_attention_path(path)
    try:
        out = ops.decode_attention(to_dev(q), to_dev(kc), to_dev(vc), None if lens is None else to_dev(lens))
        torch.cuda.synchronize()
    finally:
        _lib.lib().oxide_debug_decode_attention_path(0)
    return to_np(out)


def _check(got, exact, mag, what):
    g = bf16_to_f32(got).astype(np.float64)
    want = np.asarray(exact, np.float32)
    from oracle import oracle as orc

    d = ulp_bf16(got, orc.f32_to_bf16(want).reshape(got.shape))
    ok = (d <= 1) | (np.abs(g - exact) <= 2.0 ** -14 * mag + 1e-30)
    assert np.isfinite(g).all(), f"{what}: non-finite outputs"
    assert ok.all(), f"{what}: {np.count_nonzero(~ok)} outputs off (max {d.max()} bf16 ulp)"


CASES = [
    # (batch, q_heads, kv_heads, max_seq, lens)
    (4, 8, 8, 1024, [1024, 1, 0, 600]),            # rep 1, a single key, an empty sequence
    (3, 16, 8, 2048, [129, 128, 127]),             # rep 2, around one tile
    (2, 64, 8, 4096, [4096, 257]),                 # rep 8
    (2, 4, 1, 512, [5, 130]),                      # 3 tiles in all: fewer tiles than CTAs
    (2, 8, 2, 300, [300, 77]),                     # rep 4 (Mistral), max_seq not a tile multiple
    (200, 32, 8, 256, [int(x) for x in np.random.default_rng(7).integers(0, 257, 200)]),  # many short
    (2, 8, 2, 1024, None),                         # no lengths
]


@pytest.mark.parametrize("b,hq,hkv,m,lens", CASES)
def test_tc_decode_attention_matches_exact_and_split_kernel(cuda, orc, b, hq, hkv, m, lens):
    rng = np.random.default_rng(b * 7919 + m)
    d = 128
    q = orc.f32_to_bf16(rng.standard_normal((b, hq, d), dtype=F)).reshape(b, hq, d)
    kc = orc.f32_to_bf16(rng.standard_normal((b, hkv, m, d), dtype=F)).reshape(b, hkv, m, d)
    vc = orc.f32_to_bf16(rng.standard_normal((b, hkv, m, d), dtype=F)).reshape(b, hkv, m, d)
    lz = None if lens is None else np.array(lens, np.int32)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    exact, mag = _exact(bf16_to_f32(q), bf16_to_f32(kc), bf16_to_f32(vc), lz, scale)
    if lz is not None:  # NaN past every sequence's end: must never reach the output
        for bi, n in enumerate(lz):
            kc[bi, :, max(n, 0):] = 0x7FC0
            vc[bi, :, max(n, 0):] = 0x7FC0
    tc = _attend(q, kc, vc, lz, 0)
    _check(tc, exact, mag, "tcgen05 kernel")
    _check(_attend(q, kc, vc, lz, 1), exact, mag, "split-K kernel")
    if lz is not None:
        for bi, n in enumerate(lz):
            if n <= 0:
                assert np.all(bf16_to_f32(tc[bi]) == 0)


def test_tc_decode_attention_c3_shape(cuda, orc):
    """The benchmark's decode step: q [8, 32, 128], caches [8, 8, 32768, 128],
    the seed-2 lengths of C3; equal within the bar to the exact value, and the
    two kernels within 1 bf16 ulp of each other almost everywhere."""
    from oxide_b200.workloads import C3

    c = C3()
    _, lens, _ = c.inputs()
    rng = np.random.default_rng(3)
    b, hq, hkv, m, d = c.batch, c.heads, 8, c.keys, c.head_dim
    q = orc.f32_to_bf16(rng.standard_normal((b, hq, d), dtype=F)).reshape(b, hq, d)
    kc = orc.f32_to_bf16(rng.standard_normal((b, hkv, m, d), dtype=F)).reshape(b, hkv, m, d)
    vc = orc.f32_to_bf16(rng.standard_normal((b, hkv, m, d), dtype=F)).reshape(b, hkv, m, d)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    exact, mag = _exact(bf16_to_f32(q), bf16_to_f32(kc), bf16_to_f32(vc), lens, scale)
    tc = _attend(q, kc, vc, lens, 0)
    _check(tc, exact, mag, "tcgen05 kernel")
    split = _attend(q, kc, vc, lens, 1)
    assert np.mean(ulp_bf16(tc, split) <= 1) >= 0.999


def test_tc_wait_timeout_is_reported_and_the_context_survives(cuda, orc):
    """Failure detection without a fault: with the kernel's tile loads withheld
    (path 2) no copy ever completes, so every bounded wait runs out (two
    seconds); the launch ends by itself with NaN outputs and
    OXIDE_DEVICE_WAIT_TIMEOUT raised, and the next call on the same context
    computes the right values with no flag raised."""
    import ctypes as C
    import time

    from oxide_b200 import _lib

    flags = C.c_uint32(0)
    _lib.call("oxide_device_status", 1, C.byref(flags))  # start clear
    rng = np.random.default_rng(11)
    b, hq, hkv, m, d = 2, 8, 2, 1024, 128
    q = orc.f32_to_bf16(rng.standard_normal((b, hq, d), dtype=F)).reshape(b, hq, d)
    kc = orc.f32_to_bf16(rng.standard_normal((b, hkv, m, d), dtype=F)).reshape(b, hkv, m, d)
    vc = orc.f32_to_bf16(rng.standard_normal((b, hkv, m, d), dtype=F)).reshape(b, hkv, m, d)
    lz = np.array([1024, 77], np.int32)
    t0 = time.monotonic()
    bad = _attend(q, kc, vc, lz, 2)
    waited = time.monotonic() - t0
    _lib.call("oxide_device_status", 1, C.byref(flags))
    assert flags.value & _lib.DEVICE_WAIT_TIMEOUT, "the run-out wait was not reported"
    assert np.isnan(bf16_to_f32(bad)).all(), "an aborted launch must not leave values that look valid"
    assert 1.5 < waited < 60, f"the launch took {waited:.1f} s"
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    exact, mag = _exact(bf16_to_f32(q), bf16_to_f32(kc), bf16_to_f32(vc), lz, scale)
    _check(_attend(q, kc, vc, lz, 0), exact, mag, "the call after the timeout")
    _lib.call("oxide_device_status", 0, C.byref(flags))
    assert flags.value == 0
