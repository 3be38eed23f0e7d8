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


def assert_ulp(got: np.ndarray, ref: np.ndarray, max_ulp: int):
    d = ulp_bf16(got, ref) if got.dtype == np.uint16 else ulp_f32(got, ref)
    assert d.max(initial=0) <= max_ulp, f"max {d.max()} ulp (> {max_ulp}) at {np.argmax(d)}"
