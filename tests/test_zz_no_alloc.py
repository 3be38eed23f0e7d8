"""oxide_reduce_static_*: the whole-tensor reduction whose scratch is a fixed
array inside the library instead of a caller workspace.

Called through the C ABI and compared with oxide_reduce_* (caller workspace)
on the same input: both run the same two kernels over the same partition, so
the f64 results must agree bit for bit.  Calls come in pairs, a large input
(every scratch slot written) followed by a smaller one (fewer slots), so a
call that read a slot left over from the previous call would show up.
"""
import numpy as np
import pytest

from oxide_b200 import _lib

MAX_N = 1024 << 24  # OXIDE_REDUCE_STATIC_MAX_N


def _reduce_pair(x, op, ws, out_ws, out_static, stream):
    name = "bf16" if x.dtype.itemsize == 2 else "f32"
    n = x.numel()
    _lib.call(f"oxide_reduce_{name}", op, x.data_ptr(), n, out_ws.data_ptr(), ws.data_ptr(),
              ws.numel(), stream)
    _lib.call(f"oxide_reduce_static_{name}", op, x.data_ptr(), n, out_static.data_ptr(), stream)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("op", [_lib.RED_SUM, _lib.RED_MAX, _lib.RED_SUMSQ])
def test_static_scratch_matches_workspace_form(cuda, dtype, op):
    import torch

    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    g = torch.Generator(device=cuda).manual_seed(7 + op)
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(_lib.lib().oxide_reduce_workspace_bytes(0), dtype=torch.uint8, device=cuda)
    sizes = [(1 << 26) + 5, 12345, (1 << 20) + 3, 1, 0]  # big, then smaller: pairs in a row
    xs = [torch.randn(n, generator=g, device=cuda).to(tdt) for n in sizes]
    xs.append(xs[0][1:])  # unaligned base: the scalar stage-1 kernel
    for x in xs:
        out_ws = torch.full((1,), float("nan"), dtype=torch.float64, device=cuda)
        out_st = torch.full((1,), float("nan"), dtype=torch.float64, device=cuda)
        _reduce_pair(x, op, ws, out_ws, out_st, stream)
        torch.cuda.synchronize()
        a, b = out_ws.item(), out_st.item()
        assert a == b or (np.isnan(a) and np.isnan(b)), (x.numel(), a, b)
        # and both are the reduction (f64 of the same elements)
        ref = x.double()
        want = {0: ref.sum(), 1: ref.max() if x.numel() else torch.tensor(-np.inf),
                2: (ref * ref).sum()}[op].item()
        if op == _lib.RED_MAX:
            assert b == want, (x.numel(), b, want)  # -inf for the empty input
        else:
            scale = max(1.0, float(ref.abs().sum()) if op == 0 else float((ref * ref).sum()))
            assert abs(b - want) <= 1e-5 * scale, (x.numel(), b, want)


@pytest.mark.gpu
def test_static_scratch_two_calls_in_a_row(cuda):
    """The second of two back-to-back calls on one stream sees none of the
    first call's partials: a 2^26-element sum, then a 3-element sum."""
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    big = torch.full((1 << 26,), 1.0, dtype=torch.float32, device=cuda)
    small = torch.tensor([1.0, 2.0, 4.0], dtype=torch.float32, device=cuda)
    out = torch.zeros(2, dtype=torch.float64, device=cuda)
    _lib.call("oxide_reduce_static_f32", _lib.RED_SUM, big.data_ptr(), big.numel(),
              out.data_ptr(), stream)
    _lib.call("oxide_reduce_static_f32", _lib.RED_SUM, small.data_ptr(), small.numel(),
              out.data_ptr() + 8, stream)
    torch.cuda.synchronize()
    assert out.tolist() == [float(1 << 26), 7.0]


def test_static_scratch_rejects_oversize_n_before_any_device_work():
    """n beyond the fixed scratch's reach is an argument error, returned before
    any CUDA call.  Run only where no device is visible, so that not even a
    broken check could reach a kernel with the oversize n."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("runs without a device only")
    host = np.zeros(16, np.float32)
    out = np.zeros(1, np.float64)
    for name in ("oxide_reduce_static_f32", "oxide_reduce_static_bf16"):
        rc = _lib.raw(name, _lib.RED_SUM, host.ctypes.data, MAX_N + 1, out.ctypes.data, None)
        assert rc == _lib.ERR_INVALID_ARG
        assert "exceeds" in _lib.last_error()
        # a size within the limit gets as far as the device lookup and fails there
        rc = _lib.raw(name, _lib.RED_SUM, host.ctypes.data, 16, out.ctypes.data, None)
        assert rc == _lib.ERR_CUDA, _lib.status_name(rc)
    assert _lib.raw("oxide_reduce_static_f32", 9, host.ctypes.data, 16, out.ctypes.data,
                    None) == _lib.ERR_INVALID_ARG
