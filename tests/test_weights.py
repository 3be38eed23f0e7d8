"""Weight decoding (src/loading/safetensors.rs:48-82): the oracle's element
decode pinned against numpy and hand-derived values, the GPU decode bit-exact
against the oracle over every 16-bit pattern, and the safetensors loader
(layout, errors, round trip).  BF16 is decoded as bf16; the reference's
decode of BF16 bytes through the f16 conversion is shown to differ."""
import json
import struct

import numpy as np
import pytest

from _util import to_np

ALL16 = np.arange(65536, dtype=np.uint32).astype(np.uint16)


def _assert_bf16_equal(got, ref):
    """bf16 bits equal; a NaN is any NaN (the bf16 form stores the canonical NaN)."""
    gn = (got & 0x7FFF) > 0x7F80
    rn = (ref & 0x7FFF) > 0x7F80
    assert np.array_equal(gn, rn), "NaN positions differ"
    assert np.array_equal(got[~gn], ref[~rn])


def _blob(entries, pad=True):
    """A safetensors byte string from [(name, dtype, shape, raw bytes)]."""
    header, body = {}, b""
    for name, dt, shape, raw in entries:
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [len(body), len(body) + len(raw)]}
        body += raw
    hb = json.dumps(header).encode()
    if pad:
        hb += b" " * (-len(hb) % 8)
    return struct.pack("<Q", len(hb)) + hb + body


def test_oracle_f16_decode_matches_numpy_and_quiets_nans(orc):
    got = orc.decode_weights(ALL16.view(np.uint8), orc.WDT_F16)
    ref = ALL16.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    gb = got[nan].view(np.uint32)
    assert np.all(np.isnan(got[nan])) and np.all(gb & 0x00400000)  # quiet bit set
    assert np.array_equal((gb >> 13) & 0x1FF, ALL16[nan].astype(np.uint32) & 0x1FF)  # payload kept
    assert np.array_equal(gb >> 31, ALL16[nan].astype(np.uint32) >> 15)  # sign kept


def test_oracle_bf16_decode_is_the_high_half_and_differs_from_the_reference_bug(orc):
    got = orc.decode_weights(ALL16.view(np.uint8), orc.WDT_BF16)
    assert np.array_equal(got.view(np.uint32), ALL16.astype(np.uint32) << 16)
    b = np.array([0x3F80, 0x4049, 0xC2F7], np.uint16)  # 1.0, 3.140625, -123.5 in bf16
    assert list(orc.decode_weights(b.view(np.uint8), orc.WDT_BF16)) == [1.0, 3.140625, -123.5]
    # what the reference computes for these bytes: the f16 conversion
    bug = [orc.lib().orc_decode_f16_bits_f32(int(h)) for h in b]
    assert bug[1] != 3.140625 and abs(bug[0] - 1.875) < 1e-7


def test_oracle_f32_copy_and_bf16_rounding(orc):
    x = np.array([1.0, -2.5, np.inf, 1e-40, 3.4e38, 1.00390625], np.float32)
    assert np.array_equal(orc.decode_weights(x.view(np.uint8), orc.WDT_F32).view(np.uint32), x.view(np.uint32))
    got = orc.decode_weights(x.view(np.uint8), orc.WDT_F32, out_bf16=True)
    assert list(got) == [orc.f32_to_bf16(np.array([v], np.float32))[0] for v in x]


def test_loader_errors_follow_the_reference():
    from oxide_b200 import loading
    from oxide_b200._lib import OxideError

    with pytest.raises(OxideError, match="Dtype I64 not yet implemented for loading"):
        loading.load_from_bytes(_blob([("a", "I64", [2], b"\0" * 16)]))
    with pytest.raises(OxideError, match="Unsupported dtype in safetensors: BOOL"):
        loading.load_from_bytes(_blob([("a", "BOOL", [2], b"\0" * 2)]))
    with pytest.raises(OxideError, match="TensorInvalidInfo"):
        loading.load_from_bytes(_blob([("a", "F32", [3], b"\0" * 8)]))


def test_save_layout_matches_the_format():
    import torch

    from oxide_b200 import loading
    from oxide_b200._lib import OxideError

    t = {"w": torch.arange(6, dtype=torch.float32).reshape(2, 3), "b": torch.tensor([0.5])}
    blob = loading.save_to_bytes(t)
    n = struct.unpack("<Q", blob[:8])[0]
    assert n % 8 == 0
    h = json.loads(blob[8:8 + n])
    assert h["w"] == {"dtype": "F32", "shape": [2, 3], "data_offsets": [4, 28]}
    assert np.array_equal(np.frombuffer(blob[8 + n + 4:8 + n + 28], "<f4"), np.arange(6, dtype=np.float32))
    with pytest.raises(OxideError, match="Save not implemented for dtype BF16"):
        loading.save_to_bytes({"x": torch.zeros(2, dtype=torch.bfloat16)})


@pytest.mark.gpu
@pytest.mark.parametrize("code", [1, 2])  # F16, BF16
def test_decode_every_16bit_pattern_matches_oracle(cuda, orc, code):
    import torch

    from oxide_b200 import _lib

    raw = torch.from_numpy(ALL16.view(np.uint8).copy()).to(cuda)
    # aligned vector paths; 8-byte source alignment (the f32 output's 8-byte
    # loads, the bf16 output's element path); then the element path
    for misalign, short in ((0, 0), (8, 4), (2, 3)):
        src = torch.empty(raw.numel() + 16, dtype=torch.uint8, device=cuda)
        src[misalign:misalign + raw.numel()] = raw
        ptr = src.data_ptr() + misalign
        n = 65536 - short
        out = torch.empty(n, dtype=torch.float32, device=cuda)
        _lib.call("oxide_decode_weights_f32", ptr, n, code, out.data_ptr(), 0)
        ref = orc.decode_weights(ALL16[:n].view(np.uint8), code)
        assert np.array_equal(to_np(out).view(np.uint32), ref.view(np.uint32))
        ob = torch.empty(n, dtype=torch.bfloat16, device=cuda)
        _lib.call("oxide_decode_weights_bf16", ptr, n, code, ob.data_ptr(), 0)
        refb = orc.decode_weights(ALL16[:n].view(np.uint8), code, out_bf16=True)
        _assert_bf16_equal(to_np(ob), refb)


@pytest.mark.gpu
def test_decode_f32_copy_and_bf16_rounding(cuda, orc):
    import torch

    from oxide_b200 import _lib

    rng = np.random.default_rng(0)
    x = rng.integers(0, 2**32, size=100003, dtype=np.uint64).astype(np.uint32).view(np.float32)
    raw = torch.from_numpy(x.view(np.uint8).copy()).to(cuda)
    out = torch.empty(x.size, dtype=torch.float32, device=cuda)
    _lib.call("oxide_decode_weights_f32", raw.data_ptr(), x.size, 0, out.data_ptr(), 0)
    assert np.array_equal(to_np(out).view(np.uint32), x.view(np.uint32))
    ob = torch.empty(x.size, dtype=torch.bfloat16, device=cuda)
    _lib.call("oxide_decode_weights_bf16", raw.data_ptr(), x.size, 0, ob.data_ptr(), 0)
    _assert_bf16_equal(to_np(ob), orc.decode_weights(x.view(np.uint8), 0, out_bf16=True))
    with pytest.raises(_lib.OxideError, match="src_dtype"):
        _lib.call("oxide_decode_weights_f32", raw.data_ptr(), 4, 7, out.data_ptr(), 0)
    with pytest.raises(_lib.OxideError, match="aligned"):
        _lib.call("oxide_decode_weights_f32", raw.data_ptr() + 2, 4, 0, out.data_ptr(), 0)


@pytest.mark.gpu
def test_loader_round_trip_and_mixed_dtypes(cuda, orc, tmp_path):
    import torch

    from oxide_b200 import loading

    rng = np.random.default_rng(1)
    w = rng.standard_normal((64, 33)).astype(np.float32)
    h = rng.standard_normal(1001).astype(np.float16)
    b = orc.f32_to_bf16(rng.standard_normal((7, 5)).astype(np.float32))
    blob = _blob([("w", "F32", w.shape, w.tobytes()), ("h", "F16", h.shape, h.tobytes()),
                  ("b", "BF16", b.shape, b.tobytes()), ("e", "F32", [0], b"")])
    got = loading.load_from_bytes(blob, cuda)
    assert np.array_equal(to_np(got["w"]), w)
    assert np.array_equal(to_np(got["h"]).view(np.uint32),
                          orc.decode_weights(h.view(np.uint8), orc.WDT_F16).view(np.uint32))
    assert np.array_equal(to_np(got["b"]).view(np.uint32), (b.astype(np.uint32) << 16).reshape(7, 5))
    assert got["e"].numel() == 0 and got["w"].shape == (64, 33)
    gb = loading.load_from_bytes(blob, cuda, dtype=torch.bfloat16)
    assert np.array_equal(to_np(gb["b"]), b)
    path = tmp_path / "m.safetensors"
    loading.save_to_file({"w": torch.from_numpy(w)}, str(path))
    assert np.array_equal(to_np(loading.load_safetensors(str(path), cuda)["w"]), w)
