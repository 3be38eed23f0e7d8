"""safetensors loading with the element decode on the GPU (the reference's
SafetensorsLoader, src/loading/safetensors.rs).

The file layout is parsed on the host (an 8-byte little-endian header length,
a JSON header of {name: {dtype, shape, data_offsets}}, then the data); the data
section goes to the device in one copy and every tensor is decoded there by
oxide_decode_weights_* into an f32 tensor (the reference's result dtype) or,
on request, bf16.  BF16 sources are decoded as bf16 -- the reference runs them
through the f16 conversion, which this loader does not reproduce.  Error
messages are the reference's (convert_dtype :31-45, load_tensor_from_view
:48-82, tensor_to_bytes :114-133).
"""
from __future__ import annotations

import json
import math
import struct
from typing import Optional

import torch

from . import _lib
from ._lib import OxideError, call

# safetensors dtype names the reference maps (convert_dtype) and the ones it decodes
_KNOWN = {"F32", "F16", "BF16", "I64", "U8", "U32", "F64", "F8_E4M3"}
_DECODE = {"F32": (_lib.WDT_F32, 4), "F16": (_lib.WDT_F16, 2), "BF16": (_lib.WDT_BF16, 2)}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def load_from_bytes(data, device="cuda", dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    """SafetensorsLoader::load_from_bytes: name -> device tensor (f32 by default)."""
    if dtype not in (torch.float32, torch.bfloat16):
        raise OxideError(_lib.ERR_UNSUPPORTED, "load_from_bytes", f"result dtype {dtype} is not float32/bfloat16")
    mv = memoryview(data).cast("B")
    if len(mv) < 8:
        raise OxideError(_lib.ERR_INVALID_ARG, "load_from_bytes", "HeaderTooSmall")
    hlen = struct.unpack("<Q", mv[:8])[0]
    if 8 + hlen > len(mv):
        raise OxideError(_lib.ERR_INVALID_ARG, "load_from_bytes", "InvalidHeaderLength")
    header = json.loads(bytes(mv[8:8 + hlen]).decode("utf-8"))
    body = mv[8 + hlen:]
    entries = []
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _KNOWN:
            raise OxideError(_lib.ERR_UNSUPPORTED, "load_from_bytes", f"Unsupported dtype in safetensors: {dt}")
        if dt not in _DECODE:
            raise OxideError(_lib.ERR_INVALID_ARG, "load_from_bytes", f"Dtype {dt} not yet implemented for loading")
        code, es = _DECODE[dt]
        start, end = info["data_offsets"]
        shape = [int(v) for v in info["shape"]]
        count = math.prod(shape)
        if end - start != count * es or end > len(body) or start > end:
            raise OxideError(_lib.ERR_INVALID_ARG, "load_from_bytes", f"TensorInvalidInfo: {name}")
        entries.append((name, code, start, count, shape))
    dev = torch.device(device)
    raw = torch.empty(len(body), dtype=torch.uint8, device=dev)
    if len(body):
        host = torch.frombuffer(bytearray(body), dtype=torch.uint8).pin_memory()
        raw.copy_(host, non_blocking=True)
    sfx = "f32" if dtype == torch.float32 else "bf16"
    out = {}
    for name, code, start, count, shape in entries:
        t = torch.empty(shape, dtype=dtype, device=dev)
        call(f"oxide_decode_weights_{sfx}", raw.data_ptr() + start if count else None, count, code,
             t.data_ptr() if count else None, _stream())
        out[name] = t
    torch.cuda.current_stream().synchronize()  # raw is released on return
    return out


def load_from_file(path: str, device="cuda", dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    """SafetensorsLoader::load_from_file / load_safetensors."""
    with open(path, "rb") as f:
        return load_from_bytes(f.read(), device, dtype)


load_safetensors = load_from_file


def save_to_bytes(tensors: dict[str, torch.Tensor], metadata: Optional[dict] = None) -> bytes:
    """SafetensorsLoader::save_to_file's serialisation: f32 tensors only, as in
    the reference (tensor_to_bytes)."""
    header, chunks, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name]
        if t.dtype != torch.float32:
            name_dt = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float64: "F64"}.get(t.dtype, str(t.dtype))
            raise OxideError(_lib.ERR_UNSUPPORTED, "save_to_file", f"Save not implemented for dtype {name_dt}")
        b = t.detach().to("cpu").contiguous().numpy().astype("<f4").tobytes()
        header[name] = {"dtype": "F32", "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        chunks.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)  # the format pads the header to 8 bytes
    return struct.pack("<Q", len(hb)) + hb + b"".join(chunks)


def save_to_file(tensors: dict[str, torch.Tensor], path: str) -> None:
    with open(path, "wb") as f:
        f.write(save_to_bytes(tensors))
