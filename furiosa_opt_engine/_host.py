"""Host-side conversions of the HostTensor constructors: nested Python numbers and DLPack
exports to (shape, dtype name, little-endian bytes)."""

from __future__ import annotations

import numpy as np

_NUMPY = {
    "bool": np.bool_, "uint8": np.uint8, "int8": np.int8, "int16": np.int16, "int32": np.int32,
    "int64": np.int64, "float16": np.float16, "float32": np.float32, "float64": np.float64,
}
_TORCH_NAMES = {
    "torch.bool": "bool", "torch.uint8": "uint8", "torch.int8": "int8", "torch.int16": "int16",
    "torch.int32": "int32", "torch.int64": "int64", "torch.float16": "float16",
    "torch.bfloat16": "bfloat16", "torch.float32": "float32", "torch.float64": "float64",
    "torch.float8_e4m3fn": "float8_e4m3fn", "torch.float8_e5m2": "float8_e5m2",
}


def _shape(values) -> list[int]:
    if isinstance(values, (list, tuple)):
        if not values:
            return [0]
        inner = [_shape(v) for v in values]
        if any(s != inner[0] for s in inner):
            raise ValueError("the nesting is ragged")
        return [len(values)] + inner[0]
    return []


def _flat(values, out: list) -> None:
    if isinstance(values, (list, tuple)):
        for v in values:
            _flat(v, out)
    else:
        out.append(values)


def from_values(values, dtype: str | None):
    """Nested lists or tuples of numbers as ``dtype``: int32 when every value is an integer and
    float32 otherwise, by default."""
    shape = _shape(values)
    flat: list = []
    _flat(values, flat)
    if dtype is None:
        dtype = "int32" if all(isinstance(v, (int, bool)) and not isinstance(v, float) for v in flat) else "float32"
    if dtype in ("float8_e4m3fn", "float8_e5m2"):
        raise ValueError(f"dtype {dtype} takes values through from_dlpack")
    if dtype == "bfloat16":
        arr = np.asarray(flat, dtype=np.float32).reshape(shape)
        bits = arr.view(np.uint32)
        rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
        return shape, dtype, rounded.tobytes()
    if dtype not in _NUMPY:
        raise ValueError(f"unknown dtype: {dtype}")
    np_dtype = _NUMPY[dtype]
    arr = np.asarray(flat, dtype=np.float64 if np.issubdtype(np_dtype, np.floating) else object)
    if np.issubdtype(np_dtype, np.integer):
        info = np.iinfo(np_dtype)
        for v in flat:
            if not isinstance(v, (int, bool)) or not (info.min <= int(v) <= info.max):
                raise ValueError(f"a value does not fit {dtype}")
        arr = np.asarray([int(v) for v in flat], dtype=np_dtype)
    else:
        arr = arr.astype(np_dtype)
    return shape, dtype, arr.reshape(shape).tobytes()


def from_dlpack(value):
    """Any host tensor exporting DLPack (NumPy, PyTorch): shape, dtype name and bytes in logical
    order."""
    import torch

    try:
        t = torch.from_dlpack(value)
    except Exception as e:  # noqa: BLE001
        raise ValueError(f"the tensor does not export DLPack: {e}") from None
    if t.device.type != "cpu":
        raise ValueError("the tensor is not on the host")
    name = _TORCH_NAMES.get(str(t.dtype))
    if name is None:
        raise ValueError(f"unsupported dtype {t.dtype}")
    t = t.contiguous()
    raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
    return list(t.shape), name, raw
