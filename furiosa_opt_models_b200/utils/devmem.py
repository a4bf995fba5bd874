"""Views of engine device memory as torch tensors (tests and tools): a device address, a shape
and a dtype through the CUDA array interface, no copy."""

from __future__ import annotations

import torch

_TYPESTR = {torch.bfloat16: "<u2", torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4",
            torch.uint8: "|u1", torch.int64: "<i8"}


class _View:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def tensor(ptr: int, shape, dtype: torch.dtype, device: int | None = None) -> torch.Tensor:
    t = torch.as_tensor(_View(ptr, shape, _TYPESTR[dtype]), device="cuda" if device is None else f"cuda:{device}")
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def weights(model) -> dict:
    """Every weight of a loaded decoder, as torch views of its device memory: BF16 tensors, or
    ``QuantizedWeight`` views (codes and scales) for quantized projections."""
    from furiosa_opt_models_b200.ops.kernels import QuantizedWeight

    out = {}
    dev = model.device.ordinal
    for name in model.weight_names():
        q = model.quantized_weight(name)
        if q is None:
            ptr, shape = model.weight(name)
            out[name] = tensor(ptr, shape, torch.bfloat16, dev)
            continue
        rows, cols = q["shape"]
        fmt = q["format"]
        padded = None
        if fmt == "fp8_block":
            codes = tensor(q["codes"], (rows, cols), torch.uint8, dev)
            padded = tensor(q["scales"], ((rows + 127) // 128, cols // 128, 4), torch.float32, dev)
            scales = padded[..., 0]
        elif fmt == "fp8_rows":
            codes = tensor(q["codes"], (rows, cols), torch.uint8, dev)
            scales = tensor(q["scales"], (rows,), torch.float32, dev)
        elif fmt == "nvfp4":
            codes = tensor(q["codes"], (rows, cols // 2), torch.uint8, dev)
            scales = tensor(q["scales"], (rows, cols // 16), torch.uint8, dev)
        else:
            codes = tensor(q["codes"], (rows, cols // 2), torch.uint8, dev)
            scales = tensor(q["scales"], ((rows + 127) // 128, cols // 64, 512), torch.uint8, dev)
        out[name] = QuantizedWeight(fmt, codes, scales, rows, cols, q["tensor_scale"], q["input_scale"],
                                    gemm_scales=padded if fmt == "fp8_block" else None)
    return out
