"""Drop-in for the block-FP8 GEMM of tokenFactory's FP8 linear layers.

Qwen3_8FP8Linear._linear_op (qwen3_8/fp8_linear.py:181-201) sends every e4m3 projection to
``triton_block_fp8_linear`` (qwen3_8/fp8_triton.py:109-181) when ``can_use_triton_fp8_gemm``
allows it.  ``install()`` points both names, in ``qwen3_8.fp8_triton`` and in the
``qwen3_8.fp8_linear`` module that imported them, at ``ops.block_fp8_linear`` (same arguments,
same result: bit-exact activation quantization, the GEMM on the tcgen05 tensor cores) and a
predicate that accepts CUDA activations; ``uninstall()`` restores the reference's functions.
"""

import importlib
from typing import Dict, Tuple

import torch

from . import ops

_saved: Dict[Tuple[str, str], object] = {}


def can_use_block_fp8_gemm(x: torch.Tensor) -> bool:
    """The reference's can_use_triton_fp8_gemm (qwen3_8/fp8_triton.py:100-106) for this kernel:
    CUDA activations on a device with the 5th-generation tensor cores."""
    if not (x.is_cuda and hasattr(torch, "float8_e4m3fn")):
        return False
    return torch.cuda.get_device_capability(x.device) >= (10, 0)


def block_fp8_linear(x, weight, weight_scale_inv, bias, block_h: int = 128, block_w: int = 128):
    return ops.block_fp8_linear(x, weight, weight_scale_inv, bias, block_h, block_w)


_NAMES = {"triton_block_fp8_linear": block_fp8_linear,
          "can_use_triton_fp8_gemm": can_use_block_fp8_gemm}


def install(package: str = "qwen3_8") -> None:
    for mod_name in (f"{package}.fp8_triton", f"{package}.fp8_linear"):
        mod = importlib.import_module(mod_name)
        for name, fn in _NAMES.items():
            if hasattr(mod, name):
                _saved.setdefault((mod_name, name), getattr(mod, name))
                setattr(mod, name, fn)


def uninstall(package: str = "qwen3_8") -> None:
    for (mod_name, name), fn in list(_saved.items()):
        if mod_name.startswith(package + "."):
            setattr(importlib.import_module(mod_name), name, fn)
            del _saved[(mod_name, name)]
