"""The native quantiser plug-in the reference already looks for.

quantization/w8a8_triton_kernels.py:10-15 does ``import w8a8_cuda_quant`` and,
when ``is_available()`` is true, routes ``quantize_activation[_out]`` through
this module's four functions (:342-372) instead of its Triton kernels.  Make
this module importable under that name (``sys.modules['w8a8_cuda_quant'] =
baidu_cti_grab_b200.w8a8_cuda_quant`` before importing the reference, or put a
one-line ``from baidu_cti_grab_b200.w8a8_cuda_quant import *`` module named
w8a8_cuda_quant.py on sys.path) and the reference's W8A8 activation
quantisation runs on the sm_100a kernels with no edit to the reference.
"""

from __future__ import annotations

import torch

from . import _lib, device_ops


def is_available() -> bool:
    if not _lib.is_available():
        return False
    return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10


def load_error_message():
    return _lib.load_error_message()


def static_quantize_activation_out(x_2d: torch.Tensor, scale: torch.Tensor, xq: torch.Tensor) -> torch.Tensor:
    return device_ops.quant_static_out(x_2d.contiguous(), scale, xq)


def static_quantize_activation(x_2d: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    xq = torch.empty_like(x_2d, dtype=torch.int8)
    return static_quantize_activation_out(x_2d, scale, xq)


def dynamic_per_token_quantize_activation_out(x_2d: torch.Tensor, xq: torch.Tensor, scale: torch.Tensor):
    return device_ops.quant_dynamic_per_token_out(x_2d, xq, scale)


def dynamic_per_token_quantize_activation(x_2d: torch.Tensor):
    xq = torch.empty_like(x_2d, dtype=torch.int8)
    scale = torch.empty((x_2d.shape[0],), device=x_2d.device, dtype=torch.float32)
    return dynamic_per_token_quantize_activation_out(x_2d, xq, scale)
