"""Kernel callables with the native engine's injection signatures.

`h3b_int8_kernel` is an `Int8Kernel` and `h3b_w4a8_kernel` a `W4A8Kernel`
(model/quantization.py:19-37); pass them where the engine passes
comfy_kitchen_int8_kernel / comfy_kitchen_w4a8_kernel (quantization.py:40-95,
assembly.py:259-333) and ConvRotInt8Linear / ConvRotW4A8Linear run on B200.
"""

from __future__ import annotations

import torch

from . import ops


def h3b_int8_kernel(value: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None,
                    convrot_group_size: int) -> torch.Tensor:
    return ops.int8_linear(value, qweight, scale, bias, value.dtype, convrot=bool(convrot_group_size),
                           convrot_groupsize=convrot_group_size or 256)


def h3b_w4a8_kernel(value: torch.Tensor, qdata: torch.Tensor, s_rel: torch.Tensor, s_channel: torch.Tensor,
                    codebook: torch.Tensor | None, correction: torch.Tensor | None, bias: torch.Tensor | None,
                    group_size: int, convrot_group_size: int, output_dtype: torch.dtype) -> torch.Tensor:
    return ops.w4a8_int8_linear(value, qdata, s_rel, s_channel, codebook=codebook, correction=correction, bias=bias,
                                group_size=group_size, convrot_groupsize=convrot_group_size,
                                out_dtype=output_dtype)
