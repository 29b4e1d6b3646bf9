"""Frozen block-scaled FP8 bases for LoRA-QAD (qatfactory/quant/formats/fp8_base.py).

A pre-quantized checkpoint may ship its linears and fused experts as ``float8`` codes plus a
per-block ``scale_inv`` grid.  LoRA-QAD only reads that base, so the codes stay the frozen
parameter and one weight (or one fused expert tensor) is dequantized at a time, here by one
kernel (``qatf_fp8_block_dequant``) whose output equals the reference's torch expression
``(codes.float() * scale_inv[block]).to(dtype)`` bit for bit.  The scale grids are kept as
non-persistent buffers, as in the reference, so they neither appear in ``state_dict()`` nor
go through an FSDP2 mixed-precision cast.
"""

from __future__ import annotations

import torch
from torch import nn

from ... import _native

FP8_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2)


def is_fp8_tensor(tensor: torch.Tensor | None) -> bool:
    return tensor is not None and tensor.dtype in FP8_DTYPES


def dequantize_fp8_blocks(weight: torch.Tensor, scale_inv: torch.Tensor,
                          dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``weight`` ``[..., rows, cols]`` of FP8 codes times its ``scale_inv`` grid
    ``[..., scale_rows, scale_cols]`` (each scale covers a ``rows / scale_rows`` by
    ``cols / scale_cols`` block; leading dimensions broadcast), as ``dtype``."""

    rows, cols = weight.shape[-2:]
    scale_rows, scale_cols = scale_inv.shape[-2:]
    if rows % scale_rows or cols % scale_cols:
        raise ValueError(
            f"FP8 weight shape ({rows}, {cols}) is not divisible by its scale grid ({scale_rows}, {scale_cols})."
        )
    if weight.is_meta:
        return torch.empty(weight.shape, dtype=dtype, device="meta")
    return _native.fp8_block_dequant(weight, scale_inv, dtype)


def fp8_linear_state(module: nn.Module) -> tuple[torch.Tensor, torch.Tensor] | None:
    """``(weight, weight_scale_inv)`` of a block-FP8 linear, else None."""

    weight = getattr(module, "weight", None)
    scale_inv = getattr(module, "weight_scale_inv", None)
    if not is_fp8_tensor(weight) or scale_inv is None:
        return None
    return weight, scale_inv


def fp8_experts_state(module: nn.Module) -> dict[str, torch.Tensor] | None:
    """The FP8 codes and scale grids of a fused-experts module whose weights are FP8, else None."""

    gate_up = getattr(module, "gate_up_proj", None)
    down = getattr(module, "down_proj", None)
    if not (is_fp8_tensor(gate_up) and is_fp8_tensor(down)):
        return None
    scales = {name: getattr(module, f"{name}_scale_inv", None) for name in ("gate_up_proj", "down_proj")}
    if any(s is None for s in scales.values()):
        raise ValueError(
            "FP8 fused experts are missing their per-block scales (gate_up_proj_scale_inv / down_proj_scale_inv)."
        )
    return {"gate_up_proj": gate_up, "down_proj": down, "gate_up_proj_scale_inv": scales["gate_up_proj"],
            "down_proj_scale_inv": scales["down_proj"]}
