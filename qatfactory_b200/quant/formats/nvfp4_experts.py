"""NVFP4 fake quantization of fused routed-expert weights ``[experts, rows, in_features]``.

Recent MoE backbones keep every routed expert in fused 3-D parameters (``gate_up_proj``
``[E, 2*intermediate, hidden]``, ``down_proj`` ``[E, hidden, intermediate]``).  Each expert
slice is quantized with exactly the 2-D NVFP4 math and its own tensor amax, so one batched
kernel launch (``qatf_nvfp4_qdq_experts``) replaces the reference's slab-by-slab torch
computation (``qatfactory/quant/formats/nvfp4_experts.py:386-462``) bit for bit.

Provided here: ``fake_quantize_nvfp4_experts``, the per-expert ``_ExpertFakeQuantLinear`` and
``is_fused_experts``.  The routing modules built on them (``NVFP4Experts``,
``NVFP4ExpertLoRA``) are not part of this package.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ... import _native
from .nvfp4 import NVFP4_BLOCK_SIZE, _MaskedStraightThrough

__all__ = ["fake_quantize_nvfp4_experts", "is_fused_experts", "fused_experts_shapes"]


def fused_experts_shapes(module: nn.Module) -> tuple[int, int, int] | None:
    """``(num_experts, hidden, intermediate)`` of a fused-3D experts module, else None
    (nvfp4_experts.py:47-62)."""

    gate_up = getattr(module, "gate_up_proj", None)
    down = getattr(module, "down_proj", None)
    if not isinstance(gate_up, nn.Parameter) or not isinstance(down, nn.Parameter):
        return None
    if gate_up.ndim != 3 or down.ndim != 3 or gate_up.shape[0] != down.shape[0]:
        return None
    num_experts, gate_up_rows, hidden = gate_up.shape
    if gate_up_rows % 2:
        return None
    intermediate = gate_up_rows // 2
    if tuple(down.shape[1:]) != (hidden, intermediate):
        return None
    return num_experts, hidden, intermediate


def is_fused_experts(module: nn.Module) -> bool:
    return fused_experts_shapes(module) is not None


def _check_expert_amax(tensor_amax: torch.Tensor) -> None:
    # a host synchronisation, as in the reference (nvfp4_experts.py:433-435)
    if not bool(torch.isfinite(tensor_amax).all()) or bool((tensor_amax < 0).any()):
        raise ValueError("Expert tensor_amax values must be finite and non-negative.")


def fake_quantize_nvfp4_experts(weight: torch.Tensor, tensor_amax: torch.Tensor) -> torch.Tensor:
    """Fake-quantize a packed 3-D expert weight ``[E, rows, in_features]`` per expert with
    ``tensor_amax`` ``[E]`` (nvfp4_experts.py:386-420).  Bit-identical to quantizing the experts
    one by one with ``fake_quantize_nvfp4``; a zero-amax expert quantizes to zero with a
    pass-through gradient."""

    if weight.ndim != 3:
        raise ValueError(f"Expert fake quantization expects a 3D weight, got shape {tuple(weight.shape)}.")
    if weight.shape[-1] % NVFP4_BLOCK_SIZE:
        raise ValueError(
            f"NVFP4 expert weights require in_features divisible by {NVFP4_BLOCK_SIZE}, "
            f"got shape {tuple(weight.shape)}."
        )
    if tensor_amax.shape != (weight.shape[0],):
        raise ValueError(f"Expert tensor_amax must have shape ({weight.shape[0]},), got {tuple(tensor_amax.shape)}.")
    if weight.is_meta:
        return weight
    amax = tensor_amax.detach().to(device=weight.device, dtype=torch.float32)
    _check_expert_amax(amax)
    with torch.no_grad():
        quantized, mask = _native.nvfp4_qdq_experts(weight.detach(), amax)
    return _MaskedStraightThrough.apply(weight, quantized, mask)


class _ExpertFakeQuantLinear(torch.autograd.Function):
    """``F.linear(x, fake_quant(w))`` for one expert, with the masked straight-through gradient
    to ``w`` (nvfp4_experts.py:465-493).  As in the reference, the quantized weight and its mask
    are recomputed in backward from the latent slice instead of being kept from the forward."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, amax: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            quantized, _ = _native.nvfp4_qdq_experts(w.detach().unsqueeze(0), amax.reshape(1), want_mask=False)
        ctx.save_for_backward(x, w, amax)
        return F.linear(x, quantized[0])

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, w, amax = ctx.saved_tensors
        with torch.no_grad():
            quantized, mask = _native.nvfp4_qdq_experts(w.detach().unsqueeze(0), amax.reshape(1))
        grad_x = grad_output.matmul(quantized[0]) if ctx.needs_input_grad[0] else None
        grad_w = None
        if ctx.needs_input_grad[1]:
            grad_w = grad_output.reshape(-1, grad_output.shape[-1]).t().mm(x.reshape(-1, x.shape[-1]))
            grad_w = _native.ste_backward(grad_w.contiguous(), mask)
        return grad_x, grad_w, None
