"""MXFP4 fake quantization on B200: the ``qatfactory.quant`` MXFP4 API over libqatf.so.

E2M1 values in blocks of 32 along the input dimension with power-of-two E8M0 scales and
no tensor scale (reference qatfactory/quant/formats/mxfp4.py).  Weights use the EVEN rule
(amax threshold-rounded to a power of two, minus the E2M1 max exponent; values may clip
and then get zero gradient); activations use the CEIL rule (the smallest power of two
>= amax / 6, never clipping, all-true STE mask).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from ... import _native
from .lora import LoRAMixin, shared_base_teacher_enabled
from .nvfp4 import _MaskedStraightThrough, _pad2d, _round_up

MXFP4_BLOCK_SIZE = 32
MXFP4_MAX_VALUE = 6.0
E2M1_MAX_EXP = 2
E8M0_BIAS = 127
E8M0_MAX_EXP = 127
E8M0_MIN_EXP = -127


def dequantize_mxfp4(packed_weight: torch.Tensor, weight_scale: torch.Tensor) -> torch.Tensor:
    """Dequantize packed MXFP4 tensors to FP32 (mxfp4.py:101-116)."""

    if weight_scale.dtype != torch.uint8:
        raise ValueError(f"MXFP4 scales must be biased uint8 exponents, got {weight_scale.dtype}.")
    if packed_weight.ndim != 2 or packed_weight.dtype != torch.uint8:
        raise ValueError(f"Packed E2M1 weights must be 2D uint8, got {packed_weight.dtype} {tuple(packed_weight.shape)}.")
    if packed_weight.shape[-1] * 2 != weight_scale.shape[-1] * MXFP4_BLOCK_SIZE:
        raise ValueError(
            f"MXFP4 scale shape {tuple(weight_scale.shape)} is incompatible with "
            f"weight shape {tuple(packed_weight.shape)}."
        )
    return _native.mxfp4_dequant(packed_weight, weight_scale)


@dataclass(frozen=True)
class MXFP4QuantizationResult:
    packed_weight: torch.Tensor
    weight_scale: torch.Tensor
    reconstruction: torch.Tensor


@torch.no_grad()
def quantize_mxfp4(weight: torch.Tensor) -> MXFP4QuantizationResult:
    """Pack a 2D weight on the EVEN-rule MXFP4 lattice (mxfp4.py:126-151)."""

    if weight.ndim != 2:
        raise ValueError(f"MXFP4 packing expects a 2D weight, got shape {tuple(weight.shape)}.")
    if weight.shape[-1] % MXFP4_BLOCK_SIZE:
        raise ValueError(
            f"MXFP4 packing requires in_features divisible by {MXFP4_BLOCK_SIZE}, got {weight.shape[-1]}."
        )
    if weight.is_meta:
        raise ValueError("Cannot pack an MXFP4 lattice from a meta tensor.")
    packed, scales, recon = _native.mxfp4_pack(weight, recon=True)
    return MXFP4QuantizationResult(packed_weight=packed, weight_scale=scales, reconstruction=recon)


def fake_quantize_mxfp4(weight: torch.Tensor, block_size: int = MXFP4_BLOCK_SIZE) -> torch.Tensor:
    """EVEN-rule MXFP4 fake quant with the masked STE (mxfp4.py:177-202); the last
    dimension is zero-padded per block when not divisible by 32."""

    if block_size != MXFP4_BLOCK_SIZE:
        raise ValueError(f"MXFP4 requires block_size={MXFP4_BLOCK_SIZE}, got {block_size}.")
    if weight.ndim != 2:
        raise ValueError(f"MXFP4Linear expects a 2D weight, got shape {tuple(weight.shape)}.")
    if weight.is_meta:
        return weight
    grad = torch.is_grad_enabled() and weight.requires_grad  # else no STE mask and no autograd node
    with torch.no_grad():
        quantized, mask = _native.mxfp4_qdq_even(weight.detach(), want_mask=grad)
    return _MaskedStraightThrough.apply(weight, quantized, mask) if grad else quantized


def fake_quantize_mxfp4_activation(activation: torch.Tensor) -> torch.Tensor:
    """CEIL-rule MXFP4 activation fake quant; gradients pass unmasked (mxfp4.py:225-255)."""

    if activation.is_meta:
        return activation
    shape = activation.shape
    if shape[-1] % MXFP4_BLOCK_SIZE:
        raise ValueError(
            f"MXFP4 W4A4 requires in_features divisible by {MXFP4_BLOCK_SIZE}, got shape {tuple(shape)}."
        )
    with torch.no_grad():
        quantized = _native.mxfp4_qdq_ceil(activation.detach().reshape(-1, shape[-1])).reshape(shape)
    if not (torch.is_grad_enabled() and activation.requires_grad):
        return quantized
    return _MaskedStraightThrough.apply(activation, quantized, None)


class _MXFP4W4A4Linear(torch.autograd.Function):
    """``F.linear(fake_quantize_mxfp4_activation(x), fake_quantize_mxfp4(w))`` of the W4A4 MXFP4
    linear (mxfp4.py:285-290) on the tensor cores: one operand pass per input (codes, E8M0
    block-32 scales, dequantized copy, and for the weight the STE mask), a block-scaled MXFP4
    GEMM forward, and backward ``dX = dY @ W_q`` (the activation's straight-through gradient
    is unmasked, mxfp4.py:225-255) and ``dW = STE_w(dY^T @ X_q)`` as BF16 GEMMs.  Shapes off the
    GEMM tiles are zero-padded to them and sliced back, as for NVFP4: a zero block of 32 has zero
    codes under both rules, so the padding adds exact zeros and changes no kept value."""

    @staticmethod
    def forward(ctx, x2d, weight):
        rows, k = x2d.shape
        n = weight.shape[0]
        mp, kp, np_ = _round_up(rows, 128), _round_up(k, 256), _round_up(n, 256)
        xs = _pad2d(x2d.detach(), mp, kp)
        ws = _pad2d(weight.detach(), np_, kp)
        cx, sx, xq, _ = _native.mxfp4_operand(xs, _native.OPERAND_A, _native.MXFP4_CEIL, mask=False)
        cw, sw, wq, mw = _native.mxfp4_operand(ws, _native.OPERAND_B, _native.MXFP4_EVEN)
        y = _native.mxfp4_gemm(cx, sx, cw, sw)
        ctx.save_for_backward(xq, wq, mw)
        ctx.shape = (rows, k, n)
        return y if (mp, np_) == (rows, n) else y[:rows, :n].clone()

    @staticmethod
    def backward(ctx, grad_out):
        xq, wq, mw = ctx.saved_tensors
        rows, k, n = ctx.shape
        dy = _pad2d(grad_out.contiguous().to(torch.bfloat16), xq.shape[0], wq.shape[0])
        gx = gw = None
        if ctx.needs_input_grad[0]:
            gx = _native.bf16_gemm(dy, _native.K_MAJOR, wq, _native.MN_MAJOR)
            if gx.shape != (rows, k):
                gx = gx[:rows, :k]
        if ctx.needs_input_grad[1]:
            gw = _native.bf16_gemm(dy, _native.MN_MAJOR, xq, _native.MN_MAJOR, mw)
            if gw.shape != (n, k):
                gw = gw[:n, :k]
        return gx, gw


def mxfp4_w4a4_linear(input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """W4A4 MXFP4 linear: the tensor-core path for BF16 CUDA inputs with in features % 32 == 0
    (padded to the GEMM tiles where needed), otherwise fake-quantized operands through
    ``F.linear`` (the reference's own formulation)."""

    rows = input.numel() // input.shape[-1] if input.shape[-1] else 0
    if (input.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and input.is_cuda and rows > 0
            and weight.shape[0] > 0 and weight.shape[1] % MXFP4_BLOCK_SIZE == 0):
        y = _MXFP4W4A4Linear.apply(input.reshape(rows, input.shape[-1]), weight)
        y = y.reshape(*input.shape[:-1], weight.shape[0])
        return y if bias is None else y + bias
    return F.linear(fake_quantize_mxfp4_activation(input), fake_quantize_mxfp4(weight), bias)


class MXFP4Linear(LoRAMixin, nn.Linear):
    """Linear layer whose weight (and, for W4A4, input) is MXFP4 fake-quantized on every
    forward (mxfp4.py:258-290)."""

    @classmethod
    def from_linear(cls, module: nn.Linear) -> "MXFP4Linear":
        converted = cls(module.in_features, module.out_features, bias=module.bias is not None, device="meta")
        converted.weight = module.weight
        converted.bias = module.bias
        converted._quantize_activations = False
        return converted

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if shared_base_teacher_enabled():
            return F.linear(input, self.weight, self.bias)
        if self._quantize_activations:
            return mxfp4_w4a4_linear(input, self._effective_weight(), self.bias)
        return F.linear(input, fake_quantize_mxfp4(self._effective_weight()), self.bias)
