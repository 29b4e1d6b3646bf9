"""The tensors QATFactory's exporters and QARL weight publisher write per quantized module,
produced on the sm_100a kernels.  File I/O (safetensors writers, GGUF containers, vLLM weight
loading) stays with the caller; these functions return exactly the on-wire tensors.

    nvfp4_export_fields   compressed-tensors ``nvfp4-pack-quantized`` fields of one linear
                          (qatfactory/quant/export/nvfp4_vllm.py:709-728)
    nvfp4_publish_pack    the packed fused-family weight NVFP4WeightPublisher.sync hands to
                          vLLM every optimizer step (qatfactory/rl/vllm_nvfp4_sync.py:325-333)
    mxfp4_export_fields   compressed-tensors MXFP4 fields (quant/export/mxfp4_vllm.py:251-260)
    q4k_save_blocks       the save-time Q4_K blocks (trainer/checkpoint.py:366-391 through the
                          format's pack hook), the bytes the GGUF splice writes unchanged
"""

from __future__ import annotations

import torch

from .formats import get_quant_format
from .formats.mxfp4 import dequantize_mxfp4, quantize_mxfp4
from .formats.nvfp4 import NVFP4_SCALE_DENOMINATOR, NVFP4QuantizationResult, dequantize_nvfp4, quantize_nvfp4

__all__ = ["nvfp4_export_fields", "nvfp4_publish_pack", "mxfp4_export_fields", "q4k_save_blocks"]


@torch.no_grad()
def nvfp4_export_fields(weight: torch.Tensor, tensor_amax: torch.Tensor, input_amax: torch.Tensor | None = None,
                        *, check: bool = True) -> dict[str, torch.Tensor]:
    """``weight_packed`` (uint8 [out, in/2]), ``weight_scale`` (float8_e4m3fn [out, in/16]),
    ``weight_global_scale`` (FP32 [1], the reciprocal of weight_scale_2) and, given the
    module's finalized input amax, ``input_global_scale`` (FP32 [1], the reciprocal of
    input_amax / 2688).  With ``check`` the packed tensors are dequantized and compared with the
    reconstruction bit for bit, raising like the exporter when they differ."""

    result = quantize_nvfp4(weight, tensor_amax=tensor_amax)
    if check:
        dequantized = dequantize_nvfp4(result.packed_weight, result.weight_scale, result.weight_scale_2)
        if not torch.equal(dequantized.to(result.reconstruction.dtype), result.reconstruction):
            raise ValueError("Packed NVFP4 dequantization is not bit-equal.")
    fields = {
        "weight_packed": result.packed_weight,
        "weight_scale": result.weight_scale,
        "weight_global_scale": result.weight_scale_2.reshape(1).float().reciprocal(),
    }
    if input_amax is not None:
        # a tensor divisor: the IEEE quotient on any device (a Python-scalar divisor becomes a
        # multiply by its reciprocal on CUDA), i.e. the value finalize_nvfp4_input_scales gives
        # on the CPU
        amax = input_amax.detach().to(torch.float32)
        input_scale = (amax / torch.tensor(NVFP4_SCALE_DENOMINATOR, dtype=torch.float32, device=amax.device)).reshape(())
        fields["input_global_scale"] = input_scale.reshape(1).reciprocal()
    return fields


@torch.no_grad()
def nvfp4_publish_pack(members: list[torch.Tensor], family_amax: torch.Tensor) -> NVFP4QuantizationResult:
    """A fused family's full weights concatenated along the output dimension and packed with
    the family's shared tensor amax, without a reconstruction."""

    weight = members[0] if len(members) == 1 else torch.cat(members, dim=0)
    return quantize_nvfp4(weight, tensor_amax=family_amax, compute_reconstruction=False)


@torch.no_grad()
def mxfp4_export_fields(weight: torch.Tensor, *, check: bool = True) -> dict[str, torch.Tensor]:
    """``weight_packed`` (uint8 [out, in/2]) and ``weight_scale`` (biased E8M0 uint8
    [out, in/32]), after the exporter's bit-equal dequantization check."""

    result = quantize_mxfp4(weight)
    if check:
        dequantized = dequantize_mxfp4(result.packed_weight, result.weight_scale)
        if not torch.equal(dequantized.to(result.reconstruction.dtype), result.reconstruction):
            raise ValueError("Packed MXFP4 dequantization is not bit-equal.")
    return {"weight_packed": result.packed_weight, "weight_scale": result.weight_scale}


@torch.no_grad()
def q4k_save_blocks(weight: torch.Tensor, module=None, quant_format: str = "q4_k") -> torch.Tensor:
    """ggml ``block_q4_K`` bytes [out, in/256 * 144] on the host, as the checkpoint's save-time
    pack stores them (the module's reorders and method apply when a module is given)."""

    fmt = get_quant_format(quant_format)
    return fmt.pack_weight(weight, module).detach().cpu().contiguous()
