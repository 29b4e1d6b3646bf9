"""Drop-in replacement for ``qatfactory.quant`` (fake-quantization path) on B200.

Same public names as the reference package (qatfactory/quant/__init__.py:1-88) for the
NVFP4, MXFP4 and Q4_K formats, the format registry and the module swap; every tensor
computation runs in libqatf.so (sm_100a).  Fused routed experts train as ``NVFP4Experts``
(full-parameter) or ``NVFP4ExpertLoRA`` (LoRA, over a BF16 or block-FP8 frozen base); the
checkpoint exporters' file I/O is not part of this package.  ``NVFP4QuantizedGather`` (no
counterpart in the reference) switches FSDP2 training to gathering weights that each rank
quantized on its own shard.
"""

from .fake_quant import ConvertedModules, apply_fake_quant, is_fp8_linear
from .formats import available_quant_formats, get_quant_format
from .formats.lora import LoRAMixin, is_lora_quantized, merge_lora_weight, shared_base_teacher, shared_base_teacher_enabled
from .formats.mxfp4 import (
    MXFP4Linear,
    dequantize_mxfp4,
    fake_quantize_mxfp4,
    fake_quantize_mxfp4_activation,
    quantize_mxfp4,
)
from .formats.fp8_base import dequantize_fp8_blocks
from .formats.nvfp4_experts import NVFP4ExpertLoRA, NVFP4Experts, fake_quantize_nvfp4_experts, is_fused_experts
from .formats.nvfp4 import (
    NVFP4Linear,
    attach_nvfp4_amax_groups,
    build_nvfp4_fused_family_names,
    commit_nvfp4_input_scales,
    dequantize_nvfp4,
    fake_quantize_nvfp4,
    fake_quantize_nvfp4_activation,
    finalize_nvfp4_input_scales,
    load_nvfp4_runtime_state_dict,
    nvfp4_runtime_state_dict,
    pack_e2m1_rows,
    quantize_nvfp4,
    refresh_nvfp4_weight_amax,
    unpack_e2m1_rows,
)
from .quantized_gather import NVFP4QuantizedGather
from .formats.q4_k import (
    Q4KLinear,
    configure_q4k_reorders,
    dequantize_q4_k,
    fake_quantize_q4_k,
    pack_deploy_weight,
    quantize_q4_k,
    v_head_reorder_perm,
)

__all__ = [
    "ConvertedModules",
    "LoRAMixin",
    "MXFP4Linear",
    "NVFP4Linear",
    "Q4KLinear",
    "apply_fake_quant",
    "attach_nvfp4_amax_groups",
    "available_quant_formats",
    "build_nvfp4_fused_family_names",
    "commit_nvfp4_input_scales",
    "configure_q4k_reorders",
    "dequantize_mxfp4",
    "dequantize_nvfp4",
    "dequantize_q4_k",
    "fake_quantize_mxfp4",
    "fake_quantize_mxfp4_activation",
    "fake_quantize_nvfp4",
    "fake_quantize_nvfp4_activation",
    "fake_quantize_nvfp4_experts",
    "NVFP4Experts",
    "NVFP4ExpertLoRA",
    "is_fp8_linear",
    "dequantize_fp8_blocks",
    "NVFP4QuantizedGather",
    "is_fused_experts",
    "fake_quantize_q4_k",
    "finalize_nvfp4_input_scales",
    "get_quant_format",
    "is_lora_quantized",
    "load_nvfp4_runtime_state_dict",
    "merge_lora_weight",
    "nvfp4_runtime_state_dict",
    "pack_deploy_weight",
    "pack_e2m1_rows",
    "quantize_mxfp4",
    "quantize_nvfp4",
    "quantize_q4_k",
    "refresh_nvfp4_weight_amax",
    "shared_base_teacher",
    "shared_base_teacher_enabled",
    "unpack_e2m1_rows",
    "v_head_reorder_perm",
]
