"""Swap target ``nn.Linear`` leaves of a model for fake-quant linears and freeze the rest.

Mirrors ``apply_fake_quant`` of the reference (qatfactory/quant/fake_quant.py:158-381):
same arguments, same FQN-preserving swap, same format checks and the same invariant that
only the quantized latent weights (or, with LoRA, only the adapters) train.  Packed-3D MoE
experts become ``NVFP4Experts`` (full-parameter) or ``NVFP4ExpertLoRA`` (LoRA); block-FP8
linears among the targets keep their FP8 codes as the frozen LoRA base, and the non-target
ones are dequantized to BF16 linears.
"""

from __future__ import annotations

import logging
from collections.abc import Iterable
from dataclasses import dataclass

import torch
from torch import nn

from .formats import get_quant_format
from .formats.fp8_base import dequantize_fp8_blocks, fp8_linear_state
from .formats.nvfp4_experts import LORA_LEAVES, is_fused_experts

logger = logging.getLogger(__name__)

DEFAULT_EXCLUDE_PREFIXES = (
    "model.visual",
    "visual",
    "model.vision_tower",
    "vision_tower",
    "model.vision_adapter",
    "model.vision_projection",
    "mtp",
    "lm_head",
)

_SHARED_EXPERT_SEGMENTS = frozenset({"shared_expert", "shared_experts"})


@dataclass(frozen=True)
class ConvertedModules:
    """FQNs of the converted linears (iterates as a sorted list of target names)."""

    linears: tuple[str, ...]
    experts: tuple[str, ...] = ()
    expert_targets: tuple[str, ...] = ()
    lora: bool = False

    @property
    def all(self) -> list[str]:
        return sorted((*self.linears, *self.expert_targets))

    @property
    def trainable_parameters(self) -> set[str]:
        if self.lora:
            parameters = {f"{n}.{leaf}" for n in self.linears for leaf in ("lora_A", "lora_B")}
            for name in self.experts:  # NVFP4ExpertLoRA trains only its adapters
                parameters.update(f"{name}.{leaf}" for leaf in LORA_LEAVES)
            return parameters
        parameters = {f"{n}.weight" for n in self.linears}
        for name in self.experts:  # full-parameter NVFP4Experts train both fused latents
            parameters.update((f"{name}.gate_up_proj", f"{name}.down_proj"))
        return parameters

    def __iter__(self):
        return iter(self.all)

    def __len__(self) -> int:
        return len(self.all)


def is_fp8_linear(module: nn.Module) -> bool:
    return fp8_linear_state(module) is not None


def dequantize_remaining_fp8_linears(model: nn.Module) -> list[str]:
    """Replace every block-FP8 linear that is not a quantization target by a frozen BF16
    ``nn.Linear`` of the same dequantized weight, so no vendor FP8 matmul runs in the forward
    (fake_quant.py:25-56); returns their names."""

    replaced = []
    for parent_name, parent in list(model.named_modules()):
        for child_name, child in list(parent.named_children()):
            state = fp8_linear_state(child)
            if state is None:
                continue
            weight, scale_inv = state
            linear = nn.Linear(child.in_features, child.out_features, bias=child.bias is not None, device="meta")
            linear.weight = nn.Parameter(dequantize_fp8_blocks(weight, scale_inv, torch.bfloat16), requires_grad=False)
            linear.bias = child.bias
            setattr(parent, child_name, linear)
            replaced.append(f"{parent_name}.{child_name}" if parent_name else child_name)
    return replaced


def _mark_quantized_base_as_qat_trainable(model: nn.Module) -> None:
    """A model loaded through an HF quantizer is trainable here (only the LoRA adapters over
    the frozen quantized base train): advertise that on a per-model subclass of the quantizer,
    whose two flags are read-only properties (fake_quant.py:59-84)."""

    quantizer = getattr(model, "hf_quantizer", None)
    if quantizer is None or (quantizer.is_qat_trainable and quantizer.is_trainable):
        return
    flags = {"is_qat_trainable": property(lambda self: True), "is_trainable": property(lambda self: True)}
    quantizer.__class__ = type(f"QATTrainable{type(quantizer).__name__}", (type(quantizer),), flags)


def _excluded(name: str, prefixes: tuple[str, ...]) -> bool:
    return any(name == p or name.startswith(p + ".") for p in prefixes)


def apply_fake_quant(
    model: nn.Module,
    target_modules: Iterable[str],
    *,
    quant_format: str = "nvfp4",
    exclude_prefixes: Iterable[str] = DEFAULT_EXCLUDE_PREFIXES,
    fused_runtime_scales: bool = False,
    quantize_activations: bool = False,
    lora_rank: int = 0,
    lora_alpha: float = 0.0,
    lora_moe_hybrid_shared: bool = True,
    expert_checkpointing: bool = True,
    quantize_shared_expert: bool = True,
) -> ConvertedModules:
    """Replace target ``nn.Linear`` leaves with the format's fake-quant linear (see module doc)."""

    fmt = get_quant_format(quant_format)
    targets = set(target_modules)
    prefixes = tuple(exclude_prefixes)
    if fused_runtime_scales and not fmt.supports_fused_runtime_scales:
        raise ValueError(f"quant_format={quant_format!r} does not support fused_runtime_scales.")
    if quantize_activations and not fmt.supports_activation_quant:
        raise ValueError(f"quant_format={quant_format!r} does not support input-activation fake-quant (W4A4).")
    if quantize_activations and fmt.activation_quant_requires_runtime_scales and not fused_runtime_scales:
        raise ValueError(
            f"quant_format={quant_format!r} W4A4 requires fused_runtime_scales=True to track the "
            "activation running-max used as the static global scale."
        )
    use_lora = bool(lora_rank and lora_rank > 0)
    if use_lora and not fmt.supports_lora:
        raise ValueError(f"quant_format={quant_format!r} does not support LoRA-QAD.")
    config = getattr(model, "config", None)
    text_config = config.get_text_config() if hasattr(config, "get_text_config") else config
    is_moe = bool(text_config is not None and getattr(text_config, "num_experts", None))
    if not targets and not is_moe:
        raise ValueError("apply_fake_quant requires a non-empty target_modules set.")
    # fused routed experts: full-parameter NVFP4Experts, or NVFP4ExpertLoRA under LoRA
    if is_moe and (fmt.from_experts if use_lora else fmt.from_experts_full) is None:
        raise ValueError(
            f"quant_format={quant_format!r} does not support "
            f"{'LoRA' if use_lora else 'full-parameter'} QAD of fused routed experts."
        )
    tied = bool(getattr(config, "tie_word_embeddings", False) or getattr(text_config, "tie_word_embeddings", False))
    if tied and targets & {"embed_tokens", "lm_head"}:
        raise ValueError(
            "Tied embeddings cannot be a quantization target: remove embed_tokens/lm_head "
            "from target_modules (the shared tensor must stay frozen and unquantized)."
        )

    model.requires_grad_(False)
    converted: list[str] = []
    converted_experts: list[str] = []
    expert_targets: list[str] = []
    skipped_shared = 0
    for parent_name, parent in list(model.named_modules()):
        if _excluded(parent_name, prefixes):
            continue
        in_shared_expert = not _SHARED_EXPERT_SEGMENTS.isdisjoint(parent_name.split("."))
        for child_name, child in list(parent.named_children()):
            module_name = f"{parent_name}.{child_name}" if parent_name else child_name
            if is_moe and is_fused_experts(child):
                if use_lora:
                    replacement = fmt.from_experts(child, int(lora_rank), float(lora_alpha),
                                                   hybrid_shared=lora_moe_hybrid_shared,
                                                   expert_checkpointing=expert_checkpointing)
                else:
                    replacement = fmt.from_experts_full(child)
                setattr(parent, child_name, replacement)
                converted_experts.append(module_name)
                expert_targets.extend(replacement.target_names(module_name))
                continue
            if child_name not in targets or not isinstance(child, nn.Linear):
                continue
            if in_shared_expert and not quantize_shared_expert:
                skipped_shared += 1
                continue
            # a pre-quantized block-FP8 linear keeps its codes as the frozen base
            fp8 = fmt.from_fp8_linear is not None and fp8_linear_state(child) is not None
            setattr(parent, child_name, fmt.from_fp8_linear(child) if fp8 else fmt.from_linear(child))
            converted.append(f"{parent_name}.{child_name}" if parent_name else child_name)
    if not converted and not converted_experts:
        raise ValueError(f"No modules matched target suffixes {sorted(targets)}.")
    if is_moe and not converted_experts:
        raise ValueError(
            "MoE model (num_experts set) but no fused routed-expert modules were found to convert; "
            "only packed 3D gate_up_proj/down_proj experts (transformers>=5) are supported."
        )
    if not quantize_shared_expert and not skipped_shared:
        raise ValueError(
            "quantize_shared_expert=False but no shared-expert Linear modules were found to skip; "
            "check the model's shared-expert module naming."
        )
    if targets and not converted:
        raise ValueError(f"No linear modules matched target suffixes {sorted(targets)}.")

    for module in model.modules():
        if getattr(module, "_is_nvfp4_experts", False):
            if not use_lora:  # NVFP4ExpertLoRA's adapters are created trainable, its base frozen
                module.gate_up_proj.requires_grad_(True)
                module.down_proj.requires_grad_(True)
            continue
        if not isinstance(module, fmt.linear_cls):
            continue
        if use_lora:
            module.init_lora(int(lora_rank), float(lora_alpha))
            module.weight.requires_grad_(False)
            module.lora_A.requires_grad_(True)
            module.lora_B.requires_grad_(True)
        else:
            module.weight.requires_grad_(True)
        if module.bias is not None:
            module.bias.requires_grad_(False)
    if fused_runtime_scales:
        fmt.attach_amax_groups(model)
        for module in model.modules():
            if getattr(module, "_is_nvfp4_experts", False):
                module._track_input_amax = True
    if quantize_activations:
        for module in model.modules():
            if isinstance(module, fmt.linear_cls) or getattr(module, "_is_nvfp4_experts", False):
                module._quantize_activations = True

    result = ConvertedModules(linears=tuple(sorted(converted)), experts=tuple(sorted(converted_experts)),
                              expert_targets=tuple(sorted(expert_targets)), lora=use_lora)
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    missing = result.trainable_parameters - trainable
    unexpected = trainable - result.trainable_parameters
    if missing:
        raise RuntimeError(f"Expected trainable parameters (quantized latents or LoRA adapters) are frozen: {sorted(missing)[:8]}.")
    if unexpected:
        raise RuntimeError(
            f"Non-quantized parameters would be trained during distillation: {sorted(unexpected)[:8]}. "
            "By default only quantized-linear latent weights (or LoRA adapters) are trainable."
        )
    leftover = dequantize_remaining_fp8_linears(model)
    if leftover:
        logger.info("Dequantized %d non-target FP8 linears to BF16 (e.g. %s).", len(leftover), leftover[0])
    if use_lora:
        _mark_quantized_base_as_qat_trainable(model)
    logger.info(
        "Enabled %s %s QAD: %d quantized linears.",
        quant_format,
        "W4A4" if quantize_activations else "weight-only",
        len(result.linears),
    )
    return result
