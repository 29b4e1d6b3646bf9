"""Quantization-format registry (the reference's ``QuantFormat`` plugin interface,
qatfactory/quant/formats/__init__.py:18-192), bound to the B200 implementations.

``get_quant_format(name)`` returns the descriptor the instrumentation (``apply_fake_quant``),
trainers and exporters dispatch on; names, quantizer ids, capability flags and lifecycle
hooks match the reference for the formats this package implements: ``nvfp4``, ``mxfp4``,
``q4_k`` (min-max level-1 fit) and ``q4_k_grid_search``.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from functools import partial

from torch import nn


@dataclass(frozen=True)
class QuantFormat:
    """One fake-quant format and its optional lifecycle hooks."""

    name: str
    linear_cls: type[nn.Module]
    from_linear: Callable[[nn.Linear], nn.Module]
    quantizer_id: str
    supports_fused_runtime_scales: bool
    supports_lora: bool = True
    supports_activation_quant: bool = False
    activation_quant_requires_runtime_scales: bool = False
    commit_input_scales: Callable | None = None
    from_fp8_linear: Callable[[nn.Module], nn.Module] | None = None
    experts_cls: type[nn.Module] | None = None
    from_experts: Callable[..., nn.Module] | None = None
    from_experts_full: Callable[[nn.Module], nn.Module] | None = None
    is_fused_experts: Callable[[nn.Module], bool] = lambda module: False
    attach_amax_groups: Callable | None = None
    refresh_weight_amax: Callable | None = None
    finalize_input_scales: Callable | None = None
    runtime_state_dict: Callable | None = None
    load_runtime_state_dict: Callable | None = None
    pack_weight: Callable | None = None
    packed_weight_filename: str | None = None


def _nvfp4() -> QuantFormat:
    from . import nvfp4
    from .nvfp4_experts import NVFP4ExpertLoRA, NVFP4Experts, is_fused_experts

    return QuantFormat(
        name="nvfp4",
        linear_cls=nvfp4.NVFP4Linear,
        from_linear=nvfp4.NVFP4Linear.from_linear,
        quantizer_id="standard_max",
        supports_fused_runtime_scales=True,
        supports_activation_quant=True,
        activation_quant_requires_runtime_scales=True,
        commit_input_scales=nvfp4.commit_nvfp4_input_scales,
        attach_amax_groups=nvfp4.attach_nvfp4_amax_groups,
        refresh_weight_amax=nvfp4.refresh_nvfp4_weight_amax,
        finalize_input_scales=nvfp4.finalize_nvfp4_input_scales,
        runtime_state_dict=nvfp4.nvfp4_runtime_state_dict,
        load_runtime_state_dict=nvfp4.load_nvfp4_runtime_state_dict,
        from_fp8_linear=nvfp4.NVFP4Linear.from_fp8_linear,
        experts_cls=NVFP4ExpertLoRA,
        from_experts=NVFP4ExpertLoRA,
        from_experts_full=NVFP4Experts.from_experts,
        is_fused_experts=is_fused_experts,
    )


def _q4_k_pack_hook(default_method: str):
    def pack(weight, module=None):
        from .q4_k import pack_deploy_weight

        row_perm = getattr(module, "q4k_row_perm", None) if module is not None else None
        col_perm = getattr(module, "q4k_col_perm", None) if module is not None else None
        method = getattr(module, "quant_method", default_method) if module is not None else default_method
        return pack_deploy_weight(weight, row_perm=row_perm, col_perm=col_perm, method=method)

    return pack


def _q4_k(name: str, quantizer_id: str, method: str) -> QuantFormat:
    from .q4_k import Q4KLinear

    return QuantFormat(
        name=name,
        linear_cls=Q4KLinear,
        from_linear=partial(Q4KLinear.from_linear, method=method),
        quantizer_id=quantizer_id,
        supports_fused_runtime_scales=False,
        supports_lora=False,
        pack_weight=_q4_k_pack_hook(method),
        packed_weight_filename="q4k_weight.safetensors",
    )


def _mxfp4() -> QuantFormat:
    from .mxfp4 import MXFP4Linear

    return QuantFormat(
        name="mxfp4",
        linear_cls=MXFP4Linear,
        from_linear=MXFP4Linear.from_linear,
        quantizer_id="mx_even",
        supports_fused_runtime_scales=False,
        supports_activation_quant=True,
    )


_BUILDERS = {
    "mxfp4": _mxfp4,
    "nvfp4": _nvfp4,
    "q4_k": lambda: _q4_k("q4_k", "q4_k_minmax", "minmax"),
    "q4_k_grid_search": lambda: _q4_k("q4_k_grid_search", "q4_k_grid_search", "grid_search"),
}


def get_quant_format(name: str) -> QuantFormat:
    try:
        builder = _BUILDERS[name]
    except KeyError as exc:
        raise ValueError(f"Unknown quant_format {name!r}; supported formats: {sorted(_BUILDERS)}.") from exc
    return builder()


def available_quant_formats() -> list[str]:
    return sorted(_BUILDERS)
