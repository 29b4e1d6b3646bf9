"""LoRA merge hook and the shared-base-teacher switch used by the quantized linears.

Mirrors the reference's format-agnostic helpers (qatfactory/quant/formats/lora.py): a
quantized linear may carry a low-rank adapter ``scaling * (B @ A)`` that is folded into the
frozen base weight before fake quantization, and inside ``shared_base_teacher()`` every
quantized linear returns its plain full-precision result so one model can serve as its own
teacher.  LoRA-QAD itself is not a benchmark configuration; the hook exists so that
``_effective_weight()`` feeds the kernels exactly what the reference quantizes.
"""

from __future__ import annotations

import math
from collections.abc import Iterator
from contextlib import contextmanager
from contextvars import ContextVar

import torch
from torch import nn

_TEACHER_MODE = ContextVar("qatfactory_b200_shared_base_teacher", default=False)


def shared_base_teacher_enabled() -> bool:
    return _TEACHER_MODE.get()


@contextmanager
def shared_base_teacher() -> Iterator[None]:
    token = _TEACHER_MODE.set(True)
    try:
        yield
    finally:
        _TEACHER_MODE.reset(token)


class LoRAMixin:
    """Optional rank-r adapter on a quantized linear (reference lora.py:50-113)."""

    lora_rank: int = 0
    lora_scaling: float = 1.0

    def init_lora(self, rank: int, alpha: float) -> None:
        if rank <= 0:
            raise ValueError(f"LoRA rank must be positive, got {rank}.")
        base = self.base_weight()
        self.lora_rank = int(rank)
        self.lora_scaling = float(alpha) / float(rank)
        self.lora_A = nn.Parameter(torch.empty(rank, self.in_features, device=base.device, dtype=base.dtype))
        self.lora_B = nn.Parameter(torch.zeros(self.out_features, rank, device=base.device, dtype=base.dtype))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))

    @property
    def has_lora(self) -> bool:
        return getattr(self, "lora_A", None) is not None

    def base_weight(self) -> torch.Tensor:
        return self.weight

    def lora_delta(self) -> torch.Tensor:
        return self.lora_scaling * (self.lora_B @ self.lora_A)

    def _effective_weight(self) -> torch.Tensor:
        base = self.base_weight()
        if getattr(self, "lora_A", None) is None:
            return base
        return base + self.lora_delta().to(base.dtype)


def is_lora_quantized(module: nn.Module) -> bool:
    return isinstance(module, LoRAMixin) and getattr(module, "lora_A", None) is not None


def merge_lora_weight(weight: torch.Tensor, lora_A: torch.Tensor, lora_B: torch.Tensor, scaling: float) -> torch.Tensor:
    return weight + (scaling * (lora_B @ lora_A)).to(weight.dtype)
