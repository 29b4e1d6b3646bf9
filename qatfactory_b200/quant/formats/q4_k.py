"""Q4_K fake quantization on B200: the ``qatfactory.quant`` Q4_K API over libqatf.so.

Two-level llama.cpp ``block_q4_K`` lattice (reference qatfactory/quant/formats/q4_k.py):
256-weight super-blocks of eight 32-weight sub-blocks, 6-bit sub-block scales/mins against
FP16 super-block scales.  The training fake quant and the save-time pack call the same
encoder kernel, so the exported blocks dequantize to exactly what the student trained
with, and both match the reference's torch encoder bit for bit (``minmax`` and the
``grid_search`` of make_qkx2_quants).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from ... import _native
from .nvfp4 import _MaskedStraightThrough

QK_K = 256
Q4K_GROUP = 32
Q4K_NSUB = QK_K // Q4K_GROUP
Q4K_NMAX = 15
Q4K_L2MAX = 63
Q4K_BLOCK_BYTES = 2 + 2 + 12 + 128
Q4K_METHODS = ("grid_search", "minmax")


def _check_shape(weight: torch.Tensor) -> None:
    if weight.ndim != 2:
        raise ValueError(f"Q4_K expects a 2D weight, got shape {tuple(weight.shape)}.")
    if weight.shape[-1] % QK_K:
        raise ValueError(
            f"Q4_K requires in_features divisible by {QK_K}, got {weight.shape[-1]}. "
            "llama.cpp falls back to another type for such tensors; exclude them from the target set."
        )


def _check_method(method: str) -> None:
    if method not in Q4K_METHODS:
        raise ValueError(f"Unknown Q4_K method {method!r}; supported: {Q4K_METHODS}.")


def _inverse(perm: torch.Tensor) -> torch.Tensor:
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(perm.numel(), device=perm.device)
    return inverse


def fake_quantize_q4_k(
    weight: torch.Tensor, *, col_perm: torch.Tensor | None = None, method: str = "grid_search"
) -> torch.Tensor:
    """Fake-quantize a linear weight on the Q4_K lattice with a masked STE (q4_k.py:245-277).

    ``col_perm`` (Qwen3.5 ``out_proj``) encodes the column-permuted weight and un-permutes the
    reconstruction, so training matches the reordered GGUF value for value."""

    if weight.is_meta:
        return weight
    _check_shape(weight)
    _check_method(method)
    permuted = weight if col_perm is None else weight.index_select(1, col_perm.to(weight.device))
    with torch.no_grad():
        _, recon, mask = _native.q4k_encode(permuted.detach(), method, recon=True, mask=True, blocks=False)
    if col_perm is None:
        return _MaskedStraightThrough.apply(weight, recon, mask)
    inverse = _inverse(col_perm.to(weight.device))
    in_range = _native.unpack_mask(mask, recon.numel(), recon.shape).index_select(1, inverse)
    recon = recon.index_select(1, inverse)
    return _PermutedStraightThrough.apply(weight, recon, in_range)


class _PermutedStraightThrough(torch.autograd.Function):
    """STE with a dense bool mask (only the column-permuted path needs one)."""

    @staticmethod
    def forward(ctx, latent, quantized, in_range):
        ctx.save_for_backward(in_range)
        return quantized

    @staticmethod
    def backward(ctx, grad_output):
        (in_range,) = ctx.saved_tensors
        return grad_output * in_range, None, None


@dataclass(frozen=True)
class Q4KQuantizationResult:
    packed_weight: torch.Tensor  # [out_features, n_super * 144] uint8 (ggml block_q4_K bytes)
    reconstruction: torch.Tensor  # [out_features, in_features], weight dtype


@torch.no_grad()
def quantize_q4_k(weight: torch.Tensor, *, method: str = "grid_search") -> Q4KQuantizationResult:
    """Encode a 2D weight into ggml ``block_q4_K`` bytes plus the reconstruction (q4_k.py:318-340)."""

    if weight.is_meta:
        raise ValueError("Cannot pack a Q4_K lattice from a meta tensor.")
    _check_shape(weight)
    _check_method(method)
    blocks, recon, _ = _native.q4k_encode(weight.detach(), method, recon=True, mask=False, blocks=True)
    return Q4KQuantizationResult(packed_weight=blocks, reconstruction=recon)


def dequantize_q4_k(packed_weight: torch.Tensor, in_features: int) -> torch.Tensor:
    """Dequantize ggml ``block_q4_K`` bytes to FP32 (q4_k.py:359-385)."""

    if packed_weight.dtype != torch.uint8 or packed_weight.ndim != 2:
        raise ValueError(f"Q4_K blocks must be 2D uint8, got {packed_weight.dtype} {tuple(packed_weight.shape)}.")
    if in_features % QK_K or packed_weight.shape[1] != in_features // QK_K * Q4K_BLOCK_BYTES:
        raise ValueError(f"Q4_K blocks of shape {tuple(packed_weight.shape)} do not hold {in_features} features.")
    return _native.q4k_dequant(packed_weight, in_features)


@torch.no_grad()
def pack_deploy_weight(
    weight: torch.Tensor,
    *,
    row_perm: torch.Tensor | None = None,
    col_perm: torch.Tensor | None = None,
    method: str = "grid_search",
) -> torch.Tensor:
    """Deployed-layout Q4_K blocks with optional GGUF row/column reorders (q4_k.py:388-408)."""

    if row_perm is not None:
        weight = weight.index_select(0, row_perm.to(weight.device))
    if col_perm is not None:
        weight = weight.index_select(1, col_perm.to(weight.device))
    return quantize_q4_k(weight, method=method).packed_weight


def v_head_reorder_perm(num_k_heads: int, num_v_per_k: int, head_dim: int) -> torch.Tensor:
    """Grouped-by-K -> tiled V-head permutation with ``deployed[i] = hf[P[i]]`` (q4_k.py:411-420)."""

    total = num_k_heads * num_v_per_k * head_dim
    return torch.arange(total, dtype=torch.long).reshape(num_k_heads, num_v_per_k, head_dim).transpose(0, 1).reshape(-1)


def configure_q4k_reorders(model: nn.Module) -> int:
    """Attach Qwen3.5 linear-attention GGUF reorders to ``Q4KLinear`` targets (q4_k.py:423-461)."""

    config = model.config
    text_config = config.get_text_config() if hasattr(config, "get_text_config") else config
    num_k = int(getattr(text_config, "linear_num_key_heads", 0) or 0)
    num_v = int(getattr(text_config, "linear_num_value_heads", 0) or 0)
    if not num_k or not num_v or num_k == num_v:
        return 0
    per_k = num_v // num_k
    head_v = int(text_config.linear_value_head_dim)
    head_k = int(text_config.linear_key_head_dim)
    v_perm = v_head_reorder_perm(num_k, per_k, head_v)
    scalar_perm = v_head_reorder_perm(num_k, per_k, 1)
    qk_rows = 2 * head_k * num_k
    qkv_perm = torch.cat([torch.arange(qk_rows, dtype=torch.long), qk_rows + v_perm])
    count = 0
    for name, module in model.named_modules():
        if not isinstance(module, Q4KLinear):
            continue
        if name.endswith(".linear_attn.in_proj_qkv"):
            module.q4k_row_perm = qkv_perm
        elif name.endswith(".linear_attn.in_proj_z"):
            module.q4k_row_perm = v_perm
        elif name.endswith((".linear_attn.in_proj_a", ".linear_attn.in_proj_b")):
            module.q4k_row_perm = scalar_perm
        elif name.endswith(".linear_attn.out_proj"):
            module.q4k_col_perm = v_perm
        else:
            continue
        count += 1
    return count


class Q4KLinear(nn.Linear):
    """Linear layer whose weight is Q4_K fake-quantized on every forward (q4_k.py:464-498)."""

    @classmethod
    def from_linear(cls, module: nn.Linear, *, method: str = "grid_search") -> "Q4KLinear":
        if module.in_features % QK_K:
            raise ValueError(
                f"Q4_K requires in_features divisible by {QK_K}, got {module.in_features}; "
                "exclude this module from the target set."
            )
        _check_method(method)
        converted = cls(module.in_features, module.out_features, bias=module.bias is not None, device="meta")
        converted.weight = module.weight
        converted.bias = module.bias
        converted.quant_method = method
        converted.q4k_row_perm = None
        converted.q4k_col_perm = None
        return converted

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        method = getattr(self, "quant_method", "grid_search")
        return F.linear(input, fake_quantize_q4_k(self.weight, col_perm=self.q4k_col_perm, method=method), self.bias)
