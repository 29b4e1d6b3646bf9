"""NVFP4 fake quantization of fused routed-expert weights ``[experts, rows, in_features]``.

Recent MoE backbones keep every routed expert in fused 3-D parameters (``gate_up_proj``
``[E, 2*intermediate, hidden]``, ``down_proj`` ``[E, hidden, intermediate]``).  Each expert
slice is quantized with exactly the 2-D NVFP4 math and its own tensor amax, so one batched
kernel launch (``qatf_nvfp4_qdq_experts``) replaces the reference's slab-by-slab torch
computation (``qatfactory/quant/formats/nvfp4_experts.py:386-462``) bit for bit.

Provided here: ``fake_quantize_nvfp4_experts``, the per-expert ``_ExpertFakeQuantLinear``,
``is_fused_experts`` and the full-parameter routed-experts module ``NVFP4Experts``
(nvfp4_experts.py:496-649), whose per-expert tensor amax is one batched kernel launch per
projection.  With BF16 weights and activations on the GPU, its W4A16 forward runs every routed
expert as one grouped GEMM per projection (``torch._grouped_mm``) instead of the reference's
loop over experts; W4A4 keeps the loop.  ``NVFP4ExpertLoRA`` (nvfp4_experts.py:65-366) is the
LoRA-QAD variant: a frozen base, BF16 or block-FP8 codes dequantized per expert, with low-rank
adapters merged into every expert's weight before its fake quantization.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F
import torch.utils.checkpoint
from torch import nn

from ... import _native
from .fp8_base import dequantize_fp8_blocks, fp8_experts_state
from .lora import shared_base_teacher_enabled
from .nvfp4 import (NVFP4_BLOCK_SIZE, NVFP4_SCALE_DENOMINATOR, _MaskedStraightThrough, fake_quantize_nvfp4,
                    fake_quantize_nvfp4_activation)

__all__ = ["fake_quantize_nvfp4_experts", "is_fused_experts", "fused_experts_shapes", "NVFP4Experts",
           "NVFP4ExpertLoRA", "LORA_LEAVES"]

EXPERT_PROJECTIONS = ("w1", "w3", "w2")


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


class _GroupedExpertFakeQuantLinear(torch.autograd.Function):
    """Every routed expert's ``F.linear(x_e, fake_quant(w_e))`` as one grouped GEMM: the rows
    of ``x`` sorted by expert, group e ending at row ``offs[e]`` (int32, cumulative counts; an
    expert with no rows is an empty group).  All experts are quantized in one launch with their
    own tensor amax; as in ``_ExpertFakeQuantLinear`` the quantized weights and masks are
    recomputed in backward, where the masked straight-through gradient of every expert comes from
    one grouped GEMM (an expert without rows gets a zero gradient, as in the reference's loop)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, amax: torch.Tensor, offs: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            quantized, _ = _native.nvfp4_qdq_experts(w.detach(), amax, want_mask=False)
        ctx.save_for_backward(x, w, amax, offs)
        return torch._grouped_mm(x, quantized.transpose(1, 2), offs=offs)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x, w, amax, offs = ctx.saved_tensors
        with torch.no_grad():
            quantized, mask = _native.nvfp4_qdq_experts(w.detach(), amax)
        grad_output = grad_output.contiguous()
        grad_x = torch._grouped_mm(grad_output, quantized, offs=offs) if ctx.needs_input_grad[0] else None
        grad_w = None
        if ctx.needs_input_grad[1]:
            grad_w = torch._grouped_mm(grad_output.t(), x, offs=offs)  # [E, out, in]: g_e^T x_e per expert
            grad_w = _native.ste_backward(grad_w.contiguous(), mask).reshape(w.shape)
        return grad_x, grad_w, None, None


def grouped_experts_supported(hidden_states: torch.Tensor, *weights: torch.Tensor) -> bool:
    """The grouped path runs BF16 operands on the GPU through ``torch._grouped_mm``."""

    return (hasattr(torch, "_grouped_mm") and hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16
            and all(w.dtype == torch.bfloat16 for w in weights))


class _ExpertInputScales:
    """The W4A4 activation-scale lifecycle both expert modules share with the NVFP4 scale
    lifecycle of ``nvfp4.py`` (nvfp4_experts.py:146-187, :496-649): one static scale for the
    block input of all experts (w13) and one for the expert intermediates (w2), published from
    the running maxima between optimizer steps."""

    _is_nvfp4_experts = True
    # the two activation scales a serving fused-MoE layer carries, in export order
    INPUT_SCALE_GROUPS = (("w13", "_gate_up_input_amax"), ("w2", "_down_input_amax"))

    def _init_input_scales(self) -> None:
        self._track_input_amax = False
        self._quantize_activations = False
        self._gate_up_input_amax = None
        self._gate_up_input_amax_static = None
        self._down_input_amax = None
        self._down_input_amax_static = None

    def target_names(self, prefix: str) -> list[str]:
        """Per-expert projection names in serving (w1 / w3 / w2) naming."""

        return [f"{prefix}.{e}.{p}" for e in range(self.num_experts) for p in EXPERT_PROJECTIONS]

    @torch.no_grad()
    def commit_input_scales(self, process_group=None) -> None:
        """Publish the running input maxima as the next step's static W4A4 scales."""

        if not self._quantize_activations or self._gate_up_input_amax is None:
            return
        maxima = torch.stack([self._gate_up_input_amax, self._down_input_amax])
        if dist.is_initialized():
            dist.all_reduce(maxima, op=dist.ReduceOp.MAX, group=process_group)
        self._gate_up_input_amax, self._down_input_amax = (value.clone() for value in maxima.unbind())
        self._gate_up_input_amax_static, self._down_input_amax_static = maxima.unbind()

    @torch.no_grad()
    def finalize_input_scales(self, prefix: str, process_group=None) -> dict[str, torch.Tensor]:
        """Reduce the running maxima and return this layer's exported activation scales."""

        if self._gate_up_input_amax is None:
            raise RuntimeError(f"Missing training input-amax observations for {prefix}.")
        maxima = torch.stack([self._gate_up_input_amax, self._down_input_amax])
        if dist.is_initialized():
            dist.all_reduce(maxima, op=dist.ReduceOp.MAX, group=process_group)
        self._gate_up_input_amax, self._down_input_amax = (value.clone() for value in maxima.unbind())
        scales = {}
        for (name, _), maximum in zip(self.INPUT_SCALE_GROUPS, maxima.unbind(), strict=True):
            if not bool(torch.isfinite(maximum)) or not bool(maximum > 0):
                raise RuntimeError(f"Invalid training input amax for {prefix}.{name}.")
            scales[f"{prefix}.{name}.input_scale"] = (maximum / NVFP4_SCALE_DENOMINATOR).reshape(())
        return scales

    def runtime_state_dict(self) -> dict[str, torch.Tensor]:
        return {name: getattr(self, attribute).detach().cpu() for name, attribute in self.INPUT_SCALE_GROUPS
                if getattr(self, attribute) is not None}

    def load_runtime_state_dict(self, state: dict[str, torch.Tensor], device) -> None:
        for name, attribute in self.INPUT_SCALE_GROUPS:
            if name not in state:
                continue
            value = state[name].to(device).reshape(())
            setattr(self, attribute, value)
            setattr(self, f"{attribute}_static", value.clone())

    @staticmethod
    def _grow(running: torch.Tensor | None, value: torch.Tensor) -> torch.Tensor:
        amax = _native.tensor_amax(value.detach())
        return amax if running is None else torch.maximum(running, amax)


class NVFP4Experts(_ExpertInputScales, nn.Module):
    """Full-parameter NVFP4 QAD of fused routed experts (nvfp4_experts.py:496-649): a drop-in
    for a transformers fused experts module (``forward(hidden_states, top_k_index,
    top_k_weights)`` over ``gate_up_proj`` ``[E, 2 * intermediate, hidden]`` and ``down_proj``
    ``[E, hidden, intermediate]``).  Both 3-D latents train; every routed expert is
    fake-quantized inside its own matmul with its own tensor amax (the whole ``gate_up_proj[e]``
    slice shares one, so w1 and w3 export one global scale).  W4A4 quantizes the block input
    with one static scale for all experts (w13) and the expert intermediates with another
    (w2), with the same step-static lifecycle as the reference."""

    def __init__(self, gate_up_proj: nn.Parameter, down_proj: nn.Parameter, act_fn):
        super().__init__()
        if gate_up_proj.ndim != 3 or down_proj.ndim != 3:
            raise ValueError("NVFP4Experts requires fused 3D gate_up_proj and down_proj parameters.")
        num_experts, two_intermediate, hidden = gate_up_proj.shape
        if two_intermediate % 2 or down_proj.shape != (num_experts, hidden, two_intermediate // 2):
            raise ValueError(
                f"Inconsistent expert shapes: gate_up_proj {tuple(gate_up_proj.shape)}, "
                f"down_proj {tuple(down_proj.shape)}."
            )
        for name, parameter in (("gate_up_proj", gate_up_proj), ("down_proj", down_proj)):
            if parameter.shape[-1] % NVFP4_BLOCK_SIZE:
                raise ValueError(
                    f"NVFP4 requires {name} in_features divisible by {NVFP4_BLOCK_SIZE}, got {tuple(parameter.shape)}."
                )
        self.num_experts = num_experts
        self.hidden_dim = hidden
        self.intermediate_dim = two_intermediate // 2
        self.gate_up_proj = gate_up_proj
        self.down_proj = down_proj
        self.act_fn = act_fn
        self._init_input_scales()

    @classmethod
    def from_experts(cls, module: nn.Module) -> "NVFP4Experts":
        for attribute in ("gate_up_proj", "down_proj", "act_fn"):
            if not hasattr(module, attribute):
                raise ValueError(f"Cannot convert {type(module).__name__}: missing {attribute!r}.")
        if module.gate_up_proj.dtype == torch.float8_e4m3fn or module.down_proj.dtype == torch.float8_e4m3fn:
            raise ValueError(
                "Full-parameter expert QAD trains the expert latents and needs a BF16 base; "
                "dequantize the FP8 checkpoint first."
            )
        if getattr(module, "has_bias", False) or getattr(module, "is_transposed", False):
            raise ValueError("NVFP4 expert QAD supports only non-transposed, bias-free expert weights.")
        for name, _ in module.named_parameters():
            if name not in {"gate_up_proj", "down_proj"}:
                raise ValueError(f"Unsupported extra expert parameter {name!r} (biased experts are not supported).")
        return cls(module.gate_up_proj, module.down_proj, module.act_fn)

    def trainable_parameter_names(self, prefix: str) -> set[str]:
        return {f"{prefix}.gate_up_proj", f"{prefix}.down_proj"}

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor) -> torch.Tensor:
        tracking = self._track_input_amax and self.training
        quantize = self._quantize_activations
        if quantize:
            # W4A4: one step-static scale for the block input (all experts, like serving's w13);
            # the very first forward bootstraps it
            if self._gate_up_input_amax_static is None:
                self._gate_up_input_amax_static = _native.tensor_amax(hidden_states.detach())
            if tracking:
                self._gate_up_input_amax = self._grow(self._gate_up_input_amax, hidden_states)
            hidden_states = fake_quantize_nvfp4_activation(hidden_states, self._gate_up_input_amax_static)
        elif tracking:
            self._gate_up_input_amax = self._grow(self._gate_up_input_amax, hidden_states)

        # per-expert tensor amax of each projection: one batched launch each
        gate_up_amax = _native.tensor_amax_batched(self.gate_up_proj.detach())
        down_amax = _native.tensor_amax_batched(self.down_proj.detach())
        _check_expert_amax(gate_up_amax)
        _check_expert_amax(down_amax)
        if grouped_experts_supported(hidden_states, self.gate_up_proj, self.down_proj):
            return self._forward_grouped(hidden_states, top_k_index, top_k_weights, gate_up_amax, down_amax, tracking,
                                         quantize)
        gate_up = self.gate_up_proj.unbind(0)
        down = self.down_proj.unbind(0)

        final_hidden_states = torch.zeros_like(hidden_states)
        with torch.no_grad():
            hit_experts = torch.unique(top_k_index)
        for expert_index in hit_experts.tolist():
            if not 0 <= expert_index < self.num_experts:  # expert-parallel padding sentinel
                continue
            token_index, k_position = torch.where(top_k_index == expert_index)
            gate, up = _ExpertFakeQuantLinear.apply(
                hidden_states[token_index], gate_up[expert_index], gate_up_amax[expert_index]
            ).chunk(2, dim=-1)
            intermediate = self.act_fn(gate) * up
            if quantize:
                if self._down_input_amax_static is None:  # first-ever forward: bootstrap from this expert
                    self._down_input_amax_static = _native.tensor_amax(intermediate.detach())
                if tracking:
                    self._down_input_amax = self._grow(self._down_input_amax, intermediate)
                intermediate = fake_quantize_nvfp4_activation(intermediate, self._down_input_amax_static)
            elif tracking:
                self._down_input_amax = self._grow(self._down_input_amax, intermediate)
            expert_output = _ExpertFakeQuantLinear.apply(intermediate, down[expert_index], down_amax[expert_index])
            expert_output = expert_output * top_k_weights[token_index, k_position, None]
            final_hidden_states.index_add_(0, token_index, expert_output.to(final_hidden_states.dtype))
        return final_hidden_states

    def _forward_grouped(self, hidden_states, top_k_index, top_k_weights, gate_up_amax, down_amax, tracking,
                         quantize=False):
        """The forward of every routed expert as two grouped GEMMs (``torch._grouped_mm``)
        instead of a loop over experts: the same products, and the same sum as the reference
        (each token's expert outputs added in ascending expert order in the dtype of
        ``hidden_states``, as its one ``index_add_`` per expert does).  With W4A4 the block input
        arrives quantized; the intermediates of all experts share one static scale and the
        quantizer is row-separable, so they are quantized in one call, and the first-ever
        forward bootstraps that scale from the first routed expert's rows, as the loop does."""

        tokens, top_k = top_k_index.shape
        hidden = hidden_states.shape[-1]
        flat = top_k_index.reshape(-1)
        valid = (flat >= 0) & (flat < self.num_experts)  # expert-parallel padding sentinels take no part
        position = torch.nonzero(valid).squeeze(1)  # a host synchronisation, like the reference's expert list
        experts = flat[position]
        order = torch.argsort(experts, stable=True)
        position, experts = position[order], experts[order]
        token_index = torch.div(position, top_k, rounding_mode="floor")
        k_position = position - token_index * top_k
        offs = torch.cumsum(torch.bincount(experts, minlength=self.num_experts), 0, dtype=torch.int32)

        gate, up = _GroupedExpertFakeQuantLinear.apply(hidden_states[token_index], self.gate_up_proj, gate_up_amax,
                                                       offs).chunk(2, dim=-1)
        intermediate = self.act_fn(gate) * up
        routed = intermediate.shape[0] > 0
        if quantize and routed and self._down_input_amax_static is None:
            first_rows = int(offs[offs > 0][0])  # the rows of the lowest routed expert come first
            self._down_input_amax_static = _native.tensor_amax(intermediate[:first_rows].detach())
        if tracking and routed:
            self._down_input_amax = self._grow(self._down_input_amax, intermediate)
        if quantize and routed:
            intermediate = fake_quantize_nvfp4_activation(intermediate, self._down_input_amax_static)
        expert_output = _GroupedExpertFakeQuantLinear.apply(intermediate, self.down_proj, down_amax, offs)
        expert_output = expert_output * top_k_weights[token_index, k_position, None]

        contributions = hidden_states.new_zeros((tokens * top_k, hidden))
        contributions = contributions.index_copy(0, position, expert_output.to(hidden_states.dtype))
        contributions = contributions.view(tokens, top_k, hidden)
        slots = torch.argsort(torch.where(valid.view(tokens, top_k), top_k_index, self.num_experts), dim=1,
                              stable=True)
        final_hidden_states = torch.zeros_like(hidden_states)
        for j in range(top_k):
            picked = contributions.gather(1, slots[:, j, None, None].expand(tokens, 1, hidden)).squeeze(1)
            final_hidden_states = final_hidden_states + picked
        return final_hidden_states

    @torch.no_grad()
    def merged_projection(self, expert: int, projection: str) -> torch.Tensor:
        """One 2-D expert latent in serving naming, for export."""

        if projection == "w2":
            return self.down_proj[expert]
        gate, up = self.gate_up_proj[expert].chunk(2, dim=0)
        if projection == "w1":
            return gate
        if projection == "w3":
            return up
        raise ValueError(f"Unknown expert projection {projection!r}; expected one of {EXPERT_PROJECTIONS}.")


LORA_LEAVES = ("gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B")


class NVFP4ExpertLoRA(_ExpertInputScales, nn.Module):
    """LoRA-QAD of fused routed experts (nvfp4_experts.py:65-366): the fused base weights stay
    frozen (BF16, or block-FP8 codes dequantized per expert by ``qatf_fp8_block_dequant``) and
    every expert's merged weight ``base + scaling * B @ A`` is NVFP4 fake-quantized inside its own
    matmul (tensor amax of the merged weight, on the device), so gradients reach only the
    adapters.  ``hybrid_shared`` shares the gate/up ``A`` and the down ``B`` factors across
    experts.  The same module serves as its own teacher inside ``shared_base_teacher()`` (base
    weights, no adapters, no quantization, no statistics).  Each expert's forward is
    recomputed in its backward (``expert_checkpointing``) so the merged, quantized weights of all
    experts are never alive at once."""

    _is_nvfp4_expert_lora = True

    def __init__(self, source: nn.Module, rank: int, alpha: float, *, hybrid_shared: bool = True,
                 compute_dtype: torch.dtype = torch.bfloat16, expert_checkpointing: bool = True):
        super().__init__()
        if rank <= 0:
            raise ValueError(f"LoRA rank must be positive, got {rank}.")
        shapes = fused_experts_shapes(source)
        if shapes is None:
            raise ValueError(f"{type(source).__name__} does not expose fused 3D gate_up_proj / down_proj experts.")
        if getattr(source, "has_bias", False) or getattr(source, "is_transposed", False):
            raise ValueError("NVFP4 expert LoRA supports only non-transposed, bias-free expert weights.")
        self.num_experts, self.hidden_dim, self.intermediate_dim = shapes
        fp8 = fp8_experts_state(source)
        self.gate_up_proj = nn.Parameter(source.gate_up_proj.detach(), requires_grad=False)
        self.down_proj = nn.Parameter(source.down_proj.detach(), requires_grad=False)
        for name in ("gate_up_proj_scale_inv", "down_proj_scale_inv"):
            self.register_buffer(name, fp8[name].detach().float() if fp8 else None, persistent=False)
        self.act_fn = getattr(source, "act_fn", F.silu)
        self._compute_dtype = compute_dtype
        self.expert_checkpointing = bool(expert_checkpointing)
        self.rank = int(rank)
        self.lora_alpha = float(alpha)
        self.lora_scaling = self.lora_alpha / self.rank
        self.hybrid_shared = bool(hybrid_shared)

        E, H, I, r = self.num_experts, self.hidden_dim, self.intermediate_dim, self.rank
        kw = dict(device=self.gate_up_proj.device, dtype=compute_dtype)
        self.gate_up_lora_A = nn.Parameter(torch.empty((2, r, H) if self.hybrid_shared else (E, 2, r, H), **kw))
        self.gate_up_lora_B = nn.Parameter(torch.zeros(E, 2, I, r, **kw))
        self.down_lora_A = nn.Parameter(torch.empty(E, r, I, **kw))
        self.down_lora_B = nn.Parameter(torch.zeros((H, r) if self.hybrid_shared else (E, H, r), **kw))
        self.reset_lora_parameters()
        self._init_input_scales()

    def reset_lora_parameters(self) -> None:
        """Kaiming-uniform ``A`` slices (each ``[rank, in]`` matrix on its own, in the
        reference's order, so a seeded run draws the same values) and zero ``B``: the merged
        weight starts as the base (nvfp4_experts.py:189-195)."""

        for a, width in ((self.gate_up_lora_A, self.hidden_dim), (self.down_lora_A, self.intermediate_dim)):
            for matrix in a.reshape(-1, self.rank, width):
                nn.init.kaiming_uniform_(matrix, a=math.sqrt(5))
        nn.init.zeros_(self.gate_up_lora_B)
        nn.init.zeros_(self.down_lora_B)

    @property
    def is_fp8_base(self) -> bool:
        return self.gate_up_proj_scale_inv is not None

    def trainable_parameter_names(self, prefix: str) -> set[str]:
        return {f"{prefix}.{leaf}" for leaf in LORA_LEAVES}

    def _base(self, weight: torch.Tensor, scale_inv: torch.Tensor | None, expert) -> torch.Tensor:
        if scale_inv is None:
            return weight[expert]
        return dequantize_fp8_blocks(weight[expert], scale_inv[expert], self._compute_dtype)

    def base_gate_up(self, expert) -> torch.Tensor:
        return self._base(self.gate_up_proj, self.gate_up_proj_scale_inv, expert)

    def base_down(self, expert) -> torch.Tensor:
        return self._base(self.down_proj, self.down_proj_scale_inv, expert)

    def effective_gate_up(self, expert) -> torch.Tensor:
        """Merged ``[2 * intermediate, hidden]`` weight of one expert (w1 rows over w3 rows)."""

        base = self.base_gate_up(expert)
        a = self.gate_up_lora_A if self.hybrid_shared else self.gate_up_lora_A[expert]
        delta = torch.matmul(self.gate_up_lora_B[expert], a) * self.lora_scaling  # [2, I, H]
        return base + delta.reshape_as(base).to(base.dtype)

    def effective_down(self, expert) -> torch.Tensor:
        base = self.base_down(expert)
        b = self.down_lora_B if self.hybrid_shared else self.down_lora_B[expert]
        delta = torch.matmul(b, self.down_lora_A[expert]) * self.lora_scaling  # [H, I]
        return base + delta.to(base.dtype)

    def _gate(self, gate_up: torch.Tensor) -> torch.Tensor:
        gate, up = gate_up.chunk(2, dim=-1)
        return self.act_fn(gate) * up

    def _quantize_input(self, value: torch.Tensor, static: torch.Tensor | None) -> torch.Tensor:
        # the static scale changes only between optimizer steps: a recompute sees the same one
        if not self._quantize_activations or static is None:
            return value
        return fake_quantize_nvfp4_activation(value, static)

    def _teacher_expert(self, tokens: torch.Tensor, expert: int) -> torch.Tensor:
        return F.linear(self._gate(F.linear(tokens, self.base_gate_up(expert))), self.base_down(expert))

    def _student_expert(self, tokens: torch.Tensor, expert: int) -> torch.Tensor:
        # w1 and w3 are quantized as one tensor, so they share one NVFP4 tensor scale as served
        gated = self._gate(F.linear(self._quantize_input(tokens, self._gate_up_input_amax_static),
                                    fake_quantize_nvfp4(self.effective_gate_up(expert))))
        if self._track_input_amax and self.training:
            with torch.no_grad():  # a running maximum: a recompute of this expert changes nothing
                self._down_input_amax = self._grow(self._down_input_amax, gated)
        return F.linear(self._quantize_input(gated, self._down_input_amax_static),
                        fake_quantize_nvfp4(self.effective_down(expert)))

    def _routing(self, top_k_index: torch.Tensor):
        """Per expert, the (top-k slot, token) pairs routed to it: one device-side sort and one
        host transfer of the per-expert counts for the whole layer."""

        tokens, top_k = top_k_index.shape
        flat = top_k_index.reshape(-1)
        # rows ordered by (expert, top-k slot, token)
        slot = torch.arange(top_k, device=flat.device).repeat(tokens)
        token = torch.arange(tokens, device=flat.device).repeat_interleave(top_k)
        order = torch.argsort((flat * top_k + slot) * tokens + token)
        counts = torch.bincount(flat, minlength=self.num_experts).tolist()
        return slot[order], token[order], counts

    @torch.no_grad()
    def _bootstrap_input_scales(self, hidden_states, slots, tokens, counts) -> None:
        """Both static W4A4 scales from the first batch: the block input's maximum, and the
        maximum of every active expert's gated intermediate on the base weights (one extra pass,
        once), all-reduced so every rank starts from the same scales (nvfp4_experts.py:280-306)."""

        gate_up_max = _native.tensor_amax(hidden_states.detach())
        down_max = torch.zeros((), dtype=torch.float32, device=hidden_states.device)
        start = 0
        for expert, count in enumerate(counts):
            if count:
                rows = tokens[start:start + count]
                start += count
                gated = self._gate(F.linear(hidden_states[rows], self.base_gate_up(expert)))
                down_max = torch.maximum(down_max, _native.tensor_amax(gated))
        if dist.is_initialized():
            both = torch.stack([gate_up_max, down_max])
            dist.all_reduce(both, op=dist.ReduceOp.MAX)
            gate_up_max, down_max = both.unbind()
        self._gate_up_input_amax_static = gate_up_max.clone()
        self._down_input_amax_static = down_max.clone()

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor) -> torch.Tensor:
        teacher = shared_base_teacher_enabled()
        expert_fn = self._teacher_expert if teacher else self._student_expert
        recompute = self.expert_checkpointing and not teacher and torch.is_grad_enabled()
        with torch.no_grad():
            slots, tokens, counts = self._routing(top_k_index)
            if not teacher and self._track_input_amax:
                if self._quantize_activations and self._gate_up_input_amax_static is None:
                    self._bootstrap_input_scales(hidden_states, slots, tokens, counts)
                self._gate_up_input_amax = self._grow(self._gate_up_input_amax, hidden_states)
        final_hidden_states = torch.zeros_like(hidden_states)
        start = 0
        for expert, count in enumerate(counts):
            if not count:
                continue
            slot, token = slots[start:start + count], tokens[start:start + count]
            start += count
            rows = hidden_states[token]
            if recompute:
                out = torch.utils.checkpoint.checkpoint(expert_fn, rows, expert, use_reentrant=False)
            else:
                out = expert_fn(rows, expert)
            out = out * top_k_weights[token, slot, None]
            final_hidden_states.index_add_(0, token, out.to(final_hidden_states.dtype))
        return final_hidden_states

    @torch.no_grad()
    def merged_projection(self, expert: int, projection: str) -> torch.Tensor:
        """One merged 2-D expert projection in serving naming, for export."""

        if projection == "w2":
            return self.effective_down(expert)
        gate, up = self.effective_gate_up(expert).chunk(2, dim=0)
        if projection == "w1":
            return gate
        if projection == "w3":
            return up
        raise ValueError(f"Unknown expert projection {projection!r}; expected one of {EXPERT_PROJECTIONS}.")
