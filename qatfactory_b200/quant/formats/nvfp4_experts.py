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
loop over experts; W4A4 keeps the loop.  The LoRA variant ``NVFP4ExpertLoRA`` (frozen, possibly block-FP8 base with low-rank
adapters) is not part of this package.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from ... import _native
from .nvfp4 import NVFP4_BLOCK_SIZE, NVFP4_SCALE_DENOMINATOR, _MaskedStraightThrough, fake_quantize_nvfp4_activation

__all__ = ["fake_quantize_nvfp4_experts", "is_fused_experts", "fused_experts_shapes", "NVFP4Experts"]

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


class NVFP4Experts(nn.Module):
    """Full-parameter NVFP4 QAD of fused routed experts (nvfp4_experts.py:496-649): a drop-in
    for a transformers fused experts module (``forward(hidden_states, top_k_index,
    top_k_weights)`` over ``gate_up_proj`` ``[E, 2 * intermediate, hidden]`` and ``down_proj``
    ``[E, hidden, intermediate]``).  Both 3-D latents train; every routed expert is
    fake-quantized inside its own matmul with its own tensor amax (the whole ``gate_up_proj[e]``
    slice shares one, so w1 and w3 export one global scale).  W4A4 quantizes the block input
    with one static scale for all experts (w13) and the expert intermediates with another
    (w2), with the same step-static lifecycle as the reference."""

    _is_nvfp4_experts = True
    # the two activation scales a serving fused-MoE layer carries, in export order
    INPUT_SCALE_GROUPS = (("w13", "_gate_up_input_amax"), ("w2", "_down_input_amax"))

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
        self._track_input_amax = False
        self._quantize_activations = False
        self._gate_up_input_amax = None
        self._gate_up_input_amax_static = None
        self._down_input_amax = None
        self._down_input_amax_static = None

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

    def target_names(self, prefix: str) -> list[str]:
        """Per-expert projection names in serving (w1 / w3 / w2) naming."""

        return [f"{prefix}.{e}.{p}" for e in range(self.num_experts) for p in EXPERT_PROJECTIONS]

    def trainable_parameter_names(self, prefix: str) -> set[str]:
        return {f"{prefix}.gate_up_proj", f"{prefix}.down_proj"}

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
        if not quantize and grouped_experts_supported(hidden_states, self.gate_up_proj, self.down_proj):
            return self._forward_grouped(hidden_states, top_k_index, top_k_weights, gate_up_amax, down_amax, tracking)
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

    def _forward_grouped(self, hidden_states, top_k_index, top_k_weights, gate_up_amax, down_amax, tracking):
        """W4A16 forward of every routed expert as two grouped GEMMs (``torch._grouped_mm``)
        instead of a loop over experts: the same products, and the same sum as the reference
        (each token's expert outputs added in ascending expert order in the dtype of
        ``hidden_states``, as its one ``index_add_`` per expert does)."""

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
        if tracking:
            self._down_input_amax = self._grow(self._down_input_amax, intermediate)
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
