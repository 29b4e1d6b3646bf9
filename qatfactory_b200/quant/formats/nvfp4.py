"""NVFP4 fake quantization on B200: the ``qatfactory.quant`` NVFP4 API over libqatf.so.

Same public names, arguments, results and errors as the reference module
(qatfactory/quant/formats/nvfp4.py), with every tensor computation done by the sm_100a
kernels: block-16 E2M1 codes with E4M3 block scales and an FP32 tensor scale
(tensor amax / 2688), round-to-nearest-even ties, the masked straight-through estimator
and the fused-family / W4A4 static-scale lifecycle.  CUDA tensors only; meta tensors pass
through as in the reference.

The STE mask is kept as one bit per element (the reference keeps an int8 then a bool
tensor); the backward expands it inside the kernel, with identical gradients.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from ... import _native
from .fp8_base import dequantize_fp8_blocks, fp8_linear_state
from .lora import LoRAMixin, shared_base_teacher_enabled

NVFP4_BLOCK_SIZE = 16
NVFP4_MAX_VALUE = 6.0
E4M3_MAX_VALUE = 448.0
E4M3_MIN_SUBNORMAL = 2**-9
NVFP4_SCALE_DENOMINATOR = NVFP4_MAX_VALUE * E4M3_MAX_VALUE


class _MaskedStraightThrough(torch.autograd.Function):
    """Forward returns the quantized tensor; backward is ``grad * in_range``
    (nvfp4.py:32-41) with ``in_range`` held as a bit mask."""

    @staticmethod
    def forward(ctx, latent: torch.Tensor, quantized: torch.Tensor, mask_bits: torch.Tensor | None):
        ctx.all_true = mask_bits is None
        if mask_bits is not None:
            ctx.save_for_backward(mask_bits)
        ctx.latent_shape = latent.shape
        return quantized

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        if ctx.all_true:
            return grad_output, None, None
        (mask_bits,) = ctx.saved_tensors
        grad = _native.ste_backward(grad_output.contiguous(), mask_bits)
        return grad.reshape(ctx.latent_shape), None, None


def pack_e2m1_rows(indices: torch.Tensor) -> torch.Tensor:
    """Pack E2M1 nibbles with even columns in the low nibble (nvfp4.py:76-85)."""

    if indices.ndim != 2:
        raise ValueError(f"E2M1 packing expects a 2D tensor, got shape {tuple(indices.shape)}.")
    if indices.shape[-1] % 2:
        raise ValueError("E2M1 packing requires an even final dimension.")
    return _native.e2m1_pack_rows(indices.to(torch.uint8))


def unpack_e2m1_rows(packed: torch.Tensor) -> torch.Tensor:
    """Unpack bytes into canonical E2M1 nibbles (nvfp4.py:88-101)."""

    if packed.ndim != 2 or packed.dtype != torch.uint8:
        raise ValueError(f"Packed E2M1 weights must be 2D uint8, got {packed.dtype} {tuple(packed.shape)}.")
    return _native.e2m1_unpack_rows(packed)


def dequantize_nvfp4(
    packed_weight: torch.Tensor,
    weight_scale: torch.Tensor,
    weight_scale_2: torch.Tensor,
) -> torch.Tensor:
    """Dequantize packed NVFP4 tensors to FP32 (nvfp4.py:104-121)."""

    if packed_weight.ndim != 2 or packed_weight.dtype != torch.uint8:
        raise ValueError(f"Packed E2M1 weights must be 2D uint8, got {packed_weight.dtype} {tuple(packed_weight.shape)}.")
    if packed_weight.shape[-1] * 2 != weight_scale.shape[-1] * NVFP4_BLOCK_SIZE:
        raise ValueError(
            f"NVFP4 scale shape {tuple(weight_scale.shape)} is incompatible with "
            f"weight shape {tuple(packed_weight.shape)}."
        )
    return _native.nvfp4_dequant(packed_weight, weight_scale.view(torch.uint8), weight_scale_2)


@dataclass(frozen=True)
class NVFP4QuantizationResult:
    packed_weight: torch.Tensor
    weight_scale: torch.Tensor
    weight_scale_2: torch.Tensor
    reconstruction: torch.Tensor | None


@dataclass
class NVFP4AmaxGroup:
    """One fused family (QKV, gate/up, ...) sharing a tensor scale (nvfp4.py:134-147)."""

    member_names: tuple[str, ...]
    members: tuple["NVFP4Linear", ...]
    tensor_amax_value: torch.Tensor | None = None

    def tensor_amax(self) -> torch.Tensor:
        if self.tensor_amax_value is not None:
            return self.tensor_amax_value
        if any(hasattr(module.weight, "to_local") for module in self.members):
            raise RuntimeError("Fused NVFP4 weight amax must be refreshed after FSDP parallelization.")
        maxima = [_native.tensor_amax(module._effective_weight().detach()) for module in self.members]
        return torch.stack(maxima).amax()


def build_nvfp4_fused_family_names(module_names: list[str]) -> list[tuple[str, ...]]:
    """Group projections as the serving runtime fuses them (nvfp4.py:150-185)."""

    present_names = set(module_names)
    assigned: set[str] = set()
    families: list[tuple[str, ...]] = []
    for name in module_names:
        if name in assigned:
            continue
        parent, _, leaf = name.rpartition(".")
        partial_ok = False
        if leaf in {"q_proj", "k_proj", "v_proj"} and parent.endswith("self_attn"):
            siblings = ("q_proj", "k_proj", "v_proj")
            partial_ok = True  # Gemma-style layers without v_proj fuse the present subset
        elif leaf in {"gate_proj", "up_proj"} and (parent.endswith("mlp") or parent.endswith("shared_expert")):
            siblings = ("gate_proj", "up_proj")
        elif leaf in {"in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a"} and parent.endswith("linear_attn"):
            siblings = ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")
        else:
            siblings = None
        if siblings is None:
            family = (name,)
        else:
            candidates = tuple(f"{parent}.{s}" for s in siblings)
            family = tuple(c for c in candidates if c in present_names)
            if not partial_ok and len(family) < len(candidates):
                raise ValueError(f"Incomplete fused NVFP4 family for {name!r}: {family}.")
            family = family or (name,)
        families.append(family)
        assigned.update(family)
    if assigned != present_names:
        raise ValueError(f"Failed to assign NVFP4 modules to fused families: {sorted(present_names - assigned)}.")
    return families


def attach_nvfp4_amax_groups(model: nn.Module) -> list[NVFP4AmaxGroup]:
    by_name = {name: m for name, m in model.named_modules() if isinstance(m, NVFP4Linear)}
    groups = []
    for names in build_nvfp4_fused_family_names(list(by_name)):
        group = NVFP4AmaxGroup(names, tuple(by_name[n] for n in names))
        for module in group.members:
            module._amax_group = group
            module._track_input_amax = True
        groups.append(group)
    model._nvfp4_amax_groups = groups
    return groups


def _nvfp4_amax_groups(model: nn.Module) -> list[NVFP4AmaxGroup]:
    groups = getattr(model, "_nvfp4_amax_groups", None)
    if groups is None:
        raise RuntimeError("NVFP4 fused amax groups have not been attached to the model.")
    return groups


def _local_weight(module: "NVFP4Linear") -> torch.Tensor:
    """Local shard of the trainable weight: the FP32 latent master when the module gathers its
    weight quantized (``quant.quantized_gather``), else the weight parameter."""

    weight = module.__dict__.get("_latent_shard", module.weight)
    return weight.to_local() if hasattr(weight, "to_local") else weight


def _merged_local_weight(module: "NVFP4Linear") -> torch.Tensor:
    """Local FSDP shard of the (LoRA-merged) weight the forward quantizes (nvfp4.py:214-256)."""

    weight = module.weight
    if getattr(module, "_fp8_scale_inv", None) is not None:
        # the 128-row scale blocks of an FP8 base need not align with a row shard: dequantize
        # the gathered (frozen) codes, as the reference does (nvfp4.py:228-237)
        full = weight.full_tensor() if hasattr(weight, "full_tensor") else weight
        base = dequantize_fp8_blocks(full, module._fp8_scale_inv, module._compute_dtype)
        if getattr(module, "lora_A", None) is None:
            return base
        a = module.lora_A.full_tensor() if hasattr(module.lora_A, "full_tensor") else module.lora_A
        b = module.lora_B.full_tensor() if hasattr(module.lora_B, "full_tensor") else module.lora_B
        return base + (module.lora_scaling * (b @ a)).to(base.dtype)
    if getattr(module, "lora_A", None) is None:
        return _local_weight(module)
    scaling = module.lora_scaling
    if not hasattr(weight, "to_local"):
        return weight + (scaling * (module.lora_B @ module.lora_A)).to(weight.dtype)
    w_local = weight.to_local()
    a_full = module.lora_A.full_tensor() if hasattr(module.lora_A, "full_tensor") else module.lora_A
    b_local = module.lora_B.to_local() if hasattr(module.lora_B, "to_local") else module.lora_B
    if b_local.shape[0] != w_local.shape[0]:
        raise RuntimeError("LoRA B shard rows do not align with the weight shard")
    return w_local + (scaling * (b_local @ a_full)).to(w_local.dtype)


def _bf16_amax(weight: torch.Tensor) -> torch.Tensor:
    """``weight.to(bfloat16).abs().amax().float()`` without materialising the cast.

    Round-to-nearest-even is monotonic and odd, so max |bf16(x)| == bf16(max |x|)."""

    amax = _native.tensor_amax(weight.detach())
    return amax if weight.dtype == torch.bfloat16 else amax.to(torch.bfloat16).float()


@torch.no_grad()
def refresh_nvfp4_weight_amax(model: nn.Module, process_group=None) -> None:
    """Refresh globally reduced fused-family maxima from local FSDP shards (nvfp4.py:259-282).

    One all-reduce(MAX) of the ``[n_families]`` FP32 vector, issued in the same order on
    every rank."""

    groups = _nvfp4_amax_groups(model)
    if not groups:
        return
    local = []
    for group in groups:
        maxima = [_bf16_amax(_merged_local_weight(m)) for m in group.members]
        local.append(torch.stack(maxima).amax())
    reduced = torch.stack(local)
    if dist.is_initialized():
        dist.all_reduce(reduced, op=dist.ReduceOp.MAX, group=process_group)
    for group, value in zip(groups, reduced.unbind()):
        group.tensor_amax_value = value


@torch.no_grad()
def finalize_nvfp4_input_scales(model: nn.Module, process_group=None) -> dict[str, torch.Tensor]:
    """Reduce running training-input maxima into fused-family input scales (nvfp4.py:285-319)."""

    input_scales: dict[str, torch.Tensor] = {}
    for name, module in model.named_modules():  # routed experts first, in module order (nvfp4.py:290-292)
        if getattr(module, "_is_nvfp4_experts", False):
            input_scales.update(module.finalize_input_scales(name, process_group))
    groups = _nvfp4_amax_groups(model)
    if not groups:
        return input_scales
    local = []
    for group in groups:
        missing = [n for n, m in zip(group.member_names, group.members) if m._input_amax is None]
        if missing:
            raise RuntimeError(f"Missing training input-amax observations for {missing}.")
        local.append(torch.stack([m._input_amax for m in group.members]).amax())
    reduced = torch.stack(local).to(_local_weight(groups[0].members[0]).device)
    if dist.is_initialized():
        dist.all_reduce(reduced, op=dist.ReduceOp.MAX, group=process_group)
    for group, maximum in zip(groups, reduced.unbind()):
        if not bool(torch.isfinite(maximum)) or not bool(maximum > 0):
            raise RuntimeError(f"Invalid training input amax for fused family {group.member_names}.")
        for name, module in zip(group.member_names, group.members):
            module._input_amax = maximum.clone()
            input_scales[f"{name}.input_scale"] = (maximum / NVFP4_SCALE_DENOMINATOR).reshape(())
    return input_scales


def nvfp4_runtime_state_dict(model: nn.Module) -> dict:
    modules = {
        name: m._input_amax.detach().cpu()
        for name, m in model.named_modules()
        if isinstance(m, NVFP4Linear) and m._track_input_amax and m._input_amax is not None
    }
    experts = {}
    for name, m in model.named_modules():
        if getattr(m, "_is_nvfp4_experts", False):
            state = m.runtime_state_dict()
            if state:
                experts[name] = state
    return {"version": 1, "modules": modules, "experts": experts}


def load_nvfp4_runtime_state_dict(model: nn.Module, state_dict: dict) -> None:
    if state_dict.get("version") != 1:
        raise ValueError("Unsupported NVFP4 QAD runtime-state version.")
    saved = state_dict.get("modules", {})
    expected = {n: m for n, m in model.named_modules() if isinstance(m, NVFP4Linear) and m._track_input_amax}
    if set(saved) != set(expected):
        missing = sorted(set(expected) - set(saved))
        extra = sorted(set(saved) - set(expected))
        raise RuntimeError(f"NVFP4 runtime-state module mismatch; missing={missing[:5]}, extra={extra[:5]}.")
    for name, module in expected.items():
        module._input_amax = saved[name].to(_local_weight(module).device).reshape(())
        module._input_amax_static = module._input_amax.clone()
    saved_experts = state_dict.get("experts", {})
    for name, module in model.named_modules():
        if getattr(module, "_is_nvfp4_experts", False) and name in saved_experts:
            module.load_runtime_state_dict(saved_experts[name], module.gate_up_proj.device)


@torch.no_grad()
def commit_nvfp4_input_scales(model: nn.Module, process_group=None) -> None:
    """Publish running input maxima as the step-static W4A4 scales (nvfp4.py:361-397)."""

    for module in model.modules():
        if getattr(module, "_is_nvfp4_experts", False):
            module.commit_input_scales(process_group)
    modules = [
        m
        for m in model.modules()
        if isinstance(m, NVFP4Linear) and getattr(m, "_quantize_activations", False) and m._input_amax is not None
    ]
    if not modules:
        return
    maxima = torch.stack([m._input_amax for m in modules]).to(_local_weight(modules[0]).device)
    if dist.is_initialized():
        dist.all_reduce(maxima, op=dist.ReduceOp.MAX, group=process_group)
    for module, maximum in zip(modules, maxima.unbind()):
        module._input_amax = maximum.clone()
        module._input_amax_static = maximum.clone()


def _amax_tensor(weight: torch.Tensor, tensor_amax: torch.Tensor | None) -> torch.Tensor:
    if tensor_amax is None:
        return _native.tensor_amax(weight.detach())
    return tensor_amax.detach().to(device=weight.device, dtype=torch.float32).reshape(())


@torch.no_grad()
def quantize_nvfp4(
    weight: torch.Tensor,
    *,
    tensor_amax: torch.Tensor | None = None,
    compute_reconstruction: bool = True,
) -> NVFP4QuantizationResult:
    """Pack a 2D weight on the max-based NVFP4 lattice (nvfp4.py:400-462)."""

    if weight.ndim != 2:
        raise ValueError(f"NVFP4 packing expects a 2D weight, got shape {tuple(weight.shape)}.")
    if weight.shape[-1] % NVFP4_BLOCK_SIZE:
        raise ValueError(
            f"NVFP4 packing requires in_features divisible by {NVFP4_BLOCK_SIZE}, got {weight.shape[-1]}."
        )
    if weight.is_meta:
        raise ValueError("Cannot pack an NVFP4 lattice from a meta tensor.")
    if tensor_amax is not None and tensor_amax.numel() != 1:
        raise ValueError("NVFP4 tensor_amax must be one finite non-negative value.")
    amax = _amax_tensor(weight, tensor_amax)
    # the reference validates the scalar on the host (nvfp4.py:425-426); packing is not on
    # the per-step path, so the synchronisation is acceptable here as it is there
    value = float(amax)
    if not (value == value) or value < 0 or value == float("inf"):
        raise ValueError("NVFP4 tensor_amax must be one finite non-negative value.")
    packed, scales, scale_2, recon = _native.nvfp4_pack(weight, amax, recon=compute_reconstruction)
    return NVFP4QuantizationResult(
        packed_weight=packed,
        weight_scale=scales.view(torch.float8_e4m3fn),
        weight_scale_2=scale_2,
        reconstruction=recon,
    )


def fake_quantize_nvfp4(
    weight: torch.Tensor,
    block_size: int = NVFP4_BLOCK_SIZE,
    *,
    tensor_amax: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fake-quantize a linear weight with NVFP4 E2M1 values and E4M3 block scales
    (nvfp4.py:504-550).  The host never reads the amax: a zero tensor amax is handled in
    the kernel, so the call does not synchronise the device."""

    if block_size != NVFP4_BLOCK_SIZE:
        raise ValueError(f"NVFP4 requires block_size={NVFP4_BLOCK_SIZE}, got {block_size}.")
    if weight.ndim != 2:
        raise ValueError(f"NVFP4Linear expects a 2D weight, got shape {tuple(weight.shape)}.")
    if weight.is_meta:
        return weight
    grad = torch.is_grad_enabled() and weight.requires_grad  # else no STE mask and no autograd node
    with torch.no_grad():
        if tensor_amax is None and weight.is_contiguous():
            quantized, mask, _ = _native.nvfp4_fake_quant(weight.detach(), want_mask=grad)
        else:
            quantized, mask = _native.nvfp4_qdq(weight.detach(), _amax_tensor(weight, tensor_amax), want_mask=grad)
    return _MaskedStraightThrough.apply(weight, quantized, mask) if grad else quantized


def fake_quantize_nvfp4_activation(activation: torch.Tensor, input_amax: torch.Tensor) -> torch.Tensor:
    """NVFP4 activation fake quant with a static tensor scale (nvfp4.py:553-569)."""

    if activation.is_meta:
        return activation
    shape = activation.shape
    quantized = fake_quantize_nvfp4(activation.reshape(-1, shape[-1]), tensor_amax=input_amax.detach())
    return quantized.reshape(shape)


def _round_up(value: int, multiple: int) -> int:
    return (value + multiple - 1) // multiple * multiple


def _pad2d(t: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """``t`` zero-padded at the end to [rows, cols]; ``t`` itself when it has that shape."""

    if t.shape[0] == rows and t.shape[1] == cols:
        return t
    return F.pad(t, (0, cols - t.shape[1], 0, rows - t.shape[0]))


class _W4A4Linear(torch.autograd.Function):
    """``F.linear(fq_act(x), fq(w))`` of the W4A4 NVFP4 linear (nvfp4.py:636-658) on the tensor
    cores: one operand pass per input (codes, block scales, dequantized copy, STE mask), a
    block-scaled FP4 GEMM forward, and backward ``dX = STE_x(dY @ W_q)``,
    ``dW = STE_w(dY^T @ X_q)`` as BF16 GEMMs with the masks applied in their epilogues.

    Shapes off the GEMM tiles (token rows % 128, in or out features % 256) are zero-padded to
    them and the results sliced back.  Zero rows and columns change nothing that is kept: a
    padded block of 16 is all zeros (in features % 16 == 0, so no block mixes data and
    padding), its codes are 0, every product it meets is an exact 0, the running maximum and the
    given tensor amaxes are unchanged, and padded rows of dY are zero in the weight gradient's
    sum over tokens."""

    @staticmethod
    def forward(ctx, x2d, weight, input_amax, weight_amax, running_amax=None):
        rows, k = x2d.shape
        n = weight.shape[0]
        mp, kp, np_ = _round_up(rows, 128), _round_up(k, 256), _round_up(n, 256)
        xs = _pad2d(x2d.detach(), mp, kp)
        ws = _pad2d(weight.detach(), np_, kp)
        cx, sx, xq, mx = _native.nvfp4_operand(xs, input_amax, _native.OPERAND_A, running_amax=running_amax)
        cw, sw, wq, mw = _native.nvfp4_operand(ws, weight_amax, _native.OPERAND_B)
        y = _native.nvfp4_gemm(cx, sx, input_amax, cw, sw, weight_amax)
        ctx.save_for_backward(xq, mx, wq, mw)
        ctx.shape = (rows, k, n)
        # a sliced result is copied out: an output that is a view made inside a custom Function
        # cannot be modified in place by the caller
        return y if (mp, np_) == (rows, n) else y[:rows, :n].clone()

    @staticmethod
    def backward(ctx, grad_out):
        xq, mx, wq, mw = ctx.saved_tensors
        rows, k, n = ctx.shape
        dy = _pad2d(grad_out.contiguous().to(torch.bfloat16), xq.shape[0], wq.shape[0])
        gx = gw = None
        if ctx.needs_input_grad[0]:
            gx = _native.bf16_gemm(dy, _native.K_MAJOR, wq, _native.MN_MAJOR, mx)
            if gx.shape != (rows, k):
                gx = gx[:rows, :k]
        if ctx.needs_input_grad[1]:
            gw = _native.bf16_gemm(dy, _native.MN_MAJOR, xq, _native.MN_MAJOR, mw)
            if gw.shape != (n, k):
                gw = gw[:n, :k]
        return gx, gw, None, None, None


def w4a4_linear(input: torch.Tensor, weight: torch.Tensor, input_amax: torch.Tensor, weight_amax: torch.Tensor,
                bias: torch.Tensor | None = None, running_amax: torch.Tensor | None = None) -> torch.Tensor:
    """W4A4 NVFP4 linear: the tensor-core path for BF16 CUDA inputs with in features % 16 == 0
    (padded to the GEMM tiles where needed), otherwise fake-quantized operands through
    ``F.linear`` (the reference's own formulation).  ``running_amax`` (FP32 scalar tensor), when
    given, is raised in place to max |input|."""

    rows = input.numel() // input.shape[-1] if input.shape[-1] else 0
    if (input.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and input.is_cuda and rows > 0
            and weight.shape[0] > 0 and weight.shape[1] % 16 == 0):
        y = _W4A4Linear.apply(input.reshape(rows, input.shape[-1]), weight, input_amax.detach(), weight_amax.detach(),
                              running_amax)
        y = y.reshape(*input.shape[:-1], weight.shape[0])
        return y if bias is None else y + bias
    if running_amax is not None:
        _native.tensor_amax_update(input.detach(), running_amax)
    quantized = fake_quantize_nvfp4_activation(input, input_amax)
    return F.linear(quantized, fake_quantize_nvfp4(weight, tensor_amax=weight_amax), bias)


class NVFP4Linear(LoRAMixin, nn.Linear):
    """Linear layer whose weight (and, for W4A4, input) is NVFP4 fake-quantized on every
    forward (nvfp4.py:572-658).  State-dict keys stay ``{weight, bias}``."""

    _compute_dtype: torch.dtype = torch.bfloat16

    @classmethod
    def _empty_like(cls, module: nn.Module, in_features: int, out_features: int) -> "NVFP4Linear":
        converted = cls(in_features, out_features, bias=module.bias is not None, device="meta")
        converted.bias = module.bias
        converted.register_buffer("_fp8_scale_inv", None, persistent=False)
        converted._amax_group = None
        converted._track_input_amax = False
        converted._input_amax = None
        converted._input_amax_static = None
        converted._quantize_activations = False
        return converted

    @classmethod
    def from_linear(cls, module: nn.Linear) -> "NVFP4Linear":
        converted = cls._empty_like(module, module.in_features, module.out_features)
        converted.weight = module.weight
        return converted

    @classmethod
    def from_fp8_linear(cls, module: nn.Module, compute_dtype: torch.dtype = torch.bfloat16) -> "NVFP4Linear":
        """Wrap a block-scaled FP8 linear, its FP8 codes kept as the frozen (LoRA) base and
        dequantized per forward (nvfp4.py:610-627)."""

        state = fp8_linear_state(module)
        if state is None:
            raise ValueError(f"{type(module).__name__} is not a block-scaled FP8 linear.")
        weight, scale_inv = state
        out_features, in_features = weight.shape
        converted = cls._empty_like(module, in_features, out_features)
        converted.weight = nn.Parameter(weight.detach(), requires_grad=False)
        converted._fp8_scale_inv = scale_inv.detach().float()
        converted._compute_dtype = compute_dtype
        return converted

    def base_weight(self) -> torch.Tensor:
        if getattr(self, "_fp8_scale_inv", None) is None:
            return self.weight
        return dequantize_fp8_blocks(self.weight, self._fp8_scale_inv, self._compute_dtype)

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if shared_base_teacher_enabled():
            return F.linear(input, self.base_weight(), self.bias)
        if self._quantize_activations:
            running = None
            if self._input_amax_static is None:
                # bootstrap: all-reduced once per module, in the same first forward on every rank
                current = _native.tensor_amax(input.detach())
                if dist.is_initialized():
                    dist.all_reduce(current, op=dist.ReduceOp.MAX)
                self._input_amax_static = current.clone()
                if self._track_input_amax and self.training:
                    self._input_amax = current if self._input_amax is None else torch.maximum(self._input_amax,
                                                                                                current)
            elif self._track_input_amax and self.training:
                # the running maximum is raised by the activation's operand pass itself
                running = self._running_input_amax(input.device)
            weight = self._effective_weight()
            tensor_amax = self._amax_group.tensor_amax() if self._amax_group is not None else None
            if tensor_amax is None:
                tensor_amax = _native.tensor_amax(weight.detach())
            return w4a4_linear(input, weight, self._input_amax_static, tensor_amax, self.bias, running_amax=running)
        elif self._track_input_amax and self.training:
            self._observe_input_amax(input)
        if self.__dict__.get("_prequantized", False):
            # the weight was quantized shard by shard before FSDP2 gathered it
            return F.linear(input, self.weight, self.bias)
        tensor_amax = self._amax_group.tensor_amax() if self._amax_group is not None else None
        return F.linear(input, fake_quantize_nvfp4(self._effective_weight(), tensor_amax=tensor_amax), self.bias)

    def _running_input_amax(self, device: torch.device) -> torch.Tensor:
        """The module's own running-maximum tensor, updated in place by the kernels (+0 before
        the first observation, so the first update leaves max |input|).  A tensor assigned from
        elsewhere (a loaded state, a finalized value) is copied first and never mutated."""

        running = self._input_amax
        if running is not None and running is self.__dict__.get("_input_amax_own"):
            return running
        if running is None:
            running = torch.zeros((), dtype=torch.float32, device=device)
        else:
            running = running.detach().to(device=device, dtype=torch.float32).reshape(()).clone()
        self._input_amax = self.__dict__["_input_amax_own"] = running
        return running

    def _observe_input_amax(self, input: torch.Tensor) -> None:
        """Running maximum of |input| (nvfp4.py:654-656) in one launch."""

        _native.tensor_amax_update(input.detach(), self._running_input_amax(input.device))
