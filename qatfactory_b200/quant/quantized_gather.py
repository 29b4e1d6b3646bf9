"""Quantize-before-gather for FSDP2 training of NVFP4 W4A16 linears.

The reference fake-quantizes every ``NVFP4Linear`` weight after FSDP2 has gathered it and cast
it to BF16: in every forward, again in every activation-checkpoint recompute, and on every rank
for the whole weight (``F.linear(input, fake_quantize_nvfp4(self._effective_weight(), ...))``,
qatfactory/quant/formats/nvfp4.py:657-658).  An NVFP4 block is 16 consecutive elements of one
row and FSDP2 shards rows, so the quantized weight is the concatenation of the quantized row
shards (the reference relies on the same alignment for its shard-local amax, nvfp4.py:214-256).
Here each rank quantizes its own FP32 latent shard once per optimizer step, after the
fused-family amax refresh, and FSDP2 gathers the already-quantized weight:

* ``module.weight``: the FSDP2 parameter, holding ``fq(bf16(latent))`` widened to FP32
  (exact, so FSDP2's BF16 cast for the all-gather is lossless); the forward is ``F.linear`` on
  the gathered weight, with no quantizer in the forward or the recompute;
* ``module._latent_shard``: the FP32 latent master with the same sharding (a DTensor under
  FSDP2), the parameter the optimizer steps; the amax refresh reads it;
* ``module._shadow_mask``: the STE mask bits of the local shard.

The results are the reference's, bit for bit (finite weights).  The forward sees the same BF16
weight.  The reference multiplies the gathered BF16 weight gradient by the mask before FSDP2's
FP32 reduce-scatter; this module masks the reduced FP32 shard after it, and a 0/1 factor
commutes with the sum exactly.  With gradient accumulation the sum of masked micro-step
gradients equals the mask times their sum for the same reason.

One optimizer step::

    loss = ...; loss.backward()              # FSDP2 reduce-scatters d loss / d weight_q
    gather.gradients_to_latents()            # latent.grad = mask * weight.grad (in place)
    optimizer.step(); optimizer.zero_grad()  # over gather.parameters() + the other params
    refresh_nvfp4_weight_amax(model)         # family amax from the latent shards
    gather.requantize()                      # weight <- fq(bf16(latent)) for the next step

``model.state_dict()`` then holds the quantized weights; ``latent_state_dict()`` gives the
latents under the same keys.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _native
from .formats.nvfp4 import NVFP4Linear


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if hasattr(t, "to_local") else t


class NVFP4QuantizedGather:
    """Switches the NVFP4 W4A16 linears of ``model`` (after ``apply_fake_quant`` with fused
    runtime scales, and after ``fully_shard`` if FSDP2 is used) to quantize-before-gather."""

    def __init__(self, model: nn.Module):
        self.names: list[str] = []
        self.members: list[NVFP4Linear] = []
        for name, module in model.named_modules():
            if not isinstance(module, NVFP4Linear):
                continue
            if getattr(module, "lora_A", None) is not None or module._quantize_activations:
                raise ValueError(f"quantize-before-gather covers full-parameter W4A16 linears only ({name})")
            if module._amax_group is None:
                raise ValueError(f"{name} has no fused-family amax group (apply_fake_quant with fused runtime scales)")
            weight = module.weight
            if _local(weight).dtype != torch.float32:
                raise ValueError(f"{name}: the latent masters must be FP32")
            latent = nn.Parameter(weight.detach().clone(), requires_grad=True)
            local = _local(weight)
            # plain attributes: the latent must not become a module parameter (FSDP2 would
            # manage it and state_dict would hold it)
            module.__dict__["_latent_shard"] = latent
            module.__dict__["_shadow_mask"] = torch.empty(_native.mask_nbytes(local.numel()), dtype=torch.uint8,
                                                          device=local.device)
            module.__dict__["_prequantized"] = True
            self.names.append(name)
            self.members.append(module)
        if not self.members:
            raise ValueError("the model has no NVFP4 W4A16 linears")

    def parameters(self) -> list[nn.Parameter]:
        """The FP32 latent masters, which the optimizer steps in place of the weights."""

        return [m._latent_shard for m in self.members]

    def other_parameters(self, model: nn.Module) -> list[nn.Parameter]:
        """The model's remaining trainable parameters (everything but the quantized weights)."""

        skip = {id(m.weight) for m in self.members}
        return [p for p in model.parameters() if p.requires_grad and id(p) not in skip]

    @torch.no_grad()
    def requantize(self) -> None:
        """weight <- fq(bf16(latent)) (FP32) and the STE mask, per local shard, with the
        family's current tensor amax; call after every amax refresh."""

        for m in self.members:
            amax = m._amax_group.tensor_amax_value
            if amax is None:
                raise RuntimeError("refresh the fused-family weight amax (refresh_nvfp4_weight_amax) before requantize")
            latent = _local(m._latent_shard)
            weight = _local(m.weight)
            if latent.numel() == 0:
                continue
            _native.nvfp4_qdq_shadow(latent.reshape(-1, latent.shape[-1]), amax, weight.reshape(-1, weight.shape[-1]),
                                     m._shadow_mask)

    @torch.no_grad()
    def gradients_to_latents(self) -> None:
        """Move each weight gradient to its latent, multiplied by the STE mask (in place)."""

        for m in self.members:
            grad = m.weight.grad
            m._latent_shard.grad = None
            if grad is None:
                continue
            local = _local(grad)
            if local.numel() > 0:
                _native.ste_backward(local, m._shadow_mask, out=local)
            m._latent_shard.grad = grad
            m.weight.grad = None

    def latent_state_dict(self) -> dict[str, torch.Tensor]:
        """``{<module>.weight: latent}``: the trainable weights under the model's own keys."""

        return {f"{name}.weight": m._latent_shard.detach() for name, m in zip(self.names, self.members)}
