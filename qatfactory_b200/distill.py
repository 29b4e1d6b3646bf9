"""Forward-KL distillation loss on the fused vocabulary kernel (``qatf_kd_forward_kl``).

Mirrors ``distill_loss`` of the reference (qatfactory/distill/kd_loss.py:147-195): drop the last
position, shift the labels, keep supervised tokens, and average T^2 * KL(softmax(t/T) ||
softmax(s/T)) over them, optionally plus hard-label cross entropy.  The reference materialises
FP32 chunks of both logit sets and runs log_softmax, softmax and kl_div over them, forward and
backward; here one kernel streams each row once for the loss and once more (mostly from L2)
for the gradient, which backward only rescales.  Values agree with the reference to FP32
rounding; the order of the vocabulary sums differs, so they are not bit-identical.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _native

IGNORE_INDEX = -100


@dataclass
class DistillLossOutput:
    loss: torch.Tensor  # combined, per-token mean (differentiable)
    distill_loss: torch.Tensor  # temperature-KL component (detached)
    ce_loss: torch.Tensor  # hard-label component (detached)
    num_tokens: torch.Tensor  # supervised token count
    metrics: dict[str, torch.Tensor] = field(default_factory=dict)


class _FusedForwardKL(torch.autograd.Function):
    """sum over rows of T^2 * KL_row, times ``scale``; the gradient is written by the forward
    kernel (already multiplied by ``scale``) and scaled by the incoming gradient here."""

    @staticmethod
    def forward(ctx, student, teacher, row_valid, temperature, scale):
        row_loss, grad = _native.kd_forward_kl(student.detach(), teacher.detach(), temperature, row_valid,
                                               want_grad=student.requires_grad, grad_scale=scale)
        ctx.used = False
        if grad is not None:
            ctx.save_for_backward(grad)
        return row_loss.sum() * scale

    @staticmethod
    def backward(ctx, grad_output):
        if ctx.used:
            raise RuntimeError("the fused distillation loss supports one backward pass per forward")
        ctx.used = True
        (grad,) = ctx.saved_tensors
        return grad.mul_(grad_output.to(grad.dtype)), None, None, None, None


def distill_loss(
    student_logits: torch.Tensor,
    teacher_logits: torch.Tensor,
    labels: torch.Tensor,
    *,
    temperature: float = 1.0,
    distill_weight: float = 1.0,
    hard_label_weight: float = 0.0,
    logits_chunk_size: int = 2048,
    compute_metrics: bool = False,
    metrics_top_k: tuple[int, ...] = (1, 5, 10),
    loss_denominator: torch.Tensor | int | None = None,
) -> DistillLossOutput:
    """``distill_loss`` of kd_loss.py:147-195 with the KL term on the fused kernel.
    ``logits_chunk_size`` is accepted for signature compatibility (the kernel needs no chunks)."""

    if compute_metrics:
        raise ValueError("agreement metrics are not computed by the fused distillation loss")
    vocab = student_logits.shape[-1]
    student = student_logits[..., :-1, :].reshape(-1, vocab)
    teacher = teacher_logits[..., :-1, :].reshape(-1, vocab)
    flat_labels = labels[..., 1:].reshape(-1)
    valid = flat_labels != IGNORE_INDEX
    token_count = valid.sum()
    count = int(token_count)  # one host read, where the reference's boolean gather syncs too
    if count == 0:
        zero = student_logits.sum() * 0
        return DistillLossOutput(zero, zero.detach(), zero.detach(), token_count, {})
    # the reference's torch.as_tensor(loss_denominator).clamp_min(1): a fractional denominator
    # is kept, not truncated
    denominator = float(max(count, 1)) if loss_denominator is None else max(float(loss_denominator), 1.0)
    all_valid = count == valid.numel()
    kl_over_denominator = _FusedForwardKL.apply(student, teacher.detach(), None if all_valid else valid,
                                                float(temperature), 1.0 / denominator)
    distill_mean = kl_over_denominator.detach() * (denominator / count)
    combined = distill_weight * kl_over_denominator
    ce_mean = distill_mean * 0
    if hard_label_weight:
        rows = student if all_valid else student[valid]
        targets = flat_labels if all_valid else flat_labels[valid]
        ce_sum = F.cross_entropy(rows.float(), targets, reduction="sum")
        ce_mean = (ce_sum / max(count, 1)).detach()
        combined = combined + hard_label_weight * (ce_sum / denominator)
    return DistillLossOutput(combined, distill_mean, ce_mean, token_count, {})
