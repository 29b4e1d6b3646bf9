"""The fused forward-KL distillation loss (qatfactory_b200/distill.py, qatf_kd_forward_kl)
against the reference's formulation (FP32 chunks of log_softmax / softmax / kl_div, autograd
for the gradient).  The vocabulary sums are ordered differently, so values agree to FP32
rounding: relative 1e-5 on the loss, 1e-3 relative Frobenius on the BF16 gradient."""

import pytest
import torch
import torch.nn.functional as F

from qatfactory_b200 import distill

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def reference_loss(s, t, labels, temperature=1.0, hard_label_weight=0.0, chunk=2048):
    """kd_loss.py:147-195 restated (shift, select, FP32 chunks, kl_div sum * T^2, mean)."""

    vocab = s.shape[-1]
    flat = labels[..., 1:].reshape(-1)
    valid = flat != -100
    ss = s[..., :-1, :].reshape(-1, vocab)[valid]
    tt = t[..., :-1, :].reshape(-1, vocab)[valid]
    total = torch.zeros((), device=s.device)
    ce = torch.zeros((), device=s.device)
    for i in range(0, ss.shape[0], chunk):
        sc, tc = ss[i:i + chunk].float(), tt[i:i + chunk].float()
        total = total + F.kl_div(F.log_softmax(sc / temperature, -1), F.softmax(tc / temperature, -1),
                                 reduction="sum") * temperature ** 2
        if hard_label_weight:
            ce = ce + F.cross_entropy(sc, flat[valid][i:i + chunk], reduction="sum")
    n = valid.sum().clamp_min(1)
    return total / n + hard_label_weight * ce / n


def rel_fro(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


@pytest.mark.parametrize("shape,temperature,ignore,hard", [((2, 65, 1000), 1.0, False, 0.0),
                                                           ((1, 129, 4099), 2.0, True, 0.0),
                                                           ((2, 33, 777), 1.0, True, 0.5)])
def test_fused_distill_loss_matches_reference_formulation(shape, temperature, ignore, hard):
    g = torch.Generator().manual_seed(shape[1])
    s = (torch.randn(shape, generator=g) * 3).to(torch.bfloat16).to(DEV)
    t = (torch.randn(shape, generator=g) * 3).to(torch.bfloat16).to(DEV)
    labels = torch.randint(0, shape[-1], shape[:2], generator=g).to(DEV)
    if ignore:
        labels[:, ::3] = -100
    s1 = s.clone().requires_grad_(True)
    s2 = s.clone().requires_grad_(True)
    out = distill.distill_loss(s1, t, labels, temperature=temperature, hard_label_weight=hard)
    ref = reference_loss(s2, t, labels, temperature, hard)
    out.loss.backward()
    ref.backward()
    assert abs(float(out.loss.detach()) - float(ref.detach())) <= 1e-5 * abs(float(ref.detach())) + 1e-6
    # with a hard-label term the KL and CE gradients are each rounded to BF16 before autograd
    # sums them (the reference rounds one FP32 sum), hence the looser bound there
    assert rel_fro(s1.grad, s2.grad) < (5e-3 if hard else 1e-3)
    assert int(out.num_tokens) == int((labels[..., 1:] != -100).sum())


def test_fused_distill_loss_at_qwen3_vocabulary():
    """Configuration 5's shape: 4096 positions x vocabulary 151936, BF16 logits."""

    g = torch.Generator(device=DEV).manual_seed(5)
    s = (torch.randn((1, 4096, 151936), generator=g, device=DEV) * 2).to(torch.bfloat16)
    t = (s.float() + 0.1 * torch.randn(s.shape, generator=g, device=DEV)).to(torch.bfloat16)
    labels = torch.zeros((1, 4096), dtype=torch.long, device=DEV)
    s1 = s.clone().requires_grad_(True)
    out = distill.distill_loss(s1, t, labels)
    out.loss.backward()
    s2 = s.clone().requires_grad_(True)
    ref = reference_loss(s2, t, labels)
    ref.backward()
    assert abs(float(out.loss.detach()) - float(ref.detach())) <= 1e-5 * abs(float(ref.detach()))
    assert rel_fro(s1.grad, s2.grad) < 1e-3


def test_minus_infinity_logits_follow_kl_div():
    s = torch.randn(1, 5, 64, device=DEV)
    t = torch.randn(1, 5, 64, device=DEV)
    t[..., 3] = float("-inf")  # zero teacher probability: contributes nothing
    labels = torch.zeros(1, 5, dtype=torch.long, device=DEV)
    out = distill.distill_loss(s, t, labels)
    ref = reference_loss(s, t, labels)
    assert torch.isfinite(out.loss)
    assert abs(float(out.loss) - float(ref)) <= 1e-5 * abs(float(ref)) + 1e-6
