"""Block-FP8 frozen bases and LoRA-QAD of fused experts on the GPU.

* ``qatf_fp8_block_dequant`` equals the reference's torch expression
  ``(codes.float() * scale_inv[block]).to(dtype)`` (fp8_base.py:27-52) bit for bit: E4M3 and
  E5M2 codes (every byte value), FP32 / BF16 / FP16 outputs, the vector and the scalar path, a
  batched expert tensor and a broadcast scale grid.
* ``NVFP4ExpertLoRA`` and an FP8-based LoRA ``NVFP4Linear`` against the reference's own modules
  (nvfp4_experts.py:65-366, nvfp4.py:610-627, from ``baseline/_ref`` when installed) on the
  same adapters: outputs and adapter gradients within 5e-2 relative Frobenius (the reference's
  CUDA path rounds the tensor scale amax / 2688 as a multiply by the reciprocal, which moves
  single codes; its CPU path, which this repository follows, agrees bit for bit), and the
  shared-base teacher output exactly.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
from torch import nn

from qatfactory_b200 import _native
from qatfactory_b200.quant import NVFP4ExpertLoRA, NVFP4Linear, dequantize_fp8_blocks, shared_base_teacher

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _torch_dequant(weight, scale_inv, dtype):
    rows, cols = weight.shape[-2:]
    sr, sc = scale_inv.shape[-2:]
    blocked = weight.to(torch.float32).reshape(*weight.shape[:-2], sr, rows // sr, sc, cols // sc)
    scales = scale_inv.to(torch.float32).reshape(*scale_inv.shape[:-2], sr, 1, sc, 1)
    return (blocked * scales).reshape(weight.shape).to(dtype)


@pytest.mark.parametrize("fp8", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape,grid", [((256, 512), (2, 4)), ((3, 128, 256), (3, 1, 2)), ((96, 40), (3, 5)),
                                        ((2, 64, 48), (1, 2, 3))])
def test_fp8_block_dequant_is_the_torch_expression(fp8, dtype, shape, grid):
    g = torch.Generator().manual_seed(len(shape) * 7 + shape[-1])
    codes = torch.randint(0, 256, shape, generator=g, dtype=torch.uint8)
    codes.view(-1)[:256] = torch.arange(256, dtype=torch.uint8)[: min(256, codes.numel())]  # every byte value
    weight = codes.view(fp8).to(DEV)
    scale_inv = (torch.rand(grid, generator=g) * 4 + 1e-3).to(DEV)
    got = dequantize_fp8_blocks(weight, scale_inv, dtype)
    want = _torch_dequant(weight, scale_inv.expand(*shape[:-2], *grid[-2:]) if len(grid) < len(shape) else scale_inv,
                          dtype)
    torch.cuda.synchronize()
    finite = ~torch.isnan(want)  # NaN codes stay NaN (payload bits aside)
    assert torch.equal(torch.isnan(got), ~finite)
    bits = torch.int32 if dtype == torch.float32 else torch.int16
    assert torch.equal(got[finite].view(bits), want[finite].view(bits))


def _ref_quant():
    if not (REF_DIR / "qatfactory").is_dir():
        pytest.skip("reference not installed under baseline/_ref")
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    import qatfactory.quant as rq

    return rq


class _Experts(nn.Module):
    def __init__(self, E, H, I, seed, fp8=False):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        gu = torch.randn(E, 2 * I, H, generator=g) * 0.02
        dn = torch.randn(E, H, I, generator=g) * 0.02
        if fp8:  # block-FP8 codes with a 128 x 128 scale grid, as a pre-quantized checkpoint ships
            self.gate_up_proj_scale_inv = (torch.rand(E, 2 * I // 128, H // 128, generator=g) * 1e-3 + 1e-4).to(DEV)
            self.down_proj_scale_inv = (torch.rand(E, H // 128, I // 128, generator=g) * 1e-3 + 1e-4).to(DEV)
            gu = gu / 0.02 * 50  # well inside the E4M3 range (448)
            dn = dn / 0.02 * 50
            self.gate_up_proj = nn.Parameter(gu.to(torch.float8_e4m3fn).to(DEV), requires_grad=False)
            self.down_proj = nn.Parameter(dn.to(torch.float8_e4m3fn).to(DEV), requires_grad=False)
        else:
            self.gate_up_proj = nn.Parameter(gu.to(torch.bfloat16).to(DEV))
            self.down_proj = nn.Parameter(dn.to(torch.bfloat16).to(DEV))
        self.act_fn = nn.SiLU()


def _rel(a, b):
    a, b = a.detach().double(), b.detach().double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("fp8,hybrid,w4a4", [(False, True, False), (False, False, False), (True, True, False),
                                              (False, True, True)])
def test_expert_lora_matches_reference_module(fp8, hybrid, w4a4):
    rq = _ref_quant()
    from qatfactory.quant.formats.nvfp4_experts import NVFP4ExpertLoRA as RefLoRA

    E, H, I, T, K, r = 4, 256, 128, 64, 2, 8
    ours = NVFP4ExpertLoRA(_Experts(E, H, I, 51, fp8), r, 16.0, hybrid_shared=hybrid)
    ref = RefLoRA(_Experts(E, H, I, 51, fp8), r, 16.0, hybrid_shared=hybrid)
    g = torch.Generator().manual_seed(52)
    with torch.no_grad():
        for leaf in ("gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B"):
            value = (torch.randn(getattr(ours, leaf).shape, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
            getattr(ours, leaf).copy_(value)
            getattr(ref, leaf).copy_(value)
    for m in (ours, ref):
        m.train()
        m._track_input_amax = True
        m._quantize_activations = w4a4
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    w, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g), -1), K, dim=-1)
    idx, w = idx.to(DEV), w.to(torch.bfloat16).to(DEV)
    up = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    # the reference module on the CPU too: its torch CPU path forms the tensor scale by true
    # division, as this repository does, so only GEMM rounding separates the two
    src_cpu = _Experts(E, H, I, 51, fp8)
    src_cpu.gate_up_proj = nn.Parameter(src_cpu.gate_up_proj.detach().cpu(), requires_grad=False)
    src_cpu.down_proj = nn.Parameter(src_cpu.down_proj.detach().cpu(), requires_grad=False)
    if fp8:
        src_cpu.gate_up_proj_scale_inv = src_cpu.gate_up_proj_scale_inv.cpu()
        src_cpu.down_proj_scale_inv = src_cpu.down_proj_scale_inv.cpu()
    ref_cpu = RefLoRA(src_cpu, r, 16.0, hybrid_shared=hybrid)
    with torch.no_grad():
        for leaf in ("gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B"):
            getattr(ref_cpu, leaf).copy_(getattr(ours, leaf).cpu())
    ref_cpu.train()
    ref_cpu._track_input_amax = True
    ref_cpu._quantize_activations = w4a4

    y_ours = ours(hidden, idx, w)
    y_ours.backward(up)
    y_ref = ref(hidden, idx, w)
    y_ref.backward(up)
    y_cpu = ref_cpu(hidden.cpu(), idx.cpu(), w.cpu())
    y_cpu.backward(up.cpu())
    torch.cuda.synchronize()
    assert _rel(y_ours.cpu(), y_cpu) <= 1e-2
    # against the reference's CUDA path, whose device-side tensor scales move single codes of the
    # weights (and, with W4A4, of the 4-bit activations): measured up to 5.7e-2 with W4A4
    assert _rel(y_ours, y_ref) <= (8e-2 if w4a4 else 5e-2)
    for leaf in ("gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B"):
        g_ours, g_cpu, g_gpu = getattr(ours, leaf).grad, getattr(ref_cpu, leaf).grad, getattr(ref, leaf).grad
        assert _rel(g_ours.cpu(), g_cpu) <= 1e-2, leaf
        if w4a4:
            # with 4-bit activations the reference's CUDA path departs from its own CPU path
            # further than this module does (measured 0.26 on gate_up_lora_A)
            assert _rel(g_ours.cpu(), g_cpu) <= _rel(g_gpu.cpu(), g_cpu) + 1e-3, leaf
        else:
            assert _rel(g_ours, g_gpu) <= 5e-2, leaf
    assert torch.equal(ours._gate_up_input_amax, ref._gate_up_input_amax)
    if w4a4:
        assert torch.equal(ours._gate_up_input_amax_static, ref._gate_up_input_amax_static)
        assert _rel(ours._down_input_amax_static, ref._down_input_amax_static) <= 1e-2
    for e in range(E):  # the merged weights the quantizer sees are identical
        assert torch.equal(ours.effective_gate_up(e), ref.effective_gate_up(e))
        assert torch.equal(ours.effective_down(e), ref.effective_down(e))
    with torch.no_grad(), shared_base_teacher():
        t_ours = ours(hidden, idx, w)
    with torch.no_grad(), rq.shared_base_teacher():
        t_ref = ref(hidden, idx, w)
    assert torch.equal(t_ours, t_ref)


def test_fp8_lora_linear_matches_reference_module():
    rq = _ref_quant()
    g = torch.Generator().manual_seed(61)
    lin = nn.Linear(512, 256, bias=False)
    lin.weight = nn.Parameter((torch.randn(256, 512, generator=g) * 50).to(torch.float8_e4m3fn).to(DEV),
                              requires_grad=False)
    lin.weight_scale_inv = (torch.rand(2, 4, generator=g) * 1e-3 + 1e-4).to(DEV)
    ours = NVFP4Linear.from_fp8_linear(lin)
    ref = rq.NVFP4Linear.from_fp8_linear(lin)
    ours.init_lora(8, 16.0)
    ref.init_lora(8, 16.0)
    with torch.no_grad():
        a = (torch.randn(8, 512, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
        b = (torch.randn(256, 8, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
        for m in (ours, ref):
            m.lora_A.copy_(a)
            m.lora_B.copy_(b)
    assert torch.equal(ours.base_weight(), ref.base_weight())
    assert torch.equal(ours._effective_weight(), ref._effective_weight())
    x = torch.randn(128, 512, generator=g).to(torch.bfloat16).to(DEV)
    up = torch.randn(128, 256, generator=g).to(torch.bfloat16).to(DEV)
    y_ours = ours(x)
    y_ours.backward(up)
    y_ref = ref(x)
    y_ref.backward(up)
    torch.cuda.synchronize()
    assert _rel(y_ours, y_ref) <= 5e-2
    assert _rel(ours.lora_A.grad, ref.lora_A.grad) <= 5e-2
    assert _rel(ours.lora_B.grad, ref.lora_B.grad) <= 5e-2
