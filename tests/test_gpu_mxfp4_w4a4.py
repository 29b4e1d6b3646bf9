"""W4A4 MXFP4 linear on the tensor cores: the MXFP4 operand pass against the CPU oracle (the
codes and E8M0 scales of quantize_mxfp4 under the EVEN rule, the QDQ outputs and masks of both
rules, bit for bit), the block-scaled MXFP4 GEMM (tcgen05 kind::mxf4) against the exact product
of its operands and against the reference's BF16 matmul of the dequantized operands (relative
Frobenius error <= 1e-2), and MXFP4Linear with W4A4 against the reference formulation
F.linear(fake_quantize_mxfp4_activation(x), fake_quantize_mxfp4(w)) (mxfp4.py:285-290)."""

import numpy as np
import pytest
import torch

import oracle
from qatfactory_b200 import _native, workloads

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float64)
A, B = _native.OPERAND_A, _native.OPERAND_B
EVEN, CEIL = _native.MXFP4_EVEN, _native.MXFP4_CEIL


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def _offsets(rows: int, cols: int, role: int) -> torch.Tensor:
    """[4 (lane quarter), rows, cols / 128] byte offsets of the scale words in the layout of
    ``role``: 4 KB blocks of 128 lanes x 8 words, word v of lane L at (L / 8) * 256 + (L % 8) *
    16 + (v / 4) * 128 + (v % 4) * 4; the word of row r and 128-column K-block kb sits in the
    lanes r % 32 + 32 q."""

    r = torch.arange(rows).reshape(-1, 1)
    kb = torch.arange(cols // 128).reshape(1, -1)
    if role == A:
        blk = ((r // 128) * (cols // 256) + kb // 2) * 4096
        word = 4 * (kb % 2) + (r // 32) % 4
    else:
        blk = ((r // 256) * (cols // 128) + kb) * 4096
        word = ((r // 32) % 8).expand(rows, cols // 128)
    out = []
    for q in range(4):
        lane = r % 32 + 32 * q
        out.append(blk + (lane // 8) * 256 + (lane % 8) * 16 + (word // 4) * 128 + (word % 4) * 4)
    return torch.stack(out)


def to_layout(scales_rm: torch.Tensor, rows: int, cols: int, role: int) -> torch.Tensor:
    """Row-major [rows, cols / 32] scale bytes -> the operand layout of ``role``."""

    sc = scales_rm.reshape(rows, cols // 128, 4).cpu()
    out = torch.zeros(rows * (cols // 32) * 4, dtype=torch.uint8)
    for base in _offsets(rows, cols, role):
        for s in range(4):
            out[(base + s).reshape(-1)] = sc[:, :, s].reshape(-1)
    return out


def from_layout(scales: torch.Tensor, rows: int, cols: int, role: int) -> torch.Tensor:
    """The operand layout -> row-major [rows, cols / 32] bytes (lane quarter 0's copy), after
    checking that all four lane quarters hold the same words."""

    flat = scales.cpu()
    copies = []
    for base in _offsets(rows, cols, role):
        copies.append(torch.stack([flat[base + s] for s in range(4)], dim=-1).reshape(rows, cols // 32))
    for c in copies[1:]:
        assert torch.equal(c, copies[0])
    return copies[0]


def decode(codes: torch.Tensor, scales_rm: torch.Tensor) -> torch.Tensor:
    """Exact FP64 value of an MXFP4 operand: E2M1 code * 2^(E8M0 byte - 127)."""

    c = codes.cpu().to(torch.int64)
    nib = torch.stack([c & 0xF, c >> 4], dim=-1).reshape(c.shape[0], -1)
    val = E2M1[nib & 7] * torch.where(nib & 8 > 0, -1.0, 1.0).double()
    sc = torch.exp2(scales_rm.cpu().double() - 127.0).repeat_interleave(32, dim=1)
    return val * sc


def operand_input(rows, cols, seed):
    x = workloads.student_t_outliers((rows, cols), seed=seed, outlier_seed=seed + 1).to(torch.bfloat16)
    x[3, :64] = 0  # zero blocks
    x[5, 32:64] = 1e-32  # a tiny block
    x[6, 64:96] = -3e-39  # BF16 subnormals
    return x


@pytest.mark.parametrize("rule", [EVEN, CEIL])
@pytest.mark.parametrize("rows,cols,role", [(128, 256, A), (384, 4096, A), (256, 1024, A), (256, 128, B),
                                           (512, 4096, B)])
def test_mxfp4_operand_matches_oracle(rows, cols, role, rule):
    x = operand_input(rows, cols, seed=60 + rows + cols)
    codes, scales, deq, mask = _native.mxfp4_operand(x.to(DEV), role, rule)
    torch.cuda.synchronize()
    scales_rm = from_layout(scales, rows, cols, role)
    if rule == EVEN:
        o_packed, o_scales, _ = oracle.mxfp4_pack(x, recon=False)
        assert torch.equal(codes.cpu(), o_packed)
        assert torch.equal(scales_rm, o_scales)
        assert torch.equal(scales.cpu(), to_layout(o_scales, rows, cols, role))
        o_y, o_mask = oracle.mxfp4_qdq_even(x)
        want = torch.from_numpy(np.packbits(o_mask.reshape(-1).numpy().astype(np.uint8), bitorder="little"))
        assert torch.equal(mask.cpu(), want)
    else:
        o_y = oracle.mxfp4_qdq_ceil(x)
        assert bool((mask == 0xFF).all())
    assert torch.equal(deq.cpu().view(torch.int16), o_y.view(torch.int16))
    # the codes and scales the GEMM reads carry exactly the dequantized values
    assert torch.equal(decode(codes, scales_rm), deq.cpu().double())


def _mx_case(m, n, k, seed):
    x = operand_input(m, k, seed).to(DEV)
    w = workloads.normal((n, k), 0.02, seed=seed + 7).to(torch.bfloat16).to(DEV)
    ax = _native.mxfp4_operand(x, A, CEIL, mask=False)
    aw = _native.mxfp4_operand(w, B, EVEN)
    return ax, aw


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 512, 2048), (384, 768, 1280), (1152, 512, 512)])
def test_mxfp4_gemm_matches_exact_product_and_bf16_reference(m, n, k):
    (cx, sx, xq, _), (cw, sw, wq, _) = _mx_case(m, n, k, seed=m + n + k)
    y = _native.mxfp4_gemm(cx, sx, cw, sw)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    exact = decode(cx, from_layout(sx, m, k, A)) @ decode(cw, from_layout(sw, n, k, B)).T
    assert rel_fro(y.cpu(), exact) < 4e-3  # only the BF16 rounding of the output
    ref = torch.nn.functional.linear(xq, wq)  # the reference's BF16 matmul of the fake-quantized operands
    assert rel_fro(y, ref) < 1e-2


def test_mxfp4_gemm_config2_layer():
    """Configuration 2's tensors as one W4A4 layer: activations [16384, 4096] (CEIL) times the
    fused gate/up weight [24576, 4096] (EVEN), against the BF16 matmul of the dequantized
    operands on a row sample."""

    x = workloads.config2_activation().to(DEV)
    w = workloads.config2_weight().to(DEV)
    cx, sx, xq, _ = _native.mxfp4_operand(x, A, CEIL, mask=False)
    cw, sw, wq, _ = _native.mxfp4_operand(w, B, EVEN)
    y = _native.mxfp4_gemm(cx, sx, cw, sw)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    rows = torch.arange(0, x.shape[0], 61, device=DEV)
    ref = torch.nn.functional.linear(xq[rows], wq)
    assert rel_fro(y[rows], ref) < 1e-2


@pytest.mark.parametrize("lead,k,n", [((2, 128), 512, 768), ((7,), 512, 768), ((200,), 4128, 1000)])
def test_mxfp4_linear_w4a4_matches_reference_formulation(lead, k, n, monkeypatch):
    """MXFP4Linear with W4A4 on the tensor cores (shapes off the tiles zero-padded) against the
    reference's own formulation with its straight-through gradients: output and all three
    gradients within 1e-2."""

    from qatfactory_b200.quant.formats.mxfp4 import (MXFP4Linear, fake_quantize_mxfp4,
                                                      fake_quantize_mxfp4_activation)

    calls = []
    gemm = _native.mxfp4_gemm
    monkeypatch.setattr(_native, "mxfp4_gemm", lambda *a, **kw: calls.append(1) or gemm(*a, **kw))
    torch.manual_seed(2)
    lin = torch.nn.Linear(k, n, bias=True, device=DEV, dtype=torch.bfloat16)
    q = MXFP4Linear.from_linear(lin)
    q._quantize_activations = True
    x = workloads.student_t_outliers((*lead, k), seed=29, outlier_seed=30).to(DEV).requires_grad_(True)
    y = q(x)
    assert y.shape == (*lead, n) and calls == [1]
    g = torch.randn_like(y)
    y.backward(g)

    x2 = x.detach().clone().requires_grad_(True)
    w2 = q.weight.detach().clone().requires_grad_(True)
    b2 = q.bias.detach().clone().requires_grad_(True)
    ref = torch.nn.functional.linear(fake_quantize_mxfp4_activation(x2), fake_quantize_mxfp4(w2), b2)
    ref.backward(g)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    assert rel_fro(y.detach(), ref.detach()) < 1e-2
    assert rel_fro(x.grad, x2.grad) < 1e-2
    assert rel_fro(q.weight.grad, w2.grad) < 1e-2
    assert rel_fro(q.bias.grad, b2.grad) < 1e-2


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
def test_lora_w4a4_linear_on_the_tensor_cores_matches_reference_formulation(fmt, monkeypatch):
    """LoRA-QAD of a W4A4 linear (frozen base, adapters merged into the weight before its fake
    quant, lora.py:50-113): the tensor-core path's output, input gradient and adapter gradients
    against the reference formulation F.linear(fq_act(x), fq(W + s * B @ A)), within 1e-2."""

    from qatfactory_b200.quant.formats import mxfp4 as mx
    from qatfactory_b200.quant.formats import nvfp4 as nv

    name = "nvfp4_gemm" if fmt == "nvfp4" else "mxfp4_gemm"
    calls = []
    gemm = getattr(_native, name)
    monkeypatch.setattr(_native, name, lambda *a, **kw: calls.append(1) or gemm(*a, **kw))
    torch.manual_seed(5)
    k, n = 512, 768
    lin = torch.nn.Linear(k, n, bias=False, device=DEV, dtype=torch.bfloat16)
    q = (nv.NVFP4Linear if fmt == "nvfp4" else mx.MXFP4Linear).from_linear(lin)
    q.weight.requires_grad_(False)  # the frozen base
    q.init_lora(8, 16.0)
    with torch.no_grad():
        q.lora_B.normal_(0.0, 0.02)  # a nonzero delta, so the adapters change the quantized weight
    q._quantize_activations = True
    x = workloads.student_t_outliers((2, 128, k), seed=31, outlier_seed=32).to(DEV).requires_grad_(True)
    if fmt == "nvfp4":
        q._input_amax_static = x.detach().float().abs().amax()
    y = q(x)
    assert calls == [1]
    g = torch.randn_like(y)
    y.backward(g)

    a2 = q.lora_A.detach().clone().requires_grad_(True)
    b2 = q.lora_B.detach().clone().requires_grad_(True)
    x2 = x.detach().clone().requires_grad_(True)
    w_eff = q.weight.detach() + (q.lora_scaling * (b2 @ a2)).to(torch.bfloat16)
    if fmt == "nvfp4":
        xq = nv.fake_quantize_nvfp4_activation(x2, q._input_amax_static)
        wq = nv.fake_quantize_nvfp4(w_eff)
    else:
        xq = mx.fake_quantize_mxfp4_activation(x2)
        wq = mx.fake_quantize_mxfp4(w_eff)
    ref = torch.nn.functional.linear(xq, wq)
    ref.backward(g)
    torch.cuda.synchronize()
    assert int(_native.gemm_error_word(DEV)) == 0
    assert rel_fro(y.detach(), ref.detach()) < 1e-2
    assert rel_fro(x.grad, x2.grad) < 1e-2
    assert rel_fro(q.lora_A.grad, a2.grad) < 1e-2
    assert rel_fro(q.lora_B.grad, b2.grad) < 1e-2
    assert q.weight.grad is None
