"""GPU parity of the NVFP4 / MXFP4 kernels (through libqatf.so) with the reference.

Three layers of evidence:
  * every golden fixture produced by the reference's own torch functions is reproduced bit
    for bit (values, masks, packed bytes, scales, dequantized tensors, STE gradients);
  * seeded random tensors in every dtype and awkward shape match the CPU oracle;
  * the full benchmark configurations match SHA-256 digests of the reference outputs.
Modelled on the reference's tests/quant/test_fp4_triton.py (bitwise torch.equal on the
values and the STE mask).
"""

import hashlib
import json

import pytest
import torch

import oracle
from qatfactory_b200 import _native, workloads
from qatfactory_b200.quant import (
    dequantize_mxfp4,
    dequantize_nvfp4,
    fake_quantize_mxfp4,
    fake_quantize_mxfp4_activation,
    fake_quantize_nvfp4,
    fake_quantize_nvfp4_activation,
    pack_e2m1_rows,
    quantize_mxfp4,
    quantize_nvfp4,
    unpack_e2m1_rows,
)
from tests.golden.fixtures import GOLDEN_DIR, load_cases

pytestmark = pytest.mark.gpu

FP4 = load_cases(GOLDEN_DIR / "fp4_golden.npz")
DIGESTS = json.loads((GOLDEN_DIR / "digests.json").read_text())
DEV = "cuda"


def bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16)
    if t.dtype == torch.float32:
        return t.view(torch.int32)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8)
    return t


def assert_bits(a: torch.Tensor, b: torch.Tensor) -> None:
    assert a.shape == b.shape, (a.shape, b.shape)
    assert a.dtype == b.dtype, (a.dtype, b.dtype)
    ba, bb = bits(a), bits(b)
    if not torch.equal(ba, bb):
        diff = (ba != bb).nonzero()
        raise AssertionError(f"{diff.shape[0]} mismatches, first at {diff[0].tolist()}: {a.flatten()[0]} ...")


def digest(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous().reshape(-1)
    if t.dtype == torch.bool:
        t = t.to(torch.uint8)
    return hashlib.sha256(t.view(torch.uint8).numpy().tobytes()).hexdigest()


def names(prefix):
    return sorted(k for k in FP4 if k.startswith(prefix + "/"))


# ------------------------------------------------------------------ golden fixtures


@pytest.mark.parametrize("name", names("nvfp4_qdq"))
def test_nvfp4_qdq_golden(name):
    c = FP4[name]
    x = c["x"].to(DEV)
    y, mask = _native.nvfp4_qdq(x, torch.tensor(c["amax"], device=DEV))
    assert_bits(y, c["y"])
    assert torch.equal(_native.unpack_mask(mask, x.numel(), x.shape).cpu(), c["mask"])


@pytest.mark.parametrize("name", names("mxfp4_even"))
def test_mxfp4_even_golden(name):
    c = FP4[name]
    x = c["x"].to(DEV)
    y, mask = _native.mxfp4_qdq_even(x)
    assert_bits(y, c["y"])
    assert torch.equal(_native.unpack_mask(mask, x.numel(), x.shape).cpu(), c["mask"])


@pytest.mark.parametrize("name", names("mxfp4_ceil"))
def test_mxfp4_ceil_golden(name):
    c = FP4[name]
    assert_bits(fake_quantize_mxfp4_activation(c["x"].to(DEV)), c["y"])


@pytest.mark.parametrize("name", names("nvfp4_pack"))
def test_nvfp4_pack_golden(name):
    c = FP4[name]
    r = quantize_nvfp4(c["x"].to(DEV), tensor_amax=torch.tensor(c["amax"], device=DEV))
    assert torch.equal(r.packed_weight.cpu(), c["packed"])
    assert_bits(r.weight_scale, c["scales"])
    assert_bits(r.weight_scale_2, c["scale_2"].reshape(()))
    assert_bits(r.reconstruction, c["recon"])
    assert_bits(dequantize_nvfp4(r.packed_weight, r.weight_scale, r.weight_scale_2), c["dequant"])


@pytest.mark.parametrize("name", names("mxfp4_pack"))
def test_mxfp4_pack_golden(name):
    c = FP4[name]
    r = quantize_mxfp4(c["x"].to(DEV))
    assert torch.equal(r.packed_weight.cpu(), c["packed"])
    assert torch.equal(r.weight_scale.cpu(), c["scales"])
    assert_bits(r.reconstruction, c["recon"])
    assert_bits(dequantize_mxfp4(r.packed_weight, r.weight_scale), c["dequant"])


@pytest.mark.parametrize("name", names("ste"))
def test_ste_backward_golden(name):
    c = FP4[name]
    leaf = c["x"].to(DEV).requires_grad_()
    if name.startswith("ste/nvfp4"):
        amax = torch.tensor(float(c["x"].float().abs().amax()) * 0.5, device=DEV)
        out = fake_quantize_nvfp4(leaf, tensor_amax=amax)
    else:
        out = fake_quantize_mxfp4(leaf)
    out.backward(c["grad_out"].to(DEV))
    assert_bits(out, c["y"])
    assert_bits(leaf.grad, c["grad_in"])


def test_e2m1_nibble_packing_golden():
    c = FP4["e2m1_pack/known"]
    packed = pack_e2m1_rows(c["nibbles"].to(DEV))
    assert torch.equal(packed.cpu(), c["packed"])
    assert torch.equal(unpack_e2m1_rows(packed).cpu(), c["nibbles"])


# -------------------------------------------------------- seeded cases vs the oracle

DTYPES = (torch.bfloat16, torch.float16, torch.float32)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("magnitude", (1e-4, 1.0, 1e4))
def test_random_tensors_match_oracle(dtype, magnitude):
    g = torch.Generator().manual_seed(10)
    x = (torch.randn(257, 4096, generator=g) * magnitude).to(dtype)
    xd = x.to(DEV)
    for amax in (None, float(x.float().abs().amax()) * 1.25):
        ref_y, ref_m = oracle.nvfp4_qdq(x, amax)
        amax_t = _native.tensor_amax(xd) if amax is None else torch.tensor(amax, device=DEV)
        y, m = _native.nvfp4_qdq(xd, amax_t)
        assert_bits(y, ref_y)
        assert torch.equal(_native.unpack_mask(m, x.numel(), x.shape).cpu(), ref_m)
    ref_y, ref_m = oracle.mxfp4_qdq_even(x)
    y, m = _native.mxfp4_qdq_even(xd)
    assert_bits(y, ref_y)
    assert torch.equal(_native.unpack_mask(m, x.numel(), x.shape).cpu(), ref_m)
    assert_bits(_native.mxfp4_qdq_ceil(xd), oracle.mxfp4_qdq_ceil(x))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", ((4096, 100), (4096, 24), (1, 16), (1, 32), (3, 48), (7, 17), (5, 40), (33, 80)))
def test_padding_and_tiny_shapes_match_oracle(dtype, shape):
    g = torch.Generator().manual_seed(shape[0] * shape[1])
    x = torch.randn(shape, generator=g).to(dtype)
    xd = x.to(DEV)
    ref_y, ref_m = oracle.nvfp4_qdq(x)
    y = fake_quantize_nvfp4(xd)
    assert_bits(y, ref_y)
    ref_y, ref_m = oracle.mxfp4_qdq_even(x)
    assert_bits(fake_quantize_mxfp4(xd), ref_y)


def test_noncontiguous_and_row_strided_inputs():
    g = torch.Generator().manual_seed(3)
    base = torch.randn(100, 64, generator=g).to(torch.bfloat16)
    src = base.to(DEV).T  # transposed view: copied to a dense tensor like the reference does
    assert not src.is_contiguous()
    assert_bits(fake_quantize_nvfp4(src), oracle.nvfp4_qdq(base.T.contiguous())[0])
    wide = torch.randn(64, 512, generator=g).to(torch.bfloat16)
    view = wide.to(DEV)[:, 128:384]  # row stride 512, unit column stride: no copy
    assert view.stride() == (512, 1)
    assert_bits(fake_quantize_mxfp4(view), oracle.mxfp4_qdq_even(wide[:, 128:384].contiguous())[0])
    assert_bits(_native.mxfp4_qdq_ceil(view), oracle.mxfp4_qdq_ceil(wide[:, 128:384].contiguous()))


def test_activation_paths_on_flattened_3d():
    g = torch.Generator().manual_seed(12)
    act = torch.randn(8, 1024, 4096, generator=g).to(torch.bfloat16)
    flat = act.reshape(-1, 4096)
    amax = float(act.float().abs().amax()) * 0.75
    out = fake_quantize_nvfp4_activation(act.to(DEV), torch.tensor(amax, device=DEV))
    assert_bits(out, oracle.nvfp4_qdq(flat, amax)[0].reshape(act.shape))
    assert_bits(fake_quantize_mxfp4_activation(act.to(DEV)), oracle.mxfp4_qdq_ceil(flat).reshape(act.shape))


def test_zero_amax_paths_and_gradients():
    t = torch.zeros(3, 24, dtype=torch.bfloat16, device=DEV, requires_grad=True)
    implicit = fake_quantize_nvfp4(t)
    explicit = fake_quantize_nvfp4(t, tensor_amax=torch.zeros((), device=DEV))
    assert torch.equal(implicit, t) and torch.equal(explicit, t)
    explicit.sum().backward()
    assert torch.equal(t.grad, torch.ones_like(t))


def test_activation_gradients_pass_unmasked():
    a = torch.zeros(2, 3, 64, dtype=torch.bfloat16, device=DEV, requires_grad=True)
    with torch.no_grad():
        a[0, 0, 32] = 1e-30
    out = fake_quantize_mxfp4_activation(a)
    out.sum().backward()
    assert torch.equal(a.grad, torch.ones_like(a))
    with pytest.raises(ValueError, match="divisible by 32"):
        fake_quantize_mxfp4_activation(torch.randn(4, 33, device=DEV))


def test_pack_reconstruction_equals_fake_quant_and_dequant():
    g = torch.Generator().manual_seed(21)
    w = (torch.randn(512, 1024, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    r = quantize_nvfp4(w)
    assert torch.equal(r.reconstruction, fake_quantize_nvfp4(w))
    assert torch.equal(dequantize_nvfp4(r.packed_weight, r.weight_scale, r.weight_scale_2).to(w.dtype), r.reconstruction)
    m = quantize_mxfp4(w)
    assert torch.equal(m.reconstruction, fake_quantize_mxfp4(w))
    assert torch.equal(dequantize_mxfp4(m.packed_weight, m.weight_scale).to(w.dtype), m.reconstruction)


def test_tensor_amax_matches_torch_reduction():
    g = torch.Generator().manual_seed(5)
    for dtype in DTYPES:
        for n in (1, 7, 4096, 1_000_003):
            x = torch.randn(n, generator=g).to(dtype)
            assert float(_native.tensor_amax(x.to(DEV))) == float(x.float().abs().amax())
    x = torch.randn(1000, generator=g)
    x[123] = float("nan")
    assert torch.isnan(_native.tensor_amax(x.to(DEV)))


# --------------------------------------------- full benchmark configurations (digests)


def test_config1_nvfp4_full_size_digests():
    w = workloads.config1_weight().to(DEV)
    grad = workloads.config1_grad().to(DEV)
    amax = _native.tensor_amax(w)
    assert float(amax) == DIGESTS["config1/amax"]
    y, mask = _native.nvfp4_qdq(w, amax)
    assert digest(y) == DIGESTS["config1/nvfp4_qdq/y"]
    assert digest(_native.unpack_mask(mask, w.numel(), w.shape)) == DIGESTS["config1/nvfp4_qdq/mask"]
    assert digest(_native.ste_backward(grad, mask)) == DIGESTS["config1/nvfp4_ste/grad_in"]
    r = quantize_nvfp4(w)
    assert digest(r.packed_weight) == DIGESTS["config1/nvfp4_pack/packed"]
    assert digest(r.weight_scale.view(torch.uint8)) == DIGESTS["config1/nvfp4_pack/scales"]
    assert digest(r.weight_scale_2) == DIGESTS["config1/nvfp4_pack/scale_2"]


def test_config2_mxfp4_full_size_digests():
    w = workloads.config2_weight().to(DEV)
    y, mask = _native.mxfp4_qdq_even(w)
    assert digest(y) == DIGESTS["config2a/mxfp4_even/y"]
    assert digest(_native.unpack_mask(mask, w.numel(), w.shape)) == DIGESTS["config2a/mxfp4_even/mask"]
    r = quantize_mxfp4(w)
    assert digest(r.packed_weight) == DIGESTS["config2a/mxfp4_pack/packed"]
    assert digest(r.weight_scale) == DIGESTS["config2a/mxfp4_pack/scales"]
    del w, y, mask, r
    x = workloads.config2_activation().to(DEV)
    assert digest(_native.mxfp4_qdq_ceil(x)) == DIGESTS["config2b/mxfp4_ceil/y"]


def test_config4_operand_quantization_digests():
    x, w, _ = workloads.config4_inputs()
    x, w = x.to(DEV), w.to(DEV)
    xa = _native.tensor_amax(x)
    assert float(xa) == DIGESTS["config4/x_amax"]
    y, mask = _native.nvfp4_qdq(x, xa)
    assert digest(y) == DIGESTS["config4/x_qdq/y"]
    assert digest(_native.unpack_mask(mask, x.numel(), x.shape)) == DIGESTS["config4/x_qdq/mask"]
    y, mask = _native.nvfp4_qdq(w, _native.tensor_amax(w))
    assert digest(y) == DIGESTS["config4/w_qdq/y"]
    assert digest(_native.unpack_mask(mask, w.numel(), w.shape)) == DIGESTS["config4/w_qdq/mask"]


def test_config2_size_independent_properties():
    """At full size: pack -> dequant reproduces the fake-quant, and QDQ is idempotent."""

    w = workloads.config2_weight().to(DEV)
    y, _ = _native.mxfp4_qdq_even(w)
    y2, _ = _native.mxfp4_qdq_even(y)
    assert torch.equal(y, y2)  # E2M1 x 2^k values are fixed points of the EVEN quantizer
    r = quantize_mxfp4(w)
    assert torch.equal(dequantize_mxfp4(r.packed_weight, r.weight_scale).to(w.dtype), y)


def test_stream_rows_matches_whole_tensor_calls():
    """Host tensors streamed through the GPU in row chunks give the whole-tensor results."""

    from qatfactory_b200.host_stream import stream_rows
    from qatfactory_b200.quant import fake_quantize_mxfp4, fake_quantize_nvfp4

    x = workloads.student_t_outliers((5000, 512), seed=21, outlier_seed=22).pin_memory()
    dev = torch.device("cuda", 0)
    out = torch.empty_like(x).pin_memory()
    stream_rows(fake_quantize_mxfp4, x, out, dev, chunk_rows=640)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), fake_quantize_mxfp4(x.to(dev)).cpu().view(torch.int16))
    amax = x.to(dev).abs().amax().float()
    out2 = torch.empty_like(x).pin_memory()
    stream_rows(lambda c: fake_quantize_nvfp4(c, tensor_amax=amax), x, out2, dev, chunk_rows=1000, buffers=2)
    torch.cuda.synchronize()
    assert torch.equal(out2.view(torch.int16), fake_quantize_nvfp4(x.to(dev), tensor_amax=amax).cpu().view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_expert_fake_quant_is_bit_identical_to_per_expert_2d_and_oracle(dtype):
    """test_nvfp4_moe.py:35-43 and :59-69 on the GPU: one batched launch equals the experts one
    by one (and the CPU oracle); a zero-amax expert gives zeros and a pass-through gradient."""

    from qatfactory_b200.quant import fake_quantize_nvfp4_experts

    w = workloads.normal((6, 96, 256), 0.02, seed=31).to(dtype)
    w[2] = 0
    amax = w.float().abs().amax(dim=(1, 2))
    wd = w.to(DEV).requires_grad_(True)
    q = fake_quantize_nvfp4_experts(wd, amax.to(DEV))
    g = workloads.normal((6, 96, 256), 1.0, seed=32).to(dtype)
    q.backward(g.to(DEV))
    for e in range(6):
        ref = fake_quantize_nvfp4(w[e].to(DEV), tensor_amax=amax[e].to(DEV))
        assert torch.equal(q[e].detach(), ref)
        o_y, o_mask = oracle.nvfp4_qdq(w[e], amax[e])
        assert torch.equal(q[e].detach().cpu(), o_y)
        assert torch.equal(wd.grad[e].cpu(), g[e] * o_mask.to(dtype) if e != 2 else g[e])
    assert int(q[2].count_nonzero()) == 0


def test_expert_linear_recomputes_the_quantized_weight_in_backward():
    from qatfactory_b200.quant.formats.nvfp4_experts import _ExpertFakeQuantLinear

    w = workloads.normal((64, 128), 0.02, seed=33).to(DEV).requires_grad_(True)
    x = workloads.normal((3, 10, 128), 1.0, seed=34).to(DEV).requires_grad_(True)
    amax = w.detach().float().abs().amax()
    y = _ExpertFakeQuantLinear.apply(x, w, amax)
    g = torch.randn_like(y)
    y.backward(g)
    w2 = w.detach().clone().requires_grad_(True)
    x2 = x.detach().clone().requires_grad_(True)
    torch.nn.functional.linear(x2, fake_quantize_nvfp4(w2, tensor_amax=amax)).backward(g)
    assert torch.equal(y.detach(), torch.nn.functional.linear(x2.detach(), fake_quantize_nvfp4(w2.detach(), tensor_amax=amax)))
    torch.testing.assert_close(x.grad, x2.grad, rtol=0, atol=0)
    torch.testing.assert_close(w.grad, w2.grad, rtol=1e-2, atol=1e-3)


def _signed_zero_and_tiny_tensor(scale: float, seed: int) -> torch.Tensor:
    """BF16 [128, 4096]: N(0, scale) blocks salted with +0, -0, tiny elements of both signs
    (|x| < 2^-100) and small negatives whose codes round to zero (-0 codes)."""

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(128, 4096, generator=g) * scale
    salt = torch.tensor([0.0, -0.0, 1e-35, -1e-35, -2e-33, 3e-38, -1e-3 * scale, 1e-3 * scale])
    pos = torch.randint(0, x.numel(), (x.numel() // 5,), generator=g)
    x.view(-1)[pos] = salt[torch.randint(0, salt.numel(), pos.shape, generator=g)]
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("scale", (1.0, 1e-28))
def test_signed_zero_and_tiny_elements_match_oracle(scale):
    """The BF16 fast paths feed signed quotients to the E2M1 converter and admit blocks with
    elements below 2^-100 when the block scale is at least 2^-96: zero signs, -0 codes and
    tiny elements must still match the reference bit for bit, on both sides of that guard
    (scale 1e-28 puts block scales around 2^-96)."""

    x = _signed_zero_and_tiny_tensor(scale, seed=int(scale > 1e-10) + 77)
    xd = x.to(DEV)
    amax = oracle.tensor_amax(x)
    ref_y, ref_m = oracle.nvfp4_qdq(x, amax)
    y, m = _native.nvfp4_qdq(xd, amax.to(DEV))
    assert_bits(y, ref_y)
    assert torch.equal(_native.unpack_mask(m, x.numel(), x.shape).cpu(), ref_m)
    r = quantize_nvfp4(xd, tensor_amax=amax.to(DEV))
    p_ref, s_ref, s2_ref, rc_ref = oracle.nvfp4_pack(x, amax)
    assert torch.equal(r.packed_weight.cpu(), p_ref)
    assert torch.equal(r.weight_scale.cpu().view(torch.uint8), s_ref)
    assert_bits(r.reconstruction, rc_ref)
    codes, _, deq, mk = _native.nvfp4_operand(xd, amax.to(DEV), _native.OPERAND_A)
    assert torch.equal(codes.cpu(), p_ref)
    assert_bits(deq, ref_y)
    assert torch.equal(_native.unpack_mask(mk, x.numel(), x.shape).cpu(), ref_m)
    ref_y, ref_m = oracle.mxfp4_qdq_even(x)
    y, m = _native.mxfp4_qdq_even(xd)
    assert_bits(y, ref_y)
    assert torch.equal(_native.unpack_mask(m, x.numel(), x.shape).cpu(), ref_m)
    assert_bits(_native.mxfp4_qdq_ceil(xd), oracle.mxfp4_qdq_ceil(x))
    mp = quantize_mxfp4(xd)
    p_ref, s_ref, rc_ref = oracle.mxfp4_pack(x)
    assert torch.equal(mp.packed_weight.cpu(), p_ref)
    assert torch.equal(mp.weight_scale.cpu(), s_ref)
    assert_bits(mp.reconstruction, rc_ref)

