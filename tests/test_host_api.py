"""Host-side behaviour of the drop-in API that needs no GPU: names, registry metadata,
argument errors (same messages as the reference), meta passthrough and the absence of
any CPU compute path."""

import pytest
import torch
from torch import nn

import qatfactory_b200.quant as q
from qatfactory_b200.quant.formats.nvfp4 import NVFP4_SCALE_DENOMINATOR

REFERENCE_EXPORTS_IN_SCOPE = {
    "ConvertedModules", "LoRAMixin", "MXFP4Linear", "NVFP4Linear", "Q4KLinear", "apply_fake_quant",
    "attach_nvfp4_amax_groups", "available_quant_formats", "build_nvfp4_fused_family_names",
    "commit_nvfp4_input_scales", "configure_q4k_reorders", "dequantize_mxfp4", "dequantize_nvfp4",
    "dequantize_q4_k", "fake_quantize_mxfp4", "fake_quantize_mxfp4_activation", "fake_quantize_nvfp4",
    "fake_quantize_nvfp4_activation", "fake_quantize_q4_k", "finalize_nvfp4_input_scales", "get_quant_format",
    "is_lora_quantized", "load_nvfp4_runtime_state_dict", "merge_lora_weight", "nvfp4_runtime_state_dict",
    "pack_deploy_weight", "pack_e2m1_rows", "quantize_mxfp4", "quantize_nvfp4", "quantize_q4_k",
    "refresh_nvfp4_weight_amax", "shared_base_teacher", "shared_base_teacher_enabled", "unpack_e2m1_rows",
    "v_head_reorder_perm", "fake_quantize_nvfp4_experts", "is_fused_experts",
}


def test_public_names_match_the_reference_package():
    assert REFERENCE_EXPORTS_IN_SCOPE <= set(q.__all__)
    for name in q.__all__:
        assert hasattr(q, name)


def test_format_registry_metadata():
    assert q.available_quant_formats() == ["mxfp4", "nvfp4", "q4_k", "q4_k_grid_search"]
    nv = q.get_quant_format("nvfp4")
    assert nv.quantizer_id == "standard_max" and nv.supports_fused_runtime_scales
    assert nv.activation_quant_requires_runtime_scales and nv.commit_input_scales is q.commit_nvfp4_input_scales
    mx = q.get_quant_format("mxfp4")
    assert mx.quantizer_id == "mx_even" and mx.supports_activation_quant and not mx.supports_fused_runtime_scales
    q4 = q.get_quant_format("q4_k")
    assert q4.quantizer_id == "q4_k_minmax" and q4.pack_weight is not None and not q4.supports_lora
    assert q.get_quant_format("q4_k_grid_search").quantizer_id == "q4_k_grid_search"
    with pytest.raises(ValueError, match="Unknown quant_format"):
        q.get_quant_format("int4")
    assert NVFP4_SCALE_DENOMINATOR == 2688.0


def test_fused_family_names():
    names = [f"model.layers.0.self_attn.{p}" for p in ("q_proj", "k_proj", "v_proj", "o_proj")]
    names += [f"model.layers.0.mlp.{p}" for p in ("gate_proj", "up_proj", "down_proj")]
    fams = q.build_nvfp4_fused_family_names(names)
    assert fams[0] == tuple(names[:3])
    assert ("model.layers.0.mlp.gate_proj", "model.layers.0.mlp.up_proj") in fams
    assert q.build_nvfp4_fused_family_names(["model.layers.0.self_attn.q_proj"]) == [("model.layers.0.self_attn.q_proj",)]
    with pytest.raises(ValueError, match="Incomplete fused NVFP4 family"):
        q.build_nvfp4_fused_family_names(["model.layers.0.mlp.gate_proj"])


def test_argument_errors_match_the_reference():
    w = torch.zeros(4, 32)
    with pytest.raises(ValueError, match="block_size=16"):
        q.fake_quantize_nvfp4(w, block_size=32)
    with pytest.raises(ValueError, match="2D weight"):
        q.fake_quantize_nvfp4(torch.zeros(2, 2, 16))
    with pytest.raises(ValueError, match="block_size=32"):
        q.fake_quantize_mxfp4(w, block_size=16)
    with pytest.raises(ValueError, match="divisible by 32"):
        q.fake_quantize_mxfp4_activation(torch.zeros(4, 33))
    with pytest.raises(ValueError, match="divisible by 16"):
        q.quantize_nvfp4(torch.zeros(2, 40))
    with pytest.raises(ValueError, match="divisible"):
        q.quantize_mxfp4(torch.zeros(2, 40))
    with pytest.raises(ValueError, match="divisible by 256"):
        q.quantize_q4_k(torch.zeros(2, 300))
    with pytest.raises(ValueError, match="divisible by 256"):
        q.Q4KLinear.from_linear(nn.Linear(300, 4))
    with pytest.raises(ValueError, match="Unknown Q4_K method"):
        q.fake_quantize_q4_k(torch.zeros(2, 256), method="kmeans")
    with pytest.raises(ValueError, match="2D uint8"):
        q.unpack_e2m1_rows(torch.zeros(2, 2))


def test_meta_tensors_pass_through():
    m = torch.empty(8, 32, device="meta")
    assert q.fake_quantize_nvfp4(m) is m
    assert q.fake_quantize_mxfp4(m) is m
    assert q.fake_quantize_q4_k(torch.empty(8, 256, device="meta")) is not None
    with pytest.raises(ValueError, match="meta"):
        q.quantize_nvfp4(m)


def test_cpu_tensors_fail_loudly_instead_of_falling_back():
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        q.fake_quantize_nvfp4(torch.randn(4, 32))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        q.fake_quantize_mxfp4(torch.randn(4, 32))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        q.quantize_q4_k(torch.randn(4, 256), method="minmax")


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.self_attn = nn.Module()
        for n, o in (("q_proj", 64), ("k_proj", 32), ("v_proj", 32), ("o_proj", 64)):
            setattr(self.self_attn, n, nn.Linear(64, o, bias=False))
        self.mlp = nn.Module()
        self.mlp.gate_proj = nn.Linear(64, 128, bias=False)
        self.mlp.up_proj = nn.Linear(64, 128, bias=False)
        self.mlp.down_proj = nn.Linear(128, 64, bias=False)
        self.norm = nn.LayerNorm(64)


class _Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.config = None
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([_Block(), _Block()])
        self.lm_head = nn.Linear(64, 100, bias=False)


TARGETS = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def test_apply_fake_quant_swaps_targets_and_freezes_the_rest():
    model = _Tiny()
    keys = set(model.state_dict())
    converted = q.apply_fake_quant(model, TARGETS, quant_format="nvfp4", fused_runtime_scales=True)
    assert set(model.state_dict()) == keys
    assert len(converted) == 14
    assert isinstance(model.model.layers[0].self_attn.q_proj, q.NVFP4Linear)
    assert not isinstance(model.lm_head, q.NVFP4Linear)
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert trainable == {f"{n}.weight" for n in converted}
    groups = model._nvfp4_amax_groups
    assert len(groups) == 2 * 4  # qkv, o, gate/up, down per layer
    assert all(m._amax_group is not None for g in groups for m in g.members)


def test_apply_fake_quant_format_checks():
    with pytest.raises(ValueError, match="requires fused_runtime_scales"):
        q.apply_fake_quant(_Tiny(), TARGETS, quant_format="nvfp4", quantize_activations=True)
    with pytest.raises(ValueError, match="does not support input-activation"):
        q.apply_fake_quant(_Tiny(), ["gate_proj"], quant_format="q4_k", quantize_activations=True)
    with pytest.raises(ValueError, match="does not support fused_runtime_scales"):
        q.apply_fake_quant(_Tiny(), TARGETS, quant_format="mxfp4", fused_runtime_scales=True)
    model = _Tiny()
    q.apply_fake_quant(model, ["gate_proj", "up_proj", "down_proj"], quant_format="mxfp4", quantize_activations=True)
    flagged = [m for m in model.modules() if isinstance(m, q.MXFP4Linear)]
    assert len(flagged) == 6 and all(m._quantize_activations for m in flagged)


def test_linear_state_dict_keys_are_unchanged():
    lin = nn.Linear(32, 8, bias=True)
    for cls in (q.NVFP4Linear, q.MXFP4Linear):
        conv = cls.from_linear(lin)
        assert set(conv.state_dict()) == {"weight", "bias"}
        assert conv.weight is lin.weight
    conv = q.Q4KLinear.from_linear(nn.Linear(256, 4), method="minmax")
    assert set(conv.state_dict()) == {"weight", "bias"} and conv.quant_method == "minmax"


def test_v_head_reorder_perm():
    assert q.v_head_reorder_perm(num_k_heads=2, num_v_per_k=3, head_dim=1).tolist() == [0, 3, 1, 4, 2, 5]


def test_runtime_state_roundtrip_on_cpu_state():
    model = _Tiny()
    q.apply_fake_quant(model, TARGETS, quant_format="nvfp4", fused_runtime_scales=True)
    for m in model.modules():
        if isinstance(m, q.NVFP4Linear):
            m._input_amax = torch.tensor(3.5)
    state = q.nvfp4_runtime_state_dict(model)
    fresh = _Tiny()
    q.apply_fake_quant(fresh, TARGETS, quant_format="nvfp4", fused_runtime_scales=True)
    q.load_nvfp4_runtime_state_dict(fresh, state)
    for m in fresh.modules():
        if isinstance(m, q.NVFP4Linear):
            assert float(m._input_amax) == 3.5 and float(m._input_amax_static) == 3.5
    with pytest.raises(ValueError, match="version"):
        q.load_nvfp4_runtime_state_dict(fresh, {"version": 2})


def test_stream_rows_validates_shapes_on_the_host():
    from qatfactory_b200.host_stream import stream_rows

    with pytest.raises(ValueError):
        stream_rows(lambda c: c, torch.zeros(8), torch.zeros(8))
    with pytest.raises(ValueError):
        stream_rows(lambda c: c, torch.zeros(8, 4), torch.zeros(6, 4))


def test_expert_fake_quant_rejects_bad_shapes_like_the_reference():
    """test_nvfp4_moe.py:72-81: errors are raised before any kernel."""

    from qatfactory_b200.quant import fake_quantize_nvfp4_experts

    gate_up = torch.randn(4, 32, 32)
    with pytest.raises(ValueError, match="3D"):
        fake_quantize_nvfp4_experts(gate_up[0], gate_up.abs().amax(dim=(1, 2)))
    with pytest.raises(ValueError, match="shape"):
        fake_quantize_nvfp4_experts(gate_up, torch.ones(2))
    with pytest.raises(ValueError, match="divisible"):
        fake_quantize_nvfp4_experts(torch.randn(2, 4, 24), torch.ones(2))
    meta = torch.empty(4, 32, 32, device="meta")
    assert fake_quantize_nvfp4_experts(meta, torch.ones(4)) is meta


def test_is_fused_experts():
    from torch import nn

    from qatfactory_b200.quant import is_fused_experts

    m = nn.Module()
    m.gate_up_proj = nn.Parameter(torch.zeros(4, 32, 16))
    m.down_proj = nn.Parameter(torch.zeros(4, 16, 16))
    assert is_fused_experts(m)
    m.down_proj = nn.Parameter(torch.zeros(4, 16, 8))
    assert not is_fused_experts(m)


def _tiny_moe():
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    cfg = Qwen3MoeConfig(hidden_size=64, intermediate_size=128, moe_intermediate_size=32, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=16, num_experts=8,
                         num_experts_per_tok=2, vocab_size=128)
    return Qwen3MoeForCausalLM(cfg)


def test_apply_fake_quant_converts_fused_routed_experts():
    """MoE backbones: every fused experts module becomes a full-parameter NVFP4Experts whose two
    3-D latents train, next to the quantized attention linears (fake_quant.py:255-275)."""

    from qatfactory_b200.quant import NVFP4Experts, apply_fake_quant

    model = _tiny_moe()
    converted = apply_fake_quant(model, ("q_proj", "k_proj", "v_proj", "o_proj"), quant_format="nvfp4",
                                 fused_runtime_scales=True)
    experts = [n for n, m in model.named_modules() if isinstance(m, NVFP4Experts)]
    assert experts == ["model.layers.0.mlp.experts", "model.layers.1.mlp.experts"]
    assert converted.experts == tuple(experts)
    assert len(converted.expert_targets) == 2 * 8 * 3
    assert "model.layers.1.mlp.experts.7.w2" in converted.expert_targets
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert "model.layers.0.mlp.experts.gate_up_proj" in trainable
    assert "model.layers.0.mlp.gate.weight" not in trainable  # the router stays frozen
    assert all(m._track_input_amax for m in model.modules() if isinstance(m, NVFP4Experts))


def test_apply_fake_quant_lora_on_fused_experts():
    """LoRA-QAD of an MoE backbone: fused experts become NVFP4ExpertLoRA with a frozen base and
    only the four adapter factors training (hybrid-shared shapes by default), next to LoRA
    attention linears (fake_quant.py:264-272, nvfp4_experts.py:73-135)."""

    from qatfactory_b200.quant import NVFP4ExpertLoRA, apply_fake_quant

    model = _tiny_moe()
    converted = apply_fake_quant(model, ("q_proj",), quant_format="nvfp4", lora_rank=4, lora_alpha=8.0)
    experts = [m for m in model.modules() if isinstance(m, NVFP4ExpertLoRA)]
    assert len(experts) == 2 and converted.lora
    e = experts[0]
    assert tuple(e.gate_up_lora_A.shape) == (2, 4, e.hidden_dim)
    assert tuple(e.gate_up_lora_B.shape) == (e.num_experts, 2, e.intermediate_dim, 4)
    assert tuple(e.down_lora_A.shape) == (e.num_experts, 4, e.intermediate_dim)
    assert tuple(e.down_lora_B.shape) == (e.hidden_dim, 4)
    assert not e.gate_up_proj.requires_grad and not e.down_proj.requires_grad
    assert bool((e.gate_up_lora_B == 0).all()) and bool((e.down_lora_B == 0).all())
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert "model.layers.0.mlp.experts.down_lora_A" in trainable
    assert "model.layers.0.mlp.experts.gate_up_proj" not in trainable
    assert trainable == converted.trainable_parameters
    with torch.no_grad():  # merged weights: the base while B is zero
        assert torch.equal(e.effective_down(3), e.down_proj[3])
    assert e.merged_projection(0, "w1").shape == (e.intermediate_dim, e.hidden_dim)


def test_expert_lora_per_expert_factors_and_fp8_checks():
    from qatfactory_b200.quant import NVFP4ExpertLoRA

    src = _tiny_moe().model.layers[0].mlp.experts
    e = NVFP4ExpertLoRA(src, 2, 4.0, hybrid_shared=False)
    assert tuple(e.gate_up_lora_A.shape) == (e.num_experts, 2, 2, e.hidden_dim)
    assert tuple(e.down_lora_B.shape) == (e.num_experts, e.hidden_dim, 2)
    assert not e.is_fp8_base
    with pytest.raises(ValueError, match="rank must be positive"):
        NVFP4ExpertLoRA(src, 0, 1.0)
    src.gate_up_proj = nn.Parameter(src.gate_up_proj.detach().to(torch.float8_e4m3fn), requires_grad=False)
    src.down_proj = nn.Parameter(src.down_proj.detach().to(torch.float8_e4m3fn), requires_grad=False)
    with pytest.raises(ValueError, match="missing their per-block scales"):
        NVFP4ExpertLoRA(src, 2, 4.0)


def test_fp8_linear_conversion_keeps_the_codes_frozen():
    from qatfactory_b200.quant import NVFP4Linear, dequantize_fp8_blocks, is_fp8_linear

    lin = nn.Linear(256, 128, bias=False)
    lin.weight = nn.Parameter(lin.weight.detach().to(torch.float8_e4m3fn), requires_grad=False)
    lin.weight_scale_inv = torch.rand(1, 2) + 0.5
    assert is_fp8_linear(lin)
    q_lin = NVFP4Linear.from_fp8_linear(lin)
    assert q_lin.weight.dtype == torch.float8_e4m3fn and not q_lin.weight.requires_grad
    assert "_fp8_scale_inv" not in q_lin.state_dict()  # a non-persistent buffer
    with pytest.raises(ValueError, match="not divisible"):
        dequantize_fp8_blocks(lin.weight, torch.ones(3, 2))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        q_lin.base_weight()  # no CPU path


def test_quantized_gather_host_logic(monkeypatch):
    """NVFP4QuantizedGather without a GPU: which parameters train, and the gradient hand-over
    (the STE kernel faked on the host by the mask it would apply)."""

    model = _Tiny()
    model.float()
    q.apply_fake_quant(model, TARGETS, quant_format="nvfp4", fused_runtime_scales=True)
    gather = q.NVFP4QuantizedGather(model)
    assert len(gather.members) == 14
    latents = gather.parameters()
    assert all(isinstance(p, nn.Parameter) and p.requires_grad for p in latents)
    assert {id(p) for p in gather.other_parameters(model)}.isdisjoint({id(m.weight) for m in gather.members})
    assert not any(n.endswith("_latent_shard") for n, _ in model.named_parameters())  # not registered
    assert set(gather.latent_state_dict()) == {f"{n}.weight" for n in gather.names}

    from qatfactory_b200 import _native

    def fake_ste(grad, mask_bits, out=None):
        out = grad if out is None else out
        out.mul_(0.5)
        return out

    monkeypatch.setattr(_native, "ste_backward", fake_ste)
    m = gather.members[0]
    m.weight.grad = torch.ones_like(m.weight)
    gather.gradients_to_latents()
    assert m.weight.grad is None
    assert torch.equal(m._latent_shard.grad, torch.full_like(m.weight, 0.5))
    with pytest.raises(RuntimeError, match="refresh the fused-family weight amax"):
        gather.requantize()


def test_quantized_gather_rejects_w4a4_and_lora():
    model = _Tiny()
    model.float()
    q.apply_fake_quant(model, TARGETS, quant_format="nvfp4", fused_runtime_scales=True)
    model.model.layers[0].self_attn.q_proj._quantize_activations = True
    with pytest.raises(ValueError, match="full-parameter W4A16"):
        q.NVFP4QuantizedGather(model)


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
@pytest.mark.parametrize("rows,k,n", [(7, 48, 40), (200, 4128, 1000), (256, 512, 768)])
def test_w4a4_padding_onto_the_gemm_tiles(fmt, rows, k, n, monkeypatch):
    """The W4A4 autograd functions zero-pad token rows to 128 and in/out features to 256 before
    the operand passes, hand the backward GEMMs dY padded the same way, and slice every result
    back to the caller's shapes (the kernels are replaced by recording fakes here)."""

    from qatfactory_b200 import _native
    from qatfactory_b200.quant.formats import mxfp4 as mx
    from qatfactory_b200.quant.formats import nvfp4 as nv

    seen = {}
    mp, kp, np_ = -(-rows // 128) * 128, -(-k // 256) * 256, -(-n // 256) * 256

    def operand(x, *args, **kwargs):
        role = args[1] if fmt == "nvfp4" else args[0]
        seen[role] = x.clone()
        r, c = x.shape
        return (torch.zeros(r, c // 2, dtype=torch.uint8), torch.zeros(1, dtype=torch.uint8), x.clone(),
                torch.zeros(1, dtype=torch.uint8))

    def gemm(cx, sx, *rest):
        return torch.full((cx.shape[0], rest[-3].shape[0] if fmt == "nvfp4" else rest[0].shape[0]), 2.0,
                          dtype=torch.bfloat16)

    def bf16_gemm(a, a_layout, b, b_layout, mask=None, split_k=True):
        seen.setdefault("dy", a.clone())
        m_out = a.shape[0] if a_layout == _native.K_MAJOR else a.shape[1]
        n_out = b.shape[1] if b_layout == _native.MN_MAJOR else b.shape[0]
        return torch.ones(m_out, n_out, dtype=torch.bfloat16)

    if fmt == "nvfp4":
        monkeypatch.setattr(_native, "nvfp4_operand", operand)
        monkeypatch.setattr(_native, "nvfp4_gemm", gemm)
        fn = lambda x, w: nv._W4A4Linear.apply(x, w, torch.tensor(1.0), torch.tensor(1.0))  # noqa: E731
    else:
        monkeypatch.setattr(_native, "mxfp4_operand", operand)
        monkeypatch.setattr(_native, "mxfp4_gemm", gemm)
        fn = mx._MXFP4W4A4Linear.apply
    monkeypatch.setattr(_native, "bf16_gemm", bf16_gemm)

    g = torch.Generator().manual_seed(rows + k + n)
    x = torch.randn(rows, k, generator=g).to(torch.bfloat16).requires_grad_(True)
    w = torch.randn(n, k, generator=g).to(torch.bfloat16).requires_grad_(True)
    y = fn(x, w)
    assert y.shape == (rows, n) and bool((y == 2.0).all())
    xs, ws = seen[_native.OPERAND_A], seen[_native.OPERAND_B]
    assert xs.shape == (mp, kp) and ws.shape == (np_, kp)
    assert torch.equal(xs[:rows, :k], x.detach()) and torch.equal(ws[:n, :k], w.detach())
    assert int(xs.count_nonzero()) == int(x.detach().count_nonzero())  # the padding is zeros
    assert int(ws.count_nonzero()) == int(w.detach().count_nonzero())
    dy = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    y.backward(dy)
    assert seen["dy"].shape == (mp, np_) and torch.equal(seen["dy"][:rows, :n], dy)
    assert int(seen["dy"].count_nonzero()) == int(dy.count_nonzero())
    assert x.grad.shape == (rows, k) and w.grad.shape == (n, k)


def test_fake_quant_asks_for_the_ste_mask_only_when_a_gradient_is_needed(monkeypatch):
    """Without a gradient to propagate (weight not requiring grad, or under no_grad) the public
    fake quantizers request no STE mask and return the quantized tensor itself; with one, they
    request the mask and wrap the result in the straight-through node."""

    from qatfactory_b200 import _native
    from qatfactory_b200.quant.formats import mxfp4 as mx
    from qatfactory_b200.quant.formats import nvfp4 as nv

    asked = []

    def fake_nv(x, amax_scratch=None, want_mask=True):
        asked.append(want_mask)
        return x.clone(), (torch.zeros(x.numel() // 8, dtype=torch.uint8) if want_mask else None), None

    def fake_mx(x, want_mask=True):
        asked.append(want_mask)
        return x.clone(), (torch.zeros(x.numel() // 8, dtype=torch.uint8) if want_mask else None)

    monkeypatch.setattr(_native, "nvfp4_fake_quant", fake_nv)
    monkeypatch.setattr(_native, "mxfp4_qdq_even", fake_mx)
    for fq in (nv.fake_quantize_nvfp4, mx.fake_quantize_mxfp4):
        asked.clear()
        w = torch.randn(4, 64).to(torch.bfloat16)
        y = fq(w)
        assert asked == [False] and y.grad_fn is None
        wg = w.clone().requires_grad_(True)
        with torch.no_grad():
            y = fq(wg)
        assert asked == [False, False] and y.grad_fn is None
        y = fq(wg)
        assert asked == [False, False, True] and y.grad_fn is not None
