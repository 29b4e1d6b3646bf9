"""Generate the golden fixtures from the REFERENCE implementation itself.

Run in a container where the reference checkout is importable (it is not present on the
GPU hosts, which only read the committed fixtures):

    python tests/golden/make_golden.py --reference /path/to/QATFactory

It records, for seeded inputs and for the known-answer inputs of the reference's own tests
(tests/quant/test_nvfp4.py, test_mxfp4.py, test_q4_k.py, test_fp4_triton.py), the outputs of
the reference's PyTorch CPU functions:

    _fake_quantize_nvfp4_torch, quantize_nvfp4, dequantize_nvfp4   (formats/nvfp4.py)
    _fake_quantize_mxfp4_torch, _fake_quantize_mxfp4_activation_torch,
    quantize_mxfp4, dequantize_mxfp4                                (formats/mxfp4.py)
    quantize_q4_k, _encode_superblocks_torch, dequantize_q4_k      (formats/q4_k.py)
    the STE backward through fake_quantize_nvfp4 / fake_quantize_mxfp4 autograd

Small cases are stored whole (``fp4_golden.npz``, ``q4k_golden.npz``); the full-size
benchmark configurations are stored as SHA-256 digests of the output bytes
(``digests.json``), so a GPU run can be pinned at full size without shipping the data.

The Q4_K grid search sums 32 floats per sub-block in torch-CPU's vectorised order; the
script first checks that this host sums in the 8-lane order the oracle restates and stops
if it does not.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.fixtures import save_cases  # noqa: E402
from qatfactory_b200 import workloads  # noqa: E402

DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def _digest(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous().reshape(-1)
    if t.dtype == torch.bool:
        t = t.to(torch.uint8)
    return hashlib.sha256(t.view(torch.uint8).numpy().tobytes()).hexdigest()


def _check_sum_order() -> None:
    """The 8-lane order t[k] = ((x[k]+x[k+8])+x[k+16])+x[k+24]; sum t sequentially."""

    g = torch.Generator().manual_seed(123)
    a = torch.randn(4096, 32, generator=g) * torch.exp(torch.randn(4096, 32, generator=g) * 3)
    got = a.sum(dim=-1)
    t = ((a[:, 0:8] + a[:, 8:16]) + a[:, 16:24]) + a[:, 24:32]
    acc = torch.zeros(a.shape[0])
    for k in range(8):
        acc = acc + t[:, k]
    if not torch.equal(acc, got):
        raise SystemExit("this host's torch sums 32 floats in a different order; regenerate elsewhere")


def fp4_cases(R, M) -> dict:
    cases = {}

    def qdq_nv(name, x, amax=None):
        amax_t = None if amax is None else torch.tensor(float(amax), dtype=torch.float32)
        y, mask = R._fake_quantize_nvfp4_torch(x, tensor_amax=amax_t)
        used = float(x.float().abs().amax()) if amax is None else float(amax)
        if used == 0.0:
            # the public API's zero-amax branch (nvfp4.py:540-543)
            y = torch.zeros_like(x)
            mask = torch.ones_like(x, dtype=torch.bool)
        cases[f"nvfp4_qdq/{name}"] = {"x": x, "amax": used, "y": y, "mask": mask}

    def qdq_mx(name, x):
        y, mask = M._fake_quantize_mxfp4_torch(x)
        cases[f"mxfp4_even/{name}"] = {"x": x, "y": y, "mask": mask}

    def qdq_ceil(name, x):
        y, _ = M._fake_quantize_mxfp4_activation_torch(x)
        cases[f"mxfp4_ceil/{name}"] = {"x": x, "y": y}

    # random tensors, test_fp4_triton.py:55-69 (shapes reduced)
    for dtype in DTYPES:
        for mag in (1e-4, 1.0, 1e4):
            g = torch.Generator().manual_seed(10)
            x = (torch.randn(17, 256, generator=g) * mag).to(dtype)
            tag = f"rand_{str(dtype)[6:]}_{mag:g}"
            qdq_nv(tag, x)
            qdq_nv(tag + "_amax125", x, float(x.float().abs().amax()) * 1.25)
            qdq_mx(tag, x)
            qdq_ceil(tag, x)
    # padding and tiny shapes, test_fp4_triton.py:88-103
    for dtype in DTYPES:
        for shape in ((9, 100), (5, 24), (1, 16), (1, 32), (3, 48), (2, 17), (4, 40)):
            g = torch.Generator().manual_seed(shape[0] * shape[1])
            x = torch.randn(shape, generator=g).to(dtype)
            tag = f"pad_{str(dtype)[6:]}_{shape[0]}x{shape[1]}"
            qdq_nv(tag, x)
            qdq_mx(tag, x)
    # E2M1 ties and signed zero, test_fp4_triton.py:124-141
    bounds = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    ties = torch.cat((bounds, -bounds))
    for dtype in DTYPES:
        nv = torch.zeros(1, 32)
        nv[0, : ties.numel()] = ties
        nv[0, 14] = -0.0
        nv[0, 15] = 6.0
        qdq_nv(f"ties_{str(dtype)[6:]}", nv.to(dtype), 2688.0)
        mx = torch.zeros(1, 32)
        mx[0, : ties.numel()] = ties
        mx[0, 14] = -0.0
        mx[0, -1] = 5.0
        qdq_mx(f"ties_{str(dtype)[6:]}", mx.to(dtype))
        # zero blocks and single huge elements, test_fp4_triton.py:144-152
        zb = torch.zeros(3, 64)
        zb[0, 0] = 1e4
        zb[1, 31] = -1e4
        zb[2, 32:] = torch.linspace(-4.0, 4.0, 32)
        qdq_nv(f"zeroblocks_{str(dtype)[6:]}", zb.to(dtype))
        qdq_mx(f"zeroblocks_{str(dtype)[6:]}", zb.to(dtype))
    # fp32 subnormals, test_fp4_triton.py:155-159
    sub = torch.full((3, 32), 1e-40)
    sub[1].neg_()
    qdq_nv("subnormal_f32", sub)
    qdq_mx("subnormal_f32", sub)
    # E4M3 subnormal scale rounding, test_fp4_triton.py:162-172
    e4 = torch.zeros(1, 64)
    e4.view(4, 16)[:, 0] = torch.tensor([0.5, 1.0, 1.5, 2.5]) * (2.0**-9) * 6.0
    qdq_nv("e4m3_subnormal", e4, 2688.0)
    # known answers, test_nvfp4.py:35-73
    qdq_nv("known_values", torch.tensor([[0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0] * 2]))
    sv = torch.zeros(1, 32)
    sv[0, 0] = 2688.0
    sv[0, 16:] = 0.003
    qdq_nv("e4m3_subnormal_block", sv)
    sat = torch.zeros(1, 32)
    sat[0, 0] = 2688.0
    sat[0, 16] = 5.8
    qdq_nv("saturation_mask", sat)
    qdq_nv("zero_weight", torch.zeros(2, 17))
    qdq_nv("zero_amax_nonzero_tensor", torch.randn(2, 32, generator=torch.Generator().manual_seed(5)), 0.0)
    # W4A4 activation saturating beyond the static scale, test_nvfp4.py:363-374
    act = torch.zeros(1, 16)
    act[0, 0] = 8.0
    act[0, 1] = 1.0
    qdq_nv("static_scale_saturation", act, 6.0)
    # MXFP4 EVEN regions, test_mxfp4.py:44-63 and the clip mask :105-119
    for name, vals in (("exact", {0: 1.5, 1: 0.5}), ("clipped", {0: 1.6875}), ("promoted", {0: 1.75}),
                       ("clip_mask", {0: 1.6875, 1: 0.9})):
        w = torch.zeros(1, 32)
        for k, v in vals.items():
            w[0, k] = v
        qdq_mx(f"even_{name}", w)
        qdq_mx(f"even_{name}_bf16", w.to(torch.bfloat16))
    qdq_mx("known_values", torch.tensor([[0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0] * 4]))
    # MXFP4 CEIL boundaries and zero/tiny blocks, test_fp4_triton.py:185-206, test_mxfp4.py:323-354
    cb = torch.zeros(4, 32)
    cb[:, 0] = torch.tensor([1.5, 3.0, 6.0, 100.0])
    qdq_ceil("boundaries", cb)
    za = torch.zeros(6, 64)
    za[0, 32] = 1e-30
    za[1, 0] = 1e-38
    za[2, 5] = 0.85
    za[2, 6] = 0.4
    za[3, :] = torch.linspace(-7.0, 7.0, 64)
    qdq_ceil("zero_tiny", za)
    qdq_ceil("zero_tiny_bf16", za.to(torch.bfloat16))
    # huge magnitudes (E8M0 clamp at 2^127 / 2^-127)
    huge = torch.zeros(2, 32)
    huge[0, 0] = 3.0e38
    huge[1, 0] = 1e-38
    qdq_mx("extreme", huge)
    qdq_ceil("extreme", huge)

    # packing: quantize_nvfp4 / quantize_mxfp4 + dequantize (test_nvfp4.py:94-123, test_mxfp4.py:135-147)
    for dtype in DTYPES:
        g = torch.Generator().manual_seed(7)
        x = (torch.randn(16, 256, generator=g) * 0.05).to(dtype)
        tag = str(dtype)[6:]
        for amax_mode in ("own", "shared"):
            amax = None if amax_mode == "own" else torch.tensor(float(x.float().abs().amax()) * 1.7)
            r = R.quantize_nvfp4(x, tensor_amax=amax)
            dq = R.dequantize_nvfp4(r.packed_weight, r.weight_scale, r.weight_scale_2)
            used = float(x.float().abs().amax()) if amax is None else float(amax)
            cases[f"nvfp4_pack/{tag}_{amax_mode}"] = {
                "x": x, "amax": used, "packed": r.packed_weight, "scales": r.weight_scale,
                "scale_2": r.weight_scale_2, "recon": r.reconstruction, "dequant": dq,
            }
        r = M.quantize_mxfp4(x)
        cases[f"mxfp4_pack/{tag}"] = {
            "x": x, "packed": r.packed_weight, "scales": r.weight_scale, "recon": r.reconstruction,
            "dequant": M.dequantize_mxfp4(r.packed_weight, r.weight_scale),
        }
    zr = R.quantize_nvfp4(torch.zeros(2, 32, dtype=torch.bfloat16))
    cases["nvfp4_pack/zero"] = {
        "x": torch.zeros(2, 32, dtype=torch.bfloat16), "amax": 0.0, "packed": zr.packed_weight,
        "scales": zr.weight_scale, "scale_2": zr.weight_scale_2, "recon": zr.reconstruction,
        "dequant": R.dequantize_nvfp4(zr.packed_weight, zr.weight_scale, zr.weight_scale_2),
    }
    zm = M.quantize_mxfp4(torch.zeros(2, 64, dtype=torch.bfloat16))
    cases["mxfp4_pack/zero"] = {
        "x": torch.zeros(2, 64, dtype=torch.bfloat16), "packed": zm.packed_weight, "scales": zm.weight_scale,
        "recon": zm.reconstruction, "dequant": M.dequantize_mxfp4(zm.packed_weight, zm.weight_scale),
    }
    cases["e2m1_pack/known"] = {
        "nibbles": torch.tensor([[0x1, 0xA, 0x7, 0xF]], dtype=torch.uint8),
        "packed": R.pack_e2m1_rows(torch.tensor([[0x1, 0xA, 0x7, 0xF]], dtype=torch.uint8)),
    }

    # STE backward through the public autograd path (nvfp4.py:32-41, :550)
    for dtype in (torch.bfloat16, torch.float32):
        g = torch.Generator().manual_seed(13)
        src = torch.randn(4, 96, generator=g).to(dtype)
        src[0, 0] = 1e4  # forces saturation masks in that block
        up = torch.randn(4, 96, generator=g).to(dtype)
        up[1, 3] = -0.0
        for fmt, fn, extra in (("nvfp4", R.fake_quantize_nvfp4, {"tensor_amax": torch.tensor(float(src.float().abs().amax()) * 0.5)}),
                               ("mxfp4", M.fake_quantize_mxfp4, {})):
            leaf = src.clone().requires_grad_()
            out = fn(leaf, **extra)
            out.backward(up)
            cases[f"ste/{fmt}_{str(dtype)[6:]}"] = {"x": src, "grad_out": up, "y": out.detach(), "grad_in": leaf.grad}
    return cases


def q4k_cases(Q) -> dict:
    cases = {}

    def enc(name, x, method):
        r = Q.quantize_q4_k(x, method=method)
        e = Q._encode_superblocks_torch(Q._as_superblocks(x), method=method)
        cases[f"q4k/{name}_{method}"] = {
            "x": x, "method": method, "blocks": r.packed_weight, "recon": r.reconstruction,
            "mask": e.in_range.reshape(x.shape), "dequant": Q.dequantize_q4_k(r.packed_weight, x.shape[1]),
        }

    for method in ("minmax", "grid_search"):
        for dtype, mag, seed in ((torch.bfloat16, 0.1, 0), (torch.bfloat16, 0.02, 1), (torch.float32, 1.0, 2),
                                 (torch.float16, 0.05, 3)):
            g = torch.Generator().manual_seed(seed)
            x = (torch.randn(6, 512, generator=g) * mag).to(dtype)
            enc(f"rand_{str(dtype)[6:]}_{mag:g}", x, method)
        # hand-derived affine (test_q4_k.py:268-278) and degenerate sub-blocks
        kat = torch.tensor([[-0.3] + [0.0] * 30 + [0.6]], dtype=torch.float32).repeat(1, 8)
        enc("affine", kat, method)
        deg = torch.zeros(3, 256)
        deg[1, :] = 0.25  # constant positive: xmax != vmin (vmin clamps to 0)
        deg[2, 32:64] = -0.5  # one all-negative constant sub-block
        deg[2, 100] = 3.0
        enc("degenerate", deg, method)
        heavy = workloads.student_t_outliers((4, 512), seed=99, outlier_seed=98, n_outliers=2, dtype=torch.bfloat16)
        enc("heavy_tail", heavy, method)
        # signed zeros: torch keeps the first of equal extrema, clamp(max=0) keeps -0, and a
        # -0 code survives the reconstruction when a sub-block's min code lm is 0
        enc("all_neg_zero", torch.full((1, 256), -0.0), method)
        enc("mixed_zeros", torch.tensor([[-0.0, 0.0] * 128]), method)
        enc("zeros_then_neg_zero", torch.tensor([[0.0, -0.0] * 128]), method)
        lm0 = torch.zeros(1, 256)
        lm0[0, 0], lm0[0, 1] = -1.0, 1.0
        lm0[0, 32:64] = torch.linspace(-0.001, 0.5, 32)
        lm0[0, 64:96] = torch.linspace(-0.0004, 0.3, 32)
        enc("lm0_negative", lm0, method)
        enc("lm0_negative_bf16", lm0.to(torch.bfloat16), method)
        g = torch.Generator().manual_seed(17)
        pos = torch.rand(2, 512, generator=g)
        pos[0, 40], pos[1, 300], pos[1, 301] = -0.0, 0.0, -0.0
        enc("positive_signed_zeros", pos, method)
        zs = torch.rand(1, 256, generator=g)
        zs[0, 32:64] = 0.0
        zs[0, 35] = -0.0
        enc("positive_zero_subblock", zs.to(torch.bfloat16), method)
    return cases


def digests(R, M, Q) -> dict:
    out = {}
    # configuration 1
    w = workloads.config1_weight()
    grad = workloads.config1_grad()
    amax = w.float().abs().amax()
    y, mask = R._fake_quantize_nvfp4_torch(w, tensor_amax=amax)
    out["config1/nvfp4_qdq/y"] = _digest(y)
    out["config1/nvfp4_qdq/mask"] = _digest(mask)
    out["config1/nvfp4_ste/grad_in"] = _digest(grad * mask)
    r = R.quantize_nvfp4(w)
    out["config1/nvfp4_pack/packed"] = _digest(r.packed_weight)
    out["config1/nvfp4_pack/scales"] = _digest(r.weight_scale.view(torch.uint8))
    out["config1/nvfp4_pack/scale_2"] = _digest(r.weight_scale_2)
    out["config1/amax"] = float(amax)
    # configuration 2
    w2 = workloads.config2_weight()
    y, mask = M._fake_quantize_mxfp4_torch(w2)
    out["config2a/mxfp4_even/y"] = _digest(y)
    out["config2a/mxfp4_even/mask"] = _digest(mask)
    r = M.quantize_mxfp4(w2)
    out["config2a/mxfp4_pack/packed"] = _digest(r.packed_weight)
    out["config2a/mxfp4_pack/scales"] = _digest(r.weight_scale)
    x2 = workloads.config2_activation()
    y, _ = M._fake_quantize_mxfp4_activation_torch(x2)
    out["config2b/mxfp4_ceil/y"] = _digest(y)
    # configuration 3, layer 0.  For grid_search also record the IEEE-arithmetic oracle's
    # digests and its agreement with the reference: the reference's weights use
    # torch.sqrt, which on this host goes through a vector math library that is not
    # correctly rounded (about 0.7% of float32 inputs land one ulp away), so a few
    # super-blocks of the weighted search can end on a different encoding.
    import oracle

    agree = {"weights": 0, "weights_equal": 0, "superblocks": 0, "superblocks_differ": 0}
    for name, wl in workloads.config3_layer(0):
        for method in ("minmax", "grid_search"):
            r = Q.quantize_q4_k(wl, method=method)
            out[f"config3/layer0/{name}/{method}/blocks"] = _digest(r.packed_weight)
            out[f"config3/layer0/{name}/{method}/recon"] = _digest(r.reconstruction)
            if method == "grid_search":
                blocks, recon, _ = oracle.q4k_encode(wl, method)
                out[f"config3/layer0/{name}/{method}/oracle_blocks"] = _digest(blocks)
                out[f"config3/layer0/{name}/{method}/oracle_recon"] = _digest(recon)
                agree["weights"] += wl.numel()
                agree["weights_equal"] += int((recon.view(torch.int16) == r.reconstruction.view(torch.int16)).sum())
                sb_diff = (blocks.reshape(-1, 144) != r.packed_weight.reshape(-1, 144)).any(dim=1)
                agree["superblocks"] += sb_diff.numel()
                agree["superblocks_differ"] += int(sb_diff.sum())
    out["config3/layer0/grid_search/reference_agreement"] = agree
    # configuration 4 operands (static activation amax = bootstrap amax)
    x4, w4, _ = workloads.config4_inputs()
    xa = x4.float().abs().amax()
    y, mask = R._fake_quantize_nvfp4_torch(x4, tensor_amax=xa)
    out["config4/x_qdq/y"] = _digest(y)
    out["config4/x_qdq/mask"] = _digest(mask)
    out["config4/x_amax"] = float(xa)
    y, mask = R._fake_quantize_nvfp4_torch(w4)
    out["config4/w_qdq/y"] = _digest(y)
    out["config4/w_qdq/mask"] = _digest(mask)
    return out


def export_cases(R, M, Q) -> dict:
    """The tensors the reference's exporters and QARL publisher emit for a module, computed with
    the reference's own functions and the field expressions of its call sites:
      compressed-tensors NVFP4 export  (quant/export/nvfp4_vllm.py:709-728): weight_packed,
          weight_scale, weight_global_scale = 1 / weight_scale_2, input_global_scale =
          1 / (input_amax / 2688), after the bit-equal dequantization check;
      NVFP4WeightPublisher.sync        (rl/vllm_nvfp4_sync.py:325-333): the fused family's full
          weights concatenated along dim 0, quantize_nvfp4(..., compute_reconstruction=False);
      compressed-tensors MXFP4 export  (quant/export/mxfp4_vllm.py:251-260);
      Q4_K save-time pack              (trainer/checkpoint.py:366-391): the format's pack hook,
          i.e. quantize_q4_k blocks (q4_k.py:388-408 without reorders)."""

    cases = {}
    g = torch.Generator().manual_seed(61)
    family = [("q_proj", 64), ("k_proj", 32), ("v_proj", 32)]
    ws = [(torch.randn(rows, 256, generator=g) * 0.02).to(torch.bfloat16) for _, rows in family]
    ws[2][5, :16] = 0  # an all-zero block
    amax = torch.stack([w.float().abs().amax() for w in ws]).amax()
    input_amax = torch.tensor(7.25, dtype=torch.float32)
    input_scale = (input_amax / R.NVFP4_SCALE_DENOMINATOR).reshape(())  # finalize_nvfp4_input_scales
    for (name, _), w in zip(family, ws):
        r = R.quantize_nvfp4(w, tensor_amax=amax)
        dq = R.dequantize_nvfp4(r.packed_weight, r.weight_scale, r.weight_scale_2)
        cases[f"nvfp4_export/{name}"] = {
            "weight": w, "tensor_amax": float(amax), "input_amax": float(input_amax),
            "weight_packed": r.packed_weight, "weight_scale": r.weight_scale,
            "weight_global_scale": r.weight_scale_2.reshape(1).float().reciprocal(),
            "input_global_scale": input_scale.reshape(1).reciprocal(),
            "dequant_bit_equal": bool(torch.equal(dq.to(r.reconstruction.dtype), r.reconstruction)),
        }
    fused = torch.cat(ws, dim=0)
    p = R.quantize_nvfp4(fused, tensor_amax=amax, compute_reconstruction=False)
    cases["nvfp4_publish/qkv"] = {
        "weight": fused, "tensor_amax": float(amax), "packed_weight": p.packed_weight,
        "weight_scale": p.weight_scale, "weight_scale_2": p.weight_scale_2,
        "reconstruction_is_none": p.reconstruction is None,
    }
    wm = (torch.randn(96, 512, generator=g) * 0.02).to(torch.bfloat16)
    r = M.quantize_mxfp4(wm)
    cases["mxfp4_export/gate_proj"] = {
        "weight": wm, "weight_packed": r.packed_weight, "weight_scale": r.weight_scale,
        "dequant_bit_equal": bool(torch.equal(M.dequantize_mxfp4(r.packed_weight, r.weight_scale)
                                              .to(r.reconstruction.dtype), r.reconstruction)),
    }
    for name, shape in (("q_proj", (256, 512)), ("down_proj", (128, 1024))):
        wq = (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)
        r = Q.quantize_q4_k(wq, method="minmax")
        cases[f"q4k_pack/{name}"] = {"weight": wq, "blocks": r.packed_weight,
                                     "dequant": Q.dequantize_q4_k(r.packed_weight, shape[1])}
    return cases


def stack_file(part: str) -> Path:
    return HERE / f"config3_stack_{part}.json"


def config3_stack(Q, part: str) -> None:
    """Digests of configuration 3 as configured: every linear of all 36 layers.

    part "minmax": the reference's ``quantize_q4_k(method="minmax")`` blocks and reconstruction
    per tensor (the default Q4_K method; bit-exact target).
    part "grid": the IEEE-arithmetic oracle's grid-search blocks and reconstruction per tensor
    (the GPU's target) and, per layer, the oracle's agreement with the reference's own grid
    search (which differs where torch-CPU's float sqrt is not correctly rounded).
    Each part writes its own file (``config3_stack_minmax.json``, ``config3_stack_grid.json``),
    rewritten after every layer."""

    import oracle

    data = {}
    for layer in range(workloads.QWEN3_8B_LAYERS):
        agree = {"weights": 0, "weights_equal": 0, "superblocks": 0, "superblocks_differ": 0}
        for name, wl in workloads.config3_layer(layer):
            key = f"layer{layer}/{name}"
            if part == "minmax":
                r = Q.quantize_q4_k(wl, method="minmax")
                data[f"{key}/minmax/blocks"] = _digest(r.packed_weight)
                data[f"{key}/minmax/recon"] = _digest(r.reconstruction)
            else:
                blocks, recon, _ = oracle.q4k_encode(wl, "grid_search")
                data[f"{key}/grid_search/oracle_blocks"] = _digest(blocks)
                data[f"{key}/grid_search/oracle_recon"] = _digest(recon)
                r = Q.quantize_q4_k(wl, method="grid_search")
                agree["weights"] += wl.numel()
                agree["weights_equal"] += int((recon.view(torch.int16) == r.reconstruction.view(torch.int16)).sum())
                sb_diff = (blocks.reshape(-1, 144) != r.packed_weight.reshape(-1, 144)).any(dim=1)
                agree["superblocks"] += sb_diff.numel()
                agree["superblocks_differ"] += int(sb_diff.sum())
        if part != "minmax":
            data[f"layer{layer}/grid_search/reference_agreement"] = agree
        print(f"config3 stack {part}: layer {layer} done", flush=True)
        data["__host__"] = {"torch": torch.__version__, "cpu_capability": torch.backends.cpu.get_cpu_capability()}
        stack_file(part).write_text(json.dumps(data, indent=0, sort_keys=True) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--skip-digests", action="store_true")
    ap.add_argument("--export-only", action="store_true", help="only export_golden.npz")
    ap.add_argument("--config3-stack", choices=("minmax", "grid"),
                    help="only the 36-layer configuration-3 digests (one part)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from qatfactory.quant.formats import mxfp4 as M
    from qatfactory.quant.formats import nvfp4 as R
    from qatfactory.quant.formats import q4_k as Q

    sys.path.insert(0, str(HERE.parents[1]))
    torch.set_num_threads(max(1, torch.get_num_threads()))
    _check_sum_order()
    if args.config3_stack:
        config3_stack(Q, args.config3_stack)
        return
    save_cases(HERE / "export_golden.npz", export_cases(R, M, Q))
    if args.export_only:
        return
    save_cases(HERE / "fp4_golden.npz", fp4_cases(R, M))
    save_cases(HERE / "q4k_golden.npz", q4k_cases(Q))
    if not args.skip_digests:
        d = digests(R, M, Q)
        d["__host__"] = {"torch": torch.__version__, "cpu_capability": torch.backends.cpu.get_cpu_capability()}
        (HERE / "digests.json").write_text(json.dumps(d, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
