"""The on-wire tensors of the reference's exporters and QARL publisher, and the GGUF round trip
of the Q4_K save-time blocks, produced on the GPU kernels.

* ``nvfp4_export_fields`` / ``mxfp4_export_fields`` / ``nvfp4_publish_pack`` / ``q4k_save_blocks``
  against fixtures the reference's own functions produced with the field expressions of its
  call sites (tests/golden/make_golden.py ``export_cases``): names, dtypes, shapes and bytes,
  bit for bit (qatfactory/quant/export/nvfp4_vllm.py:709-728, mxfp4_vllm.py:251-260,
  rl/vllm_nvfp4_sync.py:325-333, trainer/checkpoint.py:366-391).
* The Q4_K blocks written into a GGUF file and read back decode, through gguf's own Q4_K
  dequantizer, to exactly this library's dequantization (the lossless check of
  quant/export/q4_k_gguf.py:304-334), and stay within the splice's closeness bound of the
  source weights (max |diff| <= 0.25 amax, q4_k_gguf.py:59, :269-280).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from qatfactory_b200.quant import dequantize_q4_k
from qatfactory_b200.quant.export_fields import (
    mxfp4_export_fields,
    nvfp4_export_fields,
    nvfp4_publish_pack,
    q4k_save_blocks,
)
from tests.golden.fixtures import GOLDEN_DIR, load_cases

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
CASES = load_cases(GOLDEN_DIR / "export_golden.npz")


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    return (a.dtype == b.dtype and a.shape == b.shape
            and torch.equal(a.reshape(-1).view(torch.uint8), b.reshape(-1).view(torch.uint8)))


@pytest.mark.parametrize("name", ["q_proj", "k_proj", "v_proj"])
def test_nvfp4_export_fields_match_the_reference_exporter(name):
    case = CASES[f"nvfp4_export/{name}"]
    assert case["dequant_bit_equal"]
    fields = nvfp4_export_fields(case["weight"].to(DEV), torch.tensor(case["tensor_amax"], device=DEV),
                                 torch.tensor(case["input_amax"], device=DEV))
    assert set(fields) == {"weight_packed", "weight_scale", "weight_global_scale", "input_global_scale"}
    for key, value in fields.items():
        assert _same(value, case[key]), key


def test_fused_family_shares_one_global_scale():
    scales = {name: nvfp4_export_fields(CASES[f"nvfp4_export/{name}"]["weight"].to(DEV),
                                        torch.tensor(CASES[f"nvfp4_export/{name}"]["tensor_amax"], device=DEV))
              ["weight_global_scale"] for name in ("q_proj", "k_proj", "v_proj")}
    assert torch.equal(scales["q_proj"], scales["k_proj"]) and torch.equal(scales["q_proj"], scales["v_proj"])


def test_publisher_pack_matches_the_reference_publisher():
    case = CASES["nvfp4_publish/qkv"]
    rows = [64, 32, 32]
    members = list(case["weight"].to(DEV).split(rows, dim=0))
    packed = nvfp4_publish_pack(members, torch.tensor(case["tensor_amax"], device=DEV))
    assert case["reconstruction_is_none"] and packed.reconstruction is None
    assert _same(packed.packed_weight, case["packed_weight"])
    assert _same(packed.weight_scale, case["weight_scale"])
    assert _same(packed.weight_scale_2, case["weight_scale_2"])


def test_mxfp4_export_fields_match_the_reference_exporter():
    case = CASES["mxfp4_export/gate_proj"]
    assert case["dequant_bit_equal"]
    fields = mxfp4_export_fields(case["weight"].to(DEV))
    assert set(fields) == {"weight_packed", "weight_scale"}
    for key, value in fields.items():
        assert _same(value, case[key]), key


def test_q4k_blocks_round_trip_through_gguf_losslessly(tmp_path):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import Q4_K

    names = ("q_proj", "down_proj")
    blocks = {}
    for name in names:
        case = CASES[f"q4k_pack/{name}"]
        blocks[name] = q4k_save_blocks(case["weight"].to(DEV))
        assert _same(blocks[name], case["blocks"]), name  # the reference's save-time bytes
    path = tmp_path / "spliced.gguf"
    writer = gguf.GGUFWriter(str(path), "llama")
    for name in names:
        writer.add_tensor(f"blk.0.{name}.weight", blocks[name].numpy(), raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()

    reader = gguf.GGUFReader(str(path))
    tensors = {t.name: t for t in reader.tensors}
    for name in names:
        case = CASES[f"q4k_pack/{name}"]
        out_f, in_f = case["weight"].shape
        t = tensors[f"blk.0.{name}.weight"]
        assert t.tensor_type == gguf.GGMLQuantizationType.Q4_K
        theirs = Q4_K.dequantize_blocks(np.asarray(t.data).reshape(-1, 144)).reshape(out_f, in_f)
        ours = dequantize_q4_k(blocks[name].to(DEV), in_f).cpu().numpy()
        assert float(np.abs(theirs - ours).max()) == 0.0, name
        assert np.array_equal(ours.view(np.uint32), case["dequant"].numpy().view(np.uint32))
        src = case["weight"].float().numpy()
        assert float(np.abs(ours - src).max()) <= 0.25 * float(np.abs(src).max())
