"""Quantize-before-gather (``quant.NVFP4QuantizedGather``) against the reference's data flow.

* ``qatf_nvfp4_qdq_shadow`` equals ``qatf_nvfp4_qdq`` on the BF16 cast of the FP32 latent,
  widened back to FP32, bit for bit (values, STE mask), including zero, tiny and
  rounding-boundary blocks and a zero tensor amax;
* ``qatf_tensor_amax_update`` is ``torch.maximum(running, x.abs().amax())``;
* the configuration-5 QAD step with the quantized gather takes exactly the same steps as the
  step that fake-quantizes the gathered weight in every forward (FSDP2, gradient checkpointing):
  identical losses and identical FP32 latents after three optimizer steps.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from qatfactory_b200 import _native, qad_step

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _latent(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * 0.02
    x[0, :16] = 0.0  # a zero block
    x[1, 16:32] = 1e-30  # a tiny block: the exact per-element path
    x[2, :16] = torch.tensor([1.0 + 2.0 ** -8 * k for k in range(16)])  # BF16 rounding ties and neighbours
    x[3, :16] = -x[2, :16]
    return x.to(DEV)


@pytest.mark.parametrize("rows,cols", [(64, 256), (384, 4096), (1, 16), (3, 48)])
def test_shadow_qdq_equals_qdq_of_the_bf16_cast(rows, cols):
    x = _latent(max(rows, 4), cols, seed=rows + cols)[:rows].contiguous()
    amax = x.to(torch.bfloat16).float().abs().amax()
    out = torch.empty_like(x)
    mask = torch.empty(_native.mask_nbytes(x.numel()), dtype=torch.uint8, device=DEV)
    _native.nvfp4_qdq_shadow(x, amax, out, mask)
    y, m = _native.nvfp4_qdq(x.to(torch.bfloat16), amax)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int32), y.float().view(torch.int32))
    assert torch.equal(mask, m)


def test_shadow_qdq_zero_amax():
    x = _latent(8, 64, seed=3)
    out = torch.full_like(x, 7.0)
    mask = torch.zeros(_native.mask_nbytes(x.numel()), dtype=torch.uint8, device=DEV)
    _native.nvfp4_qdq_shadow(x, torch.zeros((), device=DEV), out, mask)
    torch.cuda.synchronize()
    assert int(out.count_nonzero()) == 0 and bool((mask == 0xFF).all())


def test_shadow_qdq_rejects_bad_arguments():
    x = _latent(4, 32, seed=1)
    mask = torch.empty(16, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        _native.nvfp4_qdq_shadow(x.to(torch.bfloat16), x.abs().amax(), x, mask)
    with pytest.raises(RuntimeError):  # cols % 16
        _native.nvfp4_qdq_shadow(x[:, :24].contiguous(), x.abs().amax(), torch.empty(4, 24, device=DEV), mask)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_amax_update_is_a_running_maximum(dtype):
    g = torch.Generator().manual_seed(5)
    running = torch.tensor(0.5, device=DEV)
    expect = running.clone()
    for scale in (0.1, 3.0, 1.0):
        x = (torch.randn(1000, 37, generator=g) * scale).to(dtype).to(DEV)
        _native.tensor_amax_update(x, running)
        expect = torch.maximum(expect, x.float().abs().amax())
    torch.cuda.synchronize()
    assert torch.equal(running, expect)
    x = torch.ones(64, device=DEV, dtype=dtype)
    x[7] = float("nan")
    _native.tensor_amax_update(x, running)
    assert bool(torch.isnan(running))


@pytest.fixture(scope="module")
def process_group():
    import torch.distributed as dist

    created = not dist.is_initialized()
    if created:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
            os.environ.pop(key, None)
        qad_step.ensure_process_group(timeout_s=120)
    yield
    if created and dist.is_initialized():  # later tests must not find this module's group
        torch.cuda.synchronize()
        dist.destroy_process_group()


def _config():
    return qad_step.qwen3_config(num_hidden_layers=2, hidden_size=256, num_attention_heads=4, num_key_value_heads=2,
                                 head_dim=64, intermediate_size=512, vocab_size=2048, max_position_embeddings=512)


def _weights(step) -> dict[str, torch.Tensor]:
    """Full FP32 trainable weights: the latents where the step gathers quantized weights."""

    out = {}
    latents = step.gather.latent_state_dict() if step.gather is not None else {}
    for name, p in step.student.named_parameters():
        t = latents.get(name, p)
        out[name] = (t.full_tensor() if hasattr(t, "full_tensor") else t).detach().float().clone()
    return out


def test_quantized_gather_step_is_bit_identical(process_group):
    cfg = _config()
    tokens = [qad_step.synthetic_tokens(cfg.vocab_size, 256, 0, i, DEV) for i in range(3)]
    ref = qad_step.QADStep(cfg, DEV)
    ref_losses = [float(ref(t)) for t in tokens]
    ref_w = _weights(ref)
    del ref
    ours = qad_step.QADStep(cfg, DEV, quantized_gather=True)
    assert len(ours.gather.members) == 2 * 7
    losses = [float(ours(t)) for t in tokens]
    w = _weights(ours)
    torch.cuda.synchronize()
    assert losses == ref_losses, (losses, ref_losses)
    assert set(w) == set(ref_w)
    for name in w:
        assert torch.equal(w[name].view(torch.int32), ref_w[name].view(torch.int32)), name
    # the FSDP parameters hold exactly the quantized latents
    for m in ours.gather.members:
        lat = m._latent_shard.to_local() if hasattr(m._latent_shard, "to_local") else m._latent_shard
        wq = m.weight.to_local() if hasattr(m.weight, "to_local") else m.weight
        y, _ = _native.nvfp4_qdq(lat.detach().to(torch.bfloat16), m._amax_group.tensor_amax())
        assert torch.equal(wq.detach().view(torch.int32), y.float().view(torch.int32))
