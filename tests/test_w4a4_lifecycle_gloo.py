"""The W4A4 input-scale lifecycle across two ``gloo`` ranks (nvfp4.py:361-397, :285-319,
bootstrap :636-644): the bootstrap static scale, the committed running maxima and the
finalized fused-family input scales are the MAX over ranks, identical on every rank.  The
library's entry points are replaced by the CPU oracle (as in test_qad_harness.py)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.test_qad_harness import _oracle_native, _tiny

TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def _rank_main(rank: int, world: int, port: int, results):
    import torch.distributed as dist
    from transformers import Qwen3ForCausalLM

    from qatfactory_b200.quant import (apply_fake_quant, commit_nvfp4_input_scales, finalize_nvfp4_input_scales,
                                       refresh_nvfp4_weight_amax)
    from qatfactory_b200.quant.formats.nvfp4 import NVFP4Linear

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mp_ = pytest.MonkeyPatch()
        _oracle_native(mp_)
        torch.manual_seed(0)  # same weights on both ranks
        model = Qwen3ForCausalLM(_tiny()).to(torch.bfloat16)
        apply_fake_quant(model, TARGETS, quant_format="nvfp4", fused_runtime_scales=True, quantize_activations=True)
        refresh_nvfp4_weight_amax(model)
        for m in model.modules():
            if isinstance(m, NVFP4Linear):
                m._track_input_amax = True
        model.train()
        g = torch.Generator().manual_seed(100 + rank)  # different data per rank
        with torch.no_grad():
            model(input_ids=torch.randint(0, 256, (1, 16), generator=g))
        boot = {n: float(m._input_amax_static) for n, m in model.named_modules() if isinstance(m, NVFP4Linear)}
        local_running = {n: float(m._input_amax) for n, m in model.named_modules() if isinstance(m, NVFP4Linear)}
        with torch.no_grad():
            model(input_ids=torch.randint(0, 256, (1, 16), generator=g) * (rank + 1) % 256)
        local_running2 = {n: float(m._input_amax) for n, m in model.named_modules() if isinstance(m, NVFP4Linear)}
        commit_nvfp4_input_scales(model)
        committed = {n: float(m._input_amax_static) for n, m in model.named_modules() if isinstance(m, NVFP4Linear)}
        scales = {k: float(v) for k, v in finalize_nvfp4_input_scales(model).items()}
        results[rank] = (boot, local_running, local_running2, committed, scales)
        mp_.undo()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_w4a4_input_scales_are_reduced_across_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_rank_main, args=(2, _free_port(), results), nprocs=2, join=True, start_method="spawn")
        res = dict(results)
    (boot0, run0, run0b, com0, sc0), (boot1, run1, run1b, com1, sc1) = res[0], res[1]
    assert boot0 == boot1  # bootstrap all-reduced in the first forward
    for name in boot0:
        # committed static scale = MAX over ranks of each rank's running maximum
        assert com0[name] == com1[name] == max(run0b[name], run1b[name])
    assert sc0 == sc1 and len(sc0) > 0
    for key, value in sc0.items():
        assert value > 0
    # a fused family shares one scale: q, k and v of layer 0
    q = sc0["model.layers.0.self_attn.q_proj.input_scale"]
    assert q == sc0["model.layers.0.self_attn.k_proj.input_scale"] == sc0["model.layers.0.self_attn.v_proj.input_scale"]
