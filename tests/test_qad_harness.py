"""The configuration-5 QAD step harness (qatfactory_b200/qad_step.py) on the CPU.

The loss and FLOP count are checked directly; the FSDP2 step runs as two ``gloo`` ranks with
the library's entry points replaced by the CPU oracle (the CUDA path is exercised by the GPU
tests and the benchmark)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

from qatfactory_b200 import qad_step


def test_distill_loss_is_mean_forward_kl_per_supervised_token():
    g = torch.Generator().manual_seed(0)
    s = torch.randn(2, 7, 11, generator=g)
    t = torch.randn(2, 7, 11, generator=g)
    labels = torch.randint(0, 11, (2, 7), generator=g)
    labels[0, 3] = qad_step.IGNORE_INDEX
    loss = qad_step.distill_loss(s, t, labels, chunk_size=4)
    sl, tl, lab = s[:, :-1].reshape(-1, 11), t[:, :-1].reshape(-1, 11), labels[:, 1:].reshape(-1)
    keep = lab != qad_step.IGNORE_INDEX
    p = F.softmax(tl[keep], -1)
    want = (p * (p.log() - F.log_softmax(sl[keep], -1))).sum() / keep.sum()
    torch.testing.assert_close(loss, want, rtol=1e-5, atol=1e-6)


def test_step_flops_counts_teacher_student_recompute_and_backward():
    cfg = qad_step.qwen3_config(num_hidden_layers=1, hidden_size=8, num_attention_heads=2, num_key_value_heads=1,
                                head_dim=4, intermediate_size=16, vocab_size=32)
    seq = 5
    per_layer = 8 * 8 + 2 * 8 * 4 + 8 * 8 + 3 * 8 * 16
    layer = 2 * seq * per_layer + 2 * seq * seq * 8
    fwd = layer + 2 * seq * 8 * 32
    assert qad_step.step_flops(cfg, seq) == 4 * fwd + layer
    assert qad_step.step_flops(cfg, seq, gradient_checkpointing=False) == 4 * fwd


def _tiny():
    return qad_step.qwen3_config(num_hidden_layers=2, hidden_size=64, num_attention_heads=4, num_key_value_heads=2,
                                 head_dim=16, intermediate_size=128, vocab_size=256, max_position_embeddings=64,
                                 attn_implementation="eager")


def _oracle_native(monkeypatch):
    """Route the four entry points the NVFP4 linear uses through the CPU oracle."""

    import oracle
    from qatfactory_b200 import _native

    def bits(mask: torch.Tensor) -> torch.Tensor:
        return torch.from_numpy(np.packbits(mask.reshape(-1).numpy().astype(np.uint8), bitorder="little"))

    def tensor_amax(x, out=None):
        return oracle.tensor_amax(x.contiguous())

    def nvfp4_qdq(x, amax, want_mask=True):
        y, m = oracle.nvfp4_qdq(x.contiguous(), float(amax))
        return y, bits(m) if want_mask else None

    def nvfp4_fake_quant(x, amax_scratch=None, want_mask=True):
        a = oracle.tensor_amax(x.contiguous())
        y, m = nvfp4_qdq(x, a, want_mask)
        return y, m, a

    def tensor_amax_update(x, running):
        running.copy_(torch.maximum(running, oracle.tensor_amax(x.contiguous())))
        return running

    def nvfp4_qdq_shadow(latent, amax, out, mask):
        y, m = oracle.nvfp4_qdq(latent.to(torch.bfloat16).contiguous(), float(amax))
        out.copy_(y.float())
        mask[: (m.numel() + 7) // 8].copy_(bits(m))

    def ste_backward(grad, mask_bits, out=None):
        n = grad.numel()
        m = np.unpackbits(mask_bits.numpy(), bitorder="little")[:n].astype(bool)
        masked = grad * torch.from_numpy(m).reshape(grad.shape).to(grad.dtype)
        return masked if out is None else out.copy_(masked)

    def kd_forward_kl(student, teacher, temperature=1.0, row_valid=None, want_grad=True, grad_scale=1.0):
        ls = F.log_softmax(student.float() / temperature, -1)
        lt = F.log_softmax(teacher.float() / temperature, -1)
        pt = lt.exp()
        keep = torch.ones(student.shape[0]) if row_valid is None else row_valid.float()
        row = (pt * (lt - ls)).sum(-1) * temperature * temperature * keep
        grad = None
        if want_grad:
            grad = ((ls.exp() - pt) * temperature * grad_scale * keep[:, None]).to(student.dtype)
        return row, grad

    for name, fn in (("tensor_amax", tensor_amax), ("tensor_amax_update", tensor_amax_update),
                     ("nvfp4_qdq", nvfp4_qdq), ("nvfp4_qdq_shadow", nvfp4_qdq_shadow),
                     ("nvfp4_fake_quant", nvfp4_fake_quant), ("ste_backward", ste_backward),
                     ("kd_forward_kl", kd_forward_kl)):
        monkeypatch.setattr(_native, name, fn)


def _rank_main(rank: int, world: int, port: int, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mp_ = pytest.MonkeyPatch()
        _oracle_native(mp_)
        torch.manual_seed(0)
        step = qad_step.QADStep(_tiny(), torch.device("cpu"))
        from qatfactory_b200.quant.formats.nvfp4 import _nvfp4_amax_groups

        losses = [float(step(qad_step.synthetic_tokens(256, 32, rank, i, "cpu"))) for i in range(2)]
        groups = _nvfp4_amax_groups(step.student)
        got = [float(g.tensor_amax()) for g in groups]
        want = []
        for g in groups:
            fulls = [m.weight.full_tensor() for m in g.members]
            want.append(max(float(w.detach().to(torch.bfloat16).abs().amax().float()) for w in fulls))
        cfg = _tiny()
        d = cfg.head_dim
        inv = 1.0 / (cfg.rope_parameters["rope_theta"] ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
        rope_ok = all(torch.equal(m.model.rotary_emb.inv_freq, inv) for m in (step.student, step.teacher))
        weights = {n: p.full_tensor().detach().clone() for n, p in step.student.named_parameters() if p.requires_grad}
        # the same steps with each rank quantizing its own shards before FSDP2 gathers them
        torch.manual_seed(0)
        qstep = qad_step.QADStep(_tiny(), torch.device("cpu"), quantized_gather=True)
        qlosses = [float(qstep(qad_step.synthetic_tokens(256, 32, rank, i, "cpu"))) for i in range(2)]
        latents = {n: t.full_tensor().detach() for n, t in qstep.gather.latent_state_dict().items()}
        same = set(latents) == set(weights) and all(torch.equal(latents[n], weights[n]) for n in weights)
        results[rank] = (losses, got, want, len(groups), rope_ok, qlosses, same)
        mp_.undo()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_fsdp2_qad_step_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_rank_main, args=(2, _free_port(), results), nprocs=2, join=True, start_method="spawn")
        res = dict(results)
    assert set(res) == {0, 1}
    for rank in (0, 1):
        losses, got, want, n_groups, rope_ok, qlosses, same = res[rank]
        assert qlosses == losses and same  # quantize-before-gather: the same steps bit for bit
        assert rope_ok  # RoPE frequencies rebuilt after materialising the meta-initialised models
        assert n_groups == 2 * 4  # per layer: the qkv and gate_up families, o and down alone
        assert all(np.isfinite(losses)) and losses[0] > 0
        assert got == want  # family amax all-reduced over the FSDP shards of every member
    assert res[0][1] == res[1][1]
