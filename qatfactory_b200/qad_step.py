"""The QAD student step of configuration 5: the step-level caller of the fake-quant path.

A minimal FSDP2 harness standing in for QATFactory's HF-Trainer glue: it reproduces what one
optimizer step of ``QADTrainer`` does (qatfactory/trainer/qad_trainer.py:550-639), with the
fused-family amax refresh of ``FusedScaleRefreshCallback`` (qatfactory/trainer/callbacks.py:26-31)
after the optimizer step:

    teacher forward (frozen BF16, no grad) -> student forward (NVFP4 fake-quantized linears,
    gradient-checkpointed decoder layers) -> forward KL at T=1 over FP32 logit chunks
    (qatfactory/distill/kd_loss.py:147-195, on the fused kernel) -> backward (STE) -> AdamW on the FP32 latent
    masters (qatfactory/models/llm.py:247-270) -> refresh of the per-family tensor amax
    (one NCCL all-reduce MAX of the [n_families] vector).

Both models are Qwen3 causal LMs built from a config with random weights; the student's
target linears are swapped by ``apply_fake_quant`` for ``NVFP4Linear`` (fused families,
W4A16).  Every decoder layer and the root are wrapped by FSDP2 ``fully_shard`` with a BF16
compute / FP32 reduce policy, one process per GPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import quant as _b200_quant
from .distill import distill_loss as fused_distill_loss

TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
IGNORE_INDEX = -100


def qwen3_config(**overrides):
    """Qwen3-8B architecture (36 layers, hidden 4096, 32 q / 8 kv heads of dim 128, SwiGLU
    12288, vocab 151936, RoPE theta 1e6, untied head); overrides shrink it for tests."""

    from transformers import Qwen3Config

    kw = dict(hidden_size=4096, num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
              intermediate_size=12288, vocab_size=151936, rope_theta=1e6, tie_word_embeddings=False,
              max_position_embeddings=40960, rms_norm_eps=1e-6, attn_implementation="sdpa")
    kw.update(overrides)
    return Qwen3Config(**kw)


def distill_loss(student_logits: torch.Tensor, teacher_logits: torch.Tensor, labels: torch.Tensor,
                 chunk_size: int = 2048) -> torch.Tensor:
    """Forward KL(teacher || student) at T=1 per supervised token, summed in FP32 chunks and
    divided by the token count (kd_loss.py:128-195 with hard_label_weight 0): the reference's
    formulation in torch, which the step replaces with the fused kernel (``distill.py``)."""

    s = student_logits[..., :-1, :]
    t = teacher_logits[..., :-1, :]
    flat = labels[..., 1:].reshape(-1)
    valid = flat != IGNORE_INDEX
    s = s.reshape(-1, s.shape[-1])[valid]
    t = t.reshape(-1, t.shape[-1])[valid]
    total = s.new_zeros((), dtype=torch.float32)
    for start in range(0, s.shape[0], chunk_size):
        sc = s[start:start + chunk_size].float()
        tc = t[start:start + chunk_size].float()
        total = total + F.kl_div(F.log_softmax(sc, dim=-1), F.softmax(tc, dim=-1), reduction="sum")
    return total / valid.sum().clamp_min(1)


@torch.no_grad()
def _init_(model: torch.nn.Module, seed: int, std: float = 0.02) -> None:
    """N(0, std) for matrices and embeddings, ones for RMSNorm weights; the same bits on every rank."""

    g = torch.Generator(device=next(model.parameters()).device)
    for i, (name, p) in enumerate(model.named_parameters()):
        if p.ndim == 1:
            p.fill_(1.0)
        else:
            g.manual_seed(seed * 100003 + i)
            p.normal_(0.0, std, generator=g)


class Impl:
    """Where the step's fake-quant modules and distillation loss come from: this repository
    (``impl="b200"``: NVFP4Linear on the sm_100a kernels, the fused KD-loss kernel) or the
    unmodified reference (``impl="reference"``: ``qatfactory.quant`` with its Triton quantizers
    and ``qatfactory.distill.kd_loss.distill_loss``), imported from ``ref_path`` (a pip install of
    the reference, e.g. ``baseline/_ref``)."""

    def __init__(self, impl: str = "b200", ref_path=None):
        if impl == "b200":
            self.quant = _b200_quant
            self.distill_loss = fused_distill_loss
        elif impl == "reference":
            import sys

            if ref_path is not None and str(ref_path) not in sys.path:
                sys.path.append(str(ref_path))
            import qatfactory.quant as rq
            from qatfactory.distill.kd_loss import distill_loss as ref_loss

            self.quant = rq
            self.distill_loss = ref_loss
        else:
            raise ValueError(f"unknown impl {impl!r}")
        self.name = impl


def build_models(config, device: torch.device, *, student_seed: int = 9, teacher_seed: int = 10,
                 gradient_checkpointing: bool = True, impl: Impl | None = None, fsdp: bool = True):
    """Student (NVFP4 fake-quant, FP32 latent masters, FSDP2) and teacher (BF16, frozen, FSDP2)."""

    impl = impl or Impl("b200")

    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
    from transformers import Qwen3ForCausalLM

    with torch.device("meta"):
        student = Qwen3ForCausalLM(config)
        teacher = Qwen3ForCausalLM(config)
    student.to_empty(device=device)
    teacher.to_empty(device=device)
    student.to(torch.bfloat16)
    teacher.to(torch.bfloat16)
    for model in (student, teacher):  # to_empty leaves the RoPE frequency buffers uninitialised (FP32)
        model.model.rotary_emb = type(model.model.rotary_emb)(config, device=device)
    _init_(student, student_seed)
    with torch.no_grad():
        g = torch.Generator(device=device)
        for i, (ps, pt) in enumerate(zip(student.parameters(), teacher.parameters())):
            pt.copy_(ps)
            if ps.ndim > 1:
                g.manual_seed(teacher_seed * 100003 + i)
                pt.add_(torch.randn(pt.shape, generator=g, device=device, dtype=torch.float32).mul_(0.002).to(pt.dtype))
    teacher.requires_grad_(False)
    teacher.eval()

    impl.quant.apply_fake_quant(student, TARGETS, quant_format="nvfp4", fused_runtime_scales=True)
    for p in student.parameters():  # FP32 masters for the trainable latents (llm.py:247-270)
        if p.requires_grad:
            p.data = p.data.float()
    if gradient_checkpointing:
        student.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": False})
    student.config.use_cache = False
    student.train()
    if not fsdp:
        return student, teacher

    mp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
    for layer in student.model.layers:
        fully_shard(layer, mp_policy=mp)
    fully_shard(student, mp_policy=mp)
    for layer in teacher.model.layers:
        fully_shard(layer)
    fully_shard(teacher)
    return student, teacher


class QADStep:
    """One optimizer step per call on a micro-batch of token ids (mbs 1 per rank)."""

    def __init__(self, config, device: torch.device, *, lr: float = 1e-6, gradient_checkpointing: bool = True,
                 logits_chunk_size: int = 2048, impl: str = "b200", ref_path=None, fsdp: bool = True,
                 quantized_gather: bool = False):
        """``quantized_gather``: each rank quantizes its FP32 latent shards once per optimizer
        step and FSDP2 gathers the quantized weights (``quant.NVFP4QuantizedGather``), instead
        of every forward and recompute quantizing the gathered weights; same results."""

        self.device = device
        self.impl = Impl(impl, ref_path)
        self.student, self.teacher = build_models(config, device, gradient_checkpointing=gradient_checkpointing,
                                                  impl=self.impl, fsdp=fsdp)
        self.gather = None
        if quantized_gather:
            if impl != "b200":
                raise ValueError("quantized_gather runs on this repository's kernels only")
            self.gather = _b200_quant.NVFP4QuantizedGather(self.student)
            groups = [{"params": ps} for ps in (self.gather.other_parameters(self.student), self.gather.parameters())
                      if ps]
        else:
            groups = [p for p in self.student.parameters() if p.requires_grad]
        self.optimizer = torch.optim.AdamW(groups, lr=lr, betas=(0.9, 0.999), weight_decay=0.0, fused=True)
        self.chunk = logits_chunk_size
        self.impl.quant.refresh_nvfp4_weight_amax(self.student)  # FusedScaleRefreshCallback.on_train_begin
        if self.gather is not None:
            self.gather.requantize()

    def forward_backward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Teacher forward, student forward, distillation loss and its backward (gradients left
        on the student's parameters); returns the detached loss."""

        labels = input_ids
        with torch.no_grad():
            t_logits = self.teacher(input_ids=input_ids, use_cache=False).logits
        s_logits = self.student(input_ids=input_ids, use_cache=False).logits
        loss = self.impl.distill_loss(s_logits, t_logits, labels, logits_chunk_size=self.chunk).loss
        del t_logits
        loss.backward()
        return loss.detach()

    def optimizer_step(self) -> None:
        """AdamW on the gradients left by ``forward_backward``, then the amax refresh (and, with
        the quantized gather, the STE mask on the reduced gradients before and the shards'
        requantization after)."""

        if self.gather is not None:
            self.gather.gradients_to_latents()
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        self.impl.quant.refresh_nvfp4_weight_amax(self.student)  # FusedScaleRefreshCallback.on_step_end
        if self.gather is not None:
            self.gather.requantize()

    def __call__(self, input_ids: torch.Tensor) -> torch.Tensor:
        loss = self.forward_backward(input_ids)
        self.optimizer_step()
        return loss


def synthetic_tokens(vocab: int, seq: int, rank: int, step: int, device) -> torch.Tensor:
    """Uniform token ids over the vocabulary, seed 11 + rank (and the step)."""

    g = torch.Generator().manual_seed(11 + rank + 1000 * step)
    return torch.randint(0, vocab, (1, seq), generator=g).to(device)


def ensure_process_group(timeout_s: int = 600) -> tuple[int, int, int]:
    """(rank, world, local_rank); a one-rank NCCL group when not launched by torchrun."""

    import os
    from datetime import timedelta

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def step_flops(config, seq: int, gradient_checkpointing: bool = True) -> float:
    """Algorithmic matmul FLOPs of one QAD step on one sequence of ``seq`` tokens.

    Forward = decoder linears 2*seq*P_layer per layer + causal attention 2*seq^2*(heads*head_dim)
    per layer (QK^T and PV over the lower triangle) + LM head 2*seq*hidden*vocab.  One step is a
    teacher forward, a student forward, the recomputed decoder forward of gradient checkpointing
    and a student backward counted as twice the forward."""

    h = config.hidden_size
    hq = config.num_attention_heads * config.head_dim
    hkv = config.num_key_value_heads * config.head_dim
    per_layer = h * hq + 2 * h * hkv + hq * h + 3 * h * config.intermediate_size
    layers = config.num_hidden_layers * (2.0 * seq * per_layer + 2.0 * seq * seq * hq)
    head = 2.0 * seq * h * config.vocab_size
    fwd = layers + head
    return 2 * fwd + (layers if gradient_checkpointing else 0.0) + 2 * fwd
