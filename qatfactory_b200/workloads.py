"""Seeded synthetic inputs for the benchmark configurations of the fake-quantization path.

The reference measures on no dataset for this path; these generators reproduce the
shapes, value distributions and seeds of the five configurations (N(0, 0.02) latent
weights, Student-t(df=4) activations with outlier channels, N(0, 1) upstream grads).
Every tensor is drawn on the CPU from a seeded ``torch.Generator`` (or, for the Student-t
sampler, a forked global RNG) and cast to BF16, so the oracle, the reference and the CUDA
kernels all see identical bits on any host.
"""

from __future__ import annotations

import torch

# Qwen3-8B linear shapes (out_features, in_features), in the order q, k, v, o, gate, up, down.
QWEN3_8B_LINEARS = (
    ("q_proj", 4096, 4096),
    ("k_proj", 1024, 4096),
    ("v_proj", 1024, 4096),
    ("o_proj", 4096, 4096),
    ("gate_proj", 12288, 4096),
    ("up_proj", 12288, 4096),
    ("down_proj", 4096, 12288),
)
QWEN3_8B_LAYERS = 36


def normal(shape, std: float, seed: int, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype)


def student_t_outliers(shape, seed: int, outlier_seed: int, n_outliers: int = 8, dtype=torch.bfloat16) -> torch.Tensor:
    """Student-t(df=4) * 0.5 with ``n_outliers`` random channels scaled x50."""

    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        x = torch.distributions.StudentT(4.0).sample(torch.Size(shape)) * 0.5
    channels = torch.randperm(shape[-1], generator=torch.Generator().manual_seed(outlier_seed))[:n_outliers]
    x[..., channels] *= 50.0
    return x.to(dtype)


# --- configuration 1: NVFP4 W4A16 fake-quant of one [4096, 4096] weight + STE backward
def config1_weight() -> torch.Tensor:
    return normal((4096, 4096), 0.02, seed=0)


def config1_grad() -> torch.Tensor:
    return normal((4096, 4096), 1.0, seed=1)


# --- configuration 2: MXFP4 weights (fused gate/up) and activations
def config2_weight() -> torch.Tensor:
    return normal((2 * 12288, 4096), 0.02, seed=2)


def config2_activation() -> torch.Tensor:
    return student_t_outliers((16384, 4096), seed=3, outlier_seed=4)


# --- configuration 3: Q4_K over every linear of a Qwen3-8B layer stack
def config3_layer(layer: int) -> list[tuple[str, torch.Tensor]]:
    return [
        (name, normal((out_f, in_f), 0.02, seed=5 + layer * 7 + idx))
        for idx, (name, out_f, in_f) in enumerate(QWEN3_8B_LINEARS)
    ]


def config3_elements(layers: int = QWEN3_8B_LAYERS) -> int:
    return layers * sum(o * i for _, o, i in QWEN3_8B_LINEARS)


# --- configuration 4: NVFP4 W4A4 fused-QKV linear
def config4_inputs() -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    x = student_t_outliers((16384, 4096), seed=6, outlier_seed=6 + 1000)
    w = normal((6144, 4096), 0.02, seed=7)
    dy = normal((16384, 6144), 1.0, seed=8)
    return x, w, dy
