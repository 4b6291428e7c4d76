"""Seeded synthetic decode-GEMM operands (no checkpoint or dataset is used anywhere).

Distributions follow the decode-GEMM workloads: weights bf16 ~ N(0, 0.02) (the init the
reference's kernel test applies, tests/test_hand_rolled_kernels.py:154-156), activations
bf16 ~ N(0, 1). Values are drawn in fp32 with a dedicated ``torch.Generator`` per tensor and
rounded once to bf16 (nearest-even), so the same (shape, seed, device) always gives the same
bits.
"""

from __future__ import annotations

import torch

WEIGHT_STD = 0.02
ACT_STD = 1.0


def synthetic_bf16(shape, seed: int, std: float = 1.0, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(int(seed))
    t = torch.randn(tuple(shape), generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(torch.bfloat16)


def weight(N: int, K: int, seed: int, device="cpu") -> torch.Tensor:
    """Row-major [N, K] bf16 weight, as packed by the reference (engine/kernels/weights.py:10-11)."""
    return synthetic_bf16((N, K), seed, WEIGHT_STD, device)


def activation(M: int, K: int, seed: int, device="cpu") -> torch.Tensor:
    """Contiguous [M, K] bf16 decode activations."""
    return synthetic_bf16((M, K), seed, ACT_STD, device)
