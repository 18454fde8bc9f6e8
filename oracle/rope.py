"""CPU restatement of the reference's rotary position embedding (test
infrastructure only: tests and the bench's CPU baseline use it as the
checker; the product never imports it).

The reference composes RoPE from tensor ops (tests/inductor/
test_inductor_ops.py:5447-5456; param sets 2840-2858): a head row of D
elements is viewed as [2, D/2] (halves k = 0, 1), multiplied elementwise by
freqs[s] of shape [2, 2, D/2] broadcast over the output half i, and summed over
k.  On CPU fp16 tensors each product is rounded to fp16 and the sum over k is
accumulated in fp32 and rounded to fp16 once.  `rope_rows` evaluates the same
operations for rows at arbitrary positions:
    out[t, h, i * D/2 + j] = sum_k freqs[positions[t], i, k, j] * x[t, h, k * D/2 + j].
"""

from __future__ import annotations

import torch


def rope_rows(x: torch.Tensor, freqs: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """x [T, H, D] fp16, freqs [P, 2, 2, D/2] fp16, positions [T] -> [T, H, D] fp16."""
    T, H, D = x.shape
    half = D // 2
    xk = x.reshape(T, H, 1, 2, half)                       # [T, H, -, k, j]
    f = freqs[positions.long()].reshape(T, 1, 2, 2, half)  # [T, -, i, k, j]
    prod = f * xk                                          # fp16 products, [T, H, i, k, j]
    return prod.sum(dim=3).reshape(T, H, D)                # fp32-accumulated sum over k


def rope_float(x: torch.Tensor, freqs: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """The same rotation in fp32 (no intermediate rounding), for tolerance checks."""
    T, H, D = x.shape
    half = D // 2
    xk = x.float().reshape(T, H, 1, 2, half)
    f = freqs.float()[positions.long()].reshape(T, 1, 2, 2, half)
    return (f * xk).sum(dim=3).reshape(T, H, D)
