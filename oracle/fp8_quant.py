"""CPU restatement of the reference's FP8 quantize / dequantize and of fp8 KV
pages (test infrastructure only: tests, smoke and the bench's CPU baseline use
it as the checker; the product never imports it).

* `quantize_fp8_with_scale` follows the reference's decomposition of
  spyre::quantize_fp8_with_scale (torch_spyre/_inductor/decompositions.py:897-904):
  ``inv = reciprocal(scale)``; ``x * inv``; clamp to +-FP8_E4M3_MAX (448,
  torch_spyre/_inductor/constants.py:90); ``qfp8ch`` = conversion to
  float8_e4m3fn (customops.py:562-584).  Every step is a torch CPU op on fp16
  tensors, i.e. computed in fp32 and rounded to fp16, then rounded to e4m3
  (nearest even).
* `dequantize_fp8_with_scale` follows decompositions.py:846-858:
  ``x.to(float16) * scale``.
* `reference_roundtrip` is the CPU formula the reference's own tests compare
  against (tests/inductor/test_fp8_operations.py:235-272):
  ``(x / scale).clamp(-448, 448).to(e4m3).to(fp16) * scale``.
* fp8 pools are [NB, Hkv, D/128, 64, 128] e4m3: the default stick tiling of a
  [64, D] tile of 1-byte elements (128-element sticks;
  torch_spyre/csrc/spyre_tensor_impl.cpp:46-175).  `pool_from_fp16_pool`
  quantizes an fp16 pool [NB, Hkv, D/64, 64, 64] page by page and
  `fp16_pool_from_pool` dequantizes it back into the fp16 page layout, so the
  fp16 attention oracle (paged_attention.py) runs on the dequantized cache.
"""

from __future__ import annotations

import torch

FP8_E4M3_MAX = 448.0
PAGE = 64


def quantize_fp8_with_scale(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    x = x.to(torch.float16)
    inv = torch.reciprocal(scale.to(torch.float16))
    return (x * inv).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)


def dequantize_fp8_with_scale(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float16) * scale.to(torch.float16)


def reference_roundtrip(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return (x / scale).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn).to(torch.float16) * scale


def rows_of_fp16_pool(pool16: torch.Tensor) -> torch.Tensor:
    """fp16 pool [NB, Hkv, S, 64, 64] -> [NB, Hkv, 64, D] (token rows)."""
    nb, hkv, s, t, e = pool16.shape
    return pool16.permute(0, 1, 3, 2, 4).reshape(nb, hkv, t, s * e)


def fp16_pool_of_rows(rows: torch.Tensor) -> torch.Tensor:
    nb, hkv, t, d = rows.shape
    return rows.reshape(nb, hkv, t, d // 64, 64).permute(0, 1, 3, 2, 4).contiguous()


def fp8_pool_of_rows(rows8: torch.Tensor) -> torch.Tensor:
    """[NB, Hkv, 64, D] e4m3 -> fp8 pool [NB, Hkv, D/128, 64, 128]."""
    nb, hkv, t, d = rows8.shape
    return rows8.reshape(nb, hkv, t, d // 128, 128).permute(0, 1, 3, 2, 4).contiguous()


def rows_of_fp8_pool(pool8: torch.Tensor) -> torch.Tensor:
    nb, hkv, s, t, e = pool8.shape
    return pool8.permute(0, 1, 3, 2, 4).reshape(nb, hkv, t, s * e)


def pool_from_fp16_pool(pool16: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return fp8_pool_of_rows(quantize_fp8_with_scale(rows_of_fp16_pool(pool16), scale))


def fp16_pool_from_pool(pool8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return fp16_pool_of_rows(dequantize_fp8_with_scale(rows_of_fp8_pool(pool8), scale))


def append(new_rows: torch.Tensor, pool8: torch.Tensor, slots: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Slot write of fp16 rows [N, Hkv, D] into an fp8 pool, quantized with
    `scale` (negative slots are padding and skipped)."""
    out = pool8.clone()
    q = quantize_fp8_with_scale(new_rows, scale)
    nslots = pool8.shape[0] * PAGE
    for n, slot in enumerate(slots.tolist()):
        if slot < 0:
            continue
        if slot >= nslots:
            raise IndexError(f"slot {slot} outside the pool ({nslots} slots)")
        blk, t = divmod(slot, PAGE)
        out[blk, :, :, t, :] = q[n].reshape(pool8.shape[1], pool8.shape[2], 128)
    return out
