"""FP8 (e4m3) ops over libb200kv: quantize / dequantize with an fp16 scale,
and fp8 KV pages (append and decode attention).

* ``b200kv::quantize_fp8_with_scale(input, scale)`` /
  ``b200kv::dequantize_fp8_with_scale(input, scale)`` -- the reference's
  ``spyre::quantize_fp8_with_scale`` / ``spyre::dequantize_fp8_with_scale``
  (torch_spyre/_inductor/customops.py:587-653), same argument meaning: input
  ``[..., hidden]``, scale fp16 of shape ``[1]`` (one scale) or
  ``input.shape[:-1] + (1,)`` (one scale per row); results bit-identical to the
  reference's decompositions (decompositions.py:846-858, 897-904).
* fp8 pools ``float8_e4m3fn [NB, Hkv, D/128, 64, 128]`` (the stick tiling of
  1-byte elements) with one fp16 scale per pool (a device scalar tensor):
  ``b200kv::kv_append_fp8``, ``b200kv::decode_attention_fp8`` and
  ``b200kv::decode_attention_append_fp8`` mirror their fp16 counterparts in
  :mod:`torch_spyre_b200.ops`; :func:`torch_spyre_b200.ops.decode_attention`
  and friends dispatch here when the pools are fp8.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .layout import PAGE_TOKENS
from .ops import (DECODE_INPUTS_READY, _check_rope_freqs, _maybe_check_flag, _ptr, _require_cuda, _stream_ptr,
                  workspace_for)

FP8 = torch.float8_e4m3fn
FP8_E4M3_MAX = 448.0


def _check_pool8(pool: torch.Tensor, name: str) -> None:
    if pool.dtype != FP8 or pool.dim() != 5 or pool.shape[3] != PAGE_TOKENS or pool.shape[4] != 128:
        raise ValueError(f"{name} must be float8_e4m3fn [num_blocks, Hkv, D/128, 64, 128], "
                         f"got {tuple(pool.shape)} {pool.dtype}")
    if not pool.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _check_scale(scale: torch.Tensor, name: str, device: torch.device) -> None:
    if scale.dtype != torch.float16 or scale.numel() != 1 or scale.device != device:
        raise ValueError(f"{name} must be a one-element fp16 tensor on {device}")


def _row_scale(input: torch.Tensor, scale: torch.Tensor) -> tuple[torch.Tensor, int]:
    """(scale tensor, stride between rows) for a [..., hidden] input."""
    if scale.dtype != torch.float16:
        raise ValueError(f"scale must be fp16 (got {scale.dtype})")
    if scale.numel() == 1:
        return scale.contiguous(), 0
    lead = tuple(input.shape[:-1])
    if tuple(scale.shape) not in (lead + (1,), lead):
        raise ValueError(f"scale of shape {tuple(scale.shape)} does not broadcast over the rows of "
                         f"{tuple(input.shape)} (expected [1] or {lead + (1,)})")
    return scale.contiguous(), 1


# ------------------------------------------------------ quantize / dequantize --
@torch.library.custom_op("b200kv::quantize_fp8_with_scale", mutates_args=(), device_types="cuda")
def _quantize_op(input: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    _require_cuda(input, scale)
    if input.dtype != torch.float16:
        raise ValueError(f"input must be fp16 (got {input.dtype})")
    x = input.contiguous()
    sc, stride = _row_scale(x, scale)
    out = torch.empty(x.shape, dtype=FP8, device=x.device)
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // cols if cols else 0
    _lib.call("b200kv_quantize_fp8_f16", x.data_ptr(), out.data_ptr(), rows, cols, sc.data_ptr(), stride,
              _stream_ptr(x.device))
    return out


@_quantize_op.register_fake
def _(input, scale):
    return torch.empty(input.size(), dtype=FP8, device=input.device)


@torch.library.custom_op("b200kv::dequantize_fp8_with_scale", mutates_args=(), device_types="cuda")
def _dequantize_op(input: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    _require_cuda(input, scale)
    if input.dtype != FP8:
        raise ValueError(f"input must be float8_e4m3fn (got {input.dtype})")
    x = input.contiguous()
    sc, stride = _row_scale(x, scale)
    out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // cols if cols else 0
    _lib.call("b200kv_dequantize_fp8_f16", x.data_ptr(), out.data_ptr(), rows, cols, sc.data_ptr(), stride,
              _stream_ptr(x.device))
    return out


@_dequantize_op.register_fake
def _(input, scale):
    return torch.empty(input.size(), dtype=torch.float16, device=input.device)


def quantize_fp8_with_scale(input: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3(clamp(input * (1 / scale), -448, 448)), the reference's quantize."""
    return torch.ops.b200kv.quantize_fp8_with_scale(input, scale)


def dequantize_fp8_with_scale(input: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp16(input) * scale, the reference's dequantize."""
    return torch.ops.b200kv.dequantize_fp8_with_scale(input, scale)


# ----------------------------------------------------------------- pools --
def pool_shape_fp8(num_blocks: int, num_kv_heads: int, head_dim: int = 128) -> tuple[int, ...]:
    """Shape of an fp8 K or V pool: [num_blocks, Hkv, head_dim / 128, 64, 128]."""
    if head_dim % 128:
        raise ValueError("head_dim must be a multiple of 128 for fp8 pages")
    return (num_blocks, num_kv_heads, head_dim // 128, PAGE_TOKENS, 128)


def empty_pool_fp8(num_blocks: int, num_kv_heads: int, head_dim: int = 128, device=None) -> torch.Tensor:
    return torch.empty(pool_shape_fp8(num_blocks, num_kv_heads, head_dim), dtype=FP8, device=device)


def quantize_pool(pool16: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp16 pool [NB, Hkv, D/64, 64, 64] -> fp8 pool [NB, Hkv, D/128, 64, 128]
    holding quantize_fp8_with_scale(K, scale) of the same token rows."""
    nb, hkv, s, t, e = pool16.shape
    d = s * e
    rows = pool16.permute(0, 1, 3, 2, 4).reshape(nb, hkv, t, d)
    q = quantize_fp8_with_scale(rows, scale)
    return q.view(nb, hkv, t, d // 128, 128).permute(0, 1, 3, 2, 4).contiguous()


def dequantize_pool(pool8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp8 pool -> fp16 pool of the dequantized values (fp16 page layout)."""
    nb, hkv, s, t, e = pool8.shape
    d = s * e
    rows = dequantize_fp8_with_scale(pool8.permute(0, 1, 3, 2, 4).reshape(nb, hkv, t, d), scale)
    return rows.view(nb, hkv, t, d // 64, 64).permute(0, 1, 3, 2, 4).contiguous()


@torch.library.custom_op("b200kv::kv_append_fp8", mutates_args=("k_pool", "v_pool"), device_types="cuda")
def _kv_append_fp8_op(
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    slot_mapping: torch.Tensor,
    error_flag: Optional[torch.Tensor],
) -> None:
    _require_cuda(k_new, v_new, k_pool, v_pool, k_scale, v_scale, slot_mapping)
    _check_pool8(k_pool, "k_pool")
    _check_pool8(v_pool, "v_pool")
    _check_scale(k_scale, "k_scale", k_pool.device)
    _check_scale(v_scale, "v_scale", k_pool.device)
    if k_new.shape != v_new.shape or k_new.dim() != 3 or k_new.dtype != torch.float16 or v_new.dtype != torch.float16:
        raise ValueError("k_new / v_new must be fp16 [N, Hkv, D] of equal shape")
    if k_new.stride() != v_new.stride() or k_new.stride(2) != 1:
        raise ValueError("k_new / v_new must share strides with a contiguous head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 [N] tensor")
    N, Hkv, D = k_new.shape
    if slot_mapping.shape[0] != N or Hkv != k_pool.shape[1] or D != k_pool.shape[2] * 128:
        raise ValueError("k_new does not match slot_mapping / the pools")
    _lib.call(
        "b200kv_kv_append_fp8",
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(),
        slot_mapping.data_ptr(), N, Hkv, D, k_pool.shape[0], _ptr(error_flag), _stream_ptr(k_new.device),
    )
    _maybe_check_flag(error_flag, "kv_append_fp8")


@_kv_append_fp8_op.register_fake
def _(k_new, v_new, k_pool, v_pool, k_scale, v_scale, slot_mapping, error_flag):
    return None


def _check_decode_common(q, block_table, context_lens, k_pool):
    if q.dim() != 3 or q.dtype != torch.float16 or q.stride(2) != 1:
        raise ValueError(f"q must be fp16 [B, Hq, D] with a contiguous head_dim, got {tuple(q.shape)}")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be int32 [B, max_blocks] with unit column stride")
    if context_lens.dtype != torch.int32 or context_lens.dim() != 1 or not context_lens.is_contiguous():
        raise ValueError("context_lens must be a contiguous int32 [B] tensor")
    B, Hq, D = q.shape
    if D != k_pool.shape[2] * 128:
        raise ValueError(f"q head_dim {D} does not match the pools ({k_pool.shape[2] * 128})")
    if block_table.shape[0] != B or context_lens.shape[0] != B:
        raise ValueError("block_table / context_lens batch mismatch")


@torch.library.custom_op("b200kv::decode_attention_fp8", mutates_args=(), device_types="cuda")
def _decode_attention_fp8_op(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    num_splits: int,
    error_flag: Optional[torch.Tensor],
    inputs_ready: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(q, k_pool, v_pool, k_scale, v_scale, block_table, context_lens)
    _check_pool8(k_pool, "k_pool")
    _check_pool8(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must have the same shape")
    _check_scale(k_scale, "k_scale", q.device)
    _check_scale(v_scale, "v_scale", q.device)
    _check_decode_common(q, block_table, context_lens, k_pool)
    B, Hq, D = q.shape
    NB, Hkv = k_pool.shape[0], k_pool.shape[1]
    out = torch.empty((B, Hq, D), dtype=torch.float16, device=q.device)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    if B == 0:
        return out, lse
    wbytes = _lib.lib().b200kv_decode_workspace_bytes(B, Hq, Hkv, D)
    ws = workspace_for(q.device, wbytes) if wbytes > 0 else torch.empty(0, dtype=torch.uint8, device=q.device)
    args = (
        q.data_ptr(), q.stride(0), q.stride(1),
        k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(),
        block_table.data_ptr(), block_table.stride(0),
        context_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(),
        B, Hq, Hkv, D, NB, block_table.shape[1],
        float(scale), int(num_splits),
        ws.data_ptr(), ws.numel(),
        _ptr(error_flag),
    )
    if inputs_ready:
        _lib.call("b200kv_decode_attention_ex_fp8", *args, DECODE_INPUTS_READY, _stream_ptr(q.device))
    else:
        _lib.call("b200kv_decode_attention_fp8", *args, _stream_ptr(q.device))
    _maybe_check_flag(error_flag, "decode_attention_fp8")
    return out, lse


@_decode_attention_fp8_op.register_fake
def _(q, k_pool, v_pool, k_scale, v_scale, block_table, context_lens, scale, num_splits, error_flag,
      inputs_ready=False):
    B, Hq, D = q.shape
    return q.new_empty((B, Hq, D)), q.new_empty((B, Hq), dtype=torch.float32)


@torch.library.custom_op("b200kv::decode_attention_append_fp8", mutates_args=("k_pool", "v_pool"),
                         device_types="cuda")
def _decode_attention_append_fp8_op(
    q: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    num_splits: int,
    error_flag: Optional[torch.Tensor],
    rope_freqs: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale, block_table, context_lens)
    _check_pool8(k_pool, "k_pool")
    _check_pool8(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must have the same shape")
    _check_scale(k_scale, "k_scale", q.device)
    _check_scale(v_scale, "v_scale", q.device)
    _check_decode_common(q, block_table, context_lens, k_pool)
    B, Hq, D = q.shape
    NB, Hkv = k_pool.shape[0], k_pool.shape[1]
    if k_new.shape != (B, Hkv, D) or v_new.shape != k_new.shape or k_new.dtype != torch.float16 \
            or v_new.dtype != torch.float16 or k_new.stride() != v_new.stride() or k_new.stride(2) != 1:
        raise ValueError("k_new / v_new must be fp16 [B, Hkv, D] with equal strides and a contiguous head_dim")
    out = torch.empty((B, Hq, D), dtype=torch.float16, device=q.device)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    if B == 0:
        return out, lse
    wbytes = _lib.lib().b200kv_decode_workspace_bytes(B, Hq, Hkv, D)
    ws = workspace_for(q.device, wbytes) if wbytes > 0 else torch.empty(0, dtype=torch.uint8, device=q.device)
    rope = () if rope_freqs is None else (_check_rope_freqs(rope_freqs, D, q.device).data_ptr(), rope_freqs.shape[0])
    _lib.call(
        "b200kv_decode_attention_append_rope_fp8" if rope else "b200kv_decode_attention_append_fp8",
        q.data_ptr(), q.stride(0), q.stride(1),
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), *rope,
        block_table.data_ptr(), block_table.stride(0),
        context_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(),
        B, Hq, Hkv, D, NB, block_table.shape[1],
        float(scale), int(num_splits),
        ws.data_ptr(), ws.numel(),
        _ptr(error_flag), _stream_ptr(q.device),
    )
    _maybe_check_flag(error_flag, "decode_attention_append_fp8")
    return out, lse


@_decode_attention_append_fp8_op.register_fake
def _(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale, block_table, context_lens, scale, num_splits,
      error_flag, rope_freqs=None):
    B, Hq, D = q.shape
    return q.new_empty((B, Hq, D)), q.new_empty((B, Hq), dtype=torch.float32)
