"""torch.library custom ops over libb200kv (namespace ``b200kv``).

Operator surface, mirroring the reference's hot-path ops:

* ``b200kv::decode_attention(q, k_pool, v_pool, block_table, context_lens,
  scale, num_splits) -> (out, lse)`` -- decode SDPA over the paged pools; the
  reference reaches this math through
  ``aten::_scaled_dot_product_fused_attention_overrideable``
  (torch_spyre/csrc/attn_utils.cpp:22-37 -> torch_spyre/_inductor/
  decompositions.py:523-611).  :func:`sdpa_decode` is the drop-in adapter with
  the SDPA signature and the reference's output memory order (596-600).
* ``b200kv::decode_attention_append(q, k_new, v_new, k_pool!, v_pool!, ...)``
  -- the same decode fused with the append of the new token (the HF
  ``index_copy_`` + SDPA decode step, fallbacks.py:256 + decompositions.py).
* ``b200kv::kv_append(k_new, v_new, k_pool!, v_pool!, slot_mapping)`` -- the
  KV slot write, in place like ``spyre::overwrite`` (customops.py:262-295,
  ``mutates_args``) and ``Tensor.index_copy_`` (ops/fallbacks.py:256).
* ``b200kv::rope(x, freqs, positions) -> out`` -- the rotary embedding with the
  reference's formulation (tests/inductor/test_inductor_ops.py:5447-5456);
  ``decode_attention_append(..., rope_freqs=)`` applies it to q and the new K
  row inside the fused kernel.
* ``b200kv::kv_relayout(rows, pool!, block_ids)`` /
  ``b200kv::kv_unrelayout(pool, block_ids, num_tokens) -> rows`` -- the
  row-major <-> stick-page relayout (spyre_mem.cpp:176-440 as an HBM kernel).

Each op has a ``register_fake`` so it can be traced.  The CUDA library is the
only implementation: CPU tensors are rejected, there is no fallback.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch

from . import _lib
from .layout import PAGE_TOKENS

HEAD_DIM = 128
DECODE_INPUTS_READY = 1  # B200KV_DECODE_INPUTS_READY

# ---------------------------------------------------------------- helpers ---
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError(
                f"b200kv ops run on CUDA devices only (got a tensor on {t.device}); "
                "there is no CPU fallback"
            )


def workspace_for(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised decode workspace cached per (device, stream).

    The decode kernel leaves its completion counters at zero after every call,
    so one buffer serves every call ordered on the same stream.
    """
    key = (device.index if device.index is not None else torch.cuda.current_device(), _stream_ptr(device))
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _debug_checks() -> bool:
    return os.environ.get("B200KV_CHECK", "0") not in ("", "0")


def _maybe_check_flag(flag: Optional[torch.Tensor], what: str) -> None:
    if flag is not None and _debug_checks():
        v = int(flag.item())
        if v:
            raise RuntimeError(f"{what}: device error flag 0x{v:x}")


def _check_pool(pool: torch.Tensor, name: str) -> None:
    if pool.dtype != torch.float16 or pool.dim() != 5 or pool.shape[3] != PAGE_TOKENS or pool.shape[4] != 64:
        raise ValueError(f"{name} must be fp16 [num_blocks, Hkv, D/64, 64, 64], got {tuple(pool.shape)} {pool.dtype}")
    if not pool.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _is_fp8(pool: torch.Tensor) -> bool:
    return pool.dtype == torch.float8_e4m3fn


def _need(t: Optional[torch.Tensor], name: str) -> torch.Tensor:
    if t is None:
        raise ValueError(f"fp8 pools need {name} (their fp16 dequantisation scale)")
    return t


# --------------------------------------------------------- decode attention --
@torch.library.custom_op("b200kv::decode_attention", mutates_args=(), device_types="cuda")
def _decode_attention_op(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    num_splits: int,
    error_flag: Optional[torch.Tensor],
    inputs_ready: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(q, k_pool, v_pool, block_table, context_lens)
    if q.dim() != 3 or q.dtype != torch.float16:
        raise ValueError(f"q must be fp16 [B, Hq, D], got {tuple(q.shape)} {q.dtype}")
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    if k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must have the same shape")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be int32 [B, max_blocks] with unit column stride")
    if context_lens.dtype != torch.int32 or context_lens.dim() != 1 or not context_lens.is_contiguous():
        raise ValueError("context_lens must be a contiguous int32 [B] tensor")
    if q.stride(2) != 1:
        raise ValueError("q must have a contiguous head_dim")
    B, Hq, D = q.shape
    NB, Hkv = k_pool.shape[0], k_pool.shape[1]
    if D != k_pool.shape[2] * 64:
        raise ValueError(f"q head_dim {D} does not match the pools ({k_pool.shape[2] * 64})")
    if block_table.shape[0] != B or context_lens.shape[0] != B:
        raise ValueError("block_table / context_lens batch mismatch")
    out = torch.empty((B, Hq, D), dtype=torch.float16, device=q.device)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    if B == 0:
        return out, lse
    lib = _lib.lib()
    wbytes = lib.b200kv_decode_workspace_bytes(B, Hq, Hkv, D)
    # An unsupported shape has no workspace size; the call below then reports
    # the precise reason from the library's own argument checks.
    ws = workspace_for(q.device, wbytes) if wbytes > 0 else torch.empty(0, dtype=torch.uint8, device=q.device)
    args = (
        q.data_ptr(), q.stride(0), q.stride(1),
        k_pool.data_ptr(), v_pool.data_ptr(),
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
        _lib.call("b200kv_decode_attention_ex_f16", *args, DECODE_INPUTS_READY, _stream_ptr(q.device))
    else:
        _lib.call("b200kv_decode_attention_f16", *args, _stream_ptr(q.device))
    _maybe_check_flag(error_flag, "decode_attention")
    return out, lse


@_decode_attention_op.register_fake
def _(q, k_pool, v_pool, block_table, context_lens, scale, num_splits, error_flag, inputs_ready=False):
    B, Hq, D = q.shape
    return q.new_empty((B, Hq, D)), q.new_empty((B, Hq), dtype=torch.float32)


def decode_attention(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: Optional[float] = None,
    num_splits: int = 0,
    return_lse: bool = False,
    error_flag: Optional[torch.Tensor] = None,
    k_scale: Optional[torch.Tensor] = None,
    v_scale: Optional[torch.Tensor] = None,
    inputs_ready: bool = False,
):
    """Decode attention of one new token per sequence over the paged KV pools.

    q [B, Hq, D] fp16; pools fp16 [NB, Hkv, D/64, 64, 64], or float8_e4m3fn
    [NB, Hkv, D/128, 64, 128] with their fp16 dequantisation scales
    ``k_scale`` / ``v_scale`` (one-element device tensors); block_table int32
    [B, max_blocks]; context_lens int32 [B].  Returns out [B, Hq, D] fp16 (and
    the natural-log LSE [B, Hq] fp32 when ``return_lse``).

    ``inputs_ready`` (fp16 or fp8 pools): the pools, block table and context
    lengths were written before the preceding kernel on the stream began (q
    and the fp8 scales may be written by it), so the kernel may plan and start
    its page loads while that kernel finishes (B200KV_DECODE_INPUTS_READY).
    Same result either way.
    """
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if _is_fp8(k_pool):
        from . import fp8  # noqa: F401  (registers the fp8 ops)
        out, lse = torch.ops.b200kv.decode_attention_fp8(
            q, k_pool, v_pool, _need(k_scale, "k_scale"), _need(v_scale, "v_scale"), block_table, context_lens,
            float(scale), int(num_splits), error_flag, bool(inputs_ready)
        )
    else:
        out, lse = torch.ops.b200kv.decode_attention(
            q, k_pool, v_pool, block_table, context_lens, float(scale), int(num_splits), error_flag,
            bool(inputs_ready)
        )
    return (out, lse) if return_lse else out


# ------------------------------------------------- fused append + decode --
@torch.library.custom_op("b200kv::decode_attention_append", mutates_args=("k_pool", "v_pool"),
                         device_types="cuda")
def _decode_attention_append_op(
    q: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    num_splits: int,
    error_flag: Optional[torch.Tensor],
    rope_freqs: Optional[torch.Tensor] = None,
    inputs_ready: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(q, k_new, v_new, k_pool, v_pool, block_table, context_lens)
    if q.dim() != 3 or q.dtype != torch.float16 or q.stride(2) != 1:
        raise ValueError(f"q must be fp16 [B, Hq, D] with a contiguous head_dim, got {tuple(q.shape)}")
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    B, Hq, D = q.shape
    NB, Hkv = k_pool.shape[0], k_pool.shape[1]
    if k_new.shape != (B, Hkv, D) or v_new.shape != k_new.shape or k_new.dtype != torch.float16 \
            or v_new.dtype != torch.float16 or k_new.stride() != v_new.stride() or k_new.stride(2) != 1:
        raise ValueError("k_new / v_new must be fp16 [B, Hkv, D] with equal strides and a contiguous head_dim")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be int32 [B, max_blocks] with unit column stride")
    if context_lens.dtype != torch.int32 or context_lens.dim() != 1 or not context_lens.is_contiguous():
        raise ValueError("context_lens must be a contiguous int32 [B] tensor")
    out = torch.empty((B, Hq, D), dtype=torch.float16, device=q.device)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    if B == 0:
        return out, lse
    lib = _lib.lib()
    wbytes = lib.b200kv_decode_workspace_bytes(B, Hq, Hkv, D)
    ws = workspace_for(q.device, wbytes) if wbytes > 0 else torch.empty(0, dtype=torch.uint8, device=q.device)
    rope = () if rope_freqs is None else (_check_rope_freqs(rope_freqs, D, q.device).data_ptr(), rope_freqs.shape[0])
    if rope and inputs_ready:
        raise ValueError("inputs_ready is not offered with rope_freqs")
    args = (
        q.data_ptr(), q.stride(0), q.stride(1),
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        k_pool.data_ptr(), v_pool.data_ptr(), *rope,
        block_table.data_ptr(), block_table.stride(0),
        context_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        lse.data_ptr(),
        B, Hq, Hkv, D, NB, block_table.shape[1],
        float(scale), int(num_splits),
        ws.data_ptr(), ws.numel(),
        _ptr(error_flag),
    )
    if rope:
        _lib.call("b200kv_decode_attention_append_rope_f16", *args, _stream_ptr(q.device))
    elif inputs_ready:
        _lib.call("b200kv_decode_attention_append_ex_f16", *args, DECODE_INPUTS_READY, _stream_ptr(q.device))
    else:
        _lib.call("b200kv_decode_attention_append_f16", *args, _stream_ptr(q.device))
    _maybe_check_flag(error_flag, "decode_attention_append")
    return out, lse


@_decode_attention_append_op.register_fake
def _(q, k_new, v_new, k_pool, v_pool, block_table, context_lens, scale, num_splits, error_flag, rope_freqs=None,
      inputs_ready=False):
    B, Hq, D = q.shape
    return q.new_empty((B, Hq, D)), q.new_empty((B, Hq), dtype=torch.float32)


def decode_attention_append(
    q: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: Optional[float] = None,
    num_splits: int = 0,
    return_lse: bool = False,
    error_flag: Optional[torch.Tensor] = None,
    k_scale: Optional[torch.Tensor] = None,
    v_scale: Optional[torch.Tensor] = None,
    rope_freqs: Optional[torch.Tensor] = None,
    inputs_ready: bool = False,
):
    """Appends the new token's K/V rows ([B, Hkv, D], at position
    context_lens[b] - 1) to the pools and decodes, in one launch.

    ``inputs_ready`` (fp16 pools, no rope): the caller vouches that the pools
    (other than the rows appended here), block table and context lengths were
    written before the preceding kernel on the stream began, so the kernel
    starts its page loads while that kernel finishes; q and the new rows may be
    written by it.

    Same result as ``kv_append`` at those slots followed by
    ``decode_attention`` (the HF ``index_copy_`` + SDPA step of the reference).
    fp8 pools take ``k_scale`` / ``v_scale``; the new rows are quantized.
    With ``rope_freqs`` ([max_pos, 2, 2, D/2] fp16, or the reference's
    [1, max_pos, 2, 2, D/2]) q and the new K row are first rotated at position
    context_lens[b] - 1, as ``rope`` would.
    """
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if rope_freqs is not None and rope_freqs.dim() == 5:
        rope_freqs = rope_freqs[0]
    if _is_fp8(k_pool):
        from . import fp8  # noqa: F401
        out, lse = torch.ops.b200kv.decode_attention_append_fp8(
            q, k_new, v_new, k_pool, v_pool, _need(k_scale, "k_scale"), _need(v_scale, "v_scale"), block_table,
            context_lens, float(scale), int(num_splits), error_flag, rope_freqs
        )
    else:
        out, lse = torch.ops.b200kv.decode_attention_append(
            q, k_new, v_new, k_pool, v_pool, block_table, context_lens, float(scale), int(num_splits), error_flag,
            rope_freqs, bool(inputs_ready)
        )
    return (out, lse) if return_lse else out


# -------------------------------------------------------------------- rope --
def _check_rope_freqs(freqs: torch.Tensor, head_dim: int, device: torch.device) -> torch.Tensor:
    if freqs.dtype != torch.float16 or freqs.dim() != 4 or tuple(freqs.shape[1:]) != (2, 2, head_dim // 2):
        raise ValueError(f"rope freqs must be fp16 [max_pos, 2, 2, {head_dim // 2}], got {tuple(freqs.shape)}")
    if not freqs.is_contiguous() or freqs.device != device:
        raise ValueError("rope freqs must be contiguous and on the device of the rows")
    return freqs


@torch.library.custom_op("b200kv::rope", mutates_args=(), device_types="cuda")
def _rope_op(x: torch.Tensor, freqs: torch.Tensor, positions: torch.Tensor,
             error_flag: Optional[torch.Tensor]) -> torch.Tensor:
    _require_cuda(x, freqs, positions)
    if x.dim() != 3 or x.dtype != torch.float16 or x.stride(2) != 1:
        raise ValueError(f"x must be fp16 [T, H, D] with a contiguous head_dim, got {tuple(x.shape)}")
    T, H, D = x.shape
    _check_rope_freqs(freqs, D, x.device)
    if positions.dtype != torch.int32 or positions.shape != (T,) or not positions.is_contiguous():
        raise ValueError("positions must be a contiguous int32 [T] tensor")
    out = torch.empty((T, H, D), dtype=torch.float16, device=x.device)
    _lib.call("b200kv_rope_f16", x.data_ptr(), x.stride(0), x.stride(1), out.data_ptr(), out.stride(0),
              out.stride(1), freqs.data_ptr(), freqs.shape[0], positions.data_ptr(), T, H, D, _ptr(error_flag),
              _stream_ptr(x.device))
    _maybe_check_flag(error_flag, "rope")
    return out


@_rope_op.register_fake
def _(x, freqs, positions, error_flag):
    return torch.empty_like(x)


def rope(x: torch.Tensor, freqs: torch.Tensor, positions: torch.Tensor,
         error_flag: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotary embedding of rows x [T, H, D] at positions [T] (int32) with
    freqs [max_pos, 2, 2, D/2] (or the reference's [1, max_pos, 2, 2, D/2]):
    out[..., i*D/2 + j] = sum_k freqs[pos, i, k, j] * x[..., k*D/2 + j]."""
    if freqs.dim() == 5:
        freqs = freqs[0]
    return torch.ops.b200kv.rope(x, freqs, positions, error_flag)


# ------------------------------------------------------------------ append --
@torch.library.custom_op("b200kv::kv_append", mutates_args=("k_pool", "v_pool"), device_types="cuda")
def _kv_append_op(
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    slot_mapping: torch.Tensor,
    error_flag: Optional[torch.Tensor],
) -> None:
    _require_cuda(k_new, v_new, k_pool, v_pool, slot_mapping)
    _check_pool(k_pool, "k_pool")
    _check_pool(v_pool, "v_pool")
    if k_new.shape != v_new.shape or k_new.dim() != 3 or k_new.dtype != torch.float16 or v_new.dtype != torch.float16:
        raise ValueError("k_new / v_new must be fp16 [N, Hkv, D] of equal shape")
    if k_new.stride() != v_new.stride() or k_new.stride(2) != 1:
        raise ValueError("k_new / v_new must share strides with a contiguous head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 [N] tensor")
    N, Hkv, D = k_new.shape
    if slot_mapping.shape[0] != N or Hkv != k_pool.shape[1] or D != k_pool.shape[2] * 64:
        raise ValueError("k_new does not match slot_mapping / the pools")
    _lib.call(
        "b200kv_kv_append_f16",
        k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
        k_pool.data_ptr(), v_pool.data_ptr(), slot_mapping.data_ptr(),
        N, Hkv, D, k_pool.shape[0], _ptr(error_flag), _stream_ptr(k_new.device),
    )
    _maybe_check_flag(error_flag, "kv_append")


@_kv_append_op.register_fake
def _(k_new, v_new, k_pool, v_pool, slot_mapping, error_flag):
    return None


def kv_append(k_new, v_new, k_pool, v_pool, slot_mapping, error_flag=None, k_scale=None, v_scale=None) -> None:
    """Writes row n of k_new / v_new ([N, Hkv, D]) into slot slot_mapping[n]
    (quantized with k_scale / v_scale when the pools are fp8)."""
    if _is_fp8(k_pool):
        from . import fp8  # noqa: F401
        torch.ops.b200kv.kv_append_fp8(k_new, v_new, k_pool, v_pool, _need(k_scale, "k_scale"),
                                       _need(v_scale, "v_scale"), slot_mapping, error_flag)
        return
    torch.ops.b200kv.kv_append(k_new, v_new, k_pool, v_pool, slot_mapping, error_flag)


# ---------------------------------------------------------------- relayout --
@torch.library.custom_op("b200kv::kv_relayout", mutates_args=("pool",), device_types="cuda")
def _kv_relayout_op(rows: torch.Tensor, pool: torch.Tensor, block_ids: torch.Tensor,
                    error_flag: Optional[torch.Tensor]) -> None:
    _require_cuda(rows, pool, block_ids)
    _check_pool(pool, "pool")
    if rows.dim() != 3 or rows.dtype != torch.float16 or not rows.is_contiguous():
        raise ValueError("rows must be a contiguous fp16 [T, Hkv, D] tensor")
    T, Hkv, D = rows.shape
    if Hkv != pool.shape[1] or D != pool.shape[2] * 64:
        raise ValueError("rows do not match the pool's heads / head_dim")
    if block_ids.dtype != torch.int32 or block_ids.dim() != 1 or block_ids.numel() < -(-T // PAGE_TOKENS):
        raise ValueError("block_ids must be int32 [ceil(T / 64)]")
    _lib.call("b200kv_relayout_f16", rows.data_ptr(), pool.data_ptr(), block_ids.data_ptr(),
              T, Hkv, D, pool.shape[0], 0, _ptr(error_flag), _stream_ptr(rows.device))
    _maybe_check_flag(error_flag, "kv_relayout")


@_kv_relayout_op.register_fake
def _(rows, pool, block_ids, error_flag):
    return None


@torch.library.custom_op("b200kv::kv_unrelayout", mutates_args=(), device_types="cuda")
def _kv_unrelayout_op(pool: torch.Tensor, block_ids: torch.Tensor, num_tokens: int,
                      error_flag: Optional[torch.Tensor]) -> torch.Tensor:
    _require_cuda(pool, block_ids)
    _check_pool(pool, "pool")
    Hkv, D = pool.shape[1], pool.shape[2] * 64
    if block_ids.dtype != torch.int32 or block_ids.dim() != 1 or block_ids.numel() < -(-num_tokens // PAGE_TOKENS):
        raise ValueError("block_ids must be int32 [ceil(num_tokens / 64)]")
    rows = torch.empty((num_tokens, Hkv, D), dtype=torch.float16, device=pool.device)
    _lib.call("b200kv_relayout_f16", rows.data_ptr(), pool.data_ptr(), block_ids.data_ptr(),
              num_tokens, Hkv, D, pool.shape[0], 1, _ptr(error_flag), _stream_ptr(pool.device))
    _maybe_check_flag(error_flag, "kv_unrelayout")
    return rows


@_kv_unrelayout_op.register_fake
def _(pool, block_ids, num_tokens, error_flag):
    return pool.new_empty((num_tokens, pool.shape[1], pool.shape[2] * 64))


def kv_relayout(rows, pool, block_ids, error_flag=None) -> None:
    """Scatters a row-major cache [T, Hkv, D] into pages block_ids[t // 64]."""
    torch.ops.b200kv.kv_relayout(rows, pool, block_ids, error_flag)


def kv_unrelayout(pool, block_ids, num_tokens: int, error_flag=None) -> torch.Tensor:
    """Gathers pages block_ids[...] back into a row-major [T, Hkv, D] cache."""
    return torch.ops.b200kv.kv_unrelayout(pool, block_ids, int(num_tokens), error_flag)


# ------------------------------------------------------ merge split states --
def merge_attention_states(outs, lses):
    """Merges attention outputs computed over disjoint KV sets of the same
    queries: outs [n] of [..., D] (fp16 or fp32), lses [n] of [...] fp32
    (natural-log LSE, -inf for an empty set) -> (out fp16 [..., D], lse fp32).
    E.g. a shared prefix decoded once and each sequence's own pages decoded
    separately (``b200kv_lse_combine_f32``)."""
    outs, lses = list(outs), list(lses)
    if not outs or len(outs) != len(lses):
        raise ValueError("need matching non-empty lists of outputs and LSEs")
    o = torch.stack([t.contiguous() for t in outs])
    l = torch.stack([t.contiguous().float() for t in lses])
    _require_cuda(o, l)
    if o.dtype not in (torch.float16, torch.float32):
        raise ValueError("outputs must be fp16 or fp32")
    D = o.shape[-1]
    rows = o[0].numel() // D
    if l[0].numel() != rows:
        raise ValueError("each LSE must have one value per output row")
    out = torch.empty(o.shape[1:], dtype=torch.float16, device=o.device)
    lse = torch.empty(l.shape[1:], dtype=torch.float32, device=o.device)
    _lib.call("b200kv_lse_combine_f32", o.data_ptr(), o.element_size(), l.data_ptr(), o.shape[0], rows, D,
              out.data_ptr(), lse.data_ptr(), _stream_ptr(o.device))
    return out, lse


# ------------------------------------------------------------ SDPA adapter --
def _sdpa_decode_shapes(query, key, value, enable_gqa):
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4 or query.shape[2] != 1:
        raise ValueError("decode SDPA takes query [B, Hq, 1, D] and key / value [B, Hkv, S, D]")
    B, Hq, _, D = query.shape
    Hkv, S = key.shape[1], key.shape[2]
    if key.shape != value.shape or key.shape[0] != B or key.shape[3] != D:
        raise ValueError(f"key {tuple(key.shape)} / value {tuple(value.shape)} do not match query {tuple(query.shape)}")
    if Hq != Hkv and not enable_gqa:
        raise ValueError("Hq != Hkv requires enable_gqa=True")
    return B, Hq, Hkv, S, D


@torch.library.custom_op("b200kv::sdpa_decode", mutates_args=(), device_types="cuda")
def _sdpa_decode_op(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scale: Optional[float],
                    enable_gqa: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode SDPA over dense K/V in a fixed number of launches whatever the
    batch: the K and V rows of every sequence are written into stick pages by
    one append launch (sequence b owns pages [b * nblk, (b + 1) * nblk), token
    s goes to slot b * nblk * 64 + s), then the paged decode kernel runs."""
    _require_cuda(query, key, value)
    B, Hq, Hkv, S, D = _sdpa_decode_shapes(query, key, value, enable_gqa)
    nblk = max(1, -(-S // PAGE_TOKENS))
    k_pool = torch.empty((B * nblk, Hkv, D // 64, PAGE_TOKENS, 64), dtype=torch.float16, device=query.device)
    v_pool = torch.empty_like(k_pool)
    block_table = torch.arange(B * nblk, dtype=torch.int32, device=query.device).view(B, nblk)
    if B * S > 0:
        # token-major rows [B * S, Hkv, D] (one copy each when key / value are head-major)
        rows_k = key.transpose(1, 2).reshape(B * S, Hkv, D)
        rows_v = value.transpose(1, 2).reshape(B * S, Hkv, D)
        seq = torch.arange(B, dtype=torch.int64, device=query.device).unsqueeze(1) * (nblk * PAGE_TOKENS)
        slots = (seq + torch.arange(S, dtype=torch.int64, device=query.device)).reshape(-1)
        kv_append(rows_k, rows_v, k_pool, v_pool, slots)
    ctx = torch.full((B,), S, dtype=torch.int32, device=query.device)
    out, lse = decode_attention(query[:, :, 0, :], k_pool, v_pool, block_table, ctx, scale=scale, return_lse=True)
    # [B, Hq, D] -> [B, 1, Hq, D] memory order, viewed as [B, Hq, 1, D]
    return out.unsqueeze(1).transpose(1, 2), lse


@_sdpa_decode_op.register_fake
def _(query, key, value, scale, enable_gqa):
    B, Hq, _, S, D = _sdpa_decode_shapes(query, key, value, enable_gqa)
    out = query.new_empty((B, 1, Hq, D)).transpose(1, 2)
    return out, query.new_empty((B, Hq), dtype=torch.float32)


def sdpa_decode(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scale: Optional[float] = None,
    enable_gqa: bool = False,
) -> torch.Tensor:
    """Decode SDPA with the signature of F.scaled_dot_product_attention
    (``torch.ops.b200kv.sdpa_decode``, traceable by torch.compile).

    query [B, Hq, 1, D]; key/value dense [B, Hkv, S, D] fp16.  The dense K/V are
    written into stick pages on the device (identity block table) and the
    paged decode kernel runs: a constant number of launches for any B.  The
    result has shape [B, Hq, 1, D] and the memory order [B, 1, Hq, D], like the
    reference decomposition's output (torch_spyre/_inductor/decompositions.py:
    592-600).
    """
    return torch.ops.b200kv.sdpa_decode(query, key, value, scale, bool(enable_gqa))[0]


def _overrideable_tuple(query, key, value, scale, enable_gqa):
    B, Hq = query.shape[0], query.shape[1]
    out, lse = torch.ops.b200kv.sdpa_decode(query, key, value, scale, enable_gqa)
    seed = torch.empty((1,), dtype=torch.float16, device=query.device)
    offset = torch.empty((1,), dtype=torch.float16, device=query.device)
    empty = query.new_empty((0,))
    return out, lse.view(B, Hq, 1), empty, empty, 1, key.shape[2], seed, offset, empty


def _check_overrideable_args(query, key, attn_bias, dropout_p, is_causal):
    if dropout_p > 0.0:
        raise NotImplementedError("attention dropout is not implemented (as in the reference)")
    if attn_bias is not None:
        raise NotImplementedError("an attention bias is not supported by the paged decode path")
    if query.dim() != 4 or query.shape[2] != 1:
        raise NotImplementedError("only the decode case (one query position) is implemented")
    if is_causal and key.shape[2] != 1:
        raise NotImplementedError("is_causal with one query position masks every key but the first")


def scaled_dot_product_fused_attention_overrideable(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attn_bias: Optional[torch.Tensor] = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    return_debug_mask: bool = False,
    scale: Optional[float] = None,
):
    """The decode case of ``aten::_scaled_dot_product_fused_attention_overrideable``
    with the reference decomposition's signature and return tuple
    (torch_spyre/_inductor/decompositions.py:523-611):
    ``(out, logsumexp, None, None, max_q, max_k, philox_seed, philox_offset, None)``,
    out [B, Hq, 1, D] in [B, 1, Hq, D] memory order.  The logsumexp the
    reference leaves uninitialised is filled with the real one.  Query length
    must be 1; dropout, an attention bias and a causal mask (which for one
    query position would keep only key 0) are rejected.
    """
    _check_overrideable_args(query, key, attn_bias, dropout_p, is_causal)
    r = _overrideable_tuple(query, key, value, scale, query.shape[1] != key.shape[1])
    return r[0], r[1], None, None, r[4], r[5], r[6], r[7], None


# ------------------------------------------------------- SDPA dispatch route --
_aten_impl: Optional[torch.library.Library] = None


def _aten_overrideable_cuda(query, key, value, attn_bias=None, dropout_p=0.0, is_causal=False,
                            return_debug_mask=False, *, scale=None):
    _check_overrideable_args(query, key, attn_bias, dropout_p, is_causal)
    return _overrideable_tuple(query, key, value, scale, query.shape[1] != key.shape[1])


def register_sdpa_overrideable() -> None:
    """Registers this package's decode SDPA as the CUDA kernel of the ATen op
    the reference implements for its device,
    ``aten::_scaled_dot_product_fused_attention_overrideable``
    (torch_spyre/_inductor/decompositions.py:523-611).  Idempotent.  CUDA
    itself never selects that op, so nothing else changes until a caller
    calls it or enters :class:`SdpaDecodeMode`."""
    global _aten_impl
    if _aten_impl is None:
        lib = torch.library.Library("aten", "IMPL")
        lib.impl("_scaled_dot_product_fused_attention_overrideable", _aten_overrideable_cuda, "CUDA")
        _aten_impl = lib


def sdpa_decode_eligible(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
                         enable_gqa=False) -> bool:
    """Whether F.scaled_dot_product_attention with these arguments is a decode
    step the paged kernel computes: CUDA fp16, one query position, head_dim
    128, GQA group 1 / 2 / 4 / 8, no mask, dropout or causal mask."""
    if not all(isinstance(t, torch.Tensor) for t in (query, key, value)):
        return False
    if query.device.type != "cuda" or any(t.dtype != torch.float16 for t in (query, key, value)):
        return False
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4 or query.shape[2] != 1 or query.shape[3] != HEAD_DIM:
        return False
    if key.shape != value.shape or key.shape[0] != query.shape[0] or key.shape[3] != HEAD_DIM:
        return False
    hq, hkv = query.shape[1], key.shape[1]
    if hq % hkv or hq // hkv not in (1, 2, 4, 8) or (hq != hkv and not enable_gqa):
        return False
    return attn_mask is None and not dropout_p and not (is_causal and key.shape[2] != 1)


class SdpaDecodeMode(torch.overrides.TorchFunctionMode):
    """Routes decode-shaped ``F.scaled_dot_product_attention`` calls to
    ``aten::_scaled_dot_product_fused_attention_overrideable`` (this package's
    CUDA kernel) and leaves every other call to torch -- what the reference's
    ``_fused_sdp_choice`` does for its device by forcing the overrideable
    backend (torch_spyre/csrc/attn_utils.cpp:22-37).  Install it around the
    code that holds the SDPA call site (e.g. an HF model's decode step)::

        with tsb.ops.SdpaDecodeMode():
            logits = model(input_ids, past_key_values=cache).logits
    """

    def __enter__(self):
        register_sdpa_overrideable()
        return super().__enter__()

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is torch.nn.functional.scaled_dot_product_attention:
            names = ("query", "key", "value", "attn_mask", "dropout_p", "is_causal", "scale", "enable_gqa")
            bound = dict(zip(names, args))
            bound.update(kwargs)
            if sdpa_decode_eligible(bound.get("query"), bound.get("key"), bound.get("value"),
                                    bound.get("attn_mask"), bound.get("dropout_p", 0.0),
                                    bound.get("is_causal", False), bound.get("enable_gqa", False)):
                return torch.ops.aten._scaled_dot_product_fused_attention_overrideable(
                    bound["query"], bound["key"], bound["value"], None, 0.0, bool(bound.get("is_causal", False)),
                    False, scale=bound.get("scale"))[0]
        return func(*args, **kwargs)
