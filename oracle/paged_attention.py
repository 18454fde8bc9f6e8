"""CPU oracle of paged decode attention (test infrastructure only).

`decode_attention_cpu` is the reference's CPU eager path for decode SDPA: the
reference's test harness runs the user function on CPU tensors with stock
torch and treats that as the truth (compare_with_cpu,
tests/inductor/utils_inductor.py:620-703, line 661).  For a paged cache the
pages of each sequence are first gathered into a dense [Hkv, ctx, D] tensor by
the block table, then `torch.nn.functional.scaled_dot_product_attention` runs
on fp32 upcasts with `enable_gqa=True` (query head h uses KV head h // G, as in
decompositions.py:560-563) and the output is cast to fp16.

`sdpa_decomposition_cpu` restates the reference decomposition itself
(torch_spyre/_inductor/decompositions.py:549-596): sqrt(scale) applied to both
q and k, KV-head expansion, q @ k^T, softmax, @ v -- all in fp32 here.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

PAGE = 64


def gather_pages(pool: torch.Tensor, block_row: torch.Tensor, ctx: int) -> torch.Tensor:
    """Dense [Hkv, ctx, D] rows of one sequence from a [NB, Hkv, S, 64, 64] pool.

    Element (t, d) of head h sits in page block_row[t // 64] at stick d // 64,
    row t % 64, column d % 64 (the default stick tiling of a [64, D] tile).
    """
    n = -(-ctx // PAGE)
    if n == 0:
        return pool.new_empty((pool.shape[1], 0, pool.shape[2] * 64))
    pages = pool[block_row[:n].long()]              # [n, Hkv, S, 64, 64]
    dense = pages.permute(1, 0, 3, 2, 4)            # [Hkv, n, 64 t, S, 64 e]
    dense = dense.reshape(pool.shape[1], n * PAGE, pool.shape[2] * 64)
    return dense[:, :ctx]


def decode_attention_cpu(q, k_pool, v_pool, block_table, context_lens, scale=None,
                         return_lse=False):
    """Reference CPU eager decode: out [B, Hq, D] fp16 (and LSE [B, Hq] fp32)."""
    q = q.cpu()
    k_pool, v_pool = k_pool.cpu(), v_pool.cpu()
    block_table, context_lens = block_table.cpu(), context_lens.cpu()
    B, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.empty((B, Hq, D), dtype=torch.float16)
    lse = torch.empty((B, Hq), dtype=torch.float32)
    for b in range(B):
        ctx = int(context_lens[b])
        k = gather_pages(k_pool, block_table[b], ctx).float()
        v = gather_pages(v_pool, block_table[b], ctx).float()
        qb = q[b].float().unsqueeze(1)                # [Hq, 1, D]
        o = F.scaled_dot_product_attention(qb.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0),
                                           scale=scale, enable_gqa=True)
        out[b] = o[0, :, 0].to(torch.float16)
        if return_lse:
            if ctx == 0:
                lse[b] = float("-inf")
            else:
                G = Hq // k.shape[0]
                s = (qb @ k.repeat_interleave(G, 0).transpose(1, 2)) * scale  # [Hq, 1, ctx]
                lse[b] = torch.logsumexp(s[:, 0], dim=-1)
    return (out, lse) if return_lse else out


def sdpa_decomposition_cpu(query, key, value, scale=None):
    """fp32 restatement of spyre__sdpa_overrideable for dense q/k/v [B, H, S, D].

    Returns [B, Hq, Sq, D] fp32.  Follows decompositions.py:549-596: the scale is
    split as sqrt(scale) on q and on k, KV heads are expanded by
    unsqueeze/expand/flatten, then matmul -> softmax -> matmul.
    """
    query, key, value = query.float(), key.float(), value.float()
    hq, hkv = query.shape[1], key.shape[1]
    sf = scale if scale is not None else 1.0 / math.sqrt(query.shape[-1])
    sf = math.sqrt(sf)
    query = query * sf
    key = key * sf
    g = hq // hkv
    if g != 1:
        key = key.unsqueeze(2).expand(-1, -1, g, -1, -1).flatten(1, 2)
        value = value.unsqueeze(2).expand(-1, -1, g, -1, -1).flatten(1, 2)
    attn = torch.softmax(query @ key.transpose(-2, -1), dim=-1)
    return attn @ value
