"""CPU oracle of the head-sharded tensor-parallel decode step (test
infrastructure only: the checker of tests/ and of bench.py's TP parity check).

The TP step is, per rank r, the decode of its KV heads, its o_proj partial
attn_r @ W_o[:, cols_r]^T, and a SUM all-reduce of the partials
(SpyreCCLBackend::allreduce, torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494:
one tensor, ReduceOp SUM).  Summing the partials over every rank is the o_proj
of all heads, so the oracle is the reference's CPU eager decode of all heads
(`decode_attention_cpu`: paged gather + torch CPU SDPA in fp32, output cast to
fp16 as the decode op returns it) followed by the full o_proj in fp32.
"""

from __future__ import annotations

import torch

from .paged_attention import decode_attention_cpu


def tp_step_cpu(q, k_pool, v_pool, block_table, context_lens, w_o, scale=None) -> torch.Tensor:
    """All-reduced o_proj output [B, hidden] in fp32 for every head.

    q [B, Hq, D] fp16, pools [NB, Hkv, S, 64, 64] fp16 with every KV head,
    w_o [hidden, Hq * D] fp16.
    """
    attn = decode_attention_cpu(q, k_pool, v_pool, block_table, context_lens, scale=scale)
    return attn.reshape(attn.shape[0], -1).float() @ w_o.cpu().float().t()
