"""Head-sharded tensor-parallel decode step (one process per GPU).

Rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N), the G query heads of each,
their KV pages (a per-rank pool with only those heads) and the matching input
columns of the output projection W_o.  A step is

    attn_r    = decode_attention(q[:, heads_r], k_pool_r, v_pool_r, ...)   # [B, Hq/N, D]
    partial_r = attn_r.reshape(B, -1) @ W_o[:, cols_r]^T                   # [B, hidden]
    y         = all_reduce_SUM(partial_r)                                  # NCCL

The all-reduce is the reference's tensor-parallel collective: a synchronous
SUM all-reduce of one tensor (SpyreCCLBackend::allreduce,
torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494), here over NCCL on
NVLink/NVSwitch.  The block table and context lengths are replicated.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch


@dataclass(frozen=True)
class HeadShard:
    """The heads and W_o columns one rank owns."""

    rank: int
    world: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int

    def __post_init__(self):
        if self.num_kv_heads % self.world:
            raise ValueError(f"{self.num_kv_heads} KV heads do not split over {self.world} ranks")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world {self.world}")

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    @property
    def kv_heads(self) -> range:
        n = self.num_kv_heads // self.world
        return range(self.rank * n, (self.rank + 1) * n)

    @property
    def q_heads(self) -> range:
        kv = self.kv_heads
        return range(kv.start * self.group, kv.stop * self.group)

    @property
    def w_cols(self) -> slice:
        q = self.q_heads
        return slice(q.start * self.head_dim, q.stop * self.head_dim)

    def shard_q(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of q [B, Hq, D] (a strided view, no copy)."""
        return q[:, self.q_heads.start:self.q_heads.stop]

    def shard_pool(self, pool: torch.Tensor) -> torch.Tensor:
        """This rank's KV heads of a full pool [NB, Hkv, S, 64, 64] (a copy)."""
        return pool[:, self.kv_heads.start:self.kv_heads.stop].contiguous()

    def shard_w_o(self, w_o: torch.Tensor) -> torch.Tensor:
        """This rank's input columns of W_o [hidden_out, Hq * D]."""
        return w_o[:, self.w_cols].contiguous()


AttnFn = Callable[..., torch.Tensor]


def tp_decode_step(
    shard: HeadShard,
    q_local: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    w_o_local: torch.Tensor,
    group=None,
    out: Optional[torch.Tensor] = None,
    attn_fn: Optional[AttnFn] = None,
    k_scale: Optional[torch.Tensor] = None,
    v_scale: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One rank's step: local decode -> o_proj partial -> SUM all-reduce.

    attn_fn defaults to the CUDA decode op; tests on CPU ranks pass the oracle.
    k_scale / v_scale are the dequantisation scales of fp8 pools.
    Every rank must call this in the same order (it contains one collective).
    """
    if attn_fn is None:
        from .ops import decode_attention as attn_fn
    if k_scale is not None:
        attn = attn_fn(q_local, k_pool, v_pool, block_table, context_lens, k_scale=k_scale, v_scale=v_scale)
    else:
        attn = attn_fn(q_local, k_pool, v_pool, block_table, context_lens)
    B = attn.shape[0]
    flat = attn.reshape(B, -1)
    if out is not None:
        partial = torch.matmul(flat, w_o_local.t(), out=out)
    else:
        partial = torch.matmul(flat, w_o_local.t())
    if shard.world > 1:
        import torch.distributed as dist

        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
