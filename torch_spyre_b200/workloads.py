"""Seeded synthetic workloads for the paged decode path.

The reference publishes no dataset or benchmark for this path; its tests draw
fp16 N(0, 1) inputs from a generator seeded by a SHA-256 of the call arguments
(``cached_randn`` / ``_make_generator``, tests/inductor/utils_inductor.py:27-50).
`seeded_generator` / `seeded_randn` keep that seeding rule so the reference's
own test shapes (mha_decode / gqa_decode, tests/inductor/test_inductor_ops.py:
2651-2678) are reproduced value for value.

`DECODE_CONFIGS` are the five BASELINE configurations:
  mha_b1     B=1,  32/32 heads, ctx 1024, identity block table
  gqa_b16    B=16, 32/8 heads, ctx U{512..8192}, pool 2x, permuted blocks
  gqa_long   B=4,  32/8 heads, ctx {32k, 64k, 96k, 128k}, pool 2x, permuted
  tp70b      B=128, 64/8 heads, ctx U{1024..4096}, pool 2x, permuted (+ o_proj)
and the relayout/append case `RELAYOUT_CONFIG`.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from typing import Optional

import torch

from .layout import PAGE_TOKENS, pool_shape


def seeded_generator(*args, device: str = "cpu") -> torch.Generator:
    """Generator seeded by the first 32 bits of SHA-256(repr(args))."""
    seed = int(hashlib.sha256(repr(args).encode()).hexdigest()[:8], 16)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def seeded_randn(shape, differentiation=None, abs=False, dtype=torch.float16, scale=1.0) -> torch.Tensor:
    """fp16 N(0, 1) * scale on the CPU, seeded from the arguments (reference rule)."""
    gen = seeded_generator(shape, differentiation, abs, dtype, scale)
    out = torch.randn(shape, dtype=dtype, generator=gen) * scale
    return out if not abs else torch.abs(out)


@dataclass
class DecodeConfig:
    name: str
    batch: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int = 128
    ctx_fixed: Optional[list[int]] = None   # explicit context lengths
    ctx_range: Optional[tuple[int, int]] = None  # uniform integer range (inclusive)
    pool_factor: int = 2                     # pool blocks = factor * blocks needed
    permute: bool = True                     # random block order (else identity)
    hidden: int = 0                          # o_proj width (tp70b only)
    description: str = ""

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads


DECODE_CONFIGS = {
    "mha_b1": DecodeConfig("mha_b1", 1, 32, 32, ctx_fixed=[1024], pool_factor=1, permute=False,
                           description="CPU-runnable MHA decode, B=1, 32/32 heads, ctx 1024"),
    "gqa_b16": DecodeConfig("gqa_b16", 16, 32, 8, ctx_range=(512, 8192),
                            description="GQA decode, B=16, 32/8 heads, ctx U[512, 8192]"),
    "gqa_long": DecodeConfig("gqa_long", 4, 32, 8, ctx_fixed=[32768, 65536, 98304, 131072],
                             description="long-context GQA decode, B=4, ctx 32k..128k"),
    "tp70b": DecodeConfig("tp70b", 128, 64, 8, ctx_range=(1024, 4096), hidden=8192,
                          description="70B-shaped TP decode, B=128, 64/8 heads, ctx U[1024, 4096]"),
}


@dataclass
class RelayoutConfig:
    name: str = "relayout"
    append_tokens: int = 64
    num_kv_heads: int = 8
    head_dim: int = 128
    bulk_tokens: int = 131072


RELAYOUT_CONFIG = RelayoutConfig()


def context_lens_for(cfg: DecodeConfig, seed_tag: str = "") -> list[int]:
    if cfg.ctx_fixed is not None:
        return list(cfg.ctx_fixed)
    lo, hi = cfg.ctx_range
    g = seeded_generator(cfg.name, "ctx", seed_tag)
    return torch.randint(lo, hi + 1, (cfg.batch,), generator=g).tolist()


@dataclass
class DecodeInputs:
    q: torch.Tensor
    k_pool: torch.Tensor
    v_pool: torch.Tensor
    block_table: torch.Tensor
    context_lens: torch.Tensor
    ctx: list[int] = field(default_factory=list)

    k_scale: Optional[torch.Tensor] = None  # fp8 pools: fp16 dequantisation scales
    v_scale: Optional[torch.Tensor] = None

    @property
    def kv_bytes(self) -> int:
        """Algorithmic KV bytes one decode step reads (K and V, valid tokens)."""
        hkv, d = self.k_pool.shape[1], self.k_pool.shape[2] * self.k_pool.shape[4]
        return sum(self.ctx) * hkv * d * 2 * self.k_pool.element_size()

    @property
    def step_bytes(self) -> int:
        """Algorithmic bytes per step: KV + q + out + block-table entries + lens."""
        pages = sum(-(-c // PAGE_TOKENS) for c in self.ctx)
        return self.kv_bytes + 2 * self.q.numel() * 2 + pages * 4 + len(self.ctx) * 4


def make_decode_inputs(
    cfg: DecodeConfig,
    device: str | torch.device = "cpu",
    seed_tag: str = "",
    num_kv_heads: Optional[int] = None,
    ctx: Optional[list[int]] = None,
    batch: Optional[int] = None,
) -> DecodeInputs:
    """Seeded inputs of one decode step of `cfg` (N(0,1) fp16 q / K / V).

    num_kv_heads / batch / ctx override the config (head shards, small cases).
    Blocks are drawn from a pool of pool_factor x the blocks needed; the block
    table is a seeded random permutation of the pool (identity if not permuted).
    """
    device = torch.device(device)
    hkv = num_kv_heads or cfg.num_kv_heads
    hq = hkv * cfg.group
    ctx = list(ctx) if ctx is not None else context_lens_for(cfg, seed_tag)
    if batch is not None:
        ctx = ctx[:batch]
    B = len(ctx)
    pages = [max(1, -(-c // PAGE_TOKENS)) for c in ctx]
    need = sum(pages)
    nb = max(1, need * cfg.pool_factor)
    max_blocks = max(pages)
    gdev = "cuda" if device.type == "cuda" else "cpu"
    gen = seeded_generator(cfg.name, "kv", seed_tag, hkv, tuple(ctx), device=gdev)
    if cfg.permute:
        order = torch.randperm(nb, generator=seeded_generator(cfg.name, "perm", seed_tag, nb))
    else:
        order = torch.arange(nb)
    bt = torch.zeros((B, max_blocks), dtype=torch.int32)
    pos = 0
    for b, n in enumerate(pages):
        bt[b, :n] = order[pos:pos + n].to(torch.int32)
        pos += n
    shape = pool_shape(nb, hkv, cfg.head_dim)
    k_pool = torch.randn(shape, generator=gen, device=device, dtype=torch.float16)
    v_pool = torch.randn(shape, generator=gen, device=device, dtype=torch.float16)
    q = torch.randn((B, hq, cfg.head_dim), generator=gen, device=device, dtype=torch.float16)
    return DecodeInputs(
        q=q,
        k_pool=k_pool,
        v_pool=v_pool,
        block_table=bt.to(device),
        context_lens=torch.tensor(ctx, dtype=torch.int32, device=device),
        ctx=ctx,
    )


# Scale of the seeded fp8 pools: N(0, 1) values stay inside e4m3's +-448 range
# up to 7 sigma (1/64 is exact in fp16).
KV_FP8_SCALE = 1.0 / 64


def quantize_decode_inputs(inp: DecodeInputs, k_scale: float = KV_FP8_SCALE,
                           v_scale: float = KV_FP8_SCALE) -> DecodeInputs:
    """The same step with its pools quantized to fp8 pages (on the pools'
    device, by the library's quantize kernel)."""
    from .fp8 import quantize_pool

    dev = inp.k_pool.device
    ks = torch.tensor([k_scale], dtype=torch.float16, device=dev)
    vs = torch.tensor([v_scale], dtype=torch.float16, device=dev)
    return DecodeInputs(q=inp.q, k_pool=quantize_pool(inp.k_pool, ks), v_pool=quantize_pool(inp.v_pool, vs),
                        block_table=inp.block_table, context_lens=inp.context_lens, ctx=list(inp.ctx),
                        k_scale=ks, v_scale=vs)
