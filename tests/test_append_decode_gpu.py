"""Fused KV append + decode against the two-step path and the oracle.

The reference's decode step is the HF cache write ``cache.index_copy_``
(torch_spyre/ops/fallbacks.py:256; tests/inductor/test_inductor_ops.py:5715-5740)
followed by SDPA; the fused op must leave the pools bit-identical to
``kv_append`` at slot (block_table[b][(len-1)//64], (len-1) % 64) and return the
same output as ``decode_attention`` afterwards.
"""

import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import paged_attention as opa
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs

pytestmark = pytest.mark.gpu


def _two_step(inp, k_new, v_new, num_splits):
    kp, vp = inp.k_pool.clone(), inp.v_pool.clone()
    pos = inp.context_lens.long() - 1
    slots = tsb.layout.slot_of(inp.block_table, pos)
    tsb.kv_append(k_new, v_new, kp, vp, slots)
    out, lse = tsb.decode_attention(inp.q, kp, vp, inp.block_table, inp.context_lens, num_splits=num_splits,
                                    return_lse=True)
    return kp, vp, out, lse


@pytest.mark.parametrize("name,hkv", [("gqa_b16", 8), ("tp70b", 8), ("mha_b1", 32), ("gqa_b16", 16)])
@pytest.mark.parametrize("splits", [0, 1, 200])
def test_fused_equals_two_step(name, hkv, splits):
    cfg = DECODE_CONFIGS[name]
    ctx = [1, 63, 64, 65, 128, 129, 700, 4097] if name != "mha_b1" else [1024]
    inp = make_decode_inputs(cfg, device="cuda", ctx=ctx, num_kv_heads=hkv if name != "mha_b1" else None,
                             seed_tag="append")
    B, hkvv = len(ctx), inp.k_pool.shape[1]
    k_new = torch.randn((B, hkvv, 128), device="cuda", dtype=torch.float16)
    v_new = torch.randn_like(k_new)
    kp2, vp2, out2, lse2 = _two_step(inp, k_new, v_new, splits)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = tsb.decode_attention_append(inp.q, k_new, v_new, inp.k_pool, inp.v_pool, inp.block_table,
                                           inp.context_lens, num_splits=splits, return_lse=True, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    assert torch.equal(inp.k_pool.view(torch.int16), kp2.view(torch.int16))
    assert torch.equal(inp.v_pool.view(torch.int16), vp2.view(torch.int16))
    torch.testing.assert_close(out, out2, atol=0, rtol=0)
    torch.testing.assert_close(lse, lse2, atol=0, rtol=0)
    ref = opa.decode_attention_cpu(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-3, rtol=1e-2)


def test_fused_strided_new_rows():
    """k_new / v_new as views of a fused qkv projection [B, 3, Hkv, D]."""
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=[5, 300, 64], seed_tag="append2")
    qkv = torch.randn((3, 3, 8, 128), device="cuda", dtype=torch.float16)
    k_new, v_new = qkv[:, 1], qkv[:, 2]
    kp2, vp2, out2, _ = _two_step(inp, k_new, v_new, 0)
    out = tsb.decode_attention_append(inp.q, k_new, v_new, inp.k_pool, inp.v_pool, inp.block_table,
                                      inp.context_lens)
    assert torch.equal(inp.k_pool.view(torch.int16), kp2.view(torch.int16))
    torch.testing.assert_close(out, out2, atol=0, rtol=0)


def test_fused_bad_block_skips_write_and_flags():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=[100, 30], seed_tag="append3")
    inp.block_table[0, 1] = inp.k_pool.shape[0] + 3  # page of token 99
    before = inp.k_pool.clone()
    k_new = torch.randn((2, 8, 128), device="cuda", dtype=torch.float16)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.decode_attention_append(inp.q, k_new, k_new, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens,
                                error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.DEVERR_BAD_BLOCK
    blk1 = int(inp.block_table[1, 0])
    changed = (inp.k_pool != before).any(dim=(1, 2, 3, 4)).nonzero().flatten().tolist()
    assert changed == [blk1]  # only sequence 1's append landed


def test_fused_early_start_same_bits():
    """B200KV_DECODE_INPUTS_READY on the fused append: alternating two pool
    sets (so no call's pools are written by the call right before it), the
    outputs and the pools equal the default launches bit for bit."""
    cfg = DECODE_CONFIGS["gqa_b16"]
    ctx = [1, 63, 64, 65, 700, 4097]

    def run(ready):
        sets = [make_decode_inputs(cfg, device="cuda", ctx=ctx, seed_tag=f"early-append{i}") for i in range(2)]
        g = torch.Generator(device="cuda").manual_seed(5)
        outs = []
        for step in range(6):
            s = sets[step % 2]
            k_new = torch.randn((len(ctx), 8, 128), generator=g, device="cuda", dtype=torch.float16)
            v_new = torch.randn((len(ctx), 8, 128), generator=g, device="cuda", dtype=torch.float16)
            outs.append(tsb.decode_attention_append(s.q, k_new, v_new, s.k_pool, s.v_pool, s.block_table,
                                                    s.context_lens, inputs_ready=ready))
        torch.cuda.synchronize()
        return outs, sets

    ref, ref_sets = run(False)
    got, got_sets = run(True)
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    for a, b in zip(ref_sets, got_sets):
        assert torch.equal(a.k_pool.view(torch.int16), b.k_pool.view(torch.int16))
        assert torch.equal(a.v_pool.view(torch.int16), b.v_pool.view(torch.int16))
