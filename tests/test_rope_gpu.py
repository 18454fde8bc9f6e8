"""GPU parity of the rotary embedding: the standalone op bit-exact against the
oracle (itself pinned to the reference's dataflow, test_rope_cpu.py), and the
fused append + decode with RoPE identical to rope -> fused append + decode."""

import json

import numpy as np
import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import paged_attention as opa
from oracle import rope as orope
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs, quantize_decode_inputs, seeded_randn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["prefill_bs1", "prefill", "decode_bs1", "decode"])
def test_rope_op_matches_reference_cases(golden_dir, name):
    meta = json.loads((golden_dir / "rope_golden.json").read_text())[name]
    q = seeded_randn(tuple(meta["q_shape"]), dtype=torch.float16)
    freqs = seeded_randn(tuple(meta["freqs_shape"]), dtype=torch.float16)
    B, S, E = q.shape
    D = freqs.shape[-1] * 2
    rows = q.reshape(B * S, E // D, D)
    pos = torch.arange(S, dtype=torch.int32).repeat(B)
    out = tsb.rope(rows.cuda(), freqs.cuda(), pos.cuda()).cpu()
    assert torch.equal(out.view(torch.int16), orope.rope_rows(rows, freqs[0], pos).view(torch.int16))
    if S == 1:
        gold = np.load(golden_dir / "rope_golden.npz")[f"{name}_out"]
        assert torch.equal(out.reshape(meta["out_shape"]).view(torch.int16), torch.from_numpy(gold).view(torch.int16))


def test_rope_strided_rows_and_bad_position():
    g = torch.Generator().manual_seed(5)
    big = torch.randn(6, 40, 128, generator=g).to(torch.float16)
    x = big[:, 8:16]  # a head shard: strided rows
    freqs = torch.randn(32, 2, 2, 64, generator=g).to(torch.float16)
    pos = torch.tensor([0, 31, 7, 7, 3, 30], dtype=torch.int32)
    out = tsb.rope(x.cuda(), freqs.cuda(), pos.cuda()).cpu()
    assert torch.equal(out, orope.rope_rows(x, freqs, pos))
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.rope(x.cuda(), freqs.cuda(), torch.tensor([0, 32, 1, 1, 1, 1], dtype=torch.int32, device="cuda"),
             error_flag=flag)
    assert int(flag.item()) & _lib.DEVERR_BAD_LEN


def _freqs(max_pos, seed=9):
    # genuine rotations cos/sin of position * theta_j, as fp16 2x2 matrices
    j = torch.arange(64, dtype=torch.float64)
    theta = 10000.0 ** (-j / 64)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * theta
    c, s = torch.cos(ang), torch.sin(ang)
    f = torch.stack([torch.stack([c, -s], 1), torch.stack([s, c], 1)], 1)  # [P, 2, 2, 64]
    return f.to(torch.float16)


@pytest.mark.parametrize("kv", ["fp16", "fp8"])
def test_fused_rope_append_decode_matches_two_step(kv):
    ctx = [1, 64, 65, 300, 4096, 4097]
    base = make_decode_inputs(DECODE_CONFIGS["tp70b"], device="cuda", ctx=ctx, num_kv_heads=2, seed_tag="rope")
    inp = quantize_decode_inputs(base, k_scale=0.03, v_scale=0.03) if kv == "fp8" else base
    B, hkv = len(ctx), 2
    k_new = torch.randn((B, hkv, 128), device="cuda", dtype=torch.float16)
    v_new = torch.randn((B, hkv, 128), device="cuda", dtype=torch.float16)
    freqs = _freqs(5000).cuda()
    kp2, vp2 = inp.k_pool.clone(), inp.v_pool.clone()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = tsb.decode_attention_append(inp.q, k_new, v_new, inp.k_pool, inp.v_pool, inp.block_table,
                                           inp.context_lens, return_lse=True, k_scale=inp.k_scale,
                                           v_scale=inp.v_scale, rope_freqs=freqs, error_flag=flag)
    pos = inp.context_lens - 1
    q_rot = tsb.rope(inp.q, freqs, pos)
    k_rot = tsb.rope(k_new, freqs, pos)
    ref, ref_lse = tsb.decode_attention_append(q_rot, k_rot, v_new, kp2, vp2, inp.block_table, inp.context_lens,
                                               return_lse=True, k_scale=inp.k_scale, v_scale=inp.v_scale)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    bits = (lambda t: t.view(torch.uint8)) if kv == "fp8" else (lambda t: t.view(torch.int16))
    assert torch.equal(bits(inp.k_pool), bits(kp2)) and torch.equal(bits(inp.v_pool), bits(vp2))
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
    if kv == "fp16":  # and against the CPU oracle: rope, append, attention
        q_o = orope.rope_rows(inp.q.cpu(), freqs.cpu(), pos.cpu())
        oracle_out = opa.decode_attention_cpu(q_o, kp2.cpu(), vp2.cpu(), inp.block_table, inp.context_lens)
        torch.testing.assert_close(out.cpu().float(), oracle_out.float(), atol=2e-3, rtol=1e-2)
        k_o = orope.rope_rows(k_new.cpu(), freqs.cpu(), pos.cpu())
        assert torch.equal(k_o, k_rot.cpu())
