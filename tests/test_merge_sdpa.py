"""Split-KV merge (b200kv_lse_combine_f32) and the SDPA-overrideable drop-in
(the reference decomposition's signature and 9-tuple,
torch_spyre/_inductor/decompositions.py:523-611)."""

import numpy as np
import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import paged_attention as opa
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs, seeded_randn

ATOL, RTOL = 2e-3, 1e-2


def test_overrideable_rejects_unsupported_cases():
    q = torch.zeros(1, 4, 1, 128, dtype=torch.float16)
    k = torch.zeros(1, 4, 8, 128, dtype=torch.float16)
    f = tsb.scaled_dot_product_fused_attention_overrideable
    with pytest.raises(NotImplementedError, match="dropout"):
        f(q, k, k, dropout_p=0.1)
    with pytest.raises(NotImplementedError, match="bias"):
        f(q, k, k, attn_bias=torch.zeros(1))
    with pytest.raises(NotImplementedError, match="decode"):
        f(torch.zeros(1, 4, 2, 128, dtype=torch.float16), k, k)
    with pytest.raises(NotImplementedError, match="causal"):
        f(q, k, k, is_causal=True)


def test_merge_rejects_cpu_and_mismatch():
    with pytest.raises(RuntimeError, match="CUDA"):
        tsb.merge_attention_states([torch.zeros(2, 128)], [torch.zeros(2)])
    with pytest.raises(ValueError):
        tsb.merge_attention_states([torch.zeros(2, 128)], [])


@pytest.mark.gpu
@pytest.mark.parametrize("split_pages", [0, 1, 3, 40])
def test_prefix_suffix_merge_equals_full_decode(split_pages):
    ctx = [1, 64, 65, 300, 2600, 4097, 0, 129]
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=ctx, seed_tag="merge")
    ctx_t = inp.context_lens
    cut = split_pages * 64
    ctx_a = torch.clamp(ctx_t, max=cut)
    ctx_b = torch.clamp(ctx_t - cut, min=0)
    bt = inp.block_table
    bt_a = bt[:, :max(split_pages, 1)].contiguous()
    bt_b = bt[:, split_pages:].contiguous() if split_pages < bt.shape[1] else bt[:, :1].contiguous()
    oa, la = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, bt_a, ctx_a.to(torch.int32), return_lse=True)
    ob, lb = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, bt_b, ctx_b.to(torch.int32), return_lse=True)
    out, lse = tsb.merge_attention_states([oa, ob], [la, lb])
    ref, ref_lse = opa.decode_attention_cpu(inp.q, inp.k_pool, inp.v_pool, bt, ctx_t, return_lse=True)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=1e-3, rtol=1e-4)
    # fp32 parts, three of them (an empty middle part changes nothing)
    empty = torch.full_like(la, float("-inf"))
    out3, _ = tsb.merge_attention_states([oa.float(), torch.zeros_like(oa).float(), ob.float()], [la, empty, lb])
    torch.testing.assert_close(out3.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)


@pytest.mark.gpu
@pytest.mark.parametrize("case,hkv", [("mha_decode", 32), ("gqa_decode", 8)])
def test_overrideable_matches_reference_golden(golden_dir, case, hkv):
    g = np.load(golden_dir / "sdpa_decode_golden.npz")
    q = seeded_randn((2, 1, 32, 128), 1).transpose(1, 2).cuda()
    k = seeded_randn((2, 257, hkv, 128), 2).transpose(1, 2).cuda()
    v = seeded_randn((2, 257, hkv, 128), 3).transpose(1, 2).cuda()
    res = tsb.scaled_dot_product_fused_attention_overrideable(q, k, v)
    assert len(res) == 9
    out, lse, cq, ck, max_q, max_k, seed, offset, dbg = res
    assert out.shape == (2, 32, 1, 128) and out.transpose(1, 2).is_contiguous()
    assert (cq, ck, dbg) == (None, None, None) and (max_q, max_k) == (1, 257)
    assert lse.shape == (2, 32, 1) and seed.shape == (1,) and offset.shape == (1,)
    torch.testing.assert_close(out.cpu().float(), torch.from_numpy(g[f"{case}_out_fp32"]), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu()[:, :, 0], torch.from_numpy(g[f"{case}_lse"]), atol=1e-3, rtol=1e-4)
