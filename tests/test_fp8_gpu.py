"""GPU parity of the fp8 (e4m3) ops and fp8 KV pages.

* quantize / dequantize: bit-exact against the CPU restatement of the
  reference's decompositions, on the reference's own test cases
  (tests/inductor/test_fp8_operations.py:124-272) plus per-row scales, odd
  widths and out-of-range values; and within the reference's tolerances of its
  own CPU formula.
* fp8 append: bit-exact against the oracle's quantized slot write.
* fp8 decode: against the CPU decode oracle run on the dequantized pools
  (fp16(q8) * scale), tolerance 2e-3 absolute + 1e-2 relative (BASELINE
  north_star); the kernel applies the scales in fp32 instead of rounding each
  dequantized element to fp16.
"""

import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import fp8_quant as o8
from oracle import paged_attention as opa
from torch_spyre_b200 import _lib
from torch_spyre_b200.fp8 import dequantize_pool
from torch_spyre_b200.workloads import (DECODE_CONFIGS, make_decode_inputs, quantize_decode_inputs,
                                        seeded_randn)

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
FP8 = torch.float8_e4m3fn

CASES = ([((1, 2, 32), s, 0.0, std, 2.0) for s in (0.01, 0.1, 0.5, 1.0, 2.0) for std in (1.0, 5.0)]
         + [((1, 2, 32), s, 10.0, 50.0, 16.0) for s in (0.01, 0.1, 0.5, 1.0, 2.0)]
         + [((1, 2, 32), s, m, m, 32.0 * s) for s in (0.01, 0.1, 0.5, 1.0, 2.0) for m in (100.0, 200.0)])


def _bits(t):
    return t.view(torch.uint8) if t.dtype == FP8 else t.view(torch.int16)


@pytest.mark.parametrize("shape,scale,mean,std,atol", CASES)
def test_quantize_dequantize_reference_cases(shape, scale, mean, std, atol):
    x = seeded_randn(shape, dtype=torch.float16, scale=1.0) * std + mean
    s = torch.tensor([scale], dtype=torch.float16)
    q = tsb.quantize_fp8_with_scale(x.cuda(), s.cuda())
    assert q.dtype == FP8
    assert torch.equal(_bits(q.cpu()), _bits(o8.quantize_fp8_with_scale(x, s)))
    y = tsb.dequantize_fp8_with_scale(q, s.cuda())
    assert y.dtype == torch.float16
    assert torch.equal(_bits(y.cpu()), _bits(o8.dequantize_fp8_with_scale(q.cpu(), s)))
    torch.testing.assert_close(y.cpu(), o8.reference_roundtrip(x, s), atol=atol, rtol=0.0)


@pytest.mark.parametrize("shape", [(1, 128, 512), (4, 128, 512), (1, 128, 1024), (1, 128, 2048), (1, 128, 4096)])
def test_quantize_dequantize_production_shapes(shape):
    x = seeded_randn(shape, dtype=torch.float16, scale=1.0) * 2.0 + 1.0
    s = torch.tensor([1.0], dtype=torch.float16)
    y = tsb.dequantize_fp8_with_scale(tsb.quantize_fp8_with_scale(x.cuda(), s.cuda()), s.cuda()).cpu()
    assert torch.equal(_bits(y), _bits(o8.dequantize_fp8_with_scale(o8.quantize_fp8_with_scale(x, s), s)))
    torch.testing.assert_close(y, o8.reference_roundtrip(x, s), atol=0.5, rtol=0.1)


@pytest.mark.parametrize("cols", [1, 7, 8, 33, 128, 4096])
def test_per_row_scale_and_odd_widths(cols):
    g = torch.Generator().manual_seed(cols)
    x = (torch.randn((3, 5, cols), generator=g) * 300).to(torch.float16)  # beyond +-448 / scale too
    s = (torch.rand((3, 5, 1), generator=g) * 2 + 0.01).to(torch.float16)
    q = tsb.quantize_fp8_with_scale(x.cuda(), s.cuda())
    assert torch.equal(_bits(q.cpu()), _bits(o8.quantize_fp8_with_scale(x, s)))
    y = tsb.dequantize_fp8_with_scale(q, s.cuda())
    assert torch.equal(_bits(y.cpu()), _bits(o8.dequantize_fp8_with_scale(q.cpu(), s)))


def test_every_fp16_value():
    """All 65536 fp16 bit patterns except NaNs, at three scales."""
    x = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.float16)
    x = x[~torch.isnan(x)].reshape(1, -1)
    for scale in (1.0, 0.0999755859375, 7.5):
        s = torch.tensor([scale], dtype=torch.float16)
        q = tsb.quantize_fp8_with_scale(x.cuda(), s.cuda())
        assert torch.equal(_bits(q.cpu()), _bits(o8.quantize_fp8_with_scale(x, s))), scale


def test_every_e4m3_value():
    q = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(FP8)
    q = q[~torch.isnan(q.float())].reshape(1, -1)
    for scale in (1.0, 0.015625, 3.3):
        s = torch.tensor([scale], dtype=torch.float16)
        y = tsb.dequantize_fp8_with_scale(q.cuda(), s.cuda())
        assert torch.equal(_bits(y.cpu()), _bits(o8.dequantize_fp8_with_scale(q, s))), scale


def test_quantize_pool_matches_oracle():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", batch=3)
    q8 = quantize_decode_inputs(inp)
    ref = o8.pool_from_fp16_pool(inp.k_pool.cpu(), q8.k_scale.cpu())
    assert torch.equal(_bits(q8.k_pool.cpu()), _bits(ref))
    back = dequantize_pool(q8.k_pool, q8.k_scale)
    assert torch.equal(_bits(back.cpu()), _bits(o8.fp16_pool_from_pool(ref, q8.k_scale.cpu())))


def test_kv_append_fp8_bit_exact():
    nb, hkv = 6, 8
    g = torch.Generator().manual_seed(3)
    k_pool = torch.randint(0, 120, (nb, hkv, 1, 64, 128), generator=g, dtype=torch.uint8).view(FP8)
    v_pool = torch.randint(0, 120, (nb, hkv, 1, 64, 128), generator=g, dtype=torch.uint8).view(FP8)
    k_new = (torch.randn((5, hkv, 128), generator=g) * 4).to(torch.float16)
    v_new = (torch.randn((5, hkv, 128), generator=g) * 4).to(torch.float16)
    slots = torch.tensor([0, 65, -1, 383, 200], dtype=torch.int64)
    ks = torch.tensor([0.02], dtype=torch.float16)
    vs = torch.tensor([0.5], dtype=torch.float16)
    kd, vd = k_pool.cuda(), v_pool.cuda()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.kv_append(k_new.cuda(), v_new.cuda(), kd, vd, slots.cuda(), error_flag=flag, k_scale=ks.cuda(),
                  v_scale=vs.cuda())
    assert int(flag.item()) == 0
    assert torch.equal(_bits(kd.cpu()), _bits(o8.append(k_new, k_pool, slots, ks)))
    assert torch.equal(_bits(vd.cpu()), _bits(o8.append(v_new, v_pool, slots, vs)))
    bad = torch.tensor([nb * 64], dtype=torch.int64, device="cuda")
    tsb.kv_append(k_new[:1].cuda(), v_new[:1].cuda(), kd, vd, bad, error_flag=flag, k_scale=ks.cuda(),
                  v_scale=vs.cuda())
    assert int(flag.item()) & _lib.DEVERR_BAD_SLOT


def _poison_tail8(inp):
    """e4m3 NaN (0x7f) in every pool slot no sequence owns."""
    used = torch.zeros(inp.k_pool.shape[0], 64, dtype=torch.bool)
    bt = inp.block_table.cpu()
    for b, c in enumerate(inp.ctx):
        for p in range(-(-c // 64)):
            used[int(bt[b, p]), :min(64, c - 64 * p)] = True
    mask = (~used).to(inp.k_pool.device)[:, None, None, :, None].expand(inp.k_pool.shape)
    for pool in (inp.k_pool, inp.v_pool):
        pool.view(torch.uint8).masked_fill_(mask, 0x7F)


def _check8(inp, num_splits=0, poison=True):
    if poison:
        _poison_tail8(inp)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens,
                                    num_splits=num_splits, return_lse=True, error_flag=flag,
                                    k_scale=inp.k_scale, v_scale=inp.v_scale)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    ks, vs = inp.k_scale.cpu(), inp.v_scale.cpu()
    k16 = o8.fp16_pool_from_pool(inp.k_pool.cpu(), ks)
    v16 = o8.fp16_pool_from_pool(inp.v_pool.cpu(), vs)
    ref, ref_lse = opa.decode_attention_cpu(inp.q, k16, v16, inp.block_table, inp.context_lens, return_lse=True)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=1e-3, rtol=1e-4)
    return out


@pytest.mark.parametrize("name", ["mha_b1", "gqa_b16", "tp70b"])
def test_config_parity_fp8(name):
    inp = quantize_decode_inputs(make_decode_inputs(DECODE_CONFIGS[name], device="cuda"))
    _check8(inp)


@pytest.mark.parametrize("group", [1, 2, 4, 8])
@pytest.mark.parametrize("splits", [1, 4, 64, 1000])
def test_groups_and_splits_fp8(group, splits):
    ctx = [1, 63, 64, 65, 257, 1000, 4097, 0]
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=ctx, num_kv_heads=32 // group,
                             seed_tag=f"g{group}")
    inp.q = torch.randn((len(ctx), 32, 128), device="cuda", dtype=torch.float16)
    _check8(quantize_decode_inputs(inp, k_scale=0.03, v_scale=0.01), num_splits=splits)


def test_fp8_matches_fp16_kernel_on_dequantized_pools():
    inp = quantize_decode_inputs(make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", seed_tag="x"))
    out8 = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens,
                                k_scale=inp.k_scale, v_scale=inp.v_scale)
    out16 = tsb.decode_attention(inp.q, dequantize_pool(inp.k_pool, inp.k_scale),
                                 dequantize_pool(inp.v_pool, inp.v_scale), inp.block_table, inp.context_lens)
    torch.testing.assert_close(out8.float(), out16.float(), atol=1e-3, rtol=5e-3)


def test_fused_append_fp8_matches_two_step():
    ctx = [1, 64, 65, 300, 4096, 4097]
    base = make_decode_inputs(DECODE_CONFIGS["tp70b"], device="cuda", ctx=ctx, num_kv_heads=2, seed_tag="app8")
    inp = quantize_decode_inputs(base, k_scale=0.02, v_scale=0.04)
    B, hkv = len(ctx), 2
    k_new = torch.randn((B, hkv, 128), device="cuda", dtype=torch.float16)
    v_new = torch.randn((B, hkv, 128), device="cuda", dtype=torch.float16)
    kp2, vp2 = inp.k_pool.clone(), inp.v_pool.clone()
    out, lse = tsb.decode_attention_append(inp.q, k_new, v_new, inp.k_pool, inp.v_pool, inp.block_table,
                                           inp.context_lens, return_lse=True, k_scale=inp.k_scale,
                                           v_scale=inp.v_scale)
    pos = inp.context_lens.long() - 1
    slots = inp.block_table.long().gather(1, (pos // 64)[:, None])[:, 0] * 64 + pos % 64
    tsb.kv_append(k_new, v_new, kp2, vp2, slots, k_scale=inp.k_scale, v_scale=inp.v_scale)
    ref, ref_lse = tsb.decode_attention(inp.q, kp2, vp2, inp.block_table, inp.context_lens, return_lse=True,
                                        k_scale=inp.k_scale, v_scale=inp.v_scale)
    assert torch.equal(_bits(inp.k_pool), _bits(kp2)) and torch.equal(_bits(inp.v_pool), _bits(vp2))
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse)


def test_fp8_graph_capture_and_repeat():
    inp = quantize_decode_inputs(make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", batch=6))
    args = (inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)
    kw = dict(k_scale=inp.k_scale, v_scale=inp.v_scale, num_splits=16)
    eager = tsb.decode_attention(*args, **kw)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tsb.decode_attention(*args, **kw)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = tsb.decode_attention(*args, **kw)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_bad_block_id_sets_flag_fp8():
    inp = quantize_decode_inputs(make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", batch=2))
    inp.block_table[1, 0] = inp.k_pool.shape[0] + 5
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens, error_flag=flag,
                         k_scale=inp.k_scale, v_scale=inp.v_scale)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.DEVERR_BAD_BLOCK
