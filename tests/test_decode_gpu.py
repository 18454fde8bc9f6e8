"""GPU parity of the paged decode kernel against the CPU oracle.

Tolerance: 2e-3 absolute + 1e-2 relative on the fp16
output versus the reference's CPU eager path in fp32; LSE within 1e-3.
"""

import json

import numpy as np
import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import kv_relayout as okv
from oracle import paged_attention as opa
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs, seeded_randn

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _poison_tail(inp):
    """NaN every pool slot no sequence owns (unused blocks and the slots past
    ctx in each last page) so reading one would show in the output."""
    used = torch.zeros(inp.k_pool.shape[0], 64, dtype=torch.bool)
    bt = inp.block_table.cpu()
    for b, c in enumerate(inp.ctx):
        for p in range(-(-c // 64)):
            n = min(64, c - 64 * p)
            used[int(bt[b, p]), :n] = True
    mask = (~used).to(inp.k_pool.device)[:, None, None, :, None].expand_as(inp.k_pool)
    inp.k_pool.masked_fill_(mask, float("nan"))
    inp.v_pool.masked_fill_(mask, float("nan"))


def _check(inp, num_splits=0, poison=True):
    if poison:
        _poison_tail(inp)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, lse = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens,
                                    num_splits=num_splits, return_lse=True, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    ref, ref_lse = opa.decode_attention_cpu(inp.q, inp.k_pool, inp.v_pool, inp.block_table,
                                            inp.context_lens, return_lse=True)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), ref_lse, atol=1e-3, rtol=1e-4)
    return out


@pytest.mark.parametrize("case,hkv", [("mha_decode", 32), ("gqa_decode", 8)])
def test_reference_decode_golden(golden_dir, case, hkv):
    """The reference's own decode inputs (ctx 257: partial last page)."""
    g = np.load(golden_dir / "sdpa_decode_golden.npz")
    q = seeded_randn((2, 1, 32, 128), 1).transpose(1, 2)
    k = seeded_randn((2, 257, hkv, 128), 2)
    v = seeded_randn((2, 257, hkv, 128), 3)
    ids = torch.tensor([[9, 2, 7, 0, 5], [1, 8, 3, 6, 4]], dtype=torch.int32)
    kp = torch.full((10, hkv, 2, 64, 64), float("nan"), dtype=torch.float16)
    vp = kp.clone()
    kpn, vpn = kp.numpy(), vp.numpy()
    for b in range(2):
        kpn = okv.rows_to_pool(k[b].numpy(), kpn, ids[b].numpy())
        vpn = okv.rows_to_pool(v[b].numpy(), vpn, ids[b].numpy())
    out, lse = tsb.decode_attention(q[:, :, 0].contiguous().cuda(), torch.from_numpy(kpn).cuda(),
                                    torch.from_numpy(vpn).cuda(), ids.cuda(),
                                    torch.full((2,), 257, dtype=torch.int32, device="cuda"), return_lse=True)
    ref = torch.from_numpy(g[f"{case}_out_fp32"])[:, :, 0]
    torch.testing.assert_close(out.cpu().float(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), torch.from_numpy(g[f"{case}_lse"]), atol=1e-3, rtol=1e-4)


def test_sdpa_adapter_matches_golden(golden_dir):
    g = np.load(golden_dir / "sdpa_decode_golden.npz")
    q = seeded_randn((2, 1, 32, 128), 1).transpose(1, 2).cuda()
    k = seeded_randn((2, 257, 8, 128), 2).transpose(1, 2).cuda()
    v = seeded_randn((2, 257, 8, 128), 3).transpose(1, 2).cuda()
    out = tsb.sdpa_decode(q, k, v, enable_gqa=True)
    assert out.shape == (2, 32, 1, 128)
    assert out.transpose(1, 2).is_contiguous()  # the reference's [B, S, H, D] memory order
    torch.testing.assert_close(out.cpu().float(), torch.from_numpy(g["gqa_decode_out_fp32"]), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["mha_b1", "gqa_b16", "tp70b"])
def test_config_parity(name):
    inp = make_decode_inputs(DECODE_CONFIGS[name], device="cuda")
    _check(inp)


@pytest.mark.slow
def test_long_context_parity():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_long"], device="cuda")
    _check(inp, poison=False)


@pytest.mark.parametrize("group", [1, 2, 4, 8])
@pytest.mark.parametrize("splits", [1, 4, 64, 1000])
def test_groups_and_splits(group, splits):
    cfg = DECODE_CONFIGS["gqa_b16"]
    ctx = [1, 63, 64, 65, 257, 1000, 4097, 0]
    inp = make_decode_inputs(cfg, device="cuda", ctx=ctx, num_kv_heads=32 // group, seed_tag=f"g{group}")
    # keep q's heads = Hkv * group
    inp.q = torch.randn((len(ctx), (32 // group) * group, 128), device="cuda", dtype=torch.float16)
    _check(inp, num_splits=splits)


def test_strided_q_and_out_shard():
    """A head shard of q (a strided view, as a tensor-parallel rank passes it)."""
    inp = make_decode_inputs(DECODE_CONFIGS["tp70b"], device="cuda", ctx=[300, 2000, 64, 4096],
                             num_kv_heads=2)
    full_q = torch.randn(4, 64, 128, device="cuda", dtype=torch.float16)
    inp.q = full_q[:, 16:32]  # heads of KV heads 2..3 in a 64-head model
    assert not inp.q.is_contiguous()
    _check(inp)


def test_repeat_calls_are_identical_and_workspace_resets():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda")
    a = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens, num_splits=8)
    b = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens, num_splits=8)
    assert torch.equal(a, b)
    ws = tsb.ops._workspaces
    for t in ws.values():
        counters = t[: 16 * 8 * 4].view(torch.int32)
        assert int(counters.abs().sum()) == 0


def test_bad_block_id_sets_flag_without_fault():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=[100, 200], batch=2)
    inp.block_table[1, 0] = inp.k_pool.shape[0] + 5
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.DEVERR_BAD_BLOCK


def test_context_beyond_table_sets_flag():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=[100, 200], batch=2)
    inp.context_lens[0] = 10_000
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.DEVERR_BAD_LEN


def test_cuda_graph_capture():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda")
    eager = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_simt_kernel_variant_parity():
    """The CUDA-core variant (B200KV_DECODE_KERNEL=simt, read once per process)."""
    import os
    import subprocess
    import sys

    code = (
        "import torch, torch_spyre_b200 as tsb\n"
        "from oracle import paged_attention as opa\n"
        "from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs\n"
        "for name, ctx in (('gqa_b16', [1, 65, 257, 3000]), ('tp70b', [64, 129, 4096, 7])):\n"
        "    inp = make_decode_inputs(DECODE_CONFIGS[name], device='cuda', ctx=ctx)\n"
        "    out = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)\n"
        "    ref = opa.decode_attention_cpu(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)\n"
        "    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-3, rtol=1e-2)\n"
        "print('simt ok')\n"
    )
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, B200KV_DECODE_KERNEL="simt", PYTHONPATH=repo)
    r = subprocess.run([sys.executable, "-c", code], env=env, cwd=repo, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "simt ok" in r.stdout, r.stderr[-3000:]


@pytest.mark.parametrize("name,hkv", [("gqa_b16", None), ("tp70b", 1), ("mha_b1", None)])
def test_early_start_gives_the_same_bits(name, hkv):
    """B200KV_DECODE_INPUTS_READY: plan and first page loads before the wait
    for the preceding kernel.  Chained decodes where each one's q is the
    previous one's output (written by a grid that lets its dependents start
    early, so q must be read only after the wait), eager and graph-replayed,
    give the same bits as the default launch."""
    cfg = DECODE_CONFIGS[name]
    kw = {"num_kv_heads": hkv} if hkv else {}
    sets = [make_decode_inputs(cfg, device="cuda", seed_tag=f"early{i}", **kw) for i in range(2)]

    def chain(ready):
        outs, q = [], sets[0].q
        for i in range(6):
            s = sets[i % 2]
            q = tsb.decode_attention(q, s.k_pool, s.v_pool, s.block_table, s.context_lens, inputs_ready=ready)
            outs.append(q)
        return outs

    ref = chain(False)
    got = chain(True)
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        chain(True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            graphed = chain(True)
        g.replay()
    stream.synchronize()
    for a, b in zip(ref, graphed):
        assert torch.equal(a, b)
    first = opa.decode_attention_cpu(sets[0].q, sets[0].k_pool, sets[0].v_pool, sets[0].block_table,
                                     sets[0].context_lens)
    torch.testing.assert_close(got[0].cpu().float(), first.float(), atol=2e-3, rtol=1e-2)


@pytest.mark.parametrize("name", ["gqa_b16", "tp70b"])
def test_early_start_gives_the_same_bits_fp8(name):
    """The early start over e4m3 pools (b200kv_decode_attention_ex_fp8):
    chained decodes whose q is the previous output, eager and graph-replayed,
    give the same bits as the default launch."""
    from torch_spyre_b200.workloads import quantize_decode_inputs

    cfg = DECODE_CONFIGS[name]
    kw = {"num_kv_heads": 1} if name == "tp70b" else {}
    sets = [quantize_decode_inputs(make_decode_inputs(cfg, device="cuda", seed_tag=f"early8-{i}", **kw))
            for i in range(2)]

    def chain(ready):
        outs, q = [], sets[0].q
        for i in range(6):
            s = sets[i % 2]
            q = tsb.decode_attention(q, s.k_pool, s.v_pool, s.block_table, s.context_lens, k_scale=s.k_scale,
                                     v_scale=s.v_scale, inputs_ready=ready)
            outs.append(q)
        return outs

    ref = chain(False)
    got = chain(True)
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        chain(True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            graphed = chain(True)
        g.replay()
    stream.synchronize()
    for a, b in zip(ref, graphed):
        assert torch.equal(a, b)
