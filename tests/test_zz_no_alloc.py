"""The decode entry point that allocates nothing.

Some callers cannot allocate device memory when they launch decode attention
(an engine replaying a pre-planned memory layout, a plugin host that only hands
over the tensors it owns), so they cannot pass the workspace the regular entry
point needs.  b200kv_decode_attention_f16_noalloc keeps its split-KV partials
in a fixed scratch array inside the library instead.  These tests call it
through the C ABI, twice in a row (the scratch keeps the previous call's
contents), and check each result against the CPU oracle (the reference's CPU
eager decode) and against the regular entry point; they also check the size
limit the scratch sets, on both sides of it.  The file name sorts last so that
a run stopping at the first failure has run every other test first.
"""

import ctypes

import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import paged_attention as opa
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs, seeded_generator

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2  # the decode parity tolerance used by every decode test
B200KV_ERR_UNSUPPORTED = 2


def _noalloc(inp, out, lse, batch=None, hq=None, hkv=None):
    B, q_heads, D = inp.q.shape
    nb, kv_heads = inp.k_pool.shape[0], inp.k_pool.shape[1]
    return _lib.lib().b200kv_decode_attention_f16_noalloc(
        inp.q.data_ptr(), inp.q.stride(0), inp.q.stride(1),
        inp.k_pool.data_ptr(), inp.v_pool.data_ptr(),
        inp.block_table.data_ptr(), inp.block_table.stride(0),
        inp.context_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        batch or B, hq or q_heads, hkv or kv_heads, D, nb, inp.block_table.shape[1],
        ctypes.c_float(D ** -0.5), None, torch.cuda.current_stream().cuda_stream,
    )


def _check_two_calls(inp):
    ref_cpu, ref_cpu_lse = opa.decode_attention_cpu(inp.q, inp.k_pool, inp.v_pool, inp.block_table,
                                                    inp.context_lens, return_lse=True)
    ws, ws_lse = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens,
                                      return_lse=True)
    for _ in range(2):  # the second call sees the first call's scratch contents
        out = torch.full_like(ws, float("nan"))
        lse = torch.full_like(ws_lse, float("nan"))
        status = _noalloc(inp, out, lse)
        assert status == 0, _lib.last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.cpu().float(), ref_cpu.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse.cpu(), ref_cpu_lse, atol=1e-3, rtol=1e-4)
        torch.testing.assert_close(out.float(), ws.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse, ws_lse, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("name", ["gqa_b16", "tp70b"])
def test_noalloc_matches_oracle_and_workspace_entry_point(name):
    _check_two_calls(make_decode_inputs(DECODE_CONFIGS[name], device="cuda", seed_tag="noalloc"))


def test_noalloc_just_under_the_scratch_limit():
    # G = 8: 475 sequences x 8 KV heads = 3800 pairs, whose partials nearly
    # fill the 16 MiB scratch (the limit at G = 8 is about 3860 pairs)
    g = seeded_generator("noalloc", "near-limit")
    ctx = torch.randint(1, 300, (475,), generator=g).tolist()
    _check_two_calls(make_decode_inputs(DECODE_CONFIGS["tp70b"], device="cuda", ctx=ctx, seed_tag="noalloc"))


def _rejected(batch, hq, hkv):
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=[64] * 4, seed_tag="noalloc")
    out = torch.empty((4, 32, 128), dtype=torch.float16, device="cuda")
    lse = torch.empty((4, 32), dtype=torch.float32, device="cuda")
    # the sizes are rejected before anything is launched, so the small
    # buffers are never read
    status = _noalloc(inp, out, lse, batch=batch, hq=hq, hkv=hkv)
    return status, _lib.last_error()


def test_noalloc_rejects_too_many_pairs():
    status, msg = _rejected(1024, 128, 32)  # 32768 pairs > 16384
    assert status == B200KV_ERR_UNSUPPORTED
    assert "scratch" in msg


def test_noalloc_rejects_partials_beyond_the_scratch():
    status, msg = _rejected(500, 64, 8)  # 4000 pairs at G = 8: the partials do not fit
    assert status == B200KV_ERR_UNSUPPORTED
    assert "scratch" in msg
