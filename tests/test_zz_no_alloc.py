"""The decode entry point that allocates nothing.

Some callers cannot allocate device memory when they launch decode attention
(an engine replaying a pre-planned memory layout, a plugin host that only hands
over the tensors it owns), so they cannot pass the workspace the regular entry
point needs.  b200kv_decode_attention_f16_noalloc keeps its split-KV partials
in a fixed scratch array inside the library instead.  These tests call it
through the C ABI and check it against the regular entry point, twice in a row
(the scratch keeps the previous call's contents).  The file name sorts last so
that a run stopping at the first failure has run every other test first.
"""

import ctypes

import pytest
import torch

import torch_spyre_b200 as tsb
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2  # the decode parity tolerance used by every decode test


def _noalloc(inp, out, lse):
    B, hq, D = inp.q.shape
    nb, hkv = inp.k_pool.shape[0], inp.k_pool.shape[1]
    return _lib.lib().b200kv_decode_attention_f16_noalloc(
        inp.q.data_ptr(), inp.q.stride(0), inp.q.stride(1),
        inp.k_pool.data_ptr(), inp.v_pool.data_ptr(),
        inp.block_table.data_ptr(), inp.block_table.stride(0),
        inp.context_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        B, hq, hkv, D, nb, inp.block_table.shape[1],
        ctypes.c_float(D ** -0.5), None, torch.cuda.current_stream().cuda_stream,
    )


@pytest.mark.parametrize("name", ["gqa_b16", "tp70b"])
def test_noalloc_matches_workspace_entry_point(name):
    inp = make_decode_inputs(DECODE_CONFIGS[name], device="cuda", seed_tag="noalloc")
    ref, ref_lse = tsb.decode_attention(inp.q, inp.k_pool, inp.v_pool, inp.block_table,
                                        inp.context_lens, return_lse=True)
    for _ in range(2):  # the second call sees the first call's scratch contents
        out = torch.full_like(ref, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        status = _noalloc(inp, out, lse)
        assert status == 0, _lib.last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse, ref_lse, atol=1e-3, rtol=1e-4)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], device="cuda", ctx=[64] * 4, seed_tag="noalloc")
    out = torch.empty((4, 32, 128), dtype=torch.float16, device="cuda")
    lse = torch.empty((4, 32), dtype=torch.float32, device="cuda")
    status = _lib.lib().b200kv_decode_attention_f16_noalloc(
        inp.q.data_ptr(), inp.q.stride(0), inp.q.stride(1), inp.k_pool.data_ptr(), inp.v_pool.data_ptr(),
        inp.block_table.data_ptr(), inp.block_table.stride(0), inp.context_lens.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        1024, 128, 32, 128, inp.k_pool.shape[0], inp.block_table.shape[1],
        ctypes.c_float(0.088), None, torch.cuda.current_stream().cuda_stream)
    assert status == 2  # B200KV_ERR_UNSUPPORTED, checked before any launch
    assert "scratch" in _lib.last_error()
