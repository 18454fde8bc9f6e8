"""The SDPA route: F.scaled_dot_product_attention -> the reference's ATen op
aten::_scaled_dot_product_fused_attention_overrideable (CUDA kernel of this
package) -> b200kv::sdpa_decode, as the reference's _fused_sdp_choice forces
the overrideable backend for its device (torch_spyre/csrc/attn_utils.cpp:22-37,
torch_spyre/_inductor/decompositions.py:523-611).

CPU tests: which calls the mode takes, that every other call reaches torch
unchanged, and the fake (meta) kernel of the op.  GPU tests: the routed call
against the reference's golden decode outputs, a torch.compile(fullgraph=True)
trace of the op, and a launch count that does not grow with the batch.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import torch_spyre_b200 as tsb
from oracle import paged_attention as opa
from torch_spyre_b200.ops import SdpaDecodeMode, sdpa_decode_eligible
from torch_spyre_b200.workloads import seeded_randn

ATOL, RTOL = 2e-3, 1e-2


def _fake(shape, device="cuda", dtype=torch.float16):
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        return torch.empty(shape, dtype=dtype, device=device)


def test_eligibility():
    q, k = _fake((2, 32, 1, 128)), _fake((2, 8, 300, 128))
    assert sdpa_decode_eligible(q, k, k, enable_gqa=True)
    assert not sdpa_decode_eligible(q, k, k)                            # GQA without enable_gqa
    assert not sdpa_decode_eligible(_fake((2, 32, 2, 128)), k, k, enable_gqa=True)  # two query positions
    assert not sdpa_decode_eligible(q, k, k, attn_mask=_fake((2, 1, 1, 300)), enable_gqa=True)
    assert not sdpa_decode_eligible(q, k, k, dropout_p=0.1, enable_gqa=True)
    assert not sdpa_decode_eligible(q, k, k, is_causal=True, enable_gqa=True)
    assert not sdpa_decode_eligible(_fake((2, 24, 1, 128)), k, k, enable_gqa=True)  # group 3
    assert not sdpa_decode_eligible(_fake((2, 32, 1, 64)), _fake((2, 8, 300, 64)), _fake((2, 8, 300, 64)),
                                    enable_gqa=True)                    # head_dim 64
    assert not sdpa_decode_eligible(_fake((2, 32, 1, 128), dtype=torch.bfloat16), k, k, enable_gqa=True)
    cpu = torch.zeros(2, 8, 1, 128, dtype=torch.float16)
    assert not sdpa_decode_eligible(cpu, cpu, cpu)


def test_mode_passes_other_calls_to_torch():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 4, 3, 64, generator=g)
    k = torch.randn(2, 4, 10, 64, generator=g)
    ref = F.scaled_dot_product_attention(q, k, k, is_causal=True)
    with SdpaDecodeMode():
        out = F.scaled_dot_product_attention(q, k, k, is_causal=True)
        assert torch.equal(out, ref)
        assert torch.equal(torch.add(q, 1), q + 1)


def test_fake_kernel_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty((3, 32, 1, 128), dtype=torch.float16, device="cuda")
        k = torch.empty((3, 8, 77, 128), dtype=torch.float16, device="cuda")
        out, lse = torch.ops.b200kv.sdpa_decode(q, k, k, None, True)
    assert out.shape == (3, 32, 1, 128) and out.stride() == (32 * 128, 128, 32 * 128, 1)
    assert lse.shape == (3, 32) and lse.dtype == torch.float32


def _golden_inputs(hkv):
    q = seeded_randn((2, 1, 32, 128), 1).transpose(1, 2).cuda()
    k = seeded_randn((2, 257, hkv, 128), 2).transpose(1, 2).cuda()
    v = seeded_randn((2, 257, hkv, 128), 3).transpose(1, 2).cuda()
    return q, k, v


@pytest.mark.gpu
@pytest.mark.parametrize("case,hkv", [("mha_decode", 32), ("gqa_decode", 8)])
def test_routed_sdpa_matches_reference_golden(golden_dir, case, hkv):
    g = np.load(golden_dir / "sdpa_decode_golden.npz")
    q, k, v = _golden_inputs(hkv)
    with SdpaDecodeMode():
        out = F.scaled_dot_product_attention(q, k, v, enable_gqa=hkv != 32)
    torch.testing.assert_close(out.cpu().float(), torch.from_numpy(g[f"{case}_out_fp32"]), atol=ATOL, rtol=RTOL)
    # the ATen op itself, called on CUDA tensors, is this package's kernel
    res = torch.ops.aten._scaled_dot_product_fused_attention_overrideable(q, k, v)
    assert torch.equal(res[0], out) and res[4] == 1 and res[5] == 257
    torch.testing.assert_close(res[1].cpu()[:, :, 0], torch.from_numpy(g[f"{case}_lse"]), atol=1e-3, rtol=1e-4)


@pytest.mark.gpu
def test_compiled_fullgraph_matches_oracle():
    torch.manual_seed(0)
    B, S = 5, 1000
    q = torch.randn(B, 32, 1, 128, dtype=torch.float16, device="cuda")
    k = torch.randn(B, 8, S, 128, dtype=torch.float16, device="cuda")
    v = torch.randn(B, 8, S, 128, dtype=torch.float16, device="cuda")

    def step(q, k, v):
        return tsb.sdpa_decode(q, k, v, enable_gqa=True) * 2.0

    out = torch.compile(step, fullgraph=True)(q, k, v)
    eager = step(q, k, v)
    assert torch.equal(out, eager)
    ref = F.scaled_dot_product_attention(q.cpu().float(), k.cpu().float(), v.cpu().float(), enable_gqa=True)
    torch.testing.assert_close(out.cpu().float(), (ref * 2.0).half().float(), atol=2 * ATOL, rtol=RTOL)


@pytest.mark.gpu
def test_launch_count_does_not_grow_with_batch():
    from torch.profiler import ProfilerActivity, profile

    def kernels(B):
        q = torch.randn(B, 32, 1, 128, dtype=torch.float16, device="cuda")
        k = torch.randn(B, 8, 300, 128, dtype=torch.float16, device="cuda")
        tsb.sdpa_decode(q, k, k, enable_gqa=True)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            tsb.sdpa_decode(q, k, k, enable_gqa=True)
            torch.cuda.synchronize()
        return sum(1 for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA)

    # B = 1 may save the two K/V copies (its transpose is already token-major)
    n1, n2, n9 = kernels(1), kernels(2), kernels(9)
    assert n2 == n9 and n1 <= n2 <= 12, (n1, n2, n9)


@pytest.mark.gpu
def test_dense_decode_matches_oracle_ragged_length():
    # S not a multiple of 64: the last page of every sequence is partial
    torch.manual_seed(1)
    q = torch.randn(3, 16, 1, 128, dtype=torch.float16, device="cuda")
    k = torch.randn(3, 4, 131, 128, dtype=torch.float16, device="cuda")
    v = torch.randn(3, 4, 131, 128, dtype=torch.float16, device="cuda")
    out = tsb.sdpa_decode(q, k, v, enable_gqa=True)
    ref = opa.sdpa_decomposition_cpu(q.cpu(), k.cpu(), v.cpu())
    torch.testing.assert_close(out.cpu().float(), ref, atol=ATOL, rtol=RTOL)
