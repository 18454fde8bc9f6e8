"""FP8 (e4m3) oracle and host-side checks (no GPU work).

The oracle restates the reference's quantize / dequantize decompositions
(torch_spyre/_inductor/decompositions.py:846-858, 897-904); it is pinned here
against the CPU formula and tolerances of the reference's own tests
(tests/inductor/test_fp8_operations.py:124-272) on the same seeded inputs
(cached_randn == seeded_randn), and against known e4m3 answers.
"""

import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import fp8_quant as o8
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import seeded_randn

SMALL = [((1, 2, 32), s, 0.0, std) for s in (0.01, 0.1, 0.5, 1.0, 2.0) for std in (1.0, 5.0)]
MEDIUM = [((1, 2, 32), s, 10.0, 50.0) for s in (0.01, 0.1, 0.5, 1.0, 2.0)]
BOUNDARY = [((1, 2, 32), s, m, m) for s in (0.01, 0.1, 0.5, 1.0, 2.0) for m in (100.0, 200.0)]
PRODUCTION = [(1, 128, 512), (4, 128, 512), (1, 128, 1024), (1, 128, 2048), (1, 128, 4096)]


def _case_input(shape, mean, std):
    return seeded_randn(shape, dtype=torch.float16, scale=1.0) * std + mean


@pytest.mark.parametrize("shape,scale,mean,std,atol", [c + (2.0,) for c in SMALL] + [c + (16.0,) for c in MEDIUM]
                         + [c + (32.0 * c[1],) for c in BOUNDARY])
def test_oracle_within_reference_tolerance(shape, scale, mean, std, atol):
    x = _case_input(shape, mean, std)
    s = torch.tensor([scale], dtype=torch.float16)
    got = o8.dequantize_fp8_with_scale(o8.quantize_fp8_with_scale(x, s), s)
    torch.testing.assert_close(got, o8.reference_roundtrip(x, s), atol=atol, rtol=0.0)


@pytest.mark.parametrize("shape", PRODUCTION)
def test_oracle_production_shapes(shape):
    x = seeded_randn(shape, dtype=torch.float16, scale=1.0) * 2.0 + 1.0
    s = torch.tensor([1.0], dtype=torch.float16)
    got = o8.dequantize_fp8_with_scale(o8.quantize_fp8_with_scale(x, s), s)
    torch.testing.assert_close(got, o8.reference_roundtrip(x, s), atol=0.5, rtol=0.1)


def test_oracle_known_answers():
    one = torch.tensor([1.0], dtype=torch.float16)
    x = torch.tensor([1.0625, 1.1875, 448.0, 500.0, -1000.0, 2.0 ** -10, 3 * 2.0 ** -10, 30.0, -0.0],
                     dtype=torch.float16)
    q = o8.quantize_fp8_with_scale(x, one).float().tolist()
    # ties to even (1.0625 -> 1, 1.1875 -> 1.25), clamp to +-448, subnormal ties
    assert q == [1.0, 1.25, 448.0, 448.0, -448.0, 0.0, 2.0 ** -8, 30.0, -0.0]
    # scale 0.1 is 0.0999755859375 in fp16; its fp16 reciprocal is exactly 10
    s = torch.tensor([0.1], dtype=torch.float16)
    assert torch.reciprocal(s).item() == 10.0
    q = o8.quantize_fp8_with_scale(torch.tensor([3.0], dtype=torch.float16), s)
    assert q.float().item() == 30.0
    assert o8.dequantize_fp8_with_scale(q, s).item() == 3.0  # 2.99927 rounds to fp16 3.0


def test_oracle_pool_roundtrip():
    g = torch.Generator().manual_seed(0)
    pool16 = torch.randn((3, 2, 2, 64, 64), generator=g).to(torch.float16)
    s = torch.tensor([1 / 64], dtype=torch.float16)
    pool8 = o8.pool_from_fp16_pool(pool16, s)
    assert pool8.shape == (3, 2, 1, 64, 128) and pool8.dtype == torch.float8_e4m3fn
    # token row t, dim d of page (blk, h) at [blk, h, d // 128, t, d % 128]
    assert pool8[2, 1, 0, 5, 70].float() == o8.quantize_fp8_with_scale(pool16[2, 1, 1, 5, 6], s).float()
    back = o8.fp16_pool_from_pool(pool8, s)
    torch.testing.assert_close(back, o8.dequantize_fp8_with_scale(o8.quantize_fp8_with_scale(pool16, s), s))


def test_fp8_page_is_the_stick_layout_of_one_byte_elements():
    stl = tsb.SpyreTensorLayout([64, 128], torch.float8_e4m3fn)
    assert stl.device_size == [1, 64, 128] and stl.stride_map == [128, 128, 1]
    assert tsb.pool_shape_fp8(10, 8) == (10, 8, 1, 64, 128)
    with pytest.raises(ValueError):
        tsb.pool_shape_fp8(10, 8, 64)


def test_ops_reject_cpu_tensors():
    x = torch.zeros(4, 8, dtype=torch.float16)
    s = torch.ones(1, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CPU"):
        tsb.quantize_fp8_with_scale(x, s)
    with pytest.raises(RuntimeError, match="CPU"):
        tsb.dequantize_fp8_with_scale(x.to(torch.float8_e4m3fn), s)
    q = torch.zeros(1, 8, 128, dtype=torch.float16)
    pool = torch.zeros(2, 8, 1, 64, 128, dtype=torch.float8_e4m3fn)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CPU"):
        tsb.decode_attention(q, pool, pool, bt, torch.ones(1, dtype=torch.int32), k_scale=s, v_scale=s)


def test_fp8_pools_need_scales():
    q = torch.zeros(1, 8, 128, dtype=torch.float16)
    pool = torch.zeros(2, 8, 1, 64, 128, dtype=torch.float8_e4m3fn)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    with pytest.raises(ValueError, match="k_scale"):
        tsb.decode_attention(q, pool, pool, bt, torch.ones(1, dtype=torch.int32))


def test_fake_tensor_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(2, 16, 64, dtype=torch.float16, device="cuda")
        s = torch.empty(1, dtype=torch.float16, device="cuda")
        y = torch.ops.b200kv.quantize_fp8_with_scale(x, s)
        assert y.dtype == torch.float8_e4m3fn and y.shape == x.shape
        z = torch.ops.b200kv.dequantize_fp8_with_scale(y, s)
        assert z.dtype == torch.float16 and z.shape == x.shape
        q = torch.empty(3, 32, 128, dtype=torch.float16, device="cuda")
        pool = torch.empty(8, 8, 1, 64, 128, dtype=torch.float8_e4m3fn, device="cuda")
        bt = torch.empty(3, 4, dtype=torch.int32, device="cuda")
        lens = torch.empty(3, dtype=torch.int32, device="cuda")
        out, lse = torch.ops.b200kv.decode_attention_fp8(q, pool, pool, s, s, bt, lens, 0.1, 0, None)
        assert out.shape == (3, 32, 128) and lse.shape == (3, 32)


def test_c_abi_argument_checks():
    lib = _lib.lib()
    assert lib.b200kv_quantize_fp8_f16(None, None, 0, 16, None, 0, None) == 0
    assert lib.b200kv_quantize_fp8_f16(16, 16, -1, 16, 16, 0, None) == 1
    assert lib.b200kv_dequantize_fp8_f16(None, None, 4, 16, None, 0, None) == 1
    assert "null" in _lib.last_error()
    assert lib.b200kv_dequantize_fp8_f16(16, 16, 4, 16, 16, -1, None) == 1
    # append: head_dim, null scale
    assert lib.b200kv_kv_append_fp8(16, 16, 1024, 128, 16, 16, 16, 16, 16, 3, 8, 64, 4, None, None) == 2
    assert lib.b200kv_kv_append_fp8(16, 16, 1024, 128, 16, 16, None, 16, 16, 3, 8, 128, 4, None, None) == 1
    assert lib.b200kv_kv_append_fp8(None, None, 0, 0, None, None, None, None, None, 0, 8, 128, 4, None, None) == 0
    # decode: null scales are rejected before any launch
    args = [1 << 20, 4096, 128, 1 << 21, 1 << 22, None, None, 1 << 23, 4, 1 << 24, 1 << 25, 4096, 128, None,
            2, 32, 8, 128, 10, 4, 0.088, 0, 1 << 26, 1 << 40, None, None]
    assert lib.b200kv_decode_attention_fp8(*args) == 1
    assert "k_scale" in _lib.last_error()
    args[14] = 0  # empty batch
    assert lib.b200kv_decode_attention_fp8(*args) == 0
