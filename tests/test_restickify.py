"""Restickify: target layouts (the reference's restickify_device_size /
restickify_stride_map, torch_spyre/_inductor/pass_utils.py:749-781) on the
sizes of its restickify tests (tests/inductor/test_restickify.py:104-148,
test_inductor_ops_lx_planning.py:180-182), the oracle's data movement, and (on
a GPU) the one-pass device kernel bit-exact against the oracle."""

import numpy as np
import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import stick_layout as osl
from torch_spyre_b200.layout import restickify, restickify_layout

SIZES = [(256, 128), (128, 256), (128, 128), (64, 128), (128, 64), (10, 20), (7, 13), (64, 129)]

# target layouts of moving the stick of the default [s1, s2] fp16 layout to dim 0
EXPECTED = {
    (256, 128): ([4, 128, 64], [8192, 1, 128]),
    (128, 64): ([2, 64, 64], [4096, 1, 64]),
    (7, 13): ([1, 13, 64], [832, 1, 13]),
    (64, 129): ([1, 129, 64], [8256, 1, 129]),
}


@pytest.mark.parametrize("size", list(EXPECTED))
def test_target_layout_follows_reference_formula(size):
    stl = tsb.SpyreTensorLayout(list(size), torch.float16)
    r = restickify_layout(stl, size, 0)
    assert (r.device_size, r.stride_map) == EXPECTED[size]


def test_target_layout_3d_and_errors():
    stl = tsb.SpyreTensorLayout([4, 6, 200], torch.float16)
    r = restickify_layout(stl, [4, 6, 200], 1)
    assert (r.device_size, r.stride_map) == ([200, 1, 4, 64], [1, 12800, 1200, 200])
    with pytest.raises(ValueError):
        restickify_layout(stl, [4, 6, 200], 2)  # already the stick dim


@pytest.mark.parametrize("size", SIZES)
def test_oracle_restickify_round_trip(size):
    x = np.random.default_rng(sum(size)).standard_normal(size).astype(np.float16)
    a = tsb.SpyreTensorLayout(list(size), torch.float16)
    b = restickify_layout(a, size, 0)
    buf_a = osl.to_device(x, a.device_size, a.stride_map)
    buf_b = osl.restickify(buf_a, size, a.device_size, a.stride_map, b.device_size, b.stride_map)
    assert np.array_equal(buf_b.view(np.int16), osl.to_device(x, b.device_size, b.stride_map).view(np.int16))
    back = osl.restickify(buf_b, size, b.device_size, b.stride_map, a.device_size, a.stride_map)
    assert np.array_equal(back.view(np.int16), buf_a.view(np.int16))


def test_rejects_cpu():
    a = tsb.SpyreTensorLayout([8, 64], torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        restickify(torch.zeros(a.device_numel(), dtype=torch.float16), a, a, [8, 64])


@pytest.mark.gpu
@pytest.mark.parametrize("size", SIZES + [(4, 6, 200)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.float8_e4m3fn])
def test_gpu_restickify_matches_oracle(size, dtype):
    rng = np.random.default_rng(len(size) * 1000 + size[0])
    x = torch.from_numpy(rng.standard_normal(size).astype(np.float32)).to(dtype)
    a = tsb.SpyreTensorLayout(list(size), dtype)
    b = restickify_layout(a, size, len(size) - 2)
    buf_a = tsb.to_device_layout(x.cuda(), a)
    buf_b = restickify(buf_a, a, b, size)
    view = {torch.float16: np.int16, torch.float32: np.int32, torch.float8_e4m3fn: np.uint8}[dtype]
    bits = (lambda t: t.view(torch.uint8).numpy()) if dtype == torch.float8_e4m3fn else (lambda t: t.numpy().view(view))
    ref = osl.restickify(bits(buf_a.cpu()), size, a.device_size, a.stride_map, b.device_size, b.stride_map)
    assert np.array_equal(bits(buf_b.cpu()), ref)
    back = tsb.from_device_layout(restickify(buf_b, b, a, size), a, size)
    assert np.array_equal(bits(back.cpu()).reshape(-1), bits(x).reshape(-1))
