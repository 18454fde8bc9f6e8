"""General stick relayout on the GPU against the oracle's element map.

Every layout the reference's own layout tests pin (tests/tensor/
test_tensor_layout.py: default 39-66, dim_order 68-91, sparse 101-104,
explicit / padding / leading-ones 193-280) is relaid on the device; the device
buffer must equal oracle.stick_layout.to_device bit for bit and the round trip
must give the tensor back (the reference's ``x.to(device_layout=stl).cpu() == x``).
"""

import numpy as np
import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import stick_layout as osl
from test_layout import DEFAULT, DIM_ORDER, EXPLICIT

pytestmark = pytest.mark.gpu


def _check(x: torch.Tensor, dev, smap):
    stl = tsb.SpyreTensorLayout(dev, smap, torch.float16)
    buf = tsb.to_device_layout(x, stl)
    ref = osl.to_device(x.contiguous().cpu().numpy(), dev, smap)
    assert np.array_equal(buf.cpu().numpy().view(np.int16), ref.view(np.int16))
    back = tsb.from_device_layout(buf, stl, x.shape)
    assert torch.equal(back.view(torch.int16), x.contiguous().view(torch.int16))


@pytest.mark.parametrize("size,dev,smap", [c for c in DEFAULT if c[0]])
def test_default_layouts(size, dev, smap):
    _check(torch.randn(size, dtype=torch.float16, device="cuda"), dev, smap)


@pytest.mark.parametrize("size,stride,order,dev,smap", DIM_ORDER)
def test_dim_order_and_sparse_layouts(size, stride, order, dev, smap):
    _check(torch.randn(size, dtype=torch.float16, device="cuda"), dev, smap)


@pytest.mark.parametrize("size,dev,smap", EXPLICIT)
def test_explicit_layouts(size, dev, smap):
    _check(torch.randn(size, dtype=torch.float16, device="cuda"), dev, smap)


def test_strided_view_input():
    """A slice (non-contiguous storage offset) as in the reference's
    w[256:, :].to(device_layout=...) case."""
    w = torch.randn((512, 256), dtype=torch.float16, device="cuda")
    view = w[256:, :]
    dev, smap = osl.default_layout([256, 256])
    _check(view, dev, smap)
    t = torch.randn((256, 512), dtype=torch.float16, device="cuda").t()  # transposed strides
    dev, smap = osl.default_layout([512, 256])
    _check(t, dev, smap)


def test_expanding_layout():
    """[60] with stride_map [64, 0, 1]: the middle device dim repeats the row."""
    x = torch.randn(60, dtype=torch.float16, device="cuda")
    stl = tsb.SpyreTensorLayout([1, 512, 64], [64, 0, 1], torch.float16)
    buf = tsb.to_device_layout(x, stl).view(512, 64)
    assert torch.equal(buf[:, :60], x.expand(512, 60)) and int(buf[:, 60:].count_nonzero()) == 0
    assert torch.equal(tsb.from_device_layout(buf.reshape(-1), stl, [60]), x)


def test_kv_cache_layout_matches_pages():
    """A whole [T, Hkv, 128] cache in its default layout [Hkv, 2, T, 64] is the
    transpose of the paged pool's page content (same sticks, other order)."""
    T, hkv = 256, 3
    rows = torch.randn((T, hkv, 128), dtype=torch.float16, device="cuda")
    dev, smap = osl.default_layout([T, hkv, 128])
    buf = tsb.to_device_layout(rows, tsb.SpyreTensorLayout(dev, smap, torch.float16)).view(hkv, 2, T, 64)
    pool = torch.zeros((T // 64, hkv, 2, 64, 64), dtype=torch.float16, device="cuda")
    tsb.kv_relayout(rows, pool, torch.arange(T // 64, dtype=torch.int32, device="cuda"))
    assert torch.equal(buf, pool.permute(1, 2, 0, 3, 4).reshape(hkv, 2, T, 64))


def test_folded_layout_rejected():
    x = torch.randn((40, 60), dtype=torch.float16, device="cuda")
    with pytest.raises(tsb.B200KVError, match="folded"):
        tsb.to_device_layout(x, tsb.SpyreTensorLayout([38, 64], [64, 1], torch.float16))
