"""Stick layout algebra against the reference's golden layout vectors.

The vectors are restated from tests/tensor/test_tensor_layout.py (default
layouts 39-66, dim_order 68-91, sparse 101-104, explicit/padding/leading-one
round trips 193-280) and tests/test_spyre.py:384-392 (allocation size).  Both
the oracle restatement (oracle/stick_layout.py) and the product's C++ algebra
(b200kv_stick_layout in libb200kv.so, host code) must reproduce them.
"""

import numpy as np
import pytest
import torch

from oracle import stick_layout as osl

DEFAULT = [
    ([], [1, 64], [-1, -1]),
    ([120], [2, 64], [64, 1]),
    ([128], [2, 64], [64, 1]),
    ([512, 240], [4, 512, 64], [64, 240, 1]),
    ([512, 256], [4, 512, 64], [64, 256, 1]),
    ([512, 8, 240], [8, 4, 512, 64], [240, 64, 1920, 1]),
    ([512, 8, 256], [8, 4, 512, 64], [256, 64, 2048, 1]),
    # the page tile of the KV pools and a whole row-major cache
    ([64, 128], [2, 64, 64], [64, 128, 1]),
    ([131072, 8, 128], [8, 2, 131072, 64], [128, 64, 1024, 1]),
]

DIM_ORDER = [
    ([512, 256], [256, 1], [1, 0], [8, 256, 64], [16384, 1, 256]),
    ([512, 8, 256], [2048, 256, 1], [0, 2, 1], [256, 1, 512, 64], [1, 16384, 2048, 256]),
    ([512, 8, 256], [2048, 256, 1], [1, 0, 2], [512, 4, 8, 64], [2048, 64, 256, 1]),
    ([512, 8, 256], [2048, 256, 1], [1, 2, 0], [256, 8, 8, 64], [1, 131072, 256, 2048]),
    ([512, 8, 256], [2048, 256, 1], [2, 0, 1], [512, 1, 256, 64], [2048, 16384, 1, 256]),
    ([512, 8, 256], [2048, 256, 1], [2, 1, 0], [8, 8, 256, 64], [256, 131072, 1, 2048]),
    ([512, 256], [256, 1], [0, 1, -1], [256, 1, 512, 64], [1, -1, 256, -1]),  # sparse
]

# (host sizes, device_size, stride_map) explicit layouts whose round trip the
# reference checks (test_to_spyre_layout_explicit / _padding / _leading_ones)
EXPLICIT = [
    ([60], [1, 64], [64, 1]), ([64], [1, 64], [64, 1]), ([120], [2, 64], [64, 1]),
    ([128], [2, 64], [64, 1]), ([240], [4, 64], [64, 1]), ([256], [4, 64], [64, 1]),
    ([40, 60], [1, 60, 64], [3840, 1, 60]), ([40, 60], [1, 40, 64], [64, 60, 1]),
    ([40, 64], [1, 64, 64], [4096, 1, 64]), ([40, 64], [1, 40, 64], [64, 64, 1]),
    ([40, 120], [1, 120, 64], [7680, 1, 120]), ([40, 120], [2, 40, 64], [64, 120, 1]),
    ([40, 128], [1, 128, 64], [8192, 1, 128]), ([40, 128], [2, 40, 64], [64, 128, 1]),
    ([40, 240], [1, 240, 64], [15360, 1, 240]), ([40, 240], [4, 40, 64], [64, 240, 1]),
    ([40, 256], [1, 256, 64], [16384, 1, 256]), ([40, 256], [4, 40, 64], [64, 256, 1]),
    ([40, 60], [1, 512, 64], [64, 60, 1]), ([40, 128], [2, 512, 64], [64, 128, 1]),
    ([40, 256], [4, 512, 64], [64, 256, 1]), ([40, 120], [1, 512, 64], [7680, 1, 120]),
    ([60], [1, 1, 64], [64, 60, 1]), ([60], [1, 1, 1, 64], [60, 64, 60, 1]),
    ([60], [1, 1, 1, 1, 1, 64], [60, 60, 60, 64, 60, 1]),
]


@pytest.mark.parametrize("size,dev,smap", DEFAULT)
def test_default_layout_oracle(size, dev, smap):
    assert osl.default_layout(size) == (dev, smap)


@pytest.mark.parametrize("size,stride,order,dev,smap", DIM_ORDER)
def test_dim_order_oracle(size, stride, order, dev, smap):
    assert osl.layout(size, stride, 2, order) == (dev, smap)


@pytest.mark.parametrize("size,dev,smap", DEFAULT)
def test_default_layout_capi(size, dev, smap):
    from torch_spyre_b200.layout import stick_layout

    assert stick_layout(size, torch.float16) == (dev, smap)


@pytest.mark.parametrize("size,stride,order,dev,smap", DIM_ORDER)
def test_dim_order_capi(size, stride, order, dev, smap):
    from torch_spyre_b200.layout import SpyreTensorLayout

    stl = SpyreTensorLayout(size, stride, torch.float16, order)
    assert (stl.device_size, stl.stride_map) == (dev, smap)


def test_fp32_stick_holds_32():
    from torch_spyre_b200.layout import stick_layout

    assert stick_layout([100], torch.float32) == ([4, 32], [32, 1])
    assert osl.default_layout([100], elem_bytes=4) == ([4, 32], [32, 1])


def test_explicit_constructor_and_equality():
    from torch_spyre_b200.layout import SpyreTensorLayout

    x = SpyreTensorLayout([512, 256], torch.float16)
    y = SpyreTensorLayout([4, 512, 64], [64, 256, 1], torch.float16)
    z = SpyreTensorLayout([512, 256], [256, 1], torch.float16, [1, 0])
    assert x == y and hash(x) == hash(y)
    assert x != z
    assert len({x, y, z}) == 2


def test_allocation_size():
    """Two fp16 elements occupy one 128-byte stick (tests/test_spyre.py:384-392)."""
    from torch_spyre_b200.layout import SpyreTensorLayout

    stl = SpyreTensorLayout([2], torch.float16)
    assert stl.device_size_in_bytes() == 128
    assert osl.device_size_in_bytes(stl.device_size) == 128
    page = SpyreTensorLayout([64, 128], torch.float16)
    assert page.device_size_in_bytes() == 16384


def test_rank_limit_matches_reference():
    from torch_spyre_b200 import B200KVError
    from torch_spyre_b200.layout import stick_layout

    with pytest.raises(B200KVError, match="Unsupported tensor rank"):
        stick_layout([1] * 7)
    with pytest.raises(RuntimeError, match="Unsupported tensor rank"):
        osl.default_layout([1] * 7)


def test_dma_encoding_example():
    """docs/source/user_guide/tensors_and_layouts.md "DMA Encoding": for a
    (1024, 256) fp16 tensor device[i*65536 + j*64 + k] = host[j*256 + i*64 + k]."""
    x = np.arange(1024 * 256, dtype=np.int64).reshape(1024, 256)
    dev, smap = osl.default_layout([1024, 256])
    buf = osl.to_device(x, dev, smap)
    i, j, k = np.meshgrid(np.arange(4), np.arange(1024), np.arange(64), indexing="ij")
    assert np.array_equal(buf[i * 65536 + j * 64 + k], x.reshape(-1)[j * 256 + i * 64 + k])


@pytest.mark.parametrize("size,dev,smap", EXPLICIT)
def test_explicit_round_trip(size, dev, smap):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(size).astype(np.float16)
    buf = osl.to_device(x, dev, smap)
    assert buf.size == int(np.prod(dev))
    assert np.array_equal(osl.from_device(buf, size, dev, smap).view(np.int16), x.view(np.int16))


def test_page_tile_map_matches_pool_layout():
    """The generic element map of a [64, 128] page equals the pool's page order."""
    x = np.arange(64 * 128, dtype=np.int64).reshape(64, 128)
    dev, smap = osl.default_layout([64, 128])
    buf = osl.to_device(x, dev, smap).reshape(dev)      # [S=2, t=64, e=64]
    t, d = 37, 99
    assert buf[d // 64, t, d % 64] == x[t, d]
