"""Op registration: fake kernels trace, and CPU tensors are rejected loudly
(there is no CPU fallback in the product path)."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import torch_spyre_b200 as tsb  # noqa: F401  (registers torch.ops.b200kv)


def test_ops_registered():
    for name in ("decode_attention", "kv_append", "kv_relayout", "kv_unrelayout"):
        assert hasattr(torch.ops.b200kv, name)


def test_fake_decode_shapes():
    with FakeTensorMode():
        q = torch.empty(4, 32, 128, dtype=torch.float16)
        pool = torch.empty(10, 8, 2, 64, 64, dtype=torch.float16)
        bt = torch.empty(4, 3, dtype=torch.int32)
        ctx = torch.empty(4, dtype=torch.int32)
        out, lse = torch.ops.b200kv.decode_attention(q, pool, pool, bt, ctx, 0.1, 0, None)
        assert out.shape == (4, 32, 128) and lse.shape == (4, 32) and lse.dtype == torch.float32
        rows = torch.ops.b200kv.kv_unrelayout(pool, torch.empty(2, dtype=torch.int32), 100, None)
        assert rows.shape == (100, 8, 128)


def test_cpu_tensors_rejected():
    q = torch.zeros(1, 8, 128, dtype=torch.float16)
    pool = torch.zeros(2, 8, 2, 64, 64, dtype=torch.float16)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    ctx = torch.ones(1, dtype=torch.int32)
    with pytest.raises(Exception, match="CUDA"):
        tsb.decode_attention(q, pool, pool, bt, ctx)
    with pytest.raises(Exception, match="CUDA"):
        tsb.kv_append(q, q, pool, pool, torch.zeros(1, dtype=torch.int64))


def test_stick_relayout_rejects_cpu_tensors():
    x = torch.zeros(4, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        tsb.to_device_layout(x, tsb.SpyreTensorLayout([4, 64], torch.float16))
