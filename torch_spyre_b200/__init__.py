"""B200-native paged decode attention + KV relayout/append (torch-spyre hot path).

Importing the package registers the ``torch.ops.b200kv.*`` custom ops; their
CUDA library (``lib/libb200kv.so``, built by ``python -m torch_spyre_b200.build``)
is loaded on first use and is the only implementation.
"""

from . import _lib, fp8, layout, ops, workloads  # noqa: F401
from ._lib import B200KVError
from .fp8 import dequantize_fp8_with_scale, empty_pool_fp8, pool_shape_fp8, quantize_fp8_with_scale
from .layout import (SpyreTensorLayout, empty_pool, from_device_layout, page_layout, pool_shape, restickify,
                     restickify_layout, stick_layout, to_device_layout)
from .ops import (decode_attention, decode_attention_append, kv_append, kv_relayout, kv_unrelayout,
                  merge_attention_states, rope, scaled_dot_product_fused_attention_overrideable, sdpa_decode)

__all__ = [
    "B200KVError",
    "SpyreTensorLayout",
    "decode_attention",
    "decode_attention_append",
    "dequantize_fp8_with_scale",
    "empty_pool",
    "empty_pool_fp8",
    "from_device_layout",
    "to_device_layout",
    "kv_append",
    "kv_relayout",
    "kv_unrelayout",
    "merge_attention_states",
    "page_layout",
    "pool_shape",
    "pool_shape_fp8",
    "quantize_fp8_with_scale",
    "restickify",
    "restickify_layout",
    "rope",
    "scaled_dot_product_fused_attention_overrideable",
    "sdpa_decode",
    "stick_layout",
]
