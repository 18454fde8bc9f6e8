"""Stick layout algebra and the paged KV pool layout.

`SpyreTensorLayout` mirrors the reference class of the same name
(torch_spyre/csrc/spyre_tensor_impl.h:48-146, bound to Python in
torch_spyre/csrc/module.cpp): a device layout is a ``device_size`` list whose
last entry is the stick (128 bytes of elements) and a ``stride_map`` giving, for
every device dim, the host element stride it walks (-1 for dims of size one).
The arithmetic runs in libb200kv (``b200kv_stick_layout``, host code, no GPU
needed), so the kernels and Python share one implementation.

The KV pools use the default tiling of a [64, D] fp16 page:
device_size [D/64, 64, 64], stride_map [64, D, 1].
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib

PAGE_TOKENS = 64
STICK_BYTES = 128

_ELEM_BYTES = {
    torch.float16: 2,
    torch.bfloat16: 2,
    torch.float32: 4,
    torch.int32: 4,
    torch.int64: 8,
    torch.int8: 1,
    torch.uint8: 1,
    torch.float8_e4m3fn: 1,
}


def elems_per_stick(dtype: torch.dtype) -> int:
    return STICK_BYTES // _ELEM_BYTES[dtype]


def stick_layout(
    host_size: Sequence[int],
    dtype: torch.dtype = torch.float16,
    host_stride: Optional[Sequence[int]] = None,
    dim_order: Optional[Sequence[int]] = None,
) -> tuple[list[int], list[int]]:
    """(device_size, stride_map) of the default stick tiling of a host tensor."""
    rank = len(host_size)
    cap = rank + 2
    hs = (ctypes.c_int64 * max(rank, 1))(*host_size)
    st = (ctypes.c_int64 * max(rank, 1))(*host_stride) if host_stride is not None else None
    order = (ctypes.c_int32 * len(dim_order))(*dim_order) if dim_order is not None else None
    dev = (ctypes.c_int64 * cap)()
    smap = (ctypes.c_int64 * cap)()
    out_rank = ctypes.c_int32(0)
    _lib.call(
        "b200kv_stick_layout",
        ctypes.cast(hs, ctypes.c_void_p),
        ctypes.cast(st, ctypes.c_void_p) if st is not None else None,
        rank,
        ctypes.cast(order, ctypes.c_void_p) if order is not None else None,
        len(dim_order) if dim_order is not None else 0,
        _ELEM_BYTES[dtype],
        ctypes.cast(dev, ctypes.c_void_p),
        ctypes.cast(smap, ctypes.c_void_p),
        cap,
        ctypes.cast(ctypes.pointer(out_rank), ctypes.c_void_p),
    )
    n = out_rank.value
    return list(dev[:n]), list(smap[:n])


class SpyreTensorLayout:
    """Device layout of a tensor in 128-byte sticks.

    Constructors follow the reference (tests/tensor/test_tensor_layout.py):
    ``SpyreTensorLayout(host_size, dtype)``,
    ``SpyreTensorLayout(host_size, host_stride, dtype, dim_order)`` and the
    explicit ``SpyreTensorLayout(device_size, stride_map, dtype)``.
    """

    def __init__(self, *args):
        if len(args) == 2:
            size, dtype = args
            self.device_size, self.stride_map = stick_layout(list(size), dtype)
        elif len(args) == 4:
            size, stride, dtype, order = args
            self.device_size, self.stride_map = stick_layout(list(size), dtype, list(stride), list(order))
        elif len(args) == 3:
            self.device_size, self.stride_map, dtype = list(args[0]), list(args[1]), args[2]
            if len(self.device_size) != len(self.stride_map):
                raise ValueError("device_size and stride_map must have the same length")
        else:
            raise TypeError("SpyreTensorLayout(size, dtype) | (size, stride, dtype, dim_order) | "
                            "(device_size, stride_map, dtype)")
        self.device_dtype = dtype

    def device_numel(self) -> int:
        n = 1
        for x in self.device_size:
            n *= x
        return n

    def device_size_in_bytes(self) -> int:
        arr = (ctypes.c_int64 * len(self.device_size))(*self.device_size)
        return int(_lib.lib().b200kv_device_size_in_bytes(ctypes.cast(arr, ctypes.c_void_p), len(arr)))

    def _key(self):
        return (tuple(self.device_size), tuple(self.stride_map), self.device_dtype)

    def __eq__(self, other):
        return isinstance(other, SpyreTensorLayout) and self._key() == other._key()

    def __hash__(self):
        return hash(self._key())

    def __repr__(self):
        return (f"SpyreTensorLayout(device_size={self.device_size}, stride_map={self.stride_map}, "
                f"device_dtype={self.device_dtype})")


def page_layout(head_dim: int = 128) -> SpyreTensorLayout:
    """Layout of one page: the default tiling of a [64, head_dim] fp16 tile."""
    return SpyreTensorLayout([PAGE_TOKENS, head_dim], torch.float16)


def pool_shape(num_blocks: int, num_kv_heads: int, head_dim: int = 128) -> tuple[int, ...]:
    """Shape of a K or V pool: [num_blocks, Hkv, head_dim / 64, 64, 64]."""
    if head_dim % 64:
        raise ValueError("head_dim must be a multiple of 64")
    return (num_blocks, num_kv_heads, head_dim // 64, PAGE_TOKENS, 64)


def empty_pool(num_blocks: int, num_kv_heads: int, head_dim: int = 128, device=None) -> torch.Tensor:
    return torch.empty(pool_shape(num_blocks, num_kv_heads, head_dim), dtype=torch.float16, device=device)


def slot_of(block_table: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Slots (block * 64 + offset) of token `positions[b]` of each sequence b."""
    blk = block_table.gather(1, (positions // PAGE_TOKENS).long().unsqueeze(1)).squeeze(1).long()
    return blk * PAGE_TOKENS + (positions % PAGE_TOKENS).long()


def _arr64(v):
    a = (ctypes.c_int64 * len(v))(*v)
    return a, ctypes.cast(a, ctypes.c_void_p)


def _stick_relayout(src: torch.Tensor, dst: torch.Tensor, host: torch.Tensor, stl: "SpyreTensorLayout",
                    direction: int) -> None:
    if src.device.type != "cuda" or dst.device.type != "cuda":
        raise RuntimeError("stick relayout runs on CUDA devices only (there is no CPU fallback)")
    hs, hs_p = _arr64(list(host.shape) or [1])
    st, st_p = _arr64(list(host.stride()) or [1])
    ds, ds_p = _arr64(stl.device_size)
    sm, sm_p = _arr64(stl.stride_map)
    _lib.call("b200kv_stick_relayout", src.data_ptr(), dst.data_ptr(), host.element_size(),
              max(host.dim(), 1), hs_p, st_p, len(stl.device_size), ds_p, sm_p, direction,
              torch.cuda.current_stream(src.device).cuda_stream)


def to_device_layout(x: torch.Tensor, stl: SpyreTensorLayout) -> torch.Tensor:
    """Device buffer (flat, prod(device_size) elements) holding x in layout stl.

    The CUDA form of the reference's ``x.to(device_layout=stl)``
    (torch_spyre/_monkey_patch.py:73-156 -> generate_dci); x may be a strided
    view.  Stick padding is zero.
    """
    buf = torch.empty(stl.device_numel(), dtype=x.dtype, device=x.device)
    _stick_relayout(x, buf, x, stl, 0)
    return buf


def from_device_layout(buf: torch.Tensor, stl: SpyreTensorLayout, host_size, out: Optional[torch.Tensor] = None
                       ) -> torch.Tensor:
    """The host-order tensor read back from a device-layout buffer (``.cpu()``
    of the reference, on the device)."""
    if out is None:
        out = torch.empty(tuple(host_size), dtype=buf.dtype, device=buf.device)
    _stick_relayout(buf, out, out, stl, 1)
    return out


def _walked_host_dim(stride: int, host_size, cstride) -> Optional[int]:
    """The host dim a device dim of stride-map entry `stride` walks (the size > 1
    dim with the largest contiguous stride <= stride; None if there is none)."""
    best = None
    for d, (n, cs) in enumerate(zip(host_size, cstride)):
        if n != 1 and cs <= stride and (best is None or cs > cstride[best]):
            best = d
    return best


def restickify_layout(stl: SpyreTensorLayout, host_size, new_stick_dim: int) -> SpyreTensorLayout:
    """The layout that results from moving stl's stick to host dim
    ``new_stick_dim`` of a contiguous host tensor of ``host_size``.

    Follows the reference's restickify_device_size / restickify_stride_map
    (torch_spyre/_inductor/pass_utils.py:749-781): the stick dim becomes a full
    stick of the new dim, the old stick's outer device dim counts sticks of the
    new dim, and the device dim that walked the new dim now walks the old stick
    dim.
    """
    host_size = list(host_size)
    cstride, acc = [0] * len(host_size), 1
    for d in range(len(host_size) - 1, -1, -1):
        cstride[d] = acc
        acc *= host_size[d]
    dev, smap = list(stl.device_size), list(stl.stride_map)
    old_sd = _walked_host_dim(smap[-1], host_size, cstride)
    if old_sd is None or old_sd == new_stick_dim:
        raise ValueError("the stick already walks that dim, or the layout has no stick dim")
    walks = [_walked_host_dim(smap[j], host_size, cstride) if smap[j] > 0 and dev[j] > 1 else None
             for j in range(len(dev) - 1)]
    # the device dim counting sticks of the old stick dim; when it has size one
    # (a single stick) nothing walks it and a size-one device dim stands in
    old_outer = next((j for j, d in enumerate(walks) if d == old_sd),
                     next((j for j in range(len(dev) - 1) if dev[j] == 1), None))
    new_outer = next((j for j, d in enumerate(walks) if d == new_stick_dim), None)
    if old_outer is None or new_outer is None:
        raise ValueError("no device dim walks the old stick dim or the new stick dim")
    stick = dev[-1]
    new_dev = list(dev)
    new_dev[-1] = stick
    new_dev[old_outer] = -(-host_size[new_stick_dim] // stick)
    new_dev[new_outer] = host_size[old_sd]
    new_smap = list(smap)
    new_smap[-1] = cstride[new_stick_dim]
    new_smap[old_outer] = cstride[new_stick_dim] * stick
    new_smap[new_outer] = cstride[old_sd]
    return SpyreTensorLayout(new_dev, new_smap, stl.device_dtype)


def restickify(buf: torch.Tensor, src: SpyreTensorLayout, dst: SpyreTensorLayout, host_size) -> torch.Tensor:
    """The device buffer of layout ``dst`` holding the tensor that ``buf`` holds
    in layout ``src`` (the reference's ``spyre::restickify``,
    torch_spyre/_inductor/customops.py:338-342), moved on the device in one
    pass; destination padding is zero."""
    if buf.device.type != "cuda":
        raise RuntimeError("restickify runs on CUDA devices only (there is no CPU fallback)")
    out = torch.empty(dst.device_numel(), dtype=buf.dtype, device=buf.device)
    hs, hs_p = _arr64(list(host_size))
    sd, sd_p = _arr64(src.device_size)
    ss, ss_p = _arr64(src.stride_map)
    dd, dd_p = _arr64(dst.device_size)
    ds, ds_p = _arr64(dst.stride_map)
    _lib.call("b200kv_stick_restickify", buf.data_ptr(), out.data_ptr(), buf.element_size(), len(host_size), hs_p,
              len(src.device_size), sd_p, ss_p, len(dst.device_size), dd_p, ds_p,
              torch.cuda.current_stream(buf.device).cuda_stream)
    return out
