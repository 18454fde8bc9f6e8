"""Restatement of the reference's stick layout algebra (test infrastructure only).

* `default_layout` / `layout` follow SpyreTensorLayout::init
  (torch_spyre/csrc/spyre_tensor_impl.cpp:126-175): tiling rule
  get_generic_stick_layout (46-82), stick padding (160-172) and
  dim_map_to_stride_map (104-124).
* `to_device` / `from_device` apply the host<->device element map that the DMA
  descriptors encode (torch_spyre/csrc/spyre_mem.cpp:60-96 get_dim_map for the
  stride matching, 176-354 for the loop nest; worked example in
  docs/source/user_guide/tensors_and_layouts.md "DMA Encoding":
  device[i*65536 + j*64 + k] = host[j*256 + i*64 + k] for a (1024, 256) fp16
  tensor).  Device positions that map outside the host tensor (stick padding)
  are zero.

Written independently of the product's C++ implementation so the two check
each other against the reference's golden vectors.
"""

from __future__ import annotations

import numpy as np

STICK_BYTES = 128


def _tiling(order):
    # device dims: order[1:], then order[0], then the stick dim order[-1] again
    return list(order[1:]) + [order[0], order[-1]]


def layout(host_size, host_stride=None, elem_bytes=2, dim_order=None):
    """(device_size, stride_map) for a host tensor and a host dim order."""
    rank = len(host_size)
    eps = STICK_BYTES // elem_bytes
    if rank == 0:
        return [1, eps], [-1, -1]
    if rank > 6:
        raise RuntimeError(f"Unsupported tensor rank: {rank}")
    if host_stride is None:
        host_stride, s = [0] * rank, 1
        for i in range(rank - 1, -1, -1):
            host_stride[i] = s
            s *= host_size[i]
    order = list(range(rank)) if dim_order is None else list(dim_order)
    sparse = len(order) == rank + 1 and order[-1] == -1
    if len(order) != rank and not sparse:
        raise RuntimeError("Incompatible host_size and dim_order")
    dmap = _tiling(order)
    stick = dmap[-1]
    dev = []
    for d in dmap[:-1]:
        if d == stick:
            dev.append(1 if sparse else -(-host_size[d] // eps))
        else:
            dev.append(host_size[d])
    dev.append(eps)
    smap = [-1] * len(dmap)
    outer = {}
    for j in range(len(dmap) - 1, -1, -1):
        d = dmap[j]
        if d == -1 or host_size[d] == 1:
            continue
        smap[j] = outer.get(d, host_stride[d])
        outer[d] = smap[j] * dev[j]
    return dev, smap


def default_layout(host_size, elem_bytes=2):
    return layout(host_size, None, elem_bytes, None)


def _dim_map(host_size, host_stride, device_size, stride_map):
    """Host dim walked by each device dim: the host dim with the largest stride
    that is <= the device dim's stride (size-1 and expanded dims skipped)."""
    best = [0] * len(stride_map)
    dmap = [-1] * len(stride_map)
    for i, (sz, st) in enumerate(zip(host_size, host_stride)):
        if sz == 1 or st == 0:
            continue
        for j, (dsz, dst) in enumerate(zip(device_size, stride_map)):
            if dsz == 1:
                continue
            if best[j] < st <= dst:
                best[j] = st
                dmap[j] = i
    return dmap


def _element_map(host_size, device_size, stride_map):
    """(flat host index or -1) for every device element, host contiguous."""
    rank = len(host_size)
    hstride, s = [0] * rank, 1
    for i in range(rank - 1, -1, -1):
        hstride[i] = s
        s *= host_size[i]
    dmap = _dim_map(host_size, hstride, device_size, stride_map)
    idx = np.indices(device_size, dtype=np.int64).reshape(len(device_size), -1)
    coords = np.zeros((rank, idx.shape[1]), dtype=np.int64)
    for j, d in enumerate(dmap):
        if d < 0 or stride_map[j] <= 0:
            continue
        coords[d] += idx[j] * (stride_map[j] // hstride[d])
    valid = np.ones(idx.shape[1], dtype=bool)
    flat = np.zeros(idx.shape[1], dtype=np.int64)
    for d in range(rank):
        valid &= coords[d] < host_size[d]
        flat += coords[d] * hstride[d]
    return np.where(valid, flat, -1)


def to_device(x: np.ndarray, device_size, stride_map) -> np.ndarray:
    """Device buffer (flat, prod(device_size) elements) holding host tensor x."""
    m = _element_map(list(x.shape), list(device_size), list(stride_map))
    flat = np.ascontiguousarray(x).reshape(-1)
    out = np.zeros(m.shape[0], dtype=x.dtype)
    ok = m >= 0
    out[ok] = flat[m[ok]]
    return out


def from_device(buf: np.ndarray, host_size, device_size, stride_map, dtype=None) -> np.ndarray:
    """Inverse of `to_device`: the host tensor read back from a device buffer."""
    m = _element_map(list(host_size), list(device_size), list(stride_map))
    out = np.zeros(int(np.prod(host_size)), dtype=dtype or buf.dtype)
    ok = m >= 0
    out[m[ok]] = buf[ok]
    return out.reshape(host_size)


def device_size_in_bytes(device_size):
    """128 bytes per stick times the number of sticks (spyre_tensor_impl.cpp:287-293)."""
    return int(np.prod(device_size[:-1])) * STICK_BYTES


def restickify(buf: np.ndarray, host_size, src_device_size, src_stride_map, dst_device_size,
               dst_stride_map) -> np.ndarray:
    """Device buffer of layout dst holding what `buf` holds in layout src: read
    back through src's element map, written through dst's (the data movement
    of spyre::restickify, torch_spyre/_inductor/customops.py:338-342)."""
    host = from_device(buf, host_size, src_device_size, src_stride_map, dtype=buf.dtype)
    return to_device(host, dst_device_size, dst_stride_map)
