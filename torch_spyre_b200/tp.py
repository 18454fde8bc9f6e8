"""Head-sharded tensor-parallel decode step (one process per GPU).

Rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N), the G query heads of each,
their KV pages (a per-rank pool with only those heads) and the matching input
columns of the output projection W_o.  A step is

    attn_r    = decode_attention(q[:, heads_r], k_pool_r, v_pool_r, ...)   # [B, Hq/N, D]
    partial_r = attn_r.reshape(B, -1) @ W_o[:, cols_r]^T                   # [B, hidden]
    y         = all_reduce_SUM(partial_r)                                  # NCCL

The all-reduce is the reference's tensor-parallel collective: a synchronous
SUM all-reduce of one tensor (SpyreCCLBackend::allreduce,
torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494).  It runs either over NCCL
on NVLink/NVSwitch or, with a :class:`PeerAllReduce`, as one libb200kv kernel
per rank over buffers the ranks map into each other with CUDA IPC (two-shot:
push slices to their owner, owner sums and pushes the result to every rank).
The block table and context lengths are replicated.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional

import torch

from . import _lib


@dataclass(frozen=True)
class HeadShard:
    """The heads and W_o columns one rank owns."""

    rank: int
    world: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int

    def __post_init__(self):
        if self.num_kv_heads % self.world:
            raise ValueError(f"{self.num_kv_heads} KV heads do not split over {self.world} ranks")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world {self.world}")

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    @property
    def kv_heads(self) -> range:
        n = self.num_kv_heads // self.world
        return range(self.rank * n, (self.rank + 1) * n)

    @property
    def q_heads(self) -> range:
        kv = self.kv_heads
        return range(kv.start * self.group, kv.stop * self.group)

    @property
    def w_cols(self) -> slice:
        q = self.q_heads
        return slice(q.start * self.head_dim, q.stop * self.head_dim)

    def shard_q(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of q [B, Hq, D] (a strided view, no copy)."""
        return q[:, self.q_heads.start:self.q_heads.stop]

    def shard_pool(self, pool: torch.Tensor) -> torch.Tensor:
        """This rank's KV heads of a full pool [NB, Hkv, S, 64, 64] (a copy)."""
        return pool[:, self.kv_heads.start:self.kv_heads.stop].contiguous()

    def shard_w_o(self, w_o: torch.Tensor) -> torch.Tensor:
        """This rank's input columns of W_o [hidden_out, Hq * D]."""
        return w_o[:, self.w_cols].contiguous()


class _DeviceBytes:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 2, "strides": None}


class PeerAllReduce:
    """SUM all-reduce of fp16 tensors of up to ``capacity`` elements over peer
    memory (libb200kv ``b200kv_peer_allreduce_f16``).

    Every rank allocates one peer buffer, exports its CUDA IPC handle and maps
    the others' (exchanged with ``all_gather_object`` over ``group``).  The
    tensor to reduce lives in the buffer's data region: ``buffer(shape)`` is a
    view a producer writes (the o_proj GEMM), ``all_reduce(view)`` sums it in
    place across ranks on the current stream.  Every rank must call
    ``all_reduce`` the same number of times with the same sizes, like a
    collective; calls replay correctly from CUDA graphs.  Waits are bounded:
    a missing peer sets B200KV_DEVERR_TIMEOUT in ``error_flag`` after 2 s.
    """

    def __init__(self, capacity: int, group=None, device: Optional[torch.device] = None, ctas: int = 128):
        import torch.distributed as dist

        self.group = group
        self._dist = dist.is_initialized()
        # without a process group: a single rank (the fused o_proj is then a plain GEMM)
        self.rank = dist.get_rank(group) if self._dist else 0
        self.world = dist.get_world_size(group) if self._dist else 1
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        q = 8 * self.world
        self.capacity = -(-int(capacity) // q) * q
        self.ctas = int(ctas)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            buf = ctypes.c_void_p()
            _lib.call("b200kv_peer_alloc", self.capacity, self.world, ctypes.byref(buf))
            self._own = buf.value
            hbytes = lib.b200kv_ipc_handle_bytes()
            handle = (ctypes.c_char * hbytes)()
            _lib.call("b200kv_ipc_get_handle", ctypes.c_void_p(self._own), handle)
            handles = [None] * self.world
            if self._dist:
                dist.all_gather_object(handles, bytes(handle), group=group)
            else:
                handles[0] = bytes(handle)
            self._opened = []
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                _lib.call("b200kv_ipc_open_handle", ctypes.create_string_buffer(h, len(h)), ctypes.byref(p))
                self._opened.append(p.value)
                ptrs.append(p.value)
        self._table = (ctypes.c_void_p * self.world)(*ptrs)
        self._data = torch.as_tensor(_DeviceBytes(self._own, self.capacity * 2), device=self.device).view(torch.float16)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)

    def buffer(self, shape) -> torch.Tensor:
        """A view of the data region (fp16, contiguous) of the given shape."""
        n = 1
        for d in shape:
            n *= int(d)
        if n > self.capacity:
            raise ValueError(f"{n} elements exceed the peer buffer capacity {self.capacity}")
        return self._data[:n].view(*shape)

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sums ``t`` (a view from ``buffer``) over the ranks, in place."""
        if t.dtype != torch.float16 or not t.is_contiguous() or t.data_ptr() != self._data.data_ptr():
            raise ValueError("all_reduce takes a contiguous fp16 view returned by buffer()")
        _lib.call("b200kv_peer_allreduce_f16", self._table, self.rank, self.world, t.numel(), self.capacity,
                  self.ctas, self.error_flag.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        return t

    def oproj_all_reduce(self, attn: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None
                         ) -> torch.Tensor:
        """Fused o_proj + all-reduce (b200kv_oproj_allreduce_f16): returns
        sum over ranks of attn [B, K] @ w [N, K]^T as fp16 [B, N] (B <= 128),
        the GEMM on the tensor cores and every 128 x 64 output tile exchanged
        as soon as it is computed.  A collective, like ``all_reduce``."""
        if attn.dtype != torch.float16 or w.dtype != torch.float16 or attn.dim() != 2 or w.dim() != 2:
            raise ValueError("attn [B, K] and w [N, K] must be fp16 matrices")
        if attn.stride(1) != 1 or w.stride(1) != 1 or attn.shape[1] != w.shape[1]:
            raise ValueError("attn and w need unit column strides and the same K")
        B, N = attn.shape[0], w.shape[0]
        if out is None:
            out = torch.empty((B, N), dtype=torch.float16, device=attn.device)
        _lib.call("b200kv_oproj_allreduce_f16", attn.data_ptr(), attn.stride(0), w.data_ptr(), w.stride(0),
                  out.data_ptr(), out.stride(0), B, N, attn.shape[1], self._table, self.rank, self.world,
                  self.capacity, self.error_flag.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a barrier:
        no peer may still write into it)."""
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self._dist:
            dist.barrier(group=self.group)
        self._data = None
        for p in self._opened:
            _lib.call("b200kv_ipc_close_handle", ctypes.c_void_p(p))
        _lib.call("b200kv_peer_free", ctypes.c_void_p(self._own))
        self._own = None
        self._opened = []


class NvlsAllReduce:
    """SUM all-reduce of fp16 tensors of up to ``capacity`` elements through
    NVLink SHARP (libb200kv ``b200kv_nvls_allreduce_f16``): the NVSwitch adds
    the ranks' values and multicasts the sum.

    The buffer is PyTorch symmetric memory (one allocation per rank, bound to
    an NVLink multicast object by ``rendezvous``): the data region first, then
    (low-latency kernel only) the reduce-scatter and all-gather receive
    regions, then the kernel's signal area.  PyTorch only provides that memory
    and its mapping; the collective is this library's kernel.  ``low_latency``
    picks ``b200kv_nvls_allreduce_ll_f16`` (two-shot with the arrival marker
    in the data: peer stores, then one multicast store, no barrier) over
    ``b200kv_nvls_allreduce_f16`` (in-switch reduction between two flag
    barriers).  Usage matches
    :class:`PeerAllReduce`: ``buffer(shape)`` is the view a producer writes,
    ``all_reduce(view)`` sums it in place across ranks on the current stream;
    every rank makes the same calls; graph replays are supported; waits are
    bounded (B200KV_DEVERR_TIMEOUT in ``error_flag``).  Raises RuntimeError if
    the GPUs offer no multicast (``available()`` tells beforehand).
    """

    def __init__(self, capacity: int, group=None, device: Optional[torch.device] = None,
                 ctas: Optional[int] = None, low_latency: bool = True):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        q = 8 * self.world
        self.capacity = -(-int(capacity) // q) * q
        self.low_latency = bool(low_latency)
        # measured on B200 (2 MiB): the low-latency kernel gains up to 64 CTAs
        # (N = 2: 11.3 -> 9.3 us, N = 4: 13.2 -> 11.4 us), the in-switch one does not
        self.ctas = int(ctas) if ctas is not None else (64 if self.low_latency else 32)
        lib = _lib.lib()
        self._data_bytes = -(-self.capacity * 2 // 256) * 256
        sig = int(lib.b200kv_nvls_signal_bytes())
        # [data | reduce-scatter x 2 | all-gather x 2 | signals] (low latency), [data | signals]
        self._rs_off = self._data_bytes
        self._ag_off = self._rs_off + 2 * self._data_bytes
        self._sig_off = self._ag_off + 2 * self._data_bytes if self.low_latency else self._data_bytes
        with torch.cuda.device(self.device):
            try:
                self._buf = symm_mem.empty(self._sig_off + sig, dtype=torch.uint8, device=self.device)
                self._hdl = symm_mem.rendezvous(self._buf, self.group.group_name)
                mc = int(self._hdl.multicast_ptr)
            except Exception:  # no symmetric memory here: no multicast either
                self._buf = self._hdl = None
                mc = 0
            # every rank sees the same answer; decide collectively so all raise or none
            flag = torch.tensor([1 if mc else 0], dtype=torch.int32, device=self.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
            if not int(flag.item()):
                self._hdl = None
                self._buf = None
                raise RuntimeError("NVLink multicast is not available on these GPUs")
            # the receive regions hold the "not arrived" sentinel between
            # calls; every rank fills its own before any rank may write them
            if self.low_latency:
                self._buf[self._rs_off : self._sig_off].fill_(0xFF)
            self._buf[self._sig_off :].zero_()
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._mc = mc
        ptrs = [int(p) for p in self._hdl.buffer_ptrs]
        self._signals = (ctypes.c_void_p * self.world)(*[p + self._sig_off for p in ptrs])
        self._rs = (ctypes.c_void_p * self.world)(*[p + self._rs_off for p in ptrs])
        self._data = self._buf[: self.capacity * 2].view(torch.float16)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)

    @staticmethod
    def available(group=None) -> bool:
        """Whether NVLink multicast buffers can be made for ``group`` (collective)."""
        import torch.distributed as dist

        try:
            NvlsAllReduce(8 * dist.get_world_size(group), group=group).close()
            return True
        except RuntimeError:
            return False

    def buffer(self, shape) -> torch.Tensor:
        """A view of the data region (fp16, contiguous) of the given shape."""
        n = 1
        for d in shape:
            n *= int(d)
        if n > self.capacity:
            raise ValueError(f"{n} elements exceed the multicast buffer capacity {self.capacity}")
        return self._data[:n].view(*shape)

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sums ``t`` (a view from ``buffer``) over the ranks, in place."""
        if t.dtype != torch.float16 or not t.is_contiguous() or t.data_ptr() != self._data.data_ptr():
            raise ValueError("all_reduce takes a contiguous fp16 view returned by buffer()")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self.low_latency:
            base = self._buf.data_ptr()
            _lib.call("b200kv_nvls_allreduce_ll_f16", t.data_ptr(), self._rs, base + self._ag_off,
                      self._mc + self._ag_off, self._data_bytes // 2, base + self._sig_off, self.rank, self.world,
                      t.numel(), self.ctas, self.error_flag.data_ptr(), stream)
        else:
            _lib.call("b200kv_nvls_allreduce_f16", self._mc, self._signals, self.rank, self.world, t.numel(),
                      self.ctas, self.error_flag.data_ptr(), stream)
        return t

    def close(self) -> None:
        """Releases the buffer after a barrier (no rank may still use it)."""
        import torch.distributed as dist

        if self._buf is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._data = None
        self._hdl = None
        self._buf = None


AttnFn = Callable[..., torch.Tensor]


def tp_decode_step(
    shard: HeadShard,
    q_local: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    w_o_local: torch.Tensor,
    group=None,
    out: Optional[torch.Tensor] = None,
    attn_fn: Optional[AttnFn] = None,
    k_scale: Optional[torch.Tensor] = None,
    v_scale: Optional[torch.Tensor] = None,
    allreduce=None,
    fused_oproj: bool = False,
    inputs_ready: bool = False,
) -> torch.Tensor:
    """One rank's step: local decode -> o_proj partial -> SUM all-reduce.

    attn_fn defaults to the CUDA decode op; tests on CPU ranks pass the oracle.
    k_scale / v_scale are the dequantisation scales of fp8 pools.  With
    ``allreduce`` the partial is written into its peer buffer and reduced by
    the peer-memory kernel (the result is a view of that buffer, valid until
    the next step) or, with ``fused_oproj``, the o_proj GEMM and the
    all-reduce run as one kernel (``PeerAllReduce.oproj_all_reduce``);
    otherwise NCCL (``group``) reduces it.
    ``inputs_ready``: the pools, block table and context lengths were written
    before the preceding kernel on the stream began (see
    ``decode_attention``), so the decode may start its page loads while that
    kernel -- e.g. the previous step's all-reduce -- finishes.
    Every rank must call this in the same order (it contains one collective).
    """
    if attn_fn is None:
        from .ops import decode_attention as attn_fn
    if k_scale is not None:
        attn = attn_fn(q_local, k_pool, v_pool, block_table, context_lens, k_scale=k_scale, v_scale=v_scale)
    elif inputs_ready:
        attn = attn_fn(q_local, k_pool, v_pool, block_table, context_lens, inputs_ready=True)
    else:
        attn = attn_fn(q_local, k_pool, v_pool, block_table, context_lens)
    B = attn.shape[0]
    flat = attn.reshape(B, -1)
    if allreduce is not None and fused_oproj:
        return allreduce.oproj_all_reduce(flat, w_o_local, out=out)
    if allreduce is not None:
        partial = allreduce.buffer((B, w_o_local.shape[0]))
        torch.matmul(flat, w_o_local.t(), out=partial)
        return allreduce.all_reduce(partial)
    if out is not None:
        partial = torch.matmul(flat, w_o_local.t(), out=out)
    else:
        partial = torch.matmul(flat, w_o_local.t())
    if shard.world > 1:
        import torch.distributed as dist

        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
