"""ctypes binding of libb200kv.so, the C-ABI CUDA library (include/b200kv.h).

There is no fallback: if the shared library is missing the import of the ops
fails loudly, and every non-zero status of a C call is raised as
:class:`B200KVError` (a ``RuntimeError``, like the reference's TORCH_CHECK
failures, torch_spyre/csrc/spyre_mem.cpp:266-293).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libb200kv.so"

STATUS_NAMES = {
    0: "B200KV_OK",
    1: "B200KV_ERR_INVALID_ARG",
    2: "B200KV_ERR_UNSUPPORTED",
    3: "B200KV_ERR_WORKSPACE",
    4: "B200KV_ERR_CUDA",
}

DEVERR_BAD_BLOCK = 0x1
DEVERR_BAD_SLOT = 0x2
DEVERR_BAD_LEN = 0x4
DEVERR_TIMEOUT = 0x8


class B200KVError(RuntimeError):
    """A libb200kv entry point returned a non-zero status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        self.func = func
        super().__init__(f"{func}: {STATUS_NAMES.get(status, status)}: {message}")


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_p = ctypes.c_void_p
_f32 = ctypes.c_float

# (name, restype, argtypes) for every entry point of include/b200kv.h
SIGNATURES = {
    "b200kv_version": (ctypes.c_int, []),
    "b200kv_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "b200kv_stick_layout": (
        ctypes.c_int,
        [_p, _p, _i32, _p, _i32, _i32, _p, _p, _i32, _p],
    ),
    "b200kv_device_size_in_bytes": (_i64, [_p, _i32]),
    "b200kv_stick_relayout": (
        ctypes.c_int,
        [_p, _p, _i32, _i32, _p, _p, _i32, _p, _p, _i32, _p],
    ),
    "b200kv_stick_restickify": (ctypes.c_int, [_p, _p, _i32, _i32, _p, _i32, _p, _p, _i32, _p, _p, _p]),
    "b200kv_decode_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "b200kv_query_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "b200kv_lse_combine_f32": (ctypes.c_int, [_p, _i32, _p, _i64, _i64, _i64, _p, _p, _p]),
    "b200kv_decode_attention_f16": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p,  # k_pool, v_pool
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, _p,  # error_flag, stream
        ],
    ),
    "b200kv_decode_attention_ex_f16": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p,  # k_pool, v_pool
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, ctypes.c_uint32, _p,  # error_flag, flags, stream
        ],
    ),
    "b200kv_decode_attention_append_f16": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _i64, _i64,  # k_new, v_new, new_stride_b, new_stride_h
            _p, _p,  # k_pool, v_pool
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, _p,  # error_flag, stream
        ],
    ),
    "b200kv_decode_attention_append_ex_f16": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _i64, _i64,  # k_new, v_new, new_stride_b, new_stride_h
            _p, _p,  # k_pool, v_pool
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, ctypes.c_uint32, _p,  # error_flag, flags, stream
        ],
    ),
    "b200kv_decode_attention_f16_noalloc": (
        ctypes.c_int,
        [
            _p, _i64, _i64, _p, _p, _p, _i64, _p, _p, _i64, _i64, _p,
            _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _p,
        ],
    ),
    "b200kv_kv_append_f16": (
        ctypes.c_int,
        [_p, _p, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p],
    ),
    "b200kv_relayout_f16": (
        ctypes.c_int,
        [_p, _p, _p, _i64, _i64, _i64, _i64, _i32, _p, _p],
    ),
    "b200kv_rope_f16": (ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64, _p, _p]),
    "b200kv_decode_attention_append_rope_f16": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _i64, _i64,  # k_new, v_new, new_stride_b, new_stride_h
            _p, _p,  # k_pool, v_pool
            _p, _i64,  # rope_freqs, rope_max_pos
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, _p,  # error_flag, stream
        ],
    ),
    "b200kv_decode_attention_append_rope_fp8": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _i64, _i64,  # k_new, v_new, new_stride_b, new_stride_h
            _p, _p, _p, _p,  # k_pool, v_pool, k_scale, v_scale
            _p, _i64,  # rope_freqs, rope_max_pos
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, _p,  # error_flag, stream
        ],
    ),
    "b200kv_oproj_allreduce_f16": (
        ctypes.c_int,
        [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i32, _i32, _i64, _p, _p],
    ),
    "b200kv_peer_buffer_bytes": (_i64, [_i64, _i32]),
    "b200kv_peer_alloc": (ctypes.c_int, [_i64, _i32, _p]),
    "b200kv_peer_free": (ctypes.c_int, [_p]),
    "b200kv_ipc_handle_bytes": (_i32, []),
    "b200kv_ipc_get_handle": (ctypes.c_int, [_p, _p]),
    "b200kv_ipc_open_handle": (ctypes.c_int, [_p, _p]),
    "b200kv_ipc_close_handle": (ctypes.c_int, [_p]),
    "b200kv_peer_allreduce_f16": (ctypes.c_int, [_p, _i32, _i32, _i64, _i64, _i32, _p, _p]),
    "b200kv_nvls_signal_bytes": (_i64, []),
    "b200kv_nvls_allreduce_f16": (ctypes.c_int, [_p, _p, _i32, _i32, _i64, _i32, _p, _p]),
    "b200kv_nvls_allreduce_ll_f16": (ctypes.c_int, [_p, _p, _p, _p, _i64, _p, _i32, _i32, _i64, _i32, _p, _p]),
    "b200kv_quantize_fp8_f16": (ctypes.c_int, [_p, _p, _i64, _i64, _p, _i64, _p]),
    "b200kv_dequantize_fp8_f16": (ctypes.c_int, [_p, _p, _i64, _i64, _p, _i64, _p]),
    "b200kv_kv_append_fp8": (
        ctypes.c_int,
        [_p, _p, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p],
    ),
    "b200kv_decode_attention_fp8": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _p, _p,  # k_pool, v_pool, k_scale, v_scale
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, _p,  # error_flag, stream
        ],
    ),
    "b200kv_decode_attention_ex_fp8": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _p, _p,  # k_pool, v_pool, k_scale, v_scale
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, ctypes.c_uint32, _p,  # error_flag, flags, stream
        ],
    ),
    "b200kv_decode_attention_append_fp8": (
        ctypes.c_int,
        [
            _p, _i64, _i64,  # q, q_stride_b, q_stride_h
            _p, _p, _i64, _i64,  # k_new, v_new, new_stride_b, new_stride_h
            _p, _p, _p, _p,  # k_pool, v_pool, k_scale, v_scale
            _p, _i64,  # block_table, block_table_stride
            _p,  # context_lens
            _p, _i64, _i64,  # out, out_stride_b, out_stride_h
            _p,  # lse
            _i64, _i64, _i64, _i64,  # batch, Hq, Hkv, head_dim
            _i64, _i64,  # num_blocks, max_blocks_per_seq
            _f32, _i64,  # scale, num_splits
            _p, _i64,  # workspace, workspace_bytes
            _p, _p,  # error_flag, stream
        ],
    ),
}


def lib() -> ctypes.CDLL:
    """Loads libb200kv.so once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m torch_spyre_b200.build` "
                    "(there is no CPU fallback for the b200kv ops)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().b200kv_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, func: str) -> None:
    if status != 0:
        raise B200KVError(status, func, last_error())


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises on failure."""
    check(getattr(lib(), name)(*args), name)
