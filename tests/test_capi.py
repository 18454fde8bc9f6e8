"""libb200kv.so loads, exports every symbol of include/b200kv.h, and validates
arguments on the host (no GPU work is launched by these tests)."""

import ctypes
import re
from pathlib import Path

import pytest

from torch_spyre_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "b200kv.h"


def header_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"B200KV_API\s+[\w\s\*]+?\b(b200kv_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = header_symbols()
    for name in ("b200kv_decode_attention_f16", "b200kv_kv_append_f16", "b200kv_relayout_f16",
                 "b200kv_decode_workspace_bytes", "b200kv_last_error", "b200kv_stick_layout"):
        assert name in syms


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    for name in header_symbols():
        assert hasattr(lib, name), name
    assert set(header_symbols()) <= set(_lib.SIGNATURES), "ctypes signatures missing"


def test_version_and_last_error():
    lib = _lib.lib()
    assert lib.b200kv_version() >= 100
    n = lib.b200kv_last_error(None, 0)
    assert n >= 0


def test_workspace_bytes():
    lib = _lib.lib()
    w = lib.b200kv_decode_workspace_bytes(16, 32, 8, 128)
    assert w > 0 and w % 256 == 0
    assert lib.b200kv_decode_workspace_bytes(16, 32, 8, 64) == -1   # head_dim
    assert lib.b200kv_decode_workspace_bytes(16, 30, 8, 128) == -1  # Hq % Hkv


def _decode(**over):
    args = dict(q=1 << 20, qsb=4096, qsh=128, k=1 << 21, v=1 << 22, bt=1 << 23, bts=4, ctx=1 << 24,
                out=1 << 25, osb=4096, osh=128, lse=None, B=2, Hq=32, Hkv=8, D=128, NB=10, MB=4,
                scale=0.088, splits=0, ws=None, wsb=0, flag=None, stream=None)
    args.update(over)
    return _lib.lib().b200kv_decode_attention_f16(*args.values())


@pytest.mark.parametrize("over,status,msg", [
    (dict(D=64), 2, "head_dim"),
    (dict(Hq=24, Hkv=8), 2, "group size"),
    (dict(Hq=30), 1, "multiple"),
    (dict(q=None), 1, "null"),
    (dict(q=(1 << 20) + 2), 1, "aligned"),
    (dict(bts=2), 1, "block_table_stride"),
    (dict(splits=1025), 1, "num_splits"),
    (dict(B=2000), 2, "batch"),
    (dict(scale=float("nan")), 1, "scale"),
    (dict(), 3, "workspace"),
])
def test_decode_argument_checks(over, status, msg):
    assert _decode(**over) == status
    assert msg in _lib.last_error()


def test_empty_batch_is_ok_without_gpu():
    assert _decode(B=0) == 0


def test_append_and_relayout_checks():
    lib = _lib.lib()
    assert lib.b200kv_kv_append_f16(None, None, 0, 0, None, None, None, 0, 8, 128, 4, None, None) == 0
    assert lib.b200kv_kv_append_f16(None, None, 1024, 128, None, None, None, 3, 8, 128, 4, None, None) == 1
    assert lib.b200kv_kv_append_f16(16, 16, 1024, 128, 16, 16, 16, 3, 8, 96, 4, None, None) == 2
    assert lib.b200kv_relayout_f16(16, 16, 16, 64, 8, 128, 4, 2, None, None) == 1
    assert "direction" in _lib.last_error()
    assert lib.b200kv_relayout_f16(16, 16, 16, 0, 8, 128, 4, 0, None, None) == 0


def test_error_raises_runtime_error():
    with pytest.raises(RuntimeError, match="B200KV_ERR_INVALID_ARG"):
        _lib.call("b200kv_relayout_f16", 16, 16, 16, 64, 8, 128, 4, 5, None, None)


def test_peer_allreduce_host_checks():
    import ctypes

    lib = _lib.lib()
    assert lib.b200kv_ipc_handle_bytes() == 64
    assert lib.b200kv_peer_buffer_bytes(128 * 8192, 2) > 128 * 8192 * 2 * 2
    assert lib.b200kv_peer_buffer_bytes(0, 2) == -1 and lib.b200kv_peer_buffer_bytes(16, 9) == -1
    table = (ctypes.c_void_p * 2)(1 << 20, 1 << 21)
    assert lib.b200kv_peer_allreduce_f16(table, 0, 2, 12, 32, 0, None, None) == 1
    assert "multiple of 8 * world" in _lib.last_error()
    assert lib.b200kv_peer_allreduce_f16(table, 2, 2, 16, 32, 0, None, None) == 1
    assert lib.b200kv_peer_allreduce_f16(table, 0, 2, 16, 32, 129, None, None) == 1
    assert lib.b200kv_peer_allreduce_f16(table, 0, 2, 48, 32, 0, None, None) == 1  # beyond capacity
    assert lib.b200kv_peer_allreduce_f16(table, 0, 2, 0, 32, 0, None, None) == 0  # nothing to do
    bad = (ctypes.c_void_p * 2)(1 << 20, (1 << 21) + 16)
    assert lib.b200kv_peer_allreduce_f16(bad, 0, 2, 16, 32, 0, None, None) == 1
    assert "aligned" in _lib.last_error()


def test_ex_entries_reject_unknown_flags():
    lib = _lib.lib()
    base = [1 << 20, 4096, 128, 1 << 21, 1 << 22, 1 << 23, 4, 1 << 24, 1 << 25, 4096, 128, None, 2, 32, 8, 128,
            10, 4, 0.088, 0, None, 0, None]
    assert lib.b200kv_decode_attention_ex_f16(*base, 2, None) == 1
    assert "unknown flags" in _lib.last_error()
    fp8 = base[:5] + [1 << 26, 1 << 27] + base[5:]  # k_scale, v_scale after the pools
    assert lib.b200kv_decode_attention_ex_fp8(*fp8, 6, None) == 1
    assert "unknown flags" in _lib.last_error()


def test_nvls_allreduce_host_checks():
    lib = _lib.lib()
    assert lib.b200kv_nvls_signal_bytes() >= (64 + 2 * 256 * 8) * 4
    rs = (ctypes.c_void_p * 2)(1 << 20, 1 << 21)
    sig = (ctypes.c_void_p * 2)(1 << 24, 1 << 25)

    def ll(data=1 << 22, ag=1 << 23, ag_mc=1 << 26, region=1024, signal=1 << 24, rank=0, world=2, n=512,
           ctas=0, table=rs):
        return lib.b200kv_nvls_allreduce_ll_f16(data, table, ag, ag_mc, region, signal, rank, world, n, ctas,
                                                None, None)

    assert ll(n=0) == 0                                   # nothing to do, nothing launched
    for kw, msg in [(dict(world=9), "world"), (dict(rank=2), "rank"), (dict(n=24), "multiple of 8 * world"),
                    (dict(region=256), "region_elems"), (dict(region=1020), "region_elems"),
                    (dict(ctas=257), "ctas"), (dict(data=None), "aligned"), (dict(ag_mc=(1 << 26) + 8), "aligned"),
                    (dict(table=(ctypes.c_void_p * 2)(1 << 20, None)), "reduce-scatter region")]:
        assert ll(**kw) == 1, kw
        assert msg in _lib.last_error(), (kw, _lib.last_error())
    # the in-switch form: the same limits on world, size and CTAs
    assert lib.b200kv_nvls_allreduce_f16(1 << 26, sig, 0, 2, 24, 32, None, None) == 1
    assert lib.b200kv_nvls_allreduce_f16(1 << 26, sig, 0, 2, 512, 257, None, None) == 1
    assert "ctas" in _lib.last_error()
    assert lib.b200kv_nvls_allreduce_f16(1 << 26, sig, 0, 2, 0, 32, None, None) == 0
