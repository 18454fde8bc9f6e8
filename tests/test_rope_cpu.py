"""Rotary embedding oracle (pinned to the reference's rope dataflow on its own
inputs) and host-side checks of the rope op (no GPU work)."""

import hashlib
import json

import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import rope as orope
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import seeded_randn

CASES = ["prefill_bs1", "prefill", "decode_bs1", "decode"]


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def _case(meta):
    q = seeded_randn(tuple(meta["q_shape"]), dtype=torch.float16)
    freqs = seeded_randn(tuple(meta["freqs_shape"]), dtype=torch.float16)
    assert _sha(q) == meta["sha_q"] and _sha(freqs) == meta["sha_freqs"]
    B, S, E = q.shape
    D = freqs.shape[-1] * 2
    rows = q.reshape(B * S, E // D, D)
    pos = torch.arange(S, dtype=torch.int32).repeat(B)
    return q, freqs, rows, pos


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_dataflow(golden_dir, name):
    meta = json.loads((golden_dir / "rope_golden.json").read_text())[name]
    q, freqs, rows, pos = _case(meta)
    out = orope.rope_rows(rows, freqs[0], pos)
    assert _sha(out.reshape(meta["out_shape"])) == meta["sha_out"]
    torch.testing.assert_close(out.float(), orope.rope_float(rows, freqs[0], pos), atol=2e-2, rtol=2e-3)


def test_oracle_known_answers():
    x = torch.randn(3, 2, 8).to(torch.float16)
    ident = torch.zeros(5, 2, 2, 4, dtype=torch.float16)
    ident[:, 0, 0] = 1
    ident[:, 1, 1] = 1
    swap = torch.zeros_like(ident)
    swap[:, 0, 1] = 1
    swap[:, 1, 0] = 1
    pos = torch.tensor([0, 4, 2], dtype=torch.int32)
    assert torch.equal(orope.rope_rows(x, ident, pos), x)
    assert torch.equal(orope.rope_rows(x, swap, pos), torch.cat([x[..., 4:], x[..., :4]], dim=-1))
    # a quarter turn at position 2 only: (x0, x1) -> (-x1, x0)
    rot = ident.clone()
    rot[2] = 0
    rot[2, 0, 1] = -1
    rot[2, 1, 0] = 1
    out = orope.rope_rows(x, rot, pos)
    assert torch.equal(out[2], torch.cat([-x[2, :, 4:], x[2, :, :4]], dim=-1))
    assert torch.equal(out[0], x[0])


def test_rope_op_rejects_cpu_and_bad_shapes():
    x = torch.zeros(2, 4, 128, dtype=torch.float16)
    f = torch.zeros(8, 2, 2, 64, dtype=torch.float16)
    pos = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CPU"):
        tsb.rope(x, f, pos)
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        xf = torch.empty(2, 4, 128, dtype=torch.float16, device="cuda")
        ff = torch.empty(8, 2, 2, 64, dtype=torch.float16, device="cuda")
        pf = torch.empty(2, dtype=torch.int32, device="cuda")
        y = torch.ops.b200kv.rope(xf, ff, pf, None)
        assert y.shape == (2, 4, 128) and y.dtype == torch.float16


def test_c_abi_checks():
    lib = _lib.lib()
    args = [1 << 20, 512, 128, 1 << 21, 512, 128, 1 << 22, 16, 1 << 23, 4, 4, 128, None, None]
    assert lib.b200kv_rope_f16(*[a if i != 11 else 126 for i, a in enumerate(args)]) == 1  # head_dim % 4
    assert lib.b200kv_rope_f16(*[a if i != 7 else 0 for i, a in enumerate(args)]) == 1     # max_pos
    assert lib.b200kv_rope_f16(*[a if i != 0 else None for i, a in enumerate(args)]) == 1  # null x
    assert lib.b200kv_rope_f16(*[a if i != 9 else 0 for i, a in enumerate(args)]) == 0     # no tokens
