"""The CPU oracle against the reference's golden vectors and against itself."""

import json

import numpy as np
import pytest
import torch

from oracle import kv_relayout as okv
from oracle import paged_attention as opa
from oracle import stick_layout as osl
from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs, seeded_randn


def _sha(t):
    import hashlib

    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def _ref_decode_inputs(hkv):
    q = seeded_randn((2, 1, 32, 128), 1).transpose(1, 2)
    k = seeded_randn((2, 257, hkv, 128), 2).transpose(1, 2)
    v = seeded_randn((2, 257, hkv, 128), 3).transpose(1, 2)
    return q, k, v


def _dense_to_paged(k, v, perm_seed=0):
    """Packs dense [B, Hkv, S, D] K/V into shuffled pages (oracle relayout)."""
    B, hkv, S, D = k.shape
    nb = -(-S // 64)
    rng = np.random.default_rng(perm_seed)
    ids = rng.permutation(B * nb * 2)[: B * nb].reshape(B, nb).astype(np.int32)
    pool_shape = (B * nb * 2, hkv, D // 64, 64, 64)
    kp = np.full(pool_shape, np.nan, dtype=np.float16)
    vp = np.full(pool_shape, np.nan, dtype=np.float16)
    for b in range(B):
        kp = okv.rows_to_pool(k[b].transpose(0, 1).numpy(), kp, ids[b])
        vp = okv.rows_to_pool(v[b].transpose(0, 1).numpy(), vp, ids[b])
    return torch.from_numpy(kp), torch.from_numpy(vp), torch.from_numpy(ids)


@pytest.mark.parametrize("case,hkv", [("mha_decode", 32), ("gqa_decode", 8)])
def test_golden_inputs_reproduce(golden_dir, case, hkv):
    meta = json.loads((golden_dir / "sdpa_decode_golden.json").read_text())[case]
    q, k, v = _ref_decode_inputs(hkv)
    assert (_sha(q), _sha(k), _sha(v)) == (meta["sha_q"], meta["sha_k"], meta["sha_v"])


@pytest.mark.parametrize("case,hkv", [("mha_decode", 32), ("gqa_decode", 8)])
def test_oracle_matches_reference_cpu_golden(golden_dir, case, hkv):
    """Paged gather + CPU SDPA == the reference harness's CPU result (ctx 257,
    a partial last page, pages shuffled, unused pool slots NaN)."""
    g = np.load(golden_dir / "sdpa_decode_golden.npz")
    q, k, v = _ref_decode_inputs(hkv)
    kp, vp, bt = _dense_to_paged(k, v)
    ctx = torch.full((2,), 257, dtype=torch.int32)
    out, lse = opa.decode_attention_cpu(q[:, :, 0], kp, vp, bt, ctx, return_lse=True)
    ref32 = torch.from_numpy(g[f"{case}_out_fp32"])[:, :, 0]
    ref16 = torch.from_numpy(g[f"{case}_out_native"])[:, :, 0]
    torch.testing.assert_close(out.float(), ref32.float(), atol=1e-3, rtol=0)
    torch.testing.assert_close(out.float(), ref16.float(), atol=2e-3, rtol=1e-2)
    torch.testing.assert_close(lse, torch.from_numpy(g[f"{case}_lse"]), atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("hkv", [32, 8])
def test_decomposition_restatement_agrees(hkv):
    q, k, v = _ref_decode_inputs(hkv)
    a = opa.sdpa_decomposition_cpu(q, k, v)
    b = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), enable_gqa=hkv != 32)
    torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5)


def test_empty_context_is_zero():
    inp = make_decode_inputs(DECODE_CONFIGS["gqa_b16"], ctx=[0, 70], batch=2)
    out, lse = opa.decode_attention_cpu(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens,
                                        return_lse=True)
    assert torch.count_nonzero(out[0]) == 0 and torch.isinf(lse[0]).all()
    assert torch.isfinite(out[1].float()).all()


def test_relayout_round_trip_and_append():
    rng = np.random.default_rng(1)
    T, hkv, D = 200, 3, 128
    rows = rng.standard_normal((T, hkv, D)).astype(np.float16)
    pool = np.zeros((10, hkv, 2, 64, 64), dtype=np.float16)
    ids = np.array([7, 2, 9, 0], dtype=np.int32)
    pool = okv.rows_to_pool(rows, pool, ids)
    assert np.array_equal(okv.pool_to_rows(pool, ids, T).view(np.int16), rows.view(np.int16))
    # page element map == generic stick layout of a [64, D] tile
    dev, smap = osl.default_layout([64, D])
    for j in range(3):
        tile = rows[j * 64:(j + 1) * 64, 1]
        assert np.array_equal(pool[ids[j], 1].reshape(-1).view(np.int16),
                              osl.to_device(tile, dev, smap).view(np.int16))
    new = rng.standard_normal((3, hkv, D)).astype(np.float16)
    slots = np.array([7 * 64 + 5, -1, 9 * 64 + 63])
    p2 = okv.append(new, pool, slots)
    assert np.array_equal(p2[7, :, :, 5, :].reshape(hkv, D), new[0])
    assert np.array_equal(p2[9, :, :, 63, :].reshape(hkv, D), new[2])
    with pytest.raises(IndexError):
        okv.append(new, pool, np.array([10 * 64, -1, -1]))


def test_index_copy_golden(golden_dir):
    """KV append of the reference's index_copy_ tests (prefill 0-13, decode 14)
    through relayout -> append -> unrelayout equals torch CPU index_copy_."""
    meta = json.loads((golden_dir / "index_copy_golden.json").read_text())
    cache = seeded_randn((1, 8, 2048, 128))
    assert _sha(cache) == meta["sha_cache"]
    rows = cache[0].transpose(0, 1).contiguous().numpy()          # [2048, 8, 128]
    ids = np.arange(32, dtype=np.int32)[::-1].copy()
    pool = okv.rows_to_pool(rows, np.zeros((32, 8, 2, 64, 64), np.float16), ids)
    for tag, n, pos in (("prefill", 14, np.arange(14)), ("decode", 1, np.array([14]))):
        src = seeded_randn((1, 8, n, 128), tag)[0].transpose(0, 1).contiguous().numpy()
        slots = ids[pos // 64].astype(np.int64) * 64 + pos % 64
        p2 = okv.append(src, pool, slots)
        back = torch.from_numpy(okv.pool_to_rows(p2, ids, 2048)).transpose(0, 1).unsqueeze(0)
        assert _sha(back) == meta[f"sha_after_{tag}"]
