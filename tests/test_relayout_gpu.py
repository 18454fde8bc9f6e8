"""GPU KV append / relayout, bit-exact against the numpy oracle."""

import hashlib
import json

import numpy as np
import pytest
import torch

import torch_spyre_b200 as tsb
from oracle import kv_relayout as okv
from torch_spyre_b200 import _lib
from torch_spyre_b200.workloads import RELAYOUT_CONFIG, seeded_generator, seeded_randn

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.cpu().contiguous().view(torch.int16)


def test_bulk_relayout_full_size_round_trip():
    cfg = RELAYOUT_CONFIG
    T, hkv, D = cfg.bulk_tokens, cfg.num_kv_heads, cfg.head_dim
    g = seeded_generator("relayout", "bulk", device="cuda")
    rows = torch.randn((T, hkv, D), generator=g, device="cuda", dtype=torch.float16)
    nb = 2 * T // 64
    ids = torch.randperm(nb, generator=seeded_generator("relayout", "ids"))[: T // 64].to(torch.int32)
    pool = torch.zeros((nb, hkv, 2, 64, 64), dtype=torch.float16, device="cuda")
    tsb.kv_relayout(rows, pool, ids.cuda())
    back = tsb.kv_unrelayout(pool, ids.cuda(), T)
    assert torch.equal(_bits(back), _bits(rows))
    # spot-check against the oracle on a slice of pages (the full oracle is slow)
    sub = slice(0, 64 * 37)
    ref = okv.rows_to_pool(rows[sub].cpu().numpy(), np.zeros((nb, hkv, 2, 64, 64), np.float16),
                           ids[:37].numpy())
    got = pool.cpu().numpy()
    for j in range(37):
        assert np.array_equal(got[int(ids[j])].view(np.int16), ref[int(ids[j])].view(np.int16))


@pytest.mark.parametrize("T", [1, 63, 64, 65, 200, 4096 + 17])
def test_relayout_partial_pages_match_oracle(T):
    hkv, D = 3, 128
    rows = torch.randn((T, hkv, D), dtype=torch.float16)
    nb = -(-T // 64) + 3
    ids = torch.randperm(nb)[: -(-T // 64)].to(torch.int32)
    pool0 = torch.randn((nb, hkv, 2, 64, 64), dtype=torch.float16)
    pool = pool0.cuda()
    tsb.kv_relayout(rows.cuda(), pool, ids.cuda())
    ref = okv.rows_to_pool(rows.numpy(), pool0.numpy(), ids.numpy())
    assert np.array_equal(pool.cpu().numpy().view(np.int16), ref.view(np.int16))
    back = tsb.kv_unrelayout(pool, ids.cuda(), T)
    assert torch.equal(_bits(back), _bits(rows))


def test_append_config_matches_oracle():
    cfg = RELAYOUT_CONFIG
    n, hkv, D = cfg.append_tokens, cfg.num_kv_heads, cfg.head_dim
    nb = 512
    g = seeded_generator("append", "slots")
    slots = torch.randperm(nb * 64, generator=g)[:n].to(torch.int64)
    slots[5] = -1  # a padding token
    k_new = seeded_randn((n, hkv, D), "k_new")
    v_new = seeded_randn((n, hkv, D), "v_new")
    k0 = seeded_randn((nb, hkv, 2, 64, 64), "k_pool")
    v0 = seeded_randn((nb, hkv, 2, 64, 64), "v_pool")
    kp, vp = k0.cuda(), v0.cuda()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.kv_append(k_new.cuda(), v_new.cuda(), kp, vp, slots.cuda(), error_flag=flag)
    assert int(flag.item()) == 0
    kr = okv.append(k_new.numpy(), k0.numpy(), slots.numpy())
    vr = okv.append(v_new.numpy(), v0.numpy(), slots.numpy())
    assert np.array_equal(kp.cpu().numpy().view(np.int16), kr.view(np.int16))
    assert np.array_equal(vp.cpu().numpy().view(np.int16), vr.view(np.int16))


def test_append_strided_source():
    """k_new / v_new as views of a fused qkv projection output."""
    n, hkv, D = 7, 4, 128
    qkv = torch.randn((n, 3, hkv, D), dtype=torch.float16, device="cuda")
    k_new, v_new = qkv[:, 1], qkv[:, 2]
    pool_k = torch.zeros((4, hkv, 2, 64, 64), dtype=torch.float16, device="cuda")
    pool_v = torch.zeros_like(pool_k)
    slots = torch.tensor([0, 5, 64, 100, 255, 3, 7], dtype=torch.int64)
    tsb.kv_append(k_new, v_new, pool_k, pool_v, slots.cuda())
    kr = okv.append(k_new.cpu().numpy(), np.zeros((4, hkv, 2, 64, 64), np.float16), slots.numpy())
    assert np.array_equal(pool_k.cpu().numpy().view(np.int16), kr.view(np.int16))


def test_append_bad_slot_flag_no_fault():
    pool = torch.zeros((2, 1, 2, 64, 64), dtype=torch.float16, device="cuda")
    new = torch.ones((2, 1, 128), dtype=torch.float16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.kv_append(new, new, pool, pool.clone(), torch.tensor([3, 128], device="cuda"), error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.DEVERR_BAD_SLOT
    assert float(pool[0, 0, :, 3].sum()) == 128.0


def test_relayout_bad_block_flag_no_fault():
    rows = torch.ones((100, 1, 128), dtype=torch.float16, device="cuda")
    pool = torch.zeros((2, 1, 2, 64, 64), dtype=torch.float16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    tsb.kv_relayout(rows, pool, torch.tensor([1, 7], dtype=torch.int32, device="cuda"), error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & _lib.DEVERR_BAD_BLOCK
    assert float(pool[1].sum()) == 64 * 128


def test_index_copy_golden_on_gpu(golden_dir):
    """The reference's index_copy_ KV-cache tests through the GPU ops."""
    meta = json.loads((golden_dir / "index_copy_golden.json").read_text())
    cache = seeded_randn((1, 8, 2048, 128))
    rows = cache[0].transpose(0, 1).contiguous().cuda()
    ids = torch.arange(32, dtype=torch.int32).flip(0).contiguous()
    for tag, pos in (("prefill", torch.arange(14)), ("decode", torch.tensor([14]))):
        kp = torch.zeros((32, 8, 2, 64, 64), dtype=torch.float16, device="cuda")
        vp = torch.zeros_like(kp)
        tsb.kv_relayout(rows, kp, ids.cuda())
        src = seeded_randn((1, 8, len(pos), 128), tag)[0].transpose(0, 1).contiguous().cuda()
        slots = (ids[pos // 64].long() * 64 + pos % 64).cuda()
        tsb.kv_append(src, src, kp, vp, slots)
        back = tsb.kv_unrelayout(kp, ids.cuda(), 2048).cpu().transpose(0, 1).unsqueeze(0)
        h = hashlib.sha256(back.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()
        assert h == meta[f"sha_after_{tag}"]
