"""Tensor-parallel host logic on CPU ranks (gloo, world size 2).

The per-rank attention is the CPU oracle (no GPU here); what is tested is the
head/column sharding, the o_proj partials and the SUM all-reduce, against the
single-rank computation -- and that a rank that dies before the collective is
reported as an error by its peer instead of hanging it.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from torch_spyre_b200.tp import HeadShard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs

    cfg = DECODE_CONFIGS["tp70b"]
    inp = make_decode_inputs(cfg, ctx=[100, 64, 300, 7], seed_tag="tp-gloo")
    g = torch.Generator().manual_seed(7)
    w_o = (torch.randn((256, cfg.num_q_heads * cfg.head_dim), generator=g) * 0.02).to(torch.float16)
    return cfg, inp, w_o


def _oracle_attn(q, k_pool, v_pool, block_table, context_lens):
    from oracle import paged_attention as opa

    return opa.decode_attention_cpu(q, k_pool, v_pool, block_table, context_lens).float()


def _worker(rank, world, port, results, fail_rank):
    import datetime

    import torch.distributed as dist

    from torch_spyre_b200.tp import HeadShard, tp_decode_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        cfg, inp, w_o = _inputs()
        shard = HeadShard(rank, world, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
        y = tp_decode_step(shard, shard.shard_q(inp.q), shard.shard_pool(inp.k_pool), shard.shard_pool(inp.v_pool),
                           inp.block_table, inp.context_lens, shard.shard_w_o(w_o).float(), attn_fn=_oracle_attn)
        results[rank] = ("ok", y)
    except Exception as e:  # reported to the parent, never swallowed
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert not p.is_alive(), "a rank hung"
    return dict(results)


def test_head_shard_partition():
    s = [HeadShard(r, 4, 64, 8, 128) for r in range(4)]
    assert [list(x.kv_heads) for x in s] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert s[1].q_heads == range(16, 32) and s[1].w_cols == slice(2048, 4096)
    q = torch.zeros(3, 64, 128)
    assert s[3].shard_q(q).shape == (3, 16, 128)
    with pytest.raises(ValueError):
        HeadShard(0, 3, 64, 8, 128)


def test_tp_world2_matches_single_rank():
    res = _run(2)
    assert all(v[0] == "ok" for v in res.values()), res
    cfg, inp, w_o = _inputs()
    full = _oracle_attn(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens)
    ref = full.reshape(full.shape[0], -1) @ w_o.float().t()
    for r in range(2):
        torch.testing.assert_close(res[r][1], ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(res[0][1], res[1][1], atol=0, rtol=0)


def test_dead_rank_is_reported_not_hung():
    res = _run(2, fail_rank=1)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    assert res[0][0] == "error", "the surviving rank must see the collective fail"
