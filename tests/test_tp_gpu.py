"""Tensor-parallel decode over NCCL on 2 GPUs of one node (skipped with fewer).

Each rank runs the CUDA decode kernel on its KV-head shard, its o_proj partial
and an NCCL SUM all-reduce; the result must match the single-GPU computation
of all heads (decode parity tolerance, then fp16 matmul / all-reduce rounding).
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs

    cfg = DECODE_CONFIGS["tp70b"]
    inp = make_decode_inputs(cfg, ctx=[1000, 64, 3000, 17, 4096, 2000, 5, 777], seed_tag="tp-gpu")
    g = torch.Generator().manual_seed(11)
    w_o = (torch.randn((1024, cfg.num_q_heads * cfg.head_dim), generator=g) * 0.02).to(torch.float16)
    return cfg, inp, w_o


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    import torch_spyre_b200  # noqa: F401
    from torch_spyre_b200.tp import HeadShard, tp_decode_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg, inp, w_o = _inputs()
        shard = HeadShard(rank, world, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
        dev = torch.device("cuda", rank)
        y = tp_decode_step(shard, shard.shard_q(inp.q.to(dev)), shard.shard_pool(inp.k_pool).to(dev),
                           shard.shard_pool(inp.v_pool).to(dev), inp.block_table.to(dev),
                           inp.context_lens.to(dev), shard.shard_w_o(w_o).to(dev))
        torch.cuda.synchronize()
        results[rank] = ("ok", y.cpu())
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_nccl_matches_single_gpu():
    import torch_spyre_b200 as tsb

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert not p.is_alive(), "a rank hung"
    res = dict(results)
    assert all(v[0] == "ok" for v in res.values()), res
    cfg, inp, w_o = _inputs()
    attn = tsb.decode_attention(inp.q.cuda(), inp.k_pool.cuda(), inp.v_pool.cuda(), inp.block_table.cuda(),
                                inp.context_lens.cuda())
    ref = (attn.reshape(attn.shape[0], -1).float() @ w_o.cuda().float().t()).cpu()
    for r in range(2):
        torch.testing.assert_close(res[r][1].float(), ref, atol=1e-2, rtol=1e-2)
    assert torch.equal(res[0][1], res[1][1])
