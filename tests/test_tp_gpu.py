"""Head-sharded tensor-parallel decode step on 2 and 4 GPUs of one node
(skipped with fewer), checked against the CPU oracle.

Each rank runs the CUDA decode kernel on its KV-head shard and its o_proj
partial, then the SUM all-reduce (the reference's TP collective,
SpyreCCLBackend::allreduce, torch_spyre/csrc/distributed/spyre_ccl.cpp:470-494)
by each path: NCCL, the peer-memory all-reduce kernel, the fused o_proj +
all-reduce kernel, and (where the GPUs offer NVLink multicast) the two NVLink
SHARP all-reduce kernels.  Every result must match the oracle -- the
reference's CPU eager decode of all heads followed by the full o_proj in fp32
-- within 1e-2 abs + 1e-2 rel (the decode tolerance carried through an fp16
attention output and fp16 partials summed over K = 8192 / N products), and
every rank must hold the same bits.  Ranks are spawned processes (NCCL's own
NVLS off) that all run to their clean exit.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 1e-2
CTX = [1000, 64, 3000, 17, 4096, 2000, 5, 777]  # partial pages, a context shorter than one page
HIDDEN = 1024


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from torch_spyre_b200.workloads import DECODE_CONFIGS, make_decode_inputs

    cfg = DECODE_CONFIGS["tp70b"]
    inp = make_decode_inputs(cfg, ctx=CTX, seed_tag="tp-gpu")
    g = torch.Generator().manual_seed(11)
    w_o = (torch.randn((HIDDEN, cfg.num_q_heads * cfg.head_dim), generator=g) * 0.02).to(torch.float16)
    return cfg, inp, w_o


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    import torch_spyre_b200  # noqa: F401
    from torch_spyre_b200.tp import HeadShard, NvlsAllReduce, PeerAllReduce, tp_decode_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg, inp, w_o = _inputs()
        shard = HeadShard(rank, world, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
        dev = torch.device("cuda", rank)
        args = (shard, shard.shard_q(inp.q.to(dev)), shard.shard_pool(inp.k_pool).to(dev),
                shard.shard_pool(inp.v_pool).to(dev), inp.block_table.to(dev), inp.context_lens.to(dev),
                shard.shard_w_o(w_o).to(dev))
        y_nccl = tp_decode_step(*args).cpu()
        ar = PeerAllReduce(128 * HIDDEN)  # the fused kernel's receive regions cover 128 rows
        y_peer = tp_decode_step(*args, allreduce=ar).cpu().clone()
        y_fused = tp_decode_step(*args, allreduce=ar, fused_oproj=True).cpu()
        torch.cuda.synchronize()
        flag = int(ar.error_flag.item())
        ar.close()
        ys = {"nccl": y_nccl, "peer": y_peer, "fused": y_fused}
        try:  # the NVLink SHARP all-reduce, where the GPUs offer multicast
            nv = NvlsAllReduce(128 * HIDDEN, low_latency=False)
        except RuntimeError:
            nv = None
        if nv is not None:
            ys["nvls"] = tp_decode_step(*args, allreduce=nv).cpu().clone()
            torch.cuda.synchronize()
            flag |= int(nv.error_flag.item())
            nv.close()
            nv = NvlsAllReduce(128 * HIDDEN, low_latency=True)
            ys["nvls_ll"] = tp_decode_step(*args, allreduce=nv).cpu().clone()
            torch.cuda.synchronize()
            flag |= int(nv.error_flag.item())
            nv.close()
        results[rank] = ("ok", ys, flag)
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_step_matches_oracle(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle.tp_step import tp_step_cpu

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert not p.is_alive(), "a rank hung"
    res = dict(results)
    assert len(res) == world and all(v[0] == "ok" for v in res.values()), res
    cfg, inp, w_o = _inputs()
    ref = tp_step_cpu(inp.q, inp.k_pool, inp.v_pool, inp.block_table, inp.context_lens, w_o)
    for r in range(world):
        _, ys, flag = res[r]
        assert flag == 0
        for path, y in ys.items():
            torch.testing.assert_close(y.float(), ref, atol=ATOL, rtol=RTOL, msg=lambda m: f"{path}: {m}")
    for path in res[0][1]:
        for r in range(1, world):
            assert torch.equal(res[0][1][path], res[r][1][path]), f"{path}: ranks 0 and {r} differ"
