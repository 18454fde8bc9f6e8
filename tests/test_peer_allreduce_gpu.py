"""Peer-memory all-reduce (b200kv_peer_allreduce_f16) on 2 GPUs of one node.

* sums are bit-exact against fp32 accumulation in rank order rounded once;
* repeated calls and CUDA-graph replays (the epoch lives in device memory);
* the fused o_proj + all-reduce kernel against the fp32 sum of the ranks'
  o_proj products (the TP decode step through every all-reduce path is checked
  against the CPU oracle in test_tp_gpu.py);
* a peer that never joins ends the wait after its 2 s bound with
  B200KV_DEVERR_TIMEOUT, and the context stays usable.
Ranks run as spawned processes (NVLS off; the kernel uses plain peer stores).
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _partials(world, n, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(n, generator=g) * 3).to(torch.float16) for _ in range(world)]


def _expected(parts):
    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for p in parts:
        acc += p.float()
    return acc.to(torch.float16)


def _w_sums(rank, world, port, results):
    dist = _init(rank, world, port)
    from torch_spyre_b200.tp import PeerAllReduce

    try:
        ar = PeerAllReduce(128 * 8192)
        out = []
        for i, n in enumerate([128 * 8192, 16 * 8192, 8 * world, 4096 * world]):
            buf = ar.buffer((n,))
            buf.copy_(_partials(world, n, 100 + i)[rank].cuda())
            ar.all_reduce(buf)
            torch.cuda.synchronize()
            out.append(buf.cpu().clone())
        # a captured graph replayed with new inputs each time
        n = 64 * 8192
        src = torch.empty(n, dtype=torch.float16, device="cuda")
        buf = ar.buffer((n,))
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            buf.copy_(src)
            ar.all_reduce(buf)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                buf.copy_(src)
                ar.all_reduce(buf)
        torch.cuda.current_stream().wait_stream(s)
        graphed = []
        for k in range(3):
            src.copy_(_partials(world, n, 200 + k)[rank].cuda())
            g.replay()
            torch.cuda.synchronize()
            graphed.append(buf.cpu().clone())
        flag = int(ar.error_flag.item())
        del g
        ar.close()
        results[rank] = ("ok", out, graphed, flag)
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


def _run(target, world=2, timeout=300):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        assert not p.is_alive(), "a rank hung"
    res = dict(results)
    assert all(v[0] == "ok" for v in res.values()), res
    return res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce_sums_bit_exact(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run(_w_sums, world)
    sizes = [128 * 8192, 16 * 8192, 8 * world, 4096 * world]
    for r in range(world):
        _, out, graphed, flag = res[r]
        assert flag == 0
        for i, n in enumerate(sizes):
            assert torch.equal(out[i].view(torch.int16), _expected(_partials(world, n, 100 + i)).view(torch.int16))
        for k in range(3):
            exp = _expected(_partials(world, 64 * 8192, 200 + k))
            assert torch.equal(graphed[k].view(torch.int16), exp.view(torch.int16))


def _w_timeout(rank, world, port, results):
    dist = _init(rank, world, port)
    from torch_spyre_b200._lib import DEVERR_TIMEOUT
    from torch_spyre_b200.tp import PeerAllReduce

    try:
        ar = PeerAllReduce(8 * 1024)
        flag = 0
        if rank == 0:  # rank 1 never joins this call: rank 0's waits run out
            buf = ar.buffer((8 * 1024,))
            buf.fill_(1.0)
            ar.all_reduce(buf)
            torch.cuda.synchronize()
            flag = int(ar.error_flag.item())
        # the context is still usable
        x = torch.arange(16, device="cuda", dtype=torch.float32).sum().item()
        ar.close()
        results[rank] = ("ok", flag, x, DEVERR_TIMEOUT)
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


def test_missing_peer_times_out_with_status():
    res = _run(_w_timeout, 2)
    _, flag, x, timeout_bit = res[0]
    assert flag & timeout_bit
    assert x == 120.0 and res[1][2] == 120.0


def _w_fused(rank, world, port, results):
    dist = _init(rank, world, port)
    from torch_spyre_b200.tp import PeerAllReduce

    try:
        B, N, K = 128, 8192, 2048
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        attn = torch.randn((B, K), generator=g, device="cuda", dtype=torch.float16)
        w = torch.randn((N, K), generator=g, device="cuda", dtype=torch.float16) * 0.02
        ar = PeerAllReduce(B * N)
        fused = ar.oproj_all_reduce(attn, w).cpu()
        # the unfused path on the same buffers (epochs interleave), then fused again
        part = ar.buffer((B, N))
        torch.matmul(attn, w.t(), out=part)
        unfused = ar.all_reduce(part).cpu().clone()
        fused2 = ar.oproj_all_reduce(attn[:77], w).cpu()
        torch.cuda.synchronize()
        flag = int(ar.error_flag.item())
        ar.close()
        results[rank] = ("ok", fused, unfused, fused2, flag, attn.cpu(), w.cpu())
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()


def test_fused_oproj_allreduce_two_ranks():
    res = _run(_w_fused, 2)
    ref = sum((res[r][5].float() @ res[r][6].float().t()) for r in range(2))
    for r in range(2):
        _, fused, unfused, fused2, flag, _, _ = res[r]
        assert flag == 0
        torch.testing.assert_close(fused.float(), ref, atol=3e-2, rtol=1e-2)
        torch.testing.assert_close(fused.float(), unfused.float(), atol=3e-2, rtol=1e-2)
        assert torch.equal(fused2, fused[:77])
    assert torch.equal(res[0][1], res[1][1]) and torch.equal(res[0][3], res[1][3])
