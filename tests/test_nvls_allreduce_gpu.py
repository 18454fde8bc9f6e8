"""NVLink SHARP all-reduce (b200kv_nvls_allreduce_f16, and its low-latency
form b200kv_nvls_allreduce_ll_f16) on 2, 4 and 8 GPUs of one node (skipped
with fewer GPUs, or when the GPUs offer no multicast).

* every rank ends with the same bits, and each element is the sum of the
  ranks' fp16 values accumulated in fp32 and rounded once to fp16 (the
  switch's fp32 adds may associate differently from rank order, which can
  move a sum by at most one fp16 ulp);
* repeated calls of several sizes and CUDA-graph replays with new inputs
  (the epoch lives in device memory);
* the low-latency form: sums are the fp32 rank-order sums rounded once
  (bit-exact), partials with NaN and inf give the same NaN/inf sums as fp32
  arithmetic (NaN as the canonical 0x7E00), and the receive regions are
  back to their sentinel after every call.
Ranks are spawned processes; every rank runs to its clean exit (no rank
leaves while its memory is bound to the multicast object).
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


def _partials(world, n, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(n, generator=g) * 3).to(torch.float16) for _ in range(world)]


def _expected(parts):
    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for p in parts:
        acc += p.float()
    return acc.to(torch.float16)


SIZES = [128 * 8192, 16 * 8192, 4096]


def _worker(rank, world, port, results, low_latency):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ar = None
    try:
        from torch_spyre_b200.tp import NvlsAllReduce

        try:
            ar = NvlsAllReduce(128 * 8192, low_latency=low_latency)
        except RuntimeError as e:
            results[rank] = ("unavailable", str(e))
            return
        out = []
        for i, n in enumerate(SIZES):
            buf = ar.buffer((n,))
            buf.copy_(_partials(world, n, 100 + i)[rank].cuda())
            ar.all_reduce(buf)
            torch.cuda.synchronize()
            out.append(buf.cpu().clone())
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
        del g
        special = None
        if low_latency:  # NaN and inf partials, then the result region's state
            n = 8 * 8 * world
            buf = ar.buffer((n,))
            buf.copy_(_special_partials(world, n)[rank].cuda())
            ar.all_reduce(buf)
            torch.cuda.synchronize()
            special = buf.cpu().clone()
            region = ar._buf[ar._rs_off: ar._sig_off]
            assert bool((region == 0xFF).all()), "receive regions not restored"
        results[rank] = ("ok", out, graphed, int(ar.error_flag.item()), special)
    except Exception as e:
        results[rank] = ("error", f"{type(e).__name__}: {e}")
    finally:
        if ar is not None:
            ar.close()
        dist.destroy_process_group()


def _close_enough(y, exp):
    # at most one fp16 ulp apart (the switch's fp32 association), zeros exact
    d = (y.float() - exp.float()).abs()
    ulp = torch.finfo(torch.float16).eps * exp.float().abs().clamp(min=2.0 ** -14)
    return bool((d <= ulp).all())


def _special_partials(world, n):
    parts = _partials(world, n, 300)
    parts[0][0] = float("nan")
    parts[0][1] = float("inf")
    parts[world - 1][1] = float("-inf")  # inf - inf: NaN
    parts[0][2] = float("inf")           # inf + finite: inf
    parts[world - 1][3] = 60000.0        # fp16 overflow in the sum (fp32 sum > 65504 rounds to inf)
    parts[0][3] = 60000.0
    return parts


@pytest.mark.parametrize("low_latency", [False, True], ids=["two_barrier", "low_latency"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_nvls_allreduce_sums(world, low_latency):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results, low_latency)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert not p.is_alive(), "a rank hung"
    res = dict(results)
    if any(v[0] == "unavailable" for v in res.values()):
        pytest.skip("no NVLink multicast: " + next(v[1] for v in res.values() if v[0] == "unavailable"))
    assert len(res) == world and all(v[0] == "ok" for v in res.values()), res
    for r in range(world):
        _, out, graphed, flag, special = res[r]
        assert flag == 0
        for i, n in enumerate(SIZES):
            assert _close_enough(out[i], _expected(_partials(world, n, 100 + i)))
            if low_latency:  # the owner's fp32 rank-order sum, rounded once
                assert torch.equal(out[i], _expected(_partials(world, n, 100 + i)))
            assert torch.equal(out[i], res[0][1][i])
        for k in range(3):
            assert _close_enough(graphed[k], _expected(_partials(world, 64 * 8192, 200 + k)))
            if low_latency:
                assert torch.equal(graphed[k], _expected(_partials(world, 64 * 8192, 200 + k)))
            assert torch.equal(graphed[k], res[0][2][k])
        if low_latency:
            exp = _expected(_special_partials(world, 8 * 8 * world))
            assert torch.equal(special.isnan(), exp.isnan())
            fin = ~exp.isnan()
            assert torch.equal(special[fin].isinf(), exp[fin].isinf())
            assert bool((special[exp.isnan()].view(torch.int16) == 0x7E00).all())
            ok = fin & ~exp.isinf()
            assert _close_enough(special[ok], exp[ok])
            assert torch.equal(special.view(torch.int16), res[0][4].view(torch.int16))
