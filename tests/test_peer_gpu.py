"""nk_allreduce_bf16 (include/nk_comm.h) on 2+ GPUs, one process per GPU.

* Exactness: every rank gets bf16(x_0 + x_1 + ...) summed in rank order — bit-identical to the
  same fp32 sum done by PyTorch on the gathered partials — for several sizes, back-to-back
  calls (both buffer sets, reused), and replays of a CUDA graph holding the calls.
* Failure detection: when one rank does not make a call, the others' bounded wait gives up
  after ~2 s and reports NK_ERR_TIMEOUT through the device error word; no rank leaves while
  a kernel is in flight, NVLS is off and only plain peer loads and stores are used.
Skipped with fewer than two GPUs.
"""

import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

N_GPUS = torch.cuda.device_count() if torch.cuda.is_available() else 0


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def _exact_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from neokernel_b200.peer import PeerGroup
        dev = torch.device("cuda", rank)
        sizes = (4, 1020, 5120, 8 * 5120, 32 * 5120, 1 << 20)
        peer = PeerGroup(max(sizes), device=dev)
        worst = 0
        for call, n in enumerate(sizes * 2):
            g = torch.Generator(device=dev).manual_seed(1000 * call + rank)
            x = torch.randn(n, generator=g, device=dev) * 3.0
            out = torch.empty(n, dtype=torch.bfloat16, device=dev)
            peer.allreduce_bf16(x, out)
            allx = [torch.empty_like(x).cpu() for _ in range(world)]
            dist.all_gather(allx, x.cpu())
            ref = allx[0].clone()
            for r in range(1, world):
                ref += allx[r]  # rank order, fp32
            torch.cuda.synchronize(dev)
            worst = max(worst, int((out.cpu() != ref.to(torch.bfloat16)).sum()))
        # a CUDA graph of three calls on fixed buffers, replayed with new data
        n = 5120
        xs = [torch.empty(n, device=dev) for _ in range(3)]
        outs = [torch.empty(n, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        s = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(s):
            for x, o in zip(xs, outs):
                peer.allreduce_bf16(x, o)  # warm-up outside the graph, same call sequence
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for x, o in zip(xs, outs):
                peer.allreduce_bf16(x, o)
        for rep in range(3):
            for i, x in enumerate(xs):
                x.copy_(torch.randn(n, generator=torch.Generator(device=dev).manual_seed(
                    7 * rep + 31 * i + 100 * rank), device=dev))
            graph.replay()
            torch.cuda.synchronize(dev)
            for x, o in zip(xs, outs):
                allx = [torch.empty(n) for _ in range(world)]
                dist.all_gather(allx, x.cpu())
                ref = allx[0].clone()
                for r in range(1, world):
                    ref += allx[r]
                worst = max(worst, int((o.cpu() != ref.to(torch.bfloat16)).sum()))
        del graph
        import neokernel_b200 as nk
        err = nk.device_error()
        peer.close()
        dist.destroy_process_group()
        q.put((rank, "ok", worst, err))
    except Exception:
        q.put((rank, "error", traceback.format_exc(), None))


def _timeout_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        import neokernel_b200 as nk
        from neokernel_b200 import _lib
        from neokernel_b200.peer import PeerGroup
        dev = torch.device("cuda", rank)
        peer = PeerGroup(4096, device=dev)
        x = torch.ones(4096, device=dev)
        out = torch.empty(4096, dtype=torch.bfloat16, device=dev)
        peer.allreduce_bf16(x, out)  # every rank: one good call
        torch.cuda.synchronize(dev)
        good = bool((out.float() == float(world)).all())
        if rank == 0:
            peer.allreduce_bf16(x, out)  # the others never make this call
            torch.cuda.synchronize(dev)  # returns once the bounded wait has given up
            status = nk.device_error()
        else:
            status = None
        dist.barrier()  # nobody leaves while rank 0's kernel runs
        peer.close()
        q.put((rank, "ok", good, status == _lib.NK_ERR_TIMEOUT if rank == 0 else True))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc(), None))


def _run(target, world, timeout=300):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=timeout) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.skipif(N_GPUS < 2, reason="needs two or more GPUs")
def test_peer_allreduce_is_the_rank_order_sum():
    world = min(N_GPUS, 4)
    for rank, status, worst, err in _run(_exact_worker, world):
        assert status == "ok", worst
        assert worst == 0, (rank, worst)
        assert err == 0, (rank, err)


@pytest.mark.skipif(N_GPUS < 2, reason="needs two or more GPUs")
def test_peer_allreduce_reports_a_rank_that_does_not_arrive():
    for rank, status, good, timed_out in _run(_timeout_worker, 2):
        assert status == "ok", good
        assert good, rank
        assert timed_out, rank
