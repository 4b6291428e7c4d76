"""nk_gemm_bf16_allreduce (include/nk_comm.h) on 2+ GPUs, one process per GPU: the K-split
linear of a tensor-parallel group fused with its all-reduce.

* Exactness: every rank holds one K slice of x and W; every rank's output must equal, bit for
  bit, bf16 of the rank-order fp32 sum of the slices' partials — each partial computed here
  with the unfused nk_gemm_bf16_f32out on every slice (the data is seeded, so every rank can
  make all slices). Qwen3-32B o_proj / down shard shapes at TP = 2 / 4, M = 1..64, repeated
  calls (both sets of flags and slots), interleaved shapes, and replays of a CUDA graph.
* Failure detection: when one rank does not make a call, the others' bounded wait gives up
  after ~2 s, leaves y unwritten and reports NK_ERR_TIMEOUT; nobody leaves while a kernel is in
  flight, NVLS is off and only plain peer loads and stores are used.
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


def _data(M, N, K, world, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K * world, generator=g, device=dev).to(torch.bfloat16)
    W = (torch.randn(N, K * world, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return x, W


def _expected(x, W, K, world):
    import neokernel_b200 as nk
    M, N = x.shape[0], W.shape[0]
    acc = None
    for r in range(world):
        xs = x[:, r * K:(r + 1) * K].contiguous()
        ws = W[:, r * K:(r + 1) * K].contiguous()
        p = torch.empty(M, N, dtype=torch.float32, device=x.device)
        nk.mm_f32(xs, ws.t(), out=p)
        acc = p if acc is None else acc + p  # rank order, fp32
    return acc.to(torch.bfloat16)


def _exact_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        import neokernel_b200 as nk
        from neokernel_b200.peer import PeerGroup
        dev = torch.device("cuda", rank)
        H = 5120
        peer = PeerGroup(64 * H, device=dev)
        # (M, N, K per rank): o_proj (8192 / world) and down (25600 / world) shards
        shapes = [(M, H, k // world) for M in (1, 4, 16, 64) for k in (8192, 25600)]
        bad = 0
        for call, (M, N, K) in enumerate(shapes + shapes[::-1]):
            x, W = _data(M, N, K, world, seed=call, dev=dev)
            xs = x[:, rank * K:(rank + 1) * K].contiguous()
            ws = W[:, rank * K:(rank + 1) * K].contiguous()
            out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
            peer.mm_allreduce(xs, ws.t(), out=out)
            want = _expected(x, W, K, world)
            torch.cuda.synchronize(dev)
            bad += int((out != want).sum())
        # a CUDA graph holding two calls, replayed with new inputs in the same buffers
        M, N, K = 4, H, 8192 // world
        bufs = [torch.empty(M, K, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        x, W = _data(M, N, K, world, seed=99, dev=dev)
        ws = W[:, rank * K:(rank + 1) * K].contiguous()
        outs = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for b, o in zip(bufs, outs):
                peer.mm_allreduce(b, ws.t(), out=o)  # warm-up: the same call sequence
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for b, o in zip(bufs, outs):
                peer.mm_allreduce(b, ws.t(), out=o)
        for rep in range(3):
            xr = []
            for i, b in enumerate(bufs):
                xf, _ = _data(M, N, K, world, seed=1000 + 10 * rep + i, dev=dev)
                b.copy_(xf[:, rank * K:(rank + 1) * K])
                xr.append(xf)
            graph.replay()
            torch.cuda.synchronize(dev)
            for xf, o in zip(xr, outs):
                bad += int((o != _expected(xf, W, K, world)).sum())
        del graph
        err = nk.device_error()
        dist.barrier()
        peer.close()
        dist.destroy_process_group()
        q.put((rank, "ok", bad, err))
    except Exception:
        q.put((rank, "error", traceback.format_exc(), None))


def _timeout_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        import neokernel_b200 as nk
        from neokernel_b200 import _lib
        from neokernel_b200.peer import PeerGroup
        dev = torch.device("cuda", rank)
        M, N, K = 1, 5120, 4096
        peer = PeerGroup(M * N, device=dev)
        x, W = _data(M, N, K, world, seed=5, dev=dev)
        xs = x[:, rank * K:(rank + 1) * K].contiguous()
        ws = W[:, rank * K:(rank + 1) * K].contiguous()
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        peer.mm_allreduce(xs, ws.t(), out=out)  # every rank: one good call
        torch.cuda.synchronize(dev)
        good = bool(torch.equal(out, _expected(x, W, K, world)))
        status = None
        if rank == 0:
            out.fill_(float("nan"))
            peer.mm_allreduce(xs, ws.t(), out=out)  # the others never make this call
            torch.cuda.synchronize(dev)  # returns once the bounded waits have given up
            status = nk.device_error()
            untouched = bool(torch.isnan(out.float()).all())
        else:
            untouched = True
        dist.barrier()  # nobody leaves while rank 0's kernel runs
        peer.close()
        q.put((rank, "ok", good and untouched,
               status == _lib.NK_ERR_TIMEOUT if rank == 0 else True))
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
@pytest.mark.parametrize("world", (2, 4))
def test_fused_gemm_allreduce_is_the_rank_order_sum(world):
    if world > N_GPUS:
        pytest.skip(f"needs {world} GPUs")
    for rank, status, bad, err in _run(_exact_worker, world):
        assert status == "ok", bad
        assert bad == 0, (rank, bad)
        assert err == 0, (rank, err)


@pytest.mark.skipif(N_GPUS < 2, reason="needs two or more GPUs")
def test_fused_gemm_allreduce_reports_a_rank_that_does_not_arrive():
    for rank, status, good, timed_out in _run(_timeout_worker, 2):
        assert status == "ok", good
        assert good, rank
        assert timed_out, rank
