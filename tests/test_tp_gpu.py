"""Tensor-parallel decode on 2+ GPUs, CUDA-graph captured, against the single-GPU model of the
same seed on every rank, with the K-split partials summed inside the linear's own launch
(nk_gemm_bf16_allreduce), by the peer-memory all-reduce (nk_allreduce_bf16) and by NCCL.
Skipped with fewer than two GPUs."""

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


def _worker(rank, world, port, q, collective):
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        torch.backends.cuda.matmul.allow_tf32 = False
        import neokernel_b200 as nk
        from neokernel_b200 import qwen3, tp
        d = qwen3.QWEN3_8B
        layers = 4
        full = qwen3.Qwen3Weights(d, seed=21, device=dev, layers=layers)
        shard = tp.TPWeights(d, seed=21, rank=rank, world=world, device=dev, layers=layers)
        B, cap = 4, 32
        ref = qwen3.GraphDecoder(full, B, cap, nk.mm, device=dev)
        # logits stored (lm_head, then torch.max of the shard) ...
        tpg = qwen3.GraphDecoder(shard, B, cap, nk.mm, device=dev,
                                 make_hooks=tp.make_hooks(shard, collective=collective,
                                                          fused_head=False))
        # ... and the product hook: each shard's argmax from the lm_head launch itself
        tpf = qwen3.GraphDecoder(shard, B, cap, nk.mm, device=dev, fused=True,
                                 make_hooks=tp.make_hooks(shard, collective=collective))
        gen = torch.Generator(device=dev).manual_seed(77)
        worst, agree, total = 0.0, 0, 0
        vl = d.vocab // world
        for pos in range(8):
            toks = torch.randint(0, d.vocab, (B,), generator=gen, device=dev)
            for g in (ref, tpg, tpf):
                g.st.tokens.copy_(toks)
                g.st.position.fill_(pos)
                g.graph.replay()
            torch.cuda.synchronize(dev)
            local_ref = ref.st.logits[:, rank * vl:(rank + 1) * vl].float()
            worst = max(worst, (tpg.st.logits.float() - local_ref).abs().max().item())
            top2 = ref.st.logits.float().topk(2, dim=-1).values
            decisive = (top2[:, 0] - top2[:, 1]) > 0.1
            agree += int((tpg.st.next_tokens == ref.st.next_tokens)[decisive].sum())
            agree += int((tpf.st.next_tokens == ref.st.next_tokens)[decisive].sum())
            total += 2 * int(decisive.sum())
        del ref.graph, tpg.graph, tpf.graph  # graphs holding NCCL calls go before the group
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", worst, agree, total))
    except Exception:
        q.put((rank, "error", traceback.format_exc(), 0, 0))


@pytest.mark.skipif(N_GPUS < 2, reason="needs two or more GPUs")
@pytest.mark.parametrize("collective", ("fused", "peer", "nccl"))
def test_tp_decode_matches_single_gpu_model(collective):
    world = 4 if N_GPUS >= 4 else 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, collective))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=600) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, status, worst, agree, total in res:
        assert status == "ok", worst
        assert worst <= 0.25, (rank, worst)    # fp32 partial sums re-associated across ranks
        assert total > 0 and agree == total, (rank, agree, total)
