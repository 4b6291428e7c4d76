"""Tensor-parallel decode host logic on CPU ranks (gloo, world size 2).

The decode linears are emulated on the CPU with their exact semantics (bf16 operands, fp32
accumulation, one rounding; fp32 partials unrounded for the K-split linears), so these tests
check the sharding, the fp32 all-reduce, the vocab-split argmax and the failure behaviour —
not the CUDA kernels, which tests/test_tp_gpu.py runs on GPUs.
"""

import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch

TINY = dict(hidden=64, intermediate=128, heads=4, kv_heads=2, head_dim=16, layers=2, vocab=96)


def lin(a, b, out):          # bf16 in, fp32 accumulate, one rounding
    out.copy_(torch.mm(a.float(), b.float()))


def lin32(a, b, out):        # unrounded fp32 partial
    torch.mm(a.float(), b.float(), out=out)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=20):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _parity_worker(rank, world, port, q):
    try:
        torch.manual_seed(0)
        dist = _init(rank, world, port)
        from neokernel_b200 import qwen3, tp
        d = qwen3.Qwen3Dims(**TINY)
        full = qwen3.Qwen3Weights(d, seed=4, device="cpu")
        shard = tp.TPWeights(d, seed=4, rank=rank, world=world, device="cpu")
        # same model: the shard is a slice of the full matrices
        assert torch.equal(shard.layers[0].o_weight,
                           full.layers[0].o_weight[:, rank * 32:(rank + 1) * 32])
        B, cap = 3, 8
        ref = qwen3.DecodeState(full, B, cap, device="cpu")
        st = qwen3.DecodeState(shard, B, cap, device="cpu")
        row, head = tp.make_hooks(shard, linear_f32=lin32, linear=lin)(st)
        gen = torch.Generator().manual_seed(9)
        worst, agree, total = 0.0, 0, 0
        for pos in range(5):
            toks = torch.randint(0, d.vocab, (B,), generator=gen)
            for s in (ref, st):
                s.tokens.copy_(toks)
                s.position.fill_(pos)
            qwen3.decode_step(ref, full, lin)
            qwen3.decode_step(st, shard, lin, row, head)
            vl = d.vocab // world
            local_ref = ref.logits[:, rank * vl:(rank + 1) * vl].float()
            worst = max(worst, (st.logits.float() - local_ref).abs().max().item())
            # next tokens agree wherever the reference's top-2 gap is not a near-tie
            top2 = ref.logits.float().topk(2, dim=-1).values
            decisive = (top2[:, 0] - top2[:, 1]) > 0.05
            agree += int((st.next_tokens == ref.next_tokens)[decisive].sum())
            total += int(decisive.sum())
        dist.destroy_process_group()
        q.put((rank, "ok", worst, agree, total))
    except Exception:
        q.put((rank, "error", traceback.format_exc(), 0, 0))


def _run(target, world=2, extra=(), timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world):
        results.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_tp2_matches_single_process_model():
    res = _run(_parity_worker)
    for rank, status, worst, agree, total in res:
        assert status == "ok", worst
        assert worst <= 0.05, (rank, worst)
        assert total > 0 and agree == total, (rank, agree, total)


def _failure_worker(rank, world, port, q):
    try:
        dist = _init(rank, world, port, timeout_s=5)
        from neokernel_b200 import qwen3, tp
        d = qwen3.Qwen3Dims(**TINY)
        shard = tp.TPWeights(d, seed=4, rank=rank, world=world, device="cpu")
        st = qwen3.DecodeState(shard, 2, 4, device="cpu")
        row, head = tp.make_hooks(shard, linear_f32=lin32, linear=lin)(st)
        if rank == 1:
            q.put((rank, "left", None))
            q.close()
            q.join_thread()  # flush the message before leaving without cleanup
            os._exit(0)  # this rank leaves between steps, before its next collective
        try:
            qwen3.decode_step(st, shard, lin, row, head)
            q.put((rank, "no error", None))
        except Exception as e:  # the peer's departure surfaces as an error, not a hang
            q.put((rank, "raised", type(e).__name__))
    except Exception:
        q.put((rank, "setup error", traceback.format_exc()))


def test_tp_collective_fails_loudly_when_a_rank_leaves():
    res = _run(_failure_worker, timeout=90)
    by_rank = {r[0]: r for r in res}
    assert by_rank[1][1] == "left"
    assert by_rank[0][1] == "raised", by_rank[0]


def test_local_dims_validation():
    from neokernel_b200 import qwen3, tp
    d = qwen3.QWEN3_32B
    ld = tp.local_dims(d, 8)
    assert (ld.heads, ld.kv_heads, ld.intermediate, ld.vocab) == (8, 1, 3200, 18992)
    with pytest.raises(ValueError):
        tp.local_dims(d, 16)  # 8 KV heads cannot be split 16 ways
