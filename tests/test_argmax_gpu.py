"""Greedy head (nk_gemm_bf16_argmax, neokernel_b200.mm_argmax): the lm_head linear with the
lowest-index argmax folded into its epilogue, replacing ``torch.mm`` + ``torch.argmax`` at
engine/engine.py:114-116.

The argmax is over the same bf16 outputs nk_gemm_bf16 stores, so it must equal
``torch.argmax`` of our own logits exactly (indices and maxima), on every path a tile's
output can take: whole tiles, split tiles finished by rank 0 (tagged slots, counts, bulk
copies for wide token tiles) and ragged last tiles. Ties go to the lowest index, planted by
duplicating the winning weight row in another tile. The fixed workspace region that holds
the running maxima must be left zeroed, so back-to-back calls, interleaved with plain GEMMs
of other plans on the same workspace, keep giving exact answers.
"""

import pytest
import torch

import neokernel_b200 as nk

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rand(*shape, std=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=DEV) * std).to(torch.bfloat16)


SHAPES = [(1, 151936, 4096), (4, 151936, 4096), (16, 151936, 4096), (3, 1000, 256),
          (7, 129, 4096), (64, 50000, 1024), (128, 9000, 512), (200, 4096, 1024),
          (4, 75968, 4096), (8, 37984, 5120), (1, 18992, 5120)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_argmax_equals_argmax_of_own_logits(M, N, K):
    x = rand(M, K, seed=M)
    w = rand(N, K, std=0.02, seed=N + K)
    logits = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    nk.mm(x, w.t(), out=logits)
    idx = torch.full((M,), -7, dtype=torch.int64, device=DEV)
    nk.mm_argmax(x, w.t(), idx=idx)
    idx2 = torch.empty_like(idx)
    logits2 = torch.empty_like(logits)
    best = torch.empty(M, dtype=torch.bfloat16, device=DEV)
    nk.mm_argmax(x, w.t(), idx=idx2, logits=logits2, best=best)
    torch.cuda.synchronize()
    assert nk.device_error() == 0
    ref = torch.argmax(logits, dim=-1)
    assert torch.equal(idx, ref)
    assert torch.equal(idx2, ref)
    assert torch.equal(logits2, logits)
    assert torch.equal(best, logits.max(dim=-1).values)


@pytest.mark.parametrize("M,N,K", [(1, 151936, 4096), (16, 151936, 4096), (64, 20000, 1024)])
def test_ties_go_to_the_lowest_index(M, N, K):
    """Token m's winning row i_m is duplicated at j_m > i_m in another tile: both give the same
    bf16 logit, the largest of the row by far, and the lower index must win."""
    x = rand(M, K, seed=3)
    w = rand(N, K, std=0.02, seed=4)
    lo = [(5 + 997 * m) % (N // 2) for m in range(M)]
    hi = [N - 1 - 131 * m for m in range(M)]
    for m in range(M):
        row = torch.sign(x[m].float()).to(torch.bfloat16) * 0.05
        w[lo[m]] = row
        w[hi[m]] = row
    logits = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    nk.mm(x, w.t(), out=logits)
    idx = torch.empty(M, dtype=torch.int64, device=DEV)
    nk.mm_argmax(x, w.t(), idx=idx)
    torch.cuda.synchronize()
    want = torch.tensor(lo, device=DEV)
    rows = torch.arange(M, device=DEV)
    assert torch.equal(logits[rows, want], logits[rows, torch.tensor(hi, device=DEV)])
    assert torch.equal(torch.argmax(logits, dim=-1), want)
    assert torch.equal(idx, want)


def test_back_to_back_calls_share_the_workspace():
    """Calls of different plans in a row on one stream (so one workspace): the argmax region
    must come back zeroed after every call, whatever ran in between."""
    K = 4096
    w_head = rand(151936, K, std=0.02, seed=8)
    w_mlp = rand(24576, K, std=0.02, seed=9)
    w_small = rand(1000, 256, std=0.02, seed=10)
    for call in range(4):
        for M in (1, 16, 5):
            x = rand(M, K, seed=100 * call + M)
            y = torch.empty(M, 24576, dtype=torch.bfloat16, device=DEV)
            nk.mm(x, w_mlp.t(), out=y)  # split tiles: tickets and partial slots in use
            idx = torch.empty(M, dtype=torch.int64, device=DEV)
            nk.mm_argmax(x, w_head.t(), idx=idx)
            xs = rand(M, 256, seed=7 + call)
            idx_s = torch.empty(M, dtype=torch.int64, device=DEV)
            nk.mm_argmax(xs, w_small.t(), idx=idx_s)
            logits = torch.empty(M, 151936, dtype=torch.bfloat16, device=DEV)
            nk.mm(x, w_head.t(), out=logits)
            ls = torch.empty(M, 1000, dtype=torch.bfloat16, device=DEV)
            nk.mm(xs, w_small.t(), out=ls)
            torch.cuda.synchronize()
            assert torch.equal(idx, torch.argmax(logits, dim=-1)), (call, M)
            assert torch.equal(idx_s, torch.argmax(ls, dim=-1)), (call, M)
    assert nk.device_error() == 0


def test_fused_head_decode_matches_unfused():
    """Two-layer Qwen3-8B-shaped decode in CUDA graphs: the fused lm_head + argmax gives the
    same greedy tokens as lm_head then torch.argmax on the same linears."""
    from neokernel_b200 import qwen3
    d = qwen3.QWEN3_8B
    w = qwen3.Qwen3Weights(d, seed=5, layers=2)
    B, cap = 4, 40
    prompt = torch.randint(0, d.vocab, (B, 6), generator=torch.Generator(device=DEV)
                           .manual_seed(1), device=DEV)
    a = qwen3.GraphDecoder(w, B, cap, nk.mm, fused=True)
    b = qwen3.GraphDecoder(w, B, cap, nk.mm, fused=True, fused_head=True)
    ta = a.greedy(prompt, 24)
    tb = b.greedy(prompt, 24)
    torch.cuda.synchronize()
    assert torch.equal(ta, tb)
