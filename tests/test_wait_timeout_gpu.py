"""The tensor-core kernel's bounded cross-CTA wait runs out, is reported, and the workspace
recovers — made to happen without faulting or hanging anything.

A tile whose K range spans several CTAs is finished by its rank-0 CTA from the others' fp32
partials; the finisher waits for them with a bounded wait (about 2 s). ``nk_test_withhold_partial``
makes the rank-1 CTA of one tile keep its partial for the next launch, so that wait expires:
the launch still returns, the tile's outputs are left unwritten, ``nk_device_error`` reports
NK_ERR_TIMEOUT, and after ``nk_ws_init`` the same workspace gives the exact result again.
Every finishing protocol is covered: tagged slots (M <= 8), the fenced count (M > 8) and the
column-distributed finishing of wide token tiles (M > 32), where every finishing CTA of the tile
waits out.
"""

import ctypes
import time

import pytest
import torch

import neokernel_b200 as nk
from neokernel_b200 import _lib, synthetic
from oracle import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def partition(p, M):
    """(U, KB, G, split) of the partition launch_tc builds for a plain call with M tokens
    (nk_tc.cu): the tile-aligned one when the plan has slices, else the balanced one."""
    KB = -(-p.K // p.k_step)
    tiles = p.n_tiles * (-(-M // p.tile_m))
    U = tiles * KB
    if p.slices:
        return U, KB, tiles * p.slices, p.slices
    q = (p.n_tiles * p.m_tiles * KB) // p.grid
    return U, KB, max(1, min(p.grid, U // q)), 0


def cta_of(u, U, G, KB, split):
    if split:
        t, kb = divmod(u, KB)
        return t * split + ((kb + 1) * split + KB - 1) // KB - 1
    return ((u + 1) * G + U - 1) // U - 1


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 4096, 12288), (64, 4096, 4096),
                                   (128, 4096, 4096)])
def test_withheld_partial_times_out_and_workspace_recovers(M, N, K):
    L = _lib.load()
    plan = nk.plan_for(M, N, K)
    assert plan.kind == nk.KIND_TC and plan.split_k == 0
    U, KB, G, split = partition(plan.c, M)
    assert G <= 296, "the grid must be one resident wave for the waiting protocol"
    tile = 0
    assert cta_of(KB - 1, U, G, KB, split) > cta_of(0, U, G, KB, split), \
        "tile 0 must be shared by several CTAs"

    W = synthetic.weight(N, K, seed=31, device=DEV)
    x = synthetic.activation(M, K, seed=32, device=DEV)
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream
    ws = torch.empty(plan.ws_bytes, dtype=torch.uint8, device=DEV)
    assert L.nk_ws_init(ws.data_ptr(), ws.numel(), s) == 0

    def call(y):
        st = L.nk_gemm_bf16(x.data_ptr(), K, W.data_ptr(), K, y.data_ptr(), N, M, N, K,
                            plan._ref, ws.data_ptr(), ws.numel(), s)
        assert st == 0, _lib.status_string(st)

    clean = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    call(clean)
    torch.cuda.synchronize()
    assert nk.device_error() == 0
    assert (clean.float() - torch.matmul(x.float(), W.float().t())).abs().max().item() \
        <= oracle.tolerance(K)

    # The wait of tile 0's finisher runs out: the launch returns, the tile is not written.
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    assert L.nk_test_withhold_partial(tile) == 0
    t0 = time.perf_counter()
    call(y)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert nk.device_error() == _lib.NK_ERR_TIMEOUT
    assert 1.0 <= waited <= 30.0, waited
    rows = slice(tile * 128, tile * 128 + 128)
    assert torch.isnan(y[:, rows].float()).all(), "a tile whose partial never came was written"
    rest = torch.ones(N, dtype=torch.bool, device=DEV)
    rest[rows] = False
    assert torch.equal(y[:, rest], clean[:, rest]), "tiles that finished must be exact"

    # The request was consumed by that launch; after nk_ws_init the workspace is whole again.
    assert L.nk_ws_init(ws.data_ptr(), ws.numel(), s) == 0
    for _ in range(2):
        y2 = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        call(y2)
        torch.cuda.synchronize()
        assert torch.equal(y2, clean)
    assert nk.device_error() == 0


def test_withhold_request_is_validated_and_cleared():
    L = _lib.load()
    assert L.nk_test_withhold_partial(-2) == _lib.NK_ERR_ARG
    assert L.nk_test_withhold_partial(3) == 0
    assert L.nk_test_withhold_partial(-1) == 0  # cleared: the next launch withholds nothing
    M, N, K = 1, 4096, 4096
    W = synthetic.weight(N, K, seed=41, device=DEV)
    x = synthetic.activation(M, K, seed=42, device=DEV)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    nk.mm(x, W.t(), out=y)
    torch.cuda.synchronize()
    assert nk.device_error() == 0
    assert (y.float() - torch.matmul(x.float(), W.float().t())).abs().max().item() \
        <= oracle.tolerance(K)
