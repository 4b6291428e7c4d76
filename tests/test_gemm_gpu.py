"""GPU parity of the decode linears against the oracle, the reference's golden vectors,
cuBLAS (the reference's own GPU path, torch.mm) and an fp32 matmul.

Tolerance (north star): max |y - x·Wᵀ| <= 2e-2 * sqrt(K / 1024) for bf16 output with fp32
accumulation, where x·Wᵀ is computed exactly (float64 oracle) or in fp32 on the GPU with TF32
disabled. Against the sequential-fp32 oracle the kernels also agree element-wise to one bf16
ulp plus the fp32 re-association error (``pin_bound``), on almost every element bit-exactly.
"""

import os

import numpy as np
import pytest
import torch

import neokernel_b200 as nk
from neokernel_b200 import synthetic
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"

Q06 = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)]   # (N, K)
Q8B = [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288), (151936, 4096)]
REF4B = [(6144, 2560), (2560, 4096), (19456, 2560), (2560, 9728), (151936, 2560)]


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def pin_bound(a, b, K):
    fa, fb = oracle.bf16_to_f32(a), oracle.bf16_to_f32(b)
    mag = np.maximum(np.abs(fa), np.abs(fb)).astype(np.float32)
    return np.abs(fa - fb) <= np.spacing(mag) * 65536.0 + 2.0 ** -22 * np.sqrt(K)


def run(x, W, plan=None):
    y = torch.empty((x.shape[0], W.shape[0]), dtype=torch.bfloat16, device=x.device)
    nk.mm(x, W.t(), out=y, plan=plan)
    return y


def fp32_ref(x, W):
    return torch.matmul(x.float(), W.float().t())


def assert_vs_oracle(y, x, W):
    K = W.shape[1]
    xb, wb, yb = bits(x), bits(W), bits(y)
    ref = oracle.gemm_f64(xb, wb)
    err = np.abs(oracle.bf16_to_f32(yb) - ref).max()
    assert err <= oracle.tolerance(K), (err, oracle.tolerance(K))
    ob = oracle.gemm_bf16(xb, wb)
    ok = pin_bound(yb, ob, K)
    assert ok.all(), f"{(~ok).sum()} elements outside the pin bound"
    assert np.mean(yb == ob) >= 0.99


# --- reference golden vectors -----------------------------------------------------------

@pytest.mark.parametrize("site", ("qkv", "o", "gate_up", "down", "lm_head"))
@pytest.mark.parametrize("M", (1, 3, 16))
def test_golden_tiny_layer(site, M):
    g = np.load(os.path.join(GOLDEN, "tiny_layer.npz"))
    w, x, y = g[f"{site}/w"], g[f"{site}/m{M}/x"], g[f"{site}/m{M}/y"]
    Wt = torch.from_numpy(w.view(np.int16)).view(torch.bfloat16).to(DEV)
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(DEV)
    out = bits(run(xt, Wt))
    K = w.shape[1]
    assert pin_bound(out, y, K).all()
    assert np.mean(out == y) >= 0.99
    ref = oracle.gemm_f64(x, w)
    assert np.abs(oracle.bf16_to_f32(out) - ref).max() <= oracle.tolerance(K)


def test_golden_decode_shapes():
    g = np.load(os.path.join(GOLDEN, "decode_shapes.npz"))
    for name in sorted({k.split("/")[0] for k in g.files}):
        M, K, N, ws, xs = (int(v) for v in g[f"{name}/meta"])
        W = synthetic.weight(N, K, ws).to(DEV)
        x = synthetic.activation(M, K, xs).to(DEV)
        for split in (0, 1, 4):
            out = bits(run(x, W, nk.plan_for(M, N, K, split_k=split)))
            y = g[f"{name}/y"]
            assert pin_bound(out, y, K).all(), (name, split)
            assert np.mean(out == y) >= 0.99, (name, split)


# --- oracle parity across shapes, including ragged and edge cases -----------------------

@pytest.mark.parametrize("M", (1, 2, 3, 4, 5, 8, 13, 16, 17, 33))
@pytest.mark.parametrize("N,K", [(1, 256), (7, 24), (100, 1000), (1000, 8), (513, 2056),
                                 (4096, 1024), (1024, 3072)])
def test_vs_oracle(M, N, K):
    W = synthetic.weight(N, K, seed=N * 7 + K).to(DEV)
    x = synthetic.activation(M, K, seed=M * 13 + K).to(DEV)
    assert_vs_oracle(run(x, W), x, W)


@pytest.mark.parametrize("N,K", [(300, 1001), (64, 3), (5, 1), (129, 77)])
@pytest.mark.parametrize("M", (1, 4, 9))
def test_unaligned_K_generic(M, N, K):
    W = synthetic.weight(N, K, seed=N + K).to(DEV)
    x = synthetic.activation(M, K, seed=M + K).to(DEV)
    assert nk.plan_for(M, N, K, nk.KIND_GENERIC).kind == nk.KIND_GENERIC
    assert_vs_oracle(run(x, W), x, W)


def test_misaligned_pointers_and_strides():
    M, N, K = 5, 300, 512
    base_x = synthetic.activation(M, K + 9, seed=1).to(DEV)
    base_w = synthetic.weight(N, K + 9, seed=2).to(DEV)
    x = base_x[:, 1:K + 1]            # 2-byte offset: not 16-byte aligned -> generic kernel
    W = base_w[:, 3:K + 3]
    y = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    nk.mm(x, W.t(), out=y)
    assert_vs_oracle(y, x.contiguous(), W.contiguous())
    # aligned but strided rows (ldx = K + 64, ldy = N + 8) stay on the vectorised kernel
    bx = synthetic.activation(M, K + 64, seed=3).to(DEV)
    xs = bx[:, :K]
    by = torch.zeros((M, N + 8), dtype=torch.bfloat16, device=DEV)
    ys = by[:, :N]
    W2 = synthetic.weight(N, K, seed=4).to(DEV)
    nk.mm(xs, W2.t(), out=ys)
    assert_vs_oracle(ys, xs.contiguous(), W2)
    assert not by[:, N:].any(), "wrote outside the output view"


def test_guard_bands_untouched():
    """Canary bands around the output and inside a strided activation are never written."""
    M, N, K = 16, 1000, 2048
    W = synthetic.weight(N, K, seed=5).to(DEV)
    x = synthetic.activation(M, K, seed=6).to(DEV)
    big = torch.full((M * N + 2048,), 7.0, dtype=torch.bfloat16, device=DEV)
    y = big[1024:1024 + M * N].view(M, N)
    for split in (1, 3, 8):
        nk.mm(x, W.t(), out=y, plan=nk.plan_for(M, N, K, split_k=split))
        assert (big[:1024] == 7.0).all() and (big[1024 + M * N:] == 7.0).all()
    assert_vs_oracle(y, x, W)


# --- full decode shapes vs cuBLAS (the reference's GPU path) and fp32 -------------------

_W_CACHE = {}


def weight_dev(N, K, seed):
    key = (N, K, seed)
    if key not in _W_CACHE:
        _W_CACHE.clear()
        _W_CACHE[key] = synthetic.weight(N, K, seed, device=DEV)
    return _W_CACHE[key]


@pytest.mark.parametrize("N,K", Q06 + Q8B + REF4B)
@pytest.mark.parametrize("M", (1, 2, 4, 8, 16))
def test_decode_shapes_vs_cublas_and_fp32(M, N, K):
    W = weight_dev(N, K, seed=N + K)
    x = synthetic.activation(M, K, seed=M, device=DEV)
    y = run(x, W)
    tol = oracle.tolerance(K)
    ref = fp32_ref(x, W)
    err = (y.float() - ref).abs().max().item()
    assert err <= tol, (err, tol)
    cublas = torch.mm(x, W.t())
    assert (y.float() - cublas.float()).abs().max().item() <= tol
    # near-identical to cuBLAS: the only differences are fp32 re-association at rounding edges
    assert (y == cublas).float().mean().item() >= 0.98


@pytest.mark.parametrize("N,K", Q8B[:4])
@pytest.mark.parametrize("M", (1, 4, 16))
def test_split_k_sweep(M, N, K):
    W = weight_dev(N, K, seed=N + K)
    x = synthetic.activation(M, K, seed=M + 100, device=DEV)
    ref = fp32_ref(x, W)
    tol = oracle.tolerance(K)
    seen = set()
    for split in range(1, 17):
        plan = nk.plan_for(M, N, K, split_k=split)
        seen.add(plan.split_k)
        y = run(x, W, plan)
        assert (y.float() - ref).abs().max().item() <= tol, split
    assert 1 in seen and len(seen) >= 4


@pytest.mark.parametrize("kind", (nk.KIND_GEMV, nk.KIND_TC))
@pytest.mark.parametrize("M", (1, 2, 3, 4, 8, 16))
@pytest.mark.parametrize("N,K", [(100, 1000), (513, 2056), (4096, 1024), (1024, 3072), (130, 64)])
def test_families_vs_oracle(kind, M, N, K):
    W = synthetic.weight(N, K, seed=N * 3 + K).to(DEV)
    x = synthetic.activation(M, K, seed=M * 5 + K).to(DEV)
    for split in (0, 1, 3):
        y = run(x, W, nk.plan_for(M, N, K, kind=kind, split_k=split))
        assert_vs_oracle(y, x, W)


@pytest.mark.parametrize("M", (17, 32, 33, 64, 100, 128, 200, 256, 300))
@pytest.mark.parametrize("N,K", [(4096, 1024), (777, 520), (256, 4096)])
def test_tc_token_tiles_vs_oracle(M, N, K):
    W = synthetic.weight(N, K, seed=N + 2 * K).to(DEV)
    x = synthetic.activation(M, K, seed=M + 3 * K).to(DEV)
    for split in (0, 1, 2):
        plan = nk.plan_for(M, N, K, kind=nk.KIND_TC, split_k=split)
        assert plan.kind == nk.KIND_TC
        assert_vs_oracle(run(x, W, plan), x, W)


@pytest.mark.parametrize("N,K", Q8B[:4] + [(151936, 4096)])
@pytest.mark.parametrize("M", (1, 4, 8, 16))
def test_tc_decode_shapes_vs_fp32(M, N, K):
    W = weight_dev(N, K, seed=N + K)
    x = synthetic.activation(M, K, seed=M + 1, device=DEV)
    y = run(x, W, nk.plan_for(M, N, K, kind=nk.KIND_TC))
    assert (y.float() - fp32_ref(x, W)).abs().max().item() <= oracle.tolerance(K)
    y2 = run(x, W, nk.plan_for(M, N, K, kind=nk.KIND_GEMV))
    assert (y.float() - y2.float()).abs().max().item() <= oracle.tolerance(K)


@pytest.mark.parametrize("M", (64, 128, 256))
@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)])
def test_verify_shapes(M, N, K):
    W = weight_dev(N, K, seed=N + K)
    x = synthetic.activation(M, K, seed=M + 7, device=DEV)
    y = run(x, W)
    assert (y.float() - fp32_ref(x, W)).abs().max().item() <= oracle.tolerance(K)


def test_deterministic_across_runs():
    N, K, M = 4096, 12288, 4
    W = weight_dev(N, K, seed=N + K)
    x = synthetic.activation(M, K, seed=9, device=DEV)
    for kind in (nk.KIND_GEMV, nk.KIND_TC):
        for split in (1, 5, 10):
            plan = nk.plan_for(M, N, K, kind=kind, split_k=split)
            a = run(x, W, plan)
            b = run(x, W, plan)
            assert torch.equal(a, b)


@pytest.mark.parametrize("N,K", [(6144, 4096), (4096, 4096), (4096, 12288), (1024, 2048)])
@pytest.mark.parametrize("M", (1, 4, 8, 16))
def test_tile_aligned_and_balanced_schedules(M, N, K):
    """A plan with slices launches the tile-aligned schedule; the same plan with slices cleared
    launches the balanced one. Interleaved on one workspace, each is within the tolerance of
    the fp32 product, agrees with the sequential-fp32 oracle up to re-association, and gives
    the same bits every time."""
    W = weight_dev(N, K, seed=N + 5 * K)
    x = synthetic.activation(M, K, seed=M + 11, device=DEV)
    aligned = nk.plan_for(M, N, K)
    assert aligned.as_dict()["slices"] >= 4
    balanced = nk.Plan(nk.m_bucket(M), N, K)
    balanced.c.slices = 0
    ref = fp32_ref(x, W)
    first = {}
    for _ in range(2):
        for name, plan in (("aligned", aligned), ("balanced", balanced)):
            y = run(x, W, plan)
            assert (y.float() - ref).abs().max().item() <= oracle.tolerance(K), name
            if name in first:
                assert torch.equal(y, first[name]), name
            else:
                first[name] = y
                assert_vs_oracle(y, x, W)
    assert nk.device_error() == 0


def test_split_protocols_share_one_workspace():
    """Shared tiles are finished three ways: tagged partial slots (M <= 8), plain partials
    with a fence and a count (larger M), and, when a forced split makes the grid larger than
    can be resident, every rank publishing and the last arrival summing. Interleaved on one
    stream's workspace, none may leave state that changes another's result."""
    N, K = 4096, 4096
    W = weight_dev(N, K, seed=77)
    cases = [(1, 0), (16, 0), (4, 10), (8, 0), (3, 0), (12, 0)]
    xs = {M: synthetic.activation(M, K, seed=300 + M, device=DEV) for M, _ in cases}
    plans = {(M, s): nk.plan_for(M, N, K, split_k=s) for M, s in cases}
    assert plans[(4, 10)].grid > 148 * 2  # forced split: not co-resident, no-wait finishing
    first = {}
    for _ in range(3):
        for M, s in cases:
            y = run(xs[M], W, plans[(M, s)])
            assert (y.float() - fp32_ref(xs[M], W)).abs().max().item() <= oracle.tolerance(K)
            if (M, s) in first:
                assert torch.equal(y, first[(M, s)]), (M, s)
            else:
                first[(M, s)] = y
    assert nk.device_error() == 0


def test_cuda_graph_capture_and_replay():
    """Decode-style capture: side-stream warm-up x3, then capture (engine/engine.py:119-129)."""
    shapes = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072)] * 3 + [(151936, 1024)]
    Ws = [synthetic.weight(N, K, seed=i, device=DEV) for i, (N, K) in enumerate(shapes)]
    for M in (1, 4, 16):
        xs = [synthetic.activation(M, K, seed=50 + i, device=DEV) for i, (N, K) in enumerate(shapes)]
        ys = [torch.empty((M, N), dtype=torch.bfloat16, device=DEV) for (N, K) in shapes]

        def step():
            for x, W, y in zip(xs, Ws, ys):
                nk.mm(x, W.t(), out=y)

        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
        torch.cuda.current_stream().wait_stream(stream)
        eager = [y.clone() for y in ys]
        for y in ys:
            y.zero_()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        for a, b in zip(ys, eager):
            assert torch.equal(a, b)
        # new inputs in the same buffers flow through the captured graph
        for x in xs:
            x.copy_(torch.flip(x, dims=[1]))
        graph.replay()
        torch.cuda.synchronize()
        for x, W, y in zip(xs, Ws, ys):
            assert (y.float() - fp32_ref(x, W)).abs().max().item() <= oracle.tolerance(W.shape[1])
        del graph


def test_graph_survives_workspace_growth_on_its_stream():
    """A graph captured on a stream keeps working when a later eager call on that stream needs
    a larger split-K workspace: the old workspace is retired, never freed, so memory the graph
    still writes to is not handed to another tensor."""
    dev = torch.device(DEV, torch.cuda.current_device())
    stream = torch.cuda.Stream()
    N, K, M = 4096, 4096, 1
    W = synthetic.weight(N, K, seed=61, device=DEV)
    x = synthetic.activation(M, K, seed=62, device=DEV)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    plan = nk.plan_for(M, N, K)
    assert plan.ws_bytes > 0
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            nk.mm(x, W.t(), out=y, plan=plan)
    stream.synchronize()
    eager = y.clone()
    before = nk.workspace(1, dev, stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        nk.mm(x, W.t(), out=y, plan=plan)
    # Larger plans run eagerly on the same stream: the lm_head at 16 tokens and the greedy
    # head grow the stream's workspace.
    Nh = 151936
    Wh = synthetic.weight(Nh, K, seed=63, device=DEV)
    xh = synthetic.activation(16, K, seed=64, device=DEV)
    yh = torch.empty((16, Nh), dtype=torch.bfloat16, device=DEV)
    idx = torch.empty((16, 1), dtype=torch.int64, device=DEV)
    stream.wait_stream(torch.cuda.current_stream())  # the inputs were made on this stream
    with torch.cuda.stream(stream):
        nk.mm(xh, Wh.t(), out=yh)
        nk.mm_argmax(xh, Wh.t(), idx=idx)
        after = nk.workspace(1, dev, stream)
        assert after.data_ptr() != before.data_ptr() and after.numel() > before.numel()
        # Whatever memory is free now is taken and filled with a pattern the kernels would
        # misread as work in progress.
        junk = [torch.full((before.numel(),), 0xFF, dtype=torch.uint8, device=DEV)
                for _ in range(8)]
    stream.synchronize()
    assert torch.equal(idx[:, 0], yh.float().argmax(dim=-1))
    for _ in range(3):
        y.zero_()
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, eager)
    assert nk.device_error() == 0
    del graph, junk


def test_shim_errors_on_gpu():
    W = synthetic.weight(64, 128, 1, device=DEV)
    x = synthetic.activation(2, 128, 2, device=DEV)
    y = torch.empty((2, 64), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        nk.mm(x, W, out=torch.empty((2, 128), dtype=torch.bfloat16, device=DEV))  # b not W.t()
    with pytest.raises(ValueError):
        nk.mm(x, W.t(), out=y[:, :10])
    with pytest.raises(ValueError):
        nk.mm(x, W.t(), out=y, plan=nk.plan_for(1, 64, 128))  # M=2 > plan's M_max=1
    empty = torch.empty((0, 128), dtype=torch.bfloat16, device=DEV)
    nk.mm(empty, W.t(), out=torch.empty((0, 64), dtype=torch.bfloat16, device=DEV))
    z = torch.ones((2, 64), dtype=torch.bfloat16, device=DEV)
    nk.mm(x[:, :0], W[:, :0].t(), out=z)
    assert not z.any()


def test_no_device_error_left():
    torch.cuda.synchronize()
    assert nk.device_error() == 0


@pytest.mark.parametrize("N,K", [(5120, 8192), (5120, 1024), (5120, 25600), (5120, 3200)])
@pytest.mark.parametrize("M", (1, 4, 8, 32))
def test_f32_output_is_the_unrounded_sum(M, N, K):
    """mm_f32 (nk_gemm_bf16_f32out), the K-split partial of the tensor-parallel o_proj/down:
    the same fp32 sums mm rounds, so rounding it to bf16 gives mm's output bit for bit."""
    W = weight_dev(N, K, seed=N + 3 * K)
    x = synthetic.activation(M, K, seed=M + 7, device=DEV)
    y = run(x, W)
    p = torch.empty((M, N), dtype=torch.float32, device=DEV)
    nk.mm_f32(x, W.t(), out=p)
    assert torch.equal(p.to(torch.bfloat16), y)
    # fp32 against fp32 (TF32 off): only the order of the additions differs
    assert (p - fp32_ref(x, W)).abs().max().item() <= 1e-3
