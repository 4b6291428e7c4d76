"""The workspace-free entry point nk_gemm_bf16_static, called through the C ABI.

Callers that cannot allocate device memory (an operator inside a framework that owns every
allocation, a process with a fixed device-memory budget, a latency-critical path that avoids
cudaMalloc) use nk_gemm_bf16_static, whose split-K scratch is an array compiled into the
library. This file checks, on two calls in a row per shape, that its output agrees with the
regular entry point nk_gemm_bf16 (given a caller-allocated workspace) within the tolerance the
other parity tests use, 2e-2 * sqrt(K / 1024), and that plans needing more scratch than the
array holds are refused. It is collected last so that a run stopping at the first failure has
already run every other test; it needs no state from them.
"""

import ctypes

import pytest
import torch

from neokernel_b200 import _lib, synthetic
from oracle import oracle

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 8 << 20  # NK_STATIC_SCRATCH_BYTES in include/nk_gemm.h


def bind():
    L = _lib.load()
    f = L.nk_gemm_bf16_static
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32, ctypes.POINTER(_lib.NkPlan), vp]
    f.restype = i32
    return L


def make_plan(L, M, N, K):
    p = _lib.NkPlan()
    assert L.nk_plan_make(ctypes.byref(p), M, N, K, 0, _lib.KIND_TC) == 0
    return p


# (M, N, K): Qwen3-8B decode linears whose tiles are shared by several CTAs, so the scratch
# is really used, plus a verify-sized batch.
CASES = [(1, 6144, 4096), (4, 4096, 4096), (16, 4096, 12288), (8, 24576, 4096), (32, 6144, 4096)]


def test_static_entry_point_matches_regular_entry_point_twice():
    L = bind()
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    used_scratch = False
    for i, (M, N, K) in enumerate(CASES):
        W = synthetic.weight(N, K, seed=900 + i, device=dev)
        x = synthetic.activation(M, K, seed=950 + i, device=dev)
        plan = make_plan(L, M, N, K)
        need = L.nk_ws_bytes(ctypes.byref(plan))
        assert need <= STATIC_SCRATCH_BYTES
        used_scratch |= need > 0

        # regular entry point, caller-allocated workspace
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        assert L.nk_ws_init(ws.data_ptr(), need, stream) == 0
        y_ref = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        st = L.nk_gemm_bf16(x.data_ptr(), K, W.data_ptr(), K, y_ref.data_ptr(), N, M, N, K,
                            ctypes.byref(plan), ws.data_ptr() if need else None, need, stream)
        assert st == 0, _lib.status_string(st)

        tol = oracle.tolerance(K)
        exact = torch.matmul(x.float(), W.float().t())
        for call in range(2):  # two calls in a row share the library's scratch array
            y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
            st = L.nk_gemm_bf16_static(x.data_ptr(), K, W.data_ptr(), K, y.data_ptr(), N,
                                       M, N, K, ctypes.byref(plan), stream)
            assert st == 0, (M, N, K, call, _lib.status_string(st))
            torch.cuda.synchronize(dev)
            assert torch.isfinite(y.float()).all()
            assert (y.float() - y_ref.float()).abs().max().item() <= tol, (M, N, K, call)
            assert (y.float() - exact).abs().max().item() <= tol, (M, N, K, call)
    assert used_scratch
    st = ctypes.c_int(0)
    assert L.nk_device_error(stream, ctypes.byref(st)) == 0 and st.value == 0


def test_static_entry_point_refuses_oversized_or_foreign_plans():
    L = bind()
    stream = torch.cuda.current_stream().cuda_stream
    M, N, K = 16, 151936, 4096  # lm_head at M=16: its partial sums need more than 8 MiB
    plan = make_plan(L, M, N, K)
    assert L.nk_ws_bytes(ctypes.byref(plan)) > STATIC_SCRATCH_BYTES
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    st = L.nk_gemm_bf16_static(dummy.data_ptr(), K, dummy.data_ptr(), K, dummy.data_ptr(), N,
                               M, N, K, ctypes.byref(plan), stream)
    assert st == _lib.NK_ERR_WORKSPACE
    gemv = _lib.NkPlan()
    assert L.nk_plan_make(ctypes.byref(gemv), 1, 4096, 4096, 0, _lib.KIND_GEMV) == 0
    st = L.nk_gemm_bf16_static(dummy.data_ptr(), 4096, dummy.data_ptr(), 4096, dummy.data_ptr(),
                               4096, 1, 4096, 4096, ctypes.byref(gemv), stream)
    assert st == _lib.NK_ERR_PLAN


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_static_entry_point_refuses_a_stream_of_another_device():
    """The scratch array is per device: a stream of device 1 while device 0 is current would
    make the kernels use device 0's copy from device 1, so the call is refused untouched."""
    L = bind()
    M, N, K = 4, 4096, 4096
    with torch.cuda.device(0):
        plan = make_plan(L, M, N, K)
        assert L.nk_ws_bytes(ctypes.byref(plan)) > 0
        W = synthetic.weight(N, K, seed=1, device="cuda:0")
        x = synthetic.activation(M, K, seed=2, device="cuda:0")
        y = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda:0")
        other = torch.cuda.Stream(device=1)
        st = L.nk_gemm_bf16_static(x.data_ptr(), K, W.data_ptr(), K, y.data_ptr(), N, M, N, K,
                                   ctypes.byref(plan), other.cuda_stream)
        assert st == _lib.NK_ERR_DEVICE
        torch.cuda.synchronize()
        assert not y.any()
