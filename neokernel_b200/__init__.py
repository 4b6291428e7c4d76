"""neokernel_b200 — B200-native (sm_100a) decode GEMMs for the neoKernel Qwen3 engine.

The package replaces the five decode linears of the reference engine
(``torch.mm(x, W.t(), out=y)`` at engine/kernels/decode.py:54,58,64,66 and
engine/engine.py:114) with hand-written CUDA kernels reached through the C ABI of
``lib/libnkgemm.so`` (include/nk_gemm.h). The library is loaded on first use (so that
``python -m neokernel_b200.build`` can build it in a fresh checkout); an operator called
without it raises ImportError. There is no CPU or library fallback.
"""

from .gemm import (  # noqa: E402
    KIND_AUTO, KIND_GEMV, KIND_TC, KIND_GENERIC, Plan, device_error, linear_out, m_bucket, mm,
    mm_argmax, mm_f32, plan_for, workspace,
)

__all__ = ["mm", "mm_argmax", "mm_f32", "linear_out", "Plan", "plan_for", "workspace",
           "device_error", "m_bucket", "KIND_AUTO", "KIND_GEMV", "KIND_TC", "KIND_GENERIC"]
__version__ = "0.1.0"
