"""neokernel_b200 — B200-native (sm_100a) decode GEMMs for the neoKernel Qwen3 engine.

The package replaces the five decode linears of the reference engine
(``torch.mm(x, W.t(), out=y)`` at engine/kernels/decode.py:54,58,64,66 and
engine/engine.py:114) with hand-written CUDA kernels reached through the C ABI of
``lib/libnkgemm.so`` (include/nk_gemm.h). Importing the package loads that library; there is
no CPU or library fallback.
"""

from . import _lib

_lib.load()

from .gemm import (  # noqa: E402
    KIND_AUTO, KIND_GEMV, KIND_TC, KIND_GENERIC, Plan, device_error, linear_out, m_bucket, mm,
    plan_for, workspace,
)

__all__ = ["mm", "linear_out", "Plan", "plan_for", "workspace", "device_error", "m_bucket",
           "KIND_AUTO", "KIND_GEMV", "KIND_TC", "KIND_GENERIC"]
__version__ = "0.1.0"
