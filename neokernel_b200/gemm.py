"""The decode-linear operator: a drop-in for ``torch.mm(x, W.t(), out=y)``.

Reference call sites this replaces (all ``torch.mm(a, b, out=c)`` with ``a`` a contiguous
bf16 ``[M, K]`` activation, ``b = W.t()`` the transposed view of a row-major bf16 ``[N, K]``
weight and ``c`` a preallocated bf16 ``[M, N]`` buffer):

* engine/kernels/decode.py:54  ``torch.mm(self.norm, w.qkv, out=self.qkv)``
* engine/kernels/decode.py:58  ``torch.mm(self.attn_flat, w.o, out=self.branch)``
* engine/kernels/decode.py:64  ``torch.mm(self.norm, w.gate_up, out=self.gate_up)``
* engine/kernels/decode.py:66  ``torch.mm(self.product, w.down, out=self.branch)``
* engine/engine.py:114        ``torch.mm(self.buffers.norm, self.lm_head, out=self.logits)``

``mm(a, b, out=c)`` keeps that signature. It launches one hand-written sm_100a kernel on the
current stream through the C ABI of ``libnkgemm.so``: no allocation once warmed up, no host
synchronisation, capture-safe. Like the reference's wrappers (engine/kernels/decode.py:22,24,
engine/kernels/rmsnorm.py:36) it raises ``ValueError`` for an unsupported configuration
before launching anything; a CUDA failure raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import KIND_AUTO, KIND_GEMV, KIND_TC, KIND_GENERIC, NkPlan  # noqa: F401

_VALUE_ERRORS = (_lib.NK_ERR_SHAPE, _lib.NK_ERR_ALIGN, _lib.NK_ERR_WORKSPACE, _lib.NK_ERR_SPLIT,
                 _lib.NK_ERR_PLAN, _lib.NK_ERR_ARG)


def _raise(status: int, where: str):
    err = _lib.NkError(status, where)
    if status in _VALUE_ERRORS:
        raise ValueError(str(err)) from None
    raise err


def m_bucket(M: int) -> int:
    """Largest M a plan made for decode batch M serves (token tiles 1, 2, 4, 8, 16, then x16)."""
    for b in (1, 2, 4, 8, 16):
        if M <= b:
            return b
    return (M + 15) // 16 * 16


class Plan:
    """Launch plan for y[M <= M_max, N] = x · Wᵀ (kernel family, split-K, tiles)."""

    __slots__ = ("c", "ws_bytes", "_ref")

    def __init__(self, M_max: int, N: int, K: int, split_k: int = 0, kind: int = KIND_AUTO):
        L = _lib.load()
        self.c = NkPlan()
        self._ref = ctypes.byref(self.c)
        status = L.nk_plan_make(self._ref, int(M_max), int(N), int(K), int(split_k), int(kind))
        if status != _lib.NK_OK:
            _raise(status, f"nk_plan_make(M_max={M_max}, N={N}, K={K}, split_k={split_k}, "
                           f"kind={kind})")
        self.ws_bytes = int(L.nk_ws_bytes(self._ref))

    def __getattr__(self, name):
        return getattr(self.c, name)

    def as_dict(self) -> dict:
        d = self.c.as_dict()
        d["ws_bytes"] = self.ws_bytes
        return d

    def __repr__(self):
        return f"Plan({self.as_dict()})"


_PLANS: dict = {}
_WORKSPACES: dict = {}
# Workspaces replaced by a larger one. They are never freed: a CUDA graph captured while one
# of them was current still writes split-K tickets and partials into it on every replay.
_RETIRED: list = []


def plan_for(M: int, N: int, K: int, kind: int = KIND_AUTO, split_k: int = 0) -> Plan:
    """Cached plan for a decode batch of M tokens (shared by every M in the same bucket)."""
    key = (m_bucket(M), N, K, kind, split_k)
    p = _PLANS.get(key)
    if p is None:
        p = Plan(key[0], N, K, split_k=split_k, kind=kind)
        _PLANS[key] = p
    return p


def workspace(nbytes: int, device: torch.device, stream: torch.cuda.Stream) -> torch.Tensor:
    """Zeroed split-K workspace for ``stream`` on ``device``, at least ``nbytes`` long.

    One workspace per (device, stream): launches on one stream are ordered, so every plan
    on that stream can share it (the kernels leave it zeroed). It is allocated while the
    stream is not being captured — run one eager call of each shape before capturing a CUDA
    graph, as the reference engine does with its three warm-up decodes
    (engine/engine.py:119-125).

    A workspace that must grow is replaced, never freed: the old one stays allocated for the
    life of the process, because a graph captured while it was current keeps using it on
    every replay (and torch reuses stream handles, so two decoders may share a key). Sizes
    grow at least twofold, so the retired buffers total less than the current one. The new
    buffer is allocated on ``stream`` itself, so the caching allocator never hands it out
    while work of another stream may still use that memory.
    """
    key = (device.index, stream.cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("neokernel_b200: split-K workspace must be sized before CUDA "
                               "graph capture; run the call once eagerly first")
        size = max(nbytes, 1 << 20, 2 * ws.numel() if ws is not None else 0)
        size = (size + (1 << 20) - 1) >> 20 << 20
        with torch.cuda.device(device), torch.cuda.stream(stream):
            new = torch.empty(size, dtype=torch.uint8, device=device)
        status = _lib.load().nk_ws_init(new.data_ptr(), size, stream.cuda_stream)
        if status != _lib.NK_OK:
            _raise(status, "nk_ws_init")
        if ws is not None:
            _RETIRED.append(ws)
        _WORKSPACES[key] = ws = new
    return ws


def _check_tensor(t: torch.Tensor, name: str, dtype=torch.bfloat16):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {str(dtype).replace('torch.', '')}, got {t.dtype}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor, got device {t.device}")
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")


def mm(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor, plan: Plan | None = None,
       stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """``out = a @ b`` for ``b = W.t()`` (W row-major [N, K]); drop-in for ``torch.mm(a, b, out=out)``.

    a: bf16 CUDA [M, K] with unit column stride; b: bf16 CUDA [K, N] with strides (1, ldw);
    out: bf16 CUDA [M, N] with unit column stride. fp32 accumulation, one bf16 rounding.
    """
    return _mm(a, b, out, plan, stream, f32=False)


def mm_f32(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor, plan: Plan | None = None,
           stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """As ``mm`` but ``out`` is fp32 and unrounded: the partial sum of a K-split
    (tensor-parallel) linear, to be all-reduced across ranks and rounded to bf16 once."""
    return _mm(a, b, out, plan, stream, f32=True)


def _mm(a, b, out, plan, stream, f32):
    _check_tensor(a, "a")
    _check_tensor(b, "b")
    _check_tensor(out, "out", torch.float32 if f32 else torch.bfloat16)
    M, K = a.shape
    K2, N = b.shape
    if K2 != K:
        raise ValueError(f"mm: a is [{M}, {K}] but b is [{K2}, {N}]")
    if tuple(out.shape) != (M, N):
        raise ValueError(f"mm: out must be [{M}, {N}], got {tuple(out.shape)}")
    if not (a.device == b.device == out.device):
        raise ValueError("mm: a, b and out must be on the same device")
    if M == 0 or N == 0:
        return out
    if K == 0:
        return out.zero_()
    if a.stride(1) != 1 and K > 1:
        raise ValueError("mm: a must have unit stride along K (a row-major [M, K] activation)")
    if b.stride(0) != 1 and K > 1:
        raise ValueError("mm: b must be the transposed view W.t() of a row-major [N, K] weight "
                         "(strides (1, ldw)), as in engine/kernels/weights.py:12-13,24-25")
    if out.stride(1) != 1 and N > 1:
        raise ValueError("mm: out must have unit stride along N (a row-major [M, N] buffer)")
    ldx = a.stride(0) if M > 1 else K
    ldw = b.stride(1) if N > 1 else K
    ldy = out.stride(0) if M > 1 else N

    xp, wp, yp = a.data_ptr(), b.data_ptr(), out.data_ptr()
    if plan is None:
        aligned = (K % 8 == 0 and xp % 16 == 0 and wp % 16 == 0 and ldx % 8 == 0
                   and ldw % 8 == 0)
        plan = plan_for(M, N, K, KIND_AUTO if aligned else KIND_GENERIC)
    dev = a.device
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    if plan.ws_bytes:
        ws = workspace(plan.ws_bytes, dev, stream)
        wsp, wsn = ws.data_ptr(), ws.numel()
    else:
        wsp, wsn = None, 0
    L = _lib.load()
    fn = L.nk_gemm_bf16_f32out if f32 else L.nk_gemm_bf16
    if dev.index != torch.cuda.current_device():
        with torch.cuda.device(dev):
            status = fn(xp, ldx, wp, ldw, yp, ldy, M, N, K, plan._ref, wsp, wsn,
                        stream.cuda_stream)
    else:
        status = fn(xp, ldx, wp, ldw, yp, ldy, M, N, K, plan._ref, wsp, wsn, stream.cuda_stream)
    if status != _lib.NK_OK:
        _raise(status, f"nk_gemm_bf16{'_f32out' if f32 else ''}(M={M}, N={N}, K={K})")
    return out


def _rows_vector(t: torch.Tensor, M: int) -> bool:
    """``t`` holds one element per row, M elements adjacent in memory: [M] or [M, 1]."""
    if t.dim() == 2 and t.shape[1] != 1:
        return False
    if t.dim() not in (1, 2) or t.shape[0] != M:
        return False
    return M <= 1 or t.stride(0) == 1


def mm_argmax(a: torch.Tensor, b: torch.Tensor, *, idx: torch.Tensor,
              logits: torch.Tensor | None = None, best: torch.Tensor | None = None,
              plan: Plan | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Greedy head: ``idx[m] = argmax_n (a @ b)[m, n]`` over the bf16 products, lowest index on
    ties — ``torch.mm(a, b, out=logits); torch.argmax(logits, dim=-1, out=idx)`` at
    engine/engine.py:114-116 in one launch, the argmax folded into the linear's epilogue.

    a: bf16 CUDA [M, K]; b = W.t() of a row-major [N, K] weight (as ``mm``); idx: int64 CUDA
    [M] or [M, 1] — the engine's ``next_tokens`` is [B, 1] (``keepdim=True``,
    engine/engine.py:91,116). ``logits`` (bf16 [M, N], unit column stride) is written only if
    given, so the [M, N] logits need not be stored; ``best`` (bf16 [M] or [M, 1]) receives
    each row's maximum. Tensor-core plans only (16-byte aligned operands, K a multiple of 8).
    """
    _check_tensor(a, "a")
    _check_tensor(b, "b")
    M, K = a.shape
    K2, N = b.shape
    if K2 != K:
        raise ValueError(f"mm_argmax: a is [{M}, {K}] but b is [{K2}, {N}]")
    if not isinstance(idx, torch.Tensor) or idx.dtype != torch.int64 or idx.device != a.device:
        raise ValueError("mm_argmax: idx must be an int64 tensor on a's device")
    if not _rows_vector(idx, M):
        raise ValueError(f"mm_argmax: idx must be a contiguous [{M}] or [{M}, 1] tensor")
    if logits is not None:
        _check_tensor(logits, "logits")
        if tuple(logits.shape) != (M, N) or (N > 1 and logits.stride(1) != 1):
            raise ValueError(f"mm_argmax: logits must be [{M}, {N}] with unit stride along N")
    if best is not None:
        if best.dtype != torch.bfloat16 or best.device != a.device or not _rows_vector(best, M):
            raise ValueError(f"mm_argmax: best must be a contiguous bf16 [{M}] or [{M}, 1] "
                             "tensor")
    if b.device != a.device:
        raise ValueError("mm_argmax: a and b must be on the same device")
    if M == 0:
        return idx
    if N == 0 or K == 0:
        raise ValueError("mm_argmax: needs N >= 1 and K >= 1")
    if a.stride(1) != 1 and K > 1:
        raise ValueError("mm_argmax: a must have unit stride along K")
    if b.stride(0) != 1 and K > 1:
        raise ValueError("mm_argmax: b must be the transposed view W.t() of a row-major "
                         "[N, K] weight (strides (1, ldw))")
    ldx = a.stride(0) if M > 1 else K
    ldw = b.stride(1) if N > 1 else K
    ldy = (logits.stride(0) if M > 1 else N) if logits is not None else 0
    if plan is None:
        plan = plan_for(M, N, K)
    L = _lib.load()
    need = int(L.nk_gemm_argmax_ws_bytes(plan._ref))
    if need == 0:
        raise ValueError("mm_argmax: the plan is not a tensor-core plan (operands must be "
                         "16-byte aligned with K a multiple of 8)")
    dev = a.device
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    ws = workspace(need, dev, stream)
    args = (a.data_ptr(), ldx, b.data_ptr(), ldw,
            logits.data_ptr() if logits is not None else None, ldy, idx.data_ptr(),
            best.data_ptr() if best is not None else None, M, N, K, plan._ref, ws.data_ptr(),
            ws.numel(), stream.cuda_stream)
    if dev.index != torch.cuda.current_device():
        with torch.cuda.device(dev):
            status = L.nk_gemm_bf16_argmax(*args)
    else:
        status = L.nk_gemm_bf16_argmax(*args)
    if status != _lib.NK_OK:
        _raise(status, f"nk_gemm_bf16_argmax(M={M}, N={N}, K={K})")
    return idx


def linear_out(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor,
               plan: Plan | None = None) -> torch.Tensor:
    """``out = x · weightᵀ`` for a row-major [N, K] ``weight`` (same as ``mm(x, weight.t(), out=out)``)."""
    return mm(x, weight.t(), out=out, plan=plan)


def device_error(stream: torch.cuda.Stream | None = None) -> int:
    """Read and clear the device error word (NK_ERR_TIMEOUT after an expired bounded wait)."""
    stream = stream or torch.cuda.current_stream()
    st = ctypes.c_int(0)
    status = _lib.load().nk_device_error(stream.cuda_stream, ctypes.byref(st))
    if status != _lib.NK_OK:
        _raise(status, "nk_device_error")
    return st.value
