"""ORACLE — TEST INFRASTRUCTURE ONLY.

Python face of the CPU restatement in ``oracle/nk_oracle.c`` of the reference's decode
linear ``torch.mm(x, W.t(), out=y)`` (engine/kernels/decode.py:54,58,64,66;
engine/engine.py:114). Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg import this module, and only to check or time; the product package
``neokernel_b200`` never does.

All arrays are numpy ``uint16`` holding bf16 bit patterns, row-major with explicit leading
dimensions, mirroring the C ABI of the product library.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnkoracle.so")

_lib = None


def build(force: bool = False) -> str:
    """Compile nk_oracle.c with the committed Makefile (gcc)."""
    if force or not os.path.exists(LIB_PATH) or (
            os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "nk_oracle.c"))):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        f64p = ctypes.POINTER(ctypes.c_double)
        i64 = ctypes.c_int64
        L.nko_gemm_bf16.argtypes = [u16p, i64, u16p, i64, u16p, i64, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int]
        L.nko_gemm_bf16.restype = None
        L.nko_gemm_f64.argtypes = [u16p, i64, u16p, i64, f64p, i64, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int]
        L.nko_gemm_f64.restype = None
        L.nko_f32_to_bf16_array.argtypes = [ctypes.POINTER(ctypes.c_float), u16p, i64]
        L.nko_f32_to_bf16_array.restype = None
        L.nko_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.nko_bf16_to_f32.restype = ctypes.c_float
        _lib = L
    return _lib


def _ptr(a, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def _check(x, w):
    if x.dtype != np.uint16 or w.dtype != np.uint16:
        raise TypeError("oracle operands are uint16 arrays of bf16 bit patterns")
    if x.ndim != 2 or w.ndim != 2 or x.shape[1] != w.shape[1]:
        raise ValueError(f"shape mismatch: x {x.shape}, w {w.shape} (need [M,K] and [N,K])")
    return np.ascontiguousarray(x), np.ascontiguousarray(w)


def _row_blocks(N: int, threads: int):
    step = max(1, (N + threads - 1) // threads)
    return [(n0, min(N, n0 + step)) for n0 in range(0, N, step)]


def gemm_bf16(x: np.ndarray, w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """y = bf16(x · wᵀ) with fp32 accumulation in ascending k (uint16 in, uint16 out).

    ``ctypes`` releases the GIL during the foreign call, so row blocks of ``w`` run in
    parallel threads; each output element is still one sequential fp32 sum.
    """
    x, w = _check(x, w)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.uint16)
    L = lib()
    threads = threads or min(8, os.cpu_count() or 1)

    def run(block):
        n0, n1 = block
        L.nko_gemm_bf16(_ptr(x, ctypes.c_uint16), K, _ptr(w[n0:n1], ctypes.c_uint16), K,
                        ctypes.cast(y.ctypes.data + 2 * n0, ctypes.POINTER(ctypes.c_uint16)), N,
                        M, n1 - n0, K)

    blocks = _row_blocks(N, threads)
    if len(blocks) == 1:
        run(blocks[0])
    else:
        with ThreadPoolExecutor(len(blocks)) as pool:
            list(pool.map(run, blocks))
    return y


def gemm_f64(x: np.ndarray, w: np.ndarray, threads: int | None = None) -> np.ndarray:
    """Same product accumulated in double, not rounded (float64 [M, N])."""
    x, w = _check(x, w)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    L = lib()
    threads = threads or min(8, os.cpu_count() or 1)

    def run(block):
        n0, n1 = block
        L.nko_gemm_f64(_ptr(x, ctypes.c_uint16), K, _ptr(w[n0:n1], ctypes.c_uint16), K,
                       ctypes.cast(y.ctypes.data + 8 * n0, ctypes.POINTER(ctypes.c_double)), N,
                       M, n1 - n0, K)

    blocks = _row_blocks(N, threads)
    if len(blocks) == 1:
        run(blocks[0])
    else:
        with ThreadPoolExecutor(len(blocks)) as pool:
            list(pool.map(run, blocks))
    return y


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 bit patterns (nearest-even, NaN kept quiet)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    h = np.empty(f.shape, dtype=np.uint16)
    lib().nko_f32_to_bf16_array(_ptr(f, ctypes.c_float), _ptr(h, ctypes.c_uint16), f.size)
    return h


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns to float32 (exact)."""
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def tolerance(K: int) -> float:
    """North-star bound on max|y - x·wᵀ| for bf16 output with fp32 accumulation."""
    return 2e-2 * (K / 1024.0) ** 0.5


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 units-in-the-last-place between two bf16 bit-pattern arrays."""
    def ordered(h):
        h = np.asarray(h, dtype=np.uint16).astype(np.int32)
        return np.where(h & 0x8000, 0x8000 - h, h)  # monotone map of the sign-magnitude code
    return np.abs(ordered(a) - ordered(b))
