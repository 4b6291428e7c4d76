"""ctypes binding of ``libnkgemm.so`` (C ABI declared in ``include/nk_gemm.h``).

The library is built in-tree by ``neokernel_b200.build`` into ``neokernel_b200/lib/``. There is
no CPU or library fallback: if the shared object is missing, importing the operator raises.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# NK_LIB_PATH selects another build of the same library (for example one compiled with
# different tile parameters); by default the in-tree build is used.
LIB_PATH = os.environ.get("NK_LIB_PATH") or os.path.join(HERE, "lib", "libnkgemm.so")

# Status codes and kernel kinds (include/nk_gemm.h).
NK_OK = 0
NK_ERR_SHAPE = -1
NK_ERR_ALIGN = -2
NK_ERR_WORKSPACE = -3
NK_ERR_SPLIT = -4
NK_ERR_PLAN = -5
NK_ERR_CUDA = -6
NK_ERR_DEVICE = -7
NK_ERR_TIMEOUT = -8
NK_ERR_ARG = -9
NK_ERR_RANGE = -10

KIND_AUTO = 0
KIND_GEMV = 1
KIND_TC = 2
KIND_GENERIC = 3
MAX_SPLIT = 16
PLAN_MAGIC = 0x4E4B4731

# Every function the header declares; the CPU test checks the .so exports each of them.
EXPORTS = ("nk_plan_make", "nk_ws_bytes", "nk_ws_init", "nk_gemm_bf16", "nk_device_error",
           "nk_status_string", "nk_version", "nk_gemm_bf16_static", "nk_gemm_bf16_f32out",
           "nk_rmsnorm_bf16", "nk_qk_norm_rope_cache_bf16", "nk_attention_ws_bytes",
           "nk_attention_decode_bf16", "nk_silu_mul_bf16", "nk_peer_buffer_bytes", "nk_peer_alloc",
           "nk_peer_free", "nk_ipc_handle", "nk_ipc_open", "nk_ipc_close", "nk_allreduce_bf16",
           "nk_gemm_argmax_ws_bytes", "nk_gemm_bf16_argmax", "nk_test_withhold_partial",
           "nk_gemm_bf16_allreduce", "nk_gemm_bf16_qkv_rope_cache")


NK_PEER_MAX_RANKS = 8
NK_IPC_HANDLE_BYTES = 64
NK_PEER_MAX_ELEMS = 1 << 20


class NkPeerGroup(ctypes.Structure):
    """``nk_peer_group`` (include/nk_comm.h)."""
    _fields_ = [("buf", ctypes.c_void_p * NK_PEER_MAX_RANKS), ("rank", ctypes.c_int32),
                ("world", ctypes.c_int32), ("max_elems", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class NkPlan(ctypes.Structure):
    _fields_ = [
        ("magic", ctypes.c_int32),
        ("M_max", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("kind", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("k_slice", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("n_tiles", ctypes.c_int32),
        ("m_tiles", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("segments", ctypes.c_int32),
        ("k_step", ctypes.c_int32),
        ("slices", ctypes.c_int32),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class NkError(RuntimeError):
    """A non-zero status from libnkgemm.so."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (status {status})")


_lib = None


def load() -> ctypes.CDLL:
    """Load the library once; raise loudly if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libnkgemm.so not found at {LIB_PATH}; build it with "
            "`python -m neokernel_b200.build` (there is no fallback implementation)")
    L = ctypes.CDLL(LIB_PATH)
    vp = ctypes.c_void_p
    i32 = ctypes.c_int
    i64 = ctypes.c_int64
    L.nk_plan_make.argtypes = [ctypes.POINTER(NkPlan), i32, i32, i32, i32, i32]
    L.nk_plan_make.restype = i32
    L.nk_ws_bytes.argtypes = [ctypes.POINTER(NkPlan)]
    L.nk_ws_bytes.restype = ctypes.c_size_t
    L.nk_ws_init.argtypes = [vp, ctypes.c_size_t, vp]
    L.nk_ws_init.restype = i32
    L.nk_gemm_bf16.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32,
                               ctypes.POINTER(NkPlan), vp, ctypes.c_size_t, vp]
    L.nk_gemm_bf16.restype = i32
    L.nk_gemm_bf16_f32out.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32,
                                      ctypes.POINTER(NkPlan), vp, ctypes.c_size_t, vp]
    L.nk_gemm_bf16_f32out.restype = i32
    L.nk_gemm_argmax_ws_bytes.argtypes = [ctypes.POINTER(NkPlan)]
    L.nk_gemm_argmax_ws_bytes.restype = ctypes.c_size_t
    L.nk_gemm_bf16_argmax.argtypes = [vp, i64, vp, i64, vp, i64, vp, vp, i32, i32, i32,
                                      ctypes.POINTER(NkPlan), vp, ctypes.c_size_t, vp]
    L.nk_gemm_bf16_argmax.restype = i32
    f32 = ctypes.c_float
    L.nk_rmsnorm_bf16.argtypes = [vp, vp, vp, vp, i32, i32, f32, vp]
    L.nk_rmsnorm_bf16.restype = i32
    L.nk_qk_norm_rope_cache_bf16.argtypes = [vp, i64, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32,
                                             i32, i32, i32, i64, i64, i64, f32, vp]
    L.nk_qk_norm_rope_cache_bf16.restype = i32
    L.nk_gemm_bf16_qkv_rope_cache.argtypes = [vp, i64, vp, i64, i32, i32, i32,
                                              ctypes.POINTER(NkPlan), vp, ctypes.c_size_t,
                                              vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32,
                                              i64, i64, i64, f32, vp]
    L.nk_gemm_bf16_qkv_rope_cache.restype = i32
    L.nk_attention_ws_bytes.argtypes = [i32, i32, i32]
    L.nk_attention_ws_bytes.restype = ctypes.c_size_t
    L.nk_attention_decode_bf16.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i64, i64,
                                           i64, f32, vp, ctypes.c_size_t, vp]
    L.nk_attention_decode_bf16.restype = i32
    L.nk_silu_mul_bf16.argtypes = [vp, vp, i32, i32, vp]
    L.nk_silu_mul_bf16.restype = i32
    L.nk_peer_buffer_bytes.argtypes = [i32, i32]
    L.nk_peer_buffer_bytes.restype = ctypes.c_size_t
    L.nk_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
    L.nk_peer_alloc.restype = i32
    L.nk_peer_free.argtypes = [vp]
    L.nk_peer_free.restype = i32
    L.nk_ipc_handle.argtypes = [vp, vp]
    L.nk_ipc_handle.restype = i32
    L.nk_ipc_open.argtypes = [vp, ctypes.POINTER(vp)]
    L.nk_ipc_open.restype = i32
    L.nk_ipc_close.argtypes = [vp]
    L.nk_ipc_close.restype = i32
    L.nk_allreduce_bf16.argtypes = [vp, vp, i32, ctypes.POINTER(NkPeerGroup), vp]
    L.nk_allreduce_bf16.restype = i32
    L.nk_test_withhold_partial.argtypes = [i32]
    L.nk_test_withhold_partial.restype = i32
    L.nk_gemm_bf16_allreduce.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32,
                                         ctypes.POINTER(NkPlan), vp, ctypes.c_size_t,
                                         ctypes.POINTER(NkPeerGroup), vp]
    L.nk_gemm_bf16_allreduce.restype = i32
    L.nk_device_error.argtypes = [vp, ctypes.POINTER(i32)]
    L.nk_device_error.restype = i32
    L.nk_status_string.argtypes = [i32]
    L.nk_status_string.restype = ctypes.c_char_p
    L.nk_version.argtypes = []
    L.nk_version.restype = i32
    _lib = L
    return L


def status_string(status: int) -> str:
    return load().nk_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != NK_OK:
        raise NkError(status, where)
