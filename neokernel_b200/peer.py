"""All-reduce of the tensor-parallel fp32 partials over NVLink peer memory (include/nk_comm.h).

``PeerGroup`` owns one receive buffer per rank, allocated by the library and mapped into every
other rank of the process group with CUDA IPC (the handles travel over the process group), and
``allreduce_bf16(x, out)`` launches ``nk_allreduce_bf16``: out = bf16(x_0 + ... + x_{T-1}),
ranks added in rank order, on the current stream, capturable in a CUDA graph. It stands in for
``dist.all_reduce`` followed by the bf16 copy in the tensor-parallel hooks (neokernel_b200/tp.py)
for the linears split along K (engine/kernels/decode.py:58,66). ``mm_allreduce(a, b, out)``
goes one step further and launches ``nk_gemm_bf16_allreduce``: the K-slice linear itself,
whose kernel stores each output tile's fp32 values straight into every rank's buffer and
adds up the ranks' values of the tile. A group serves one of the two kinds of call. Every
rank must make the same sequence of calls.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .gemm import _raise


class PeerGroup:
    def __init__(self, max_elems: int, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= _lib.NK_PEER_MAX_RANKS:
            raise ValueError(f"peer all-reduce needs 2..{_lib.NK_PEER_MAX_RANKS} ranks, "
                             f"got {self.world}")
        max_elems = (int(max_elems) + 3) // 4 * 4
        if not 1 <= max_elems <= _lib.NK_PEER_MAX_ELEMS:
            raise ValueError(f"peer all-reduce of {max_elems} elements is out of range")
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        L = _lib.load()
        self._L = L
        nbytes = int(L.nk_peer_buffer_bytes(max_elems, self.world))
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            st = L.nk_peer_alloc(nbytes, ctypes.byref(own))
            if st != _lib.NK_OK:
                _raise(st, "nk_peer_alloc")
            handle = (ctypes.c_char * _lib.NK_IPC_HANDLE_BYTES)()
            st = L.nk_ipc_handle(own, handle)
            if st != _lib.NK_OK:
                _raise(st, "nk_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self._own = own
            self._opened = []
            self.c = _lib.NkPeerGroup()
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.c.buf[r] = own.value
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_char * _lib.NK_IPC_HANDLE_BYTES).from_buffer_copy(h)
                st = L.nk_ipc_open(buf, ctypes.byref(p))
                if st != _lib.NK_OK:
                    _raise(st, f"nk_ipc_open(rank {r})")
                self._opened.append(p)
                self.c.buf[r] = p.value
        self.c.rank, self.c.world, self.c.max_elems = self.rank, self.world, max_elems
        self._ref = ctypes.byref(self.c)
        dist.barrier(group=group)  # every rank has mapped every buffer before the first call

    def allreduce_bf16(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out = bf16(sum over ranks of x); x fp32, out bf16, same number of elements."""
        if not (x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
                and out.is_cuda and out.dtype == torch.bfloat16 and out.is_contiguous()
                and x.numel() == out.numel()):
            raise ValueError("allreduce_bf16: contiguous fp32 x and bf16 out of one size")
        s = torch.cuda.current_stream(x.device).cuda_stream
        st = self._L.nk_allreduce_bf16(x.data_ptr(), out.data_ptr(), x.numel(), self._ref, s)
        if st != _lib.NK_OK:
            _raise(st, "nk_allreduce_bf16")
        return out

    def mm_allreduce(self, a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor,
                     plan=None) -> torch.Tensor:
        """out = bf16(sum over ranks of a_r @ b_r), ranks added in rank order: this rank's K
        slice of a tensor-parallel linear fused with its all-reduce in one launch
        (``nk_gemm_bf16_allreduce``). a: bf16 [M, K_r]; b = W_r.t() of a row-major [N, K_r]
        weight slice; out: bf16 [M, N] contiguous. The group must be made for at least M * N
        elements and serve no ``allreduce_bf16`` calls; every rank makes the same calls."""
        from . import gemm
        gemm._check_tensor(a, "a")
        gemm._check_tensor(b, "b")
        gemm._check_tensor(out, "out")
        M, K = a.shape
        K2, N = b.shape
        if K2 != K or tuple(out.shape) != (M, N):
            raise ValueError(f"mm_allreduce: a [{M}, {K}], b [{K2}, {N}], out {tuple(out.shape)}")
        if a.stride(1) != 1 or b.stride(0) != 1 or not out.is_contiguous():
            raise ValueError("mm_allreduce: a row-major, b = W.t() of a row-major weight, "
                             "out contiguous")
        if M * N > self.c.max_elems:
            raise ValueError(f"mm_allreduce: {M} x {N} outputs exceed the group's "
                             f"{self.c.max_elems} elements")
        plan = plan or gemm.plan_for(M, N, K)
        dev = a.device
        stream = torch.cuda.current_stream(dev)
        ws = gemm.workspace(max(plan.ws_bytes, 1), dev, stream) if plan.ws_bytes else None
        st = self._L.nk_gemm_bf16_allreduce(
            a.data_ptr(), a.stride(0) if M > 1 else K, b.data_ptr(), b.stride(1) if N > 1 else K,
            out.data_ptr(), N, M, N, K, plan._ref, ws.data_ptr() if ws is not None else None,
            ws.numel() if ws is not None else 0, self._ref, stream.cuda_stream)
        if st != _lib.NK_OK:
            _raise(st, f"nk_gemm_bf16_allreduce(M={M}, N={N}, K={K})")
        return out

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still writes into another's buffer
        for p in self._opened:
            self._L.nk_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)  # every mapping of this rank's buffer is gone
        if self._own is not None:
            self._L.nk_peer_free(self._own)
            self._own = None
