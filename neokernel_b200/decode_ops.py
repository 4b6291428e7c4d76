"""Python face of the fused decode kernels (include/nk_decode.h).

Same conventions as ``neokernel_b200.mm``: caller-owned CUDA tensors, launch on the current
stream, ``ValueError`` before launching for an unsupported configuration, no allocation, no
host synchronisation. Each replaces one of the reference engine's Triton wrappers:

* ``rmsnorm``            <- ``norm_out``            (engine/kernels/rmsnorm.py:28-41)
* ``qk_norm_rope_cache`` <- ``qk_rope_cache_out``   (engine/kernels/elementwise.py:63-78)
* ``qkv_rope_cache``     <- ``torch.mm(norm, w.qkv, out=qkv)`` + ``qk_rope_cache_out``
                            (engine/kernels/decode.py:54-55): the QKV linear and its consumer
                            in one launch, qkv never stored
* ``attention_decode``   <- ``attention_out``       (engine/kernels/attention.py:53-62)
* ``silu_mul``           <- ``silu_mul_out``        (engine/kernels/elementwise.py:91-101)
"""

from __future__ import annotations

import math

import torch

from . import _lib
from .gemm import _raise

HEAD_DIM = 128


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(cond, msg):
    if not cond:
        raise ValueError(msg)


def _bf16_cuda(*ts):
    for t in ts:
        _need(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.bfloat16,
              "decode ops take bf16 CUDA tensors")


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, eps: float,
            branch: torch.Tensor | None = None) -> torch.Tensor:
    """out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight); with ``branch``, first
    x <- bf16(x + branch) in place (the fused residual add of the reference's
    ``norm_out(branch, w, out, eps, x, x)``)."""
    _bf16_cuda(x, weight, out, *([branch] if branch is not None else []))
    _need(x.dim() == 2 and x.is_contiguous() and out.shape == x.shape and out.is_contiguous(),
          "rmsnorm: x and out must be contiguous [rows, width]")
    _need(branch is None or (branch.shape == x.shape and branch.is_contiguous()),
          "rmsnorm: branch must match x")
    st = _lib.load().nk_rmsnorm_bf16(x.data_ptr(), branch.data_ptr() if branch is not None else None,
                                      weight.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1],
                                      float(eps), _stream(x))
    if st != _lib.NK_OK:
        _raise(st, "nk_rmsnorm_bf16")
    return out


def qk_norm_rope_cache(qkv, q_norm, k_norm, cos, sin, position, q_out, k_cache, v_cache,
                       heads: int, kv_heads: int, eps: float):
    """Q/K head RMSNorm + RoPE at ``position`` (device int64 [1]); queries to ``q_out``
    [B, heads*128], keys and values into the [B, kv_heads, capacity, 128] caches. A position
    outside the caches writes nothing and is reported by ``device_error()``."""
    _bf16_cuda(qkv, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    _need(position.is_cuda and position.dtype == torch.int64, "position: CUDA int64 tensor")
    B = qkv.shape[0]
    _need(qkv.stride(1) == 1 and q_out.is_contiguous() and cos.is_contiguous()
          and sin.is_contiguous() and k_cache.stride(3) == 1 and v_cache.stride() == k_cache.stride(),
          "qk_norm_rope_cache: unsupported layout")
    st = _lib.load().nk_qk_norm_rope_cache_bf16(
        qkv.data_ptr(), qkv.stride(0), q_norm.data_ptr(), k_norm.data_ptr(), cos.data_ptr(),
        sin.data_ptr(), position.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(),
        v_cache.data_ptr(), B, heads, kv_heads, HEAD_DIM, k_cache.shape[2], k_cache.stride(0),
        k_cache.stride(1), k_cache.stride(2), float(eps), _stream(qkv))
    if st != _lib.NK_OK:
        _raise(st, "nk_qk_norm_rope_cache_bf16")


def qkv_rope_cache(x, w_qkv_t, q_norm, k_norm, cos, sin, position, q_out, k_cache, v_cache,
                   heads: int, kv_heads: int, eps: float, plan=None):
    """``qk_norm_rope_cache`` of ``x @ w_qkv_t`` without storing the product: the QKV linear
    (``w_qkv_t`` = Wqkv.t() of the packed row-major weight, as ``mm`` takes it) whose kernel
    finishes each 128-row head tile with that head's RMSNorm + RoPE and writes queries, keys
    and values where the attention reads them. Same bits as ``mm`` then
    ``qk_norm_rope_cache``. Decode batches of up to 16 tokens."""
    from . import gemm
    gemm._check_tensor(x, "x")
    gemm._check_tensor(w_qkv_t, "w_qkv_t")
    _bf16_cuda(q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    _need(position.is_cuda and position.dtype == torch.int64, "position: CUDA int64 tensor")
    M, K = x.shape
    K2, N = w_qkv_t.shape
    _need(K2 == K and N == (heads + 2 * kv_heads) * HEAD_DIM,
          f"qkv_rope_cache: x [{M}, {K}] and w_qkv_t [{K2}, {N}] for {heads}+2x{kv_heads} heads")
    _need(1 <= M <= 16, "qkv_rope_cache: decode batches of 1 to 16 tokens")
    _need(x.stride(1) == 1 and w_qkv_t.stride(0) == 1 and q_out.is_contiguous()
          and cos.is_contiguous() and sin.is_contiguous() and k_cache.stride(3) == 1
          and v_cache.stride() == k_cache.stride(), "qkv_rope_cache: unsupported layout")
    plan = plan or gemm.plan_for(M, N, K)
    dev = x.device
    stream = torch.cuda.current_stream(dev)
    ws = gemm.workspace(plan.ws_bytes, dev, stream) if plan.ws_bytes else None
    st = _lib.load().nk_gemm_bf16_qkv_rope_cache(
        x.data_ptr(), x.stride(0) if M > 1 else K, w_qkv_t.data_ptr(), w_qkv_t.stride(1), M, N, K,
        plan._ref, ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        q_norm.data_ptr(), k_norm.data_ptr(), cos.data_ptr(), sin.data_ptr(), position.data_ptr(),
        q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), heads, kv_heads,
        k_cache.shape[2], k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), float(eps),
        stream.cuda_stream)
    if st != _lib.NK_OK:
        _raise(st, "nk_gemm_bf16_qkv_rope_cache")


def attention_workspace(batch: int, heads: int, capacity: int, device) -> torch.Tensor:
    n = _lib.load().nk_attention_ws_bytes(batch, heads, capacity)
    return torch.empty(max(int(n), 16), dtype=torch.uint8, device=device)


def attention_decode(q, k_cache, v_cache, position, out, ws, heads: int, kv_heads: int,
                     scale: float | None = None):
    """Grouped split-KV decode attention over slots [0, position]: q, out [B, heads*128]."""
    _bf16_cuda(q, k_cache, v_cache, out)
    _need(q.is_contiguous() and out.is_contiguous() and k_cache.stride(3) == 1
          and v_cache.stride() == k_cache.stride(), "attention_decode: unsupported layout")
    B, cap = q.shape[0], k_cache.shape[2]
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else scale
    st = _lib.load().nk_attention_decode_bf16(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), position.data_ptr(),
        out.data_ptr(), B, heads, kv_heads, HEAD_DIM, cap, k_cache.stride(0), k_cache.stride(1),
        k_cache.stride(2), float(scale), ws.data_ptr(), ws.numel(), _stream(q))
    if st != _lib.NK_OK:
        _raise(st, "nk_attention_decode_bf16")


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor):
    """out = bf16(bf16(silu(gate)) * up) for gate_up = [gate | up] rows."""
    _bf16_cuda(gate_up, out)
    _need(gate_up.is_contiguous() and out.is_contiguous()
          and gate_up.shape[1] == 2 * out.shape[1] and gate_up.shape[0] == out.shape[0],
          "silu_mul: gate_up [rows, 2I] and out [rows, I] contiguous")
    st = _lib.load().nk_silu_mul_bf16(gate_up.data_ptr(), out.data_ptr(), out.shape[0],
                                       out.shape[1], _stream(out))
    if st != _lib.NK_OK:
        _raise(st, "nk_silu_mul_bf16")
