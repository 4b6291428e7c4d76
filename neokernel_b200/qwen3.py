"""Qwen3 greedy-decode step on fixed buffers: the caller context of the decode linears.

This mirrors the reference engine's decode graph (engine/engine.py:100-117, one
``DecodeBuffers.layer`` per layer, engine/kernels/decode.py:42-68) closely enough to run the
decode linears where the engine runs them and to measure decode tokens/s:

    x = embed[token]
    per layer:  norm -> QKV linear -> per-head q/k RMSNorm + RoPE -> K/V cache write at the
                device-side position -> grouped attention over positions <= position ->
                o_proj linear -> residual add -> norm -> gate_up linear -> bf16(silu(g)) * u
                -> down linear -> residual add
    final norm -> lm_head linear -> argmax (lowest index on ties)

The five linears go through a pluggable ``linear(a, b, out)`` with ``torch.mm``'s signature:
``neokernel_b200.mm`` (the product) or ``torch.mm`` (the reference's own call, cuBLAS), so the
two differ only in the decode linears. Everything else is PyTorch on the GPU with the
reference's bf16 cast points (RMSNorm rounds the normalised value to bf16 before the gain,
engine/kernels/rmsnorm.py:12-25; RoPE rounds each product before the sum,
engine/kernels/elementwise.py:50-54; the SiLU is rounded to bf16 before the product,
engine/kernels/elementwise.py:81-88). Every buffer is allocated once in ``prepare`` and the
position lives on the device, so a step can be captured in one CUDA graph and replayed (the
reference captures its decode the same way, engine/engine.py:119-129).

Weights are random and seeded; no checkpoint is used. Two initialisations (``init``):

* ``"decisive"`` (default): every greedy choice is made by a wide margin, so two correct
  implementations of the step emit the same tokens. The embedding is N(0, 1), so the residual
  stream is led by the current token; QKV and gate_up are N(0, 0.02); the residual projections
  o_proj and down are N(0, 0.02 / sqrt(2 * layers)) (the scaled residual init of GPT-2-style
  models), so the 2 * layers branch outputs add up to about the embedding's size; the
  lm_head's row v is the embedding row of token perm(v) scaled by 1 / sqrt(hidden), for a
  seeded random permutation ``perm``, so the token after t is most often perm^-1(t) with
  a logit near 1 * sqrt(hidden) * gain, tens of logits above the rest; every norm gain is
  drawn from U(0.5, 1.5), so no multiplication by a gain is the identity.
* ``"reference"``: the reference kernel test's init (tests/test_hand_rolled_kernels.py:
  154-156): ``normal_(0, 0.02)`` for every matrix and ones for the norm gains. Its logits are
  nearly flat (top-2 gaps of a few hundredths), so greedy tokens flip on genuine near-ties
  between any two valid fp32-accumulating GEMMs.
"""

from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class Qwen3Dims:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    layers: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    tie_embeddings: bool = False

    @property
    def q_width(self):
        return self.heads * self.head_dim

    @property
    def kv_width(self):
        return self.kv_heads * self.head_dim

    @property
    def qkv_width(self):
        return self.q_width + 2 * self.kv_width


QWEN3_0_6B = Qwen3Dims(1024, 3072, 16, 8, 128, 28, 151936, tie_embeddings=True)
QWEN3_4B = Qwen3Dims(2560, 9728, 32, 8, 128, 36, 151936, tie_embeddings=True)
QWEN3_8B = Qwen3Dims(4096, 12288, 32, 8, 128, 36, 151936)
QWEN3_32B = Qwen3Dims(5120, 25600, 64, 8, 128, 64, 151936)


INITS = ("decisive", "reference")

# True: the fused decode step runs the QKV linear and its q/k-norm + RoPE + cache consumer as
# one launch (nk_gemm_bf16_qkv_rope_cache) when the linear is neokernel_b200.mm. Off by
# default: measured on B200 (Qwen3-8B, KV 1024, CUDA graph), the step takes 3.61 / 4.59 ms at
# batch 1 / 16 with it and 3.37 / 4.25 ms with the two launches — the consumer then runs in
# the tail of the linear's finishing CTAs (one per head, after the split-K sum) instead of as
# a separate, fully parallel launch that overlaps the linear's tail.
FUSE_QKV = False


def _randn(shape, gen, device, std=0.02):
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    return t.mul_(std).to(torch.bfloat16)


def _gain(n, gen, device, init):
    """A norm gain: ones (reference init) or U(0.5, 1.5) (decisive init)."""
    if init == "reference":
        return torch.ones(n, device=device, dtype=torch.bfloat16)
    t = torch.rand(n, generator=gen, device=device, dtype=torch.float32)
    return t.add_(0.5).to(torch.bfloat16)


def _check_init(init):
    if init not in INITS:
        raise ValueError(f"init must be one of {INITS}, not {init!r}")


class LayerWeights:
    """One layer's weights in the reference's packed layout (engine/kernels/weights.py:10-25):
    row-major ``qkv_weight [Nq+2Nkv, H]`` and ``gate_up_weight [2I, H]``; the linears take
    their ``.t()`` views. Drawn in a fixed order from ``gen``."""

    def __init__(self, d: Qwen3Dims, gen, device, init: str = "decisive"):
        _check_init(init)
        H, I = d.hidden, d.intermediate
        res_std = 0.02 if init == "reference" else 0.02 / math.sqrt(2 * d.layers)
        self.qkv_weight = _randn((d.qkv_width, H), gen, device)
        self.o_weight = _randn((H, d.q_width), gen, device, res_std)
        self.gate_up_weight = _randn((2 * I, H), gen, device)
        self.down_weight = _randn((H, I), gen, device, res_std)
        self.qkv = self.qkv_weight.t()
        self.o = self.o_weight.t()
        self.gate_up = self.gate_up_weight.t()
        self.down = self.down_weight.t()
        self.input_norm = _gain(H, gen, device, init)
        self.post_norm = _gain(H, gen, device, init)
        self.q_norm = _gain(d.head_dim, gen, device, init)
        self.k_norm = _gain(d.head_dim, gen, device, init)


def draw_embedding(d: Qwen3Dims, gen, device, init: str):
    """The token embedding [vocab, hidden]: the first draw of a model."""
    return _randn((d.vocab, d.hidden), gen, device, 0.02 if init == "reference" else 1.0)


def draw_head(d: Qwen3Dims, embed, gen, device, init: str):
    """(final-norm gain, lm_head weight [vocab, hidden]): the last draws of a model. Tied
    models use the embedding itself; an untied decisive model the permuted, scaled embedding
    rows (row v = embed[perm[v]] / sqrt(hidden))."""
    final_norm = _gain(d.hidden, gen, device, init)
    if d.tie_embeddings:
        return final_norm, embed
    if init == "reference":
        return final_norm, _randn((d.vocab, d.hidden), gen, device)
    perm = torch.randperm(d.vocab, generator=gen, device=device)
    head = (embed.index_select(0, perm).float() * (1.0 / math.sqrt(d.hidden))).to(torch.bfloat16)
    return final_norm, head


class Qwen3Weights:
    def __init__(self, d: Qwen3Dims, seed: int = 0, device="cuda", layers: int | None = None,
                 init: str = "decisive"):
        _check_init(init)
        self.dims, self.init = d, init
        gen = torch.Generator(device=device).manual_seed(seed)
        self.embed = draw_embedding(d, gen, device, init)
        n = d.layers if layers is None else layers
        self.layers = [LayerWeights(d, gen, device, init) for _ in range(n)]
        self.final_norm, self.lm_head_weight = draw_head(d, self.embed, gen, device, init)
        self.lm_head = self.lm_head_weight.t()  # engine/engine.py:70


def rope_tables(d: Qwen3Dims, capacity: int, device):
    """Rotary cos/sin [capacity, head_dim] in bf16 (Qwen3 rotary embedding: inverse
    frequencies theta^(-2i/D) in fp32, angles duplicated across the two halves)."""
    inv = 1.0 / (d.rope_theta ** (torch.arange(0, d.head_dim, 2, device=device,
                                                dtype=torch.float32) / d.head_dim))
    pos = torch.arange(capacity, device=device, dtype=torch.float32)
    freqs = torch.outer(pos, inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def rms_norm(x, weight, eps, out=None):
    """bf16(x / rms(x)) * weight with the normalised value rounded to bf16 first."""
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.bfloat16)
    if out is None:
        return n * weight
    return torch.mul(n, weight, out=out)


def rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class DecodeState:
    """Fixed buffers for batch ``B`` and cache ``capacity`` (reference: DecodeBuffers,
    engine/kernels/decode.py:10-39, and Engine.prepare, engine/engine.py:76-98)."""

    def __init__(self, w: Qwen3Weights, batch: int, capacity: int, device="cuda"):
        d = w.dims
        bf = dict(device=device, dtype=torch.bfloat16)
        self.batch, self.capacity = batch, capacity
        self.tokens = torch.zeros(batch, device=device, dtype=torch.int64)
        self.position = torch.zeros(1, device=device, dtype=torch.int64)
        self.x = torch.empty(batch, d.hidden, **bf)
        self.norm = torch.empty(batch, d.hidden, **bf)
        self.qkv = torch.empty(batch, d.qkv_width, **bf)
        self.attn = torch.empty(batch, d.q_width, **bf)
        self.branch = torch.empty(batch, d.hidden, **bf)
        self.gate_up = torch.empty(batch, 2 * d.intermediate, **bf)
        self.product = torch.empty(batch, d.intermediate, **bf)
        self.logits = torch.empty(batch, d.vocab, **bf)
        self.next_tokens = torch.zeros(batch, device=device, dtype=torch.int64)
        n = len(w.layers)
        self.k_cache = [torch.zeros(batch, d.kv_heads, capacity, d.head_dim, **bf) for _ in range(n)]
        self.v_cache = [torch.zeros(batch, d.kv_heads, capacity, d.head_dim, **bf) for _ in range(n)]
        self.cos, self.sin = rope_tables(d, capacity, device)
        self.slots = torch.arange(capacity, device=device)
        self.q = torch.empty(batch, d.q_width, **bf)
        self.attn_ws = None  # fused path: split-KV partials, made on first fused step


def attention(q, k_cache, v_cache, position, slots, d: Qwen3Dims):
    """Grouped decode attention over cache positions <= position (fp32 scores and softmax)."""
    B = q.shape[0]
    G = d.heads // d.kv_heads
    qf = q.view(B, d.kv_heads, G, d.head_dim).float()
    scores = torch.matmul(qf, k_cache.float().transpose(-1, -2)) * (1.0 / math.sqrt(d.head_dim))
    scores = scores.masked_fill((slots > position).view(1, 1, 1, -1), float("-inf"))
    p = torch.softmax(scores, dim=-1)
    out = torch.matmul(p, v_cache.float())  # [B, Hkv, G, D]
    return out.reshape(B, d.q_width).to(torch.bfloat16)


def layer_step(st: DecodeState, w: LayerWeights, k_cache, v_cache, d: Qwen3Dims, linear,
               row_linear=None):
    """One decoder layer. ``row_linear`` computes o_proj and down (the K-split linears of the
    tensor-parallel mode, which all-reduce before rounding); by default it is ``linear``."""
    row_linear = row_linear or linear
    B = st.batch
    rms_norm(st.x, w.input_norm, d.eps, out=st.norm)
    linear(st.norm, w.qkv, out=st.qkv)                                   # decode.py:54
    q = st.qkv[:, :d.q_width].view(B, d.heads, d.head_dim)
    k = st.qkv[:, d.q_width:d.q_width + d.kv_width].view(B, d.kv_heads, d.head_dim)
    v = st.qkv[:, d.q_width + d.kv_width:].view(B, d.kv_heads, d.head_dim)
    q = rms_norm(q, w.q_norm, d.eps)
    k = rms_norm(k, w.k_norm, d.eps)
    cos = torch.index_select(st.cos, 0, st.position).view(1, 1, -1)
    sin = torch.index_select(st.sin, 0, st.position).view(1, 1, -1)
    q = (q * cos) + (rotate_half(q) * sin)
    k = (k * cos) + (rotate_half(k) * sin)
    k_cache.index_copy_(2, st.position, k.unsqueeze(2))
    v_cache.index_copy_(2, st.position, v.unsqueeze(2))
    st.attn.copy_(attention(q, k_cache, v_cache, st.position, st.slots, d))
    row_linear(st.attn, w.o, out=st.branch)                              # decode.py:58
    torch.add(st.x, st.branch, out=st.x)
    rms_norm(st.x, w.post_norm, d.eps, out=st.norm)
    linear(st.norm, w.gate_up, out=st.gate_up)                           # decode.py:64
    I = d.intermediate
    g = st.gate_up[:, :I].float()
    act = (g / (1.0 + torch.exp(-g))).to(torch.bfloat16)   # elementwise.py:86
    torch.mul(act, st.gate_up[:, I:], out=st.product)
    row_linear(st.product, w.down, out=st.branch)                        # decode.py:66
    torch.add(st.x, st.branch, out=st.x)


def layer_step_fused(st: DecodeState, w: LayerWeights, k_cache, v_cache, d: Qwen3Dims, linear,
                     row_linear=None, carry=False):
    """The same layer on the fused kernels (neokernel_b200.decode_ops), with the reference's
    fuse_norm_residual scheme (engine/kernels/decode.py:42-68): the down projection's output
    stays in ``branch`` and the next RMSNorm adds it into ``x`` (``carry``)."""
    from . import decode_ops as ops
    from . import gemm
    row_linear = row_linear or linear
    ops.rmsnorm(st.x, w.input_norm, st.norm, d.eps, branch=st.branch if carry else None)
    if FUSE_QKV and linear is gemm.mm and st.batch <= 16:
        # decode.py:54-55 in one launch: the QKV linear finishes each head with its norm, RoPE
        # and cache write (qkv is not stored)
        ops.qkv_rope_cache(st.norm, w.qkv, w.q_norm, w.k_norm, st.cos, st.sin, st.position,
                           st.q, k_cache, v_cache, d.heads, d.kv_heads, d.eps)
    else:
        linear(st.norm, w.qkv, out=st.qkv)                               # decode.py:54
        ops.qk_norm_rope_cache(st.qkv, w.q_norm, w.k_norm, st.cos, st.sin, st.position, st.q,
                               k_cache, v_cache, d.heads, d.kv_heads, d.eps)
    ops.attention_decode(st.q, k_cache, v_cache, st.position, st.attn, st.attn_ws,
                         d.heads, d.kv_heads)
    row_linear(st.attn, w.o, out=st.branch)                              # decode.py:58
    ops.rmsnorm(st.x, w.post_norm, st.norm, d.eps, branch=st.branch)
    linear(st.norm, w.gate_up, out=st.gate_up)                           # decode.py:64
    ops.silu_mul(st.gate_up, st.product)
    row_linear(st.product, w.down, out=st.branch)                        # decode.py:66


def greedy_head(st: DecodeState, lm_head, linear):
    linear(st.norm, lm_head, out=st.logits)                               # engine.py:114
    torch.argmax(st.logits, dim=-1, out=st.next_tokens)                  # lowest index on ties


def fused_greedy_head(st: DecodeState, lm_head, linear):
    """lm_head and the lowest-index argmax in one launch (nk_gemm_bf16_argmax,
    engine.py:114-116): ``next_tokens`` without storing the [B, vocab] logits, so
    ``st.logits`` is left untouched."""
    from . import gemm
    gemm.mm_argmax(st.norm, lm_head, idx=st.next_tokens)


def decode_step(st: DecodeState, w: Qwen3Weights, linear, row_linear=None, head=None,
                fused=False):
    """One greedy decode step for every sequence at ``st.position``; writes ``st.next_tokens``.

    ``row_linear`` (o_proj, down) and ``head`` (lm_head + argmax) are the hooks the
    tensor-parallel mode replaces (neokernel_b200.tp); by default the step is single-GPU.
    ``fused`` runs the non-linear ops on the fused CUDA kernels instead of PyTorch ops."""
    d = w.dims
    torch.index_select(w.embed, 0, st.tokens, out=st.x)
    if fused:
        from . import decode_ops as ops
        if st.attn_ws is None:
            st.attn_ws = ops.attention_workspace(st.batch, d.heads, st.capacity, st.x.device)
        for i, lw in enumerate(w.layers):
            layer_step_fused(st, lw, st.k_cache[i], st.v_cache[i], d, linear, row_linear,
                             carry=i > 0)
        ops.rmsnorm(st.x, w.final_norm, st.norm, d.eps,
                    branch=st.branch if w.layers else None)
    else:
        for i, lw in enumerate(w.layers):
            layer_step(st, lw, st.k_cache[i], st.v_cache[i], d, linear, row_linear)
        rms_norm(st.x, w.final_norm, d.eps, out=st.norm)
    (head or greedy_head)(st, w.lm_head, linear)
    return st.next_tokens


class GraphDecoder:
    """A decode step captured once in a CUDA graph (reference: Engine.capture_decode,
    engine/engine.py:119-129: side-stream warm-up x3, then capture) and replayed per token."""

    def __init__(self, w: Qwen3Weights, batch: int, capacity: int, linear, device="cuda",
                 make_hooks=None, fused=False, fused_head=False):
        """``make_hooks(state) -> (row_linear, head)`` supplies the tensor-parallel hooks,
        built once per state so their buffers are fixed before capture; ``fused`` selects the
        fused CUDA kernels for the non-linear ops; ``fused_head`` the lm_head + argmax launch
        (no logits are stored, so ``teacher_forced_logits`` needs it off)."""
        self.w, self.linear = w, linear
        self.st = DecodeState(w, batch, capacity, device)
        row_linear, head = make_hooks(self.st) if make_hooks else (None, None)
        if fused_head and head is None:
            head = fused_greedy_head
        # The captured graph holds raw pointers into the buffers these hooks own (partial sums,
        # per-shard maxima, peer buffers), so the hooks live exactly as long as the graph.
        self.hooks = (row_linear, head)
        step = lambda: decode_step(self.st, w, linear, row_linear, head, fused)  # noqa: E731
        stream = torch.cuda.Stream(device=device)
        self.stream = stream
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
        stream.synchronize()
        self.reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            step()
        torch.cuda.current_stream(device).wait_stream(stream)

    def reset(self):
        for c in self.st.k_cache + self.st.v_cache:
            c.zero_()
        self.st.position.zero_()

    def step(self):
        """Replay one step, then advance: next token becomes the input, position += 1."""
        self.graph.replay()
        self.st.tokens.copy_(self.st.next_tokens)
        self.st.position.add_(1)

    def greedy(self, prompt: torch.Tensor, new_tokens: int) -> torch.Tensor:
        """Feed ``prompt`` [B, P] one token per step, then decode ``new_tokens`` greedily.
        Returns the generated tokens [B, new_tokens]."""
        self.reset()
        B, P = prompt.shape
        out = torch.empty(B, new_tokens, dtype=torch.int64, device=prompt.device)
        for i in range(P):
            self.st.tokens.copy_(prompt[:, i])
            self.graph.replay()
            self.st.position.add_(1)
        self.st.tokens.copy_(self.st.next_tokens)
        for j in range(new_tokens):
            out[:, j] = self.st.tokens
            if j + 1 < new_tokens:
                self.step()
        return out

    def teacher_forced_logits(self, prompt: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        """Logits [B, T, V] (fp32) predicting ``tokens[:, t]`` after ``prompt`` and
        ``tokens[:, :t]`` — the replay the reference judge uses (neokernel/judge.py:89-107)."""
        self.reset()
        B, P = prompt.shape
        T = tokens.shape[1]
        logits = torch.empty(B, T, self.st.logits.shape[1], dtype=torch.float32,
                             device=prompt.device)
        seq = torch.cat([prompt, tokens], dim=1)
        for i in range(P + T - 1):
            self.st.tokens.copy_(seq[:, i])
            self.graph.replay()
            if i >= P - 1:
                logits[:, i - P + 1] = self.st.logits.float()
            self.st.position.add_(1)
        return logits
