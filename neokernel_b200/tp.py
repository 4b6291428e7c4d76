"""Tensor-parallel decode for the Qwen3 shapes (one process per GPU, torch.distributed).

The reference engine is single-GPU (engine/engine.py:65,79,84 hard-code ``cuda:0``); this mode
shards the decode linears where their weights shard naturally:

* QKV (engine/kernels/decode.py:54) is split by output column, whole heads per rank: rank r
  holds query heads [r*Hq/T, (r+1)*Hq/T) and KV heads [r*Hkv/T, (r+1)*Hkv/T), so grouped
  attention runs on local heads with no exchange;
* gate_up (decode.py:64) is split by output column with the gate and up slices paired, so
  bf16(silu(gate)) * up is local;
* o_proj (decode.py:58) and down (decode.py:66) are split along K: each rank computes an
  unrounded fp32 partial, the partials are summed across ranks and the sum is rounded to bf16
  once — the single-GPU rounding. On GPUs the product fuses the linear with that sum
  (``nk_gemm_bf16_allreduce``, neokernel_b200/peer.py): one launch per rank whose output tiles
  go straight into every rank's buffer over NVLink and are added up in rank order there.
  ``collective="peer"`` keeps the two launches (``mm_f32``, then ``nk_allreduce_bf16``),
  ``collective="nccl"`` uses NCCL's all-reduce (as CPU process groups always do);
* lm_head (engine.py:114) is split by vocabulary row: each rank takes its local max and its
  lowest index — on GPUs in the lm_head launch itself (``mm_argmax``, the fused greedy head),
  so the [B, vocab / T] logits are not stored — and an all-gather of (value, index) picks the
  global maximum, ties to the lowest vocabulary index as torch.argmax does (engine.py:116).

Embedding and norms are replicated. Every rank issues the same collectives in the same order
in warm-up, capture and replay. The weights of a rank are the slices of exactly the matrices
``qwen3.Qwen3Weights`` draws for the same seed, so a tensor-parallel run and a single-GPU run
of the same seed use the same model.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import qwen3
from .qwen3 import Qwen3Dims


def local_dims(d: Qwen3Dims, world: int) -> Qwen3Dims:
    """The per-rank shapes of a ``world``-way split."""
    for what, n in (("heads", d.heads), ("kv_heads", d.kv_heads),
                    ("intermediate", d.intermediate), ("vocab", d.vocab)):
        if n % world:
            raise ValueError(f"tensor parallel size {world} does not divide {what}={n}")
    return Qwen3Dims(d.hidden, d.intermediate // world, d.heads // world, d.kv_heads // world,
                     d.head_dim, d.layers, d.vocab // world, d.eps, d.rope_theta,
                     d.tie_embeddings)


class TPLayerWeights:
    """Rank r's slices of one layer, in the same packed layout as the full layer."""

    def __init__(self, full: qwen3.LayerWeights, d: Qwen3Dims, rank: int, world: int):
        D = d.head_dim
        hq, hkv = d.heads // world, d.kv_heads // world
        I = d.intermediate
        il = I // world
        q = full.qkv_weight[rank * hq * D:(rank + 1) * hq * D]
        k0 = d.q_width
        k = full.qkv_weight[k0 + rank * hkv * D:k0 + (rank + 1) * hkv * D]
        v0 = d.q_width + d.kv_width
        v = full.qkv_weight[v0 + rank * hkv * D:v0 + (rank + 1) * hkv * D]
        self.qkv_weight = torch.cat((q, k, v)).contiguous()
        self.o_weight = full.o_weight[:, rank * hq * D:(rank + 1) * hq * D].contiguous()
        g = full.gate_up_weight[rank * il:(rank + 1) * il]
        u = full.gate_up_weight[I + rank * il:I + (rank + 1) * il]
        self.gate_up_weight = torch.cat((g, u)).contiguous()
        self.down_weight = full.down_weight[:, rank * il:(rank + 1) * il].contiguous()
        self.qkv = self.qkv_weight.t()
        self.o = self.o_weight.t()
        self.gate_up = self.gate_up_weight.t()
        self.down = self.down_weight.t()
        self.input_norm, self.post_norm = full.input_norm, full.post_norm
        self.q_norm, self.k_norm = full.q_norm, full.k_norm


class TPWeights:
    """Rank r's shard of the random-init model ``qwen3.Qwen3Weights(d, seed)``: each full
    matrix is drawn in the same order with the same generator (one layer at a time, so a rank
    never holds more than one full layer), sliced, and the full copy released."""

    def __init__(self, d: Qwen3Dims, seed: int, rank: int, world: int, device="cuda",
                 layers: int | None = None, init: str = "decisive"):
        self.full_dims = d
        self.dims = local_dims(d, world)
        self.rank, self.world, self.init = rank, world, init
        gen = torch.Generator(device=device).manual_seed(seed)
        self.embed = qwen3.draw_embedding(d, gen, device, init)
        n = d.layers if layers is None else layers
        self.layers = []
        for _ in range(n):
            full = qwen3.LayerWeights(d, gen, device, init)
            self.layers.append(TPLayerWeights(full, d, rank, world))
            del full
        self.final_norm, head = qwen3.draw_head(d, self.embed, gen, device, init)
        vl = d.vocab // world
        self.lm_head_weight = head[rank * vl:(rank + 1) * vl].contiguous()
        self.lm_head = self.lm_head_weight.t()
        self.vocab_offset = rank * vl


# Batches up to which "auto" fuses the K-split linears with their all-reduce. Measured on
# B200, Qwen3-32B TP=2 (ms per step, fused / unfused peer pair / NCCL): B=1 8.95 / 8.92 / 8.94,
# B=8 9.89 / 9.94 / 9.88, B=32 14.52 / 13.10 / 12.93 — at 32 tokens each tile's finishing CTA
# moves 32 columns to every rank in its own critical path, so NCCL's pipelined all-reduce wins.
FUSED_MAX_M = 8


def make_hooks(w: TPWeights, group=None, linear_f32=None, linear=None, collective="auto",
               fused_head: bool = True):
    """Return ``make(state) -> (row_linear, head)`` for ``qwen3.GraphDecoder`` / ``decode_step``.

    ``linear_f32(a, b, out)`` computes an unrounded fp32 partial (default:
    ``neokernel_b200.mm_f32``); ``linear(a, b, out)`` the bf16 lm_head shard (default:
    ``neokernel_b200.mm``). ``collective`` sums the partials of the K-split linears: "fused"
    (the linear and the sum in one launch, ``PeerGroup.mm_allreduce``), "peer" (``mm_f32`` then
    ``nk_allreduce_bf16`` over NVLink peer memory), "nccl" (``mm_f32``, ``dist.all_reduce``,
    then the bf16 copy) or "auto": fused on a CUDA process group of 2+ ranks for batches of up
    to ``FUSED_MAX_M``, else all_reduce. ``fused_head`` (CUDA states only)
    takes each rank's (max, lowest index) from the lm_head launch (``neokernel_b200.mm_argmax``)
    instead of storing the logits and reducing them; ``state.logits`` is then left untouched.
    Buffers are allocated here, once per state, so the hooks are capture-safe.
    """
    if collective not in ("auto", "fused", "peer", "nccl"):
        raise ValueError(f"collective must be auto, fused, peer or nccl, not {collective!r}")
    if linear_f32 is None or linear is None:
        import neokernel_b200 as nk
        linear_f32 = linear_f32 or nk.mm_f32
        linear = linear or nk.mm
    world, vocab_offset = w.world, w.vocab_offset

    def make(st: qwen3.DecodeState):
        B, H = st.batch, w.dims.hidden
        dev = st.x.device
        gpu_group = world > 1 and dev.type == "cuda" and dist.get_backend(group) == "nccl"
        use_fused = world > 1 and (collective == "fused" or (
            collective == "auto" and gpu_group and B <= FUSED_MAX_M))
        use_peer = not use_fused and world > 1 and collective == "peer"
        peer = None
        if use_fused or use_peer:
            from .peer import PeerGroup
            peer = PeerGroup(B * H, group=group, device=dev)
        partial = torch.empty(B, H, device=dev, dtype=torch.float32)
        use_fused_head = fused_head and dev.type == "cuda"
        best_bf16 = torch.empty(B, device=dev, dtype=torch.bfloat16)
        best = torch.empty(B, device=dev, dtype=torch.float32)
        best_idx = torch.empty(B, device=dev, dtype=torch.int64)
        all_best = torch.empty(world * B, device=dev, dtype=torch.float32)
        all_idx = torch.empty(world * B, device=dev, dtype=torch.int64)

        def row_linear(a, b, out):
            if use_fused:  # the K-slice linear and the rank-order sum in one launch
                peer.mm_allreduce(a, b, out=out)
                return
            linear_f32(a, b, out=partial)
            if peer is not None:
                peer.allreduce_bf16(partial, out)  # rank-order sum, one rounding to bf16
                return
            if world > 1:
                dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
            out.copy_(partial)  # the one rounding to bf16 (nearest-even)

        def head(state, lm_head, _linear):
            if use_fused_head:
                from .gemm import mm_argmax
                # this shard's lowest-index maximum, from the lm_head launch itself
                mm_argmax(state.norm, lm_head, idx=best_idx, best=best_bf16)
                best.copy_(best_bf16)  # exact: every bf16 value is an fp32 value
            else:
                linear(state.norm, lm_head, out=state.logits)
                torch.max(state.logits.float(), dim=-1, out=(best, best_idx))  # first max index
            best_idx.add_(vocab_offset)
            if world > 1:
                dist.all_gather_into_tensor(all_best, best, group=group)
                dist.all_gather_into_tensor(all_idx, best_idx, group=group)
                r = torch.argmax(all_best.view(world, B), dim=0)  # lowest rank among maxima
                torch.gather(all_idx.view(world, B), 0, r.view(1, B), out=state.next_tokens.view(1, B))
            else:
                state.next_tokens.copy_(best_idx)

        return row_linear, head

    return make
