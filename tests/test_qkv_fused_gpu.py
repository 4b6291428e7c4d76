"""nk_gemm_bf16_qkv_rope_cache (neokernel_b200.decode_ops.qkv_rope_cache): the QKV linear and
its consumer in one launch, against the two launches it replaces — the QKV linear
(``neokernel_b200.mm``, itself checked against the oracle and cuBLAS) and
``nk_qk_norm_rope_cache_bf16`` (checked against its PyTorch restatement, which is pinned to
transformers' Qwen3 modules) — bit for bit: queries, the written key and value rows, and no
other cache row touched. Head layouts of Qwen3-8B and of Qwen3-32B tensor-parallel shards;
decode batches 1..16; positions at both ends of the cache; a position outside the cache writes
nothing and reports NK_ERR_RANGE."""

import pytest
import torch

import neokernel_b200 as nk
from neokernel_b200 import _lib, decode_ops as ops, qwen3

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rand(*shape, std=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=DEV) * std).to(torch.bfloat16)


# (hidden K, query heads, kv heads): Qwen3-8B, Qwen3-32B at TP = 2, 8
LAYOUTS = [(4096, 32, 8), (5120, 32, 4), (5120, 8, 1)]


@pytest.mark.parametrize("K,hq,hkv", LAYOUTS)
@pytest.mark.parametrize("B", (1, 3, 8, 16))
def test_fused_qkv_equals_linear_then_rope_cache(K, hq, hkv, B):
    N = (hq + 2 * hkv) * 128
    cap = 40
    x = rand(B, K, seed=B)
    w = rand(N, K, std=0.02, seed=K + hq)
    qn = rand(128, std=0.25, seed=4) + 1  # non-unit gains
    kn = rand(128, std=0.25, seed=5) + 1
    d = qwen3.Qwen3Dims(K, 4 * K, hq, hkv, 128, 1, 16)
    cos, sin = qwen3.rope_tables(d, cap, DEV)
    for pos in (0, 17, cap - 1):
        position = torch.tensor([pos], device=DEV)
        # two launches: the linear, then the consumer
        qkv = torch.empty(B, N, dtype=torch.bfloat16, device=DEV)
        nk.mm(x, w.t(), out=qkv)
        q1 = torch.empty(B, hq * 128, dtype=torch.bfloat16, device=DEV)
        k1 = rand(B, hkv, cap, 128, seed=7)
        v1 = rand(B, hkv, cap, 128, seed=8)
        ops.qk_norm_rope_cache(qkv, qn, kn, cos, sin, position, q1, k1, v1, hq, hkv, 1e-6)
        # one launch
        q2 = torch.empty_like(q1)
        k2 = rand(B, hkv, cap, 128, seed=7)
        v2 = rand(B, hkv, cap, 128, seed=8)
        ops.qkv_rope_cache(x, w.t(), qn, kn, cos, sin, position, q2, k2, v2, hq, hkv, 1e-6)
        torch.cuda.synchronize()
        assert torch.equal(q1, q2), (pos, (q1.float() - q2.float()).abs().max().item())
        assert torch.equal(k1, k2), pos   # the written row, and every other row untouched
        assert torch.equal(v1, v2), pos
        assert not torch.equal(k2[:, :, pos], rand(B, hkv, cap, 128, seed=7)[:, :, pos])
    assert nk.device_error() == 0


def test_fused_qkv_position_outside_the_cache_writes_nothing():
    K, hq, hkv, B, cap = 4096, 32, 8, 4, 16
    N = (hq + 2 * hkv) * 128
    x = rand(B, K, seed=1)
    w = rand(N, K, std=0.02, seed=2)
    qn = kn = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cos, sin = qwen3.rope_tables(qwen3.Qwen3Dims(K, 4 * K, hq, hkv, 128, 1, 16), cap, DEV)
    q = torch.zeros(B, hq * 128, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(B, hkv, cap, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.zeros_like(k)
    for bad in (cap, -1):
        ops.qkv_rope_cache(x, w.t(), qn, kn, cos, sin, torch.tensor([bad], device=DEV), q, k, v,
                           hq, hkv, 1e-6)
        torch.cuda.synchronize()
        assert nk.device_error() == _lib.NK_ERR_RANGE
        assert not q.any() and not k.any() and not v.any()


def test_fused_qkv_rejects_bad_arguments():
    x = rand(4, 4096, seed=1)
    w = rand(48 * 128, 4096, std=0.02, seed=2)
    qn = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cos = sin = torch.zeros(8, 128, dtype=torch.bfloat16, device=DEV)
    q = torch.empty(4, 32 * 128, dtype=torch.bfloat16, device=DEV)
    k = v = torch.empty(4, 8, 8, 128, dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    with pytest.raises(ValueError):  # 32 + 2 * 7 heads do not make 6144 rows
        ops.qkv_rope_cache(x, w.t(), qn, qn, cos, sin, pos, q, k, v, 32, 7, 1e-6)
    with pytest.raises(ValueError):  # beyond the decode token tile
        ops.qkv_rope_cache(rand(17, 4096), w.t(), qn, qn, cos, sin, pos, q, k, v, 32, 8, 1e-6)
    with pytest.raises(ValueError):  # a forced split-K plan is not the balanced schedule
        ops.qkv_rope_cache(x, w.t(), qn, qn, cos, sin, pos, q, k, v, 32, 8, 1e-6,
                           plan=nk.plan_for(4, 6144, 4096, split_k=4))
