"""Fused decode kernels (include/nk_decode.h) against the PyTorch formulation of the same ops
in neokernel_b200.qwen3 (the reference's cast points). Cases follow the reference's kernel
tests (tests/test_hand_rolled_kernels.py:75-145): norm with and without the residual, q/k
norm + RoPE + cache write for both cache layouts and several positions, attention against an
fp32 softmax with inactive slots poisoned by NaN, SiLU·up.

Element-wise agreement is exact except where an fp32 reduction (sum of squares, softmax)
is ordered differently, which moves a value across a bf16 rounding boundary: we require
>= 99 % bit-identical elements and every element within one bf16 ulp (2^-7 relative) plus a
small absolute slack.
"""

import math

import pytest
import torch

from neokernel_b200 import decode_ops as ops
from neokernel_b200 import qwen3

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rand(*shape, std=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=DEV) * std).to(torch.bfloat16)


def close(a, b, abs_slack=1e-3, exact_frac=0.99):
    a, b = a.float(), b.float()
    ok = (a - b).abs() <= b.abs() * 2.0 ** -7 + abs_slack
    assert ok.all(), f"{(~ok).sum().item()} elements off, max diff {(a - b).abs().max().item()}"
    assert (a == b).float().mean().item() >= exact_frac


@pytest.mark.parametrize("rows", (1, 4, 16, 32))
@pytest.mark.parametrize("width", (8, 1024, 2560, 4096, 5120))
@pytest.mark.parametrize("residual", (False, True))
def test_rmsnorm(rows, width, residual):
    x = rand(rows, width, seed=1)
    b = rand(rows, width, seed=2)
    w = rand(width, seed=3)
    out = torch.empty_like(x)
    ref_x = (x + b) if residual else x.clone()
    ref = qwen3.rms_norm(ref_x, w, 1e-6)
    ops.rmsnorm(x, w, out, 1e-6, branch=b if residual else None)
    torch.cuda.synchronize()
    assert torch.equal(x, ref_x)          # the residual sum is stored exactly as bf16(x + b)
    close(out, ref, exact_frac=0.99 if width > 8 else 0.8)


def _torch_qk(qkv, qn, kn, cos, sin, pos, H, Hkv, eps):
    B = qkv.shape[0]
    D = 128
    q = qkv[:, :H * D].view(B, H, D)
    k = qkv[:, H * D:(H + Hkv) * D].view(B, Hkv, D)
    v = qkv[:, (H + Hkv) * D:].view(B, Hkv, D)
    q = qwen3.rms_norm(q, qn, eps)
    k = qwen3.rms_norm(k, kn, eps)
    c, s = cos[pos].view(1, 1, D), sin[pos].view(1, 1, D)
    q = (q * c) + (qwen3.rotate_half(q) * s)
    k = (k * c) + (qwen3.rotate_half(k) * s)
    return q.reshape(B, H * D), k, v


@pytest.mark.parametrize("B", (1, 4))
@pytest.mark.parametrize("H,Hkv", [(32, 8), (64, 8), (16, 8), (4, 1)])
@pytest.mark.parametrize("layout", ("bhsd", "bshd"))
def test_qk_norm_rope_cache(B, H, Hkv, layout):
    cap = 130
    d = qwen3.Qwen3Dims(1024, 1024, H, Hkv, 128, 1, 64)
    cos, sin = qwen3.rope_tables(d, cap, DEV)
    qn, kn = rand(128, seed=4), rand(128, seed=5)
    for pos in (0, 5, 63, 64, cap - 1):
        qkv = rand(B, (H + 2 * Hkv) * 128, seed=pos)
        if layout == "bhsd":
            kc = torch.zeros(B, Hkv, cap, 128, dtype=torch.bfloat16, device=DEV)
            vc = torch.zeros_like(kc)
        else:  # [B, S, Hkv, D] storage seen as [B, Hkv, S, D] (engine/kernels/decode.py:71-77)
            kc = torch.zeros(B, cap, Hkv, 128, dtype=torch.bfloat16, device=DEV).transpose(1, 2)
            vc = torch.zeros(B, cap, Hkv, 128, dtype=torch.bfloat16, device=DEV).transpose(1, 2)
        q_out = torch.empty(B, H * 128, dtype=torch.bfloat16, device=DEV)
        position = torch.tensor([pos], device=DEV)
        ops.qk_norm_rope_cache(qkv, qn, kn, cos, sin, position, q_out, kc, vc, H, Hkv, 1e-6)
        torch.cuda.synchronize()
        q_ref, k_ref, v_ref = _torch_qk(qkv, qn, kn, cos, sin, pos, H, Hkv, 1e-6)
        close(q_out, q_ref, abs_slack=2e-3)
        close(kc[:, :, pos], k_ref, abs_slack=2e-3)
        assert torch.equal(vc[:, :, pos], v_ref)
        others = torch.ones(cap, dtype=torch.bool, device=DEV)
        others[pos] = False
        assert kc[:, :, others].count_nonzero().item() == 0
        assert vc[:, :, others].count_nonzero().item() == 0


@pytest.mark.parametrize("B", (1, 3))
@pytest.mark.parametrize("H,Hkv", [(32, 8), (64, 8), (8, 8), (16, 8)])
@pytest.mark.parametrize("cap", (64, 100, 1088))
def test_attention_decode(B, H, Hkv, cap):
    d = qwen3.Qwen3Dims(1024, 1024, H, Hkv, 128, 1, 64)
    kc = rand(B, Hkv, cap, 128, seed=7)
    vc = rand(B, Hkv, cap, 128, seed=8)
    ws = ops.attention_workspace(B, H, cap, DEV)
    slots = torch.arange(cap, device=DEV)
    for pos in sorted({0, 1, 63, min(64, cap - 1), cap // 2, cap - 1}):
        q = rand(B, H * 128, seed=100 + pos)
        position = torch.tensor([pos], device=DEV)
        out = torch.empty_like(q)
        ops.attention_decode(q, kc, vc, position, out, ws, H, Hkv)
        torch.cuda.synchronize()
        ref = qwen3.attention(q.view(B, H, 128), kc, vc, position, slots, d)
        close(out, ref, abs_slack=4e-3, exact_frac=0.97)
        # masked capacity has no influence: poison the inactive slots (attention.py test)
        if pos + 1 < cap:
            kp, vp = kc.clone(), vc.clone()
            kp[:, :, pos + 1:] = float("nan")
            vp[:, :, pos + 1:] = float("nan")
            out2 = torch.empty_like(q)
            ops.attention_decode(q, kp, vp, position, out2, ws, H, Hkv)
            torch.cuda.synchronize()
            assert torch.isfinite(out2.float()).all()
            assert torch.equal(out2, out)


@pytest.mark.parametrize("B,H,Hkv,cap", [(16, 32, 8, 1088), (32, 64, 8, 300), (8, 32, 8, 4160),
                                         (40, 16, 8, 200)])
def test_attention_decode_several_chunks_per_split(B, H, Hkv, cap):
    """With many (sequence, kv head) pairs each split walks several chunks with the next one's
    copies in flight (at 40 x 8 pairs every split covers the whole cache); positions where
    the chunks divide unevenly over the splits, or number fewer than the splits."""
    d = qwen3.Qwen3Dims(1024, 1024, H, Hkv, 128, 1, 64)
    kc = rand(B, Hkv, cap, 128, seed=17)
    vc = rand(B, Hkv, cap, 128, seed=18)
    ws = ops.attention_workspace(B, H, cap, DEV)
    slots = torch.arange(cap, device=DEV)
    for pos in sorted({0, 65, 190, cap // 2 + 3, cap - 1}):
        q = rand(B, H * 128, seed=300 + pos)
        position = torch.tensor([pos], device=DEV)
        out = torch.empty_like(q)
        ops.attention_decode(q, kc, vc, position, out, ws, H, Hkv)
        torch.cuda.synchronize()
        ref = qwen3.attention(q.view(B, H, 128), kc, vc, position, slots, d)
        close(out, ref, abs_slack=4e-3, exact_frac=0.97)
        if pos + 1 < cap:
            kp, vp = kc.clone(), vc.clone()
            kp[:, :, pos + 1:] = float("nan")
            vp[:, :, pos + 1:] = float("nan")
            out2 = torch.empty_like(q)
            ops.attention_decode(q, kp, vp, position, out2, ws, H, Hkv)
            torch.cuda.synchronize()
            assert torch.equal(out2, out)


@pytest.mark.parametrize("H,Hkv", [(32, 8), (8, 1)])
def test_attention_decode_8_byte_aligned_cache(H, Hkv):
    """Caches whose rows are only 8-byte aligned (row pitch 132 elements, base offset 4)
    take the 8-byte copy path and give the same result as a packed copy."""
    B, cap = 2, 150
    d = qwen3.Qwen3Dims(1024, 1024, H, Hkv, 128, 1, 64)
    kst = rand(B, Hkv, cap, 132, seed=11)
    vst = rand(B, Hkv, cap, 132, seed=12)
    kc, vc = kst[..., 4:], vst[..., 4:]
    assert kc.data_ptr() % 16 == 8 and kc.stride(2) == 132
    kp, vp = kc.contiguous(), vc.contiguous()
    ws = ops.attention_workspace(B, H, cap, DEV)
    slots = torch.arange(cap, device=DEV)
    for pos in (0, 70, cap - 1):
        q = rand(B, H * 128, seed=200 + pos)
        position = torch.tensor([pos], device=DEV)
        out, out_p = torch.empty_like(q), torch.empty_like(q)
        ops.attention_decode(q, kc, vc, position, out, ws, H, Hkv)
        ops.attention_decode(q, kp, vp, position, out_p, ws, H, Hkv)
        torch.cuda.synchronize()
        assert torch.equal(out, out_p)
        ref = qwen3.attention(q.view(B, H, 128), kp, vp, position, slots, d)
        close(out, ref, abs_slack=4e-3, exact_frac=0.97)


def test_attention_decode_position_clamped_to_capacity():
    """A position past the cache attends over the whole cache, reading nothing beyond it, and
    is reported; a negative one writes nothing."""
    import neokernel_b200 as nk
    from neokernel_b200 import _lib
    assert nk.device_error() == 0
    B, H, Hkv, cap = 2, 32, 8, 100
    kc = rand(B, Hkv, cap, 128, seed=13)
    vc = rand(B, Hkv, cap, 128, seed=14)
    ws = ops.attention_workspace(B, H, cap, DEV)
    q = rand(B, H * 128, seed=15)
    a, b = torch.empty_like(q), torch.empty_like(q)
    ops.attention_decode(q, kc, vc, torch.tensor([cap - 1], device=DEV), a, ws, H, Hkv)
    assert nk.device_error() == 0
    ops.attention_decode(q, kc, vc, torch.tensor([cap + 37], device=DEV), b, ws, H, Hkv)
    assert nk.device_error() == _lib.NK_ERR_RANGE
    assert torch.equal(a, b)
    c = torch.full_like(q, 7.0)
    ops.attention_decode(q, kc, vc, torch.tensor([-1], device=DEV), c, ws, H, Hkv)
    assert nk.device_error() == _lib.NK_ERR_RANGE
    assert (c.float() == 7.0).all()


@pytest.mark.parametrize("pos_off", (0, 5))
def test_qk_norm_rope_cache_position_outside_cache(pos_off):
    """A position at or past the capacity (or negative) writes nothing and is reported."""
    import neokernel_b200 as nk
    from neokernel_b200 import _lib
    B, H, Hkv, cap = 2, 32, 8, 40
    d = qwen3.Qwen3Dims(1024, 1024, H, Hkv, 128, 1, 64)
    cos, sin = qwen3.rope_tables(d, cap, DEV)
    qn, kn = rand(128, seed=4), rand(128, seed=5)
    qkv = rand(B, (H + 2 * Hkv) * 128, seed=6)
    kc = torch.zeros(B, Hkv, cap, 128, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q_out = torch.full((B, H * 128), 3.0, dtype=torch.bfloat16, device=DEV)
    for pos in (cap + pos_off, -1 - pos_off):
        ops.qk_norm_rope_cache(qkv, qn, kn, cos, sin, torch.tensor([pos], device=DEV), q_out,
                               kc, vc, H, Hkv, 1e-6)
        assert nk.device_error() == _lib.NK_ERR_RANGE
    assert kc.count_nonzero().item() == 0 and vc.count_nonzero().item() == 0
    assert (q_out.float() == 3.0).all()


@pytest.mark.parametrize("rows", (1, 16))
@pytest.mark.parametrize("I", (8, 3072, 12288))
def test_silu_mul(rows, I):
    gu = rand(rows, 2 * I, std=3.0, seed=9)
    out = torch.empty(rows, I, dtype=torch.bfloat16, device=DEV)
    ops.silu_mul(gu, out)
    torch.cuda.synchronize()
    g = gu[:, :I].float()
    act = (g / (1.0 + torch.exp(-g))).to(torch.bfloat16)
    ref = act * gu[:, I:]
    close(out, ref, exact_frac=0.99 if I > 8 else 0.8)


def test_fused_step_matches_unfused_step():
    import neokernel_b200 as nk
    d = qwen3.QWEN3_8B
    w = qwen3.Qwen3Weights(d, seed=3, layers=2)
    B, cap = 4, 80
    a = qwen3.DecodeState(w, B, cap)
    b = qwen3.DecodeState(w, B, cap)
    gen = torch.Generator(device=DEV).manual_seed(5)
    for pos in range(6):
        toks = torch.randint(0, d.vocab, (B,), generator=gen, device=DEV)
        for st in (a, b):
            st.tokens.copy_(toks)
            st.position.fill_(pos)
        qwen3.decode_step(a, w, nk.mm, fused=True)
        qwen3.decode_step(b, w, nk.mm, fused=False)
        torch.cuda.synchronize()
        scale = b.logits.float().abs().max().item()
        assert (a.logits.float() - b.logits.float()).abs().max().item() <= 0.02 * scale
        # with the deferred residual the fused state holds x before the last down output;
        # the final norm added it, so the final normalised rows agree
        assert (a.norm.float() - b.norm.float()).abs().max().item() <= 0.05

