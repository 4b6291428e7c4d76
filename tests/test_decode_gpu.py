"""Decode-step parity: the Qwen3 decode graph with the decode linears on neokernel_b200.mm
against the same graph on torch.mm (the reference's own call, engine/kernels/decode.py:54-66,
engine/engine.py:114), random-init weights, CUDA-graph replay. The torch.mm graph with PyTorch
ops (qwen3.layer_step) is pinned to transformers' Qwen3 modules on the CPU
(tests/test_step_model_cpu.py).

With the decisive random init (qwen3.py) every greedy choice is made by a wide margin, and
the north-star criterion holds as stated: identical greedy tokens over a 128-token decode, for
the linears alone and for the whole product step (fused kernels, fused greedy head).

With the reference test's init (N(0, 0.02) everywhere, unit gains) the logits are nearly flat
(top-2 gaps of a few hundredths among 151,936 entries), so a flip is legitimate where the
reference's own logits were within rounding of a tie: every step where the tokens differ must
pass the reference judge's margin rule (neokernel/judge.py:71-86) — the token we chose scores
within 2.0 of the maximum of the torch.mm path's teacher-forced logits — and in practice within
a few bf16 ulps. Identical-token counts are printed.
"""

import json

import pytest
import torch

import neokernel_b200 as nk
from neokernel_b200 import qwen3

pytestmark = pytest.mark.gpu

MARGIN = 2.0  # neokernel/judge.py MARGIN, used by check_logits (judge.py:71-86)


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def margins(ref_logits, tokens):
    """max(ref) - ref[chosen] per (b, t), as check_logits computes it."""
    best = ref_logits.max(dim=-1).values
    chosen = ref_logits.gather(-1, tokens.unsqueeze(-1)).squeeze(-1)
    return best - chosen


def test_two_layer_step_matches_torch_mm():
    d = qwen3.QWEN3_8B
    w = qwen3.Qwen3Weights(d, seed=3, layers=2)
    B, cap = 4, 64
    ours = qwen3.DecodeState(w, B, cap)
    ref = qwen3.DecodeState(w, B, cap)
    gen = torch.Generator(device="cuda").manual_seed(5)
    for pos in range(6):
        toks = torch.randint(0, d.vocab, (B,), generator=gen, device="cuda")
        for st in (ours, ref):
            st.tokens.copy_(toks)
            st.position.fill_(pos)
        qwen3.decode_step(ours, w, nk.mm)
        qwen3.decode_step(ref, w, torch.mm)
        torch.cuda.synchronize()
        diff = (ours.logits.float() - ref.logits.float()).abs().max().item()
        scale = ref.logits.float().abs().max().item()
        assert diff <= 0.02 * scale, (pos, diff, scale)
        for a, b in zip(ours.k_cache + ours.v_cache, ref.k_cache + ref.v_cache):
            assert (a.float() - b.float()).abs().max().item() <= 0.05


@pytest.mark.parametrize("batch", (1, 4))
def test_qwen3_8b_128_identical_greedy_tokens(batch):
    """Decisive init: 128 identical greedy tokens per sequence on the reference's step (torch.mm,
    PyTorch ops), on it with neokernel_b200.mm as the five linears, and on the product step
    (fused decode kernels, neokernel_b200.mm, fused greedy head)."""
    d = qwen3.QWEN3_8B
    w = qwen3.Qwen3Weights(d, seed=11, init="decisive")
    prompt_len, new = 8, 128
    cap = prompt_len + new
    gen = torch.Generator(device="cuda").manual_seed(20260922)
    prompt = torch.randint(0, d.vocab, (batch, prompt_len), generator=gen, device="cuda")
    ref = qwen3.GraphDecoder(w, batch, cap, torch.mm)
    t_ref = ref.greedy(prompt, new)
    lr = ref.teacher_forced_logits(prompt, t_ref)
    top2 = lr.topk(2, dim=-1).values
    gap = (top2[..., 0] - top2[..., 1]).flatten()
    report = {"test": f"qwen3-8b/decisive/B{batch}", "tokens": batch * new,
              "distinct_tokens": int(t_ref.unique().numel()),
              "top2_margin": {"min": float(gap.min()), "p1": float(gap.quantile(0.01)),
                              "median": float(gap.median()), "max": float(gap.max())}}
    ours = qwen3.GraphDecoder(w, batch, cap, nk.mm)
    t_ours = ours.greedy(prompt, new)
    lo = ours.teacher_forced_logits(prompt, t_ref)
    report["linears_identical_tokens"] = int((t_ours == t_ref).sum())
    report["linears_teacher_forced_max_logit_diff"] = float((lo - lr).abs().max())
    del ours
    prod = qwen3.GraphDecoder(w, batch, cap, nk.mm, fused=True, fused_head=True)
    t_prod = prod.greedy(prompt, new)
    report["product_identical_tokens"] = int((t_prod == t_ref).sum())
    print(json.dumps(report), flush=True)
    assert torch.equal(t_ours, t_ref), report
    assert torch.equal(t_prod, t_ref), report
    assert report["distinct_tokens"] > new // 2, report  # a walk through the vocabulary
    # the margins the init is chosen for: far above the logit noise of either path
    assert report["top2_margin"]["min"] > 8 * max(report["linears_teacher_forced_max_logit_diff"],
                                                  0.125), report
    del ref, prod
    torch.cuda.empty_cache()


@pytest.mark.parametrize("batch", (1, 4))
def test_qwen3_8b_reference_init_flips_only_at_near_ties(batch):
    d = qwen3.QWEN3_8B
    w = qwen3.Qwen3Weights(d, seed=11, init="reference")
    prompt_len, new = 8, 128
    cap = prompt_len + new
    gen = torch.Generator(device="cuda").manual_seed(20260922)
    prompt = torch.randint(0, d.vocab, (batch, prompt_len), generator=gen, device="cuda")

    ours = qwen3.GraphDecoder(w, batch, cap, nk.mm)
    ref = qwen3.GraphDecoder(w, batch, cap, torch.mm)
    # Control: another valid fp32-accumulating GEMM (cuBLAS fp32 on the same bf16 values,
    # rounded once) — shows how soon any change of summation order flips a near-tie.
    ctrl = qwen3.GraphDecoder(w, batch, cap,
                              lambda a, b, out: out.copy_(torch.mm(a.float(), b.float())))
    t_ours = ours.greedy(prompt, new)
    t_ref = ref.greedy(prompt, new)
    t_ctrl = ctrl.greedy(prompt, new)
    torch.cuda.synchronize()
    same = (t_ours == t_ref)

    def first_divergence(a, b):
        eq = a == b
        return [int(eq[i].logical_not().nonzero()[0]) if not eq[i].all() else None
                for i in range(a.shape[0])]

    # Teacher-forced replay of our tokens on the reference path (neokernel/judge.py:89-107).
    ref_logits = ref.teacher_forced_logits(prompt, t_ours)
    m = margins(ref_logits, t_ours)
    first_diff = first_divergence(t_ours, t_ref)
    # Teacher-forced on the reference's own trajectory: per-step argmax agreement with the
    # reference, for our kernels and for the control GEMM.
    lo = ours.teacher_forced_logits(prompt, t_ref)
    lr = ref.teacher_forced_logits(prompt, t_ref)
    lc = ctrl.teacher_forced_logits(prompt, t_ref)
    agree = (lo.argmax(-1) == lr.argmax(-1)).float().mean().item()
    agree_ctrl = (lc.argmax(-1) == lr.argmax(-1)).float().mean().item()
    report = {"test": f"qwen3-8b/reference-init/B{batch}", "identical_tokens": int(same.sum()),
              "tokens": batch * new, "first_divergence": first_diff,
              "control_first_divergence": first_divergence(t_ctrl, t_ref),
              "teacher_forced_argmax_agreement": agree,
              "control_teacher_forced_argmax_agreement": agree_ctrl,
              "teacher_forced_max_logit_diff": float((lo - lr).abs().max()),
              "control_teacher_forced_max_logit_diff": float((lc - lr).abs().max()),
              "worst_margin": float(m.max()), "mean_margin": float(m.mean())}
    print(json.dumps(report), flush=True)
    # Our kernels agree with the reference's own GEMM as well as another valid
    # fp32-accumulating GEMM does (a few percent of slack for the 128-sample noise).
    assert agree >= agree_ctrl - 0.05, report
    assert float((lo - lr).abs().max()) <= 2 * float((lc - lr).abs().max()) + 0.0625, report
    assert torch.isfinite(ref_logits).all()
    assert float(m.max()) <= MARGIN, report
    # Up to its first divergence a sequence has seen identical inputs on both paths, so the
    # token that differs there must be a near-tie of the reference's own logits: within the
    # logit noise another valid fp32-accumulating GEMM shows on the same inputs (the control's
    # teacher-forced max logit difference), and never beyond 8 bf16 ulps at |logit| < 8.
    tie_bound = min(max(0.125, float((lc - lr).abs().max())), 0.25)
    for b in range(batch):
        if first_diff[b] is not None:
            assert float(m[b, first_diff[b]]) <= tie_bound, report
    del ours, ref, ctrl
    torch.cuda.empty_cache()
