"""Pins the oracle (oracle/nk_oracle.c) before it is trusted as the checker.

The reference's decode linear is ``torch.mm(x, W.t(), out=y)`` on bf16 tensors
(engine/kernels/decode.py:54,58,64,66; engine/engine.py:114). The golden vectors in
tests/golden/ were produced by that exact call on the reference's own weight packing
(engine/kernels/weights.py:6-29), see tests/golden/make_golden.py.
"""

import os

import numpy as np
import pytest
import torch

from neokernel_b200 import synthetic
from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SITES = ("qkv", "o", "gate_up", "down", "lm_head")


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def pin_bound(a, b, K):
    """Per-element agreement bound between two fp32-accumulating bf16 GEMMs that differ only
    in summation order: one bf16 ulp at the larger magnitude (a rounding boundary between
    the two fp32 sums) plus the fp32 re-association error ~ 2^-22 * sqrt(K)."""
    fa, fb = oracle.bf16_to_f32(a), oracle.bf16_to_f32(b)
    mag = np.maximum(np.abs(fa), np.abs(fb)).astype(np.float32)
    ulp = np.spacing(mag) * 65536.0  # bf16 ulp = fp32 ulp << 16
    return np.abs(fa - fb) <= ulp + 2.0 ** -22 * np.sqrt(K)


def test_bf16_rounding_known_answers():
    specials = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan,
                         1.00390625,        # exactly halfway 1 and 1+2^-7: tie -> even (1.0)
                         1.01171875,        # halfway 1+2^-7 and 1+2^-6: tie -> even (1+2^-6)
                         3.4e38, -3.4e38,   # rounds past bf16 max -> inf
                         1e-40, -1e-40,     # fp32 subnormals
                         2.0 ** -133, 65504.0, 0.1, -0.3], dtype=np.float32)
    rng = np.random.default_rng(0)
    vals = np.concatenate([specials, rng.standard_normal(10000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 10000)]).astype(np.float32)
    ours = oracle.f32_to_bf16(vals)
    ref = bits(torch.from_numpy(vals).to(torch.bfloat16))
    nan = np.isnan(vals)
    assert np.array_equal(ours[~nan], ref[~nan])
    assert np.all((ours[nan] & 0x7f80) == 0x7f80) and np.all(ours[nan] & 0x7f)
    assert ours[7] == 0x3f80 and ours[8] == 0x3f82


def test_bf16_widen_is_exact():
    h = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    f = oracle.bf16_to_f32(h)
    t = torch.from_numpy(h.view(np.int16)).view(torch.bfloat16).float().numpy()
    finite = np.isfinite(t)
    assert np.array_equal(f[finite], t[finite])


@pytest.mark.parametrize("site", SITES)
@pytest.mark.parametrize("M", (1, 3, 16))
def test_oracle_matches_reference_golden_tiny_layer(site, M):
    g = np.load(os.path.join(GOLDEN, "tiny_layer.npz"))
    w, x, y = g[f"{site}/w"], g[f"{site}/m{M}/x"], g[f"{site}/m{M}/y"]
    ours = oracle.gemm_bf16(x, w)
    exact = np.mean(ours == y)
    assert exact >= 0.999, exact
    assert pin_bound(ours, y, w.shape[1]).all()


def _decode_cases():
    g = np.load(os.path.join(GOLDEN, "decode_shapes.npz"))
    return sorted({k.split("/")[0] for k in g.files})


@pytest.mark.parametrize("name", _decode_cases())
def test_oracle_matches_reference_golden_decode_shapes(name):
    import hashlib
    g = np.load(os.path.join(GOLDEN, "decode_shapes.npz"))
    M, K, N, ws, xs = (int(v) for v in g[f"{name}/meta"])
    W = synthetic.weight(N, K, ws)
    x = synthetic.activation(M, K, xs)
    # the regenerated inputs are the ones the golden outputs were computed from
    assert hashlib.sha256(bits(W).tobytes()).hexdigest() == str(g[f"{name}/sha_w"])
    assert hashlib.sha256(bits(x).tobytes()).hexdigest() == str(g[f"{name}/sha_x"])
    y = g[f"{name}/y"]
    ours = oracle.gemm_bf16(bits(x), bits(W))
    assert np.mean(ours == y) >= 0.999
    assert pin_bound(ours, y, K).all()
    # and the golden itself meets the north-star tolerance against exact arithmetic
    ref = oracle.gemm_f64(bits(x), bits(W))
    assert np.abs(oracle.bf16_to_f32(y) - ref).max() <= oracle.tolerance(K)


def test_oracle_planted_error_is_caught():
    """A mistake planted in the oracle's output (on the CPU) must fail the pin."""
    g = np.load(os.path.join(GOLDEN, "tiny_layer.npz"))
    w, x, y = g["down/w"], g["down/m16/x"], g["down/m16/y"]
    ours = oracle.gemm_bf16(x, w).copy()
    ours[3, 5] ^= 0x0004  # flip a low mantissa bit: 4 ulps off
    assert not pin_bound(ours, y, w.shape[1]).all()


def test_oracle_zero_and_identity():
    K = 64
    x = oracle.f32_to_bf16(np.eye(K, dtype=np.float32)[:5])
    w = oracle.f32_to_bf16(np.arange(K * 7, dtype=np.float32).reshape(7, K) / 64.0)
    y = oracle.gemm_bf16(x, w)
    assert np.array_equal(oracle.bf16_to_f32(y), oracle.bf16_to_f32(w)[:, :5].T)
    z = oracle.gemm_bf16(np.zeros((2, K), np.uint16), w)
    assert not z.any()
