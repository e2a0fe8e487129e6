"""Kimi K3 latent MoE (row a14: kimi_k3::moe::latent_moe, src/kimi_k3/moe.rs:64-116).

CPU: the oracle restatement against an independent float64 composition of the same steps (the
shape of the reference's own latent_moe tests, which check latent_moe against a naive
re-derivation), and its Situ / RMSNorm pieces against their formulas.
GPU: rmoe_latent_moe against the oracle -- routing ids bit-exact, output within the north star's
1e-2 relative L2 -- at a small size and at the real K3 checkpoint's shapes."""
import math

import numpy as np
import pytest

from helpers import build_layer, oracle_latent, x_device
from oracle import oracle as orc
from rabbit_b200 import synth
from refvec import rel_l2

OUT_RTOL = 1e-2


def _situ64(g, u, beta, lb):
    g = g.astype(np.float64)
    u = u.astype(np.float64)
    if lb is not None:
        u = lb * np.tanh(u / lb)
    return beta * np.tanh(g / beta) / (1.0 + np.exp(-g)) * u


def test_situ_matches_formula():
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(4096) * 6).astype(np.float32)
    u = (rng.standard_normal(4096) * 40).astype(np.float32)
    for lb in (25.0, None):
        got = orc.act_mul(g, u, ("situ", 4.0, lb))
        want = _situ64(g, u, 4.0, lb)
        assert np.max(np.abs(got - want) / (np.abs(want) + 1e-3)) < 1e-5


def test_rmsnorm_rows_matches_formula():
    rng = np.random.default_rng(4)
    v = rng.standard_normal((3, 3584)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(3584)).astype(np.float32)
    got = orc.rmsnorm_rows(v, w, 1e-5)
    v64 = v.astype(np.float64)
    want = v64 / np.sqrt(np.mean(v64 ** 2, axis=1, keepdims=True) + 1e-5) * w
    assert rel_l2(got, want) < 1e-6


def _dense(data, bs, rows, cols):
    return np.stack([orc.row_f32_mxfp4(data, bs, cols, r) for r in range(rows)]).astype(np.float64)


def test_oracle_latent_matches_naive_float64():
    """Route, project down, every expert as a dense float64 matmul on the dequantized weights,
    SituAndMul, weighted sum, RMSNorm, project up -- against the oracle's f32 restatement."""
    cfg = synth.CONFIGS["c5_tiny_latent"]
    x = synth.activations(cfg, tokens=3)
    out, ids, w = oracle_latent(cfg, x)
    down, up, norm = synth.latent_weights(cfg)
    xl = x.astype(np.float64) @ down.astype(np.float64).T
    routed = np.zeros((x.shape[0], cfg.hidden))
    for t in range(x.shape[0]):
        for j in range(cfg.topk):
            ex = synth.expert(cfg, int(ids[t, j]))
            g = _dense(ex["gate"], ex["gate_scale"], cfg.inter, cfg.hidden) @ xl[t]
            u = _dense(ex["up"], ex["up_scale"], cfg.inter, cfg.hidden) @ xl[t]
            h = _situ64(g, u, cfg.situ_beta, cfg.situ_linear_beta)
            routed[t] += w[t, j] * (_dense(ex["down"], ex["down_scale"], cfg.hidden, cfg.inter) @ h)
    routed = routed / np.sqrt(np.mean(routed ** 2, axis=1, keepdims=True) + 1e-5) * norm
    want = routed @ up.astype(np.float64).T
    assert rel_l2(out, want) < 1e-5
    assert math.isfinite(float(np.abs(out).max()))


# ------------------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_latent_tiny_matches_oracle(cuda_ctx):
    cfg = synth.CONFIGS["c5_tiny_latent"]
    L = build_layer(cuda_ctx, cfg, max_tokens=cfg.tokens)
    x = synth.activations(cfg)
    for T in (1, cfg.tokens):
        out, ids, w = L.latent_moe(x_device(cfg, x[:T]), return_routing=True)
        want, want_ids, want_w = oracle_latent(cfg, x[:T])
        assert np.array_equal(ids.cpu().numpy(), want_ids)
        assert np.max(np.abs(w.cpu().numpy() - want_w)) < 1e-5
        assert rel_l2(out.cpu().numpy(), want) < OUT_RTOL
    with pytest.raises(Exception):
        L.moe_forward(x_device(cfg, x[:1]))  # a latent layer only runs through rmoe_latent_moe
    L.close()


@pytest.mark.gpu
def test_latent_k3_shapes_match_oracle(cuda_ctx):
    """The real K3 shapes (7168 -> 3584, 896 experts, top-16, inter 3072, Situ, norm)."""
    cfg = synth.CONFIGS["c5_k3_latent"]
    L = build_layer(cuda_ctx, cfg, max_tokens=4)
    x = synth.activations(cfg, tokens=2)
    out, ids, _ = L.latent_moe(x_device(cfg, x), return_routing=True)
    want, want_ids, _ = oracle_latent(cfg, x)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert rel_l2(out.cpu().numpy(), want) < OUT_RTOL
    L.close()
