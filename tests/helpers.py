"""Shared test plumbing: build a device layer from a synthetic config, and the matching CPU
oracle run on exactly the same bytes."""
from __future__ import annotations

import numpy as np

from rabbit_b200 import synth
from rabbit_b200.synth import build_layer, gpu_expert, x_device  # noqa: F401  (re-exported)


def oracle_routing(cfg, x, seed=0, layer=0):
    """Routing the reference computes for x: ids/weights [T, k]."""
    from oracle import oracle as orc

    router = synth.router_weights(cfg, seed, layer)
    T = x.shape[0]
    if cfg.router == "softmax":
        logits = orc.matmul(x, router, T, cfg.hidden, cfg.n_experts)
        b = synth.logit_bias(cfg, seed, layer)
        if b is not None:
            logits = (logits + b[None, :]).astype(np.float32)
        k = min(cfg.topk, cfg.n_experts)
        ids = np.zeros((T, k), np.int32)
        w = np.zeros((T, k), np.float32)
        for t in range(T):
            r = orc.qwen_route(logits[t], cfg.topk)
            ids[t] = [i for i, _ in r]
            w[t] = [v for _, v in r]
        return ids, w
    return orc.glm_route(x, router, synth.correction_bias(cfg, seed, layer), T, cfg.hidden,
                         cfg.n_experts, cfg.topk, cfg.n_group, cfg.topk_group, cfg.norm_topk,
                         cfg.routed_scale)


def oracle_forward(cfg, x, seed=0, layer=0, scale_dtype="f32", tier="scalar"):
    """The reference layer output for x (experts regenerated on the host, touched ones only).
    tier "avx512": the reference's AVX-512 MXFP4 tier (within 1e-4 of the scalar one) for large
    token counts of softmax-routed MXFP4 layers."""
    from oracle import oracle as orc

    ids, _ = oracle_routing(cfg, x, seed, layer)
    experts = {int(e): synth.expert(cfg, int(e), seed, layer) for e in np.unique(ids) if e >= 0}
    shared = synth.expert(cfg, cfg.n_experts, seed, layer) if cfg.shared_inter else None
    router = synth.router_weights(cfg, seed, layer)
    if cfg.router == "softmax":
        return orc.moe_forward_qwen(x, router, experts, cfg.n_experts, cfg.topk, cfg.inter,
                                    shared=shared, shared_gate=synth.shared_gate(cfg, seed, layer),
                                    logit_bias=synth.logit_bias(cfg, seed, layer),
                                    shared_inter=cfg.shared_inter, fmt=cfg.fmt_id,
                                    gs=cfg.group_size, tier=tier)
    return orc.moe_glm(x, router, synth.correction_bias(cfg, seed, layer), experts, cfg.n_experts,
                       cfg.topk, cfg.inter, cfg.n_group, cfg.topk_group, cfg.norm_topk,
                       cfg.routed_scale, shared=shared, shared_inter=cfg.shared_inter,
                       fmt=cfg.fmt_id, gs=cfg.group_size)


def oracle_latent(cfg, x, seed=0, layer=0):
    """The reference latent MoE (kimi_k3::moe::latent_moe) for x [T, router_hidden]: (out, ids, w)."""
    from oracle import oracle as orc

    router = synth.router_weights(cfg, seed, layer)
    bias = synth.correction_bias(cfg, seed, layer)
    ids, _ = orc.glm_route(x, router, bias, x.shape[0], cfg.full_hidden, cfg.n_experts, cfg.topk, cfg.n_group,
                           cfg.topk_group, cfg.norm_topk, cfg.routed_scale)
    experts = {int(e): synth.expert(cfg, int(e), seed, layer) for e in np.unique(ids) if e >= 0}
    down, up, norm = synth.latent_weights(cfg, seed, layer)
    return orc.latent_moe(x, router, bias, experts, cfg.n_experts, cfg.topk, cfg.n_group, cfg.topk_group,
                          cfg.norm_topk, cfg.routed_scale, down, up, norm, 1e-5, cfg.hidden, cfg.inter,
                          act=cfg.act, fmt=cfg.fmt_id, gs=cfg.group_size)


def per_token_rel_l2(got, want):
    """Relative L2 error of each token's output row."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return np.linalg.norm(got - want, axis=1) / np.maximum(np.linalg.norm(want, axis=1), 1e-30)


def hard_prefill_tokens(ids, mt=32, n_popular=3, at_least=64, seed=1):
    """Tokens that decide the hardest prefill outputs: for the n_popular most-picked experts (the
    ones split into several position chunks of mt rows), the first and last token of every chunk
    of their ascending-token row list; topped up with seeded random tokens to at_least."""
    ids = np.asarray(ids)
    T = ids.shape[0]
    counts = np.bincount(ids[ids >= 0].ravel(), minlength=int(ids.max()) + 1)
    sel = {0, T - 1}
    for e in np.argsort(-counts, kind="stable")[:n_popular]:
        rows = np.nonzero((ids == e).any(axis=1))[0]
        for c0 in range(0, len(rows), mt):
            chunk = rows[c0:c0 + mt]
            sel.update((int(chunk[0]), int(chunk[-1])))
    rng = np.random.default_rng(seed)
    while len(sel) < at_least:
        sel.add(int(rng.integers(T)))
    return sorted(sel)
