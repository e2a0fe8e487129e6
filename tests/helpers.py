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


def oracle_forward(cfg, x, seed=0, layer=0, scale_dtype="f32"):
    """The reference layer output for x (experts regenerated on the host, touched ones only)."""
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
                                    gs=cfg.group_size)
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
