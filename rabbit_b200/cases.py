"""Workload drivers for profiling (one GPU): build a synthetic layer of a config and run forwards,
optionally with the last one inside a cudaProfilerStart/Stop range so that
`ncu --profile-from-start off` captures exactly that call.

    python -m rabbit_b200.cases prefill [--experts NE] [--forwards N] [--profile-last]
    python -m rabbit_b200.cases latent  [--forwards N] [--profile-last]
    python -m rabbit_b200.cases decode  [--experts NE] [--forwards N] [--profile-last]

prefill: c2_qwen_prefill (2048 tokens per forward); latent: c5_k3_latent, one token per forward
(Kimi K3 latent MoE); decode: c1_qwen_decode, one token per forward. NE shrinks the resident
experts (same shapes) so a full-metric capture stays small.
"""
from __future__ import annotations

import argparse
import dataclasses

from . import synth


def main(argv=None):
    import torch

    from . import moe as rb
    from .synth import build_layer, x_device

    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["prefill", "latent", "decode"])
    ap.add_argument("--experts", type=int, default=0)
    ap.add_argument("--forwards", type=int, default=3)
    ap.add_argument("--profile-last", action="store_true")
    a = ap.parse_args(argv)
    name = {"prefill": "c2_qwen_prefill", "latent": "c5_k3_latent", "decode": "c1_qwen_decode"}[a.case]
    cfg = synth.CONFIGS[name]
    if a.experts:
        cfg = dataclasses.replace(cfg, n_experts=a.experts)
    ctx = rb.Context(0)
    tokens = cfg.tokens
    layer = build_layer(ctx, cfg, max_tokens=tokens)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for i in range(a.forwards):
        x = x_device(cfg, synth.activations(cfg, tokens=tokens, token_offset=100_000 + i * tokens))
        flush.zero_()
        torch.cuda.synchronize()
        last = i == a.forwards - 1
        if last and a.profile_last:
            torch.cuda.cudart().cudaProfilerStart()
        if a.case == "latent":
            layer.latent_moe(x)
        else:
            layer.moe_forward(x)
        torch.cuda.synchronize()
        if last and a.profile_last:
            torch.cuda.cudart().cudaProfilerStop()
    errs = layer.stats()["device_error_flags"]
    layer.close()
    ctx.close()
    print(f"{a.case}: {a.forwards} forwards, device error flags {errs}")
    return 0 if errs == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
