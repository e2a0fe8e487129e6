"""Writes small .safetensors checkpoints for the loader tests, the way the reference's own tests
build theirs (build_safetensors, src/safetensors.rs:620-639: an 8-byte little-endian header
length, a JSON header with a __metadata__ entry and name -> {dtype, shape, data_offsets}, then
the tensors' bytes back to back), and lays a synthetic MoE layer out under the reference's
checkpoint tensor names (src/expert_cache.rs:155-207, src/qwen38/model.rs:319-326,
src/glm52/model.rs:249-253)."""
from __future__ import annotations

import json
import os
import struct

import numpy as np

from rabbit_b200 import synth


def build_safetensors(entries) -> bytes:
    """entries: [(name, dtype, shape, bytes)] -> the file's bytes."""
    header = {"__metadata__": {"format": "rabbit-test"}}
    data = bytearray()
    for name, dtype, shape, raw in entries:
        start = len(data)
        data += bytes(raw)
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [start, len(data)]}
    hb = json.dumps(header).encode()
    return struct.pack("<Q", len(hb)) + hb + bytes(data)


def write(path, entries):
    with open(path, "wb") as f:
        f.write(build_safetensors(entries))


def _u8(a):
    return np.ascontiguousarray(a).view(np.uint8).tobytes()


def layer_entries(cfg, naming: str, family: str, layer: int = 0, seed: int = 0):
    """The synthetic layer (synth's weights of cfg) as checkpoint tensors: routed experts under
    `naming`, router / bias / shared expert under `family`'s names."""
    h, i = cfg.hidden, cfg.inter
    out = []

    def mx_pair(base, packed_suffix, rows, cols, data, scale):
        out.append((base + packed_suffix, "U8", [rows, (cols + 1) // 2], _u8(data)))
        out.append((base + ".weight_scale", "U8", [rows, (cols + 31) // 32], _u8(scale)))

    def qs_pair(name, rows, cols, data, scale):
        out.append((name, "U8", [rows, (cols + 1) // 2], _u8(data)))
        out.append((name + ".qs", "F32", [rows, (cols + cfg.group_size - 1) // cfg.group_size],
                    _u8(np.asarray(scale, np.float32))))

    for eid in range(cfg.n_experts):
        ex = synth.expert(cfg, eid, seed, layer)
        if naming in ("qwen38_mxfp4", "kimi_k3_mxfp4"):
            if naming == "qwen38_mxfp4":
                pre, names, suf = f"model.layers.{layer}.mlp.experts.{eid}.", ("gate_proj", "up_proj", "down_proj"), ".weight"
            else:
                pre, names, suf = (f"language_model.model.layers.{layer}.block_sparse_moe.experts.{eid}.",
                                   ("w1", "w3", "w2"), ".weight_packed")
            for nm, key, (r, c) in zip(names, ("gate", "up", "down"), ((i, h), (i, h), (h, i))):
                mx_pair(pre + nm, suf, r, c, ex[key], ex[key + "_scale"])
        elif naming == "glm52_fused_gate_up":
            pre = f"model.layers.{layer}.mlp.experts.{eid}."
            qs_pair(pre + "gate_up_proj.weight", 2 * i, h, np.concatenate([ex["gate"], ex["up"]]),
                    np.concatenate([ex["gate_scale"], ex["up_scale"]]))
            qs_pair(pre + "down_proj.weight", h, i, ex["down"], ex["down_scale"])
        else:
            pre = {"glm52": f"model.layers.{layer}.mlp.experts.{eid}.",
                   "kimi_linear": f"model.layers.{layer}.block_sparse_moe.experts.{eid}.",
                   "kimi_k3": f"language_model.model.layers.{layer}.block_sparse_moe.experts.{eid}."}[naming]
            names = ("gate_proj", "up_proj", "down_proj") if naming == "glm52" else ("w1", "w3", "w2")
            for nm, key, (r, c) in zip(names, ("gate", "up", "down"), ((i, h), (i, h), (h, i))):
                qs_pair(pre + nm + ".weight", r, c, ex[key], ex[key + "_scale"])
    mp = f"model.layers.{layer}.mlp."
    router = synth.router_weights(cfg, seed, layer)
    if cfg.bf16_inputs:
        out.append((mp + "gate.weight", "BF16", [cfg.n_experts, h], _u8(synth.f32_to_bf16_bits(router))))
    else:
        out.append((mp + "gate.weight", "F32", [cfg.n_experts, h], _u8(router)))
    if family == "glm52":
        out.append((mp + "gate.e_score_correction_bias", "F32", [cfg.n_experts],
                    _u8(synth.correction_bias(cfg, seed, layer))))
    if cfg.shared_inter:
        sh = synth.expert(cfg, cfg.n_experts, seed, layer)
        si = cfg.shared_inter
        sp = mp + ("shared_expert." if family == "qwen38" else "shared_experts.")
        for nm, key, (r, c) in (("gate_proj", "gate", (si, h)), ("up_proj", "up", (si, h)),
                                ("down_proj", "down", (h, si))):
            if cfg.fmt == "mxfp4":
                mx_pair(sp + nm, ".weight", r, c, sh[key], sh[key + "_scale"])
            else:
                qs_pair(sp + nm + ".weight", r, c, sh[key], sh[key + "_scale"])
        if family == "qwen38" and cfg.shared_gated:
            out.append((mp + "shared_expert_gate.weight", "F32", [1, h], _u8(synth.shared_gate(cfg, seed, layer))))
    return out


def write_layer(dirpath, cfg, naming, family, layer=0, n_files=2):
    """The layer's tensors split over n_files shards (model-0000k-of-0000n.safetensors)."""
    ents = layer_entries(cfg, naming, family, layer)
    per = (len(ents) + n_files - 1) // n_files
    for k in range(n_files):
        write(os.path.join(dirpath, f"model-{k + 1:05d}-of-{n_files:05d}.safetensors"), ents[k * per:(k + 1) * per])
