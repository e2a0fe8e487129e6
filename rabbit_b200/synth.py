"""Seeded synthetic inputs for the routed-MoE configs (host side, numpy).

One counter-based generator feeds the CPU oracle, the parity tests and the bench, so any subset
of a tensor (say, only the experts a batch routes to) can be regenerated on its own:

* ``u64(key, i)`` is the i-th SplitMix64 output from state ``key``:
  ``fmix64(key + (i + 1) * 0x9E3779B97F4A7C15)``.
* uniform bytes: byte j = byte (j % 8) of ``u64(key, j // 8)`` (E2M1 nibbles and offset-binary
  int4 codes are both "uniform over 16 codes" per nibble).
* E8M0 bytes in [127+lo, 127+hi]: ``127 + lo + (u64(key, j) >> 32) % (hi - lo + 1)``.
* normals: Box-Muller in double on ``u64(key, 2p)``, ``u64(key, 2p+1)``; then round-to-nearest-even
  to f32 and, where a config says bf16, again to bf16.

The byte generators are integer-exact, so the CUDA fill kernel (``rmoe_synth_bytes``) writes the
identical bytes on the device; normals are only generated here.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_TAGMUL = 0xD1B54A32D192ED03
MASK64 = (1 << 64) - 1

# tensor roles inside a stream tag
ROLE_ROUTER, ROLE_X, ROLE_DATA, ROLE_SCALE, ROLE_ZIPF, ROLE_SHGATE, ROLE_BIAS = 1, 2, 3, 4, 5, 6, 7
ROLE_LATENT = 8  # latent MoE wrapper: tensor 0 down_proj, 1 up_proj, 2 norm
GATE, UP, DOWN = 0, 1, 2


def fmix64_int(z: int) -> int:
    z &= MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def stream_key(seed: int, tag: int) -> int:
    return fmix64_int(((seed ^ ((tag * _TAGMUL) & MASK64)) + 0x9E3779B97F4A7C15) & MASK64)


def tag(layer: int, role: int, expert: int = 0, tensor: int = 0) -> int:
    return (layer << 40) | (role << 32) | (expert << 8) | tensor


def u64(key: int, start: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(key) + i * GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform_bytes(key: int, n: int) -> np.ndarray:
    words = u64(key, 0, (n + 7) // 8)
    return words.view(np.uint8)[:n].copy()  # little-endian: byte j%8 of word j//8


def e8m0_bytes(key: int, n: int, lo: int, hi: int) -> np.ndarray:
    r = (u64(key, 0, n) >> np.uint64(32)) % np.uint64(hi - lo + 1)
    return (127 + lo + r.astype(np.int64)).astype(np.uint8)


def normals(key: int, n: int) -> np.ndarray:
    """float64 N(0,1) values by Box-Muller."""
    npair = (n + 1) // 2
    w = u64(key, 0, 2 * npair).reshape(npair, 2)
    u1 = ((w[:, 0] >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53  # (0, 1]
    u2 = (w[:, 1] >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty((npair, 2), np.float64)
    z[:, 0] = r * np.cos(2.0 * math.pi * u2)
    z[:, 1] = r * np.sin(2.0 * math.pi * u2)
    return z.reshape(-1)[:n]


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    rounding = ((b >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((b + rounding) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(a: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


@dataclasses.dataclass(frozen=True)
class MoeConfig:
    name: str
    tokens: int
    hidden: int
    n_experts: int
    topk: int
    inter: int
    shared_inter: int
    router: str = "softmax"          # "softmax" (Qwen) | "sigmoid_grouped" (GLM)
    fmt: str = "mxfp4"               # "mxfp4" | "int4g"
    e8m0_lo: int = -6
    e8m0_hi: int = -2
    bf16_inputs: bool = True         # router / x / shared gate rounded to bf16
    zipf: float = 0.0                # Zipf exponent of the harness logit bias (0 = none)
    shared_gated: bool = True
    n_group: int = 1
    topk_group: int = 1
    routed_scale: float = 1.0
    norm_topk: bool = True
    group_size: int = 32
    int4_scale_sigma: float = 0.01
    bias_sigma: float = 0.01
    n_layers: int = 1
    # Kimi K3 latent MoE: the router and x are router_hidden wide, the experts `hidden` wide
    router_hidden: int = 0
    activation: str = "silu"         # "silu" | "situ" (Kimi K3 SituAndMul)
    situ_beta: float = 0.0
    situ_linear_beta: float = 0.0    # 0 = none
    latent_norm: bool = False

    @property
    def full_hidden(self) -> int:
        """Width of the router and of the layer's input x."""
        return self.router_hidden or self.hidden

    @property
    def act(self):
        """The activation as the oracle takes it."""
        if self.activation == "silu":
            return ("silu",)
        return ("situ", self.situ_beta, self.situ_linear_beta or None)

    @property
    def fmt_id(self) -> int:
        return 0 if self.fmt == "mxfp4" else 1

    def expert_bytes(self, scale_bytes: int = 4) -> int:
        """Bytes of one routed expert in the reference layout (gate + up + down)."""
        h, i = self.hidden, self.inter
        data = 2 * i * ((h + 1) // 2) + h * ((i + 1) // 2)
        if self.fmt == "mxfp4":
            return data + 2 * i * ((h + 31) // 32) + h * ((i + 31) // 32)
        gs = self.group_size
        return data + scale_bytes * (2 * i * ((h + gs - 1) // gs) + h * ((i + gs - 1) // gs))


CONFIGS = {
    "c0_tiny": MoeConfig("c0_tiny", tokens=4, hidden=256, n_experts=16, topk=2, inter=128,
                         shared_inter=128, e8m0_lo=-6, e8m0_hi=-2, bf16_inputs=False),
    "c1_qwen_decode": MoeConfig("c1_qwen_decode", tokens=1, hidden=8192, n_experts=512, topk=10,
                                inter=2048, shared_inter=2048, e8m0_lo=-8, e8m0_hi=-3, zipf=1.1),
    "c2_qwen_prefill": MoeConfig("c2_qwen_prefill", tokens=2048, hidden=8192, n_experts=512,
                                 topk=10, inter=2048, shared_inter=2048, e8m0_lo=-8, e8m0_hi=-3,
                                 zipf=1.1),
    "c3_qwen_ep": MoeConfig("c3_qwen_ep", tokens=4096, hidden=8192, n_experts=512, topk=10,
                            inter=2048, shared_inter=2048, e8m0_lo=-8, e8m0_hi=-3, zipf=1.1,
                            n_layers=4),
    "c4_glm_int4": MoeConfig("c4_glm_int4", tokens=512, hidden=6144, n_experts=256, topk=8,
                             inter=2048, shared_inter=2048, router="sigmoid_grouped",
                             fmt="int4g", shared_gated=False, n_group=8, topk_group=4,
                             routed_scale=2.5, norm_topk=True),
    # Kimi K3's latent MoE at the real checkpoint's shapes (hidden 7168 routed, experts at 3584,
    # moe_intermediate 3072, 896 experts, top-16, sigmoid router, Situ beta 4 / linear 25, norm
    # on; src/kimi_k3/config.rs:255-265). Not a BASELINE config: the supplementary row a14.
    "c5_k3_latent": MoeConfig("c5_k3_latent", tokens=1, hidden=3584, n_experts=896, topk=16,
                              inter=3072, shared_inter=0, router="sigmoid_grouped", shared_gated=False,
                              e8m0_lo=-8, e8m0_hi=-3, router_hidden=7168, activation="situ",
                              situ_beta=4.0, situ_linear_beta=25.0, latent_norm=True),
    "c5_tiny_latent": MoeConfig("c5_tiny_latent", tokens=6, hidden=512, n_experts=32, topk=4,
                                inter=512, shared_inter=0, router="sigmoid_grouped", shared_gated=False,
                                e8m0_lo=-6, e8m0_hi=-3, router_hidden=1024, activation="situ",
                                situ_beta=4.0, situ_linear_beta=25.0, latent_norm=True),
}


def _normal_tensor(seed, t, n, sigma, bf16):
    v = (normals(stream_key(seed, t), n) * sigma).astype(np.float32)
    return round_bf16(v) if bf16 else v


def router_weights(cfg: MoeConfig, seed: int = 0, layer: int = 0) -> np.ndarray:
    """[E, H] f32 (bf16-representable when the config is bf16): N(0, 0.02)."""
    n = cfg.n_experts * cfg.full_hidden
    return _normal_tensor(seed, tag(layer, ROLE_ROUTER), n, 0.02, cfg.bf16_inputs).reshape(
        cfg.n_experts, cfg.full_hidden)


def activations(cfg: MoeConfig, seed: int = 0, layer: int = 0, tokens: int | None = None,
                token_offset: int = 0) -> np.ndarray:
    """[T, H] f32 (bf16-representable when the config is bf16): N(0, 1)."""
    t = cfg.tokens if tokens is None else tokens
    key = stream_key(seed, tag(layer, ROLE_X))
    h = cfg.full_hidden
    # token rows are independent slices of one stream, so any token range can be regenerated
    z = normals_range(key, token_offset * h, t * h).astype(np.float32)
    z = round_bf16(z) if cfg.bf16_inputs else z
    return z.reshape(t, h)


def normals_range(key: int, start: int, n: int) -> np.ndarray:
    """Elements [start, start+n) of the normal stream ``key``."""
    p0 = start // 2
    p1 = (start + n + 1) // 2
    w = u64(key, 2 * p0, 2 * (p1 - p0)).reshape(-1, 2)
    u1 = ((w[:, 0] >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
    u2 = (w[:, 1] >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty((w.shape[0], 2), np.float64)
    z[:, 0] = r * np.cos(2.0 * math.pi * u2)
    z[:, 1] = r * np.sin(2.0 * math.pi * u2)
    off = start - 2 * p0
    return z.reshape(-1)[off:off + n]


def logit_bias(cfg: MoeConfig, seed: int = 0, layer: int = 0) -> np.ndarray | None:
    """Harness popularity skew for the softmax router: b_e = -zipf * ln(rank_e), rank_e from a
    seeded permutation of 1..E. None when the config has no Zipf skew."""
    if cfg.router != "softmax" or cfg.zipf == 0.0:
        return None
    keys = u64(stream_key(seed, tag(layer, ROLE_ZIPF)), 0, cfg.n_experts)
    order = np.argsort(keys, kind="stable")
    rank = np.empty(cfg.n_experts, np.int64)
    rank[order] = np.arange(1, cfg.n_experts + 1)
    return (-cfg.zipf * np.log(rank.astype(np.float64))).astype(np.float32)


def correction_bias(cfg: MoeConfig, seed: int = 0, layer: int = 0) -> np.ndarray | None:
    """GLM noaux_tc per-expert correction bias N(0, bias_sigma) f32."""
    if cfg.router != "sigmoid_grouped":
        return None
    return (normals(stream_key(seed, tag(layer, ROLE_BIAS)), cfg.n_experts) *
            cfg.bias_sigma).astype(np.float32)


def latent_weights(cfg: MoeConfig, seed: int = 0, layer: int = 0):
    """(down_proj [hidden, router_hidden], up_proj [router_hidden, hidden]) as bf16-representable
    f32 with N(0, 1/fan_in) entries, and the norm weight [hidden] = 1 + 0.1 N(0, 1) (None when
    the config has no norm)."""
    rh, h = cfg.router_hidden, cfg.hidden
    down = _normal_tensor(seed, tag(layer, ROLE_LATENT, 0, 0), h * rh, 1.0 / math.sqrt(rh), True).reshape(h, rh)
    up = _normal_tensor(seed, tag(layer, ROLE_LATENT, 0, 1), rh * h, 1.0 / math.sqrt(h), True).reshape(rh, h)
    norm = None
    if cfg.latent_norm:
        norm = (1.0 + 0.1 * normals(stream_key(seed, tag(layer, ROLE_LATENT, 0, 2)), h)).astype(np.float32)
    return down, up, norm


def shared_gate(cfg: MoeConfig, seed: int = 0, layer: int = 0) -> np.ndarray | None:
    """Qwen shared_expert_gate [H]: N(0, 0.02)."""
    if not cfg.shared_gated:
        return None
    return _normal_tensor(seed, tag(layer, ROLE_SHGATE), cfg.hidden, 0.02, cfg.bf16_inputs)


def tensor_shape(cfg: MoeConfig, tensor: int, shared: bool = False):
    i = cfg.shared_inter if shared else cfg.inter
    return (i, cfg.hidden) if tensor in (GATE, UP) else (cfg.hidden, i)


def expert_tensor(cfg: MoeConfig, eid: int, tensor: int, seed: int = 0, layer: int = 0,
                  shared: bool = False, scale_dtype: str = "f32"):
    """(data bytes, scales) of one expert matrix in the reference layout. ``eid`` = n_experts
    addresses the shared expert. MXFP4 scales are E8M0 bytes; int4 scales are |N(0, sigma)|
    rounded to bf16 (returned as f32, or as bf16 bits with scale_dtype="bf16")."""
    rows, cols = tensor_shape(cfg, tensor, shared)
    data = uniform_bytes(stream_key(seed, tag(layer, ROLE_DATA, eid, tensor)),
                         rows * ((cols + 1) // 2))
    skey = stream_key(seed, tag(layer, ROLE_SCALE, eid, tensor))
    if cfg.fmt == "mxfp4":
        sc = e8m0_bytes(skey, rows * ((cols + 31) // 32), cfg.e8m0_lo, cfg.e8m0_hi)
    else:
        n = rows * ((cols + cfg.group_size - 1) // cfg.group_size)
        v = np.abs(normals(skey, n) * cfg.int4_scale_sigma).astype(np.float32)
        bits = f32_to_bf16_bits(v)
        # a zero scale is legal but useless; keep the draw as is (it is bf16-exact either way)
        sc = bits if scale_dtype == "bf16" else bf16_bits_to_f32(bits)
    return data, sc


def expert(cfg: MoeConfig, eid: int, seed: int = 0, layer: int = 0, scale_dtype: str = "f32"):
    """All six arrays of one expert (``eid == n_experts`` -> the shared expert)."""
    shared = eid == cfg.n_experts
    out = {}
    for t, name in ((GATE, "gate"), (UP, "up"), (DOWN, "down")):
        d, s = expert_tensor(cfg, eid, t, seed, layer, shared, scale_dtype)
        out[name] = d
        out[name + "_scale"] = s
    return out


# ------------------------------------------------------------------------------ device layers
TENSORS = ((GATE, "gate"), (UP, "up"), (DOWN, "down"))


def gpu_expert(cfg, eid, seed=0, layer=0, device="cuda", scale_dtype="f32"):
    """The six tensors of expert ``eid`` (``n_experts`` = shared) generated on the device."""
    import torch

    from . import moe as rb

    shared = eid == cfg.n_experts
    out = {}
    for t, name in TENSORS:
        rows, cols = tensor_shape(cfg, t, shared)
        data = torch.empty(rows * ((cols + 1) // 2), dtype=torch.uint8, device=device)
        rb.synth_bytes(data, stream_key(seed, tag(layer, ROLE_DATA, eid, t)), 0)
        if cfg.fmt == "mxfp4":
            sc = torch.empty(rows * ((cols + 31) // 32), dtype=torch.uint8, device=device)
            rb.synth_bytes(sc, stream_key(seed, tag(layer, ROLE_SCALE, eid, t)), 1,
                           cfg.e8m0_lo, cfg.e8m0_hi)
        else:
            _, s_host = expert_tensor(cfg, eid, t, seed, layer, shared, scale_dtype)
            sc = torch.from_numpy(s_host.view(np.uint8).copy()).to(device)
        out[name] = data
        out[name + "_scale"] = sc
    return out


def build_layer(ctx, cfg, max_tokens, seed=0, layer=0, scale_dtype="f32", ep_rank=0, ep_size=1):
    """A MoeLayer holding cfg's synthetic weights (all local experts resident)."""
    import torch

    from . import moe as rb

    L = rb.MoeLayer(ctx, cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk,
                    shared_inter=cfg.shared_inter, router=cfg.router, n_group=cfg.n_group,
                    topk_group=cfg.topk_group, norm_topk=cfg.norm_topk,
                    routed_scale=cfg.routed_scale, fmt=cfg.fmt, group_size=cfg.group_size,
                    scale_dtype=scale_dtype, shared_gated=cfg.shared_gated,
                    max_tokens=max_tokens, ep_rank=ep_rank, ep_size=ep_size,
                    activation=cfg.activation, situ_beta=cfg.situ_beta,
                    situ_linear_beta=cfg.situ_linear_beta, router_hidden=cfg.router_hidden)
    router = router_weights(cfg, seed, layer)
    if cfg.bf16_inputs:
        L.upload_router(f32_to_bf16_bits(router))
    else:
        L.upload_router(router)
    bias = logit_bias(cfg, seed, layer) if cfg.router == "softmax" else correction_bias(cfg, seed, layer)
    if bias is not None:
        L.upload_router_bias(bias)
    n_loc = cfg.n_experts // ep_size
    for eid in range(ep_rank * n_loc, (ep_rank + 1) * n_loc):
        ex = gpu_expert(cfg, eid, seed, layer, scale_dtype=scale_dtype)
        L.upload_expert_dict(eid, ex)
    torch.cuda.synchronize()
    if cfg.router_hidden:
        down, up, norm = latent_weights(cfg, seed, layer)
        L.upload_latent(f32_to_bf16_bits(down), f32_to_bf16_bits(up), norm)
    if cfg.shared_inter:
        sh = gpu_expert(cfg, cfg.n_experts, seed, layer, scale_dtype=scale_dtype)
        L.upload_shared(sh["gate"], sh["gate_scale"], sh["up"], sh["up_scale"], sh["down"],
                        sh["down_scale"], shared_gate(cfg, seed, layer))
    torch.cuda.synchronize()
    return L


def x_device(cfg, x_f32):
    """Activations as the config's dtype on the device (bf16 configs keep bf16)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x_f32)).cuda()
    return t.to(torch.bfloat16) if cfg.bf16_inputs else t
