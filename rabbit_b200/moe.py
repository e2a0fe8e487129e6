"""Python mirror of rabbit's MoE-block interface over the C ABI (include/rmoe.h).

Names and argument meaning follow the reference (ferrumox/rabbit v0.29.1):

* ``matmul`` / ``matmul_mxfp4`` / ``matmul_i4_grouped``: ``y[S,O] = x[S,I] . W^T`` with the
  reference's argument order ``(y, x, w..., s, i, o)`` (src/kernels.rs:113, :233, :276).
* ``MoeLayer.route``: router matmul + ``qwen38::moe::route`` / ``glm52::moe::route``.
* ``MoeLayer.moe_forward``: ``qwen38::generate::moe_forward`` / ``glm52::moe::moe``; ``out`` is
  overwritten, as there.
* Errors surface as ``RmoeError`` (the reference's ``Result<_, ModelError>``), shape bugs as
  ``RmoeError`` with status SHAPE_MISMATCH instead of a panic.

All compute runs in librmoe.so on the GPU; torch only holds device memory and streams.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import (DT_BF16, DT_F32, FMT_I4_GROUPED, FMT_MXFP4, ROUTER_SIGMOID_GROUPED,
                   ROUTER_SOFTMAX_TOPK, STAGES, LayerDesc, LayerStats, Profile, RmoeError,
                   check)

try:
    import torch
except ImportError:  # pragma: no cover - torch is in the image; kept optional for the C ABI checks
    torch = None


def _ptr(a):
    """Address of a numpy array or torch tensor (host or device)."""
    if a is None:
        return None
    if torch is not None and isinstance(a, torch.Tensor):
        return a.data_ptr()
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    raise TypeError(f"expected a numpy array or torch tensor, got {type(a)}")


def _nbytes(a):
    if torch is not None and isinstance(a, torch.Tensor):
        return a.numel() * a.element_size()
    return a.nbytes


def _dtype_code(a):
    if torch is not None and isinstance(a, torch.Tensor):
        if a.dtype == torch.bfloat16:
            return DT_BF16
        if a.dtype == torch.float32:
            return DT_F32
        raise TypeError(f"activations must be float32 or bfloat16, got {a.dtype}")
    if a.dtype == np.float32:
        return DT_F32
    if a.dtype == np.uint16:  # bf16 bit patterns
        return DT_BF16
    raise TypeError(f"activations must be float32 or bf16 bits (uint16), got {a.dtype}")


def _stream(stream=None):
    if stream is not None:
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream
    if torch is not None and torch.cuda.is_available():
        return torch.cuda.current_stream().cuda_stream
    return None


def _require_cuda(*ts):
    for t in ts:
        if torch is None or not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RmoeError(1, "device entry points take CUDA tensors")
        if not t.is_contiguous():
            raise RmoeError(1, "tensors must be contiguous")


class Context:
    """One GPU (rmoe_init)."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        h = C.c_void_p()
        check(self.lib.rmoe_init(device, C.byref(h)))
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            self.lib.rmoe_shutdown(self.handle)
            self.handle = None


class MoeLayer:
    """One routed-MoE block with every local expert resident in HBM."""

    def __init__(self, ctx: Context, hidden: int, moe_inter: int, n_experts: int, topk: int, *,
                 shared_inter: int = 0, router: str = "softmax", n_group: int = 1,
                 topk_group: int = 1, norm_topk: bool = True, routed_scale: float = 1.0,
                 fmt: str = "mxfp4", group_size: int = 32, scale_dtype: str = "f32",
                 shared_gated: bool = False, max_tokens: int = 1, ep_rank: int = 0,
                 ep_size: int = 1, activation: str = "silu", situ_beta: float = 0.0,
                 situ_linear_beta: float = 0.0, router_hidden: int = 0):
        self.lib = ctx.lib
        self.ctx = ctx
        d = LayerDesc()
        d.hidden, d.moe_inter, d.shared_inter = hidden, moe_inter, shared_inter
        d.n_experts, d.topk = n_experts, topk
        d.router_kind = ROUTER_SOFTMAX_TOPK if router == "softmax" else ROUTER_SIGMOID_GROUPED
        d.n_group, d.topk_group, d.norm_topk = n_group, topk_group, int(norm_topk)
        d.routed_scale = routed_scale
        d.weight_format = FMT_MXFP4 if fmt == "mxfp4" else FMT_I4_GROUPED
        d.group_size = group_size
        d.scale_dtype = DT_BF16 if scale_dtype == "bf16" else DT_F32
        d.shared_gated, d.max_tokens = int(shared_gated), max_tokens
        d.ep_rank, d.ep_size = ep_rank, ep_size
        d.activation = 1 if activation == "situ" else 0
        d.situ_beta, d.situ_linear_beta = situ_beta, situ_linear_beta
        d.router_hidden = router_hidden
        self.desc = d
        h = C.c_void_p()
        check(self.lib.rmoe_layer_create(ctx.handle, C.byref(d), C.byref(h)))
        self.handle = h
        self.hidden, self.topk, self.n_experts = hidden, topk, n_experts
        self.router_hidden = router_hidden or hidden
        self.max_tokens = max_tokens

    # ---- lifetime
    def close(self):
        if self.handle:
            self.lib.rmoe_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def stats(self) -> dict:
        s = LayerStats()
        check(self.lib.rmoe_layer_get_stats(self.handle, C.byref(s)))
        return {f: getattr(s, f) for f, _ in LayerStats._fields_}

    def check(self, stream=None):
        """Synchronize and raise RmoeError(TIMEOUT) if a bounded device wait of this layer's
        kernels ran out since the last check (the layer is usable again afterwards)."""
        check(self.lib.rmoe_layer_check(self.handle, _stream(stream)))

    def set_wait_limit(self, ns: int = 0):
        """Limit of the kernels' waits on other CTAs in nanoseconds (0: the default 2 s)."""
        check(self.lib.rmoe_layer_set_wait_limit(self.handle, int(ns)))

    def set_route_config(self, cache_route: bool, route_j: int = 2, route_m: int = 12, resident=None):
        """CACHE_ROUTE (glm52::moe::RouteConfig; sigmoid routers only). resident: [E] bool/uint8
        array of resident experts, None = all."""
        r = None if resident is None else np.ascontiguousarray(resident, np.uint8)
        check(self.lib.rmoe_set_route_config(self.handle, int(cache_route), route_j, route_m, _ptr(r)))

    def set_profiling(self, on: bool = True):
        check(self.lib.rmoe_layer_set_profiling(self.handle, int(on)))

    def profile(self) -> dict:
        """Summed per-stage device milliseconds since the last read, and the call count."""
        p = Profile()
        check(self.lib.rmoe_layer_get_profile(self.handle, C.byref(p)))
        out = {name: p.stage_ms[i] for i, name in enumerate(STAGES)}
        out["calls"] = p.calls
        return out

    # ---- weights (reference byte layout; host or device buffers)
    def upload_router(self, w):
        dt = DT_BF16 if ((torch is not None and isinstance(w, torch.Tensor) and w.dtype == torch.bfloat16)
                         or (isinstance(w, np.ndarray) and w.dtype == np.uint16)) else DT_F32
        check(self.lib.rmoe_upload_router(self.handle, _ptr(w), dt, _nbytes(w)))

    def upload_router_bias(self, b):
        b = np.ascontiguousarray(b, np.float32)
        check(self.lib.rmoe_upload_router_bias(self.handle, _ptr(b), b.size))

    def upload_expert(self, eid, gate, gate_scale, up, up_scale, down, down_scale):
        check(self.lib.rmoe_upload_expert(self.handle, eid, _ptr(gate), _nbytes(gate),
                                          _ptr(gate_scale), _nbytes(gate_scale), _ptr(up),
                                          _nbytes(up), _ptr(up_scale), _nbytes(up_scale),
                                          _ptr(down), _nbytes(down), _ptr(down_scale),
                                          _nbytes(down_scale)))

    def upload_expert_fused(self, eid, gate_up, gate_up_scale, down, down_scale):
        check(self.lib.rmoe_upload_expert_fused(self.handle, eid, _ptr(gate_up), _nbytes(gate_up),
                                                _ptr(gate_up_scale), _nbytes(gate_up_scale),
                                                _ptr(down), _nbytes(down), _ptr(down_scale),
                                                _nbytes(down_scale)))

    def upload_shared(self, gate, gate_scale, up, up_scale, down, down_scale, shared_gate=None):
        sg = None if shared_gate is None else np.ascontiguousarray(shared_gate, np.float32)
        check(self.lib.rmoe_upload_shared(self.handle, _ptr(gate), _nbytes(gate), _ptr(gate_scale),
                                          _nbytes(gate_scale), _ptr(up), _nbytes(up),
                                          _ptr(up_scale), _nbytes(up_scale), _ptr(down),
                                          _nbytes(down), _ptr(down_scale), _nbytes(down_scale),
                                          _ptr(sg)))

    def load_expert(self, shards: "Shards", naming: str, layer_index: int, eid: int):
        """One routed expert of a checkpoint layer into this layer (rmoe_load_expert)."""
        check(self.lib.rmoe_load_expert(self.handle, shards.handle, _lib.NAMINGS[naming], layer_index, eid))

    def load_experts(self, shards: "Shards", naming: str, layer_index: int):
        """Every expert resident on this layer's EP rank."""
        st = self.stats()
        for eid in range(st["local_expert_begin"], st["local_expert_end"]):
            self.load_expert(shards, naming, layer_index, eid)

    def load_moe_weights(self, shards: "Shards", family: str, layer_index: int):
        """Router (+ GLM correction bias) and shared expert of a checkpoint layer."""
        check(self.lib.rmoe_load_moe_weights(self.handle, shards.handle, _lib.FAMILIES[family], layer_index))

    def upload_expert_dict(self, eid, ex: dict):
        self.upload_expert(eid, ex["gate"], ex["gate_scale"], ex["up"], ex["up_scale"],
                           ex["down"], ex["down_scale"])

    # ---- hot path (CUDA tensors)
    def route(self, x, stream=None):
        _require_cuda(x)
        T = x.shape[0]
        ids = torch.empty((T, self.topk), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.topk), dtype=torch.float32, device=x.device)
        check(self.lib.rmoe_route(self.handle, _ptr(x), _dtype_code(x), T, _ptr(ids), _ptr(w),
                                  _stream(stream)))
        return ids, w

    def dispatch(self, ids, stream=None):
        _require_cuda(ids)
        T = ids.shape[0]
        n_loc = self.n_experts // max(1, self.desc.ep_size)
        dev = ids.device
        counts = torch.zeros(n_loc, dtype=torch.int32, device=dev)
        offsets = torch.zeros(n_loc + 1, dtype=torch.int32, device=dev)
        perm = torch.zeros(T * self.topk, dtype=torch.int32, device=dev)
        uniq = torch.zeros(n_loc, dtype=torch.int32, device=dev)
        n_uniq = torch.zeros(1, dtype=torch.int32, device=dev)
        check(self.lib.rmoe_dispatch(self.handle, _ptr(ids), T, _ptr(counts), _ptr(offsets),
                                     _ptr(perm), _ptr(uniq), _ptr(n_uniq), _stream(stream)))
        return {"counts": counts, "offsets": offsets, "perm_token": perm,
                "uniq": uniq, "n_uniq": n_uniq}

    def moe_forward(self, x, out=None, return_routing=False, stream=None):
        _require_cuda(x)
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
        ids = w = None
        if return_routing:
            ids = torch.empty((T, self.topk), dtype=torch.int32, device=x.device)
            w = torch.empty((T, self.topk), dtype=torch.float32, device=x.device)
        check(self.lib.rmoe_moe_forward(self.handle, _ptr(x), _dtype_code(x), T, _ptr(out),
                                        _ptr(ids), _ptr(w), _stream(stream)))
        return (out, ids, w) if return_routing else out

    def forward_routed(self, x, ids, weights, with_shared=True, out=None, stream=None):
        """The expert loop with given routing (apply_single_expert over a Routing,
        src/glm52/moe.rs:463-513): out[t] = sum_j w[t][j] * expert_{ids[t][j]}(x[t]) (+ shared).
        Slots with id -1 or a non-resident expert contribute nothing."""
        _require_cuda(x, ids, weights)
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
        check(self.lib.rmoe_moe_forward_routed(self.handle, _ptr(x), _dtype_code(x), T, _ptr(ids), _ptr(weights),
                                               1 if with_shared else 0, _ptr(out), _stream(stream)))
        return out

    def row_payload(self, x, stream=None):
        """What expert parallelism sends for rows x [T, H]: on the MXFP4 tensor-core path their
        activation terms (rmoe_activation_terms: uint8 [T, 4 * H/2] and [T, 4 * H/32], 17 bytes per
        32 columns), else x itself."""
        _require_cuda(x)
        if getattr(self, "_terms_ok", True):
            T, H = x.shape[0], self.hidden
            terms = torch.empty((T, 2 * H), dtype=torch.uint8, device=x.device)
            scales = torch.empty((T, H // 8), dtype=torch.uint8, device=x.device)
            st = self.lib.rmoe_activation_terms(self.handle, _ptr(x), _dtype_code(x), T, _ptr(terms), _ptr(scales),
                                                _stream(stream))
            if st == _lib.RMOE_NOT_SUPPORTED:
                self._terms_ok = False
            else:
                check(st)
                return (terms, scales)
        return (x,)

    def forward_routed_payload(self, payload, ids, weights, out=None, stream=None):
        """forward_routed without the shared expert on rows given as row_payload() returned them
        (gathered from every rank): the same outputs bit for bit."""
        if len(payload) == 1:
            return self.forward_routed(payload[0], ids, weights, with_shared=False, out=out, stream=stream)
        terms, scales = payload
        _require_cuda(terms, scales, ids, weights)
        T = terms.shape[0]
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=terms.device)
        check(self.lib.rmoe_moe_forward_routed_terms(self.handle, _ptr(terms.contiguous()), _ptr(scales.contiguous()), T,
                                                     _ptr(ids), _ptr(weights), _ptr(out), _stream(stream)))
        return out

    def sum_rank_parts(self, parts, last=None, out=None, stream=None):
        """parts [N, T, H] f32 -> out [T, H] = parts[0] + ... + parts[N-1] (+ last), in rank
        order (rmoe_sum_rank_parts): expert parallelism's owner-side combine."""
        _require_cuda(parts)
        parts = parts.contiguous()
        n, T, H = parts.shape
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=parts.device)
        check(self.lib.rmoe_sum_rank_parts(_ptr(out), _ptr(parts), n, T, H,
                                           _ptr(last) if last is not None else None, _stream(stream)))
        return out

    def upload_latent(self, down_proj, up_proj, norm=None, eps=1e-5):
        """LatentMoeWeights (src/kimi_k3/moe.rs:42-56): down_proj [hidden, router_hidden] and
        up_proj [router_hidden, hidden] (f32 numpy, or bf16 bits as uint16 numpy / bf16 torch),
        norm [hidden] f32 or None."""
        down = down_proj if torch is not None and isinstance(down_proj, torch.Tensor) else np.ascontiguousarray(down_proj)
        up = up_proj if torch is not None and isinstance(up_proj, torch.Tensor) else np.ascontiguousarray(up_proj)
        dt = _dtype_code(down)
        nrm = None if norm is None else np.ascontiguousarray(norm, np.float32)
        check(self.lib.rmoe_upload_latent(self.handle, _ptr(down), _ptr(up), dt, _ptr(nrm), float(eps)))

    def latent_moe(self, x, out=None, return_routing=False, stream=None):
        """kimi_k3::moe::latent_moe (src/kimi_k3/moe.rs:64-116): x [T, router_hidden] -> out
        [T, router_hidden] f32 (routed experts only, the caller adds the shared expert)."""
        _require_cuda(x)
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.router_hidden), dtype=torch.float32, device=x.device)
        ids = w = None
        if return_routing:
            ids = torch.empty((T, self.topk), dtype=torch.int32, device=x.device)
            w = torch.empty((T, self.topk), dtype=torch.float32, device=x.device)
        check(self.lib.rmoe_latent_moe(self.handle, _ptr(x), _dtype_code(x), T, _ptr(out), _ptr(ids), _ptr(w),
                                       _stream(stream)))
        return (out, ids, w) if return_routing else out

    def moe_forward_host(self, x, out=None):
        """Host buffers in and out (x: f32 or bf16 bits as uint16; pinned torch tensors work
        too): the signature rabbit's moe_forward call sites have."""
        T = x.shape[0]
        if out is None:
            out = np.empty((T, self.hidden), np.float32)
        check(self.lib.rmoe_moe_forward_host(self.handle, _ptr(x), _dtype_code(x), T, _ptr(out),
                                             None, None))
        return out


# ---- generic matmul_qt entry points (device tensors), reference argument order
def matmul_mxfp4(y, x, data, block_scale, s, i, o, stream=None):
    """kernels::matmul_mxfp4 (src/kernels.rs:233-244)."""
    _require_cuda(y, x, data, block_scale)
    check(_lib.load().rmoe_matmul_mxfp4(_ptr(y), _ptr(x), _dtype_code(x), _ptr(data),
                                        _ptr(block_scale), s, i, o, _stream(stream)))
    return y


def matmul_mxfp4_tc(y, x, data, block_scale, s, i, o, stream=None):
    """matmul_mxfp4 on the tcgen05 tensor cores (weights as stored; x as a 4-term E2M1 expansion)."""
    _require_cuda(y, x, data, block_scale)
    check(_lib.load().rmoe_matmul_mxfp4_tc(_ptr(y), _ptr(x), _dtype_code(x), _ptr(data),
                                           _ptr(block_scale), s, i, o, _stream(stream)))
    return y


def matmul_mxfp4_noalloc(y, x, data, block_scale, s, i, o, stream=None):
    """matmul_mxfp4 with its activation scratch in a fixed device array (no allocation; shapes
    whose scratch exceeds the array raise INVALID_ARG; overlapping calls on one device race)."""
    _require_cuda(y, x, data, block_scale)
    check(_lib.load().rmoe_matmul_mxfp4_noalloc(_ptr(y), _ptr(x), _dtype_code(x), _ptr(data),
                                                _ptr(block_scale), s, i, o, _stream(stream)))
    return y


def matmul_i4_grouped(y, x, q4, scale, group_size, s, i, o, stream=None):
    """kernels::matmul_i4_grouped (src/kernels.rs:276-296); scale f32 or bf16."""
    _require_cuda(y, x, q4, scale)
    sdt = DT_BF16 if scale.dtype == torch.bfloat16 else DT_F32
    check(_lib.load().rmoe_matmul_i4_grouped(_ptr(y), _ptr(x), _dtype_code(x), _ptr(q4), _ptr(scale),
                                             sdt, group_size, s, i, o, _stream(stream)))
    return y


def matmul(y, x, w, s, i, o, stream=None):
    """kernels::matmul (src/kernels.rs:113-124), bit-exact per element."""
    _require_cuda(y, x, w)
    check(_lib.load().rmoe_matmul_f32(_ptr(y), _ptr(x), _dtype_code(x), _ptr(w), _dtype_code(w),
                                      s, i, o, _stream(stream)))
    return y


def matmul_qt(y, x, kind: str, data, scale, s, i, o, group_size=32, stream=None):
    """kernels::matmul_qt (src/kernels.rs:1104-1132) for a weight of QT kind `kind`
    ("f32", "i8", "i4", "i2", "i4_grouped", "mxfp4")."""
    _require_cuda(y, x, data)
    check(_lib.load().rmoe_matmul_qt(_ptr(y), _ptr(x), _dtype_code(x), _lib.QT_KINDS[kind], _ptr(data), _ptr(scale),
                                     group_size, s, i, o, _stream(stream)))
    return y


def synth_bytes(t, key: int, mode: int = 0, lo: int = 0, hi: int = 0, stream=None):
    """Fill a CUDA uint8 tensor with the seeded synthetic byte stream (see synth.py)."""
    _require_cuda(t)
    check(_lib.load().rmoe_synth_bytes(_ptr(t), _nbytes(t), C.c_uint64(key), mode, lo, hi,
                                       _stream(stream)))
    return t


class Shards:
    """A checkpoint's .safetensors shards (rabbit's Shards::open_multi): headers parsed once,
    tensors read on demand. Host-only: works without a GPU."""

    def __init__(self, *dirs):
        self.lib = _lib.load()
        arr = (C.c_char_p * len(dirs))(*[os.fsencode(d) for d in dirs])
        h = C.c_void_p()
        check(self.lib.rmoe_shards_open(arr, len(dirs), C.byref(h)))
        self.handle = h

    def close(self):
        if self.handle:
            self.lib.rmoe_shards_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self):
        n = C.c_int64()
        check(self.lib.rmoe_shards_count(self.handle, C.byref(n)))
        return n.value

    def tensor(self, name: str) -> dict:
        """dtype, shape and byte count of one tensor (RmoeError MISSING_TENSOR when absent)."""
        dt = C.create_string_buffer(_lib.DTYPE_NAME_BYTES)
        shape = (C.c_uint64 * _lib.MAX_TENSOR_DIMS)()
        nd, nb = C.c_int32(), C.c_uint64()
        check(self.lib.rmoe_shards_tensor(self.handle, name.encode(), dt, shape, C.byref(nd), C.byref(nb)))
        return {"dtype": dt.value.decode(), "shape": [shape[i] for i in range(nd.value)], "nbytes": nb.value}

    def has(self, name: str) -> bool:
        try:
            self.tensor(name)
            return True
        except RmoeError as e:
            if e.status_name == "MISSING_TENSOR":
                return False
            raise

    def read_raw(self, name: str) -> np.ndarray:
        """The tensor's bytes verbatim (uint8)."""
        out = np.empty(self.tensor(name)["nbytes"], np.uint8)
        check(self.lib.rmoe_shards_read_raw(self.handle, name.encode(), out.ctypes.data, out.nbytes))
        return out
