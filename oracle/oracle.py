"""ctypes view of oracle/liboracle.so -- the CPU restatement of rabbit's routed-MoE path.

TEST INFRASTRUCTURE ONLY. Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm may import this module; the product package ``rabbit_b200`` never does.
Each wrapper names the reference function (ferrumox/rabbit v0.29.1) its C body restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
U8P = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
SZ = C.c_size_t


class OrcExpert(C.Structure):
    _fields_ = [("gate", C.c_void_p), ("gate_scale", C.c_void_p),
                ("up", C.c_void_p), ("up_scale", C.c_void_p),
                ("down", C.c_void_p), ("down_scale", C.c_void_p)]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (the checker, not the product)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.orc_e2m1_decode.restype = C.c_float
        L.orc_e2m1_decode.argtypes = [C.c_uint8]
        L.orc_e8m0_decode.restype = C.c_float
        L.orc_e8m0_decode.argtypes = [C.c_uint8]
        L.orc_e2m1_encode.restype = C.c_uint8
        L.orc_e2m1_encode.argtypes = [C.c_float]
        L.orc_choose_block_scale.argtypes = [C.c_float, C.POINTER(C.c_uint8), C.POINTER(C.c_float)]
        L.orc_pack_mxfp4.argtypes = [F32P, U8P, U8P, SZ, SZ]
        L.orc_quant_int4_grouped.argtypes = [F32P, SZ, SZ, C.c_int, SZ, U8P, F32P]
        L.orc_row_f32_mxfp4.argtypes = [U8P, U8P, SZ, SZ, F32P]
        L.orc_matmul_f32.argtypes = [F32P, F32P, F32P, SZ, SZ, SZ]
        L.orc_matmul_mxfp4.argtypes = [F32P, F32P, U8P, U8P, SZ, SZ, SZ]
        L.orc_matmul_mxfp4_avx512.argtypes = [F32P, F32P, U8P, U8P, SZ, SZ, SZ]
        L.orc_matmul_i4_grouped.argtypes = [F32P, F32P, U8P, F32P, SZ, SZ, SZ, SZ]
        L.orc_siluf.restype = C.c_float
        L.orc_siluf.argtypes = [C.c_float]
        L.orc_sigmoid.restype = C.c_float
        L.orc_sigmoid.argtypes = [C.c_float]
        L.orc_qwen_route.restype = SZ
        L.orc_qwen_route.argtypes = [F32P, SZ, SZ, I32P, F32P]
        L.orc_top2_sum.restype = C.c_float
        L.orc_top2_sum.argtypes = [F32P, SZ]
        L.orc_rank_top_grouped.restype = SZ
        L.orc_rank_top_grouped.argtypes = [F32P, F32P, SZ, SZ, SZ, SZ, I32P, F32P]
        L.orc_glm_route.argtypes = [F32P, F32P, F32P, SZ, SZ, SZ, SZ, SZ, SZ, C.c_int, C.c_float,
                                    I32P, F32P]
        L.orc_glm_route_cache.argtypes = [F32P, F32P, F32P, SZ, SZ, SZ, SZ, SZ, SZ, C.c_void_p, C.c_int,
                                          C.c_float, C.c_void_p, C.c_void_p]
        L.orc_cache_route_select.restype = SZ
        L.orc_cache_route_select.argtypes = [F32P, F32P, SZ, SZ, SZ, SZ, C.c_void_p, I32P, F32P]
        L.orc_qrow_i8.restype = C.c_float
        L.orc_qrow_i8.argtypes = [F32P, SZ, C.c_void_p]
        L.orc_dot_i8i8.restype = C.c_int32
        L.orc_dot_i8i8.argtypes = [C.c_void_p, C.c_void_p, SZ]
        L.orc_dot_i4i8.restype = C.c_int32
        L.orc_dot_i4i8.argtypes = [C.c_void_p, C.c_void_p, SZ]
        L.orc_matmul_qt_kind.argtypes = [F32P, F32P, C.c_int, C.c_void_p, C.c_void_p, SZ, SZ, SZ, SZ]
        L.orc_unique_experts.restype = SZ
        L.orc_unique_experts.argtypes = [I32P, SZ, SZ, I32P]
        L.orc_expert_rows.restype = SZ
        L.orc_expert_rows.argtypes = [I32P, F32P, SZ, SZ, C.c_int32, I32P, F32P]
        L.orc_moe_forward_qwen.argtypes = [F32P, SZ, SZ, SZ, SZ, SZ, SZ, F32P, C.c_void_p,
                                           C.POINTER(OrcExpert), C.c_void_p, C.c_void_p, C.c_int,
                                           SZ, F32P, C.c_void_p, C.c_void_p]
        L.orc_moe_forward_qwen_fast.argtypes = [F32P, SZ, SZ, SZ, SZ, SZ, SZ, F32P, C.c_void_p,
                                                C.POINTER(OrcExpert), C.c_void_p, C.c_void_p,
                                                F32P, C.c_void_p, C.c_void_p]
        L.orc_moe_glm.argtypes = [F32P, SZ, SZ, SZ, SZ, SZ, SZ, F32P, F32P, SZ, SZ, C.c_int,
                                  C.c_float, C.POINTER(OrcExpert), C.c_void_p, C.c_int, SZ, F32P,
                                  C.c_void_p, C.c_void_p]
        L.orc_has_avx512.restype = C.c_int
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data


# ---------------------------------------------------------------- formats (quant.rs)
def e2m1_decode(nibble: int) -> float:
    return lib().orc_e2m1_decode(nibble)


def e8m0_decode(byte: int) -> float:
    return lib().orc_e8m0_decode(byte)


def e2m1_encode(v: float) -> int:
    return lib().orc_e2m1_encode(v)


def choose_block_scale(amax: float):
    b, s = C.c_uint8(), C.c_float()
    lib().orc_choose_block_scale(amax, C.byref(b), C.byref(s))
    return b.value, s.value


def pack_mxfp4(w, rows, cols):
    w = _f32(w).reshape(-1)
    q = np.zeros(rows * ((cols + 1) // 2), np.uint8)
    bs = np.zeros(rows * ((cols + 31) // 32), np.uint8)
    lib().orc_pack_mxfp4(w, q, bs, rows, cols)
    return q, bs


def quant_int4_grouped(w, rows, cols, bits, gs):
    w = _f32(w).reshape(-1)
    q = np.zeros(rows * ((cols + 1) // 2), np.uint8)
    sc = np.zeros(rows * ((cols + gs - 1) // gs), np.float32)
    lib().orc_quant_int4_grouped(w, rows, cols, bits, gs, q, sc)
    return q, sc


def row_f32_mxfp4(data, bs, cols, row):
    out = np.zeros(cols, np.float32)
    lib().orc_row_f32_mxfp4(np.ascontiguousarray(data), np.ascontiguousarray(bs), cols, row, out)
    return out


# ---------------------------------------------------------------- kernels.rs
def matmul(x, w, s, i, o):
    y = np.zeros(s * o, np.float32)
    lib().orc_matmul_f32(y, _f32(x).reshape(-1), _f32(w).reshape(-1), s, i, o)
    return y.reshape(s, o)


def matmul_mxfp4(x, data, bs, s, i, o, tier="scalar"):
    y = np.zeros(s * o, np.float32)
    fn = lib().orc_matmul_mxfp4 if tier == "scalar" else lib().orc_matmul_mxfp4_avx512
    fn(y, _f32(x).reshape(-1), np.ascontiguousarray(data).reshape(-1),
       np.ascontiguousarray(bs).reshape(-1), s, i, o)
    return y.reshape(s, o)


QT_KINDS = {"f32": 0, "i8": 1, "i4": 2, "i2": 3, "i4_grouped": 4, "mxfp4": 5}


def qrow_i8(x):
    """kernels::qrow_i8 -> (int8 array, scale)."""
    x = _f32(x).reshape(-1)
    q = np.zeros(x.size, np.int8)
    sc = lib().orc_qrow_i8(x, x.size, q.ctypes.data)
    return q, np.float32(sc)


def dot_i8i8(w, x):
    w, x = np.ascontiguousarray(w, np.int8), np.ascontiguousarray(x, np.int8)
    return int(lib().orc_dot_i8i8(w.ctypes.data, x.ctypes.data, w.size))


def dot_i4i8(w4, x, n):
    w4, x = np.ascontiguousarray(w4, np.uint8), np.ascontiguousarray(x, np.int8)
    return int(lib().orc_dot_i4i8(w4.ctypes.data, x.ctypes.data, n))


def matmul_qt(x, kind, data, scale, s, i, o, gs=32):
    """kernels::matmul_qt for a QT of `kind` (QT_KINDS): y [s, o] f32."""
    y = np.zeros(s * o, np.float32)
    d = np.ascontiguousarray(data)
    sc = np.ascontiguousarray(scale)
    lib().orc_matmul_qt_kind(y, _f32(x).reshape(-1), QT_KINDS[kind], d.ctypes.data, sc.ctypes.data, gs, s, i, o)
    return y.reshape(s, o)


def matmul_i4_grouped(x, q4, scale, gs, s, i, o):
    y = np.zeros(s * o, np.float32)
    lib().orc_matmul_i4_grouped(y, _f32(x).reshape(-1), np.ascontiguousarray(q4).reshape(-1),
                                _f32(scale).reshape(-1), gs, s, i, o)
    return y.reshape(s, o)


def siluf(x: float) -> float:
    return lib().orc_siluf(x)


def sigmoid(x: float) -> float:
    return lib().orc_sigmoid(x)


# ---------------------------------------------------------------- routers
def qwen_route(logits, topk):
    logits = _f32(logits).reshape(-1)
    n = logits.size
    k = min(topk, n)
    ids = np.zeros(max(k, 1), np.int32)
    w = np.zeros(max(k, 1), np.float32)
    kk = lib().orc_qwen_route(logits, n, topk, ids, w)
    return [(int(ids[j]), float(w[j])) for j in range(kk)]


def top2_sum(vals):
    v = _f32(vals)
    return lib().orc_top2_sum(v, v.size)


def rank_top_grouped(choice, logit, k, n_group, topk_group):
    c, l = _f32(choice), _f32(logit)
    ids = np.zeros(max(k, 1), np.int32)
    w = np.zeros(max(k, 1), np.float32)
    kk = lib().orc_rank_top_grouped(c, l, c.size, k, n_group, topk_group, ids, w)
    return [(int(ids[j]), float(w[j])) for j in range(kk)]


def glm_route_cache(x, router, bias, s, d, e, k, route_j, route_m, resident, norm_topk, routed_scale):
    """CACHE_ROUTE selection (glm52::moe::route_cache_aware); resident: [E] bool or None."""
    ids = np.zeros(s * k, np.int32)
    w = np.zeros(s * k, np.float32)
    res = None if resident is None else np.ascontiguousarray(resident, np.uint8)
    lib().orc_glm_route_cache(_f32(x).reshape(-1), _f32(router).reshape(-1), _f32(bias).reshape(-1), s, d, e, k,
                              route_j, route_m, res.ctypes.data if res is not None else None, int(norm_topk),
                              routed_scale, ids.ctypes.data, w.ctypes.data)
    return ids.reshape(s, k), w.reshape(s, k)


def cache_route_select(choice, logit, k, route_j, route_m, resident=None):
    """glm52::moe::cache_route_select on given choice/logit vectors -> [(id, weight)]."""
    choice, logit = _f32(choice), _f32(logit)
    ids = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    res = None if resident is None else np.ascontiguousarray(resident, np.uint8)
    n = lib().orc_cache_route_select(choice, logit, choice.size, k, route_j, route_m,
                                     res.ctypes.data if res is not None else None, ids, w)
    return [(int(ids[j]), float(w[j])) for j in range(n)]


def glm_route(x, router, bias, s, d, e, k, n_group, topk_group, norm_topk, routed_scale):
    ids = np.zeros(s * k, np.int32)
    w = np.zeros(s * k, np.float32)
    lib().orc_glm_route(_f32(x).reshape(-1), _f32(router).reshape(-1), _f32(bias).reshape(-1),
                        s, d, e, k, n_group, topk_group, int(norm_topk), routed_scale, ids, w)
    return ids.reshape(s, k), w.reshape(s, k)


def unique_experts(ids):
    ids = np.ascontiguousarray(ids, np.int32)
    s, k = ids.shape
    out = np.zeros(s * k + 1, np.int32)
    n = lib().orc_unique_experts(ids.reshape(-1), s, k, out)
    return out[:n].copy()


def expert_rows(ids, w, eid):
    ids = np.ascontiguousarray(ids, np.int32)
    w = _f32(w)
    s, k = ids.shape
    rows = np.zeros(s, np.int32)
    rw = np.zeros(s, np.float32)
    n = lib().orc_expert_rows(ids.reshape(-1), w.reshape(-1), s, k, eid, rows, rw)
    return rows[:n].copy(), rw[:n].copy()


# ---------------------------------------------------------------- layer forward
def _expert_struct(ex):
    """ex: dict with gate/gate_scale/up/up_scale/down/down_scale numpy arrays."""
    st = OrcExpert()
    for f, _ in OrcExpert._fields_:
        setattr(st, f, ex[f].ctypes.data)
    return st


def _experts_array(experts, n):
    arr = (OrcExpert * n)()
    keep = []
    for eid in range(n):
        ex = experts.get(eid) if isinstance(experts, dict) else experts[eid]
        if ex is None:
            continue
        arr[eid] = _expert_struct(ex)
        keep.append(ex)
    return arr, keep


def moe_forward_qwen(x, router, experts, e, k, inter, shared=None, shared_gate=None,
                     logit_bias=None, shared_inter=None, fmt=0, gs=32, tier="scalar"):
    """Qwen moe_forward (qwen38/generate.rs:262-351) minus the cache. ``experts`` maps expert id
    -> dict of byte arrays; only routed ids need to be present."""
    x = _f32(x)
    s, d = x.shape
    out = np.zeros(s * d, np.float32)
    kk = min(k, e)
    ids = np.zeros(s * kk, np.int32)
    w = np.zeros(s * kk, np.float32)
    arr, keep = _experts_array(experts, e)
    sh = _expert_struct(shared) if shared is not None else None
    sg = _f32(shared_gate) if shared_gate is not None else None
    lb = _f32(logit_bias) if logit_bias is not None else None
    shi = shared_inter if shared_inter is not None else inter
    if tier == "scalar":
        lib().orc_moe_forward_qwen(x.reshape(-1), s, d, e, k, inter, shi, _f32(router).reshape(-1),
                                   _ptr(lb), arr, C.addressof(sh) if sh is not None else None,
                                   _ptr(sg), fmt, gs, out, ids.ctypes.data, w.ctypes.data)
    else:
        lib().orc_moe_forward_qwen_fast(x.reshape(-1), s, d, e, k, inter, shi,
                                        _f32(router).reshape(-1), _ptr(lb), arr,
                                        C.addressof(sh) if sh is not None else None, _ptr(sg),
                                        out, ids.ctypes.data, w.ctypes.data)
    del keep
    return out.reshape(s, d), ids.reshape(s, kk), w.reshape(s, kk)


def moe_glm(x, router, bias, experts, e, k, inter, n_group, topk_group, norm_topk, routed_scale,
            shared=None, shared_inter=None, fmt=1, gs=32):
    """GLM moe() (glm52/moe.rs:350-451) minus the cache."""
    x = _f32(x)
    s, d = x.shape
    out = np.zeros(s * d, np.float32)
    ids = np.zeros(s * k, np.int32)
    w = np.zeros(s * k, np.float32)
    arr, keep = _experts_array(experts, e)
    sh = _expert_struct(shared) if shared is not None else None
    shi = shared_inter if shared_inter is not None else inter
    lib().orc_moe_glm(x.reshape(-1), s, d, e, k, inter, shi, _f32(router).reshape(-1),
                      _f32(bias).reshape(-1), n_group, topk_group, int(norm_topk), routed_scale,
                      arr, C.addressof(sh) if sh is not None else None, fmt, gs, out,
                      ids.ctypes.data, w.ctypes.data)
    del keep
    return out.reshape(s, d), ids.reshape(s, k), w.reshape(s, k)


# ---------------------------------------------------------------- Kimi K3 latent MoE
def act_mul(g, u, act=("silu",)):
    """glm52::moe::Activation::combine (src/glm52/moe.rs:58-70) elementwise in f32: SiLU via the
    C oracle's siluf, or ("situ", beta, linear_beta) = beta tanh(g / beta) sigmoid(g) * u'
    with u' = lb tanh(u / lb) when lb is not None (kimi_linear::ops::situ_and_mul,
    src/kimi_linear/ops.rs); numpy's float32 tanh/exp stand for Rust's f32 libm calls."""
    g = _f32(g)
    u = _f32(u)
    if act[0] == "silu":
        sg = np.array([siluf(float(v)) for v in g.reshape(-1)], np.float32).reshape(g.shape)
        return (sg * u).astype(np.float32)
    beta, lb = np.float32(act[1]), act[2]
    if lb is not None:
        lb = np.float32(lb)
        u = (lb * np.tanh(u / lb)).astype(np.float32)
    sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    situ = ((beta * np.tanh(g / beta)).astype(np.float32) * sig).astype(np.float32)
    return (situ * u).astype(np.float32)


def rmsnorm_rows(v, w, eps):
    """kimi_linear::ops::rmsnorm (src/kimi_linear/ops.rs:46-53) on each row: the mean of squares
    summed sequentially in f64, r = 1 / sqrt(f32(ms / n) + eps) in f32, v *= r * w."""
    v = _f32(v).copy()
    w = _f32(w)
    n = v.shape[1]
    for row in v:
        ms = np.add.accumulate(row.astype(np.float64) ** 2)[-1]
        r = np.float32(1.0) / np.sqrt(np.float32(ms / n) + np.float32(eps))
        row *= (r * w).astype(np.float32)
    return v


def latent_moe(x, router, bias, experts, e, k, n_group, topk_group, norm_topk, routed_scale, down_proj,
               up_proj, norm, eps, moe_hidden, inter, act=("silu",), fmt=0, gs=32):
    """kimi_k3::moe::latent_moe (src/kimi_k3/moe.rs:64-116) minus the cache: route on the full-width
    x (glm52 routing, :84-86), x_latent = x . down_proj^T (:91-92), apply_single_expert for every
    unique expert in first-occurrence order at the latent width (:94-104,
    src/glm52/moe.rs:463-513), RMSNorm of each summed row if norm is not None (:106-110),
    out = routed . up_proj^T (:112). Returns (out, ids, weights)."""
    x = _f32(x)
    s, hf = x.shape
    ids, w = glm_route(x, router, bias, s, hf, e, k, n_group, topk_group, norm_topk, routed_scale)
    xl = matmul(x, down_proj, s, hf, moe_hidden)
    routed = np.zeros((s, moe_hidden), np.float32)
    for eid in unique_experts(ids):
        rows, rw = expert_rows(ids, w, int(eid))
        ex = experts[int(eid)]
        xs = np.ascontiguousarray(xl[rows])
        nr = len(rows)
        if fmt == 0:
            g = matmul_mxfp4(xs, ex["gate"], ex["gate_scale"], nr, moe_hidden, inter)
            u = matmul_mxfp4(xs, ex["up"], ex["up_scale"], nr, moe_hidden, inter)
            h = act_mul(g, u, act)
            y = matmul_mxfp4(h, ex["down"], ex["down_scale"], nr, inter, moe_hidden)
        else:
            g = matmul_i4_grouped(xs, ex["gate"], ex["gate_scale"], gs, nr, moe_hidden, inter)
            u = matmul_i4_grouped(xs, ex["up"], ex["up_scale"], gs, nr, moe_hidden, inter)
            h = act_mul(g, u, act)
            y = matmul_i4_grouped(h, ex["down"], ex["down_scale"], gs, nr, inter, moe_hidden)
        for r, t in enumerate(rows):
            routed[t] = (routed[t] + (np.float32(rw[r]) * y[r]).astype(np.float32)).astype(np.float32)
    if norm is not None:
        routed = rmsnorm_rows(routed, norm, eps)
    out = matmul(routed, up_proj, s, moe_hidden, hf)
    return out, ids, w


def set_threads(n: int):
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


def has_avx512() -> bool:
    return bool(lib().orc_has_avx512())
