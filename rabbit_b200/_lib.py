"""ctypes binding of librmoe.so (include/rmoe.h). Loading fails loudly: there is no fallback."""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librmoe.so")

RMOE_OK = 0
RMOE_NOT_SUPPORTED = 6
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "SHAPE_MISMATCH", 3: "CUDA_ERROR", 4: "NCCL_ERROR",
                5: "TIMEOUT", 6: "NOT_SUPPORTED", 7: "OUT_OF_MEMORY", 8: "IO_ERROR", 9: "MISSING_TENSOR"}
ROUTER_SOFTMAX_TOPK, ROUTER_SIGMOID_GROUPED = 0, 1
FMT_MXFP4, FMT_I4_GROUPED = 0, 1
DT_F32, DT_BF16 = 0, 1
# rmoe_expert_naming / rmoe_model_family
NAMINGS = {"glm52": 0, "glm52_fused_gate_up": 1, "kimi_linear": 2, "kimi_k3": 3, "kimi_k3_mxfp4": 4,
           "qwen38_mxfp4": 5}
FAMILIES = {"qwen38": 0, "glm52": 1}
DTYPE_NAME_BYTES, MAX_TENSOR_DIMS = 16, 8
QT_KINDS = {"f32": 0, "i8": 1, "i4": 2, "i2": 3, "i4_grouped": 4, "mxfp4": 5}


class RmoeError(RuntimeError):
    """A non-OK rmoe_status, with rmoe_last_error()'s message (the Rust side's ModelError)."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.status_name}: {message}")


class LayerDesc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("moe_inter", C.c_int32), ("shared_inter", C.c_int32),
                ("n_experts", C.c_int32), ("topk", C.c_int32), ("router_kind", C.c_int32),
                ("n_group", C.c_int32), ("topk_group", C.c_int32), ("norm_topk", C.c_int32),
                ("routed_scale", C.c_float), ("weight_format", C.c_int32),
                ("group_size", C.c_int32), ("scale_dtype", C.c_int32),
                ("shared_gated", C.c_int32), ("max_tokens", C.c_int32), ("ep_rank", C.c_int32),
                ("ep_size", C.c_int32), ("activation", C.c_int32), ("situ_beta", C.c_float),
                ("situ_linear_beta", C.c_float), ("router_hidden", C.c_int32)]


class LayerStats(C.Structure):
    _fields_ = [("forward_calls", C.c_uint64), ("tokens_routed", C.c_uint64),
                ("kernel_launches", C.c_uint64), ("router_fallbacks", C.c_uint64), ("router_order_resolved", C.c_uint64),
                ("device_error_flags", C.c_uint64),
                ("device_bytes", C.c_uint64), ("local_expert_begin", C.c_int32),
                ("local_expert_end", C.c_int32)]


STAGES = ("router_logits", "topk", "prep", "dispatch", "gate_up", "quant_h", "down", "combine")


class Profile(C.Structure):
    _fields_ = [("calls", C.c_uint64), ("stage_ms", C.c_double * len(STAGES))]


# every entry point of include/rmoe.h: name -> (restype, argtypes)
P, SZ, I32, F32 = C.c_void_p, C.c_size_t, C.c_int32, C.c_float
PROTOTYPES = {
    "rmoe_last_error": (C.c_char_p, []),
    "rmoe_status_string": (C.c_char_p, [C.c_int]),
    "rmoe_abi_version": (C.c_int, []),
    "rmoe_init": (C.c_int, [C.c_int, C.POINTER(P)]),
    "rmoe_shutdown": (C.c_int, [P]),
    "rmoe_layer_create": (C.c_int, [P, C.POINTER(LayerDesc), C.POINTER(P)]),
    "rmoe_layer_destroy": (C.c_int, [P]),
    "rmoe_layer_get_stats": (C.c_int, [P, C.POINTER(LayerStats)]),
    "rmoe_layer_get_desc": (C.c_int, [P, C.POINTER(LayerDesc)]),
    "rmoe_shards_open": (C.c_int, [C.POINTER(C.c_char_p), I32, C.POINTER(P)]),
    "rmoe_shards_close": (C.c_int, [P]),
    "rmoe_shards_count": (C.c_int, [P, C.POINTER(C.c_int64)]),
    "rmoe_shards_tensor": (C.c_int, [P, C.c_char_p, P, P, C.POINTER(I32), C.POINTER(C.c_uint64)]),
    "rmoe_shards_read_raw": (C.c_int, [P, C.c_char_p, P, SZ]),
    "rmoe_load_expert": (C.c_int, [P, P, I32, I32, I32]),
    "rmoe_load_moe_weights": (C.c_int, [P, P, I32, I32]),
    "rmoe_layer_check": (C.c_int, [P, P]),
    "rmoe_layer_set_wait_limit": (C.c_int, [P, C.c_uint64]),
    "rmoe_set_route_config": (C.c_int, [P, I32, I32, I32, P]),
    "rmoe_layer_set_profiling": (C.c_int, [P, C.c_int]),
    "rmoe_layer_get_profile": (C.c_int, [P, C.POINTER(Profile)]),
    "rmoe_upload_router": (C.c_int, [P, P, I32, SZ]),
    "rmoe_upload_latent": (C.c_int, [P, P, P, I32, P, F32]),
    "rmoe_latent_moe": (C.c_int, [P, P, I32, I32, P, P, P, P]),
    "rmoe_upload_router_bias": (C.c_int, [P, P, SZ]),
    "rmoe_upload_expert": (C.c_int, [P, I32, P, SZ, P, SZ, P, SZ, P, SZ, P, SZ, P, SZ]),
    "rmoe_upload_expert_fused": (C.c_int, [P, I32, P, SZ, P, SZ, P, SZ, P, SZ]),
    "rmoe_upload_shared": (C.c_int, [P, P, SZ, P, SZ, P, SZ, P, SZ, P, SZ, P, SZ, P]),
    "rmoe_route": (C.c_int, [P, P, I32, I32, P, P, P]),
    "rmoe_dispatch": (C.c_int, [P, P, I32, P, P, P, P, P, P]),
    "rmoe_moe_forward": (C.c_int, [P, P, I32, I32, P, P, P, P]),
    "rmoe_moe_forward_routed": (C.c_int, [P, P, I32, I32, P, P, I32, P, P]),
    "rmoe_moe_forward_host": (C.c_int, [P, P, I32, I32, P, P, P]),
    "rmoe_sum_rank_parts": (C.c_int, [P, P, I32, C.c_int64, I32, P, P]),
    "rmoe_activation_terms": (C.c_int, [P, P, I32, I32, P, P, P]),
    "rmoe_moe_forward_routed_terms": (C.c_int, [P, P, P, I32, P, P, P, P]),
    "rmoe_matmul_mxfp4": (C.c_int, [P, P, I32, P, P, I32, I32, I32, P]),
    "rmoe_matmul_mxfp4_tc": (C.c_int, [P, P, I32, P, P, I32, I32, I32, P]),
    "rmoe_matmul_mxfp4_noalloc": (C.c_int, [P, P, I32, P, P, I32, I32, I32, P]),
    "rmoe_matmul_i4_grouped": (C.c_int, [P, P, I32, P, P, I32, I32, I32, I32, I32, P]),
    "rmoe_matmul_f32": (C.c_int, [P, P, I32, P, I32, I32, I32, I32, P]),
    "rmoe_matmul_qt": (C.c_int, [P, P, I32, I32, P, P, I32, I32, I32, I32, P]),
    "rmoe_synth_bytes": (C.c_int, [P, SZ, C.c_uint64, I32, I32, I32, P]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load librmoe.so. Raises ImportError when the CUDA library has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build the CUDA library first (python -m rabbit_b200.build). "
            "rabbit_b200 has no CPU fallback.")
    lib = C.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != RMOE_OK:
        msg = load().rmoe_last_error()
        raise RmoeError(status, msg.decode() if msg else "")
