"""rabbit_b200: a B200-native routed-MoE layer (router + top-k, dispatch, MXFP4/int4 SwiGLU
experts, weighted combine with the gated shared expert) behind a C ABI (include/rmoe.h)."""
from ._lib import RmoeError, load as load_library
from .moe import (Context, MoeLayer, Shards, matmul, matmul_i4_grouped, matmul_mxfp4, matmul_qt,
                  matmul_mxfp4_noalloc, matmul_mxfp4_tc, synth_bytes)

__all__ = ["RmoeError", "load_library", "Context", "MoeLayer", "Shards", "matmul", "matmul_mxfp4", "matmul_mxfp4_noalloc", "matmul_mxfp4_tc",
           "matmul_i4_grouped", "matmul_qt", "synth_bytes"]
