"""The reference's in-test generators, restated so its known-answer tests can be replayed.

xorshift / random_vec: src/kernels.rs:1311-1321 and src/quant.rs:551-561 (f32 arithmetic);
lcg_logits: src/qwen38/moe.rs:103-111.
"""
import numpy as np

_U32MAX_F32 = np.float32(4294967295.0)


def xorshift_stream(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        v = (np.float32(s) / _U32MAX_F32 - np.float32(0.5)) * np.float32(2.0)
        out[i] = v
    return out


def random_vec(n: int, seed: int) -> np.ndarray:
    return xorshift_stream(seed, n)


def lcg_logits(n: int, seed: int) -> np.ndarray:
    s = max(seed, 1) & 0xFFFFFFFF
    out = np.empty(n, np.float32)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(((s >> 8) % 2000)) / np.float32(100.0) - np.float32(10.0)
    return out


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
