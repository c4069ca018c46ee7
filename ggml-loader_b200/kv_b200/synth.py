"""Seeded synthetic inputs of the path: which generator stream feeds which tensor.

normal(seed, stream, i) is the Irwin-Hall sum of twelve 16-bit uniforms from a
splitmix64 stream (mean 0, variance 1, exact in F32); uniform(seed, stream, i)
is a 23-bit uniform.  The device generator (kv_fill_synthetic,
kv_gen_normal_device) and this numpy version produce identical bits.
"""
import numpy as np

STREAM_CACHE = 1 << 20            # + 2*layer (K) / + 2*layer + 1 (V)
STREAM_QKV = 2 << 20              # + step*1024 + layer: fused rows [n_new][row_width]
STREAM_NORM = 3 << 20             # + 2*layer (q gamma) / + 2*layer + 1 (k gamma)

_M30 = np.uint64(30)
_M27 = np.uint64(27)
_M31 = np.uint64(31)
_C1 = np.uint64(0xBF58476D1CE4E5B9)
_C2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _mix64(x):
    with np.errstate(over="ignore"):
        x = x ^ (x >> _M30)
        x = x * _C1
        x = x ^ (x >> _M27)
        x = x * _C2
        x = x ^ (x >> _M31)
    return x


def _key(seed, stream):
    with np.errstate(over="ignore"):
        s = _mix64(np.uint64(stream) + np.uint64(0x6B76B200))
        return _mix64(np.uint64(seed) ^ s)


def bits(seed, stream, idx):
    idx = np.asarray(idx, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix64(_key(seed, stream) + idx * _GOLD)


def normal(seed, stream, n, idx0=0):
    idx = np.arange(idx0, idx0 + n, dtype=np.uint64) * np.uint64(3)
    key = _key(seed, stream)
    total = np.zeros(n, dtype=np.uint64)
    mask = np.uint64(0xFFFF)
    with np.errstate(over="ignore"):
        for j in range(3):
            w = _mix64(key + (idx + np.uint64(j)) * _GOLD)
            for sh in (0, 16, 32, 48):
                total += (w >> np.uint64(sh)) & mask
    s = (total + np.uint64(6)).astype(np.float32)
    return (s * np.float32(1.0 / 65536.0) - np.float32(6.0)).astype(np.float32)


def uniform(seed, stream, n, lo, hi, idx0=0):
    b = bits(seed, stream, np.arange(idx0, idx0 + n, dtype=np.uint64))
    u = (b >> np.uint64(41)).astype(np.float32) * np.float32(1.0 / 8388608.0)
    return (np.float32(lo) + u * (np.float32(hi) - np.float32(lo))).astype(np.float32)


def qkv_rows(spec, step, layer, n_new):
    """One layer's fused input rows [n_new][row_width] for decode step `step`."""
    w = (spec["n_head"] + 2 * spec["n_head_kv"]) * spec["head_dim"]
    return normal(spec["seed"], STREAM_QKV + step * 1024 + layer, n_new * w).reshape(n_new, w)


def norm_weights(spec, layer):
    d = spec["head_dim"]
    q = uniform(spec["seed"], STREAM_NORM + 2 * layer, d, 0.5, 1.5)
    k = uniform(spec["seed"], STREAM_NORM + 2 * layer + 1, d, 0.5, 1.5)
    return q, k
