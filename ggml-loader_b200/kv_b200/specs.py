"""Model shapes and per-architecture attention flags of the path.

The flags mirror load_hparams() in the reference (src/model.cpp:131-160):
  rope_neox   = arch != llama            (model.cpp:159)
  qkv_fused   = arch == phi3             (model.cpp:155)
  has_qkv_bias= arch == qwen2            (model.cpp:156)
  qk_norm     = arch in (qwen3, qwen35)  (model.cpp:157)
The five workloads are the benchmark configurations of this path (decode on a
prefilled cache, and one chunked-prefill case).
"""
import math

import numpy as np

ROPE_NORMAL = 0
ROPE_NEOX = 2


def arch_flags(arch):
    return {
        "rope_mode": ROPE_NORMAL if arch == "llama" else ROPE_NEOX,
        "qkv_fused": arch == "phi3",
        "qkv_bias": arch == "qwen2",
        "qk_norm": arch in ("qwen3", "qwen35"),
    }


def llama3_freq_factors(n_rot, base, factor, low_freq_factor=1.0, high_freq_factor=4.0, orig_ctx=8192):
    """Per-pair divisors of the RoPE frequency for llama-3.x context extension
    (Meta's published llama3 rope scaling; what a llama-3.1/3.2 gguf stores as
    rope_freqs.weight).  High-frequency pairs keep their frequency, low ones are
    divided by `factor`, and the band between is interpolated smoothly."""
    low_wavelen = orig_ctx / low_freq_factor
    high_wavelen = orig_ctx / high_freq_factor
    out = []
    for i in range(0, n_rot, 2):
        freq = 1.0 / (base ** (i / n_rot))
        wavelen = 2.0 * math.pi / freq
        if wavelen < high_wavelen:
            out.append(1.0)
        elif wavelen > low_wavelen:
            out.append(factor)
        else:
            smooth = (orig_ctx / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
            out.append(1.0 / ((1.0 - smooth) / factor + smooth))
    return np.asarray(out, dtype=np.float32)


def _spec(name, index, arch, n_layer, n_head, n_head_kv, head_dim, rope_base, n_ctx, n_past, n_new, steps,
          rope_freq_factors=None, rms_eps=1e-6, rope_mode=None, note=""):
    f = arch_flags(arch)
    return {
        "name": name, "index": index, "arch": arch,
        "n_layer": n_layer, "n_head": n_head, "n_head_kv": n_head_kv, "head_dim": head_dim,
        "n_rot": head_dim,
        "rope_mode": f["rope_mode"] if rope_mode is None else rope_mode,
        "rope_base": float(rope_base), "rope_freq_scale": 1.0, "rope_attn_factor": 1.0,
        "rope_ext_factor": 0.0, "rope_beta_fast": 0.0, "rope_beta_slow": 0.0, "n_ctx_orig": 0,
        "rope_freq_factors": rope_freq_factors,
        "qk_norm": f["qk_norm"], "rms_eps": rms_eps, "qkv_fused": f["qkv_fused"],
        "n_ctx": n_ctx, "n_past": n_past, "n_new": n_new, "steps": steps,
        "seed": 0x6B760000 + index, "note": note,
    }


def specs():
    """The five configurations, keyed by name."""
    s = [
        _spec("qwen2-0.5b", 0, "qwen2", 24, 14, 2, 64, 1e6, 4096, 2048, 1, 1,
              note="decode, cache rows 0..2047, one step at pos 2048"),
        _spec("llama3.2-3b", 1, "llama", 28, 24, 8, 128, 5e5, 32768, 32000, 1, 256,
              rope_freq_factors=llama3_freq_factors(128, 5e5, 32.0),
              note="decode, cache filled to 32000, 256 steps, llama3 factor-32 RoPE scaling"),
        _spec("phi3-mini", 2, "phi3", 32, 32, 32, 96, 1e4, 4096, 3968, 1, 128,
              note="MHA decode, fused QKV rows, head_dim 96, NEOX RoPE as the reference rotates phi3"),
        _spec("qwen3-8b-prefill", 3, "qwen3", 36, 32, 8, 128, 1e6, 40960, 16384, 512, 1,
              note="512-token chunk at offset 16384, QK-Norm eps 1e-6, gamma ~ U(0.5,1.5)"),
        _spec("llama3.1-8b-128k", 4, "llama", 32, 32, 8, 128, 5e5, 131072, 131000, 1, 64,
              rope_freq_factors=llama3_freq_factors(128, 5e5, 8.0),
              note="128k decode, cache filled to 131000, 64 steps, llama3 factor-8 RoPE scaling"),
    ]
    return {x["name"]: x for x in s}


def get(name):
    sp = specs()
    if name not in sp:
        raise KeyError("unknown config %r (have %s)" % (name, ", ".join(sp)))
    return dict(sp[name])


def row_width(spec):
    """Floats per token of one layer's fused Q|K|V input row."""
    return (spec["n_head"] + 2 * spec["n_head_kv"]) * spec["head_dim"]


def cache_bytes(spec, n_ctx=None):
    """kv_cache_bytes of the reference (model.cpp:869-885)."""
    n = spec["n_ctx"] if n_ctx is None else n_ctx
    return spec["n_layer"] * spec["head_dim"] * spec["n_head_kv"] * 2 * 2 * n
