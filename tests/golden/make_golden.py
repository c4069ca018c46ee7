"""Generate the committed golden fixtures of the path from the CPU oracle.

    python tests/golden/make_golden.py          # rewrite tests/golden/*.npz

Each case is one layer of one of the benchmark shapes at a reduced context
(so the fixture stays small): the cache rows [0, n_past) come from the seeded
generator, the new tokens' fused Q|K|V rows too, and the oracle produces the
appended K/V rows (F16 bits), the rotated Q (F32) and the attention output
(F32).  The reference has no fixtures of its own for this path (ggml is not
vendored), so these pin the oracle against regressions and give the GPU
tests a fixed target; the oracle itself restates ggml's op semantics
(see oracle/kv_oracle.h, assumptions A1-A5).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "ggml-loader_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

from kv_b200 import specs, synth  # noqa: E402

# phi3 LongRoPE-style parameters (model.cpp:1312-1316, 555-557) with synthetic
# short factors: exercises the YaRN ramp and mscale path of the RoPE table.
LONGROPE = dict(rope_ext_factor=1.0, rope_beta_fast=32.0, rope_beta_slow=1.0, n_ctx_orig=4096,
                rope_attn_factor=1.1902381, longrope_clamp=True,
                rope_freq_factors=(1.0 + 0.05 * np.arange(48, dtype=np.float32) / 48.0).astype(np.float32))

CASES = [
    dict(name="qwen2-0.5b_decode", spec="qwen2-0.5b", n_ctx=256, n_past=200, n_new=1),
    dict(name="qwen2-0.5b_chunk5", spec="qwen2-0.5b", n_ctx=256, n_past=150, n_new=5),
    dict(name="llama3.2-3b_decode", spec="llama3.2-3b", n_ctx=192, n_past=130, n_new=1),
    dict(name="phi3-mini_decode", spec="phi3-mini", n_ctx=96, n_past=70, n_new=1),
    dict(name="phi3-mini-normalrope_decode", spec="phi3-mini", n_ctx=96, n_past=70, n_new=1,
         overrides=dict(rope_mode=0)),
    dict(name="phi3-longrope_chunk3", spec="phi3-mini", n_ctx=96, n_past=40, n_new=3, overrides=LONGROPE),
    dict(name="qwen3-8b_chunk8", spec="qwen3-8b-prefill", n_ctx=128, n_past=64, n_new=8),
    dict(name="llama3.1-8b_decode", spec="llama3.1-8b-128k", n_ctx=192, n_past=140, n_new=1),
]


def case_spec(case):
    sp = specs.get(case["spec"])
    sp.update(case.get("overrides", {}))
    sp["n_layer"] = 1
    sp["n_ctx"] = case["n_ctx"]
    return sp


def case_inputs(case):
    """Cache rows [0, n_past) (uint16), fused rows, q/k/v views, gammas."""
    import kv_oracle as O
    sp = case_spec(case)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    n_ctx, n_past, n_new = case["n_ctx"], case["n_past"], case["n_new"]
    kc = np.zeros((n_ctx, hkv, d), np.uint16)
    vc = np.zeros((n_ctx, hkv, d), np.uint16)
    kc[:n_past] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 0, 0, n_past, hkv, d)
    vc[:n_past] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 1, 0, n_past, hkv, d)
    rows = synth.qkv_rows(sp, 0, 0, n_new)
    q = rows[:, : hq * d]
    k = rows[:, hq * d: (hq + hkv) * d]
    v = rows[:, (hq + hkv) * d:]
    qn = kn = None
    if sp["qk_norm"]:
        qn, kn = synth.norm_weights(sp, 0)
    return sp, kc, vc, rows, q, k, v, qn, kn


def run_oracle(case, n_threads=0):
    import kv_oracle as O
    sp, kc, vc, rows, q, k, v, qn, kn = case_inputs(case)
    orc = O.Oracle(sp)
    q_roped = orc.append(kc, vc, case["n_past"], q, k, v, qn, kn)
    out = orc.attend(kc, vc, case["n_past"], q_roped, n_threads=n_threads)
    n0, n1 = case["n_past"], case["n_past"] + case["n_new"]
    return dict(k_new=kc[n0:n1].copy(), v_new=vc[n0:n1].copy(), q_roped=q_roped, out=out)


def path(case):
    return os.path.join(HERE, case["name"] + ".npz")


def load(case):
    z = np.load(path(case))
    return {k: z[k] for k in ("k_new", "v_new", "q_roped", "out")}


def main():
    for case in CASES:
        res = run_oracle(case)
        meta = {k: v for k, v in case.items() if k != "overrides"}
        np.savez_compressed(path(case), meta=json.dumps(meta), **res)
        print("%-32s k_new %s out %s" % (case["name"], res["k_new"].shape, res["out"].shape))


if __name__ == "__main__":
    main()
