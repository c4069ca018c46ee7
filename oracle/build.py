"""Build recipe for the CPU oracle (test infrastructure only).

Outputs (git-ignored, but carried to the GPU box with the repo snapshot):
  oracle/lib/libkv_oracle.so       -- the C restatement in kv_oracle.c
  oracle/_ref/libmoe_scalar.so     -- the reference's own scalar math backend,
                                      compiled from its sources where they lie
                                      (src/moe_stream/compute_backend.c and
                                      dequant.c)
  oracle/_ref/libref_attention.so  -- the reference's own single-token
                                      attention (src/moe_stream/qwen_model.c,
                                      attention_block and its RoPE table) in the
                                      harness oracle/ref_attention.c, with the
                                      moe_stream sources qwen_model.c needs
The two reference builds happen only when a reference checkout is found: the
directory named by KV_REFERENCE_ROOT, else a checkout named `reference` beside
this repository's root.  Without one (e.g. on a GPU box) they are skipped and
the tests that use them skip.

The reference's dense path (ggml) cannot be built: the ggml submodule is not
vendored in the checkout.  The MoE engine's scalar backend and its ggml-free
attention are the reference's own arithmetic for this path's ops that compile
from their own few files (plain gcc, no build system); they are used to
cross-check the oracle's semantics.  They are compiled with IEEE semantics
(no -ffast-math, unlike the reference's own Makefile): the builds pin op
semantics, not speed.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "lib", "libkv_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libmoe_scalar.so")
REF_ATTN_LIB = os.path.join(HERE, "_ref", "libref_attention.so")
# moe_stream sources the attention harness links besides the qwen_model.c it includes
_ATTN_DEPS = ("moe_stream.c", "gguf_index.c", "expert_loader.c", "lru_cache.c", "memtrack.c", "dequant.c",
              "compute_backend.c")


def reference_root():
    """The reference checkout: $KV_REFERENCE_ROOT, else `reference` beside the
    repository root; None when neither holds src/moe_stream."""
    cands = [os.environ.get("KV_REFERENCE_ROOT"), os.path.join(os.path.dirname(HERE), os.pardir, "reference")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "src", "moe_stream")):
            return os.path.realpath(c)
    return None


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_oracle(force=False):
    srcs = [os.path.join(HERE, "kv_oracle.c"), os.path.join(HERE, "kv_oracle.h")]
    if not force and not _newer(LIB, srcs):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cmd = ["gcc", "-std=c11", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-pthread", "-Wall", "-Wextra", "-o", LIB, srcs[0], "-lm"]
    subprocess.check_call(cmd)
    return LIB


def build_ref(force=False):
    """Compile the reference's scalar backend and its attention harness from
    the reference's sources in place; returns the scalar backend's path, or
    None without a reference checkout."""
    root = reference_root()
    if root is None:
        return None
    d = os.path.join(root, "src", "moe_stream")
    srcs = [os.path.join(d, "compute_backend.c"), os.path.join(d, "dequant.c")]
    if not all(os.path.exists(s) for s in srcs):
        return None
    os.makedirs(os.path.dirname(REF_LIB), exist_ok=True)
    if force or _newer(REF_LIB, srcs):
        cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-D_GNU_SOURCE", "-I", d,
               "-o", REF_LIB] + srcs + ["-lm"]
        subprocess.check_call(cmd)
    harness = os.path.join(HERE, "ref_attention.c")
    deps = [os.path.join(d, s) for s in _ATTN_DEPS]
    if all(os.path.exists(s) for s in deps + [os.path.join(d, "qwen_model.c")]) and \
            (force or _newer(REF_ATTN_LIB, [harness, os.path.join(d, "qwen_model.c")] + deps)):
        cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-D_GNU_SOURCE", "-D_FILE_OFFSET_BITS=64",
               "-pthread", "-I", d, "-o", REF_ATTN_LIB, harness] + deps + ["-lm", "-Wl,--no-undefined"]
        subprocess.check_call(cmd)
    return REF_LIB


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
