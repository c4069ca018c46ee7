"""Build recipe for the CPU oracle (test infrastructure only).

Outputs (git-ignored, but carried to the GPU box with the repo snapshot):
  oracle/lib/libkv_oracle.so   -- the C restatement in kv_oracle.c
  oracle/_ref/libmoe_scalar.so -- the reference's own scalar math backend,
                                  compiled from its sources where they lie
                                  (src/moe_stream/compute_backend.c and
                                  dequant.c); only built when the reference
                                  checkout is present.

The reference's dense path (ggml) cannot be built: the ggml submodule is not
vendored in the checkout.  The scalar MoE backend is the only piece of the
reference's own arithmetic for this path's ops (RMSNorm, NEOX RoPE, softmax)
that compiles from its own few files; it is used to cross-check semantics.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "lib", "libkv_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libmoe_scalar.so")
REF_SRC = os.environ.get("KV_REFERENCE_ROOT", "/root/reference")


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
    """Compile the reference's scalar backend from its sources in place."""
    d = os.path.join(REF_SRC, "src", "moe_stream")
    srcs = [os.path.join(d, "compute_backend.c"), os.path.join(d, "dequant.c")]
    if not all(os.path.exists(s) for s in srcs):
        return None  # reference checkout absent (e.g. on the GPU box)
    if not force and not _newer(REF_LIB, srcs):
        return REF_LIB
    os.makedirs(os.path.dirname(REF_LIB), exist_ok=True)
    # IEEE semantics (no -ffast-math): this build pins op semantics, not speed.
    cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-D_GNU_SOURCE", "-I", d,
           "-o", REF_LIB] + srcs + ["-lm"]
    subprocess.check_call(cmd)
    return REF_LIB


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
