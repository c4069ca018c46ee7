"""Build the KV path library in-tree: ggml-loader_b200/lib/libkv_b200.so.

Every CUDA source is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); host sources go through nvcc to
g++.  -ffp-contract=off on both sides keeps the bit-exact pieces (RoPE table,
append arithmetic) free of fused multiply-adds.  Objects are cached under
ggml-loader_b200/_build and rebuilt when a source or header is newer.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libkv_b200.so")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-I", INCLUDE, "-I", CSRC,
          "-Xcompiler", "-fPIC,-ffp-contract=off,-Wall", "--fmad=false"]
# --fmad=false: device float mul/add are never contracted implicitly; the
# kernels that want FMAs (dot products) call fmaf explicitly.


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose, obj_dir=OBJ, defines=()):
    obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [NVCC] + ARCH + COMMON + ["-D" + d for d in defines] + ["-c", src, "-o", obj]
    if verbose and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, " ".join(cmd), r.stderr))
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose=False, lib=LIB, obj_dir=OBJ, defines=()):
    """Compile and link the library.  `defines` builds a variant (e.g.
    KV_PHASE_STAMPS, the per-CTA phase stamps of the decode kernel, for
    measurement) into its own `lib` and `obj_dir`."""
    os.makedirs(obj_dir, exist_ok=True)
    os.makedirs(os.path.dirname(lib), exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, obj_dir, defines), srcs))
    if _stale(lib, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", lib] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr))
    return lib


# the phase-stamp measurement build (kv_debug_stamps; python -m kv_b200.stamps)
STAMPS_LIB = os.path.join(HERE, "lib", "stamps", "libkv_b200.so")
STAMPS_OBJ = os.path.join(HERE, "_build", "stamps")


def build_stamps(verbose=False):
    return build(verbose, STAMPS_LIB, STAMPS_OBJ, ("KV_PHASE_STAMPS",))


if __name__ == "__main__":
    if "--stamps" in sys.argv:
        print(build_stamps(verbose="-v" in sys.argv))
    else:
        print(build(verbose="-v" in sys.argv))
