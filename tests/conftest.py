"""Shared test set-up.

Markers: `gpu` -- needs a CUDA device (run on the B200 box with -m gpu).
Everything else runs on CPU: the oracle against its golden fixtures, the
reference's own scalar backend (oracle/_ref, when built), host-side logic of
the library (sizing, RoPE table, shard geometry) and multi-rank decomposition
on gloo ranks.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "ggml-loader_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def _build_once():
    import importlib.util
    for name, path, fn in (("_oracle_build", os.path.join(ROOT, "oracle", "build.py"), "build_oracle"),
                           ("_kv_build", os.path.join(ROOT, "ggml-loader_b200", "build.py"), "build")):
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        try:
            getattr(mod, fn)()
        except Exception as e:  # e.g. no nvcc on this host: the prebuilt .so is used
            sys.stderr.write("note: %s.%s() skipped: %s\n" % (name, fn, e))
    try:
        import importlib.util as u
        spec = u.spec_from_file_location("_oracle_build2", os.path.join(ROOT, "oracle", "build.py"))
        mod = u.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build_ref()
    except Exception as e:
        sys.stderr.write("note: oracle/_ref not built: %s\n" % e)


_build_once()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
