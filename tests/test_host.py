"""CPU tests of the library's host side (no GPU needed): the C ABI loads and
exports every function its headers declare, the sizing rules equal the
reference's (model.cpp:869-885, 1002-1059), the RoPE table that kv_alloc
uploads equals the oracle's bit for bit, the shard geometry, and clean
failure (an error code, no crash) of kv_alloc where there is no GPU.
"""
import ctypes
import os
import re
import sys

import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden as G  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for h in ("kv_api.h", "kv_bench.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(kv_[a-z_0-9]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_library_loads_and_exports_every_declared_function():
    L = K.lib()
    names = _declared_functions()
    assert len(names) >= 20, names
    for n in names:
        assert hasattr(L, n), "missing export %s" % n


def test_config_defaults():
    c = K.KvConfig()
    assert K.lib().kv_config_init(ctypes.byref(c)) == 0
    assert c.rope_mode == 2 and c.rope_base == 10000.0 and c.rope_freq_scale == 1.0
    assert c.rope_attn_factor == 1.0 and c.n_batch_max == 512 and c.device == -1 and c.n_shards == 1
    assert abs(c.rms_eps - 1e-6) < 1e-12


@pytest.mark.parametrize("name", list(specs.specs()))
def test_cache_bytes_equals_reference_rule(name):
    sp = specs.get(name)
    cfg = K.make_config(sp)
    for n_ctx in (1, 64, sp["n_ctx"]):
        assert K.cache_bytes(cfg, n_ctx) == O.kv_cache_bytes(sp["n_layer"], sp["n_head_kv"], sp["head_dim"], n_ctx)


@pytest.mark.parametrize("name", list(specs.specs()))
@pytest.mark.parametrize("shards", [1, 2])
def test_auto_n_ctx_equals_reference_rule(name, shards):
    sp = specs.get(name)
    if sp["n_head_kv"] % shards:
        pytest.skip("heads do not shard")
    cfg = K.make_config(sp, n_shards=shards)
    # per-position bytes of one shard: its cache rows plus one RoPE table row
    per_tok = sp["n_layer"] * (sp["n_head_kv"] // shards) * sp["head_dim"] * 4 + (sp["n_rot"] // 2) * 8
    for free in (-1, 0, 300 << 20, 1 << 30, 24 << 30, 180 << 30):
        for train in (0, 4096, 131072):
            cfg.n_ctx_train = train
            assert K.auto_n_ctx(cfg, free) == O.auto_n_ctx(free, per_tok, train), (free, train)


def test_auto_n_ctx_longrope_clamp():
    sp = specs.get("phi3-mini")
    sp.update({k: v for k, v in G.LONGROPE.items()})
    cfg = K.make_config(sp)
    assert K.auto_n_ctx(cfg, 180 << 30) == 4096
    cfg.longrope_clamp = 0
    assert K.auto_n_ctx(cfg, 180 << 30) > 4096


ROPE_CASES = ["qwen2-0.5b", "llama3.2-3b", "phi3-mini", "qwen3-8b-prefill", "llama3.1-8b-128k", "longrope",
              "partial"]


@pytest.mark.parametrize("name", ROPE_CASES)
def test_rope_table_bitexact_vs_oracle(name):
    if name == "longrope":
        sp = specs.get("phi3-mini")
        sp.update({k: v for k, v in G.LONGROPE.items()})
    elif name == "partial":
        sp = specs.get("phi3-mini")
        sp["n_rot"] = 64
    else:
        sp = specs.get(name)
    cfg = K.make_config(sp)
    orc = O.Oracle(sp)
    for pos0, npos in ((0, 300), (4000, 200), (131000, 72), (262000, 8)):
        got = K.rope_table_host(cfg, pos0, npos)
        want = orc.rope_table(pos0, npos)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (name, pos0)


def test_shard_geometry():
    sp = specs.get("llama3.1-8b-128k")
    for G_ in (1, 2, 4, 8):
        cfg = K.make_config(sp, n_shards=G_)
        seen_q, seen_kv = [], []
        for g in range(G_):
            q0, nq, kv0, nkv = K.shard_geometry(cfg, g)
            assert nkv == 8 // G_ and nq == 4 * nkv
            assert q0 == kv0 * 4          # a KV head's GQA group stays on its shard
            seen_q += list(range(q0, q0 + nq))
            seen_kv += list(range(kv0, kv0 + nkv))
        assert seen_q == list(range(32)) and seen_kv == list(range(8))
    bad = K.make_config(specs.get("qwen2-0.5b"), n_shards=4)   # 2 KV heads do not split 4 ways
    with pytest.raises(K.KvError) as e:
        K.shard_geometry(bad, 0)
    assert e.value.code == K.KV_E_ARG


def test_bad_shapes_rejected():
    sp = specs.get("llama3.2-3b")
    for field, val in (("head_dim", 80), ("n_rot", 7), ("rope_mode", 1), ("n_head", 25)):
        cfg = K.make_config(sp)
        setattr(cfg, field, val)
        with pytest.raises(K.KvError) as e:
            K.rope_table_host(cfg, 0, 1)
        assert e.value.code == K.KV_E_ARG


def test_ring_and_head_dim_256_shape_rules():
    """Ring caches need explicit positions; head_dim 256 and the nGPT norm rotate
    whole heads; qk_norm is 0, 1 or 2.  (shape_ok runs before any CUDA call.)"""
    sp = specs.get("llama3.2-3b")
    bad = []
    c = K.make_config(sp, n_ctx=0, ring_cells=1024)
    bad.append(c)
    c = K.make_config(sp, ring_cells=-1)
    bad.append(c)
    c = K.make_config(sp)
    c.head_dim, c.n_rot = 256, 128
    bad.append(c)
    c = K.make_config(sp)
    c.qk_norm, c.n_rot = 2, 64
    bad.append(c)
    c = K.make_config(sp)
    c.qk_norm = 3
    bad.append(c)
    for cfg in bad:
        with pytest.raises(K.KvError) as e:
            K.rope_table_host(cfg, 0, 1)
        assert e.value.code == K.KV_E_ARG
    ok = K.make_config(sp)
    ok.head_dim, ok.n_rot, ok.qk_norm = 256, 256, 2
    K.rope_table_host(ok, 0, 1)


def test_oversized_contexts_are_refused_and_sizes_saturate():
    """n_ctx above 2^31 positions is a shape error (checked before any CUDA
    call, so kv_alloc's sizing never overflows); kv_cache_bytes saturates
    instead of wrapping."""
    import ctypes
    sp = specs.get("llama3.1-8b-128k")
    for n_ctx in ((1 << 31) + 64, 1 << 40, (1 << 62) + 64):
        cfg = K.make_config(sp, n_ctx=n_ctx)
        with pytest.raises(K.KvError) as e:
            K.rope_table_host(cfg, 0, 1)
        assert e.value.code == K.KV_E_ARG and "2^31" in str(e.value)
        h = ctypes.c_void_p()
        assert K.lib().kv_alloc(ctypes.byref(cfg), ctypes.byref(h)) == K.KV_E_ARG and not h.value
    cfg = K.make_config(sp, n_ctx=1 << 31)
    K.rope_table_host(cfg, 0, 1)
    assert K.cache_bytes(cfg, 1 << 31) == 32 * 8 * 128 * 4 * (1 << 31)
    assert K.cache_bytes(cfg, 1 << 62) == 2 ** 64 - 1


def test_ring_cache_bytes():
    """A ring holds min(ring_cells, n_ctx) rows (dory_kv_cost, dory.c:373-389)."""
    sp = specs.get("llama3.2-3b")
    lin = K.make_config(sp, n_ctx=8192)
    ring = K.make_config(sp, n_ctx=8192, ring_cells=1024)
    assert K.cache_bytes(ring, 8192) * 8 == K.cache_bytes(lin, 8192)
    assert K.cache_bytes(ring, 512) == K.cache_bytes(lin, 512)


def test_alloc_without_gpu_returns_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    cfg = K.make_config(specs.get("qwen2-0.5b"), n_ctx=256)
    h = ctypes.c_void_p()
    rc = K.lib().kv_alloc(ctypes.byref(cfg), ctypes.byref(h))
    assert rc == K.KV_E_CUDA and not h.value
    assert "cuda" in K.last_error().lower()


def test_bench_reference_arm_prints_one_contract_line():
    """bench.py --impl reference (the CPU restatement on the host cores) prints
    exactly one JSON line with the contract's keys, in both branches."""
    import json
    import subprocess
    import sys as _sys
    for extra in ([], ["--flash"]):
        r = subprocess.run([_sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                            "--warmup", "1", "--config", "qwen2-0.5b"] + extra,
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        lines = [l for l in r.stdout.splitlines() if l.strip()]
        assert len(lines) == 1, r.stdout
        d = json.loads(lines[0])
        for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                    "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
            assert key in d, key
        assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["kind"] == "port"
        assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
        assert d["config"]["branch"].startswith("flash" if extra else "default")


def test_noalloc_refuses_oversized_shapes_before_any_device_work():
    """kv_attend_decode_noalloc: key counts or head counts whose sizing would
    overflow are refused with KV_E_RANGE by the argument checks, which run
    before the device is touched (the placeholder addresses are never used)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = K.lib()
    kc, vc, q, out = 0x10000, 0x20000, 0x30000, 0x40000
    for n_head, n_kv_heads, n_kv in ((32, 8, 1 << 40), (32, 8, (1 << 62) + 1), (1 << 20, 1 << 20, 100)):
        rc = lib.kv_attend_decode_noalloc(kc, vc, n_head, n_kv_heads, 128, n_kv, q, out, None)
        assert rc == K.KV_E_RANGE, (n_head, n_kv_heads, n_kv, rc)
        assert "scratch" in K.last_error()
    # a shape within the bounds reaches the device query, which fails here
    assert lib.kv_attend_decode_noalloc(kc, vc, 32, 8, 128, 4096, q, out, None) == K.KV_E_CUDA


@pytest.mark.parametrize("name,unit,want", [
    ("qwen2-0.5b", "GB", 0.0254),        # 24 layers, 2049 keys
    ("llama3.2-3b", "GB", 3.686),        # 28 layers, 32001..32256 keys, mean of 256 steps
    ("phi3-mini", "GB", 1.588),          # 32 MHA layers, 3969..4096 keys, mean of 128 steps
    ("llama3.1-8b-128k", "GB", 17.18),   # 32 layers, 131001..131064 keys, mean of 64 steps
    ("qwen3-8b-prefill", "TFLOP", 5.025),  # 512 causal queries after 16384 rows
])
def test_bench_algorithmic_work_per_token(name, unit, want):
    """The roofline's numerator: bytes per decode token (K and V read once in
    F16, the new rows written, k/v read and q/o in F32; split partials and
    re-reads not counted) and causal FLOPs per chunk (4*d*Hq per visible
    query-key pair), averaged over the configuration's steps."""
    import importlib
    import statistics
    import sys as _sys
    _sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    sp = specs.get(name)
    pos = bench.positions(sp, 0, sp["steps"])
    L, hq, hkv, d = sp["n_layer"], sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    if unit == "TFLOP":
        got = statistics.mean(bench.step_flops(sp, p, sp["n_new"]) for p in pos) / 1e12
        n = sp["n_new"]
        keys = sum(sp["n_past"] + i + 1 for i in range(n))
        assert bench.step_flops(sp, sp["n_past"], n) == 4 * d * keys * hq * L
    else:
        got = statistics.mean(bench.step_bytes(sp, p) for p in pos) / 1e9
        p0 = sp["n_past"]
        assert bench.step_bytes(sp, p0) == L * ((p0 + 1) * hkv * d * 4 + hkv * d * 4 + hkv * d * 8 + hq * d * 8)
    assert abs(got - want) / want < 2e-3, (got, want)


def test_cpu_baseline_sample_at_two_thread_counts():
    """The GPU arm's cpu_baseline samples the CPU path on every core and on the
    reference's own 8 threads, reusing one set of generated cache rows."""
    import importlib
    import sys as _sys
    _sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    sp = specs.get("qwen2-0.5b")
    g_all, us_all, desc, th_all, _, cp = bench.cpu_sample(sp, 0.2, 4)
    g8, us8, desc8, th8, _, cp8 = bench.cpu_sample(sp, 0.2, 4, n_threads=8, cp=cp)
    assert cp8 is cp and th8 == 8 and "8 threads" in desc8
    assert th_all == cp.O.online_cores() >= 1
    assert g_all > 0 and g8 > 0 and us_all > 0 and us8 > 0
    assert "%d threads" % th_all in desc


def test_headers_compile_as_c_and_cpp(tmp_path):
    """include/*.h are a C ABI: they compile in a C99 and a C++17 translation unit."""
    import shutil
    import subprocess
    src = ("#include \"kv_api.h\"\n#include \"kv_bench.h\"\n"
           "int f(void) { kv_config c; kv_config_init(&c); return (int)c.n_layer + KV_ATTN_FLASH + KV_MASK_F16; }\n")
    for compiler, ext, std in (("gcc", "c", "-std=c99"), ("g++", "cpp", "-std=c++17")):
        if not shutil.which(compiler):
            pytest.skip(compiler + " missing")
        p = tmp_path / ("abi." + ext)
        p.write_text(src)
        r = subprocess.run([compiler, std, "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                            str(p)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_decode_split_cta_counts():
    """kv_decode_ctas (the decode kernel's split, host arithmetic): a multiple of
    the KV heads when that idles at most 5 % of the SMs, one CTA per SM at most,
    >= 256 (head, key) rows a CTA, >= one CTA a head."""
    def n_cta(sm, hkv, n_kv):
        out = ctypes.c_int32()
        assert K.lib().kv_decode_ctas(sm, hkv, n_kv, ctypes.byref(out)) == K.KV_OK
        return out.value
    assert n_cta(148, 8, 32001) == 144            # llama-3.2-3B / 3.1-8B: 18 CTAs a head
    assert n_cta(148, 4, 131001) == 148           # 4 divides 148
    assert n_cta(148, 1, 131001) == 148           # one-head shard
    assert n_cta(148, 32, 3969) == 148            # phi3: 128 would idle 13.5 %
    assert n_cta(148, 2, 2049) == 17              # qwen2-0.5B: ceil(4098 rows / 256); 16 would idle 6 %
    assert n_cta(148, 8, 1) == 8                  # never fewer than the heads
    assert n_cta(148, 3, 100000) == 147
    for hkv in (1, 2, 3, 4, 6, 8, 12, 16, 24, 32, 40, 64):
        for n_kv in (1, 7, 300, 4096, 32768, 131072):
            c = n_cta(148, hkv, n_kv)
            assert hkv <= c <= max(hkv, 148) and c <= hkv * n_kv
            # a CTA's range covers at most one head's keys: it spans at most two heads
            assert (hkv * n_kv + c - 1) // c <= n_kv
    out = ctypes.c_int32()
    assert K.lib().kv_decode_ctas(0, 8, 100, ctypes.byref(out)) == K.KV_E_ARG


def test_decode_grid_residency_check():
    """kv_decode_grid_fits: the decode kernel's CTAs wait on one another, so
    kv_alloc accepts a device only if its largest grid is resident at once
    (SMs x resident CTAs an SM >= CTAs)."""
    fits = K.lib().kv_decode_grid_fits
    assert fits(148, 1, 148) == 1                 # one CTA per SM, the whole grid
    assert fits(148, 1, 149) == 0                 # one CTA more than the SMs
    assert fits(148, 0, 1) == 0                   # the kernel does not fit on an SM at all
    assert fits(74, 2, 148) == 1                  # two CTAs an SM
    assert fits(100, 1, 144) == 0                 # a device (or partition) with fewer SMs
    assert fits(0, 1, 1) == 0 and fits(148, 1, 0) == 0
    # every grid kv_decode_ctas produces fits one CTA per SM on that SM count
    out = ctypes.c_int32()
    for sm in (16, 74, 132, 148):
        for hkv in (1, 2, 8, 32):
            for n_kv in (1, 2049, 32001, 131001):
                if hkv > sm:
                    continue
                assert K.lib().kv_decode_ctas(sm, hkv, n_kv, ctypes.byref(out)) == K.KV_OK
                assert fits(sm, 1, out.value) == 1


def test_decode_cluster_shapes():
    """kv_decode_shape (host arithmetic): one cluster of <= 8 CTAs per head when
    the head's keys fit it (>= 256 keys a CTA) at >= 85 % of the plain split's
    CTAs; otherwise no clusters; never a cluster size the device cannot hold."""
    def shape(sm, hkv, n_kv, mc):
        arr = None
        if mc is not None:
            arr = (ctypes.c_int32 * 9)(*[mc.get(q, 0) for q in range(9)])
        out = [ctypes.c_int32() for _ in range(3)]
        assert K.lib().kv_decode_shape(sm, hkv, n_kv, arr, *[ctypes.byref(o) for o in out]) == K.KV_OK
        return tuple(o.value for o in out)
    roomy = {q: 148 // q for q in range(2, 9)}
    b200 = {2: 74, 3: 45, 4: 33, 5: 0, 6: 22, 7: 0, 8: 15}   # measured at 216 KB of shared memory a CTA
    assert shape(148, 2, 2049, b200) == (16, 8, 1)         # qwen2-0.5B: a cluster of 8 per head
    assert shape(148, 32, 3969, b200) == (128, 4, 1)       # phi3-mini: a cluster of 4 per head
    assert shape(148, 1, 32001, b200) == (126, 1, 1)       # one-head shard: the plain split
    assert shape(148, 8, 32001, b200) == (144, 1, 1)       # llama-3.2-3B: the plain split
    assert shape(148, 8, 32001, None) == (144, 1, 1)       # no cluster support: the plain split
    assert shape(148, 32, 3969, {4: 31}) == (148, 1, 1)    # 32 clusters of 4 do not fit
    assert shape(148, 2, 2049, {8: 1, 4: 4}) == (17, 1, 1)  # 2 clusters of 8 do not fit; 4s keep too few CTAs
    for hkv in (1, 2, 4, 8, 32):
        for n_kv in (1, 300, 2049, 4096, 32001, 131001):
            c, q, ncl = shape(148, hkv, n_kv, roomy)
            assert c <= 148 and q <= 8 and ncl == 1
            if q > 1:                                     # one cluster a head, within the device's capacity
                assert c == hkv * q and roomy[q] >= hkv and (n_kv + 255) // 256 >= q


def test_phase_stamps_only_in_the_measurement_build():
    """kv_debug_stamps is exported by every build; outside the phase-stamp
    build (build.py --stamps) it reports KV_E_UNSUPPORTED without touching
    its arguments."""
    r, m = ctypes.c_int32(-5), ctypes.c_int32(-5)
    rc = K.lib().kv_debug_stamps(None, None, ctypes.byref(r), ctypes.byref(m))
    assert rc == K.KV_E_UNSUPPORTED
    assert (r.value, m.value) == (-5, -5)
    assert "KV_PHASE_STAMPS" in K.lib().kv_last_error().decode()


def test_bench_shard_of_rejects_a_non_divisor():
    import subprocess
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--shard-of", "3"],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode != 0 and "does not divide" in (r.stdout + r.stderr)
