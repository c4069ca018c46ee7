"""CPU tests of the oracle (oracle/kv_oracle.c) -- the checker the GPU path is
compared against.  The reference ships no fixtures for this path (ggml is not
vendored), so the oracle is pinned by: (1) exhaustive/numpy checks of its F16
rounding, (2) the reference's own scalar math backend
(src/moe_stream/compute_backend.c, built by oracle/build.py into oracle/_ref)
for the NEOX rotation, RMSNorm and softmax formulas, (3) the reference's own
decode attention and RoPE table (src/moe_stream/qwen_model.c:456-524 and
:346-353, driven by oracle/ref_attention.c into oracle/_ref) at the benchmark
shapes, (4) an independent float64 numpy restatement of the attention, and
(5) the committed golden fixtures (regression pin).
"""
import ctypes
import math
import os
import sys

import numpy as np
import pytest

import kv_oracle as O
from kv_b200 import specs, synth

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden as G  # noqa: E402

f32p = ctypes.POINTER(ctypes.c_float)


def _fp(a):
    return a.ctypes.data_as(f32p)


# ---------------------------------------------------------------------------
# F16 conversion (A3)
# ---------------------------------------------------------------------------

def test_f16_to_f32_all_halves():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([O.lib().kvo_f16_to_f32(int(b)) for b in bits], np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(1)
    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    finite = halves[np.isfinite(halves)].astype(np.float32)
    # exact halves, exact ties between neighbours, and random floats over the whole range
    with np.errstate(over="ignore"):
        nxt = np.nextafter(finite.astype(np.float16), np.float16(np.inf)).astype(np.float32)
    ties = ((finite.astype(np.float64) + nxt.astype(np.float64)) / 2).astype(np.float32)
    rnd = np.concatenate([
        rng.standard_normal(200000).astype(np.float32),
        (rng.standard_normal(100000) * 1e-5).astype(np.float32),      # subnormal halves
        (rng.standard_normal(100000) * 3e4).astype(np.float32),       # near overflow
        np.array([65504, 65519.99, 65520, 65536, 1e-8, 2.0 ** -25, 2.0 ** -24, -0.0, np.inf, -np.inf],
                 np.float32),
    ])
    x = np.concatenate([finite, ties[np.isfinite(ties)], rnd]).astype(np.float32)
    got = O.f32_to_f16_bits(x)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


# ---------------------------------------------------------------------------
# seeded generator: C oracle == numpy (and the device generator, in GPU tests)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("seed,stream,idx0", [(0x6B760001, synth.STREAM_CACHE, 0), (7, 12345, 10 ** 9)])
def test_generator_c_matches_numpy(seed, stream, idx0):
    n = 20000
    a = O.gen_normal_f32(seed, stream, n, idx0)
    b = synth.normal(seed, stream, n, idx0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    ua = O.gen_uniform_f32(seed, stream, n, 0.5, 1.5, idx0)
    ub = synth.uniform(seed, stream, n, 0.5, 1.5, idx0)
    assert np.array_equal(ua.view(np.uint32), ub.view(np.uint32))
    assert abs(float(a.mean())) < 0.03 and abs(float(a.var()) - 1.0) < 0.05
    assert ua.min() >= 0.5 and ua.max() < 1.5


def test_cache_rows_use_global_head_index():
    hkv, d = 8, 128
    full = O.gen_cache_rows(5, synth.STREAM_CACHE, 10, 3, hkv, d)
    part = O.gen_cache_rows(5, synth.STREAM_CACHE, 10, 3, hkv, d, h0=2, nh=3)
    assert np.array_equal(full[:, 2:5], part)
    idx0 = 10 * hkv * d
    ref = synth.normal(5, synth.STREAM_CACHE, 3 * hkv * d, idx0).astype(np.float16).view(np.uint16)
    assert np.array_equal(full.reshape(-1), ref)


# ---------------------------------------------------------------------------
# RoPE (A2)
# ---------------------------------------------------------------------------

def _cfg(name, **kw):
    sp = specs.get(name)
    sp.update(kw)
    return sp


@pytest.mark.parametrize("name", ["qwen2-0.5b", "llama3.2-3b", "phi3-mini", "llama3.1-8b-128k"])
def test_rope_table_is_iterated_float_schedule(name):
    sp = _cfg(name)
    orc = O.Oracle(sp)
    pos = [0, 1, 17, 4095, 32000, 131063]
    n_rot = sp["n_rot"]
    step = np.float32(np.float32(sp["rope_base"]) ** np.float32(-2.0 / n_rot))
    ff = sp["rope_freq_factors"]
    for p in pos:
        t = orc.rope_table(p, 1)[0]
        theta = np.float32(p)
        for i in range(n_rot // 2):
            f = np.float32(1.0) if ff is None else ff[i]
            ang = np.float32(theta / f)
            # libm float cos/sin of the float angle; compare loosely to numpy's
            assert abs(float(t[i, 0]) - math.cos(float(ang))) < 2e-6 * max(1.0, abs(float(ang))) + 1e-6
            assert abs(float(t[i, 1]) - math.sin(float(ang))) < 2e-6 * max(1.0, abs(float(ang))) + 1e-6
            theta = np.float32(theta * step)


def test_rope_yarn_corr_dims_and_mscale():
    sp = _cfg("phi3-mini", **{k: v for k, v in G.LONGROPE.items()})
    orc = O.Oracle(sp)
    dims = orc.corr_dims()
    # corr_dim(n_turns) = n_dims * ln(n_ctx_orig / (2 pi n_turns)) / (2 ln base)
    def cd(b):
        return 96 * math.log(4096 / (2 * math.pi * b)) / (2 * math.log(1e4))
    assert dims[0] == max(0.0, math.floor(cd(32.0)))
    assert dims[1] == min(95.0, math.ceil(cd(1.0)))
    t0 = orc.rope_table(0, 1)[0]
    # at position 0 every angle is 0: cos = mscale = attn_factor (freq_scale 1 -> no extra term)
    assert np.all(t0[:, 0] == np.float32(sp["rope_attn_factor"]))
    assert np.all(t0[:, 1] == 0.0)


def test_rope_neox_matches_reference_scalar_backend():
    ref = O.reference_scalar_backend()
    if ref is None:
        pytest.skip("oracle/_ref not built (no reference checkout on this host)")
    sp = _cfg("qwen3-8b-prefill")
    orc = O.Oracle(sp)
    rng = np.random.default_rng(3)
    d = sp["head_dim"]
    for p in (0, 5, 16384, 40000):
        cs = orc.rope_table(p, 1)[0]
        x = rng.standard_normal(d).astype(np.float32)
        ours = orc.rope_row(cs, x)
        v = x.copy()
        c = np.ascontiguousarray(cs[:, 0])
        s = np.ascontiguousarray(cs[:, 1])
        ref.rope(None, _fp(v), d, _fp(c), _fp(s))  # compute_backend.c:56-66 (NEOX halves)
        assert np.array_equal(ours.view(np.uint32), v.view(np.uint32))


def test_rope_normal_pairs_adjacent():
    sp = _cfg("llama3.2-3b")
    orc = O.Oracle(sp)
    cs = orc.rope_table(1234, 1)[0]
    x = np.arange(128, dtype=np.float32) / 7.0
    y = orc.rope_row(cs, x)
    for i in range(64):
        c, s = cs[i]
        a, b = x[2 * i], x[2 * i + 1]
        assert y[2 * i] == np.float32(np.float32(a * c) - np.float32(b * s))
        assert y[2 * i + 1] == np.float32(np.float32(a * s) + np.float32(b * c))


def test_rope_partial_rotation_passes_tail_through():
    sp = _cfg("phi3-mini", n_rot=64)
    orc = O.Oracle(sp)
    cs = orc.rope_table(99, 1)[0]
    x = np.random.default_rng(0).standard_normal(96).astype(np.float32)
    y = orc.rope_row(cs, x)
    assert np.array_equal(y[64:], x[64:])
    assert not np.array_equal(y[:64], x[:64])


# ---------------------------------------------------------------------------
# RMSNorm (A1) and softmax (A5) against the reference scalar backend
# ---------------------------------------------------------------------------

def test_rmsnorm_matches_reference_scalar_backend():
    ref = O.reference_scalar_backend()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(4)
    for n in (64, 96, 128):
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        ours = np.empty(n, np.float32)
        O.lib().kvo_rms_norm_mul(_fp(x), _fp(w), n, 1e-6, _fp(ours))
        theirs = np.empty(n, np.float32)
        ref.rmsnorm(None, _fp(theirs), _fp(x), _fp(w), n, 1e-6)  # compute_backend.c:42-54
        # the reference's scalar backend sums squares in float, ggml in double
        assert np.max(np.abs(ours - theirs) / np.maximum(np.abs(theirs), 1e-3)) < 2e-6
        # and the double-sum restatement exactly
        sq = (x * x).astype(np.float64)
        mean = np.float32(np.cumsum(sq)[-1] / n)
        sc = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(1e-6)))
        want = ((x * sc).astype(np.float32) * w).astype(np.float32)
        assert np.array_equal(ours.view(np.uint32), want.view(np.uint32))


def _np_attention(sp, n_past, q_roped, kc, vc):
    """Independent float64 restatement of model.cpp:1416-1445 with ggml's F16
    conversions of Q and of P (A4) and a double softmax sum (A5)."""
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    r = hq // hkv
    n_new = q_roped.shape[0]
    n_kv = n_past + n_new
    scale = np.float32(1.0) / np.sqrt(np.float32(d))
    K = kc[:n_kv].view(np.float16).astype(np.float64)
    V = vc[:n_kv].view(np.float16).astype(np.float64)
    q16 = q_roped.astype(np.float16).astype(np.float64)
    out = np.zeros((n_new, hq * d))
    for t in range(n_new):
        lim = n_past + t
        for h in range(hq):
            kv = h // r  # GQA: contiguous groups (moe_stream/qwen_model.c:499)
            s = (K[: lim + 1, kv] @ q16[t, h]).astype(np.float32) * scale
            e = np.exp((s - s.max()).astype(np.float64)).astype(np.float32)
            p = (e * np.float32(1.0 / e.astype(np.float64).sum())).astype(np.float16).astype(np.float64)
            out[t, h * d:(h + 1) * d] = p @ V[: lim + 1, kv]
    return out


@pytest.mark.parametrize("case", G.CASES, ids=[c["name"] for c in G.CASES])
def test_attention_matches_float64_restatement(case):
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    q_roped = orc.append(kc, vc, case["n_past"], q, k, v, qn, kn)
    got = orc.attend(kc, vc, case["n_past"], q_roped)
    want = _np_attention(sp, case["n_past"], q_roped, kc, vc)
    err = np.abs(got - want)
    # the two restatements accumulate scores in different orders, so an
    # occasional p lands on the neighbouring F16 value: one F16 ulp of p
    # (<= 2^-11 p) times |v| (<= 6) bounds the per-element difference
    assert err.max() < 1e-4
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 3e-5


def test_softmax_semantics_against_reference_scalar_backend():
    ref = O.reference_scalar_backend()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    case = G.CASES[2]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    q_roped = orc.append(kc, vc, case["n_past"], q, k, v, qn, kn)
    got = orc.attend(kc, vc, case["n_past"], q_roped)
    d, r = sp["head_dim"], sp["n_head"] // sp["n_head_kv"]
    n_kv = case["n_past"] + 1
    K = kc[:n_kv].view(np.float16).astype(np.float32)
    V = vc[:n_kv].view(np.float16).astype(np.float32)
    for h in range(sp["n_head"]):
        kvh = h // r
        s = (K[:, kvh] @ q_roped[0, h].astype(np.float16).astype(np.float32)) * np.float32(1 / math.sqrt(d))
        s = np.ascontiguousarray(s, np.float32)
        ref.softmax(None, _fp(s), n_kv)   # compute_backend.c:68-86
        o = s.astype(np.float16).astype(np.float32) @ V[:, kvh]
        assert np.allclose(o, got[0, h * d:(h + 1) * d], rtol=0, atol=2e-5)


# ---------------------------------------------------------------------------
# the reference's own decode attention (moe_stream/qwen_model.c:456-524) and
# RoPE table (:346-353), compiled into oracle/_ref/libref_attention.so
# ---------------------------------------------------------------------------

def _ref_attention_case(tmp_path, name, pos, use_norm=False, **overrides):
    """One decode step at `pos` through the reference's attention_block and the
    oracle, on the same F16-representable cache and the same Q/K/V rows."""
    ra = O.reference_attention()
    if ra is None:
        pytest.skip("oracle/_ref/libref_attention.so not built (no reference checkout on this host)")
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import ref_gguf
    sp = specs.get(name)
    sp.update(overrides)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    qn, kn = synth.norm_weights(sp, 0) if use_norm else (None, None)
    gguf = ref_gguf.write(str(tmp_path / "model.gguf"), hq, hkv, d, sp["rope_base"], sp["rms_eps"], qn, kn)
    assert ra.geometry(gguf, pos + 1)[:3] == (hq, hkv, d)
    kc = np.zeros((pos + 1, hkv, d), np.uint16)
    vc = np.zeros_like(kc)
    kc[:pos] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE, 0, pos, hkv, d)
    vc[:pos] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 1, 0, pos, hkv, d)
    rows = synth.qkv_rows(sp, 0, 0, 1)
    q, k, v = rows[:, :hq * d], rows[:, hq * d:(hq + hkv) * d], rows[:, (hq + hkv) * d:]
    ref = ra.step(gguf, pos + 1, pos, kc[:pos].view(np.float16).astype(np.float32),
                  vc[:pos].view(np.float16).astype(np.float32), q, k, v, use_norm, hq, hkv, d)
    orc = O.Oracle(sp)
    q_roped = orc.append(kc, vc, pos, q, k, v, qn, kn)
    ours = orc.attend(kc, vc, pos, q_roped)[0]
    return sp, orc, kc, vc, rows, ref, ours


# The reference's MoE engine keeps an F32 cache and F32 weights: the oracle's
# ggml roundings (F16 Q and P in mul_mat, A4) and angle schedule (A2) are not
# its; the outputs agree within the north-star tolerance, which an error in
# the shared semantics (GQA mapping h / (Hq/Hkv), scale 1/sqrt(hd), the causal
# range 0..pos, softmax, P.V, NEOX pairs) would exceed by orders of magnitude.
@pytest.mark.parametrize("name,pos,use_norm,over", [
    ("qwen2-0.5b", 2048, False, {}),                                     # config 1
    ("llama3.2-3b", 4096, False, {"rope_mode": 2, "rope_freq_factors": None}),   # config 2's heads
    ("llama3.2-3b", 32000, False, {"rope_mode": 2, "rope_freq_factors": None}),  # ... at its context
    ("phi3-mini", 3968, False, {}),                                      # config 3 (MHA, head_dim 96)
    ("qwen3-8b-prefill", 2000, True, {}),                                # config 4's heads, QK-Norm
])
def test_attention_matches_reference_attention_block(tmp_path, name, pos, use_norm, over):
    sp, orc, kc, vc, rows, ref, ours = _ref_attention_case(tmp_path, name, pos, use_norm, **over)
    out = ref[0].astype(np.float64)
    d = ours - out
    assert np.abs(d).max() <= 2e-3
    assert np.linalg.norm(d) / np.linalg.norm(out) <= 1e-3
    # the stored V row: the reference keeps the F32 input, the oracle its RNE F16
    assert np.array_equal(ref[2].astype(np.float16).view(np.uint16), vc[pos].reshape(-1))


@pytest.mark.parametrize("name,pos,over", [
    ("qwen2-0.5b", 2048, {}),
    ("llama3.2-3b", 32000, {"rope_mode": 2, "rope_freq_factors": None}),
    ("phi3-mini", 3968, {}),
])
def test_rotation_matches_reference_given_its_table(tmp_path, name, pos, over):
    """The reference's stored K row (NEOX RoPE by its scalar backend with its
    own table) equals, bit for bit, the oracle's rotation of the same row with
    the reference's table entries at pos: the pairing and the separately
    rounded products and sums are the same; only the angles differ (A2)."""
    sp, orc, kc, vc, rows, ref, ours = _ref_attention_case(tmp_path, name, pos, **over)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    cs = np.stack([ref[3][pos], ref[4][pos]], axis=1)
    k = rows[0, hq * d:(hq + hkv) * d].reshape(hkv, d)
    got = np.concatenate([orc.rope_row(cs, k[h]) for h in range(hkv)])
    assert np.array_equal(got.view(np.uint32), ref[1].view(np.uint32))


@pytest.mark.parametrize("name,n_pos", [("qwen2-0.5b", 4096), ("llama3.2-3b", 32768), ("phi3-mini", 4096)])
def test_rope_table_against_reference_table(tmp_path, name, n_pos):
    """The oracle's angle table (ggml's schedule: theta_i by iterated float
    products, angle pos * theta_i in float, A2) against the reference MoE
    engine's (pos * base^(-2i/hd) in double, qwen_model.c:346-353) for NEOX
    without freq factors: every entry within (pos + 1) * 2^-22 + 2^-22 -- the
    float angle's relative error is a few 2^-24, times an angle of up to pos
    radians."""
    ra = O.reference_attention()
    if ra is None:
        pytest.skip("oracle/_ref/libref_attention.so not built (no reference checkout on this host)")
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import ref_gguf
    sp = specs.get(name)
    sp.update(rope_mode=2, rope_freq_factors=None)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    gguf = ref_gguf.write(str(tmp_path / "model.gguf"), hq, hkv, d, sp["rope_base"])
    z = np.zeros((1, hkv * d), np.float32)
    ref = ra.step(gguf, n_pos, 0, z[:0], z[:0], np.zeros(hq * d, np.float32), z, z, False, hq, hkv, d)
    tab = O.Oracle(sp).rope_table(0, n_pos)
    bound = (np.arange(n_pos, dtype=np.float64)[:, None] + 2.0) * 2.0 ** -22
    assert np.all(np.abs(tab[:, :, 0] - ref[3]) <= bound)
    assert np.all(np.abs(tab[:, :, 1] - ref[4]) <= bound)
    # position 0 exactly: cos 1, sin 0
    assert np.all(tab[0, :, 0] == 1.0) and np.all(ref[3][0] == 1.0)


def _causal_mask(n_past, n_new, stride, dtype):
    m = np.full((n_new, stride), -np.inf, dtype)
    for t in range(n_new):
        m[t, : n_past + t + 1] = 0
    return m


def _np_attention_masked(sp, n_past, q_roped, kc, vc, mask, flash):
    """float64 restatement with an explicit additive mask: the default branch
    (A5, F16-rounded normalised weights) or the flash branch (A6, exact)."""
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    r = hq // hkv
    n_new = q_roped.shape[0]
    n_kv = n_past + n_new
    scale = np.float32(1.0) / np.sqrt(np.float32(d))
    K = kc[:n_kv].view(np.float16).astype(np.float64)
    V = vc[:n_kv].view(np.float16).astype(np.float64)
    q16 = q_roped.astype(np.float16).astype(np.float64)
    out = np.zeros((n_new, hq * d))
    for t in range(n_new):
        mrow = mask[t, :n_kv].astype(np.float32)
        for h in range(hq):
            kv = h // r
            s = ((K[:, kv] @ q16[t, h]).astype(np.float32) * scale + mrow).astype(np.float32)
            if flash:
                if s.max() == -np.inf:
                    continue
                e = np.exp(s.astype(np.float64) - float(s.max()))
                out[t, h * d:(h + 1) * d] = (e / e.sum()) @ V[:, kv]
            else:
                e = np.exp((s - s.max()).astype(np.float64)).astype(np.float32)
                p = (e * np.float32(1.0 / e.astype(np.float64).sum())).astype(np.float16).astype(np.float64)
                out[t, h * d:(h + 1) * d] = p @ V[:, kv]
    return out


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_explicit_causal_mask_equals_implicit(dtype):
    """kvo_attend_ex with the causal mask of model.cpp:1579-1586 (padded rows)
    is kvo_attend bit for bit: adding 0 after the scale changes no score."""
    case = G.CASES[6]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    n_past = case["n_past"]
    q_roped = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    n_new = q_roped.shape[0]
    mask = _causal_mask(n_past, n_new, n_past + n_new + 13, dtype)
    a = orc.attend(kc, vc, n_past, q_roped)
    b = orc.attend_ex(kc, vc, n_past, q_roped, mask=mask)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("flash", [False, True])
def test_window_mask_matches_float64_restatement(flash):
    """A sliding-window F16 mask (keys in (pos - 96, pos]) in both branches."""
    case = G.CASES[6]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    n_past = case["n_past"]
    q_roped = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    n_new = q_roped.shape[0]
    mask = np.full((n_new, n_past + n_new), -np.inf, np.float16)
    for t in range(n_new):
        pos = n_past + t
        mask[t, max(0, pos - 95): pos + 1] = 0
    got = orc.attend_ex(kc, vc, n_past, q_roped, mask=mask, flash=flash)
    want = _np_attention_masked(sp, n_past, q_roped, kc, vc, mask, flash)
    assert np.abs(got - want).max() < 1e-4
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 3e-5


def test_flash_branch_and_fully_masked_rows():
    """The flash branch equals exact softmax(s) . V; a row whose keys are all
    masked gives 0 there and NaN in the default branch (ggml's soft_max)."""
    case = G.CASES[6]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    n_past = case["n_past"]
    q_roped = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    n_new = q_roped.shape[0]
    mask = _causal_mask(n_past, n_new, n_past + n_new, np.float32)
    mask[0, :] = -np.inf                      # token 0 sees nothing
    fl = orc.attend_ex(kc, vc, n_past, q_roped, mask=mask, flash=True)
    de = orc.attend_ex(kc, vc, n_past, q_roped, mask=mask, flash=False)
    assert np.all(fl[0] == 0.0) and np.all(np.isnan(de[0]))
    want = _np_attention_masked(sp, n_past, q_roped, kc, vc, mask, True)
    assert np.abs(fl[1:] - want[1:]).max() < 2e-6
    # the two branches differ by the F16 rounding of the normalised weights only
    assert np.abs(fl[1:] - de[1:]).max() < 1e-3


def _dory_mask(n_cells, pos0, n_tokens):
    """dory_fill_attn_mask (dory.c:553-575), restated with Python's floor mod."""
    head = pos0 + n_tokens - 1
    m = np.full((n_tokens, n_cells), -np.inf, np.float32)
    for q in range(n_tokens):
        for c in range(n_cells):
            lw = head - ((head - c) % n_cells)
            if 0 <= lw <= pos0 + q:
                m[q, c] = 0.0
    return m


@pytest.mark.parametrize("n_cells,pos0,n_tokens", [(8, 0, 1), (8, 5, 3), (4, 6, 3), (16, 40, 16), (7, 3, 7),
                                                   (32, 100, 1), (1, 9, 1)])
def test_ring_mask_matches_dory_rule(n_cells, pos0, n_tokens):
    assert np.array_equal(O.ring_mask(n_cells, pos0, n_tokens), _dory_mask(n_cells, pos0, n_tokens))


def test_ring_append_rows_and_attention():
    """kvo_append_ring puts position p in cell p % n_cells with the linear
    append's bits; attend_ring over the cells equals the linear attention
    restricted to the visible positions (a ring holding the last n_cells)."""
    case = G.CASES[6]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    hkv, d = sp["n_head_kv"], sp["head_dim"]
    n_cells, n_pos = 16, 40
    lin_k = np.zeros((n_pos, hkv, d), np.uint16)
    lin_v = np.zeros((n_pos, hkv, d), np.uint16)
    ring_k = np.zeros((n_cells, hkv, d), np.uint16)
    ring_v = np.zeros((n_cells, hkv, d), np.uint16)
    for pos0 in range(0, n_pos, 5):
        rr = synth.qkv_rows(sp, pos0, 0, 5)
        hq = sp["n_head"]
        qq, kk, vv = rr[:, :hq * d], rr[:, hq * d:(hq + hkv) * d], rr[:, (hq + hkv) * d:]
        a = orc.append(lin_k, lin_v, pos0, qq, kk, vv, qn, kn)
        b = orc.append_ring(ring_k, ring_v, pos0, qq, kk, vv, qn, kn)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        for t in range(5):
            assert np.array_equal(ring_k[(pos0 + t) % n_cells], lin_k[pos0 + t])
            assert np.array_equal(ring_v[(pos0 + t) % n_cells], lin_v[pos0 + t])
        got = orc.attend_ring(ring_k, ring_v, pos0, b)
        # the same attention on the linear cache: keys (head - n_cells, p] visible
        head = pos0 + 4
        mask = np.full((5, pos0 + 5), -np.inf, np.float32)
        for t in range(5):
            mask[t, max(0, head - n_cells + 1): pos0 + t + 1] = 0
        want = orc.attend_ex(lin_k, lin_v, pos0, b, mask=mask)
        assert np.abs(got - want).max() < 2e-6


def test_ngpt_norm_matches_ggml_arithmetic():
    """dory's L2 norm (dory.c:577-580) as ggml computes it: A1's rms_norm with
    eps 1e-6/n (float squares summed in double), then * (1/sqrt(n)) and the
    squared scale, each a rounded float multiply."""
    rng = np.random.default_rng(5)
    n = 256
    x = rng.standard_normal(n).astype(np.float32)
    w = rng.uniform(2.0, 6.0, n).astype(np.float32)
    sq = (x * x).astype(np.float32)
    mean = np.float32(np.cumsum(sq.astype(np.float64))[-1] / n)
    sc = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(np.float32(1e-6) / np.float32(n))))
    post = np.float32(1.0) / np.sqrt(np.float32(n))
    want = (((x * sc).astype(np.float32) * post).astype(np.float32) * w).astype(np.float32)
    got = np.zeros(n, np.float32)
    O.lib().kvo_ngpt_norm(_fp(x), _fp(w), n, 1e-6, _fp(got))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_ngpt_append_rotates_then_normalises():
    """qk_norm 2: the cached K row is rope(k) normalised (unit RMS * 1/16 at
    head_dim 256: L2 norm 1), Q additionally scaled."""
    sp = specs.get("llama3.2-3b")
    sp.update(n_layer=1, n_head=16, n_head_kv=4, head_dim=256, n_rot=256, rope_mode=2, rope_base=1e4,
              rope_freq_factors=None, qk_norm=2)
    orc = O.Oracle(sp)
    kc = np.zeros((8, 4, 256), np.uint16)
    vc = np.zeros((8, 4, 256), np.uint16)
    rows = synth.qkv_rows(sp, 1, 0, 3)
    q, k, v = rows[:, :16 * 256], rows[:, 16 * 256:20 * 256], rows[:, 20 * 256:]
    qs = np.full(16 * 256, 3.0, np.float32)
    qr = orc.append_ring(kc, vc, 5, q, k, v, qs, None)
    kn = np.linalg.norm(kc[5:8].view(np.float16).astype(np.float64), axis=-1)
    assert np.allclose(kn, 1.0, atol=2e-3)
    assert np.allclose(np.linalg.norm(qr.astype(np.float64), axis=-1), 3.0, atol=1e-4)


def test_masked_and_flash_attention_thread_count_invariant():
    """The masked and flash restatements do not depend on the thread count either."""
    case = G.CASES[6]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    n_past = case["n_past"]
    q_roped = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    n_new = q_roped.shape[0]
    mask = np.full((n_new, n_past + n_new), -np.inf, np.float16)
    for t in range(n_new):
        mask[t, max(0, n_past + t - 30): n_past + t + 1] = 0
    for flash in (False, True):
        a = orc.attend_ex(kc, vc, n_past, q_roped, mask=mask, flash=flash, n_threads=1)
        b = orc.attend_ex(kc, vc, n_past, q_roped, mask=mask, flash=flash, n_threads=7)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_attention_thread_count_invariant():
    case = G.CASES[6]
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    q_roped = orc.append(kc, vc, case["n_past"], q, k, v, qn, kn)
    a = orc.attend(kc, vc, case["n_past"], q_roped, n_threads=1)
    b = orc.attend(kc, vc, case["n_past"], q_roped, n_threads=8)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_append_matches_numpy_restatement():
    """kvo_append == numpy float32 ops (no FMA) with the oracle's RoPE table."""
    case = G.CASES[6]   # qwen3: QK-Norm + NEOX
    sp, kc, vc, rows, q, k, v, qn, kn = G.case_inputs(case)
    orc = O.Oracle(sp)
    n_past, n_new, d = case["n_past"], case["n_new"], sp["head_dim"]
    q_roped = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    cs = orc.rope_table(n_past, n_new)
    half = d // 2

    def norm(x, w):
        sq = (x * x).astype(np.float32).astype(np.float64)
        mean = np.float32(np.cumsum(sq)[-1] / d)
        sc = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(sp["rms_eps"])))
        return ((x * sc).astype(np.float32) * w).astype(np.float32)

    def rope(x, c):
        y = x.copy()
        a, b = x[:half], x[half:]
        y[:half] = (a * c[:, 0]).astype(np.float32) - (b * c[:, 1]).astype(np.float32)
        y[half:] = (a * c[:, 1]).astype(np.float32) + (b * c[:, 0]).astype(np.float32)
        return y

    hkv = sp["n_head_kv"]
    for t in range(n_new):
        for h in range(hkv):
            x = k[t, h * d:(h + 1) * d]
            want = rope(norm(x, kn), cs[t]).astype(np.float16).view(np.uint16)
            assert np.array_equal(kc[n_past + t, h], want)
            assert np.array_equal(vc[n_past + t, h], v[t, h * d:(h + 1) * d].astype(np.float16).view(np.uint16))
        for h in range(sp["n_head"]):
            want = rope(norm(q[t, h * d:(h + 1) * d], qn), cs[t])
            assert np.array_equal(q_roped[t, h].view(np.uint32), want.view(np.uint32))


# ---------------------------------------------------------------------------
# sizing (model.cpp:869-885, 1002-1059)
# ---------------------------------------------------------------------------

def test_kv_cache_bytes_reference_rule():
    for sp in specs.specs().values():
        want = sp["n_layer"] * sp["head_dim"] * sp["n_head_kv"] * 2 * 2 * sp["n_ctx"]
        assert O.kv_cache_bytes(sp["n_layer"], sp["n_head_kv"], sp["head_dim"], sp["n_ctx"]) == want
    # 128k llama-3.1-8B cache: 16 GiB
    assert O.kv_cache_bytes(32, 8, 128, 131072) == 16 * 2 ** 30


def test_auto_n_ctx_reference_rule():
    MiB = 2 ** 20
    assert O.auto_n_ctx(-1, 1000) == 4096                          # unreadable -> N_CTX_DEFAULT
    per = 131072                                                   # 128 KiB / position
    avail = 4096 * MiB
    raw = int((avail - 384 * MiB) * 0.8) // per
    assert O.auto_n_ctx(avail, per) == (raw // 64) * 64
    assert O.auto_n_ctx(avail, per, n_ctx_train=2048) == 2048      # clamp to trained ctx
    assert O.auto_n_ctx(400 * MiB, per) == 512                     # floor
    assert O.auto_n_ctx(400 * MiB, per, n_ctx_train=256) == 256    # floor never above the limit
    assert O.auto_n_ctx(10 ** 15, per) == 262144                   # default cap
    assert O.auto_n_ctx(10 ** 15, per, 131072, longrope_orig=4096) == 4096


# ---------------------------------------------------------------------------
# golden fixtures (regression pin of the oracle)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", G.CASES, ids=[c["name"] for c in G.CASES])
def test_golden_fixture(case):
    want = G.load(case)
    got = G.run_oracle(case)
    for key in ("k_new", "v_new"):
        assert np.array_equal(got[key], want[key]), key
    for key in ("q_roped", "out"):
        assert np.array_equal(got[key].view(np.uint32), want[key].view(np.uint32)), key
