"""GPU parity tests of the path through the C ABI (include/kv_api.h).

Bar: appended cache bytes bit-exact against the CPU oracle; attention outputs
within max-abs 2e-3 and relative L2 1e-3 (F32) of the oracle -- the tolerance
set for the path's floating-point outputs.  Covers the golden fixtures of every
benchmark shape, the full-size decode of the 32k and 128k shapes, and the
edge cases of the reference's cache contract (first token, rewind by
overwrite, multi-pass query rows, separate/fused/unaligned input rows).
"""
import os
import sys

import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden as G  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
REL_L2 = 1e-3


def assert_close(got, want, max_abs=MAX_ABS, rel_l2=REL_L2):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.all(np.isfinite(got))
    d = got - want
    ma = float(np.abs(d).max())
    rl = float(np.linalg.norm(d) / max(np.linalg.norm(want), 1e-30))
    assert ma <= max_abs and rl <= rel_l2, "max-abs %.3g (tol %.1g), rel-L2 %.3g (tol %.1g)" % (
        ma, max_abs, rl, rel_l2)
    return ma, rl


class Run:
    """One layer-0 context of a golden case, filled and driven on the GPU."""

    def __init__(self, case, cuda, n_batch_max=None):
        import torch
        self.torch = torch
        self.case = case
        self.sp = G.case_spec(case)
        sp = self.sp
        self.cfg = K.make_config(sp, n_ctx=case["n_ctx"], n_batch_max=n_batch_max or max(16, case["n_new"]))
        self.ctx = K.Context(self.cfg)
        self.stream = torch.cuda.current_stream()
        if case["n_past"] > 0:
            self.ctx.fill_synthetic(sp["seed"], 0, case["n_past"], stream=self.stream)
        self.hq, self.hkv, self.d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        self.width = (self.hq + 2 * self.hkv) * self.d
        self.qn = self.kn = None
        if sp["qk_norm"]:
            qn, kn = synth.norm_weights(sp, 0)
            self.qn = torch.from_numpy(qn).to(cuda)
            self.kn = torch.from_numpy(kn).to(cuda)
        self.cuda = cuda

    def step(self, rows_np, n_past, layer=0):
        torch = self.torch
        n_new = rows_np.shape[0]
        rows = torch.from_numpy(np.ascontiguousarray(rows_np, np.float32)).to(self.cuda)
        base = rows.data_ptr()
        w = rows_np.shape[1]
        self.ctx.append(layer, n_past, n_new, base, w, base + 4 * self.hq * self.d, w,
                        base + 4 * (self.hq + self.hkv) * self.d, w, self.qn, self.kn, stream=self.stream)
        out = torch.full((n_new, self.hq * self.d), float("nan"), device=self.cuda)
        self.ctx.attend(layer, n_past, n_new, out, stream=self.stream)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    def rows(self, which, row0, nrows, layer=0):
        return self.ctx.export_rows(layer, which, row0, nrows)


@pytest.mark.parametrize("case", G.CASES, ids=[c["name"] for c in G.CASES])
def test_golden_case(case, cuda):
    run = Run(case, cuda)
    n_past, n_new = case["n_past"], case["n_new"]
    # the device generator filled rows [0, n_past) with the oracle's bits
    want_k = O.gen_cache_rows(run.sp["seed"], synth.STREAM_CACHE + 0, 0, n_past, run.hkv, run.d)
    assert np.array_equal(run.rows(0, 0, n_past), want_k)
    out = run.step(synth.qkv_rows(run.sp, 0, 0, n_new), n_past)
    gold = G.load(case)
    assert np.array_equal(run.rows(0, n_past, n_new), gold["k_new"]), "K rows differ from the CPU path"
    assert np.array_equal(run.rows(1, n_past, n_new), gold["v_new"]), "V rows differ from the CPU path"
    assert_close(out, gold["out"])


def test_gen_normal_device_matches_host(cuda):
    import torch
    n = 100003
    dst = torch.empty(n, dtype=torch.float32, device=cuda)
    K.gen_normal_device(dst, 0x1234, synth.STREAM_QKV + 7, n, idx0=99)
    torch.cuda.synchronize()
    want = synth.normal(0x1234, synth.STREAM_QKV + 7, n, idx0=99)
    assert np.array_equal(dst.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_separate_and_unaligned_inputs_give_same_bits(cuda):
    """q, k, v as three contiguous tensors, and rows with an odd stride
    (scalar-load path), append the same bytes as the fused row."""
    import torch
    case = dict(G.CASES[6])  # qwen3 chunk of 8: QK-Norm + NEOX
    run = Run(case, cuda)
    n_past, n_new = case["n_past"], case["n_new"]
    rows = synth.qkv_rows(run.sp, 0, 0, n_new)
    hq, hkv, d = run.hq, run.hkv, run.d
    gold = G.load(case)
    # separate tensors
    q = torch.from_numpy(np.ascontiguousarray(rows[:, :hq * d])).to(cuda)
    k = torch.from_numpy(np.ascontiguousarray(rows[:, hq * d:(hq + hkv) * d])).to(cuda)
    v = torch.from_numpy(np.ascontiguousarray(rows[:, (hq + hkv) * d:])).to(cuda)
    run.ctx.append(0, n_past, n_new, q, hq * d, k, hkv * d, v, hkv * d, run.qn, run.kn, stream=run.stream)
    out = torch.zeros(n_new, hq * d, device=cuda)
    run.ctx.attend(0, n_past, n_new, out, stream=run.stream)
    torch.cuda.synchronize()
    assert np.array_equal(run.rows(0, n_past, n_new), gold["k_new"])
    assert_close(out.cpu().numpy(), gold["out"])
    # odd row stride, misaligned base
    pad = np.zeros((n_new, rows.shape[1] + 3), np.float32)
    pad[:, 1:1 + rows.shape[1]] = rows
    t = torch.from_numpy(pad).to(cuda)
    base = t.data_ptr() + 4
    w = pad.shape[1]
    run.ctx.append(0, n_past, n_new, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w,
                   run.qn, run.kn, stream=run.stream)
    run.ctx.attend(0, n_past, n_new, out, stream=run.stream)
    torch.cuda.synchronize()
    assert np.array_equal(run.rows(0, n_past, n_new), gold["k_new"])
    assert np.array_equal(run.rows(1, n_past, n_new), gold["v_new"])
    assert_close(out.cpu().numpy(), gold["out"])


def _oracle_layer(sp, n_ctx, n_past_fill):
    hkv, d = sp["n_head_kv"], sp["head_dim"]
    kc = np.zeros((n_ctx, hkv, d), np.uint16)
    vc = np.zeros((n_ctx, hkv, d), np.uint16)
    if n_past_fill:
        kc[:n_past_fill] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE, 0, n_past_fill, hkv, d)
        vc[:n_past_fill] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 1, 0, n_past_fill, hkv, d)
    return kc, vc


def _split(sp, rows):
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    return rows[:, :hq * d], rows[:, hq * d:(hq + hkv) * d], rows[:, (hq + hkv) * d:]


def test_first_token_and_rewind(cuda):
    """n_past = 0 (a single visible key), then a rewind: rows are overwritten
    and only rows < n_past + n_new are read (cmd_chat.cpp:749-764)."""
    case = dict(name="rewind", spec="llama3.2-3b", n_ctx=256, n_past=0, n_new=1)
    run = Run(case, cuda)
    sp = run.sp
    orc = O.Oracle(sp)
    kc, vc = _oracle_layer(sp, 256, 0)
    n_past = 0
    for step in range(40):                       # 40 decode steps from an empty cache
        rows = synth.qkv_rows(sp, step, 0, 1)
        out = run.step(rows, n_past)
        q, k, v = _split(sp, rows)
        qr = orc.append(kc, vc, n_past, q, k, v)
        if step in (0, 1, 39):
            assert_close(out, orc.attend(kc, vc, n_past, qr))
        n_past += 1
    # rewind to 10 and write different tokens over rows 10..14
    n_past = 10
    rows = synth.qkv_rows(sp, 1000, 0, 5)
    out = run.step(rows, n_past)
    q, k, v = _split(sp, rows)
    qr = orc.append(kc, vc, n_past, q, k, v)
    assert np.array_equal(run.rows(0, 0, 40), kc[:40])
    assert np.array_equal(run.rows(1, 0, 40), vc[:40])
    assert_close(out, orc.attend(kc, vc, n_past, qr))


@pytest.mark.parametrize("name,n_past,n_new", [
    ("llama3.2-3b", 3000, 1), ("phi3-mini", 3968, 1), ("qwen2-0.5b", 2048, 1),
    ("qwen3-8b-prefill", 4000, 33), ("llama3.1-8b-128k", 5000, 2),
])
def test_mid_size_matches_oracle(name, n_past, n_new, cuda):
    sp = specs.get(name)
    sp["n_layer"] = 1
    n_ctx = n_past + 128
    case = dict(name=name, spec=name, n_ctx=n_ctx, n_past=n_past, n_new=n_new)
    run = Run(case, cuda, n_batch_max=64)
    run.sp = sp
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    rows = synth.qkv_rows(sp, 3, 0, n_new)
    out = run.step(rows, n_past)
    q, k, v = _split(sp, rows)
    qn, kn = synth.norm_weights(sp, 0) if sp["qk_norm"] else (None, None)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    assert np.array_equal(run.rows(1, n_past, n_new), vc[n_past:n_past + n_new])
    assert_close(out, orc.attend(kc, vc, n_past, qr))


@pytest.mark.parametrize("n_new", [1, 24])
def test_no_rope_layers_match_oracle(n_new, cuda):
    """Attention layers without positional encoding (nemotron_h: model.cpp:1389
    skips ggml_rope_ext when hp.no_rope) are a context with n_rot = 0: the
    append stores the raw (normalised) K rows, decode and chunk alike."""
    sp = specs.get("llama3.2-3b")
    sp.update(n_layer=1, n_rot=0, rope_freq_factors=None)
    n_past = 3000
    n_ctx = n_past + 64
    case = dict(name="no-rope", spec="llama3.2-3b", n_ctx=n_ctx, n_past=n_past, n_new=n_new)
    run = Run(case, cuda, n_batch_max=64)
    run.sp = sp
    run.ctx.close()
    run.cfg = K.make_config(sp, n_ctx=n_ctx, n_batch_max=64)
    run.ctx = K.Context(run.cfg)
    run.ctx.fill_synthetic(sp["seed"], 0, n_past, stream=run.stream)
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    rows = synth.qkv_rows(sp, 4, 0, n_new)
    out = run.step(rows, n_past)
    q, k, v = _split(sp, rows)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v)
    hkv, d = sp["n_head_kv"], sp["head_dim"]
    # the stored K rows are the inputs rounded to F16, unrotated
    assert np.array_equal(kc[n_past:n_past + n_new], O.f32_to_f16_bits(k.reshape(n_new, hkv, d)))
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    assert np.array_equal(run.rows(1, n_past, n_new), vc[n_past:n_past + n_new])
    assert_close(out, orc.attend(kc, vc, n_past, qr))


@pytest.mark.parametrize("name,n_past,n_new", [
    ("qwen3-8b-prefill", 64, 8),       # one key tile per pair: every pair written by its own CTA
    ("qwen3-8b-prefill", 300, 200),    # pairs split over CTAs (fold), a last block with an empty tile B
    ("llama3.2-3b", 1000, 40),         # r = 3: 42 tokens per tile, 2 rows of each tile unused
    ("qwen2-0.5b", 150, 5),            # head_dim 64, r = 7
    ("qwen3-8b-prefill", 16384, 512),  # the benchmark chunk
    ("qwen3-8b-prefill", 40000, 40),   # past 32k keys: the exact two passes
    ("llama3.1-8b-128k", 120000, 33),  # 128k-class context, exact passes, pairs over many CTAs
    ("phi3-mini", 3000, 64),           # head_dim 96 on the 128 kernel (zero-filled columns), MHA
    ("phi3-mini", 500, 300),           # head_dim 96, pairs split over CTAs (fold writes 96 columns)
])
def test_prefill_chunk_matches_oracle(name, n_past, n_new, cuda):
    """The tensor-core chunk path against the oracle's ggml softmax, within the
    attention tolerance: the one-pass online softmax up to 32k keys, the exact
    statistics + output passes beyond (where ggml's F16 rounding of normalised
    weights, subnormal at long context, matters)."""
    sp = specs.get(name)
    sp["n_layer"] = 1
    n_ctx = n_past + n_new + 64
    case = dict(name=name, spec=name, n_ctx=n_ctx, n_past=n_past, n_new=n_new)
    run = Run(case, cuda, n_batch_max=max(64, n_new))
    run.sp = sp
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    rows = synth.qkv_rows(sp, 3, 0, n_new)
    run.ctx.profile(True)
    out = run.step(rows, n_past)
    # the tensor-core path ran: one pass (on CTA pairs at head_dim 128), or the exact two
    one_pass = n_past + n_new <= 32768
    pair = one_pass and sp["head_dim"] == 128
    assert run.ctx.profile_read("prefill2")[0] == (1 if pair else 0)
    assert run.ctx.profile_read("prefill")[0] == (0 if pair else 1 if one_pass else 2)
    q, k, v = _split(sp, rows)
    qn, kn = synth.norm_weights(sp, 0) if sp["qk_norm"] else (None, None)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    assert_close(out, orc.attend(kc, vc, n_past, qr))


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("name,n_past,n_new", [
    ("qwen3-8b-prefill", 16384, 512),  # the benchmark chunk: 4 blocks of 128 tokens a KV head
    ("qwen3-8b-prefill", 300, 200),    # a last block with two tiles past the chunk's end, pairs split (fold)
    ("qwen3-8b-prefill", 64, 40),      # one block: the odd CTA's tiles lie past the query buffer's rows
    ("llama3.2-3b", 5000, 90),         # r = 3 (42 tokens a tile, 126 rows), three of the four tiles in use
])
def test_prefill_on_cta_pairs_matches_oracle(name, n_past, n_new, pair, cuda, monkeypatch):
    """The one-pass chunk kernel on CTA pairs (2-CTA clusters, tcgen05
    cta_group::2: M = 256 MMAs over both SMs, each CTA staging half of every K
    and V tile) and the one-CTA kernel (KV_B200_PREFILL_PAIR=0) on the same
    chunks, both within the attention tolerance of the oracle."""
    monkeypatch.setenv("KV_B200_PREFILL_PAIR", pair)
    sp = specs.get(name)
    sp["n_layer"] = 1
    n_ctx = n_past + n_new + 64
    case = dict(name=name, spec=name, n_ctx=n_ctx, n_past=n_past, n_new=n_new)
    run = Run(case, cuda, n_batch_max=n_new)
    run.sp = sp
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    rows = synth.qkv_rows(sp, 4, 0, n_new)
    run.ctx.profile(True)
    out = run.step(rows, n_past)
    assert run.ctx.profile_read("prefill2")[0] == (1 if pair == "1" else 0)
    assert run.ctx.profile_read("prefill")[0] == (0 if pair == "1" else 1)
    q, k, v = _split(sp, rows)
    qn, kn = synth.norm_weights(sp, 0) if sp["qk_norm"] else (None, None)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    assert_close(out, orc.attend(kc, vc, n_past, qr))
    run.ctx.status()


@pytest.mark.parametrize("n_new", [1, 40])
def test_qkv_bias_matches_oracle(n_new, cuda):
    """kv_append_bias: qwen2's projection biases (model.cpp:1099-1102, ggml_add
    in F32) added inside the append -- the fused decode append (one token) and
    the chunk kernel -- give the oracle's cache bytes after the same add."""
    import torch
    sp = specs.get("qwen2-0.5b")
    sp["n_layer"] = 1
    n_past = 700
    case = dict(name="bias", spec="qwen2-0.5b", n_ctx=1024, n_past=n_past, n_new=n_new)
    run = Run(case, cuda, n_batch_max=64)
    run.sp = sp
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    rng = np.random.default_rng(7)
    bq = rng.uniform(-2, 2, hq * d).astype(np.float32)
    bk = rng.uniform(-2, 2, hkv * d).astype(np.float32)
    bv = rng.uniform(-2, 2, hkv * d).astype(np.float32)
    rows = synth.qkv_rows(sp, 5, 0, n_new)
    t = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
    tb = [torch.from_numpy(x).to(cuda) for x in (bq, bk, bv)]
    b, w = t.data_ptr(), rows.shape[1]
    run.ctx.append_bias(0, n_past, n_new, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w,
                        None, None, tb[0], tb[1], tb[2], stream=run.stream)
    out = torch.full((n_new, hq * d), float("nan"), device=cuda)
    run.ctx.attend(0, n_past, n_new, out, stream=run.stream)
    torch.cuda.synchronize()
    kc, vc = _oracle_layer(sp, case["n_ctx"], n_past)
    q, k, v = _split(sp, rows)
    # ggml_add: one F32 add per element, before RoPE
    q, k, v = (np.ascontiguousarray(x + bb, np.float32) for x, bb in ((q, bq), (k, bk), (v, bv)))
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v)
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    assert np.array_equal(run.rows(1, n_past, n_new), vc[n_past:n_past + n_new])
    assert_close(out.cpu().numpy(), orc.attend(kc, vc, n_past, qr))


def test_qk_norm_fallback_rows_match_oracle_bits(cuda):
    """QK-Norm rows whose sum of squares is tiny, or whose squares span many
    binades, leave the exact-integer fast path for the sequential double sum;
    the cache bytes still equal the oracle's."""
    sp = specs.get("qwen3-8b-prefill")
    sp["n_layer"] = 1
    n_past, n_new = 100, 40
    case = dict(name="qkn", spec="qwen3-8b-prefill", n_ctx=256, n_past=n_past, n_new=n_new)
    run = Run(case, cuda, n_batch_max=64)
    run.sp = sp
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    rows = synth.qkv_rows(sp, 11, 0, n_new).astype(np.float32)
    k0 = hq * d
    rows[0:8, k0:k0 + hkv * d] *= np.float32(1e-17)            # tiny sums: below the fast path's range
    rows[8:16, :hq * d] *= np.float32(1e-19)
    rows[16:24, k0:k0 + d] = np.float32(1e-30)                   # squares 2^-200 apart from ...
    rows[16:24, k0] = np.float32(3.0)                            # ... one large element
    rows[24:32, k0 + 3 * d:k0 + 4 * d:2] = 0.0                   # half the elements zero
    kc, vc = _oracle_layer(sp, case["n_ctx"], n_past)
    out = run.step(rows, n_past)
    q, k, v = _split(sp, rows)
    qn, kn = synth.norm_weights(sp, 0)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    assert np.array_equal(run.rows(1, n_past, n_new), vc[n_past:n_past + n_new])
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("name", ["llama3.2-3b", "llama3.1-8b-128k"])
def test_full_context_decode_matches_oracle(name, cuda):
    """One layer at the benchmark's full context (32001 / 131001 keys)."""
    sp = specs.get(name)
    sp["n_layer"] = 1
    n_past = sp["n_past"]
    case = dict(name=name, spec=name, n_ctx=sp["n_ctx"], n_past=n_past, n_new=1)
    run = Run(case, cuda)
    run.sp = sp
    kc, vc = _oracle_layer(sp, sp["n_ctx"], n_past)
    rows = synth.qkv_rows(sp, 0, 0, 1)
    out = run.step(rows, n_past)
    q, k, v = _split(sp, rows)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v)
    assert np.array_equal(run.rows(0, n_past, 1), kc[n_past:n_past + 1])
    # spot-check the device fill at the far end of the context
    assert np.array_equal(run.rows(1, n_past - 3, 3), vc[n_past - 3:n_past])
    assert_close(out, orc.attend(kc, vc, n_past, qr))


def test_doubling_v_doubles_output_exactly(cuda):
    """Size-independent property: P does not depend on V, and scaling V by 2 is
    exact in F16 and in every F32 product and sum, so out doubles bit for bit."""
    case = dict(name="lin", spec="llama3.2-3b", n_ctx=20000, n_past=19000, n_new=1)
    run = Run(case, cuda)
    rows = synth.qkv_rows(run.sp, 0, 0, 1)
    out1 = run.step(rows, 19000)
    v = run.rows(1, 0, 19001).view(np.float16)
    run.ctx.import_rows(0, 1, 0, (v * np.float16(2)).view(np.uint16))
    rows2 = rows.copy()
    hq, hkv, d = run.hq, run.hkv, run.d
    rows2[:, (hq + hkv) * d:] *= 2
    out2 = run.step(rows2, 19000)
    assert np.array_equal((out1 * 2).view(np.uint32), out2.view(np.uint32))


def test_forward_all_layers(cuda):
    import torch
    sp = specs.get("qwen3-8b-prefill")
    sp["n_layer"] = 3
    n_ctx, n_past, n_new = 512, 300, 4
    cfg = K.make_config(sp, n_ctx=n_ctx, n_batch_max=16)
    ctx = K.Context(cfg)
    ctx.fill_synthetic(sp["seed"], 0, n_past)
    hq, d = sp["n_head"], sp["head_dim"]
    w = specs.row_width(sp)
    rows = np.stack([synth.qkv_rows(sp, 0, l, n_new) for l in range(3)])
    norms = [synth.norm_weights(sp, l) for l in range(3)]
    qn = np.stack([n[0] for n in norms])
    kn = np.stack([n[1] for n in norms])
    tr = torch.from_numpy(rows).to(cuda)
    tqn, tkn = torch.from_numpy(qn).to(cuda), torch.from_numpy(kn).to(cuda)
    out = torch.zeros(3, n_new, hq * d, device=cuda)
    b = tr.data_ptr()
    ctx.forward(n_past, n_new, b, w, b + 4 * hq * d, w, b + 4 * (hq + 8) * d, w, n_new * w,
                tqn, tkn, d, out, n_new * hq * d)
    torch.cuda.synchronize()
    out = out.cpu().numpy()
    orc = O.Oracle(sp)
    for l in range(3):
        hkv = sp["n_head_kv"]
        kc = np.zeros((n_ctx, hkv, d), np.uint16)
        vc = np.zeros((n_ctx, hkv, d), np.uint16)
        kc[:n_past] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 2 * l, 0, n_past, hkv, d)
        vc[:n_past] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 2 * l + 1, 0, n_past, hkv, d)
        q, k, v = _split(sp, rows[l])
        qr = orc.append(kc, vc, n_past, q, k, v, qn[l], kn[l])
        assert np.array_equal(ctx.export_rows(l, 0, 0, n_past + n_new), kc[:n_past + n_new])
        assert_close(out[l], orc.attend(kc, vc, n_past, qr))
    ctx.close()


def test_errors_are_codes_not_crashes(cuda):
    import torch
    sp = specs.get("llama3.2-3b")
    sp["n_layer"] = 2
    ctx = K.Context(K.make_config(sp, n_ctx=128, n_batch_max=8))
    out = torch.zeros(16, sp["n_head"] * sp["head_dim"], device=cuda)
    rows = torch.zeros(16, specs.row_width(sp), device=cuda)
    w = specs.row_width(sp)
    with pytest.raises(K.KvError) as e:       # attend before any append
        ctx.attend(0, 0, 1, out)
    assert e.value.code == K.KV_E_STATE
    with pytest.raises(K.KvError) as e:       # past the end of the cache
        ctx.append(0, 127, 2, rows, w, rows, w, rows, w)
    assert e.value.code == K.KV_E_RANGE
    with pytest.raises(K.KvError) as e:       # above n_batch_max
        ctx.append(0, 0, 9, rows, w, rows, w, rows, w)
    assert e.value.code == K.KV_E_RANGE
    with pytest.raises(K.KvError) as e:
        ctx.append(2, 0, 1, rows, w, rows, w, rows, w)
    assert e.value.code == K.KV_E_ARG
    ctx.append(1, 5, 1, rows, w, rows, w, rows, w)
    with pytest.raises(K.KvError) as e:       # attend of another layer than the append
        ctx.attend(0, 5, 1, out)
    assert e.value.code == K.KV_E_STATE
    ctx.close()


def test_auto_n_ctx_allocation(cuda):
    sp = specs.get("qwen2-0.5b")
    sp["n_ctx_train"] = 8192
    cfg = K.make_config(sp, n_ctx=0)
    with K.Context(cfg) as ctx:
        assert ctx.n_ctx == 8192


def test_expired_wait_reports_timeout_and_context_recovers(cuda):
    """Failure detection without a fault: the test hook makes the tile producer
    withhold one tile, so the consumers' bounded mbarrier wait (shortened to
    50 ms here) expires.  The kernel records the error word and returns; the
    host reads KV_E_TIMEOUT from kv_status, and the next call is correct."""
    case = dict(name="inject", spec="llama3.2-3b", n_ctx=4096, n_past=3000, n_new=1)
    run = Run(case, cuda)
    sp = run.sp
    rows = synth.qkv_rows(sp, 0, 0, 1)
    run.ctx.debug_inject(1, limit_ns=50_000_000)
    run.step(rows, 3000)
    with pytest.raises(K.KvError) as e:
        run.ctx.status()
    assert e.value.code == K.KV_E_TIMEOUT
    assert run.ctx.status() == K.KV_OK          # the record was cleared
    out = run.step(rows, 3000)                   # same call again, no injection
    assert run.ctx.status() == K.KV_OK
    kc, vc = _oracle_layer(sp, 4096, 3000)
    orc = O.Oracle(sp)
    q, k, v = _split(sp, rows)
    qr = orc.append(kc, vc, 3000, q, k, v)
    assert_close(out, orc.attend(kc, vc, 3000, qr))
