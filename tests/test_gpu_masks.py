"""GPU parity of kv_attend_mask: the reference's explicit additive mask
(model.cpp:1579-1586, F32 for ggml_soft_max_ext at :1437, F16 for the flash
branch at :1431) and the flash-attn branch (model.cpp:1426-1434), through the
C ABI, against the CPU oracle's kvo_attend_ex.

Covers the decode kernel (fused single-token append, and the multi-row path of
short chunks), the tensor-core chunk kernel (one pass, the exact two passes of
the default branch past 32k keys, the one-pass flash branch at any length),
sliding-window masks, rows whose keys are all masked, and mask rows that do
not start on 16-byte boundaries.  Bar: max-abs 2e-3 and rel-L2 1e-3 in F32;
an explicit causal mask on the decode kernel gives the implicit mask's bits.
"""
import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth

from test_gpu_path import Run, _oracle_layer, _split, assert_close

pytestmark = pytest.mark.gpu


def _case(name, n_past, n_new, extra=64):
    sp = specs.get(name)
    sp["n_layer"] = 1
    n_ctx = n_past + n_new + extra
    return sp, dict(name=name, spec=name, n_ctx=n_ctx, n_past=n_past, n_new=n_new)


def _window_mask(n_past, n_new, stride, window, dtype):
    """keys in (pos - window, pos] visible for the token at pos = n_past + t"""
    m = np.full((n_new, stride), -np.inf, dtype)
    for t in range(n_new):
        pos = n_past + t
        m[t, max(0, pos - window + 1): pos + 1] = 0
    return m


def _run_masked(name, n_past, n_new, mask_np, flash, cuda, seed=3):
    import torch
    sp, case = _case(name, n_past, n_new)
    run = Run(case, cuda, n_batch_max=max(64, n_new))
    run.sp = sp
    kc, vc = _oracle_layer(sp, case["n_ctx"], n_past)
    rows = synth.qkv_rows(sp, seed, 0, n_new)
    t_rows = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
    base, w = t_rows.data_ptr(), rows.shape[1]
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    run.ctx.append(0, n_past, n_new, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w,
                   run.qn, run.kn, stream=run.stream)
    out = torch.full((n_new, hq * d), float("nan"), device=cuda)
    mask = None if mask_np is None else torch.from_numpy(mask_np).to(cuda)
    run.ctx.profile(True)
    run.ctx.attend_mask(0, n_past, n_new, mask, out, flash=flash, stream=run.stream)
    torch.cuda.synchronize()
    q, k, v = _split(sp, rows)
    qn, kn = synth.norm_weights(sp, 0) if sp["qk_norm"] else (None, None)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    want = orc.attend_ex(kc, vc, n_past, qr, mask=mask_np, flash=flash)
    assert np.array_equal(run.rows(0, n_past, n_new), kc[n_past:n_past + n_new])
    return out.cpu().numpy(), want, run


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_decode_explicit_causal_mask_gives_implicit_bits(dtype, cuda):
    """Fused decode: the causal mask passed explicitly changes no bit."""
    import torch
    name, n_past = "llama3.2-3b", 3000
    sp, case = _case(name, n_past, 1)
    mask = np.zeros((1, n_past + 1 + 7), dtype)
    mask[0, n_past + 1:] = -np.inf
    outs = []
    for use_mask in (False, True):
        run = Run(case, cuda)
        run.sp = sp
        rows = synth.qkv_rows(sp, 5, 0, 1)
        t_rows = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
        base, w = t_rows.data_ptr(), rows.shape[1]
        hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        run.ctx.append(0, n_past, 1, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w,
                       stream=run.stream)
        out = torch.full((1, hq * d), float("nan"), device=cuda)
        if use_mask:
            run.ctx.attend_mask(0, n_past, 1, torch.from_numpy(mask).to(cuda), out, stream=run.stream)
        else:
            run.ctx.attend(0, n_past, 1, out, stream=run.stream)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
        run.ctx.close()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


@pytest.mark.parametrize("name,n_past,n_new", [
    ("llama3.2-3b", 3000, 1),     # fused decode, r = 3
    ("qwen2-0.5b", 2048, 1),      # head_dim 64, r = 7
    ("phi3-mini", 3968, 1),       # head_dim 96, MHA
    ("llama3.2-3b", 1000, 3),     # 9 query rows: the decode kernel's multi-row path
])
@pytest.mark.parametrize("flash", [False, True])
def test_decode_window_mask_matches_oracle(name, n_past, n_new, flash, cuda):
    mask = _window_mask(n_past, n_new, n_past + n_new + 5, 700, np.float16)
    got, want, run = _run_masked(name, n_past, n_new, mask, flash, cuda)
    assert run.ctx.profile_read("attn")[0] >= 1
    assert_close(got, want)


@pytest.mark.parametrize("name,n_past,n_new,stride_pad,dtype", [
    ("qwen3-8b-prefill", 300, 200, 0, np.float16),      # pairs split over CTAs (fold)
    ("qwen3-8b-prefill", 2000, 512, 3, np.float16),     # odd row stride: element loads
    ("llama3.2-3b", 1000, 40, 0, np.float32),           # F32 mask, r = 3
    ("qwen2-0.5b", 150, 64, 0, np.float32),             # head_dim 64
    ("phi3-mini", 1000, 100, 0, np.float16),            # head_dim 96 on the 128 kernel
])
@pytest.mark.parametrize("flash", [False, True])
def test_prefill_window_mask_matches_oracle(name, n_past, n_new, stride_pad, dtype, flash, cuda):
    mask = _window_mask(n_past, n_new, n_past + n_new + stride_pad, 256, dtype)
    got, want, run = _run_masked(name, n_past, n_new, mask, flash, cuda)
    assert run.ctx.profile_read("prefill")[0] + run.ctx.profile_read("prefill2")[0] >= 1   # the tensor-core path ran
    assert_close(got, want)


@pytest.mark.parametrize("flash", [False, True])
def test_long_context_branches_match_oracle(flash, cuda):
    """Past 32k keys the default branch takes the exact two passes and the
    flash branch one online pass; both against their oracle."""
    name, n_past, n_new = "qwen3-8b-prefill", 40000, 40
    mask = _window_mask(n_past, n_new, n_past + n_new, 1 << 30, np.float16)   # causal, explicit
    got, want, run = _run_masked(name, n_past, n_new, mask, flash, cuda)
    # (the one pass runs on CTA pairs at head_dim 128)
    assert run.ctx.profile_read("prefill")[0] + run.ctx.profile_read("prefill2")[0] == (1 if flash else 2)
    assert_close(got, want)


def test_flash_without_mask_matches_oracle(cuda):
    """KV_ATTN_FLASH with the implicit causal mask (mask NULL)."""
    got, want, _ = _run_masked("llama3.1-8b-128k", 5000, 2, None, True, cuda)
    assert_close(got, want)
    got, want, _ = _run_masked("qwen3-8b-prefill", 16384, 512, None, True, cuda)
    assert_close(got, want)


@pytest.mark.parametrize("name,n_past,n_new", [("llama3.2-3b", 500, 1), ("llama3.2-3b", 500, 3),
                                               ("qwen3-8b-prefill", 300, 100)])
def test_fully_masked_rows(name, n_past, n_new, cuda):
    """A token whose keys are all masked: 0 in the flash branch, NaN in the
    default one (ggml's soft_max of an all -inf row); the other tokens match."""
    mask = _window_mask(n_past, n_new, n_past + n_new, 1 << 30, np.float32)
    mask[0, :] = -np.inf
    for flash in (True, False):
        got, want, _ = _run_masked(name, n_past, n_new, mask, flash, cuda)
        if flash:
            assert np.all(got[0] == 0.0)
        else:
            assert np.all(np.isnan(got[0]))
        if n_new > 1:
            assert_close(got[1:], want[1:])


def test_mask_arguments_are_checked(cuda):
    import torch
    sp, case = _case("llama3.2-3b", 100, 1)
    run = Run(case, cuda)
    out = torch.zeros((1, sp["n_head"] * sp["head_dim"]), device=cuda)
    m = torch.zeros((1, 101), device=cuda)
    lib = K.lib()
    assert lib.kv_attend_mask(run.ctx.h, 0, 100, 1, m.data_ptr(), 7, 101, 0, out.data_ptr(), None) == K.KV_E_ARG
    assert lib.kv_attend_mask(run.ctx.h, 0, 100, 1, m.data_ptr(), 0, 101, 4, out.data_ptr(), None) == K.KV_E_ARG
    # a stride shorter than the keys attended (checked once the call follows its append)
    rows = torch.zeros((1, (sp["n_head"] + 2 * sp["n_head_kv"]) * sp["head_dim"]), device=cuda)
    base, w, hd = rows.data_ptr(), rows.shape[1], sp["head_dim"]
    run.ctx.append(0, 100, 1, base, w, base + 4 * sp["n_head"] * hd, w,
                   base + 4 * (sp["n_head"] + sp["n_head_kv"]) * hd, w)
    assert lib.kv_attend_mask(run.ctx.h, 0, 100, 1, m.data_ptr(), 0, 50, 0, out.data_ptr(), None) == K.KV_E_ARG


def test_session_flash_flag_routes_kv_attend(cuda):
    """kv_config.flash_attn (decode_session::use_flash_attn, model.h:381-384):
    kv_attend then takes the flash branch, fused decode and chunk alike."""
    import torch
    for name, n_past, n_new in (("llama3.2-3b", 3000, 1), ("qwen3-8b-prefill", 1000, 100)):
        sp, case = _case(name, n_past, n_new)
        cfg = K.make_config(sp, n_ctx=case["n_ctx"], n_batch_max=max(16, n_new), flash_attn=True)
        ctx = K.Context(cfg)
        st = torch.cuda.current_stream()
        ctx.fill_synthetic(sp["seed"], 0, n_past, stream=st)
        kc, vc = _oracle_layer(sp, case["n_ctx"], n_past)
        rows = synth.qkv_rows(sp, 3, 0, n_new)
        t_rows = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
        base, w = t_rows.data_ptr(), rows.shape[1]
        hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        qn, kn = synth.norm_weights(sp, 0) if sp["qk_norm"] else (None, None)
        tq = None if qn is None else torch.from_numpy(qn).to(cuda)
        tk = None if kn is None else torch.from_numpy(kn).to(cuda)
        ctx.append(0, n_past, n_new, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w, tq, tk, stream=st)
        out = torch.full((n_new, hq * d), float("nan"), device=cuda)
        ctx.attend(0, n_past, n_new, out, stream=st)
        torch.cuda.synchronize()
        q, k, v = _split(sp, rows)
        orc = O.Oracle(sp)
        qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
        assert_close(out.cpu().numpy(), orc.attend_ex(kc, vc, n_past, qr, flash=True))
        ctx.close()
