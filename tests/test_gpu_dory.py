"""GPU parity of the pieces a dory block (dory.c:603-672) needs: head_dim 256,
the nGPT Q/K handling (RoPE, then rms_norm(x, 1e-6/256) / 16, Q times its
squared learned scale; qk_norm = 2) and the sliding-window ring, through the C
ABI against the oracle (kvo_append_ring with qk_norm 2, kvo_ring_mask,
kvo_attend_ex).  Also head_dim 256 on a linear cache, with the fused
single-token append and with qwen3's QK-Norm.  Bar: cache bytes bit-exact,
outputs within max-abs 2e-3 / rel-L2 1e-3.

Shapes: n_head 16, n_head_kv 4, head_dim 256, NEOX RoPE over the whole head,
base 1e4 (the sliding blocks' base), as dory.h describes its model; the learned
scales are synthetic (uniform 2..6 after squaring), not a checkpoint's.
"""
import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth

from test_gpu_path import _oracle_layer, _split, assert_close
from test_gpu_ring import Ring

pytestmark = pytest.mark.gpu


def _dory_spec(qk_norm=2, base=1e4, rope_mode=2):
    sp = specs.get("llama3.2-3b")
    sp.update(n_layer=1, n_head=16, n_head_kv=4, head_dim=256, n_rot=256, rope_mode=rope_mode,
              rope_base=float(base), rope_freq_factors=None, qk_norm=qk_norm)
    return sp


class DoryRing(Ring):
    """A Ring whose context and oracle use the dory spec; Q's scale in q_norm_w."""

    def __init__(self, n_cells, n_pos, cuda):
        import torch
        self.torch = torch
        self.sp = sp = _dory_spec()
        self.cfg = K.make_config(sp, n_ctx=n_pos, n_batch_max=64, ring_cells=n_cells)
        self.ctx = K.Context(self.cfg)
        self.stream = torch.cuda.current_stream()
        self.cuda = cuda
        self.hq, self.hkv, self.d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        self.kc = np.zeros((n_cells, self.hkv, self.d), np.uint16)
        self.vc = np.zeros((n_cells, self.hkv, self.d), np.uint16)
        self.orc = O.Oracle(sp)
        s = synth.uniform(sp["seed"], 777, self.hq * self.d, 1.4, 2.4)
        self.qn_np = (s * s).astype(np.float32)            # the squared learned scale, [n_head][D]
        self.kn_np = None
        self.qn = torch.from_numpy(self.qn_np).to(cuda)
        self.kn = None
        self.n_cells = n_cells


def test_dory_ring_decode_across_the_wrap(cuda):
    r = DoryRing(96, 2048, cuda)
    for pos in range(220):
        check = pos in (0, 95, 96, 150, 219)
        got, want = r.step(pos, 1, 11 + pos, check=check)
        if check:
            assert_close(got, want)
    assert np.array_equal(r.cells(0), r.kc)
    assert np.array_equal(r.cells(1), r.vc)


@pytest.mark.parametrize("flash", [False, True])
def test_dory_ring_chunk(flash, cuda):
    """A 5-token batch across the wrap (20 query rows: the decode kernel's
    multi-row path at head_dim 256), dory's mask built on the device or passed
    as the F16 mask of the flash branch."""
    r = DoryRing(128, 2048, cuda)
    p = 0
    while p < 300:
        r.step(p, 20, 3000 + p, check=False)
        p += 20
    mask = None
    if flash:
        n_used = min(128, p + 5)
        mask = np.ascontiguousarray(O.ring_mask(128, p, 5)[:, :n_used].astype(np.float16))
    got, want = r.step(p, 5, 9, mask=mask, flash=flash)
    assert_close(got, want)
    assert np.array_equal(r.cells(0), r.kc)


@pytest.mark.parametrize("qk_norm,rope_mode", [(0, 0), (1, 2)])
def test_head_dim_256_linear_decode(qk_norm, rope_mode, cuda):
    """head_dim 256 on a linear cache: the single-token append fused into the
    attention kernel (NORMAL RoPE, no norm; NEOX with QK-Norm) at 3000 keys."""
    import torch
    sp = _dory_spec(qk_norm=qk_norm, base=5e5, rope_mode=rope_mode)
    n_past, n_ctx = 3000, 3200
    cfg = K.make_config(sp, n_ctx=n_ctx, n_batch_max=16)
    ctx = K.Context(cfg)
    st = torch.cuda.current_stream()
    ctx.fill_synthetic(sp["seed"], 0, n_past, stream=st)
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    qn = kn = None
    if qk_norm:
        qn, kn = synth.norm_weights(sp, 0)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    orc = O.Oracle(sp)
    for step in range(3):
        rows = synth.qkv_rows(sp, 40 + step, 0, 1)
        t_rows = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
        base, w = t_rows.data_ptr(), rows.shape[1]
        tq = None if qn is None else torch.from_numpy(qn).to(cuda)
        tk = None if kn is None else torch.from_numpy(kn).to(cuda)
        ctx.append(0, n_past, 1, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w, tq, tk, stream=st)
        out = torch.full((1, hq * d), float("nan"), device=cuda)
        ctx.attend(0, n_past, 1, out, stream=st)
        torch.cuda.synchronize()
        q, k, v = _split(sp, rows)
        qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
        assert np.array_equal(ctx.export_rows(0, 0, n_past, 1), kc[n_past:n_past + 1])
        assert_close(out.cpu().numpy(), orc.attend(kc, vc, n_past, qr))
        n_past += 1


@pytest.mark.parametrize("qk_norm,n_past,n_new", [(0, 3000, 100), (1, 1000, 256), (0, 40000, 40)])
def test_head_dim_256_chunk_on_tensor_cores(qk_norm, n_past, n_new, cuda):
    """head_dim 256 chunks on the tcgen05 kernel's one-tile form (one 128-row
    query tile a CTA, O in TMEM columns 256-511, N = 256 P.V MMAs): the one-pass
    mode, and past 32k keys the exact two passes."""
    import torch
    sp = _dory_spec(qk_norm=qk_norm, base=5e5, rope_mode=2)
    n_ctx = n_past + n_new + 64
    cfg = K.make_config(sp, n_ctx=n_ctx, n_batch_max=max(64, n_new))
    ctx = K.Context(cfg)
    st = torch.cuda.current_stream()
    ctx.fill_synthetic(sp["seed"], 0, n_past, stream=st)
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    qn = kn = None
    if qk_norm:
        qn, kn = synth.norm_weights(sp, 0)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    rows = synth.qkv_rows(sp, 7, 0, n_new)
    t_rows = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
    base, w = t_rows.data_ptr(), rows.shape[1]
    tq = None if qn is None else torch.from_numpy(qn).to(cuda)
    tk = None if kn is None else torch.from_numpy(kn).to(cuda)
    ctx.profile(True)
    ctx.append(0, n_past, n_new, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w, tq, tk, stream=st)
    out = torch.full((n_new, hq * d), float("nan"), device=cuda)
    ctx.attend(0, n_past, n_new, out, stream=st)
    torch.cuda.synchronize()
    assert ctx.profile_read("prefill")[0] == (1 if n_past + n_new <= 32768 else 2)
    q, k, v = _split(sp, rows)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    assert np.array_equal(ctx.export_rows(0, 0, n_past, n_new), kc[n_past:n_past + n_new])
    assert_close(out.cpu().numpy(), orc.attend(kc, vc, n_past, qr))


@pytest.mark.parametrize("flash", [False, True])
def test_dory_ring_chunk_on_tensor_cores(flash, cuda):
    """A 64-token dory batch across the ring's wrap: 256 query rows on the
    tensor-core kernel with dory's mask (built on the device, or the caller's
    F16 mask in the flash branch)."""
    r = DoryRing(256, 4096, cuda)
    p = 0
    while p < 400:
        r.step(p, 50, 5000 + p, check=False)
        p += 50
    mask = None
    if flash:
        n_used = min(256, p + 64)
        mask = np.ascontiguousarray(O.ring_mask(256, p, 64)[:, :n_used].astype(np.float16))
    r.ctx.profile(True)
    got, want = r.step(p, 64, 21, mask=mask, flash=flash)
    assert r.ctx.profile_read("prefill")[0] + r.ctx.profile_read("prefill2")[0] >= 1
    assert_close(got, want)
    assert np.array_equal(r.cells(0), r.kc)
