"""kv_attend_decode_noalloc: decode attention that allocates no device memory.

It serves callers that cannot call cudaMalloc -- a host framework that owns and
plans all device memory up front and runs this op as a callback mid-compute.
They keep their own cache and buffers, and the library's scratch comes from a
fixed array built into it.  These tests call it through the C ABI with
caller-owned buffers and check it against kv_attend (the context path) on two
calls in a row, with the tolerance the other parity tests use, and check that
a shape too large for the built-in scratch is refused with an error.

(The file name sorts last so that a run stopping at the first failure has
already run every other test.)
"""
import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
REL_L2 = 1e-3


def _close(got, want):
    d = np.asarray(got, np.float64) - np.asarray(want, np.float64)
    assert np.all(np.isfinite(got))
    ma = float(np.abs(d).max())
    rl = float(np.linalg.norm(d) / np.linalg.norm(want))
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)


def test_noalloc_matches_kv_attend_on_two_calls_in_a_row(cuda):
    import torch
    sp = specs.get("llama3.2-3b")
    sp["n_layer"] = 1
    n_ctx, n_past = 8192, 6000
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    w = specs.row_width(sp)
    ctx = K.Context(K.make_config(sp, n_ctx=n_ctx, n_batch_max=4))
    ctx.fill_synthetic(sp["seed"], 0, n_past)
    orc = O.Oracle(sp)      # only to form the rotated query a caller would hold
    scratch_k = np.zeros((n_ctx, hkv, d), np.uint16)
    scratch_v = np.zeros((n_ctx, hkv, d), np.uint16)
    # caller-owned device buffers (allocated by the caller, not by the library)
    kc = torch.zeros((n_ctx, hkv, d), dtype=torch.float16, device=cuda)
    vc = torch.zeros((n_ctx, hkv, d), dtype=torch.float16, device=cuda)
    for call in range(2):
        n = n_past + call
        rows = synth.qkv_rows(sp, 10 + call, 0, 1)
        tr = torch.from_numpy(rows).to(cuda)
        b = tr.data_ptr()
        out_ref = torch.full((1, hq * d), float("nan"), device=cuda)
        ctx.append(0, n, 1, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w)
        ctx.attend(0, n, 1, out_ref)
        torch.cuda.synchronize()
        kc[: n + 1] = torch.from_numpy(ctx.export_rows(0, 0, 0, n + 1).view(np.float16)).to(cuda)
        vc[: n + 1] = torch.from_numpy(ctx.export_rows(0, 1, 0, n + 1).view(np.float16)).to(cuda)
        q_roped = orc.append(scratch_k, scratch_v, n, rows[:, :hq * d], rows[:, hq * d:(hq + hkv) * d],
                             rows[:, (hq + hkv) * d:])
        q = torch.from_numpy(np.ascontiguousarray(q_roped.reshape(-1))).to(cuda)
        out = torch.full((hq * d,), float("nan"), device=cuda)
        K.attend_decode_noalloc(kc, vc, hq, hkv, d, n + 1, q, out)
        torch.cuda.synchronize()
        _close(out.cpu().numpy(), out_ref.cpu().numpy()[0])
    ctx.close()


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda):
    import torch
    kc = torch.zeros((16, 8, 128), dtype=torch.float16, device=cuda)
    q = torch.zeros(32 * 128, device=cuda)
    out = torch.zeros(32 * 128, device=cuda)
    with pytest.raises(K.KvError) as e:
        K.attend_decode_noalloc(kc, kc, 32, 8, 128, 200000, q, out)   # ~100 MB of scores
    assert e.value.code == K.KV_E_RANGE
    assert "scratch" in str(e.value)
