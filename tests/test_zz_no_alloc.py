"""kv_attend_decode_noalloc: decode attention that allocates no device memory.

It serves callers that cannot call cudaMalloc -- a host framework that owns and
plans all device memory up front and runs this op as a callback mid-compute.
They keep their own cache and buffers, and the library's scratch comes from a
fixed array built into it.  These tests call it through the C ABI with
caller-owned buffers and check it against the CPU oracle and against kv_attend
(the context path), with the tolerance the other parity tests use, on two
calls in a row: at head_dim 64 (a GQA group of 7), 96 (MHA, 32 heads), 128
(8 KV heads) and 128 with a group of 12 query heads (two row groups a call),
and at a context near the built-in scratch's limit.  A shape too large for the
scratch is refused with an error.

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


CASES = [
    ("qwen2-0.5b", 2048, {}),
    ("phi3-mini", 3968, {}),
    ("llama3.2-3b", 6000, {}),
    ("llama3.2-3b", 5000, {"n_head": 24, "n_head_kv": 2}),
    ("llama3.2-3b", 52000, {}),          # ~15 MiB of the 16 MiB scratch
]


@pytest.mark.parametrize("name,n_past,over", CASES, ids=["%s-%d-%s" % (c[0], c[1], c[2].get("n_head_kv", ""))
                                                          for c in CASES])
def test_noalloc_matches_oracle_and_kv_attend_on_two_calls_in_a_row(name, n_past, over, cuda):
    import torch
    sp = specs.get(name)
    sp["n_layer"] = 1
    sp.update(over)
    n_ctx = n_past + 8
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    w = specs.row_width(sp)
    ctx = K.Context(K.make_config(sp, n_ctx=n_ctx, n_batch_max=4))
    ctx.fill_synthetic(sp["seed"], 0, n_past)
    orc = O.Oracle(sp)
    kc_o = np.zeros((n_ctx, hkv, d), np.uint16)
    vc_o = np.zeros((n_ctx, hkv, d), np.uint16)
    kc_o[:n_past] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE, 0, n_past, hkv, d)
    vc_o[:n_past] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 1, 0, n_past, hkv, d)
    # caller-owned device buffers (allocated by the caller, not by the library)
    kc = torch.zeros((n_ctx, hkv, d), dtype=torch.float16, device=cuda)
    vc = torch.zeros((n_ctx, hkv, d), dtype=torch.float16, device=cuda)
    kc[:n_past] = torch.from_numpy(kc_o[:n_past].view(np.float16)).to(cuda)
    vc[:n_past] = torch.from_numpy(vc_o[:n_past].view(np.float16)).to(cuda)
    for call in range(2):
        n = n_past + call
        rows = synth.qkv_rows(sp, 10 + call, 0, 1)
        tr = torch.from_numpy(rows).to(cuda)
        b = tr.data_ptr()
        out_ref = torch.full((1, hq * d), float("nan"), device=cuda)
        ctx.append(0, n, 1, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w)
        ctx.attend(0, n, 1, out_ref)
        # the caller's own append: the oracle's rotated K and V row at n
        q_roped = orc.append(kc_o, vc_o, n, rows[:, :hq * d], rows[:, hq * d:(hq + hkv) * d],
                             rows[:, (hq + hkv) * d:])
        kc[n] = torch.from_numpy(kc_o[n].view(np.float16)).to(cuda)
        vc[n] = torch.from_numpy(vc_o[n].view(np.float16)).to(cuda)
        q = torch.from_numpy(np.ascontiguousarray(q_roped.reshape(-1))).to(cuda)
        out = torch.full((hq * d,), float("nan"), device=cuda)
        K.attend_decode_noalloc(kc, vc, hq, hkv, d, n + 1, q, out)
        torch.cuda.synchronize()
        want = orc.attend(kc_o, vc_o, n, q_roped)[0]
        got = out.cpu().numpy()
        _close(got, want)
        _close(got, out_ref.cpu().numpy()[0])
    ctx.close()


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda):
    import torch
    # buffers that hold every row asked for, so a refusal is the only outcome
    # that depends on the scratch size
    kc = torch.zeros((200000, 8, 128), dtype=torch.float16, device=cuda)
    q = torch.zeros(32 * 128, device=cuda)
    out = torch.zeros(32 * 128, device=cuda)
    with pytest.raises(K.KvError) as e:
        K.attend_decode_noalloc(kc, kc, 32, 8, 128, 200000, q, out)   # ~50 MB of scores
    assert e.value.code == K.KV_E_RANGE
    assert "scratch" in str(e.value)
    with pytest.raises(K.KvError) as e:
        # just past the exact limit: 144 CTAs x 29 score tiles of 4 KB
        K.attend_decode_noalloc(kc, kc, 32, 8, 128, 64000, q, out)
    assert e.value.code == K.KV_E_RANGE
    assert "scratch" in str(e.value)
