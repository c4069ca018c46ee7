"""GPU parity of the decode kernel's cluster mode (thread-block clusters that
exchange the per-head statistics and partial outputs through distributed
shared memory) against the CPU oracle, with the plain grid beside it.

KV_B200_CLUSTER, read by kv_alloc, selects the grid: unset = the library's
policy, 0 = no clusters, q = clusters of q CTAs.  Every case checks the
appended cache rows bit for bit and the outputs within max-abs 2e-3 / rel-L2
1e-3, over two decode steps in a row (the second launch reuses the barriers'
layout and the statistics slots with the next epoch).
"""
import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth
from test_gpu_path import _oracle_layer, _split, assert_close

pytestmark = pytest.mark.gpu


def _decode(cuda, monkeypatch, name, n_past, cluster, over=None, steps=2, mask=None, flash=False):
    import torch
    if cluster is None:
        monkeypatch.delenv("KV_B200_CLUSTER", raising=False)
    else:
        monkeypatch.setenv("KV_B200_CLUSTER", str(cluster))
    sp = specs.get(name)
    sp["n_layer"] = 1
    sp.update(over or {})
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    n_ctx = n_past + steps + 8
    ctx = K.Context(K.make_config(sp, n_ctx=n_ctx, n_batch_max=4))
    st = torch.cuda.current_stream()
    ctx.fill_synthetic(sp["seed"], 0, n_past, stream=st)
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    orc = O.Oracle(sp)
    qn = kn = None
    if sp["qk_norm"]:
        qn, kn = synth.norm_weights(sp, 0)
    for s in range(steps):
        n = n_past + s
        rows = synth.qkv_rows(sp, 20 + s, 0, 1)
        t = torch.from_numpy(rows).to(cuda)
        b, w = t.data_ptr(), rows.shape[1]
        tq = tk = None
        if qn is not None:
            tq, tk = torch.from_numpy(qn).to(cuda), torch.from_numpy(kn).to(cuda)
        ctx.append(0, n, 1, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w, tq, tk, stream=st)
        out = torch.full((1, hq * d), float("nan"), device=cuda)
        q, k, v = _split(sp, rows)
        qr = orc.append(kc, vc, n, q, k, v, qn, kn)
        if mask is not None or flash:
            m = None if mask is None else np.ascontiguousarray(mask(n + 1))
            tm = None if m is None else torch.from_numpy(m).to(cuda)
            ctx.attend_mask(0, n, 1, tm, out, flash=flash, stream=st)
            want = orc.attend_ex(kc, vc, n, qr, mask=m, flash=flash)
        else:
            ctx.attend(0, n, 1, out, stream=st)
            want = orc.attend(kc, vc, n, qr)
        torch.cuda.synchronize()
        ctx.status()
        assert np.array_equal(ctx.export_rows(0, 0, n, 1), kc[n:n + 1]), "K row differs"
        assert np.array_equal(ctx.export_rows(0, 1, n, 1), vc[n:n + 1]), "V row differs"
        assert_close(out.cpu().numpy(), want)
    ctx.close()


# (name, n_past, overrides): one cluster a head (qwen2, phi3), several (one-
# and two-head shards of the 3B/8B shapes), 8 heads, and GQA groups beyond
# the kernel's 8 query rows (two row groups a layer)
SHAPES = [
    ("qwen2-0.5b", 2048, {}),
    ("phi3-mini", 3968, {}),
    ("llama3.2-3b", 20000, {"n_head": 3, "n_head_kv": 1}),
    ("llama3.2-3b", 9000, {"n_head": 6, "n_head_kv": 2}),
    ("llama3.2-3b", 6000, {}),
    ("qwen3-8b-prefill", 3000, {}),
    ("llama3.2-3b", 5000, {"n_head": 24, "n_head_kv": 2}),
]


@pytest.mark.parametrize("cluster", [None, 0, 2, 4, 8])
@pytest.mark.parametrize("name,n_past,over", SHAPES, ids=[s[0] + "-%d-%s" % (s[1], s[2].get("n_head_kv", "")) for s in SHAPES])
def test_cluster_decode_matches_oracle(name, n_past, over, cluster, cuda, monkeypatch):
    _decode(cuda, monkeypatch, name, n_past, cluster, over)


@pytest.mark.parametrize("cluster", [None, 0])
@pytest.mark.parametrize("flash", [False, True])
def test_cluster_decode_mask_and_flash(flash, cluster, cuda, monkeypatch):
    """The caller's mask (a sliding window of 700 keys) and the flash-attn
    branch on the qwen2 shape (one cluster a head under the policy)."""
    def window(n_kv):
        m = np.full((1, n_kv), -np.inf, np.float32)
        m[0, max(0, n_kv - 700):] = 0.0
        return m
    _decode(cuda, monkeypatch, "qwen2-0.5b", 2048, cluster, mask=window, flash=flash)
    _decode(cuda, monkeypatch, "llama3.2-3b", 7000, cluster, {"n_head": 3, "n_head_kv": 1}, flash=flash)


def test_cluster_decode_shape_policy(cuda):
    """On this device the policy gives one cluster a head on the qwen2 and phi3
    shapes (the statistics and outputs stay in the clusters' shared memory)."""
    import ctypes
    # the device's cluster capacity, as kv_alloc queries it, is not exported;
    # the shapes below only need clusters of 8 and of 4 for 2 and 32 heads
    mc = (ctypes.c_int32 * 9)(0, 0, 74, 49, 37, 29, 24, 21, 18)
    out = [ctypes.c_int32() for _ in range(3)]
    assert K.lib().kv_decode_shape(148, 2, 2049, mc, *[ctypes.byref(o) for o in out]) == K.KV_OK
    assert tuple(o.value for o in out) == (16, 8, 1)
    assert K.lib().kv_decode_shape(148, 32, 3969, mc, *[ctypes.byref(o) for o in out]) == K.KV_OK
    assert tuple(o.value for o in out) == (128, 4, 1)


@pytest.mark.parametrize("cluster", [None, 8])
def test_cluster_expired_wait_reports_timeout_and_recovers(cluster, cuda, monkeypatch):
    """A withheld tile (test hook) in cluster mode: every bounded wait ends,
    kv_status reports KV_E_TIMEOUT, and the next call on the context is
    correct."""
    import torch
    if cluster is None:
        monkeypatch.delenv("KV_B200_CLUSTER", raising=False)
    else:
        monkeypatch.setenv("KV_B200_CLUSTER", str(cluster))
    sp = specs.get("qwen2-0.5b")
    sp["n_layer"] = 1
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    n_past, n_ctx = 2048, 2100
    ctx = K.Context(K.make_config(sp, n_ctx=n_ctx, n_batch_max=4))
    ctx.fill_synthetic(sp["seed"], 0, n_past)
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    orc = O.Oracle(sp)
    rows = synth.qkv_rows(sp, 5, 0, 1)
    t = torch.from_numpy(rows).to(cuda)
    b, w = t.data_ptr(), rows.shape[1]
    out = torch.zeros((1, hq * d), device=cuda)
    ctx.debug_inject(1, limit_ns=50_000_000)
    ctx.append(0, n_past, 1, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w)
    ctx.attend(0, n_past, 1, out)
    torch.cuda.synchronize()
    with pytest.raises(K.KvError) as e:
        ctx.status()
    assert e.value.code == K.KV_E_TIMEOUT
    ctx.debug_inject(0, limit_ns=1_000_000_000)
    q, k, v = _split(sp, rows)
    qr = orc.append(kc, vc, n_past, q, k, v)
    ctx.append(0, n_past, 1, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w)
    ctx.attend(0, n_past, 1, out)
    torch.cuda.synchronize()
    ctx.status()
    assert_close(out.cpu().numpy(), orc.attend(kc, vc, n_past, qr))
    ctx.close()
