"""Seeded random shapes through the C ABI against the CPU oracle.

Each case draws, from a fixed seed, a base shape (head_dim 64, 96 or 128 with
its RoPE table), a KV-head count, a GQA group size (1 to 16 query heads a KV
head: one or two row groups of the decode kernel, 8 to 128 tokens a chunk
tile), the RoPE mode, QK-Norm on or off, how many cache rows are filled (none,
tile boundaries, thousands) and the chunk length (a single token, short
chunks that run the decode kernel in row groups, tensor-core chunks, a chunk
that fills the cache to its last row).  The bar is the path's: appended K/V
rows bit-exact, outputs within max-abs 2e-3 / rel-L2 1e-3 of the oracle.
"""
import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth
from test_gpu_path import _oracle_layer, _split, assert_close

pytestmark = pytest.mark.gpu

BASES = ["qwen2-0.5b", "phi3-mini", "llama3.2-3b", "qwen3-8b-prefill"]
GROUPS = [1, 2, 3, 4, 5, 7, 8, 12, 16]
FILLS = [0, 1, 127, 128, 129, 1000, 2047, 4500]
CHUNKS = [1, 1, 1, 2, 5, 16, 31, 33, 64, 100, 257]


def case(i):
    """Case i's shape, drawn from a generator seeded by i (stable across runs)."""
    g = np.random.default_rng(0x6B76F000 + i)
    sp = specs.get(BASES[int(g.integers(len(BASES)))])
    sp["n_layer"] = 1
    hkv = int(g.choice([1, 2, 3, 4, 8]))
    r = int(g.choice(GROUPS))
    sp["n_head_kv"], sp["n_head"] = hkv, hkv * r
    sp["rope_mode"] = int(g.choice([specs.ROPE_NORMAL, specs.ROPE_NEOX]))
    sp["qk_norm"] = bool(g.integers(2))
    n_past = int(g.choice(FILLS))
    n_new = int(g.choice(CHUNKS))
    if n_new >= 100:
        n_past = min(n_past, 2047)   # keeps the oracle's chunk in seconds
    full = bool(g.integers(4) == 0)   # the chunk's last row is the cache's last row
    n_ctx = n_past + n_new + (0 if full else 24)
    sp["seed"] = 0x6B76F000 + i
    return sp, n_past, n_new, n_ctx


@pytest.mark.parametrize("i", range(240))
def test_random_shape_matches_oracle(i, cuda):
    import torch
    sp, n_past, n_new, n_ctx = case(i)
    hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    ctx = K.Context(K.make_config(sp, n_ctx=n_ctx, n_batch_max=max(16, n_new)))
    st = torch.cuda.current_stream()
    if n_past:
        ctx.fill_synthetic(sp["seed"], 0, n_past, stream=st)
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    rows = synth.qkv_rows(sp, 7, 0, n_new)
    t = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(cuda)
    b, w = t.data_ptr(), rows.shape[1]
    qn = kn = tq = tk = None
    if sp["qk_norm"]:
        qn, kn = synth.norm_weights(sp, 0)
        tq, tk = torch.from_numpy(qn).to(cuda), torch.from_numpy(kn).to(cuda)
    ctx.append(0, n_past, n_new, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w, tq, tk, stream=st)
    out = torch.full((n_new, hq * d), float("nan"), device=cuda)
    ctx.attend(0, n_past, n_new, out, stream=st)
    torch.cuda.synchronize()
    ctx.status()
    q, k, v = _split(sp, rows)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    assert np.array_equal(ctx.export_rows(0, 0, n_past, n_new), kc[n_past:n_past + n_new]), "K rows differ"
    assert np.array_equal(ctx.export_rows(0, 1, n_past, n_new), vc[n_past:n_past + n_new]), "V rows differ"
    assert_close(out.cpu().numpy(), orc.attend(kc, vc, n_past, qr))
    ctx.close()
