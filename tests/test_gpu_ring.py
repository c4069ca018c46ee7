"""GPU parity of the ring cache (kv_config.ring_cells; dory.c:391-575): the
token at position p in cell p % ring_cells, RoPE at p, attention over the cells
in use with dory_fill_attn_mask's visibility (built on the device), through the
C ABI against the oracle's kvo_append_ring / kvo_ring_mask.

Covers decode across the wrap (every cell rewritten), chunks that cross the
wrap on the tensor-core kernel and on the decode kernel's multi-row path,
QK-Norm, the caller's own mask and the flash branch over a ring, and a batch
longer than the ring (an error).  Bar: cache bytes bit-exact, outputs within
max-abs 2e-3 / rel-L2 1e-3.
"""
import numpy as np
import pytest

import kv_b200 as K
import kv_oracle as O
from kv_b200 import specs, synth

from test_gpu_path import _split, assert_close

pytestmark = pytest.mark.gpu


class Ring:
    """A one-layer ring context and its oracle twin."""

    def __init__(self, name, n_cells, n_pos, cuda, n_batch_max=64):
        import torch
        self.torch = torch
        self.sp = sp = specs.get(name)
        sp["n_layer"] = 1
        self.cfg = K.make_config(sp, n_ctx=n_pos, n_batch_max=n_batch_max, ring_cells=n_cells)
        self.ctx = K.Context(self.cfg)
        self.stream = torch.cuda.current_stream()
        self.cuda = cuda
        self.hq, self.hkv, self.d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        self.kc = np.zeros((n_cells, self.hkv, self.d), np.uint16)
        self.vc = np.zeros((n_cells, self.hkv, self.d), np.uint16)
        self.orc = O.Oracle(sp)
        self.qn = self.kn = None
        self.qn_np = self.kn_np = None
        if sp["qk_norm"]:
            self.qn_np, self.kn_np = synth.norm_weights(sp, 0)
            self.qn = torch.from_numpy(self.qn_np).to(cuda)
            self.kn = torch.from_numpy(self.kn_np).to(cuda)
        self.n_cells = n_cells

    def step(self, pos0, n_new, seed, mask=None, flash=False, check=True):
        torch = self.torch
        rows = synth.qkv_rows(self.sp, seed, 0, n_new)
        t_rows = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(self.cuda)
        base, w = t_rows.data_ptr(), rows.shape[1]
        hq, hkv, d = self.hq, self.hkv, self.d
        self.ctx.append(0, pos0, n_new, base, w, base + 4 * hq * d, w, base + 4 * (hq + hkv) * d, w,
                        self.qn, self.kn, stream=self.stream)
        out = torch.full((n_new, hq * d), float("nan"), device=self.cuda)
        if mask is None and not flash:
            self.ctx.attend(0, pos0, n_new, out, stream=self.stream)
        else:
            tm = None if mask is None else torch.from_numpy(mask).to(self.cuda)
            self.ctx.attend_mask(0, pos0, n_new, tm, out, flash=flash, stream=self.stream)
        torch.cuda.synchronize()
        q, k, v = _split(self.sp, rows)
        qr = self.orc.append_ring(self.kc, self.vc, pos0, q, k, v, self.qn_np, self.kn_np)
        if not check:
            return None, None
        want = self.orc.attend_ring(self.kc, self.vc, pos0, qr, mask=mask, flash=flash)
        return out.cpu().numpy(), want

    def cells(self, which):
        return self.ctx.export_rows(0, which, 0, self.n_cells)


def test_ring_decode_across_the_wrap(cuda):
    """One token at a time from position 0 past 2.5 turns of a 128-cell ring."""
    r = Ring("llama3.2-3b", 128, 4096, cuda)
    for pos in range(330):
        check = pos in (0, 1, 127, 128, 129, 255, 256, 329)
        got, want = r.step(pos, 1, 7 + pos, check=check)
        if check:
            assert_close(got, want)
    assert np.array_equal(r.cells(0), r.kc)
    assert np.array_equal(r.cells(1), r.vc)


@pytest.mark.parametrize("name,n_cells,pos0,n_new", [
    ("llama3.2-3b", 256, 230, 40),      # 120 query rows: the tensor-core kernel, the chunk wraps
    ("llama3.2-3b", 256, 250, 3),       # 9 rows: the decode kernel's multi-row path, wraps
    ("qwen3-8b-prefill", 1024, 1900, 200),   # QK-Norm, a later turn of the ring
    ("qwen2-0.5b", 512, 700, 64),       # head_dim 64, r = 7
])
def test_ring_chunk_matches_oracle(name, n_cells, pos0, n_new, cuda):
    r = Ring(name, n_cells, pos0 + n_new + 64, cuda, n_batch_max=max(64, n_new))
    # fill the ring with the positions before pos0, in chunks (their outputs unchecked)
    p = max(0, pos0 - n_cells)
    while p < pos0:
        n = min(64, pos0 - p)
        r.step(p, n, 1000 + p, check=False)
        p += n
    got, want = r.step(pos0, n_new, 3)
    assert_close(got, want)
    assert np.array_equal(r.cells(0), r.kc)
    assert np.array_equal(r.cells(1), r.vc)


@pytest.mark.parametrize("flash", [False, True])
def test_ring_with_callers_mask(flash, cuda):
    """kv_attend_mask over a ring's cells: dory's F16 mask passed by the caller,
    in both branches (dory attends with ggml_flash_attn_ext, dory.c:653)."""
    r = Ring("llama3.2-3b", 256, 2048, cuda)
    p = 0
    while p < 300:
        r.step(p, 50, 2000 + p, check=False)
        p += 50
    n_new = 40
    n_used = min(256, p + n_new)
    mask = np.ascontiguousarray(O.ring_mask(256, p, n_new)[:, :n_used].astype(np.float16))
    got, want = r.step(p, n_new, 5, mask=mask, flash=flash)
    assert_close(got, want)


def test_ring_batch_longer_than_ring_is_an_error(cuda):
    import torch
    r = Ring("llama3.2-3b", 32, 1024, cuda)
    rows = torch.zeros((40, (r.hq + 2 * r.hkv) * r.d), device=cuda)
    base, w = rows.data_ptr(), rows.shape[1]
    rc = K.lib().kv_append(r.ctx.h, 0, 0, 40, base, w, base + 4 * r.hq * r.d, w, base + 4 * (r.hq + r.hkv) * r.d, w,
                           None, None, None)
    assert rc == K.KV_E_RANGE
