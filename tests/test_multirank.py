"""Multi-rank (KV-head sharded) decomposition on CPU ranks over gloo.

The cache shards by KV head: shard g owns KV heads [g*Hkv/G, (g+1)*Hkv/G) of
every layer and their GQA query heads (kv_shard_geometry, the product's host
code), and the only exchange is the all-gather of each layer's head outputs.
Here two gloo ranks each run the path (CPU oracle) on their own shard, gather
the outputs in the layout kv_attend returns ([n_new][G][Hq/G*d], i.e. heads
outer) and compare with the unsharded path: results must be bit-identical,
because no arithmetic crosses a KV-head boundary.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _paths():
    for p in (os.path.join(ROOT, "ggml-loader_b200"), os.path.join(ROOT, "oracle"),
              os.path.join(ROOT, "tests", "golden")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _shard_spec(sp, nq, nkv):
    s = dict(sp)
    s["n_head"], s["n_head_kv"] = nq, nkv
    return s


def _cache(O, synth, sp, n_past, n_cells, hkv_total, d, h0=0, nh=None):
    """The cache before the step: rows 0..n_past-1, or for a ring of n_cells the
    positions (n_past - n_cells, n_past) in cells p % n_cells."""
    nh = hkv_total if nh is None else nh
    rows = n_cells or (n_past + 16)
    kc = np.zeros((rows, nh, d), np.uint16)
    vc = np.zeros((rows, nh, d), np.uint16)
    p0 = max(0, n_past - n_cells) if n_cells else 0
    if n_past > p0:
        k = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE, p0, n_past - p0, hkv_total, d, h0=h0, nh=nh)
        v = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 1, p0, n_past - p0, hkv_total, d, h0=h0, nh=nh)
        cells = np.arange(p0, n_past) % rows if n_cells else np.arange(p0, n_past)
        kc[cells] = k
        vc[cells] = v
    return kc, vc


def _attend(O, orc, kc, vc, n_past, qr, variant):
    n_new = qr.shape[0]
    if variant == "ring":
        return orc.attend_ring(kc, vc, n_past, qr)
    if variant == "window_flash":
        m = np.full((n_new, n_past + n_new), -np.inf, np.float16)
        for t in range(n_new):
            m[t, max(0, n_past + t - 40): n_past + t + 1] = 0
        return orc.attend_ex(kc, vc, n_past, qr, mask=m, flash=True)
    return orc.attend(kc, vc, n_past, qr)


def _worker(rank, world, port, name, n_past, n_new, q, variant="causal"):
    try:
        _paths()
        import kv_b200 as K
        import kv_oracle as O
        from kv_b200 import specs, synth
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        sp = specs.get(name)
        sp["n_layer"] = 1
        n_cells = 64 if variant == "ring" else 0
        hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        cfg = K.make_config(sp, n_ctx=n_past + n_new + 8, n_shards=world, ring_cells=n_cells)
        q0, nq, kv0, nkv = K.shard_geometry(cfg, rank)
        # this shard's cache rows: generated from the global head index
        kc, vc = _cache(O, synth, sp, n_past, n_cells, hkv, d, h0=kv0, nh=nkv)
        rows = synth.qkv_rows(sp, 0, 0, n_new)
        # read only this shard's heads out of the replicated input rows
        qs = rows[:, q0 * d:(q0 + nq) * d]
        ks = rows[:, (hq + kv0) * d:(hq + kv0 + nkv) * d]
        vs = rows[:, (hq + hkv + kv0) * d:(hq + hkv + kv0 + nkv) * d]
        qn = kn = None
        if sp["qk_norm"]:
            qn, kn = synth.norm_weights(sp, 0)
        orc = O.Oracle(_shard_spec(sp, nq, nkv))
        qr = orc.append_ring(kc, vc, n_past, np.ascontiguousarray(qs), np.ascontiguousarray(ks),
                             np.ascontiguousarray(vs), qn, kn) if n_cells else \
            orc.append(kc, vc, n_past, np.ascontiguousarray(qs), np.ascontiguousarray(ks),
                       np.ascontiguousarray(vs), qn, kn)
        local = torch.from_numpy(_attend(O, orc, kc, vc, n_past, qr, variant))   # [n_new][nq*d]
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        out = torch.cat(parts, dim=1).numpy()                           # [n_new][Hq*d], heads outer
        new_rows = (np.arange(n_past, n_past + n_new) % n_cells) if n_cells else np.arange(n_past, n_past + n_new)
        k_rows = torch.from_numpy(kc[new_rows].astype(np.int32))
        kparts = [torch.empty_like(k_rows) for _ in range(world)]
        dist.all_gather(kparts, k_rows)
        k_all = torch.cat(kparts, dim=1).numpy().astype(np.uint16)     # [n_new][Hkv][d]
        if rank == 0:
            fk, fv = _cache(O, synth, sp, n_past, n_cells, hkv, d)
            full = O.Oracle(sp)
            app = full.append_ring if n_cells else full.append
            fqr = app(fk, fv, n_past, rows[:, :hq * d], rows[:, hq * d:(hq + hkv) * d],
                      rows[:, (hq + hkv) * d:], qn, kn)
            want = _attend(O, full, fk, fv, n_past, fqr, variant)
            ok = np.array_equal(out.view(np.uint32), want.view(np.uint32)) and \
                np.array_equal(k_all, fk[new_rows])
            q.put(("ok" if ok else "mismatch", float(np.abs(out - want).max())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put(("error", repr(e)))


@pytest.mark.parametrize("name,n_past,n_new,variant", [
    ("llama3.1-8b-128k", 200, 1, "causal"), ("qwen3-8b-prefill", 120, 5, "causal"), ("phi3-mini", 60, 2, "causal"),
    ("qwen3-8b-prefill", 120, 5, "window_flash"),   # the caller's mask and the flash branch
    ("llama3.2-3b", 150, 7, "ring"),                 # a ring cache after its wrap
])
def test_two_gloo_ranks_match_unsharded(name, n_past, n_new, variant):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, n_past, n_new, q, variant)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    results = []
    while not q.empty():
        results.append(q.get())
    assert results and all(r[0] == "ok" for r in results), results
