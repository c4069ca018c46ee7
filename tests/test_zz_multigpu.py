"""KV-head sharded path on two, four and eight GPUs: one process per GPU,
checked against the unsharded oracle.  Decode exchanges the head outputs
inside the attention kernel over NVLink (every shard writes its heads into
every peer's receive buffer); chunks use the library's NCCL all-gather into
the gather buffer and the unshard kernel.

Each case is skipped unless enough GPUs are visible.  Each rank fills only its
shard of the cache (kv_fill_synthetic generates rows from the global head
index) and reads only its heads out of the replicated input rows; every rank
must return the same full [n_new][Hq*d] output.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _paths():
    for p in (os.path.join(ROOT, "ggml-loader_b200"), os.path.join(ROOT, "oracle"),
              os.path.join(ROOT, "tests", "golden")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _rank(rank, world, name, n_past, n_new, idq, outq):
    try:
        _paths()
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        import torch
        import kv_b200 as K
        from kv_b200 import specs, synth
        torch.cuda.set_device(rank)
        if rank == 0:
            cid = K.comm_unique_id()
            for _ in range(world - 1):
                idq.put(cid)
        else:
            cid = idq.get(timeout=120)
        sp = specs.get(name)
        sp["n_layer"] = 1
        n_ctx = n_past + n_new + 64
        cfg = K.make_config(sp, n_ctx=n_ctx, n_batch_max=max(16, n_new), device=rank, n_shards=world, shard=rank,
                            comm_id=cid)
        ctx = K.Context(cfg)
        dev = torch.device("cuda", rank)
        st = torch.cuda.current_stream(dev)
        ctx.fill_synthetic(sp["seed"], 0, n_past, stream=st)
        hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        rows = synth.qkv_rows(sp, 3, 0, n_new)
        t = torch.from_numpy(np.ascontiguousarray(rows, np.float32)).to(dev)
        w = rows.shape[1]
        qn = kn = None
        if sp["qk_norm"]:
            qn, kn = [torch.from_numpy(x).to(dev) for x in synth.norm_weights(sp, 0)]
        out = torch.full((n_new, hq * d), float("nan"), device=dev)
        b = t.data_ptr()
        ctx.append(0, n_past, n_new, b, w, b + 4 * hq * d, w, b + 4 * (hq + hkv) * d, w, qn, kn, stream=st)
        ctx.attend(0, n_past, n_new, out, stream=st)
        torch.cuda.synchronize(dev)
        ctx.status()
        outq.put((rank, "ok", out.cpu().numpy()))
        ctx.close()
    except Exception as e:  # report instead of hanging the parent
        outq.put((rank, "error", repr(e)))


def _run_shards(world, name, n_past, n_new):
    """Run `world` shards of one layer, one process per GPU; check every shard
    returns the same bits and that they match the unsharded oracle."""
    import torch.multiprocessing as mp
    _paths()
    import kv_oracle as O
    from kv_b200 import specs, synth
    from test_gpu_path import _oracle_layer, _split, assert_close
    ctxm = mp.get_context("spawn")
    idq, outq = ctxm.Queue(), ctxm.Queue()
    procs = [ctxm.Process(target=_rank, args=(r, world, name, n_past, n_new, idq, outq)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        try:
            r, status, val = outq.get(timeout=300)
        except Exception:
            break
        res[r] = (status, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(res) == world and all(v[0] == "ok" for v in res.values()), res
    sp = specs.get(name)
    sp["n_layer"] = 1
    n_ctx = n_past + n_new + 64
    kc, vc = _oracle_layer(sp, n_ctx, n_past)
    rows = synth.qkv_rows(sp, 3, 0, n_new)
    q, k, v = _split(sp, rows)
    qn, kn = synth.norm_weights(sp, 0) if sp["qk_norm"] else (None, None)
    orc = O.Oracle(sp)
    qr = orc.append(kc, vc, n_past, q, k, v, qn, kn)
    want = orc.attend(kc, vc, n_past, qr)
    for r in range(1, world):
        assert np.array_equal(res[0][1].view(np.uint32), res[r][1].view(np.uint32)), r
    assert_close(res[0][1], want)


@pytest.mark.gpu
@pytest.mark.parametrize("name,n_past,n_new", [("llama3.1-8b-128k", 3000, 1), ("qwen3-8b-prefill", 2000, 40),
                                               ("llama3.2-3b", 1500, 3),
                                               ("qwen2-0.5b", 2048, 1)])   # one KV head a shard
def test_two_gpu_shards_match_oracle(name, n_past, n_new):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_shards(2, name, n_past, n_new)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("name,n_past,n_new", [("llama3.1-8b-128k", 5000, 1), ("llama3.2-3b", 1500, 3)])
def test_wider_shards_match_oracle(name, n_past, n_new, world):
    """Four and eight shards (two and one KV heads each on these shapes): the
    decode exchange reaches every peer, the chunk goes through NCCL."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    _run_shards(world, name, n_past, n_new)
