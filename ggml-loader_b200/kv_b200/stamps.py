"""Per-CTA phase stamps of the decode kernel (the measurement build).

Runs decode steps of a configuration -- or of one shard of it, on one GPU
(--hq/--hkv), or of a sharded run under torch.distributed.run -- through the
phase-stamp build of the library (ggml-loader_b200/lib/stamps/, made by
`python ggml-loader_b200/build.py --stamps`), and prints one JSON line per
rank: the time per layer (CUDA events over the steps) and, per phase, the
median / latest / earliest time over the stamped launches' CTAs, in µs from
each launch's first CTA entry (medians over the launches).

    python ggml-loader_b200/kv_b200/stamps.py llama3.2-3b [--hq 3 --hkv 1] [--steps 8] [--layers 8]

The phases: entry, tma0 (first tile issued), tmaNS (first tile past the
ring's depth issued), wait (griddepcontrol.wait returned), q (query rows
rotated), Kdone, pub (statistics published), stats (the head's statistics
known), Vdone, ticket (partial output added, ticket taken), coll0 / coll1
(the collector of a sharded run starts / ends polling the peers' words), exit.
"""
import argparse
import json
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
if PKG not in sys.path:
    sys.path.insert(0, PKG)

PHASES = {0: "entry", 10: "tma0", 11: "tmaNS", 1: "wait", 2: "q", 3: "Kdone", 4: "pub", 5: "stats", 6: "Vdone",
          7: "ticket", 8: "coll0", 9: "coll1", 12: "exit"}
ORDER = ["entry", "tma0", "tmaNS", "wait", "q", "Kdone", "pub", "stats", "Vdone", "ticket", "coll0", "coll1", "exit"]


def summarise(stamps, launches):
    """Per phase: (median, latest, earliest) over one launch's CTAs, in µs from
    its first entry; then the median of each over the launches."""
    rows = []
    for li in launches:
        x = stamps[li].astype("int64")
        x = x[x[:, 0] > 0]
        if not len(x):
            continue
        t0 = x[:, 0].min()
        r = {}
        for k, name in PHASES.items():
            v = x[:, k]
            v = v[v > 0] - t0
            if len(v):
                r[name] = (float(statistics.median(v)) / 1e3, float(v.max()) / 1e3, float(v.min()) / 1e3)
        r["ncta"] = int(len(x))
        rows.append(r)
    out = {}
    for name in ORDER:
        got = [r[name] for r in rows if name in r]
        if got:
            out[name] = [round(statistics.median(g[j] for g in got), 2) for j in range(3)]
    return out, (rows[-1]["ncta"] if rows else 0)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("config")
    ap.add_argument("--hq", type=int, help="query heads (one shard's, on one GPU)")
    ap.add_argument("--hkv", type=int, help="KV heads (one shard's, on one GPU)")
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--layers", type=int)
    ap.add_argument("--n-past", type=int)
    ap.add_argument("--tag", default="")
    a = ap.parse_args()

    import numpy as np
    import torch
    import kv_b200 as K
    from kv_b200 import specs, synth
    if not os.environ.get("KV_B200_LIBRARY"):
        K.LIB_PATH = os.path.join(PKG, "lib", "stamps", "libkv_b200.so")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    cid = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        buf = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            buf.copy_(torch.tensor(list(K.comm_unique_id()), dtype=torch.uint8))
        dist.broadcast(buf, 0)
        cid = bytes(buf.cpu().tolist())

    sp = specs.get(a.config)
    for key, val in (("n_head", a.hq), ("n_head_kv", a.hkv), ("n_layer", a.layers), ("n_past", a.n_past)):
        if val:
            sp[key] = val
    L, hq, hkv, d = sp["n_layer"], sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    W = (hq + 2 * hkv) * d
    cfg = K.make_config(sp, n_ctx=sp["n_past"] + a.steps + 64, n_batch_max=16, device=local, n_shards=world,
                        shard=rank, comm_id=cid)
    ctx = K.Context(cfg)
    st = torch.cuda.current_stream()
    ctx.fill_synthetic(sp["seed"], 0, sp["n_past"], stream=st)
    inp = torch.empty((L, 1, W), dtype=torch.float32, device=dev)
    K.gen_normal_device(inp, sp["seed"], synth.STREAM_QKV, inp.numel(), stream=st)
    out = torch.empty((L, 1, hq * d), dtype=torch.float32, device=dev)
    qn = kn = None
    if sp["qk_norm"]:
        ws = [synth.norm_weights(sp, l) for l in range(L)]
        qn = torch.from_numpy(np.stack([w[0] for w in ws])).to(dev)
        kn = torch.from_numpy(np.stack([w[1] for w in ws])).to(dev)
    b = inp.data_ptr()

    def step(s):
        ctx.forward(sp["n_past"] + s, 1, b, W, b + 4 * hq * d, W, b + 4 * (hq + hkv) * d, W, W, qn, kn, d, out,
                    hq * d, stream=st)

    for s in range(4):
        step(s)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for s in range(a.steps):
        step(4 + s)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    stamps, n = ctx.debug_stamps()
    ring = stamps.shape[0]
    last = min(L * a.steps, ring)
    launches = [(n - 1 - i) % ring for i in range(last)][::-1]
    phases, ncta = summarise(stamps, launches)
    print(json.dumps({"tag": a.tag, "rank": rank, "world": world, "config": a.config, "hq": hq, "hkv": hkv,
                      "ncta": ncta, "ms_per_step": round(ms / a.steps, 5),
                      "us_per_layer": round(ms / a.steps / L * 1e3, 3), "phases": phases}))
    sys.stdout.flush()
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
