#!/usr/bin/env python
"""Benchmark of the KV-cache append + attention path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Metric: decode KV-append+attention us/token and HBM GB/s (% of
roofline) at 1/2/4/8 B200.  A step is one decode step of the path across every
layer of the model -- per layer one kv_append (QK-Norm/RoPE/F16 append) and
one kv_attend (attention over the whole cache, plus the per-layer all-gather
of head outputs when the cache is sharded by KV head over N GPUs) -- at
positions n_past, n_past+1, ... (cycling over the configuration's step count).
`value` is the whole-job algorithmic HBM traffic per second (GB/s): per layer
n_kv*Hkv*d*2*2 (read K and V) + Hkv*d*2*2 (append) + Hkv*d*4*2 (read k, v) +
Hq*d*4*2 (read q, write o), summed over layers and steps, divided by the max
over ranks of the device-timed region.  Inputs are synthetic (seeded
generator) with the configuration's shapes.  Where a step's cache reads exceed
twice the L2 (GiBs on the 3B/8B/phi3 caches) the steps run back to back in
one timed span; where they fit (qwen2-0.5B, 25 MB) each step is timed alone,
with a write of four times L2's size between the spans.

Default workload: llama-3.2-3B shape, 32k context (the single-GPU decode
configuration); `--config llama3.1-8b-128k` runs the 128k configuration.
`--impl reference` times the CPU restatement of the reference's path (the
oracle; the reference's own ggml backend is not vendored) on the host cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ggml-loader_b200"))

METRIC = "decode KV-append+attention µs/token and HBM GB/s (% of roofline) at 1/2/4/8 B200"
METRIC_PREFILL = "chunked-prefill KV-append+attention TFLOP/s (% of tensor roofline) on B200"
DEFAULT_CONFIG = "llama3.2-3b"
NOMINAL_HBM_GBS = 8000.0
L2_BYTES = 126 * 2 ** 20      # B200 L2
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# algorithmic bytes
# ---------------------------------------------------------------------------

def layer_bytes(sp, n_kv, n_new=1, shards=1):
    hq, hkv, d = sp["n_head"] // shards, sp["n_head_kv"] // shards, sp["head_dim"]
    return (n_kv * hkv * d * 2 * 2 + n_new * hkv * d * 2 * 2 + n_new * hkv * d * 4 * 2 + n_new * hq * d * 4 * 2)


def step_bytes(sp, n_past, n_new=1):
    return sp["n_layer"] * layer_bytes(sp, n_past + n_new, n_new)


def layer_flops(sp, n_past, n_new, shards=1):
    """Algorithmic attention FLOPs of one layer: 4*d*Hq per visible (query, key)
    pair -- S = QK^T and O = PV, masked keys count 0."""
    keys = n_new * n_past + n_new * (n_new + 1) // 2
    return 4 * sp["head_dim"] * (sp["n_head"] // shards) * keys


def step_flops(sp, n_past, n_new):
    return sp["n_layer"] * layer_flops(sp, n_past, n_new)


def positions(sp, first_step, count):
    cyc = max(1, sp["steps"])
    return [sp["n_past"] + ((first_step + i) % cyc) for i in range(count)]


def measured_peak(key="hbm_gbs"):
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j[key]), "measured"
    except Exception:
        return (FALLBACK_HBM_GBS if key == "hbm_gbs" else FALLBACK_BF16_TFLOPS), "fallback"


def committed_traffic(config, kernel):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return j.get(config, {}).get(kernel)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), line.strip()))

    def mark(self, which):
        if which == "start":
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        parsed = []
        for t, line in self.rows:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                parsed.append((t, float(f[2]), float(f[3]), f[4], f[5:]))
            except ValueError:
                continue
        inside = [p for p in parsed if self.t0 and self.t1 and self.t0 - 0.06 <= p[0] <= self.t1 + 0.06]
        use = inside or parsed[-3:]
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for p in use:
            for n, v in zip(names[1:], p[4][1:]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(p[1] for p in use), "sm_max_mhz": max(p[2] for p in use),
                "reasons": sorted(reasons), "samples": len(use), "in_region": bool(inside)}


# ---------------------------------------------------------------------------
# CPU legs (the oracle: test infrastructure, used here only as the baseline)
# ---------------------------------------------------------------------------

class CpuPath:
    """The CPU restatement of the reference path (the oracle) on a sample of the
    workload: the first few layers of the model with their cache rows
    generated on the host, decode steps at the configuration's positions."""

    def __init__(self, sp, max_steps, n_threads=0, flash=False):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        self.flash = flash
        import numpy as np
        import kv_oracle as O
        from kv_b200 import synth
        self.sp, self.O, self.synth = sp, O, synth
        hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        self.max_steps = max(1, min(max_steps, sp["steps"]))
        n_ctx = sp["n_past"] + self.max_steps + sp["n_new"]
        per_layer_cache = 2 * n_ctx * hkv * d * 2
        if sp["n_new"] == 1:
            # decode: every layer whose cache fits in 8 GB of host memory (all
            # of them up to the 32k configuration), so the per-token time is
            # measured over the whole model where it can be
            self.n_lay = max(1, min(sp["n_layer"], int(8e9 // per_layer_cache)))
        else:
            # a prefill chunk costs the CPU about a second per layer: 4 layers
            self.n_lay = max(1, min(sp["n_layer"], 4, int(2e9 // per_layer_cache)))
        self.caches = [None] * self.n_lay

        def fill(l):
            kc = np.zeros((n_ctx, hkv, d), np.uint16)
            vc = np.zeros((n_ctx, hkv, d), np.uint16)
            kc[:sp["n_past"]] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 2 * l, 0, sp["n_past"], hkv, d)
            vc[:sp["n_past"]] = O.gen_cache_rows(sp["seed"], synth.STREAM_CACHE + 2 * l + 1, 0, sp["n_past"],
                                                 hkv, d)
            self.caches[l] = (kc, vc)

        import concurrent.futures as cf   # the generator releases the GIL
        with cf.ThreadPoolExecutor(max_workers=max(1, min(8, O.online_cores()))) as ex:
            list(ex.map(fill, range(self.n_lay)))
        self.orc = O.Oracle(sp)
        self.threads = n_threads if n_threads > 0 else O.online_cores()
        self.norms = [synth.norm_weights(sp, l) if sp["qk_norm"] else (None, None) for l in range(self.n_lay)]
        self.n_new = sp["n_new"]
        self.inputs = [[synth.qkv_rows(sp, s, l, self.n_new) for l in range(self.n_lay)]
                       for s in range(self.max_steps)]

    def step(self, s):
        """One step over the sample layers; returns (seconds, bytes, layer-steps, FLOPs)."""
        sp = self.sp
        hq, hkv, d = sp["n_head"], sp["n_head_kv"], sp["head_dim"]
        s %= self.max_steps
        n_past = sp["n_past"] + s
        t = 0.0
        for l in range(self.n_lay):
            rows = self.inputs[s][l]
            q, k, v = rows[:, :hq * d], rows[:, hq * d:(hq + hkv) * d], rows[:, (hq + hkv) * d:]
            kc, vc = self.caches[l]
            t0 = time.perf_counter()
            qr = self.orc.append(kc, vc, n_past, q, k, v, self.norms[l][0], self.norms[l][1])
            if self.flash:   # the flash-attn branch's restatement (oracle A6)
                self.orc.attend_ex(kc, vc, n_past, qr, flash=True, n_threads=self.threads)
            else:
                self.orc.attend(kc, vc, n_past, qr, n_threads=self.threads)
            t += time.perf_counter() - t0
        return (t, self.n_lay * layer_bytes(sp, n_past + self.n_new, self.n_new), self.n_lay,
                self.n_lay * layer_flops(sp, n_past, self.n_new))

    def describe(self, steps):
        sp = self.sp
        what = "decode step(s)" if self.n_new == 1 else "%d-token chunk(s)" % self.n_new
        if self.n_lay == sp["n_layer"]:
            return "%d %s x all %d layers at n_past %d, %d threads; measured, not extrapolated" % (
                steps, what, sp["n_layer"], sp["n_past"], self.threads)
        return ("%d %s x first %d of %d layers at n_past %d, %d threads; per-step time extrapolated x%.2f "
                "from %d of %d layers" % (steps, what, self.n_lay, sp["n_layer"], sp["n_past"], self.threads,
                                          sp["n_layer"] / self.n_lay, self.n_lay, sp["n_layer"]))


def cpu_sample(sp, seconds, max_steps, flash=False, n_threads=0, cp=None):
    """(GB/s, us per token, description, threads, TFLOP/s, path) of the CPU path
    over about `seconds` on `n_threads` host threads (0: every online core).
    Passing the `cp` of an earlier sample reuses its generated cache rows."""
    if cp is None:
        cp = CpuPath(sp, max_steps, flash=flash)
    cp.threads = n_threads if n_threads > 0 else cp.O.online_cores()
    t_total, nbytes, nls, s, fl = 0.0, 0, 0, 0, 0
    while s < cp.max_steps and (t_total < seconds or s == 0):
        t, b, n, f = cp.step(s)
        t_total += t
        nbytes += b
        nls += n
        fl += f
        s += 1
    return (nbytes / t_total / 1e9, t_total / nls * sp["n_layer"] * 1e6, cp.describe(s), cp.threads,
            fl / t_total / 1e12, cp)


def run_reference(args, sp):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cp = CpuPath(sp, args.warmup + args.steps, flash=args.flash)
    t_total, nbytes, nls, fl = 0.0, 0, 0, 0
    for i in range(args.warmup + args.steps):
        t, b, n, f = cp.step(i)
        if i >= args.warmup:
            t_total += t
            nbytes += b
            nls += n
            fl += f
    gbs = nbytes / t_total / 1e9
    if sp["n_new"] > 1:   # prefill: the tensor-bound metric
        tf = fl / t_total / 1e12
        emit({
            "impl": "reference", "metric": METRIC_PREFILL, "value": round(tf, 5), "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_total / nls * sp["n_layer"] * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 cache, f32 math",
            "data": "synthetic (seeded generator, configuration shapes)",
            "config": {"workload": sp["name"], "n_past": sp["n_past"], "n_new": sp["n_new"],
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": round(tf, 5), "unit": "TFLOP/s", "cores": cp.threads, "kind": "port",
                             "sample": "each step: " + cp.describe(1)},
            "e2e": {"value": round(tf, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "CPU restatement of model.cpp:1382-1445 (ggml not vendored, reference backend unbuildable)"})
        return 0
    us = t_total / nls * sp["n_layer"] * 1e6
    desc = cp.describe(1)
    threads = cp.threads
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1000.0, 4),
        "us_per_token": round(us, 1), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16 cache, f32 math", "data": "synthetic (seeded generator, configuration shapes)",
        "config": {"workload": sp["name"], "n_layer": sp["n_layer"], "n_head": sp["n_head"],
                   "n_head_kv": sp["n_head_kv"], "head_dim": sp["head_dim"], "n_ctx": sp["n_ctx"],
                   "n_past": sp["n_past"], "parallelism": "host threads",
                   "branch": "flash-attn (use_flash_attn)" if args.flash else "default (soft_max_ext + mul_mat)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "each step: " + desc},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU restatement of model.cpp:1382-1445 (ggml not vendored, reference backend unbuildable)",
    }
    emit(line)
    return 0


# ---------------------------------------------------------------------------
# the GPU arm
# ---------------------------------------------------------------------------

def run_ours(args, sp):
    import numpy as np
    import torch
    import kv_b200 as K
    from kv_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log("note: --gpus %d but WORLD_SIZE %d; using WORLD_SIZE" % (args.gpus, world))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    if sp["n_head_kv"] % world:
        raise SystemExit("n_head_kv %d does not shard over %d GPUs" % (sp["n_head_kv"], world))

    comm_id = None
    if world > 1:
        buf = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            buf.copy_(torch.tensor(list(K.comm_unique_id()), dtype=torch.uint8))
        dist.broadcast(buf, 0)
        comm_id = bytes(buf.cpu().tolist())

    n_new = sp["n_new"]
    L, hq, hkv, d = sp["n_layer"], sp["n_head"], sp["n_head_kv"], sp["head_dim"]
    W = (hq + 2 * hkv) * d
    cfg = K.make_config(sp, n_ctx=sp["n_ctx"], n_batch_max=max(16, n_new), device=local, n_shards=world,
                        shard=rank, comm_id=comm_id, flash_attn=args.flash)
    ctx = K.Context(cfg)
    stream = torch.cuda.current_stream()
    t0 = time.time()
    ctx.fill_synthetic(sp["seed"], 0, sp["n_past"], stream=stream)
    cyc = max(1, sp["steps"])
    inputs = torch.empty((cyc, L, n_new, W), dtype=torch.float32, device=dev)
    K.gen_normal_device(inputs, sp["seed"], synth.STREAM_QKV, inputs.numel(), stream=stream)
    qn = kn = None
    if sp["qk_norm"]:
        ws = [synth.norm_weights(sp, l) for l in range(L)]
        qn = torch.from_numpy(np.stack([w[0] for w in ws])).to(dev)
        kn = torch.from_numpy(np.stack([w[1] for w in ws])).to(dev)
    out = torch.empty((L, n_new, hq * d), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    log("rank %d: cache %.2f GiB filled, inputs ready in %.1f s" % (
        rank, K.cache_bytes(cfg, sp["n_ctx"]) / world / 2 ** 30, time.time() - t0))

    def step(s, src=None):
        base = (src if src is not None else inputs[s % cyc]).data_ptr()
        n_past = sp["n_past"] + (s % cyc)
        ctx.forward(n_past, n_new, base, W, base + 4 * hq * d, W, base + 4 * (hq + hkv) * d, W, n_new * W,
                    qn, kn, d, out, n_new * hq * d, stream=stream)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up
    for s in range(args.warmup):
        step(s)
    barrier()

    # timed region (the clock sampler runs on rank 0 for its own GPU)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    smi_index = vis.split(",")[local].strip() if vis else str(local)
    sampler = ClockSampler(smi_index)
    if rank == 0:
        sampler.start()
    # a step whose cache reads fit in L2 (qwen2-0.5B: 25 MB) would find them
    # there on the next step: such steps are timed one by one, with a write of
    # a buffer four times L2's size between them, outside the timed spans
    per_gpu_bytes = statistics.mean(step_bytes(sp, sp["n_past"] + i, n_new) for i in range(cyc)) / world
    flush = per_gpu_bytes < 2 * L2_BYTES
    scrub = torch.empty(4 * L2_BYTES // 4, dtype=torch.float32, device=dev) if flush else None
    lead = args.lead   # untimed steps on every rank while the sampler starts
    for s in range(args.warmup, args.warmup + lead):
        step(s)
    barrier()
    first = args.warmup + lead
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.launch_count()
    barrier()
    sampler.mark("start")
    h0 = time.perf_counter()
    if flush:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            scrub.fill_(float(i))
            ev[i][0].record(stream)
            step(first + i)
            ev[i][1].record(stream)
        host_ms = (time.perf_counter() - h0) * 1e3
        ev[-1][1].synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev)
    else:
        e0.record(stream)
        for i in range(args.steps):
            step(first + i)
        host_ms = (time.perf_counter() - h0) * 1e3   # host submission time of the timed steps
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
    sampler.mark("end")
    launches = ctx.launch_count() - launches0
    barrier()
    if rank == 0:
        sampler.stop()
    ms = max_over_ranks(ms)
    pos = positions(sp, first, args.steps)
    total_bytes = sum(step_bytes(sp, p, n_new) for p in pos)
    value = total_bytes / (ms / 1e3) / 1e9
    ms_step = ms / args.steps
    prefill = n_new > 1
    if prefill:   # tensor-bound: algorithmic attention TFLOP/s of the whole job
        value = sum(step_flops(sp, p, n_new) for p in pos) / (ms / 1e3) / 1e12

    # per-kernel durations (separate pass, CUDA events around each launch)
    prof_steps = min(args.steps, 32)
    ctx.profile(True)
    ctx.profile_reset()
    pfirst = first + args.steps
    for i in range(prof_steps):
        step(pfirst + i)
    torch.cuda.synchronize()
    kern = {}
    for name in ("append", "attn", "prefill", "prefill2", "pfold", "gather"):
        n, tms = ctx.profile_read(name)
        kern[name] = (n, tms)
    ctx.profile(False)
    ppos = positions(sp, pfirst, prof_steps)
    mean_nkv = statistics.mean(p + n_new for p in ppos)
    hkv_l, hq_l = hkv // world, hq // world
    # per launch: a decode launch performs the append itself (no append kernel
    # runs), so it carries the layer's whole byte count
    append_bytes = n_new * (hkv_l * d * (4 * 2 + 2 * 2) + hq_l * d * 4)
    layer_total = layer_bytes(sp, mean_nkv, n_new, world)
    algo = {
        "append": append_bytes,
        "attn": layer_total - (append_bytes if kern["append"][0] else 0),
    }
    # the dominant kernel's launch duration inside the timed region: the
    # region's time x the kernel's share of device time (from the per-launch
    # pass) / its launches in the region; per-launch events alone would add
    # their own gaps and break the programmatic-launch overlap
    prof_launches = sum(v[0] for v in kern.values())
    prof_ms = sum(v[1] for v in kern.values())

    def in_region_us(name):
        n, t = kern[name]
        if not n or not prof_ms:
            return None
        n_region = launches * n / prof_launches
        return ms * (t / prof_ms) / n_region * 1e3

    dom = "attn"
    peak, peak_kind = measured_peak()
    dom_us = in_region_us(dom)
    achieved = algo[dom] / (dom_us / 1e6) / 1e9 if dom_us else None
    if prefill:
        # the tensor-core kernel carries the layer's algorithmic FLOPs (one
        # launch per layer; the fold is timed apart)
        # (the chunk kernel on CTA pairs at head_dim 128, else the one-CTA kernel)
        dom = "prefill2" if kern["prefill2"][0] else "prefill"
        peak, peak_kind = measured_peak("bf16_tflops")
        lf = statistics.mean(layer_flops(sp, p, n_new, world) for p in ppos)
        dom_us = in_region_us(dom)
        achieved = lf / (dom_us / 1e6) / 1e12 if dom_us else None
        algo[dom] = lf
    # the per-launch pass: events around every launch (serialised, no overlap)
    kernel_table = {k: {"launches": v[0], "total_ms": round(v[1], 4),
                        "avg_us_isolated": round(v[1] / v[0] * 1e3, 3) if v[0] else None,
                        "share": round(v[1] / prof_ms, 4) if prof_ms else None} for k, v in kern.items()}

    # end to end through the C ABI with host buffers: H2D inputs, D2H outputs, every step
    h2d = L * n_new * W * 4
    d2h = L * n_new * hq * d * 4
    e2e = None
    if not args.no_e2e:
        host_in = torch.empty((cyc, L, n_new, W), dtype=torch.float32, pin_memory=True)
        host_in.copy_(inputs.cpu())
        host_out = torch.empty((L, n_new, hq * d), dtype=torch.float32, pin_memory=True)
        staging = torch.empty((L, n_new, W), dtype=torch.float32, device=dev)
        e2e_steps = args.steps
        efirst = pfirst + prof_steps
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_ms = 0.0
        f0.record(stream)
        for i in range(e2e_steps):
            s = efirst + i
            if flush:   # (the flush between the steps' timed spans, as above)
                scrub.fill_(float(i))
                f0.record(stream)
            staging.copy_(host_in[s % cyc], non_blocking=True)
            step(s, src=staging)
            host_out.copy_(out, non_blocking=True)
            if flush:
                f1.record(stream)
            stream.synchronize()
            if flush:
                e2e_ms += f0.elapsed_time(f1)
        if not flush:
            f1.record(stream)
            f1.synchronize()
            e2e_ms = f0.elapsed_time(f1)
        e2e_ms = max_over_ranks(e2e_ms)
        epos = positions(sp, efirst, e2e_steps)
        e2e_value = sum(step_bytes(sp, p, n_new) for p in epos) / (e2e_ms / 1e3) / 1e9
        if prefill:
            e2e_value = sum(step_flops(sp, p, n_new) for p in epos) / (e2e_ms / 1e3) / 1e12
        e2e = {"value": round(e2e_value, 2), "unit": "TFLOP/s" if prefill else "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "us_per_token": round(e2e_ms / e2e_steps * 1e3, 2),
               "note": "pinned host inputs copied in and outputs copied out every step, host sync per step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, us, desc, threads, tfs, cp = cpu_sample(sp, args.cpu_seconds, 64, flash=args.flash)
        cpu = {"value": round(tfs, 5) if prefill else round(gbs, 4), "unit": "TFLOP/s" if prefill else "GB/s",
               "cores": threads, "kind": "port", "sample": desc, "us_per_token": round(us, 1)}
        if threads != 8:
            # the reference's own thread count: init_backend(..., 8) (cmd_bench.cpp:107)
            g8, u8, d8, _, t8, _ = cpu_sample(sp, args.cpu_seconds, 64, n_threads=8, cp=cp)
            cpu["threads_8"] = {"value": round(t8, 5) if prefill else round(g8, 4), "cores": 8,
                                "sample": d8, "us_per_token": round(u8, 1)}

    clocks = sampler.summary() if rank == 0 else None
    barrier()
    if rank == 0:
        us_tok = ms_step * 1e3
        ideal_us = statistics.mean(step_bytes(sp, p, n_new) for p in pos) / (peak * world * 1e9) * 1e6
        if prefill:
            ideal_us = statistics.mean(step_flops(sp, p, n_new) for p in pos) / (peak * world * 1e12) * 1e6
        line = {
            "metric": METRIC_PREFILL if prefill else METRIC, "value": round(value, 2),
            "unit": "TFLOP/s" if prefill else "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "us_per_token": round(us_tok, 2),
            "pct_of_roofline": round(100.0 * value / (peak * world), 2),
            ("pct_of_nominal_2250tflops" if prefill else "pct_of_nominal_8tbs"):
                round(100.0 * value / ((2250.0 if prefill else NOMINAL_HBM_GBS) * world), 2),
            "ideal_us_per_token": round(ideal_us, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 cache, f32 math",
            "data": "synthetic (seeded splitmix64/Irwin-Hall generator, configuration shapes; no weights)",
            "config": {"workload": sp["name"], "n_layer": L, "n_head": hq, "n_head_kv": hkv, "head_dim": d,
                       "n_ctx": sp["n_ctx"], "n_past": sp["n_past"], "n_new": n_new,
                       "positions": "n_past + (step mod %d)" % cyc, "global_batch": 1,
                       "branch": "flash-attn (use_flash_attn)" if args.flash else "default (soft_max_ext + mul_mat)",
                       "parallelism": ("kv-head shards x%d + per-layer all-gather" % world) if world > 1
                       else "single GPU",
                       "l2": ("flushed: each step reads %.1f MB of cache a GPU (< 2 x 126 MB L2), so the "
                              "steps are timed one by one with a %d MB write between them" % (
                                  per_gpu_bytes / 1e6, 4 * L2_BYTES // 10 ** 6)) if flush else
                             ("no flush: each step reads %.2f GB of cache a GPU (> 2 x 126 MB L2)" % (
                                 per_gpu_bytes / 1e9))},
            "roofline": {"bound": "tensor" if prefill else "hbm", "kernel": "kv_" + dom,
                         "achieved": round(achieved, 1) if achieved else None,
                         "peak": peak, "unit": "TFLOP/s" if prefill else "GB/s",
                         "frac": round(achieved / peak, 4) if achieved else None,
                         "peak_source": peak_kind + (" dense bf16/f16 burst" if prefill else " copy bandwidth"),
                         # the chunk runs under the power cap for the whole timed region:
                         # its fraction of the sustained GEMM figure beside the burst one
                         **({"frac_of_sustained": round(achieved / measured_peak("bf16_tflops_sustained")[0], 4)
                             if achieved else None} if prefill else {}),
                         ("algorithmic_flops_per_layer" if prefill else "algorithmic_bytes_per_launch"): int(algo[dom]),
                         "launch_us": round(dom_us, 3) if dom_us else None,
                         "launch_us_source": "timed region x device-time share / launches in the region",
                         "traffic": committed_traffic(sp["name"], "kv_" + dom),
                         "kernels": kernel_table},
            "e2e": e2e,
            "gpu_launches": int(launches),
            "host_submit_ms_per_step": round(host_ms / args.steps, 4),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        emit(line)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


_JSON_OUT = None


def emit(line):
    """The one JSON line, on the process's original standard output."""
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    # Everything else printed at any level (NCCL's version banner, library
    # messages) goes to standard error, so standard output carries only the
    # JSON line.
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[1])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) pass")
    ap.add_argument("--flash", action="store_true",
                    help="the reference's flash-attn branch (use_flash_attn) instead of its default one")
    ap.add_argument("--lead", type=int, default=100,
                    help="untimed steps between warm-up and the timed region (clock sampler start-up)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (small profiling cases only; the bench line is invalid)")
    ap.add_argument("--shard-of", type=int, default=None,
                    help="run one GPU's share of a G-way KV-head shard (n_head/G, n_head_kv/G) on one GPU, "
                         "without the exchange (profiling cases only; the bench line is invalid)")
    args = ap.parse_args()
    from kv_b200 import specs
    sp = specs.get(args.config)
    if args.layers:
        sp["n_layer"] = args.layers
        sp["name"] += "-%dlayers" % args.layers
    if args.shard_of:
        g = args.shard_of
        if g < 1 or sp["n_head_kv"] % g:
            raise SystemExit("--shard-of %d does not divide %d KV heads" % (g, sp["n_head_kv"]))
        sp["n_head"] //= g
        sp["n_head_kv"] //= g
        sp["name"] += "-shard1of%d" % g
    if args.steps is None:
        # the configuration's positions, and at least 16 steps (qwen2-0.5B's
        # single position is timed 16 times, each step rewriting the same row)
        args.steps = max(sp["steps"], 16)
    if args.warmup < 3:
        log("note: raising --warmup to 3")
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args, sp)
    return run_ours(args, sp)


if __name__ == "__main__":
    sys.exit(main())
