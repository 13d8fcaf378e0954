#!/usr/bin/env python3
"""MoE-layer tokens/s of the routed Q4_0 expert FFN on B200 (sm_100a).

Contract (one JSON line from rank 0):
  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Workload (synthetic, seeded):
  config 4 (default, the largest single-GPU config): 16 micro-batches of 1,024
  tokens through a stack of L=48 MoE layers with independent seeded weights
  (43.6 GB, far above the 126 MB L2), uniform top-10 routing from logits
  ~N(0,1), 512 experts + 1 shared, H=2048, I=512, Q4_0 experts; each layer
  adds its FFN output into the residual stream: MoE-layer tokens/s =
  tokens x layers x K / time.  config 1: decode T=1; config 2: ragged decode
  T=8; config 3: T=4096 with Zipf(1.1) routing; config 5: T=32768 mixed
  batch (8 layers).  With --gpus N > 1 (torchrun) the layer is
  expert-parallel: rank r owns experts [r*512/N, (r+1)*512/N).
Timing: W warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, CUDA events on the launching stream,
max over ranks.  Each step is one CUDA-graph replay of the L layer forwards.
`e2e` repeats the K steps through the public API with the inputs in pinned
host memory: every step copies x and the L layers' router logits host->device
and reads the final residual device->host inside the timed region, one
micro-batch at a time on two copy streams, so micro-batch u+1's inputs cross
while micro-batch u computes (a step's copies start once the previous step
has finished with its buffers).
`roofline` covers the dominant kernel (the grouped gate/up weight-streaming
kernel): algorithmic bytes per launch / its mean duration from CUDA events
around each launch in an eager pass of the same K steps.
`cpu_baseline` times the reference's own CPU expert path (oracle/_ref, the
reference's CpuExpertPool on the host's physical cores) on one layer pass.
"""
import argparse
import json
import math
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E, K_TOP = 2048, 512, 512, 10
EXPERT_BYTES = 1769472            # one Q4_0 expert (gate + up + down)
GATE_UP_BYTES = 2 * 589824        # gate + up of one expert
DOWN_BYTES = 589824
METRIC = "MoE-layer tokens/s (Q4_0 experts)"

CONFIGS = {
    1: dict(name="decode_T1", tokens=1, ubatches=1, layers=48, routing="normal", steps=20),
    2: dict(name="decode_T8_ragged", tokens=8, ubatches=1, layers=48, routing="normal", steps=20),
    3: dict(name="prefill_T4096_zipf1.1", tokens=4096, ubatches=1, layers=48, routing="zipf", steps=10),
    4: dict(name="prefill_16384_ubatch1024_48layers", tokens=1024, ubatches=16, layers=48, routing="normal", steps=5),
    5: dict(name="mixed_T32768", tokens=32768, ubatches=1, layers=8, routing="mixed", steps=5),
}


def zipf_logits(rng, T, s=1.1):
    perm = rng.permutation(E)
    base = -s * np.log1p(perm.astype(np.float64))
    g = -np.log(-np.log(rng.random((T, E))))
    return (base[None, :] + g).astype(np.float32)


def make_logits(rng, cfg, T):
    if cfg["routing"] == "zipf":
        return zipf_logits(rng, T)
    return rng.standard_normal((T, E)).astype(np.float32)


def profile_traffic(name):
    """DRAM bytes (read + write) per launch recorded in a committed ncu summary."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clocks and clock-event reasons sampled through NVML every 2 ms while the
    timed region runs (a decode step's timed region is tens of milliseconds, shorter
    than nvidia-smi's start-up), recorded as csv lines in the order of nvidia-smi's
    --query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.*."""

    PERIOD_S = 0.002
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    # NVML clocks-event reason bits, in NAMES order
    BITS = (0x8, 0x40, 0x20, 0x4)

    def __init__(self, device, path=""):
        self.device = device
        self.path = path
        self.thread = None
        self.rows = []

    def _handle(self, nvml):
        import torch
        try:
            p = torch.cuda.get_device_properties(self.device)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return nvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nvml.nvmlDeviceGetHandleByIndex(self.device)

    def start(self):
        import threading
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            h = self._handle(nvml)
            mx = nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM)
        except Exception:
            self.thread = None
            return
        self.stop_evt = threading.Event()
        self.rows = []

        def run():
            while True:
                try:
                    sm = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
                    rs = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    pw = nvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    self.rows.append((sm, mx, pw, rs))
                except Exception:
                    pass
                if self.stop_evt.wait(self.PERIOD_S):
                    break
        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        # the first sample lands before the timed region starts
        while not self.rows and self.thread.is_alive():
            time.sleep(0.0005)

    def stop(self):
        if not self.thread:
            return None
        self.stop_evt.set()
        self.thread.join(timeout=5)
        if self.path:
            try:
                with open(self.path, "w") as fh:
                    for sm, mx, pw, rs in self.rows:
                        flags = ["Active" if rs & b else "Not Active" for b in self.BITS]
                        fh.write(f"{self.device}, {sm}, {mx}, {pw:.2f}, 0x{rs:016x}, " + ", ".join(flags) + "\n")
            except OSError:
                pass
        if not self.rows:
            return None
        reasons = sorted({n for _, _, _, rs in self.rows for n, b in zip(self.NAMES, self.BITS) if rs & b})
        return {"sm_mhz": float(np.median([r[0] for r in self.rows])), "sm_max_mhz": float(self.rows[0][1]),
                "reasons": reasons, "samples": len(self.rows), "source": "NVML, 2 ms period"}


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, value):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def expected_distinct(T, experts=E, k=K_TOP):
    """Expected number of routed experts touched by T tokens with uniform routing."""
    return experts * (1.0 - (1.0 - k / experts) ** T)


# ---------------------------------------------------------------- CPU baseline
def cpu_pools(R, O):
    """The reference's CpuExpertPool over every allowed physical core, split
    into equal pools of at most 15 workers (its per-pool limit), workers pinned."""
    import ctypes
    cpus = np.zeros(4096, np.int32)
    n = ctypes.c_size_t(0)
    pin = R.ref_allowed_physical_cpus(O.ptr(cpus), cpus.size, ctypes.byref(n)) == 0 and n.value > 0
    ncores = n.value if pin else (os.cpu_count() or 1)
    npools = (ncores + 14) // 15
    sizes = [ncores // npools + (1 if i < ncores % npools else 0) for i in range(npools)]
    pools, start = [], 0
    for k in sizes:
        p = R.ref_pool_new(k, 1 if pin else 0, O.ptr(cpus[start:start + k]) if pin else None, k if pin else 0)
        if not p:
            raise RuntimeError("CpuExpertPool creation failed")
        pools.append((p, k))
        start += k
    return pools, ncores


class CpuReference:
    """The reference's CPU expert path on one MoE-layer pass over
    min(T, max_tokens) tokens: the reference's quantize_q8 order (restated),
    router softmax and select_routes (restated), RouteGroups::prepare (the
    reference's), whole CpuExpert jobs of <= 3 columns on the reference's
    CpuExpertPool (AVX2, pinned workers on every allowed physical core), and the
    rank-order fold and shared sigmoid add (restated).  Set up once; each
    `one_pass()` is one timed unit."""

    def __init__(self, cfg, seed, max_tokens=1024):
        import ctypes
        import oracle as O
        R = O.ref()
        if R is None:
            raise RuntimeError("oracle/_ref was not built (the reference tree was absent at build time)")
        self.O, self.R, self.ctypes = O, R, ctypes
        T = self.T = min(cfg["tokens"], max_tokens)
        rng = np.random.default_rng(seed)
        self.x = rng.standard_normal((T, H)).astype(np.float32)
        self.logits = make_logits(rng, cfg, T)
        self.gv = (rng.standard_normal(H) * 0.02).astype(np.float32)
        probs, _ = O.router_softmax(self.logits)
        ids0, _ = O.select_routes(probs)
        self.experts = sorted(set(int(e) for e in ids0.ravel())) + [E]
        self.wts = {e: O.synth_expert(seed, 0, e) for e in self.experts}
        self.handles = {e: R.ref_expert_new(O.ptr(w[0]), O.ptr(w[1]), O.ptr(w[2]), w[0].size, w[2].size, H, I)
                        for e, w in self.wts.items()}
        self.pools, _ = cpu_pools(R, O)
        self.workers = sum(k for _, k in self.pools)
        self.rg = R.ref_routes_new(max(T, 1), 0 if T <= 1024 else 1)
        self.xq = np.zeros((T, H // 32), O.Q8_DTYPE)
        self.row_bytes = (H // 32) * 36
        self.out_all = np.zeros((T * (K_TOP + 1), H), np.float32)   # staging rows: routed pairs, then shared
        self.ticket = ctypes.c_size_t(0)
        self.njobs = 0

    def run_jobs(self, jobs):
        """Submit (expert, token rows, first output row) jobs round-robin over
        the pools; a pool is drained only when its 30 tickets are in use, so
        the other pools keep working meanwhile."""
        R, ctypes = self.R, self.ctypes
        used = [0] * len(self.pools)
        keep = []
        xq_base, out_base = self.xq.ctypes.data, self.out_all.ctypes.data
        for i, (e, toks, row0) in enumerate(jobs):
            pi = i % len(self.pools)
            p, _ = self.pools[pi]
            if used[pi] == 30:
                assert R.ref_pool_drain(p) == 0
                R.ref_pool_reset(p)
                used[pi] = 0
            inp = (ctypes.c_void_p * 3)(*[xq_base + int(t) * self.row_bytes for t in toks] + [None] * (3 - len(toks)))
            keep.append(inp)
            st = R.ref_pool_submit(p, self.handles[e], len(toks), inp, H // 32, 0,
                                   ctypes.c_void_p(out_base + row0 * H * 4), len(toks) * H, ctypes.byref(self.ticket))
            assert st == 0, st
            used[pi] += 1
        for p, _ in self.pools:
            assert R.ref_pool_drain(p) == 0
            R.ref_pool_reset(p)

    def one_pass(self):
        O, R, T = self.O, self.R, self.T
        O.lib().o_quantize_q8_1(O.ptr(self.x), self.x.size, O.ptr(self.xq))
        pr, _ = O.router_softmax(self.logits)
        ids_, w_ = O.select_routes(pr)
        assert R.ref_routes_prepare(self.rg, O.ptr(ids_), O.ptr(w_), ids_.size, T) == 0
        a = np.zeros(ids_.size, O.ASSIGN_DTYPE)
        R.ref_routes_assignments(self.rg, O.ptr(a), a.size)
        # one job per <= 3 consecutive pairs of a group; each job's output rows
        # are contiguous staging rows, scattered to [token][rank] afterwards
        jobs, staged, row = [], [], 0
        e_of = a["expert"]
        bounds = list(np.flatnonzero(np.r_[True, e_of[1:] != e_of[:-1]])) + [len(a)]
        for g0, g1 in zip(bounds[:-1], bounds[1:]):
            for c0 in range(g0, g1, 3):
                chunk = a[c0:min(g1, c0 + 3)]
                jobs.append((int(chunk[0]["expert"]), chunk["token"], row))
                staged.append((row, chunk))
                row += len(chunk)
        shared0 = row
        jobs += [(E, np.arange(c0, min(T, c0 + 3)), shared0 + c0) for c0 in range(0, T, 3)]
        self.run_jobs(jobs)
        contrib = np.empty((T, K_TOP, H), np.float32)
        for r0, chunk in staged:
            contrib[chunk["token"], chunk["rank"]] = self.out_all[r0:r0 + len(chunk)]
        res = np.empty((T, H), np.float32)
        O.lib().o_routed_fold(O.ptr(contrib), O.ptr(np.ascontiguousarray(w_)), T, H, O.ptr(res))
        O.lib().o_shared_add(O.ptr(self.x), O.ptr(self.gv),
                             O.ptr(np.ascontiguousarray(self.out_all[shared0:shared0 + T])), T, H, O.ptr(res))
        self.njobs = len(jobs)
        return res

    def job_ms(self):
        """One 3-column whole-expert job on one worker (the unit of the pass)."""
        R, ctypes = self.R, self.ctypes
        p1, _ = self.pools[0]
        base = self.xq.ctypes.data
        single = (ctypes.c_void_p * 3)(*[base + i * self.row_bytes if i < self.T else None for i in range(3)])
        t1 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t1 < 0.3:
            assert R.ref_pool_submit(p1, self.handles[self.experts[0]], min(3, self.T), single, H // 32, 0,
                                     self.O.ptr(self.out_all), min(3, self.T) * H, ctypes.byref(self.ticket)) == 0
            assert R.ref_pool_drain(p1) == 0
            R.ref_pool_reset(p1)
            reps += 1
        return (time.perf_counter() - t1) / reps * 1e3

    def describe(self, passes, pass_ms):
        job = self.job_ms()
        ideal = self.njobs / self.workers * job
        return (f"{passes} passes of one MoE layer over T={self.T} tokens ({len(self.experts)} experts incl. shared, "
                f"{self.njobs} whole-expert jobs of <= 3 columns) through the reference CpuExpertPool (AVX2, "
                f"{len(self.pools)} pinned pool(s) of {'/'.join(str(k) for _, k in self.pools)} workers); routing "
                f"and fold restated; {pass_ms:.1f} ms per pass vs {ideal:.1f} ms = jobs/workers x one 3-column job "
                f"({job:.2f} ms)")

    def close(self):
        for p, _ in self.pools:
            self.R.ref_pool_free(p)
        for h in self.handles.values():
            self.R.ref_expert_free(h)
        self.R.ref_routes_free(self.rg)


def cpu_baseline(cfg, seed, budget_s=8.0, max_tokens=1024):
    """cpu_baseline record: CpuReference passes for about `budget_s` seconds."""
    import oracle as O
    if O.ref() is None:
        return cpu_baseline_port(cfg, seed, budget_s)
    ref = CpuReference(cfg, seed, max_tokens)
    ref.one_pass()
    t0 = time.perf_counter()
    passes = 0
    while True:
        ref.one_pass()
        passes += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = (time.perf_counter() - t0) / passes
    rec = {"value": ref.T / dt, "unit": "tokens/s", "cores": int(ref.workers), "kind": "reference",
           "sample": ref.describe(passes, dt * 1e3)}
    ref.close()
    return rec


def cpu_baseline_port(cfg, seed, budget_s=8.0):
    import oracle as O
    T = min(cfg["tokens"], 8)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H)).astype(np.float32)
    logits = make_logits(rng, cfg, T)
    gv = (rng.standard_normal(H) * 0.02).astype(np.float32)
    cache = {}

    def fn(e):
        if e not in cache:
            cache[e] = O.synth_expert(seed, 0, e)
        return cache[e]
    O.moe_layer(x, logits, fn, fn(E), gv)
    t0 = time.perf_counter()
    passes = 0
    while time.perf_counter() - t0 < budget_s:
        O.moe_layer(x, logits, fn, fn(E), gv)
        passes += 1
    dt = (time.perf_counter() - t0) / max(passes, 1)
    return {"value": T / dt, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{passes} passes of one layer over T={T} tokens, scalar C restatement, 1 thread"}


# ------------------------------------------------------------------- GPU arm
def run_ours(args, cfg):
    import torch
    world, rank, local = dist_setup(args)
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    dev = torch.device("cuda", local)
    T, U, L = cfg["tokens"], cfg["ubatches"], args.layers or cfg["layers"]
    seed = args.seed + 1000 * rank
    rng = np.random.default_rng(seed)
    desc = pkg.make_desc(device=local, max_tokens=T)
    ep = world > 1    # N GPUs: expert-parallel, rank r owns experts [r*512/N, (r+1)*512/N) of every layer
    weights = []
    for l in range(L):
        w = pkg.EpWeights(desc, rank, world) if ep else pkg.MoeWeights(desc)
        w.synthesize(args.seed, l)      # the global experts' bits, sharded or whole
        w.upload_shared_gate((np.random.default_rng(args.seed + l).standard_normal(H) * 0.02).astype(np.float32))
        weights.append(w)
    if ep:
        layer = pkg.EpLayer(desc, rank, world)
        layer.connect(pkg.exchange_handles)   # CUDA IPC handles all-gathered over the process group
    else:
        layer = pkg.MoeLayer(desc)
    x_host = torch.from_numpy(rng.standard_normal((U, T, H)).astype(np.float32)).pin_memory()
    lg_host = torch.from_numpy(np.stack([make_logits(rng, cfg, T) for _ in range(U * L)]).reshape(U, L, T, E)).pin_memory()
    x_dev = x_host.to(dev)
    lg_dev = lg_host.to(dev)
    h = torch.empty(U, T, H, device=dev)
    out_host = torch.empty(U, T, H).pin_memory()
    stream = torch.cuda.Stream(device=dev)

    # Each layer reads the step's (already normalised) FFN input x and adds its
    # output into the residual h: h = x + sum_l FFN_l(x).  Feeding h back as
    # the next layer's input would need the model's RMS norm between layers.
    def step_device(s):
        h.copy_(x_dev)
        for u in range(U):
            for l in range(L):
                layer.forward(weights[l], x_dev[u], lg_dev[u, l], h[u], accumulate=True, stream=s)

    # warm-up (eager), then capture one step into a CUDA graph
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step_device(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_device(stream)
    torch.cuda.synchronize()
    flags = layer.read_flags()
    if flags:
        raise RuntimeError(f"numeric flags {flags} raised during warm-up")
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()

    clocks = ClockSampler(local, args.clocks_csv.replace("{rank}", str(rank)) if args.clocks_csv else "")
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t_start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end) / args.steps
    ms = max_over_ranks(world, ms)

    # e2e through the public API with pinned host buffers: per micro-batch, the
    # inputs go up on h2d while the previous micro-batch computes, and its
    # residual comes back on d2h as soon as its layers are done
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(U)]
    ev_done = [torch.cuda.Event() for _ in range(U)]
    ev_step = torch.cuda.Event()

    def step_e2e():
        h2d_s.wait_event(ev_step)     # the previous step is done with x_dev, lg_dev and h
        for u in range(U):
            with torch.cuda.stream(h2d_s):
                x_dev[u].copy_(x_host[u], non_blocking=True)
                lg_dev[u].copy_(lg_host[u], non_blocking=True)
                ev_in[u].record(h2d_s)
        for u in range(U):
            stream.wait_event(ev_in[u])
            with torch.cuda.stream(stream):
                h[u].copy_(x_dev[u])
                for l in range(L):
                    layer.forward(weights[l], x_dev[u], lg_dev[u, l], h[u], accumulate=True, stream=stream)
                ev_done[u].record(stream)
            d2h_s.wait_event(ev_done[u])
            with torch.cuda.stream(d2h_s):
                out_host[u].copy_(h[u], non_blocking=True)
        ev_step.record(d2h_s)
        stream.wait_event(ev_step)

    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        ev_step.record(stream)        # no copy starts before the timed region does
        for _ in range(args.steps):
            step_e2e()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(world, e0.elapsed_time(e1) / args.steps)
    h2d = x_host.numel() * 4 + lg_host.numel() * 4
    d2h = out_host.numel() * 4

    if ep:
        result = ep_result(args, cfg, world, rank, ms, e2e_ms, h2d, d2h, clk, lg_host, T, U, L)
        if rank == 0:
            print(json.dumps(result), flush=True)
        graph.reset() if hasattr(graph, "reset") else None
        del graph
        barrier(world)
        layer.close()
        barrier(world)
        import torch.distributed as dist
        dist.destroy_process_group()
        return

    # dominant-kernel durations: eager pass with events around gate/up and down
    nprof = min(args.steps, 4)
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(U * L)] for _ in range(nprof)]
    with torch.cuda.stream(stream):
        for ks in evs:              # torch creates the CUDA event on first record
            for trio in ks:
                for e in trio:
                    e.record(stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for k in range(nprof):
            h.copy_(x_dev)
            for u in range(U):
                for l in range(L):
                    layer.forward_profiled(weights[l], x_dev[u], lg_dev[u, l], h[u], evs[k][u * L + l], stream=stream)
    torch.cuda.synchronize()
    gu = [e[0].elapsed_time(e[1]) for ks in evs for e in ks]
    dn = [e[1].elapsed_time(e[2]) for ks in evs for e in ks]
    gu_ms, dn_ms = float(np.mean(gu)), float(np.mean(dn))

    # algorithmic bytes of one gate/up launch: distinct experts touched (incl. shared)
    touched = []
    for u in range(U):
        for l in range(L):
            ids = np.argsort(-lg_host[u, l].numpy(), axis=1, kind="stable")[:, :K_TOP]
            touched.append(len(np.unique(ids)) + 1)
    n_exp = float(np.mean(touched))
    gu_bytes = n_exp * GATE_UP_BYTES + T * (H + H // 32 * 8) + T * 11 * (I + I // 32 * 8)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    int8 = 2.0 * float(peaks.get("bf16_tflops", 1590.0))   # dense int8 rate = 2x dense bf16 rate on B200
    src = "MEASURED_PEAKS.json (of measured)" if peaks else "profiling-recipe fallback"
    ops = 2.0 * T * (K_TOP + 1) * (2 * I) * H          # int8 ops of the gate/up contraction, routed + shared
    gbs, tops = gu_bytes / (gu_ms * 1e-3) / 1e9, ops / (gu_ms * 1e-3) / 1e12
    # the binding roofline is the one with the longer ideal time for this launch
    hbm_bound = gu_bytes / (hbm * 1e9) >= ops / (int8 * 1e12)
    kernel = "stream_gate_up_kernel" if T <= 32 else "tc_rows_kernel<gate/up>"
    traffic_file = {8: "stream_gate_up_decode_T8.md", 1024: "tc_rows_gate_up_T1024.md",
                    4096: "tc_rows_gate_up_T4096_zipf.md"}.get(T)
    roof = {"bound": "hbm" if hbm_bound else "tensor", "kernel": kernel,
            "achieved": gbs if hbm_bound else tops, "peak": hbm if hbm_bound else int8,
            "unit": "GB/s" if hbm_bound else "TOP/s (int8)",
            "traffic": profile_traffic(traffic_file) if traffic_file else None,
            "bytes_per_launch": gu_bytes, "ops_per_launch": ops,
            "achieved_gbs": gbs, "achieved_int8_tops": tops, "int8_frac": tops / int8, "hbm_frac": gbs / hbm,
            "peak_source": f"{src}: hbm_gbs {hbm:.0f} GB/s; int8 = 2 x bf16_tflops = {int8:.0f} TOP/s"}
    peak = roof["peak"]
    roof["frac"] = roof["achieved"] / peak
    roof["launch_ms"] = gu_ms
    roof["down_launch_ms"] = dn_ms

    tokens_per_step = T * U * L * world
    result = {
        "metric": METRIC, "value": tokens_per_step / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_0xq8_1->int32,fp32",
        "data": "synthetic (seeded Q4_0 weights, x~N(0,1), router logits per BASELINE config)",
        "config": {"workload": cfg["name"], "tokens_per_ubatch": T, "ubatches": U, "layers_per_step": L,
                   "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "shared_experts": 1,
                   "parallelism": f"replica{world}" if world > 1 else "single",
                   "l2": f"weights rotate over {L} distinct layer copies ({L * 907.7:.0f} MB) > 126 MB L2",
                   "graph": "one CUDA graph per step"},
        "e2e": {"value": tokens_per_step / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms},
        "roofline": roof,
        # per layer: fused routing + 2 streaming kernels (T <= 32); else quantise, 4 routing
        # kernels, operand gather, tensor-core gate/up and down
        "gpu_launches": args.steps * U * L * (3 if T <= 32 else 8),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            result["cpu_baseline"] = cpu_baseline(cfg, args.seed)
        except Exception as ex:  # the baseline is reported, never required
            result["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
    if rank == 0:
        print(json.dumps(result), flush=True)
    graph.reset() if hasattr(graph, "reset") else None
    del graph
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def ep_result(args, cfg, world, rank, ms, e2e_ms, h2d, d2h, clk, lg_host, T, U, L):
    """JSON line of an expert-parallel run: whole-step bandwidth of this
    rank's expert shard (weights of the local experts any rank's tokens
    touched, plus the shared expert) as the roofline figure."""
    import torch.distributed as dist
    ecount = E // world
    mine = []
    for u in range(U):
        for l in range(L):
            ids = np.argsort(-lg_host[u, l].numpy(), axis=1, kind="stable")[:, :K_TOP]
            mine.append(np.unique(ids).astype(np.int16).tobytes())
    every = [None] * world
    dist.all_gather_object(every, mine)
    touched = 0
    for k in range(U * L):
        union = set()
        for r in range(world):
            union |= set(np.frombuffer(every[r][k], np.int16).tolist())
        touched += sum(1 for e in union if rank * ecount <= e < (rank + 1) * ecount) + 1
    step_bytes = touched * EXPERT_BYTES
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = max_over_ranks(world, -step_bytes / (ms * 1e-3) / 1e9)   # min over ranks
    achieved = -achieved
    roof = {"bound": "hbm", "kernel": "whole expert-parallel step (route, dispatch, experts, combine)",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
            "bytes_per_step_rank": step_bytes,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else "fallback 6650 GB/s"}
    tokens_per_step = T * U * L * world
    per_layer = (5 if T <= 32 else 17)
    return {
        "metric": METRIC, "value": tokens_per_step / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_0xq8_1->int32,fp32",
        "data": "synthetic (seeded Q4_0 weights, x~N(0,1), router logits per BASELINE config)",
        "config": {"workload": cfg["name"], "tokens_per_ubatch_per_rank": T, "ubatches": U, "layers_per_step": L,
                   "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "shared_experts": 1,
                   "parallelism": f"ep{world}", "experts_per_rank": ecount,
                   "transport": "peer stores/loads on CUDA IPC mappings (dispatch, combine), bounded epoch flags",
                   "l2": f"weights rotate over {L} distinct layer shards > 126 MB L2",
                   "graph": "one CUDA graph per step"},
        "e2e": {"value": tokens_per_step / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_ms},
        "roofline": roof,
        # per layer (T <= 32): routing+dispatch, grouping, 2 expert kernels, done+combine;
        # larger T: quantise, 4 routing, plan, dispatch, wait, 4 grouping, 4 expert kernels, done+combine
        "gpu_launches": args.steps * U * L * per_layer,
        "clocks": clk,
    }


def run_reference(args, cfg):
    """The reference's own CPU expert path (oracle/_ref: the reference's
    RouteGroups and CpuExpertPool on every allowed physical core) on the same
    workload, metric and unit: each step is one MoE-layer pass over the
    config's first min(T, 1024) tokens.  Under torchrun only rank 0 runs."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    if O.ref() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference's CPU code) was not built"}),
              flush=True)
        return
    ref = CpuReference(cfg, args.seed)
    for _ in range(args.warmup):
        ref.one_pass()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref.one_pass()
    total = time.perf_counter() - t0
    ms = total / args.steps * 1e3
    value = ref.T / (ms * 1e-3)
    base = {"value": value, "unit": "tokens/s", "cores": int(ref.workers), "kind": "reference",
            "sample": ref.describe(args.steps, ms)}
    ref.close()
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_0xq8_1->int32,fp32",
        "data": "synthetic (seeded Q4_0 weights, x~N(0,1), router logits per BASELINE config)",
        "config": {"workload": cfg["name"], "tokens_per_ubatch": cfg["tokens"], "layers_per_step": 1,
                   "sampled_tokens": ref.T},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": total,
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="timed steps (default per config)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=4, choices=sorted(CONFIGS))
    ap.add_argument("--layers", type=int, default=0, help="layers per step (default per config)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--clocks-csv", default="", help="also write the sampled SM clocks to this csv file")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.steps <= 0:
        args.steps = cfg["steps"]
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
