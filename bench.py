#!/usr/bin/env python
"""FlashHead decode-step LM-head benchmark.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flashhead|reference]
                    [--workload llama1b-fp8|llama1b-bf16|llama8b-fp8] [--no-sweep]

One step = one greedy FlashHead decode step (stage-1 centroid scores, top-p
probe selection, fused stage-2 gather + logits + argmax) for a batch of
hidden states already resident in HBM. The default workload is the
Llama-3.2-1B-shaped head (D=2048, V=128256, K=8016 clusters of 16, p=256)
with fp8-e4m3 stage-1 centroids at batch 1, on a seeded synthetic head.

Timing: K steps are captured in one CUDA graph and replayed between CUDA
events after W warm-up steps. Every step reads a different replica of the
head (at least 3x the 126 MB L2 of bytes between two uses of one replica), so
no step is served from L2. Stage durations come from graphs of single-stage
launches timed the same way. Under torchrun (N > 1) every rank serves its
own batches on its own replica set (data-parallel replicas, weak scaling);
the step time is the max over ranks.

The reference arm (--impl reference) times the reference's CPU path (the
torch port in oracle/reference_cpu.py) on this host's cores.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "flash-head_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "LM-head µs/decode step at batch 1/64/256 + achieved HBM GB/s vs dense head"
L2_BYTES = 126 * 2**20
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------
def workloads():
    from flash_head.synthetic import LLAMA31_8B, LLAMA32_1B
    return {
        "llama1b-fp8": dict(shape=LLAMA32_1B, stage1="fp8", rows=1, sweep=[1, 8, 64, 256],
                            name="Llama-3.2-1B head"),
        "llama1b-bf16": dict(shape=LLAMA32_1B, stage1="model", rows=1, sweep=[1, 8, 64, 256],
                             name="Llama-3.2-1B head"),
        "llama8b-fp8": dict(shape=LLAMA31_8B, stage1="fp8", rows=1, sweep=[1, 32, 256],
                            name="Llama-3.1-8B head"),
    }


def workload_label(wl, rows):
    s = wl["shape"]
    st = "fp8-e4m3 stage 1 (per-row scale)" if wl["stage1"] == "fp8" else "bf16 stage 1"
    return (f"FlashHead greedy decode step, {wl['name']} D={s.hidden} V={s.vocab} "
            f"K={s.n_clusters}x{s.cluster_size} p={s.n_probes}, batch {rows}, {st}, bf16 stage 2")


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self, n_gpus):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist.group.WORLD
        else:
            torch.cuda.set_device(0)

    def barrier(self):
        import torch
        torch.cuda.synchronize()
        if self.pg is not None:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    def max(self, x: float) -> float:
        if self.pg is None:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            import torch.distributed as dist
            dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Clock sampling (nvidia-smi, during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu_id],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for_smi(local_rank: int) -> str:
    import torch
    try:
        u = str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[local_rank]
        return str(local_rank)


# ---------------------------------------------------------------------------
# Timing helpers
# ---------------------------------------------------------------------------
def capture(fn_list):
    """CUDA graph running every callable of fn_list once, in order."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for fn in fn_list[:2]:
            fn()  # warm caches/allocations outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for fn in fn_list:
            fn()
    return g


def time_graph(g, dist: Dist, repeats: int = 1) -> float:
    """Seconds for `repeats` replays between CUDA events (max over ranks)."""
    import torch
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeats):
        g.replay()
    end.record()
    dist.barrier()
    return dist.max(start.elapsed_time(end) / 1e3)


# ---------------------------------------------------------------------------
# FlashHead arm
# ---------------------------------------------------------------------------
def build_replicas(wl, n_rep, seed, device):
    """n_rep NativeHeads with identical contents at distinct addresses."""
    import torch

    from flash_head.native import NativeHead, derive_buffers
    from flash_head.synthetic import make_head
    shape = wl["shape"]
    head = make_head(shape, seed=seed, device=device)
    K, cap, D = shape.n_clusters, shape.cluster_size, shape.hidden
    from flash_head.flash_head import vocab_maps_from_assignments
    vm = vocab_maps_from_assignments(head.assignments, K)
    c32 = head.centroids.float()
    cw = (c32 / c32.norm(dim=0, keepdim=True)).t().contiguous()
    w_perm = head.weight.index_select(0, vm.reshape(-1)).view(K, cap, D)
    bufs = derive_buffers(w_perm, vm, cw, head.centroids, torch.zeros(0, dtype=torch.int64),
                          wl["stage1"])
    reps = [NativeHead(bufs, D, cap, shape.n_probes)]
    for _ in range(n_rep - 1):
        b2 = {k: (None if v is None else v.clone()) for k, v in bufs.items()}
        reps.append(NativeHead(b2, D, cap, shape.n_probes))
    return head, reps


def step_bytes(wl, rows, U):
    """Algorithmic HBM bytes of one step: stage-1 matrix (+scales) + hidden in,
    the U distinct probed clusters' rows, ids out."""
    s = wl["shape"]
    s1 = s.n_clusters * s.hidden * (1 if wl["stage1"] == "fp8" else 2)
    s1 += s.n_clusters * 4 if wl["stage1"] == "fp8" else 0
    s1 += rows * s.hidden * 2
    s3 = U * s.cluster_size * s.hidden * 2 + rows * s.hidden * 2 + rows * 8
    return s1, s3


def n_replicas_for(bytes_per_step):
    return max(1, min(16, math.ceil(3 * L2_BYTES / max(bytes_per_step, 1))))


def measure_flashhead(wl, reps, rows, steps, warmup, dist, hidden_pool):
    """Step time, stage times and distinct-probe counts for one batch size."""
    import torch
    nh = len(hidden_pool)
    Hs = [h[:rows].contiguous() for h in hidden_pool]
    for r in reps:
        r.workspace(rows)
    outs = [torch.empty(rows, dtype=torch.int64, device="cuda") for _ in range(max(steps, warmup))]
    probes = [reps[0].top_clusters(h) for h in Hs]
    U = statistics.mean(int(torch.unique(p).numel()) for p in probes)
    R = len(reps)

    def step(i):
        return lambda: reps[i % R].next_token(Hs[i % nh], out=outs[i])

    g_warm = capture([step(i) for i in range(warmup)])
    g_main = capture([step(i) for i in range(steps)])
    scores = [torch.empty((rows, wl["shape"].n_clusters), device="cuda") for _ in range(R)]
    g_s1 = capture([(lambda i=i: reps[i % R].cluster_scores(Hs[i % nh], out=scores[i % R]))
                    for i in range(steps)])
    g_s3 = capture([(lambda i=i: reps[i % R].stage2_next_token(Hs[i % nh], probes[i % nh],
                                                               out=outs[i]))
                    for i in range(steps)])
    g_warm.replay()
    t_main = time_graph(g_main, dist)
    t_s1 = time_graph(g_s1, dist)
    t_s3 = time_graph(g_s3, dist)
    return {"graph": g_main, "step_s": t_main / steps, "s1_s": t_s1 / steps,
            "s3_s": t_s3 / steps, "U": U}


def measure_dense(head, rows, steps, dist, hidden_pool):
    """Dense bf16 head: cuBLAS h @ W^T + argmax over the full vocabulary."""
    import torch
    W = head.weight  # [V, D] bf16, 525 MB+ (> L2)
    Hs = [h[:rows].contiguous() for h in hidden_pool]
    outs = [torch.empty(rows, dtype=torch.int64, device="cuda") for _ in range(steps)]

    def step(i):
        def f():
            torch.argmax(Hs[i % len(Hs)] @ W.t(), dim=-1, out=outs[i])
        return f
    g = capture([step(i) for i in range(steps)])
    g.replay()
    return time_graph(g, dist) / steps


def measure_library_dense(reps, rows, steps, dist, hidden_pool):
    """The library's exact dense head (fh_dense_next_token; greedy from 16 rows:
    one tcgen05 GEMM + argmax kernel and the id publish), rotating head
    replicas."""
    import torch
    Hs = [h[:rows].contiguous() for h in hidden_pool]
    for r in reps:
        r.workspace(rows)
    outs = [torch.empty(rows, dtype=torch.int64, device="cuda") for _ in range(steps)]
    R = len(reps)
    g = capture([(lambda i=i: reps[i % R].dense_next_token(Hs[i % len(Hs)], out=outs[i]))
                 for i in range(steps)])
    g.replay()
    return time_graph(g, dist) / steps


def measure_e2e(reps, rows, steps, warmup, dist, D):
    """Through the C-ABI call with host buffers (fh_get_next_token_host): per
    step the library copies the pinned host hidden states to the device, runs
    the step, copies the ids to pinned host memory and synchronises."""
    import torch

    from flash_head.synthetic import make_hidden
    from flash_head import _lib
    n_host = 8
    host_h = [make_hidden(rows, D, seed=9000 + i).pin_memory() for i in range(n_host)]
    host_out = torch.empty(rows, dtype=torch.int64).pin_memory()
    R = len(reps)
    # The C function bound once, its arguments resolved up front: per step the
    # host makes exactly the library call a C caller would make.
    fn = reps[0].lib.fh_get_next_token_host
    stream = _lib.stream_ptr()
    wss = [r.workspace(rows, host=True) for r in reps]
    args = [(reps[j].handle, wss[j].data_ptr(), wss[j].numel()) for j in range(R)]
    hp = [h.data_ptr() for h in host_h]
    op = host_out.data_ptr()

    def one(i):
        handle, wp, wn = args[i % R]
        st = fn(handle, hp[i % n_host], rows, op, wp, wn, stream)
        if st != 0:
            raise RuntimeError(_lib.last_error())

    for i in range(warmup):
        one(i)
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        one(i)
    end.record()
    dist.barrier()
    secs = dist.max(start.elapsed_time(end) / 1e3)
    return secs / steps, rows * D * 2, rows * 8


def cpu_reference_rate(head_cpu, rows, budget_s=12.0, max_steps=4000, warmup=2):
    """Reference CPU path (greedy gather-and-argmax branch, per row) on this host."""
    import torch

    from flash_head.synthetic import make_hidden
    from oracle.reference_cpu import ReferenceHeadCPU
    torch.set_num_threads(os.cpu_count() or 1)
    ref = ReferenceHeadCPU(head_cpu.weight, head_cpu.centroids, head_cpu.assignments,
                           n_probes=head_cpu.shape.n_probes)
    H = make_hidden(64, head_cpu.shape.hidden, seed=4242)

    def step(i):
        for r in range(rows):
            x = H[(i * rows + r) % 64].view(1, 1, -1)
            top = ref.top_clusters(x)
            logits, _, ids = ref.gather_logits(x, top, False)
            ids[logits.argmax(dim=-1, keepdim=True)]

    with torch.no_grad():
        for i in range(warmup):
            step(i)
        t0 = time.perf_counter()
        n = 0
        while n < max_steps and time.perf_counter() - t0 < budget_s:
            step(n)
            n += 1
        dt = time.perf_counter() - t0
    import platform
    cpu_model = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    cpu_model = ln.split(":", 1)[1].strip()
                    break
    except Exception:
        pass
    return {"value": n * rows / dt, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "ms_per_step": dt / n * 1e3,
            "sample": (f"{n} greedy decode steps of batch {rows} ({dt:.1f} s) through the "
                       f"reference's CPU gather-and-argmax branch (torch port, bf16), "
                       f"{cpu_model}")}


def run_flashhead(args, dist):
    import torch
    wl = workloads()[args.workload]
    rows = args.rows or wl["rows"]
    shape = wl["shape"]
    peak, peak_kind = measured_peaks()
    from flash_head.synthetic import make_hidden

    # replicas sized for the smallest batch measured (largest rotation need)
    s1b, s3b = step_bytes(wl, rows, min(shape.n_clusters, shape.n_probes * rows))
    n_rep = n_replicas_for(s1b + s3b)
    head, reps = build_replicas(wl, n_rep, seed=0, device="cuda")
    max_rows = max([rows] + (wl["sweep"] if args.sweep else []))
    hidden_pool = [make_hidden(max_rows, shape.hidden, seed=1000 + 97 * dist.rank + i,
                               device="cuda") for i in range(8)]

    res = measure_flashhead(wl, reps, rows, args.steps, args.warmup, dist, hidden_pool)
    s1_bytes, s3_bytes = step_bytes(wl, rows, res["U"])
    # clocks: sample over a ~0.5 s load window that ends with the timed region
    gid = gpu_id_for_smi(dist.local)
    g = res["graph"]
    with ClockSampler(gid) as cs:
        t_end = time.time() + 0.6
        while time.time() < t_end:
            g.replay()
        torch.cuda.synchronize()
        t_main = time_graph(g, dist)
    clocks = cs.summary()
    step_s = t_main / args.steps
    dense_s = measure_dense(head, rows, args.steps, dist, hidden_pool)

    launches = reps[0].step_kernel_count(rows)
    if launches == 1:
        # the whole step is one kernel: its duration is the step time
        kernels = {"k_fused_step": (step_s, s1_bytes + s3_bytes)}
    else:
        kernels = {"stage1_scores": (res["s1_s"], s1_bytes),
                   "stage2_gather_argmax": (res["s3_s"], s3_bytes)}
    dom = max(kernels, key=lambda k: kernels[k][0])
    dur, dbytes = kernels[dom]
    traffic = None
    tpath = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                traffic = json.load(f).get(args.workload, {}).get(dom)
        except Exception:
            traffic = None
    roofline = {"bound": "hbm", "kernel": dom, "achieved": dbytes / dur / 1e9, "peak": peak,
                "peak_kind": f"{peak_kind} (copy bandwidth)", "unit": "GB/s",
                "frac": dbytes / dur / 1e9 / peak, "traffic": traffic,
                "bytes_per_launch": dbytes, "us_per_launch": dur * 1e6}
    chain = (s1_bytes + s3_bytes) / step_s / 1e9
    stage_us = {"stage1_scores_kernel": res["s1_s"] * 1e6,
                "stage2_gather_argmax_kernel": res["s3_s"] * 1e6,
                "full_step": step_s * 1e6,
                "note": "stage kernels of the three-kernel path, each timed alone"}

    sweep = []
    if args.sweep:
        for b in wl["sweep"]:
            r = measure_flashhead(wl, reps, b, args.steps, args.warmup, dist, hidden_pool) \
                if b != rows else dict(res, step_s=step_s)
            d = measure_dense(head, b, args.steps, dist, hidden_pool) if b != rows else dense_s
            a1, a3 = step_bytes(wl, b, r["U"])
            sweep.append({"rows": b, "us_per_step": r["step_s"] * 1e6,
                          "tokens_per_s": b * dist.world / r["step_s"],
                          "distinct_probes": r["U"], "bytes_per_step": a1 + a3,
                          "achieved_gbs": (a1 + a3) / r["step_s"] / 1e9,
                          "frac_hbm": (a1 + a3) / r["step_s"] / 1e9 / peak,
                          "stage1_us": r["s1_s"] * 1e6, "stage2_us": r["s3_s"] * 1e6,
                          "dense_us_per_step": d * 1e6, "speedup_vs_dense": d / r["step_s"]})
            # FlashHead.get_next_token runs the dense head above 10 rows
            # (flash_head.py:292-301): the library's tcgen05 dense kernel
            if b > 10:
                ld = measure_library_dense(reps, b, args.steps, dist, hidden_pool)
                sweep[-1].update({"library_dense_us": ld * 1e6, "library_dense_vs_dense": d / ld,
                                  "get_next_token_path": "dense (more than 10 rows)",
                                  "get_next_token_us": ld * 1e6,
                                  "get_next_token_vs_dense": d / ld})
            else:
                sweep[-1].update({"get_next_token_path": "probes",
                                  "get_next_token_us": r["step_s"] * 1e6,
                                  "get_next_token_vs_dense": d / r["step_s"]})

    e2e_s, h2d, d2h = measure_e2e(reps, rows, args.steps, args.warmup, dist, shape.hidden)

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = cpu_reference_rate(_cpu_head(head), rows)

    out = {
        "metric": METRIC, "value": rows * dist.world / step_s, "unit": "tokens/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "us_per_step": step_s * 1e6, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if wl["stage1"] != "fp8" else "bf16 (stage-1 centroids fp8-e4m3)",
        "data": "synthetic: seeded centre+noise head (centres N(0,0.02^2), noise N(0,0.005^2)), "
                "hidden states N(0,0.25) bf16",
        "config": {"workload": workload_label(wl, rows), "global_batch": rows * dist.world,
                   "seq_len": 1,
                   "parallelism": "replicas" if dist.world > 1 else "single-gpu",
                   "l2": f"inputs larger than L2: {n_rep} rotating head replicas "
                         f"({n_rep * (s1_bytes + s3_bytes) / 1e6:.0f} MB touched per cycle)",
                   "timing": "CUDA graph of K steps between CUDA events, max over ranks"},
        "roofline": roofline,
        "roofline_step": {"bound": "hbm", "achieved": chain, "peak": peak, "unit": "GB/s",
                          "frac": chain / peak, "bytes_per_step": s1_bytes + s3_bytes},
        "stage_us": stage_us,
        "dense_us_per_step": dense_s * 1e6, "speedup_vs_dense": dense_s / step_s,
        "distinct_probes": res["U"],
        "sweep": sweep,
        "e2e": {"value": rows * dist.world / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "us_per_step": e2e_s * 1e6,
                "path": "C-ABI fh_get_next_token_host: pinned host buffers, copies and stream sync inside the call"},
        "gpu_launches": launches * args.steps,
        "step_kernels": launches,
        "clocks": clocks,
    }
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return out


def _cpu_head(head):
    from flash_head.synthetic import SyntheticHead
    return SyntheticHead(weight=head.weight.cpu(), centroids=head.centroids.cpu(),
                         assignments=head.assignments.cpu(), shape=head.shape, seed=head.seed)


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU path on this host
# ---------------------------------------------------------------------------
def run_reference(args):
    import torch

    from flash_head.synthetic import make_head, make_hidden
    from oracle.reference_cpu import ReferenceHeadCPU
    wl = workloads()[args.workload]
    rows = args.rows or wl["rows"]
    torch.set_num_threads(os.cpu_count() or 1)
    head = make_head(wl["shape"], seed=0)
    ref = ReferenceHeadCPU(head.weight, head.centroids, head.assignments,
                           n_probes=wl["shape"].n_probes)
    H = make_hidden(64, wl["shape"].hidden, seed=4242)

    def step(i):
        for r in range(rows):
            x = H[(i * rows + r) % 64].view(1, 1, -1)
            logits, _, ids = ref.gather_logits(x, ref.top_clusters(x), False)
            ids[logits.argmax(dim=-1, keepdim=True)]

    with torch.no_grad():
        for i in range(args.warmup):
            step(i)
        t0 = time.perf_counter()
        for i in range(args.steps):
            step(i)
        dt = time.perf_counter() - t0
    value = args.steps * rows / dt
    sample = (f"{args.steps} greedy decode steps of batch {rows} through the reference's CPU "
              f"gather-and-argmax branch (torch port of flash_head.py:190-261, bf16)")
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded centre+noise head, hidden states N(0,0.25) bf16",
        "config": {"workload": workload_label(wl, rows), "global_batch": rows, "seq_len": 1,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_profile(args):
    """Small eager run for ncu: one head replica (about 0.6 GB), W warm-up steps,
    then --profile-steps greedy steps launched one by one (no graphs); with
    --profile-path dense the steps are the dense head (fh_dense_next_token)."""
    import torch

    from flash_head.synthetic import make_hidden
    wl = workloads()[args.workload]
    rows = args.rows or wl["rows"]
    torch.cuda.set_device(0)
    _, reps = build_replicas(wl, 1, seed=0, device="cuda")
    nh = reps[0]
    H = [make_hidden(rows, wl["shape"].hidden, seed=1000 + i, device="cuda") for i in range(8)]
    out = torch.empty(rows, dtype=torch.int64, device="cuda")
    step = nh.dense_next_token if args.profile_path == "dense" else nh.next_token
    for i in range(args.warmup):
        step(H[i % 8], out=out)
    torch.cuda.synchronize()
    for i in range(args.profile_steps):
        step(H[i % 8], out=out)
    torch.cuda.synchronize()
    print(json.dumps({"profile_steps": args.profile_steps, "rows": rows,
                      "workload": workload_label(wl, rows), "last_ids": out.tolist()}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["flashhead", "reference"], default="flashhead")
    ap.add_argument("--workload", default="llama1b-fp8")
    ap.add_argument("--rows", type=int, default=0)
    ap.add_argument("--no-sweep", dest="sweep", action="store_false")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="eager profiling run (for ncu) instead of the benchmark")
    ap.add_argument("--profile-path", choices=["step", "dense"], default="step")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.profile_steps:
        run_profile(args)
        return

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        print(json.dumps(run_reference(args)), flush=True)
        return

    dist = Dist(args.gpus)
    try:
        out = run_flashhead(args, dist)
        if dist.rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
