"""Benchmark: soft Smith-Waterman forward + backward GCUPS on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Metric: GCUPS = valid DP cells per second for one forward that
produces value + marginals plus ``value.sum().backward()``.  Default workload is
soft_sw, fp32 scores [256, 512, 512] ~ N(0,1) (seed 0), gap -1,
temperature 1, no masks.  Weak scaling: every rank runs its own 256-problem batch
(seeded from the global seed and its rank) and the per-sequence values are
gathered with NCCL every step -- the only collective on the path.

``value`` is measured with the inputs resident in HBM (scores 268 MB > L2 126 MB,
so every step streams from DRAM; no extra L2 flush).  ``e2e`` is the same step
through the public API with every step's scores copied from pinned host memory
and its values copied back; the copy for the next step overlaps the current
step's compute (a copy stream and two device buffers), all inside the timed
region.
``strong`` (N > 1) is the same step with the config's batch split across the
ranks (rank r takes the contiguous slice ``shard_bounds(B, N, r)`` of one
globally seeded batch), timed the same way: the fixed-total-work curve.
``hvp`` times the Hessian-vector product over the same batch (every family
but affine SW).
``--config nw2`` / ``nwa2`` / ``dtw2`` run soft Needleman-Wunsch (linear and
affine gaps) and soft DTW at config 2's shape (the same step through
``soft_nw`` / ``soft_nw_affine`` / ``soft_dtw``); their reference leg is the
reference's own CPU kernels of that family (value + marginals, whose marginals
are the gradient of value.sum()).
``--config emb2`` runs soft SW of scores built from bf16 embeddings on the
tensor cores (``soft_sw_embed``: the tcgen05 score producer, then the DP) with
the gradient down to the embeddings; its line adds a ``producer`` object (the
producer kernel alone against the measured HBM and bf16 peaks).
The MUFU roofline denominator is measured in the same run (``d2p_mufu_probe``,
an ex2.approx throughput kernel).
``--impl reference`` times the reference's own CPU operators (oracle/_ref, built
from the reference sources: its schemas, CPU bindings, autograd and kernels)
through ``torch.ops.d2p`` with ``value.sum().backward()``, on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "soft_sw fwd+bwd GCUPS (DP cells/s) at 1/2/4/8 B200; % of HBM/MUFU roofline"

# BASELINE.json configs (C1..C5)
CONFIGS = {
    "c1": dict(family="linear", B=2, L1=100, L2=120, gap=-1.0, T=1.0, scale=1.0, lengths=False,
               dtype="f32", desc="soft_sw [2,100,120] fp32, gap -1, T 1"),
    "c2": dict(family="linear", B=256, L1=512, L2=512, gap=-1.0, T=1.0, scale=1.0, lengths=False,
               dtype="f32", desc="soft_sw [256,512,512] fp32, gap -1, T 1, no masks"),
    "c3": dict(family="linear", B=1024, L1=512, L2=512, gap=-0.5, T=0.5, scale=1.0, lengths=True,
               dtype="f32", desc="soft_sw [1024,512,512] fp32, lengths U[64,512] (seed 1), gap -0.5, T 0.5"),
    "c4": dict(family="affine", B=64, L1=1024, L2=1024, gap=(-2.0, -0.5), T=1.0, scale=1.0, lengths=False,
               dtype="bf16", desc="soft_sw_affine [64,1024,1024] bf16 -> fp32, open -2, ext -0.5, T 1"),
    "c5": dict(family="linear", B=32, L1=4096, L2=4096, gap=-1.0, T=1.0, scale=0.5, lengths=False,
               dtype="f32", desc="soft_sw [32,4096,4096] fp32 0.5*N(0,1), gap -1, T 1"),
    # soft Needleman-Wunsch at config 2's shape (a widening of the path, not a BASELINE config)
    "nw2": dict(family="nw", B=256, L1=512, L2=512, gap=-1.0, T=1.0, scale=1.0, lengths=False,
                dtype="f32", desc="soft_nw [256,512,512] fp32, gap -1, T 1, no masks"),
    "nwa2": dict(family="nw_affine", B=256, L1=512, L2=512, gap=(-2.0, -0.5), T=1.0, scale=1.0, lengths=False,
                 dtype="f32", desc="soft_nw_affine [256,512,512] fp32, open -2, ext -0.5, T 1, no masks"),
    # soft SW of scores built from bf16 embeddings on the tensor cores (score producer + DP)
    "emb2": dict(family="embed", B=256, L1=512, L2=512, D=128, gap=-1.0, T=1.0, scale=1.0, lengths=False,
                 dtype="bf16", desc="soft_sw_embed: bf16 embeddings [256,512,128] x [256,512,128] -> scores "
                                    "[256,512,512], gap -1, T 1"),
    "dtw2": dict(family="dtw", B=256, L1=512, L2=512, gap=None, T=1.0, scale=1.0, lengths=False,
                 dtype="f32", desc="soft_dtw [256,512,512] fp32 N(0,1) costs, T 1, no band, no masks"),
}

# Algorithmic cost per valid cell (a fixed convention from the log-domain algorithm,
# independent of how this implementation does the work):
#   fused DP kernel (value + marginals): read scores 4 B (bf16: 2 B) + write marginals 4 B;
#     MUFU 10 (forward LSE 4 ex2 + 1 lg2, reverse 1 ex2 beta_init + 4 ex2 weights);
#     affine: 22 MUFU.
#   value backward kernel: read marginals 4 B + write grad 4 B.
#   soft NW: as linear; affine NW: 21 (three 3-way LSEs forward, nine weights reverse);
#   soft DTW: 7 (one 3-way softmin forward, three weights reverse).
MUFU_PER_CELL = {"linear": 10, "affine": 22, "nw": 10, "nw_affine": 21, "dtw": 7}
MUFU_PER_SM_CLK = 16


def profile_kernels(fn):
    """{kernel name: (launches, device us)} of one call of fn, from the profiler."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    out = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            n, t = out.get(e.name, (0, 0.0))
            out[e.name] = (n + 1, t + e.device_time_total)
    return out


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("sm_max_mhz", 1965.0)), "measured"
    except Exception:
        return 6650.0, 1965.0, "fallback"


def measure_mufu_peak(dev) -> float:
    """ex2.approx operations per second of the whole GPU, by d2p_mufu_probe
    (best of 5 launches after 3 warm-ups, CUDA events on the launching stream)."""
    import ctypes

    import torch

    lib = ctypes.CDLL(os.path.join(ROOT, "d2p_b200", "libd2p_b200.so"))
    lib.d2p_mufu_probe.restype = ctypes.c_int
    lib.d2p_mufu_probe.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    threads, chains = 512, 8  # D2P_MUFU_PROBE_THREADS, D2P_MUFU_PROBE_CHAINS
    blocks = 4 * torch.cuda.get_device_properties(dev).multi_processor_count
    iters = 4096
    out = torch.empty(blocks * threads, device=dev)
    st = torch.cuda.current_stream(dev)
    best = None
    for k in range(8):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        rc = lib.d2p_mufu_probe(ctypes.c_void_p(out.data_ptr()), blocks, iters, ctypes.c_void_p(st.cuda_stream))
        e1.record(st)
        if rc != 0:
            raise RuntimeError(f"d2p_mufu_probe failed: {rc}")
        torch.cuda.synchronize(dev)
        if k >= 3:
            t = e0.elapsed_time(e1) * 1e-3
            best = t if best is None else min(best, t)
    return blocks * threads * chains * iters / best


# ----------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ----------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampler: lines are timestamped on arrival by a reader thread;
    the summary keeps the samples taken within 0.15 s of the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.rows = []
        self.t0 = self.t1 = None

    def start(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                self.rows.append((time.monotonic(), [p.strip() for p in line.split(",")]))

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        t_end = time.monotonic() + 5.0
        while not self.rows and time.monotonic() < t_end:   # wait until it is emitting
            time.sleep(0.02)

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        t0 = (self.t0 or 0) - 0.15
        t1 = (self.t1 or time.monotonic()) + 0.15
        rows = [r for (t, r) in self.rows if t0 <= t <= t1 and len(r) >= 9]
        if not rows:
            return None

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        pw = [v for v in (num(r[3]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------
# inputs
# ----------------------------------------------------------------------------
def make_inputs(cfg, rank: int):
    import torch

    g = torch.Generator().manual_seed(0 + 7919 * rank)
    s = torch.randn(cfg["B"], cfg["L1"], cfg["L2"], generator=g) * cfg["scale"]
    if cfg["dtype"] == "bf16":
        s = s.to(torch.bfloat16)
    lengths = None
    if cfg["lengths"]:
        g1 = torch.Generator().manual_seed(1 + 7919 * rank)
        lengths = torch.randint(64, 513, (cfg["B"], 2), generator=g1, dtype=torch.int32)
    return s, lengths


def valid_cells(cfg, lengths) -> int:
    if lengths is None:
        return cfg["B"] * cfg["L1"] * cfg["L2"]
    l = lengths.to(dtype=__import__("torch").int64)
    return int((l[:, 0] * l[:, 1]).sum().item())


# ----------------------------------------------------------------------------
# our implementation
# ----------------------------------------------------------------------------
def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    import d2p_b200 as d2p
    from d2p_b200.shard import gather_values

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    s_host, lengths = make_inputs(cfg, rank)
    cells = valid_cells(cfg, lengths)
    fam = cfg["family"]
    gap = cfg["gap"]
    T = cfg["T"]
    s_dev = s_host.to(dev).requires_grad_(True)
    len_dev = lengths.to(dev) if lengths is not None else None
    vals_all = torch.empty(world * cfg["B"], device=dev)

    def fwd(scores, ln):
        if fam == "linear":
            return d2p.soft_sw(scores, gap=gap, temperature=T, lengths=ln)
        if fam == "nw":
            return d2p.soft_nw(scores, gap=gap, temperature=T, lengths=ln)
        if fam == "nw_affine":
            return d2p.soft_nw_affine(scores, gap_open=gap[0], gap_ext=gap[1], temperature=T, lengths=ln)
        if fam == "dtw":
            return d2p.soft_dtw(scores, temperature=T, lengths=ln)
        return d2p.soft_sw_affine(scores, gap_open=gap[0], gap_ext=gap[1], temperature=T, lengths=ln)

    def step(scores):
        res = fwd(scores, len_dev)
        (grad,) = torch.autograd.grad(res[0].sum(), scores)
        v = res[0].detach()
        if world > 1:  # rank r owns problems [r*B, (r+1)*B) of the global batch
            vals_all.copy_(gather_values(v, world * cfg["B"]))
        return v, grad

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()

    # ---------------- device-resident timing ----------------
    for _ in range(args.warmup):
        step(s_dev)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    clocks.mark_start()
    e0.record()
    for _ in range(args.steps):
        step(s_dev)
    e1.record()
    barrier()
    clocks.mark_end()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # ---------------- dominant kernel alone (same stream, CUDA events) ----------------
    nk = max(3, args.steps)
    with torch.no_grad():
        def kern():
            # the op the forward calls when the gap parameters and T need no gradient
            if fam == "linear":
                return torch.ops.d2p.soft_sw_float(s_dev, gap, T, len_dev)
            if fam == "nw":
                return torch.ops.d2p.soft_nw_float(s_dev, gap, T, len_dev)
            if fam == "nw_affine":
                return torch.ops.d2p.soft_nw_affine_float(s_dev, gap[0], gap[1], T, len_dev)
            if fam == "dtw":
                return torch.ops.d2p.soft_dtw_float(s_dev, T, len_dev, None)
            return torch.ops.d2p.soft_sw_affine_float(s_dev, gap[0], gap[1], T, len_dev)
        for _ in range(2):
            kern()
        torch.cuda.synchronize()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        for _ in range(nk):
            kern()
        k1.record()
        torch.cuda.synchronize()
        k_ms = k0.elapsed_time(k1) / nk

    # ---------------- what one step launches (outside the timed regions) ----------------
    # One step under the profiler: this library's kernels by name, their
    # count (the line's gpu_launches) and the one with the most device time
    # (the roofline's kernel).
    step_kernels = profile_kernels(lambda: step(s_dev))
    ours = {n.replace("void ", "", 1): v for n, v in step_kernels.items() if "d2pb::" in n}
    dom = max(ours, key=lambda n: ours[n][1]) if ours else "unknown"
    launches_per_step = sum(v[0] for v in ours.values())

    # ---------------- end to end from pinned host memory ----------------
    # Every step copies its scores host -> device from pinned memory and its
    # values device -> host.  As in an input pipeline, the copy for step k+1
    # runs on a copy stream while step k computes (two device buffers); every
    # copy lies inside the timed region.
    s_pin = s_host.pin_memory()
    v_host = torch.empty(cfg["B"], pin_memory=True)
    bufs = [torch.empty_like(s_dev), torch.empty_like(s_dev)]
    main = torch.cuda.current_stream(dev)
    cstream = torch.cuda.Stream(device=dev)
    freed = [torch.cuda.Event(), torch.cuda.Event()]   # buffer i no longer read by a step
    loaded = [torch.cuda.Event(), torch.cuda.Event()]  # buffer i holds the next step's scores

    def issue_copy(i):
        cstream.wait_event(freed[i])
        with torch.cuda.stream(cstream):
            bufs[i].copy_(s_pin, non_blocking=True)
        loaded[i].record(cstream)

    def e2e_run(n):
        for i in range(2):
            freed[i].record(main)
        issue_copy(0)
        for k in range(n):
            i = k % 2
            if k + 1 < n:
                issue_copy(1 - i)
            main.wait_event(loaded[i])
            x = bufs[i].requires_grad_(True)
            v, _ = step(x)
            v_host.copy_(v, non_blocking=True)
            x.requires_grad_(False)
            freed[i].record(main)

    e2e_run(max(1, min(args.warmup, 2)))
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    e2e_run(args.steps)
    x1.record()
    barrier()
    e2e_ms = x0.elapsed_time(x1) / args.steps
    te = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())

    # ---------------- strong scaling: one global batch split across the ranks ----------------
    # Rank r computes the slice shard_bounds(B, N, r) of the globally seeded
    # batch (seed 0: rank 0's own inputs above) and the values are gathered,
    # as soft_sw_sharded does.  At N = 1 this is the step timed above.
    strong = None
    if world > 1:
        from d2p_b200.shard import shard_bounds

        g_host, g_len = make_inputs(cfg, 0)
        lo, hi = shard_bounds(cfg["B"], world, rank)
        sh_dev = g_host[lo:hi].to(dev).requires_grad_(True)
        sh_len = g_len[lo:hi].to(dev) if g_len is not None else None
        del g_host
        vals_g = torch.empty(cfg["B"], device=dev)

        def strong_step():
            res = fwd(sh_dev, sh_len)
            torch.autograd.grad(res[0].sum(), sh_dev)
            vals_g.copy_(gather_values(res[0].detach(), cfg["B"]))

        for _ in range(args.warmup):
            strong_step()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            strong_step()
        s1.record()
        barrier()
        ts = torch.tensor([s0.elapsed_time(s1) / args.steps], device=dev)
        dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        st_ms = float(ts.item())
        g_cells = valid_cells(cfg, g_len)
        strong = {"value": round(g_cells / (st_ms * 1e-3) / 1e9, 3), "unit": "GCUPS", "ms_per_step": round(st_ms, 4),
                  "global_batch": cfg["B"], "per_rank_batch": hi - lo,
                  "note": "fixed total work: the config's batch split across the ranks, values all-gathered"}
        del sh_dev

    total_cells = cells * world
    gcups = total_cells / (ms_max * 1e-3) / 1e9
    e2e_gcups = total_cells / (e2e_ms * 1e-3) / 1e9

    hbm_gbs, sm_max_mhz, peak_src = load_peaks()
    sm_clock_mhz = (clk or {}).get("sm_mhz") or sm_max_mhz
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    score_bytes = 2 if cfg["dtype"] == "bf16" else 4
    padded = cfg["B"] * cfg["L1"] * cfg["L2"]
    # fused DP kernel algorithmic traffic: scores read + marginals write (padding
    # cells of the marginals are zero-filled: 4 B each)
    k_bytes = cells * score_bytes + padded * 4
    k_mufu = cells * MUFU_PER_CELL[fam]
    mufu_nominal = sm_count * MUFU_PER_SM_CLK * sm_max_mhz * 1e6  # ops/s at max SM clock
    mufu_peak = measure_mufu_peak(dev)  # measured ex2.approx throughput, this GPU, this run
    t_hbm = k_bytes / (hbm_gbs * 1e9)
    t_mufu = k_mufu / mufu_peak
    bound = "mufu" if t_mufu >= t_hbm else "hbm"
    k_s = k_ms * 1e-3
    if bound == "mufu":
        achieved, peak, unit = k_mufu / k_s / 1e12, mufu_peak / 1e12, "Tops/s (MUFU)"
    else:
        achieved, peak, unit = k_bytes / k_s / 1e9, hbm_gbs, "GB/s"
    traffic = None
    tp = os.path.join(ROOT, "profiles", f"traffic_{args.config}.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get("bytes_per_launch")
        except Exception:
            traffic = None
    roofline = {
        "bound": bound, "achieved": round(achieved, 4), "peak": round(peak, 4), "unit": unit,
        "frac": round(achieved / peak, 4), "traffic": traffic,
        "kernel": dom.split("(")[0].split("<")[0] + " (value+marginals: " +
                  {"linear": "d2p_sw", "affine": "d2p_sw_affine", "nw": "d2p_nw",
                   "nw_affine": "d2p_nw_affine", "dtw": "d2p_dtw"}[fam] + "_forward_backward)",
        "kernel_ms": round(k_ms, 4), "time_bound_ms": round(max(t_hbm, t_mufu) * 1e3, 4),
        "hbm_gbs_achieved": round(k_bytes / k_s / 1e9, 2), "hbm_peak_gbs": hbm_gbs,
        "mufu_tops_achieved": round(k_mufu / k_s / 1e12, 3), "mufu_peak_tops": round(mufu_peak / 1e12, 3),
        "mufu_nominal_tops": round(mufu_nominal / 1e12, 3),
        "peak_source": (f"HBM: {peak_src} (MEASURED_PEAKS.json hbm_gbs); MUFU: measured in this run by "
                        f"d2p_mufu_probe (ex2.approx throughput; nominal {sm_count} SM x 16/clk x "
                        f"{sm_max_mhz:.0f} MHz = {mufu_nominal / 1e12:.3f} Tops/s)"),
        "step_frac": round((max(t_hbm, t_mufu) + (8.0 * padded) / (hbm_gbs * 1e9)) / (ms_max * 1e-3), 4),
    }

    # ---------------- Hessian-vector product (BASELINE config 5 reports it) ----------------
    hvp = None
    if fam in ("linear", "nw", "nw_affine", "dtw") and not args.no_hvp:
        gv = torch.Generator().manual_seed(2 + 1000 * rank)
        v_dev = torch.randn(s_host.shape, generator=gv).to(dev)
        with torch.no_grad():
            def hvp_step():
                if fam == "nw":
                    return torch.ops.d2p.soft_nw_hvp(s_dev, v_dev, gap, T, len_dev)
                if fam == "nw_affine":
                    return torch.ops.d2p.soft_nw_affine_hvp(s_dev, v_dev, gap[0], gap[1], T, len_dev)
                if fam == "dtw":
                    return torch.ops.d2p.soft_dtw_hvp(s_dev, v_dev, T, len_dev, None)
                return torch.ops.d2p.soft_sw_hvp(s_dev, v_dev, gap, T, len_dev)
            for _ in range(2):
                hvp_step()
            barrier()
            h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            h0.record()
            for _ in range(nk):
                hvp_step()
            h1.record()
            barrier()
            h_ms = h0.elapsed_time(h1) / nk
        th = torch.tensor([h_ms], device=dev)
        if world > 1:
            dist.all_reduce(th, op=dist.ReduceOp.MAX)
        h_ms = float(th.item())
        # convention: 12 B (scores, V, H) and the family's MUFU count per valid cell
        h_bound = max(12.0 * cells / (hbm_gbs * 1e9), MUFU_PER_CELL[fam] * cells / mufu_peak)
        h_kernel = {"linear": "ltan::lin_tan_kernel (d2p_sw_hvp)",
                    "nw": "nwt::nw_wave_tan_kernel<HVP> (d2p_nw_hvp)",
                    "nw_affine": "nwa::nwa_kernel<HVP> (d2p_nw_affine_hvp)",
                    "dtw": "dtww::dtw_wave_tan_kernel<HVP> (d2p_dtw_hvp)"}[fam]
        hvp = {"value": round(total_cells / (h_ms * 1e-3) / 1e9, 3), "unit": "GCUPS", "ms_per_step": round(h_ms, 4),
               "kernel": h_kernel, "time_bound_ms": round(h_bound * 1e3, 4),
               "frac": round(h_bound / (h_ms * 1e-3), 4),
               # fwd + bwd step and one HVP over the same cells, timed as above
               "combined": {"value": round(total_cells / ((ms_max + h_ms) * 1e-3) / 1e9, 3), "unit": "GCUPS",
                            "ms_per_step": round(ms_max + h_ms, 4)}}
        del v_dev

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, args.cpu_seconds)

    if world > 1:
        dist.barrier()
    if rank == 0:
        h2d = s_host.numel() * s_host.element_size()
        line = {
            "metric": METRIC, "value": round(gcups, 3), "unit": "GCUPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if cfg["dtype"] == "f32" else "bf16-in/f32",
            "data": "synthetic (seeded N(0,1) scores, BASELINE shapes)",
            "config": {"workload": f"{args.config}: {cfg['desc']}", "per_rank_batch": cfg["B"],
                       "global_batch": cfg["B"] * world, "L1": cfg["L1"], "L2": cfg["L2"],
                       "valid_cells_per_rank": cells, "step": "forward (value+marginals) + value.sum().backward()",
                       "l2": "inputs larger than L2 (scores+marginals stream from DRAM every step)",
                       "parallelism": f"batch x{world} (one process per GPU), NCCL all_gather of values"},
            "e2e": {"value": round(e2e_gcups, 3), "unit": "GCUPS", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": cfg["B"] * 4, "ms_per_step": round(e2e_ms, 4)},
            # this library's kernels in one profiled step (outside the timed
            # region), times the timed steps
            "gpu_launches": args.steps * launches_per_step,
            "step_kernels": {n.split("(")[0]: v[0] for n, v in ours.items()},
            "roofline": roofline,
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if hvp is not None:
            line["hvp"] = hvp
        if strong is not None:
            line["strong"] = strong
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# soft SW from embeddings (score producer on tcgen05 + the strip kernel)
# ----------------------------------------------------------------------------
def run_embed(args, cfg):
    """One step = soft_sw_embed (scores = x y^T on the tensor cores, soft SW of
    them) + value.sum().backward() down to the embeddings.  Single process; the
    producer kernel is also timed alone against the measured bf16 and HBM peaks."""
    import torch

    import d2p_b200 as d2p

    # one process per GPU when launched by torchrun: each rank times its own
    # copy of the workload (no collective); rank 0 prints its line
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, L1, L2, D = cfg["B"], cfg["L1"], cfg["L2"], cfg["D"]
    g = torch.Generator().manual_seed(0)
    x_host = (torch.randn(B, L1, D, generator=g) / D ** 0.25).to(torch.bfloat16)
    y_host = (torch.randn(B, L2, D, generator=g) / D ** 0.25).to(torch.bfloat16)
    x = x_host.to(dev).requires_grad_(True)
    y = y_host.to(dev).requires_grad_(True)
    gap, T = cfg["gap"], cfg["T"]

    def step(xa, ya):
        res = d2p.soft_sw_embed(xa, ya, gap=gap, temperature=T)
        gx, gy = torch.autograd.grad(res.value.sum(), (xa, ya))
        return res.value.detach(), gx, gy

    for _ in range(args.warmup):
        step(x, y)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    clocks.mark_start()
    e0.record()
    for _ in range(args.steps):
        step(x, y)
    e1.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps

    # the producer alone (same stream, CUDA events)
    with torch.no_grad():
        xd, yd = x.detach(), y.detach()
        for _ in range(3):
            torch.ops.d2p_b200.embed_scores(xd, yd, 1.0)
        torch.cuda.synchronize()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nk = max(3, args.steps)
        p0.record()
        for _ in range(nk):
            torch.ops.d2p_b200.embed_scores(xd, yd, 1.0)
        p1.record()
        torch.cuda.synchronize()
        p_ms = p0.elapsed_time(p1) / nk

    step_kernels = profile_kernels(lambda: step(x, y))
    ours = {n.replace("void ", "", 1): v for n, v in step_kernels.items() if "d2pb::" in n or "embed_scores" in n}
    launches = sum(v[0] for v in ours.values())

    # end to end: every step's embeddings copied from pinned host memory, its
    # values back; as in an input pipeline, step k+1's copy runs on a copy
    # stream while step k computes (two device buffers), all inside the timed region
    xp, yp = x_host.pin_memory(), y_host.pin_memory()
    v_host = torch.empty(B, pin_memory=True)
    bx = [torch.empty_like(x.detach()), torch.empty_like(x.detach())]
    by = [torch.empty_like(y.detach()), torch.empty_like(y.detach())]
    main = torch.cuda.current_stream(dev)
    cstream = torch.cuda.Stream(device=dev)
    freed = [torch.cuda.Event(), torch.cuda.Event()]
    loaded = [torch.cuda.Event(), torch.cuda.Event()]

    def issue_copy(i):
        cstream.wait_event(freed[i])
        with torch.cuda.stream(cstream):
            bx[i].copy_(xp, non_blocking=True)
            by[i].copy_(yp, non_blocking=True)
        loaded[i].record(cstream)

    def e2e_run(n):
        for i in range(2):
            freed[i].record(main)
        issue_copy(0)
        for k in range(n):
            i = k % 2
            if k + 1 < n:
                issue_copy(1 - i)
            main.wait_event(loaded[i])
            v, _, _ = step(bx[i].requires_grad_(True), by[i].requires_grad_(True))
            v_host.copy_(v, non_blocking=True)
            bx[i].requires_grad_(False)
            by[i].requires_grad_(False)
            freed[i].record(main)

    e2e_run(2)
    torch.cuda.synchronize()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    e2e_run(args.steps)
    x1.record()
    torch.cuda.synchronize()
    e2e_ms = x0.elapsed_time(x1) / args.steps

    cells = B * L1 * L2
    hbm_gbs, _, peak_src = load_peaks()
    try:
        bf16_peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
    except Exception:
        bf16_peak = 1590.0
    flops = 2.0 * B * L1 * L2 * D
    wbytes = 4.0 * cells + 2.0 * B * (L1 + L2) * D   # scores written, embeddings read
    t_tensor = flops / (bf16_peak * 1e12)
    t_hbm = wbytes / (hbm_gbs * 1e9)
    bound = "hbm" if t_hbm >= t_tensor else "tensor"
    p_s = p_ms * 1e-3
    producer = {
        "kernel": "d2pb::emb::embed_scores_kernel (tcgen05.mma kind::f16, TMA, TMEM; d2p_embed_scores)",
        "kernel_ms": round(p_ms, 4), "bound": bound,
        "achieved": round(wbytes / p_s / 1e9, 2) if bound == "hbm" else round(flops / p_s / 1e12, 2),
        "peak": hbm_gbs if bound == "hbm" else bf16_peak, "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
        "frac": round((t_hbm if bound == "hbm" else t_tensor) / p_s, 4),
        "tflops": round(flops / p_s / 1e12, 2), "gbs": round(wbytes / p_s / 1e9, 2),
        "peak_source": f"MEASURED_PEAKS.json ({peak_src}): hbm_gbs and bf16_tflops (burst)",
    }
    line = {
        "metric": "soft_sw_embed fwd+bwd GCUPS (DP cells/s), scores built from bf16 embeddings on the tensor cores",
        "value": round(cells / (ms * 1e-3) / 1e9, 3), "unit": "GCUPS", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16-in/f32", "data": "synthetic (seeded N(0,1)/D^0.25 embeddings)",
        "config": {"workload": f"{args.config}: {cfg['desc']}", "B": B, "L1": L1, "L2": L2, "D": D,
                   "step": "soft_sw_embed (value + marginals) + value.sum().backward() to x and y",
                   "l2": "scores (268 MB) and marginals larger than L2"},
        "e2e": {"value": round(cells / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GCUPS",
                "h2d_bytes_per_step": int(x_host.numel() * 2 + y_host.numel() * 2), "d2h_bytes_per_step": B * 4,
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": args.steps * launches,
        "step_kernels": {n.split("(")[0]: v[0] for n, v in ours.items()},
        "producer": producer,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# reference CPU (oracle/_ref = the reference's own CPU kernels)
# ----------------------------------------------------------------------------
REF_OPS = os.path.join(ROOT, "oracle", "_ref", "libref_sw_ops.so")
REF_CUDA_OPS = os.path.join(ROOT, "oracle", "_ref", "libref_sw_cuda_ops.so")


def _ref_inputs(cfg):
    """The config's seeded inputs as the reference takes them: fp32 scores (bf16
    scores upcast, as the reference's autocast rule does) and int32 lengths."""
    s_host, lengths = make_inputs(cfg, 0)
    return s_host.float(), lengths


def _ref_fwd_bwd(cfg, s, ln):
    """One step through the reference's own operators: forward (value +
    marginals) and value.sum().backward() through its autograd Function."""
    x = s.detach().requires_grad_(True)
    if cfg["family"] == "linear":
        v, m = __import__("torch").ops.d2p.soft_sw_float(x, cfg["gap"], cfg["T"], ln)
    else:
        v, m = __import__("torch").ops.d2p.soft_sw_affine_float(x, cfg["gap"][0], cfg["gap"][1], cfg["T"], ln)
    v.sum().backward()
    return v, x.grad


def _cells(cfg, ln, nb):
    import numpy as np

    if ln is None:
        return nb * cfg["L1"] * cfg["L2"]
    ln = ln.cpu().numpy()
    return int(np.sum(ln[:, 0].astype(np.int64) * ln[:, 1]))


def _ref_cpu(cfg, steps: int, warmup: int, budget_s: float):
    """The reference's CPU operators on every host core, on a bounded sample of
    the config (the first nb problems, nb doubled until one step takes about
    budget_s / 2).  Returns (GCUPS, ms per step, cores, sample, kind)."""
    import torch

    ncores = os.cpu_count() or 1
    torch.set_num_threads(ncores)
    s_all, ln_all = _ref_inputs(cfg)
    kind = "reference"
    if os.path.exists(REF_OPS) and cfg["family"] in ("linear", "affine"):
        torch.ops.load_library(REF_OPS)
        step = lambda s, ln: _ref_fwd_bwd(cfg, s, ln)  # noqa: E731
        path = "torch.ops.d2p (reference CPU operators) + value.sum().backward()"
    else:  # no operator build: the reference's CPU kernels, or the port, through the oracle
        import oracle

        kind = "reference" if oracle.ref_available() else "port"
        impl = "ref" if kind == "reference" else "f32"

        def step(s, ln):
            lnp = None if ln is None else ln.numpy()
            if cfg["family"] == "linear":
                return oracle.sw_linear(s.numpy(), lnp, cfg["gap"], cfg["T"], impl)
            # NW / DTW: value + marginals; d value.sum() / d scores is the marginals
            if cfg["family"] == "nw":
                return oracle.nw_linear(s.numpy(), lnp, cfg["gap"], cfg["T"], impl)
            if cfg["family"] == "nw_affine":
                return oracle.nw_affine(s.numpy(), lnp, cfg["gap"][0], cfg["gap"][1], cfg["T"], impl)
            if cfg["family"] == "dtw":
                return oracle.dtw(s.numpy(), lnp, cfg["T"], -1, impl)
            return oracle.sw_affine(s.numpy(), lnp, cfg["gap"][0], cfg["gap"][1], cfg["T"], impl)
        path = f"CPU kernels ({impl}) through ctypes"
    nb = min(cfg["B"], max(1, ncores))
    while True:
        sub, ln = s_all[:nb], (ln_all[:nb] if ln_all is not None else None)
        t0 = time.perf_counter()
        step(sub, ln)
        dt = time.perf_counter() - t0
        if dt * 2 > budget_s or nb >= cfg["B"]:
            break
        nb = min(cfg["B"], nb * 2)
    for _ in range(warmup):
        step(sub, ln)
    t0 = time.perf_counter()
    for _ in range(steps):
        step(sub, ln)
    dt = (time.perf_counter() - t0) / steps
    g = _cells(cfg, ln, nb) / dt / 1e9
    sample = (f"{nb} of {cfg['B']} problems of {cfg['L1']}x{cfg['L2']} ({args_config_name(cfg)}) per step, "
              f"fwd+bwd via {path}")
    return g, dt * 1e3, ncores, sample, kind


def _ref_cuda(cfg, budget_s: float):
    """The reference's CUDA operators (its torch_cuda.cpp + kernels.cu built for
    sm_100a) on cuda:0: fwd + value.sum().backward() through its autograd,
    timed with CUDA events, on the first nb problems of the config (nb halved
    from the full batch until one step fits budget_s).  None when unavailable."""
    import torch

    if cfg["family"] not in ("linear", "affine") or not (torch.cuda.is_available() and os.path.exists(REF_CUDA_OPS)):
        return None  # the operator build holds the reference's SW and affine SW CUDA operators only
    torch.ops.load_library(REF_CUDA_OPS)
    s_all, ln_all = _ref_inputs(cfg)
    dev = torch.device("cuda", 0)
    nb = cfg["B"]
    while True:
        s = s_all[:nb].to(dev)
        ln = ln_all[:nb].to(dev) if ln_all is not None else None
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _ref_fwd_bwd(cfg, s, ln)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if dt <= budget_s or nb == 1:
            break
        nb = max(1, nb // 2)
    _ref_fwd_bwd(cfg, s, ln)  # warm-up
    reps = max(1, min(5, int(budget_s / max(dt, 1e-3))))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        _ref_fwd_bwd(cfg, s, ln)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    cells = _cells(cfg, ln, nb)
    return {"value": round(cells / (ms * 1e-3) / 1e9, 4), "unit": "GCUPS", "ms_per_step": round(ms, 3),
            "sample": f"{nb} of {cfg['B']} problems of {cfg['L1']}x{cfg['L2']}, fwd+bwd, {reps} steps",
            "build": "reference src/sw{,_affine}/{torch_cuda.cpp,kernels.cu}, nvcc -gencode "
                     "arch=compute_100a,code=sm_100a (oracle/Makefile)"}


def cpu_baseline(cfg, seconds: float):
    """The reference's CPU operators timed on the host cores, in a child process
    (its operators register the same torch.ops.d2p names as this library)."""
    name = args_config_name(cfg)
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--cpu-only",
           "--steps", "2", "--warmup", "3", "--config", name, "--ref-step-seconds", str(seconds)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ, RANK="0", WORLD_SIZE="1"))
    for line in r.stdout.splitlines()[::-1]:
        if line.startswith("{"):
            d = json.loads(line)
            return d["cpu_baseline"]
    return {"value": None, "unit": "GCUPS", "cores": os.cpu_count(), "kind": "reference",
            "sample": "failed: " + (r.stderr.strip().splitlines() or ["no output"])[-1][:200]}


def args_config_name(cfg):
    for k, v in CONFIGS.items():
        if v["desc"] == cfg["desc"]:
            return k
    return "custom"


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    g, ms, ncores, sample, kind = _ref_cpu(cfg, args.steps, args.warmup, args.ref_step_seconds)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(g, 5), "unit": "GCUPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": f"{args.config}: {cfg['desc']}", "sample": sample},
        "cpu_baseline": {"value": round(g, 5), "unit": "GCUPS", "cores": ncores, "kind": kind, "sample": sample},
        "e2e": {"value": round(g, 5), "unit": "GCUPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.cpu_only:
        try:
            rc = _ref_cuda(cfg, args.ref_cuda_seconds)
        except Exception as exc:  # reported, not fatal: the CPU figure is the arm's value
            rc = {"value": None, "error": f"{type(exc).__name__}: {str(exc)[:200]}"}
        if rc is not None:
            line["ref_cuda"] = rc
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=4.0)
    ap.add_argument("--ref-step-seconds", type=float, default=6.0)
    ap.add_argument("--cpu-only", action="store_true", help="reference arm: skip the reference CUDA leg")
    ap.add_argument("--ref-cuda-seconds", type=float, default=5.0)
    ap.add_argument("--batch", type=int, default=0, help="override the per-rank batch (profiling on a small case)")
    ap.add_argument("--no-hvp", action="store_true",
                    help="skip the Hessian-vector product leg (timed by default for every family but affine SW)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.batch > 0:
        cfg["B"] = args.batch
        cfg["desc"] = cfg["desc"] + f" (batch overridden to {args.batch})"
    if args.impl == "reference":
        if cfg["family"] == "embed":   # the reference has no embedding operator: einsum + its CPU soft_sw
            cfg = dict(cfg, family="linear")
        run_reference(args, cfg)
    elif cfg["family"] == "embed":
        run_embed(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
