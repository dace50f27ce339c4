"""Benchmark of the anchored transport score, forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): AnchoredExact(h=1, tau=1, all events as anchors, 16 slices, exposure
correction on) + DenseLinearFlow on a 2x480x640 per-pixel flow, loss.backward() down to the flow
grid, on one synthetic window of 1M events (640x480, density proportional to the gradient magnitude
of a random texture, times uniform over 100 ms, flow = Gaussian low-pass noise sigma 32 px scaled to
max |v| = 20 px per window).  With N GPUs every rank runs its own window (windows are independent:
weak scaling, no collective on the data path).

``--impl ours``       libatlb200 kernels; value = events/s with inputs resident in HBM, L2 flushed
                      before every step; e2e = the same step from pinned host buffers (H2D of the
                      events and the step's noise, D2H of the loss) inside the timed region.
``--impl reference``  the reference's own CPU path (its unmodified Python package from baseline/_ref
                      plus its OpenMP kernels compiled by oracle/Makefile) on all host cores.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "anchored-score fwd+bwd events/sec/GPU at 1M ev 640×480; % of HBM/atomic roofline"
N_EVENTS, H, W = 1_000_000, 480, 640
WORKLOAD = ("config2: AnchoredExact(h=1, tau=1, n_anchors=None, n_slices=16, visibility) + "
            "DenseLinearFlow(2x480x640) fwd+bwd, 1M events/window")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--events", type=int, default=N_EVENTS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--windows", type=int, default=8, help="--workload splat: windows of --events events")
    ap.add_argument("--dropin", action="store_true",
                    help="config2 through the stage-by-stage drop-in ops (device plan + ats_pair_fwd/bwd extension "
                         "calls, as atl's objective makes them) instead of the fused pipeline")
    ap.add_argument("--workload", default="config2", choices=["config2", "config3", "config5", "splat", "tiles"],
                    help="config2: one 1M-event window per GPU (the headline); config5: one 64M-event window "
                         "on 1280x720 shared by all GPUs (sources split across ranks, NCCL all-reduce); splat: the "
                         "Gaussian splat forward + backward of one slice of configuration 3 (sigma 1.5, 8 x 2M); "
                         "tiles: the bilinear splat, gather and voxel grid on 1M points")
    ap.add_argument("--no-strong", action="store_true",
                    help="leave out the strong-scaling legs of the default line (configuration 5a and 3 sharded "
                         "over the --gpus ranks)")
    ap.add_argument("--cpu-worker", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--record-traffic", nargs=2, metavar=("CSV", "COMMAND"), default=None,
                    help="write the per-launch DRAM traffic of the pair kernels from an ncu raw CSV export")
    return ap.parse_args()


def window_data(rank: int, n: int):
    """Seeded synthetic window of rank ``rank`` (CPU tensors; identical for both implementations)."""
    from x_b200 import synth
    ev = synth.textured_window(n, H, W, duration=0.1, seed=1000 + rank)
    flow = synth.lowpass_flow(1, H, W, sigma=32.0, vmax=20.0, seed=2000 + rank)
    return ev, flow


# ------------------------------------------------------------------------------------------------ reference
def run_reference_steps(xy, t, p, b, flow, steps, warmup, budget_s=None):
    """The reference's AnchoredExact + DenseLinearFlow on CPU tensors; returns per-step seconds."""
    import torch
    from oracle.refload import load_reference
    atl = load_reference()
    from atl.core.events import EventPacket
    from atl.motion import DenseLinearFlow
    from atl.objectives import AnchoredExact
    torch.set_num_threads(os.cpu_count() or 1)
    ev = EventPacket(xy, t, p, b, 1, H, W)
    m = DenseLinearFlow(1, H, W, grid=(H, W), mode="linear", init=flow)
    obj = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=7, visibility=True)

    def step():
        m.grid.grad = None
        out = obj(ev, m)
        out["loss"].backward()
        return float(out["loss"])

    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_start > budget_s:
            break
    return times


def run_port_steps(xy, t, b, flow, steps, warmup, budget_s=None):
    """The C restatement of the reference's path (oracle/atl_oracle.c, OpenMP) on the same window and the same
    per-step work as the reference's objective: the host draws of the dequantisation and smoothing noise (the
    objective's CPU generator), the pair plan, pair sums, window counts, exposure correction, score and the
    backward to the flow grid.  Returns per-step seconds."""
    import numpy as np
    import torch
    from oracle import oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    xy_n, t_n, b_n, flow_n = xy.numpy(), t.numpy(), b.numpy(), flow.numpy()
    n = t_n.shape[0]
    anchors = np.arange(n, dtype=np.int64)
    gen = torch.Generator().manual_seed(7)

    def step():
        u = torch.rand((n, 2), generator=gen).numpy()
        z = torch.randn((n, 2), generator=gen).numpy()
        xs = (xy_n + (u - np.float32(0.5))).astype(np.float32)
        xa = (xs + z).astype(np.float32)
        return O.anchored_exact("dense", flow_n, xs, t_n, b_n, 1, H, W, anchors, xa)["loss"]

    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_start > budget_s:
            break
    return times


def reference_or_port(xy, t, p, b, flow, steps, warmup, budget_s):
    """Times the reference's own CPU path (kind "reference"); where its package or its compiled extension is
    not present on this host, the C restatement of the same path (kind "port").  Returns (times, kind, note)."""
    try:
        from oracle.refload import load_reference
        load_reference()
    except ImportError as e:
        note = f"reference not importable here ({str(e)[:120]}); timed the C port of its CPU path"
        return run_port_steps(xy, t, b, flow, steps, warmup, budget_s), "port", note
    return run_reference_steps(xy, t, p, b, flow, steps, warmup, budget_s), "reference", ""


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        ev, flow = window_data(0, args.events)
        budget = 150.0
        times, kind, note = reference_or_port(ev.xy, ev.t, ev.p, ev.b, flow, args.steps, min(args.warmup, 1), budget)
    except Exception as e:  # neither the reference nor its C port could run here
        print(json.dumps({"impl": "reference", "unavailable": f"{type(e).__name__}: {e}"[:300]}))
        return
    ms = 1000 * statistics.mean(times)
    value = args.events / (ms / 1000)
    cores = os.cpu_count() or 1
    what = ("reference AnchoredExact + its OpenMP kernels" if kind == "reference"
            else "C port of the reference's CPU path (OpenMP)")
    sample = (f"full workload per step ({args.events} events, all anchors, host noise draws included; {what}); "
              f"{len(times)} timed steps" + (" (capped by a 150 s budget)" if len(times) < args.steps else "")
              + f", {min(args.warmup, 1)} warm-up" + (f"; {note}" if note else ""))
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "events/s", "n_gpus": args.gpus,
        "steps": len(times), "warmup": min(args.warmup, 1), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "events_per_window": args.events, "device": "cpu"},
        "cpu_baseline": {"value": value, "unit": "events/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "events/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def cpu_worker(path):
    """Subprocess body of the cpu_baseline leg: time the reference (or its C port) on the saved window."""
    import torch
    d = torch.load(path)
    times, kind, note = reference_or_port(d["xy"], d["t"], d["p"], d["b"], d["flow"], steps=3, warmup=1,
                                          budget_s=25.0)
    print(json.dumps({"times": times, "kind": kind, "note": note}))


def cpu_baseline(ev, flow, n):
    """The reference's CPU path timed on this host (bounded: 1 warm-up + up to 3 steps, <= ~25 s), in a child
    process without the GPU.  A failure reports the child's own error output."""
    import torch
    cores = os.cpu_count()
    try:
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "win.pt")
            torch.save({"xy": ev.xy.cpu(), "t": ev.t.cpu(), "p": ev.p.cpu(), "b": ev.b.cpu(), "flow": flow.cpu()}, path)
            env = dict(os.environ, OMP_NUM_THREADS=str(cores or 1), CUDA_VISIBLE_DEVICES="")
            r = subprocess.run([sys.executable, __file__, "--cpu-worker", path], capture_output=True, text=True,
                               env=env, timeout=600)
    except Exception as e:
        return {"value": None, "unit": "events/s", "cores": cores, "kind": "reference",
                "sample": f"unavailable: {type(e).__name__}: {str(e)[:200]}"}
    lines = [ln for ln in r.stdout.strip().splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"value": None, "unit": "events/s", "cores": cores, "kind": "reference",
                "sample": f"unavailable: child exited {r.returncode}: {r.stderr.strip()[-300:]}"}
    d = json.loads(lines[-1])
    times, kind = d["times"], d["kind"]
    what = ("reference AnchoredExact + its OpenMP kernels" if kind == "reference"
            else "C port of the reference's CPU path")
    return {"value": n / statistics.mean(times), "unit": "events/s", "cores": cores, "kind": kind,
            "sample": f"the same 1M-event window, full fwd+bwd with the host noise draws, {len(times)} timed steps "
                      f"after 1 warm-up ({what}, {cores} threads)" + (f"; {d['note']}" if d.get("note") else "")}


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples every 20 ms while the timed region runs; ``mark()`` brackets the region and
    ``summary()`` keeps the samples whose own timestamps fall inside it (the nearest one if none does)."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc, self.path, self.gpu = None, None, gpu_index
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            deadline = time.time() + 5.0  # wait for the first sample so the region is covered
            while time.time() < deadline and os.path.getsize(self.path) == 0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def mark(self, end=False):
        if end:
            self.t1 = time.time()
        else:
            self.t0 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        import datetime
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 10:
                try:
                    ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                rows.append((ts, f[1:]))
        os.unlink(self.path)
        if not rows:
            return None
        t0 = self.t0 if self.t0 is not None else rows[0][0]
        t1 = self.t1 if self.t1 is not None else rows[-1][0]
        inside = [r for ts, r in rows if t0 <= ts <= t1]
        if not inside:
            inside = [min(rows, key=lambda x: abs(x[0] - 0.5 * (t0 + t1)))[1]]
        num = lambda v: v.replace(".", "", 1).isdigit()  # noqa: E731
        sm = [float(r[1]) for r in inside if num(r[1])]
        mx = [float(r[2]) for r in inside if num(r[2])]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in inside:
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(inside), "region_s": round(t1 - t0, 4)}


# ------------------------------------------------------------------------------------------------ ours
PROFILE_TRAFFIC = ROOT / "profiles" / "traffic.config2_1M.json"


def candidate_pairs(plan) -> int:
    """Anchor-candidate pairs the pair kernels evaluate: for every anchor, the plan entries of the 3x3 cells
    around its cell (clipped to the grid).  Every candidate runs the acceptance test and one exp2."""
    import torch
    cnt = plan.cell_start[1:] - plan.cell_start[:-1]
    g = cnt.view(-1, plan.GH, plan.GW).to(torch.float64)
    pad = torch.nn.functional.pad(g, (1, 1, 1, 1))
    nb = sum(pad[:, 1 + dy:1 + dy + plan.GH, 1 + dx:1 + dx + plan.GW] for dy in (-1, 0, 1) for dx in (-1, 0, 1))
    ac = plan.anc_cell
    return int(nb[ac[:, 0], ac[:, 2], ac[:, 1]].sum().item())


# FP32 lane operations per candidate pair, counted from the arithmetic the kernels must do for the reference's
# exactly rounded test: r = x_i - (y_j + v_j dt_i) (2 mul, 2 add, 2 sub), d^2 = rx^2 + ry^2 (2 mul, 1 add),
# the d^2 test, the exponent scale and the accumulation (forward: 12); the backward adds dt = t_i - t_j,
# gS k, (.) dt and the two gradient multiply-adds (16).  One exp2 per candidate in both.
FP32_OPS_PER_CANDIDATE = {"k_pair_fwd": 12, "k_pair_bwd": 16}


def compute_roofline(kernel, candidates, entries, alg_bytes, avg_ms, rates):
    """T_roof = max(bytes / HBM, fp32 / FP32 rate, exp2 / SFU rate, reductions / red rate) for one pair kernel,
    with the rates measured on this GPU; frac = T_roof / the kernel's CUDA-event time."""
    hbm, _ = measured_peak()
    fp32_rate = max(rates["fp32_lane_ops"], rates["fp32x2_lane_ops"])
    terms = {"hbm": alg_bytes / (hbm * 1e9), "fp32": candidates * FP32_OPS_PER_CANDIDATE[kernel] / fp32_rate,
             "sfu": candidates / rates["ex2"]}
    if kernel == "k_pair_bwd":
        terms["red"] = entries / rates["red_v4"]  # one red.global.add.v2.f32 per plan entry at most
    bound = max(terms, key=terms.get)
    t_roof = terms[bound]
    return {"bound": bound, "t_roof_ms": t_roof * 1e3, "t_measured_ms": avg_ms, "frac": t_roof / (avg_ms * 1e-3),
            "terms_ms": {k: v * 1e3 for k, v in terms.items()}, "candidates": candidates,
            "fp32_lane_ops_per_candidate": FP32_OPS_PER_CANDIDATE[kernel], "exp2_per_candidate": 1}


def profiled_traffic(kernel):
    """DRAM bytes (read + write) per launch of ``kernel`` from the ncu capture of this workload recorded in
    PROFILE_TRAFFIC (written by ``--record-traffic``), or None."""
    try:
        d = json.load(open(PROFILE_TRAFFIC))
        return int(d["kernels"][kernel]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


def record_traffic(csv_path, command):
    """Writes PROFILE_TRAFFIC from an ncu raw-page CSV export (``ncu -i <report> --page raw --csv``): per kernel
    (matched by the pair-kernel names the bench times), the mean of dram__bytes_read.sum + dram__bytes_write.sum
    over the captured launches."""
    import csv
    names = {"k_pair_fwd": "k_pair_fwd", "k_pair_bwd": "k_pair_bwd"}
    rows = list(csv.reader(open(csv_path)))
    head = rows[0]
    col = {h: i for i, h in enumerate(head)}
    units = rows[1] if len(rows) > 1 and not rows[1][col["Kernel Name"]].strip() else None
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9}
    acc = {}
    for r in rows[2 if units else 1:]:
        kname = r[col["Kernel Name"]]
        key = next((k for k, pat in names.items() if pat in kname), None)
        if key is None:
            continue
        tot = 0.0
        for m_ in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            v = float(r[col[m_]].replace(",", ""))
            tot += v * (scale.get(units[col[m_]], 1) if units else 1)
        acc.setdefault(key, []).append(tot)
    out = {"source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, mean over the captured launches",
           "command": command,
           "kernels": {k: {"dram_bytes_per_launch": int(sum(v) / len(v)), "launches": len(v)} for k, v in acc.items()}}
    PROFILE_TRAFFIC.write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out))


def measured_peak():
    try:
        d = json.load(open(ROOT / "MEASURED_PEAKS.json"))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ours_arm(args):
    import torch
    import torch.distributed as dist
    from x_b200 import _lib
    from x_b200.events import EventPacket
    from x_b200.motion import DenseLinearFlow
    from x_b200.objectives import AnchoredExact

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    ev_cpu, flow_cpu = window_data(rank, args.events)
    ev = ev_cpu.to(dev)
    m = DenseLinearFlow(1, H, W, grid=(H, W), mode="linear", init=flow_cpu).to(dev)
    obj = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=7 + rank, visibility=True,
                        fused=not args.dropin)
    anchors, u, z = obj.draw(ev)
    noise = (anchors, u, z)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step(e, nz):
        m.grid.grad = None
        out = obj(e, m, noise=nz)
        out["loss"].backward()
        return out["loss"]

    for _ in range(max(args.warmup, 3)):
        step(ev, noise)
    torch.cuda.synchronize()
    L = _lib.load_library()
    L.atlb_timing_enable(1)
    for k in ("k_pair_fwd", "k_pair_bwd"):
        _lib.timing_read(k, reset=True)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    launches0 = L.atlb_kernel_launches()
    with ClockSampler(local) as clk:
        clk.mark()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step(ev, noise)
            ends[i].record()
        torch.cuda.synchronize()
        clk.mark(end=True)
        barrier()
    launches = L.atlb_kernel_launches() - launches0
    ktime = {k: _lib.timing_read(k, reset=True) for k in ("k_pair_fwd", "k_pair_bwd")}
    L.atlb_timing_enable(0)
    clocks = clk.summary()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t)
    ms_step = total_ms / args.steps
    value = world * args.events / (ms_step / 1000)

    # ---- end to end: every step's inputs copied from pinned host memory, its loss read back.  The copies
    # go through a second stream into two device buffers, so step i+1's inputs load while step i computes;
    # the timed region is the whole job, from the first copy to the last loss read.
    # The anchors are all events (n_anchors=None): the objective builds that index on the device
    # (objectives._pick_anchors), so it is made there each step rather than copied.
    # Two pipelines: (a) the reference's noise, drawn on the host with the objective's CPU generator and
    # copied with the events (the draws themselves are timed separately: host_rng_ms); (b) device_rng, the
    # opt-in device draws inside the fused pipeline, so only the events are copied.
    obj_dev = AnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=7 + rank, visibility=True,
                            fused=not args.dropin, device_rng=True)

    def e2e_pipeline(with_noise: bool):
        keys = (("xy", ev_cpu.xy), ("t", ev_cpu.t), ("b", ev_cpu.b)) + ((("u", u.cpu()), ("z", z.cpu()))
                                                                       if with_noise else ())
        pin = {k: v.pin_memory() for k, v in keys}
        h2d = sum(v.numel() * v.element_size() for v in pin.values())
        bufs = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in pin.items()} for _ in range(2)]
        cstream = torch.cuda.Stream(device=dev)
        copied = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]
        loss_host = torch.empty(2, 1, dtype=torch.float32).pin_memory()

        def issue_copy(slot):
            with torch.cuda.stream(cstream):
                cstream.wait_event(freed[slot])  # the step that last read this buffer is done
                for k, v in pin.items():
                    bufs[slot][k].copy_(v, non_blocking=True)
                copied[slot].record(cstream)

        def one_step(d):
            e2 = EventPacket(d["xy"], d["t"], ev.p, d["b"], 1, H, W)
            if with_noise:
                return step(e2, (torch.arange(args.events, device=dev), d["u"], d["z"]))
            m.grid.grad = None
            out = obj_dev(e2, m)
            out["loss"].backward()
            return out["loss"]

        def run(nsteps):
            """nsteps end-to-end steps; returns their device time in ms (events around the whole job)."""
            for e in freed:
                e.record()
            barrier()
            torch.cuda.synchronize()
            e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e_start.record()
            cstream.wait_event(e_start)
            issue_copy(0)
            losses = []
            for i in range(nsteps):
                slot = i % 2
                torch.cuda.current_stream().wait_event(copied[slot])
                if i + 1 < nsteps:
                    issue_copy(1 - slot)
                loss = one_step(bufs[slot])
                freed[slot].record()
                # the step's loss goes to pinned host memory asynchronously and is read on the host one step
                # later, so the host enqueues step i + 1 while step i runs
                loss_host[slot].copy_(loss.detach().reshape(1), non_blocking=True)
                read[slot].record()
                if i > 0:
                    read[1 - slot].synchronize()
                    losses.append(float(loss_host[1 - slot]))
            read[(nsteps - 1) % 2].synchronize()
            losses.append(float(loss_host[(nsteps - 1) % 2]))
            e_end.record()
            torch.cuda.synchronize()
            assert len(losses) == nsteps and all(math.isfinite(v) for v in losses)
            return e_start.elapsed_time(e_end)

        run(max(args.warmup, 3))  # untimed: the pipeline's first use of its buffers
        ms = run(args.steps) / args.steps
        t_ = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        return float(t_), h2d

    e2e_ms, h2d = e2e_pipeline(True)
    e2e_dev_ms, h2d_dev = e2e_pipeline(False)
    # the reference's per-step host draws (ats.py:84-88): uniforms for every event, normals for every anchor,
    # from one CPU generator (single-threaded by construction: one sequential stream)
    gen = torch.Generator().manual_seed(7)
    for _ in range(2):
        torch.rand((args.events, 2), generator=gen); torch.randn((args.events, 2), generator=gen)
    t0 = time.perf_counter()
    nrep = 5
    for _ in range(nrep):
        torch.rand((args.events, 2), generator=gen); torch.randn((args.events, 2), generator=gen)
    host_rng_ms = 1000 * (time.perf_counter() - t0) / nrep
    strong = None if args.no_strong else strong_scaling(world, dev)
    if world > 1:
        dist.destroy_process_group()

    if rank != 0:
        return
    # ---- roofline of the dominant kernel.  Algorithmic bytes of the fused path's compact layout:
    # forward (tau covering the window): per plan entry its (y, v) float4; per anchor its (x, y, t, self)
    # record, original index and S out (ls follows in its own kernel).  Backward: per plan entry (y, v) +
    # (t, id) = 24 B; per anchor (x, y, t - c_s, t - c_s) + (dL/dS, t) = 24 B read as 20 algorithmic B;
    # per event its (gx, gy) out.
    dom = max(ktime, key=lambda k: ktime[k][0])
    dom_ms, dom_n = ktime[dom]
    with torch.no_grad():
        from x_b200 import functional as F
        xs = ev.xy + (u - 0.5)
        xa = xs[anchors] + z
        v = m.velocity(xs, ev.t, ev.b)
        plan = F.build_pair_plan(xs, ev.t, v, ev.b, 1, H, W, anchors, 1.0, 1.0, 3.0, 16, anchor_xy=xa)
        Ns, M = plan.src_y.shape[0], plan.anc_x.shape[0]
        cand = candidate_pairs(plan)
        del plan
    alg = {"k_pair_fwd": Ns * 16 + M * (16 + 4 + 4), "k_pair_bwd": Ns * 24 + M * 20 + args.events * 8}
    if args.dropin:  # the reference's plan layout: (y, v, t, int64 id) 28 B per entry, anchors bucketed 28 B
        alg = {"k_pair_fwd": Ns * 28 + M * 32, "k_pair_bwd": Ns * 28 + M * 32 + args.events * 8}
    rates = _lib.unit_rates(dev)
    compute = {k: compute_roofline(k, cand, Ns, alg[k], ktime[k][0] / max(ktime[k][1], 1), rates)
               for k in ("k_pair_fwd", "k_pair_bwd")}
    alg_bytes = alg[dom]
    avg_ms = dom_ms / max(dom_n, 1)
    peak, peak_kind = measured_peak()
    achieved = alg_bytes / (avg_ms / 1000) / 1e9
    traffic = None if args.dropin else profiled_traffic(dom)
    cores = os.cpu_count()
    cpu = None if (args.no_cpu_baseline or world > 1) else cpu_baseline(ev_cpu, flow_cpu, args.events)
    line = {
        "metric": METRIC, "value": value, "unit": "events/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD + (" [stage-by-stage drop-in ops]" if args.dropin else ""),
                   "events_per_window": args.events, "windows_per_gpu": 1,
                   "anchors_per_window": M, "plan_entries": Ns, "l2": "flushed (256 MB write) before every step",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "kernel": dom, "avg_launch_ms": avg_ms, "algorithmic_bytes": alg_bytes,
                     "peak_source": peak_kind, "traffic_source": PROFILE_TRAFFIC.name if traffic else None},
        "roofline_compute": compute,
        "unit_rates": {**{k: v for k, v in rates.items()}, "source": "atlb_measure_unit_rates on this GPU, after the timed region"},
        "kernels_ms_per_step": {k: v[0] / max(v[1], 1) for k, v in ktime.items()},
        "e2e": {"value": world * args.events / (e2e_ms / 1000), "unit": "events/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "timing": "whole job, first H2D to last loss read, after untimed warm-up steps of the same "
                          "pipeline; H2D of step i+1 overlaps step i (two buffers); every step's loss is copied "
                          "to pinned host memory and read on the host one step later (the last after the loop); "
                          "the step's noise (the reference's host draws) is copied with the events, its drawing "
                          "is host_rng_ms",
                "host_rng_ms": host_rng_ms,
                "host_rng": "the reference's per-step draws on the host (torch CPU generator: (N,2) uniforms + "
                            "(M,2) normals), not in value: a caller that draws them serially per step adds them"},
        "e2e_device_rng": {"value": world * args.events / (e2e_dev_ms / 1000), "unit": "events/s",
                           "ms_per_step": e2e_dev_ms, "h2d_bytes_per_step": h2d_dev, "d2h_bytes_per_step": 4,
                           "timing": "as e2e, with AnchoredExact(device_rng=True): the noise is drawn on the device "
                                     "inside the fused pipeline (opt-in; another stream than the reference's), so "
                                     "only the events are copied"},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if strong is not None:
        line["strong_scaling"] = strong
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------ strong scaling
def _timed_steps(step, steps, warmup, world, dev):
    """Device ms per step (CUDA events around each step, summed; max over ranks), after untimed warm-up."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    tot = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(starts, ends))], device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    return float(tot) / steps


def strong_scaling(world: int, dev, steps: int = 3, warmup: int = 3) -> dict:
    """The two sharded workloads at this run's number of GPUs (total work fixed as N grows):
    configuration 5a, one 64M-event window on 1280x720 under AnchoredExact + DenseLinearFlow, sources split
    across the ranks (NCCL all-reduce of the M partial sums and of the flow gradient); and configuration 3,
    AnchoredSliced + Bezier PixelTrajectories on 8 x 2M events, events split across the ranks (NCCL
    all-reduce of the slices x 8 x 480 x 640 density stack, its gradient, the counts and the coefficient
    gradient).  The windows are drawn on the device (seeded, identical on every rank)."""
    import torch
    from x_b200 import synth
    from x_b200.distributed import ShardedAnchoredExact, ShardedAnchoredSliced
    from x_b200.motion import DenseLinearFlow, PixelTrajectories
    out = {}
    # configuration 5a
    n5, H5, W5 = 64_000_000, 720, 1280
    ev = synth.textured_window(n5, H5, W5, duration=0.2, seed=5000, device=dev, draw_on_device=True)
    flow = synth.lowpass_flow(1, H5, W5, sigma=32.0, vmax=20.0, seed=5001).to(dev)
    m = DenseLinearFlow(1, H5, W5, grid=(H5, W5), mode="linear", init=flow).to(dev)
    obj = ShardedAnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=5002, visibility=True)
    noise = obj.draw(ev)

    def step5():
        m.grid.grad = None
        ls, _ = obj.log_scores(ev, m, noise=noise)
        (-ls.mean()).backward()

    ms = _timed_steps(step5, steps, warmup, world, dev)
    out["config5a"] = {"value": n5 / (ms / 1000), "unit": "events/s", "ms_per_step": ms, "n_gpus": world,
                       "steps": steps, "warmup": warmup, "events": n5,
                       "workload": "one 64M-event window, 1280x720, AnchoredExact(h=1, tau=1, all anchors, 16 slices, "
                                   "visibility) + DenseLinearFlow, fwd+bwd; sources split across the ranks"}
    del ev, m, obj, noise, flow
    torch.cuda.empty_cache()
    # configuration 3
    B3, n3, K = 8, 2_000_000, 10
    ev = synth.textured_window(n3, H, W, duration=0.1, seed=3100, batch=B3, device=dev, draw_on_device=True)
    g = torch.Generator(device=dev).manual_seed(3101)
    raw = torch.nn.functional.avg_pool2d(torch.randn(B3, 2 * K, H, W, generator=g, device=dev), 17, 1, 8)
    coeff = (raw / raw.abs().amax() * 15.0 / K).requires_grad_(True)
    mt = PixelTrajectories(coeff, K, basis_kind="bezier", tile=4)
    obj3 = ShardedAnchoredSliced(n_slices=10, sigma=1.5, seed=3102)
    noise3 = obj3.draw(ev)

    def step3():
        coeff.grad = None
        obj3(ev, mt, noise=noise3)["loss"].backward()
        obj3.reduce_gradients([coeff])

    ms = _timed_steps(step3, steps, warmup, world, dev)
    out["config3"] = {"value": B3 * n3 / (ms / 1000), "unit": "events/s", "ms_per_step": ms, "n_gpus": world,
                      "steps": steps, "warmup": warmup, "events": B3 * n3,
                      "workload": "AnchoredSliced(10 slices, sigma 1.5) + PixelTrajectories(K=10 Bezier, tile 4), "
                                  "8 x 2M events on 640x480, fwd+bwd; events split across the ranks"}
    del ev, mt, obj3, noise3, coeff
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------------ config 5
def config5_arm(args):
    """One window of --events (default 64M) events on 1280x720 (times over 200 ms, dense flow as in
    configuration 2), sources split across the ranks (x_b200.distributed): strong scaling."""
    import torch
    import torch.distributed as dist
    from x_b200 import _lib, synth
    from x_b200.distributed import ShardedAnchoredExact
    from x_b200.events import EventPacket
    from x_b200.motion import DenseLinearFlow

    H5, W5 = 720, 1280
    n = args.events if args.events != N_EVENTS else 64_000_000
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    ev_cpu = synth.textured_window(n, H5, W5, duration=0.2, seed=5000)   # the same window on every rank
    flow = synth.lowpass_flow(1, H5, W5, sigma=32.0, vmax=20.0, seed=5001)
    ev = ev_cpu.to(dev)
    m = DenseLinearFlow(1, H5, W5, grid=(H5, W5), mode="linear", init=flow).to(dev)
    obj = ShardedAnchoredExact(h=1.0, tau=1.0, n_anchors=None, n_slices=16, seed=5002, visibility=True)
    noise = obj.draw(ev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def step():
        m.grid.grad = None
        ls, _ = obj.log_scores(ev, m, noise=noise)
        loss = -ls.mean()
        loss.backward()
        return loss

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    L = _lib.load_library()
    L.atlb_timing_enable(1)
    for k in ("k_pair_fwd", "k_pair_bwd"):
        _lib.timing_read(k, reset=True)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    launches0 = L.atlb_kernel_launches()
    with ClockSampler(local) as clk:
        clk.mark()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
        clk.mark(end=True)
        barrier()
    launches = L.atlb_kernel_launches() - launches0
    ktime = {k: _lib.timing_read(k, reset=True) for k in ("k_pair_fwd", "k_pair_bwd")}
    L.atlb_timing_enable(0)
    clocks = clk.summary()
    total = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(starts, ends))], device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
        dist.destroy_process_group()
    ms_step = float(total) / args.steps
    if rank != 0:
        return
    dom = max(ktime, key=lambda k: ktime[k][0])
    dom_ms = ktime[dom][0] / max(ktime[dom][1], 1)
    ns = n // world
    alg = {"k_pair_fwd": ns * 16 * 16 + n * 36, "k_pair_bwd": ns * 16 * 24 + n * 20 + ns * 8}[dom]  # 16 slices, tau = 1
    peak, peak_kind = measured_peak()
    achieved = alg / (dom_ms / 1000) / 1e9
    print(json.dumps({
        "metric": METRIC, "value": n / (ms_step / 1000), "unit": "events/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config5a: one {n}-event window on 1280x720, AnchoredExact(h=1, tau=1, all anchors, "
                               "16 slices, visibility) + DenseLinearFlow(2x720x1280), sources split across ranks",
                   "events_per_window": n, "windows": 1, "l2": "flushed (256 MB write) before every step",
                   "parallelism": f"source shards x{world}, NCCL all-reduce of S (M floats) and of the flow grad"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": dom, "avg_launch_ms": dom_ms, "algorithmic_bytes": alg,
                     "peak_source": peak_kind},
        "kernels_ms_per_step": {k: v[0] / max(v[1], 1) for k, v in ktime.items()},
        "gpu_launches": int(launches), "clocks": clocks,
    }))


# ------------------------------------------------------------------------------------------------ splat
def splat_arm(args):
    """The sliced path's Gaussian splat (configuration 3: --windows windows of --events events on 640x480,
    sigma = 1.5, R = 5, weight 1), forward + backward of one slice on one GPU: taps/s."""
    import torch
    from x_b200 import _lib, get_ext, synth
    n = args.events if args.events != N_EVENTS else 2_000_000
    B, sigma = args.windows, 1.5
    R = int(math.ceil(3 * sigma))
    ev = synth.textured_window(n, H, W, duration=0.1, seed=3000, batch=B)
    g = torch.Generator().manual_seed(3001)
    pos = (ev.xy + (torch.rand(ev.xy.shape, generator=g) - 0.5)).cuda()
    w = torch.ones(pos.shape[0], device="cuda")
    b = ev.b.cuda()
    gimg = torch.randn(B, H, W, generator=g).cuda()
    ext = get_ext()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def step():
        img = ext.splat_gauss_fwd(pos, w, b, B, H, W, sigma, R)
        gp, gw = ext.splat_gauss_bwd(gimg, pos, w, b, sigma, R)
        return img, gp, gw

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    L = _lib.load_library()
    L.atlb_timing_enable(1)
    for k in ("k_gsplat_fwd", "k_gsplat_bwd"):
        _lib.timing_read(k, reset=True)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches0 = L.atlb_kernel_launches()
    with ClockSampler(0) as clk:
        clk.mark()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
        clk.mark(end=True)
    launches = L.atlb_kernel_launches() - launches0
    kt = {k: _lib.timing_read(k, reset=True) for k in ("k_gsplat_fwd", "k_gsplat_bwd")}
    L.atlb_timing_enable(0)
    ms = sum(a.elapsed_time(e) for a, e in zip(starts, ends)) / args.steps
    taps = pos.shape[0] * (2 * R + 1) ** 2
    print(json.dumps({
        "metric": "Gaussian splat fwd+bwd taps/s (configuration 3, one slice)", "value": taps / (ms / 1000),
        "unit": "taps/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"splat: {B} windows x {n} events, 640x480, sigma {sigma}, R {R}", "taps": taps},
        "kernels_ms_per_step": {k: v[0] / max(v[1], 1) for k, v in kt.items()},
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }))


# ------------------------------------------------------------------------------------------------ tiled ops
def tiles_arm(args):
    """The tiled bilinear ops on a configuration-2-sized input (--windows windows of --events points on
    640x480, weights 1): bilinear splat forward + backward, bilinear gather forward + backward (the image
    tiles staged by TMA), and the 5-bin voxel grid.  value = points per second through all five ops."""
    import torch
    from x_b200 import _lib, get_ext, synth
    n = args.events
    B, C = args.windows if args.windows != 8 else 1, 5
    ev = synth.textured_window(n, H, W, duration=0.1, seed=4000, batch=B)
    g = torch.Generator().manual_seed(4001)
    pos = (ev.xy + (torch.rand(ev.xy.shape, generator=g) - 0.5)).cuda()
    w = torch.ones(pos.shape[0], device="cuda")
    b, t, p = ev.b.cuda(), ev.t.cuda(), ev.p.cuda()
    img = torch.randn(B, H, W, generator=g).cuda()
    gval = torch.randn(pos.shape[0], generator=g).cuda()
    ext = get_ext()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ops = {
        "splat_bilinear_fwd": lambda: ext.splat_bilinear_fwd(pos, w, b, B, H, W),
        "splat_bilinear_bwd": lambda: ext.splat_bilinear_bwd(img, pos, w, b),
        "gather_bilinear_fwd": lambda: ext.gather_bilinear_fwd(img, pos, b),
        "gather_bilinear_bwd": lambda: ext.gather_bilinear_bwd(gval, img, pos, b),
        "voxel_grid": lambda: ext.voxel_grid(pos, t, p, b, B, C, H, W),
    }
    # algorithmic bytes per point: positions 8, batch index 8, plus weight / value / time / polarity 4 each and
    # the per-point outputs; the images are L2-resident (one read or write of B x H x W floats per call)
    per_pt = {"splat_bilinear_fwd": 20, "splat_bilinear_bwd": 20 + 12, "gather_bilinear_fwd": 16 + 4,
              "gather_bilinear_bwd": 20 + 8, "voxel_grid": 24}
    for _ in range(max(args.warmup, 3)):
        for f in ops.values():
            f()
    torch.cuda.synchronize()
    L = _lib.load_library()
    launches0 = L.atlb_kernel_launches()
    per_op = {k: 0.0 for k in ops}
    with ClockSampler(0) as clk:
        clk.mark()
        for i in range(args.steps):
            for k, f in ops.items():
                flush.zero_()
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                f()
                e.record()
                e.synchronize()
                per_op[k] += a.elapsed_time(e)
        clk.mark(end=True)
    launches = L.atlb_kernel_launches() - launches0
    per_op = {k: v / args.steps for k, v in per_op.items()}
    ms = sum(per_op.values())
    npts = pos.shape[0]
    peak, peak_kind = measured_peak()
    print(json.dumps({
        "metric": "tiled bilinear ops (splat fwd+bwd, gather fwd+bwd, voxel grid) points/s", "value": npts / (ms / 1000),
        "unit": "points/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"tiles: {B} window(s) x {n} points, 640x480, voxel bins {C}",
                   "l2": "flushed (256 MB write) before every op"},
        "ops_ms": per_op,
        "ops_gbs_of_algorithmic_bytes": {k: npts * per_pt[k] / (v / 1000) / 1e9 for k, v in per_op.items()},
        "hbm_peak_gbs": peak, "peak_source": peak_kind,
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }))


# ------------------------------------------------------------------------------------------------ config 3
def config3_arm(args):
    """Configuration 3: AnchoredSliced(n_slices=10, sigma=1.5) + Bezier PixelTrajectories (K = 10 control
    displacements on the 160x120 tile grid, random smooth, |disp| <= 15 px) over --windows windows of --events
    events on 640x480, forward + backward to the coefficient grid, one GPU."""
    import torch
    from x_b200 import _lib, synth
    from x_b200.motion import PixelTrajectories
    from x_b200.objectives import AnchoredSliced
    n = args.events if args.events != N_EVENTS else 2_000_000
    B, K = args.windows, 10
    ev = synth.textured_window(n, H, W, duration=0.1, seed=3100, batch=B).to("cuda")
    g = torch.Generator().manual_seed(3101)
    raw = torch.nn.functional.avg_pool2d(torch.randn(B, 2 * K, H, W, generator=g), 17, 1, 8)
    coeff = (raw / raw.abs().amax() * 15.0 / K).cuda().requires_grad_(True)  # sum_k |c_k| g_k <= 15 px
    m = PixelTrajectories(coeff, K, basis_kind="bezier", tile=4)
    obj = AnchoredSliced(n_slices=10, sigma=1.5, seed=3102)
    noise = obj.draw(ev)  # the reference's CPU-generator draws, once (as for configuration 2)

    def step():
        coeff.grad = None
        ls, _ = obj.log_scores(ev, m, noise=noise)
        loss = -ls.mean()
        loss.backward()
        return loss

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    L = _lib.load_library()
    L.atlb_timing_enable(1)
    names = ("k_gsplat_fwd", "k_gsplat_bwd", "k_traj_fwd", "k_traj_bwd", "k_traj_records_fwd", "k_traj_records_bwd",
             "k_traj_targets_fwd", "k_traj_targets_bwd", "k_traj_vis")
    for k in names:
        _lib.timing_read(k, reset=True)
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = L.atlb_kernel_launches()
    with ClockSampler(0) as clk:
        clk.mark()
        s_ev.record()
        for _ in range(args.steps):
            step()
        e_ev.record()
        torch.cuda.synchronize()
        clk.mark(end=True)
    launches = L.atlb_kernel_launches() - launches0
    kt = {k: _lib.timing_read(k, reset=True) for k in names}
    L.atlb_timing_enable(0)
    ms = s_ev.elapsed_time(e_ev) / args.steps
    print(json.dumps({
        "metric": "anchored-score (sliced) fwd+bwd events/s, configuration 3", "value": B * n / (ms / 1000),
        "unit": "events/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config3: AnchoredSliced(10 slices, sigma 1.5) + PixelTrajectories(K=10 Bezier, tile 4) "
                               f"on {B} x {n} events, 640x480", "events": B * n},
        "kernels_ms_per_step": {k: v[0] / args.steps for k, v in kt.items()},
        "gpu_launches": int(launches), "clocks": clk.summary(),
    }))


def main():
    args = parse()
    if args.cpu_worker:
        cpu_worker(args.cpu_worker)
        return
    if args.record_traffic:
        record_traffic(*args.record_traffic)
        return
    if args.impl == "reference":
        reference_arm(args)
    elif args.workload == "config5":
        config5_arm(args)
    elif args.workload == "splat":
        splat_arm(args)
    elif args.workload == "tiles":
        tiles_arm(args)
    elif args.workload == "config3":
        config3_arm(args)
    else:
        ours_arm(args)


if __name__ == "__main__":
    main()
