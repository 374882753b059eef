#!/usr/bin/env python
"""Benchmark of the B200 flash-Sinkhorn path (one JSON line on rank 0).

On one GPU a step is one forward + IFT backward of flash-Sinkhorn attention at
B=2, H=8, N=384, d=32 (the configuration the headline metric is quoted on):
bf16 Q/K/V ~ N(0,1), eps=1, 20 iterations, uniform marginals, upstream
dO ~ N(0,1), CG tol 1e-6 / max 50 / zero start.  The line also carries a
single-GPU measurement of the long-sequence workload below (``config4_1gpu``),
the N = 1 point of its strong-scaling curve.

On N > 1 GPUs (torchrun, one rank per GPU) the default workload is the
long-sequence row-sharded one: B=1 H=16 N=8192 d=64, 30 iterations, CG tol
1e-5 / max 40, every problem's rows split over the ranks, potentials exchanged
through NVLink peer stores each half-iteration (strong scaling: one call is the
whole configuration's forward + backward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|triton]
                    [--config 2|3|4|transport|dense]

``--config 3`` (B=8 H=16 padded N=1024 d=64, variable lengths, softmax
marginals, eps 0.5, 50 iterations) spreads the (batch, head) problems over the
ranks with a length^2-balanced partition (no data-path collective).

``--config transport`` times the trunk block's balanced transport
(balanced_sinkhorn_transport, fwd+bwd) at the shapes the reference publishes
timings for (B=1 H=16 d_h=32 K=20, N = 64 ... 768) and prints them beside those.

``--config dense`` times the dense-cost entry points beyond the resident range
(sinkhorn_solve + compute_transport_output on a given 1 GiB fp32 cost, B=1 H=16
N=4096) against the measured HBM bandwidth.

``--impl reference`` times the reference's own CPU path -- dense cost, its
``sinkhorn_solve`` and ``compute_transport_output``, torch autograd -- from the
reference package pip-installed into ``baseline/_ref`` (restated in
``oracle/sinkhorn_torch.py`` where that install is absent), in float32 on all
host threads, on the same workload, and prints the same metric.

``--impl triton`` times the reference's own GPU path (``flash_sinkhorn``,
Triton forward and unrolled Triton backward, from ``baseline/_ref``) on this
GPU on config 2 or 3: the GPU bar, not one of the driver's arms.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "deepfold-linear_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "Sinkhorn attn fwd+IFT-bwd calls/sec & TFLOP/s vs bf16 peak, 1/2/4/8 B200"
UNIT = "calls/s"
CFG = dict(B=2, H=8, N=384, d=32, eps=1.0, K_iter=20, cg_rtol=1e-6, cg_max_iter=50)
L2_FLUSH_BYTES = 256 << 20       # > 126 MB L2: written between timed steps


def quiet_gc():
    """Collect once and move every object alive now out of the collector's view
    (gc.freeze): a full cyclic collection over the interpreter's heap (torch's
    objects included) pauses the host for tens of milliseconds, and on several
    GPUs the other ranks wait for the paused one inside the next collective.
    Called after set-up and warm-up, before any timed region."""
    import gc
    gc.collect()
    gc.freeze()


def workload_name():
    c = CFG
    return (f"config2: flash-Sinkhorn fwd+IFT-bwd B={c['B']} H={c['H']} N={c['N']} d={c['d']} bf16 "
            f"eps={c['eps']} K={c['K_iter']} uniform marginals, CG tol {c['cg_rtol']} max {c['cg_max_iter']}")


def flops_per_call(n_cg_mean):
    """Algorithmic flops (recompute included) of one fwd and one bwd call."""
    c = CFG
    per = c["N"] ** 2 * c["d"] * c["B"] * c["H"]
    fwd = (4 * c["K_iter"] + 4) * per
    bwd = (14 + 2 * n_cg_mean) * per
    useful = 4 * per
    return fwd, bwd, useful


class CopyPipeline:
    """Host<->device copies of an end-to-end loop, overlapped with the compute of
    the neighbouring steps: the inputs of step i+1 are copied in on a side stream
    while step i computes (two device input buffers), and the results of step i
    are read back on the side stream while step i+1 computes.  Every step still
    copies its own inputs in from pinned host memory and its own results out
    inside the timed region (the end event waits for the last read-back)."""

    def __init__(self, host: dict, device, compute):
        self.host, self.compute = host, compute
        self.side = torch.cuda.Stream(device)
        self.bufs = [{k: torch.empty(v.shape, dtype=v.dtype, device=device) for k, v in host.items()}
                     for _ in range(2)]
        self.loaded = [torch.cuda.Event() for _ in range(2)]
        self.freed = [None, None]
        self.outs = [None, None]

    def start(self):
        """Call after recording the start event: the first inputs go in behind it."""
        self.side.wait_stream(self.compute)
        self.prefetch(0)

    def prefetch(self, i):
        b = i % 2
        with torch.cuda.stream(self.side):
            if self.freed[b] is not None:
                self.side.wait_event(self.freed[b])
            for k, v in self.host.items():
                self.bufs[b][k].copy_(v, non_blocking=True)
            self.loaded[b].record(self.side)

    def inputs(self, i):
        self.compute.wait_event(self.loaded[i % 2])
        return self.bufs[i % 2]

    def finish_step(self, i, results):
        """Step i's compute is queued: release its input buffer and read its results back."""
        b = i % 2
        done = torch.cuda.Event()
        done.record(self.compute)
        self.freed[b] = done
        if self.outs[b] is None:
            self.outs[b] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in results]
        self.side.wait_event(done)
        with torch.cuda.stream(self.side):
            for o, r in zip(self.outs[b], results):
                r.record_stream(self.side)
                o.copy_(r, non_blocking=True)
        return sum(o.numel() * o.element_size() for o in self.outs[b])

    def end(self):
        self.compute.wait_stream(self.side)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "resident_bwd_config2.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("dram_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


def gpu_bus_id(dev) -> str:
    """PCI bus id of a torch device, in nvidia-smi's form: nvidia-smi counts GPUs by
    physical index and ignores CUDA_VISIBLE_DEVICES, so the torch index can name
    another GPU; the bus id cannot."""
    p = torch.cuda.get_device_properties(dev)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region, of the GPU
    this process runs on (selected by PCI bus id)."""

    def __init__(self, dev):
        index = dev.index
        self.index = index
        self.bus_id = gpu_bus_id(dev)
        self.proc = None
        # the raw samples go where DFS_CLOCK_LOG_DIR points (kept for inspection), else to a temp file
        log_dir = os.environ.get("DFS_CLOCK_LOG_DIR")
        self.path = (os.path.join(log_dir, f"clocks_rank{index}.csv") if log_dir
                     else f"/tmp/dfs_clocks_{os.getpid()}_{index}.csv")

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", self.bus_id, "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "gpu_pci_bus_id": self.bus_id}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def make_shard(dev, seed):
    c = CFG
    g = torch.Generator().manual_seed(seed)
    B, H, N, d = c["B"], c["H"], c["N"], c["d"]
    host = dict(
        Q=torch.randn(B, H, N, d, generator=g).to(torch.bfloat16),
        K=torch.randn(B, H, N, d, generator=g).to(torch.bfloat16),
        V=torch.randn(B, H, N, d, generator=g).to(torch.bfloat16),
        dO=torch.randn(B, H, N, d, generator=g).to(torch.bfloat16),
    )
    host = {k: v.pin_memory() for k, v in host.items()}
    eps = torch.full((H,), c["eps"], device=dev)
    lm = torch.full((B, H, N), -math.log(N), device=dev)
    return host, eps, lm


def run_ours(args):
    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    from deepfold import _native as nat
    from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn

    nat.lib()
    c = CFG
    host, eps, lm = make_shard(dev, 1000 + rank)
    dQKV = {k: host[k].to(dev) for k in host}
    cg = dict(rtol=c["cg_rtol"], atol=0.0, max_iter=c["cg_max_iter"])
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step_resident():
        Q = dQKV["Q"].requires_grad_(True)
        K = dQKV["K"].requires_grad_(True)
        V = dQKV["V"].requires_grad_(True)
        O, _, _, _ = flash_sinkhorn(Q, K, V, None, None, None, eps, None, lm, lm, K_iter=c["K_iter"],
                                    lam=float("inf"), cg_opts=cg)
        dQ, dK, dV = torch.autograd.grad(O, (Q, K, V), grad_outputs=dQKV["dO"].float())
        return dQ, dK, dV

    # Device-time path: the two C-ABI launches back to back on pre-allocated
    # buffers (the same kernels the autograd path runs), so host overhead never
    # leaves the GPU idle inside the events.
    B, H, N, d = c["B"], c["H"], c["N"], c["d"]
    f32 = dict(device=dev, dtype=torch.float32)
    O = torch.empty(B, H, N, d, **f32)
    lu, lv = torch.empty(B, H, N, **f32), torch.empty(B, H, N, **f32)
    dO32 = dQKV["dO"].float()
    grads = [torch.empty(B, H, N, d, **f32) for _ in range(3)]
    iters = torch.empty(B * H, device=dev, dtype=torch.int32)
    resid = torch.empty(B * H, **f32)
    st_f, st_b = torch.zeros(1, device=dev, dtype=torch.int32), torch.zeros(1, device=dev, dtype=torch.int32)
    prob = nat.make_problem(B, H, N, d, torch.bfloat16, c["K_iter"], float("inf"), 10.0)
    fargs = nat.DfsFwdArgs(Q=dQKV["Q"].data_ptr(), K=dQKV["K"].data_ptr(), V=dQKV["V"].data_ptr(),
                           eps=eps.data_ptr(), log_mu=lm.data_ptr(), log_nu=lm.data_ptr(), O=O.data_ptr(),
                           log_u=lu.data_ptr(), log_v=lv.data_ptr(), status=st_f.data_ptr())
    cgp = nat.DfsCgParams(rtol=c["cg_rtol"], atol=0.0, max_iter=c["cg_max_iter"], reserved=0)
    bargs = nat.DfsBwdArgs(Q=dQKV["Q"].data_ptr(), K=dQKV["K"].data_ptr(), V=dQKV["V"].data_ptr(),
                           eps=eps.data_ptr(), log_mu=lm.data_ptr(), log_nu=lm.data_ptr(), log_u=lu.data_ptr(),
                           log_v=lv.data_ptr(), dO=dO32.data_ptr(), dQ=grads[0].data_ptr(),
                           dK=grads[1].data_ptr(), dV=grads[2].data_ptr(), cg_iters=iters.data_ptr(),
                           cg_residual=resid.data_ptr(), status=st_b.data_ptr())
    L = nat.lib()
    sp = stream.cuda_stream
    fwd_ms, bwd_ms = [], []

    def step_kernels():
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        nat.check(L.dfs_fwd(prob, fargs, None, 0, sp), "dfs_fwd")
        e1.record(stream)
        nat.check(L.dfs_bwd(prob, cgp, bargs, None, 0, sp), "dfs_bwd")
        e2.record(stream)
        return e0, e1, e2

    # the clock sampler starts before the warm-up (nvidia-smi's start-up stays out of the timed steps)
    sampler = ClockSampler(dev) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(args.warmup):
        step_resident()
        step_kernels()
    torch.cuda.synchronize()
    quiet_gc()

    # ---- timed region: value (inputs resident in HBM, L2 flushed between steps)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs = []
    for _ in range(args.steps):
        flush.fill_(1)
        evs.append(step_kernels())
    torch.cuda.synchronize()
    for e0, e1, e2 in evs:
        fwd_ms.append(e0.elapsed_time(e1))
        bwd_ms.append(e1.elapsed_time(e2))
    step_ms = [f + b for f, b in zip(fwd_ms, bwd_ms)]
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    n_cg = float(iters.float().mean().item())
    status = int(st_f.item()) | int(st_b.item())

    # ---- e2e: public API, host buffers, H2D inputs + D2H gradients inside the timed region.
    # The step's inputs Q, K, V, dO sit in one pinned block and go in with one copy,
    # on a side stream while the previous step computes (two device buffers); the
    # three gradients (one buffer: the op casts them together) come back with one
    # copy on a second side stream while the next step computes.  Every step
    # copies its own inputs in and its own results out inside the timed region.
    hblock = torch.stack([host[k] for k in ("Q", "K", "V", "dO")]).pin_memory()
    dbufs = [torch.empty(hblock.shape, dtype=hblock.dtype, device=dev) for _ in range(2)]
    gshape = (3, B, H, N, d)
    gout = [torch.empty(gshape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    side_in, side_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    h2d = hblock.numel() * hblock.element_size()
    d2h = gout[0].numel() * gout[0].element_size()

    def copy_in(b, after=None):
        with torch.cuda.stream(side_in):
            if after is not None:
                side_in.wait_event(after)  # the step that read this buffer has finished
            dbufs[b].copy_(hblock, non_blocking=True)
            ev_in[b].record(side_in)

    def e2e_loop(n):
        side_in.wait_stream(stream)
        copy_in(0)
        for i in range(n):
            b = i % 2
            stream.wait_event(ev_in[b])
            if i + 1 < n:
                copy_in(1 - b, ev_done[1 - b] if i >= 1 else None)
            x = dbufs[b]
            Q = x[0].detach().requires_grad_(True)
            K = x[1].detach().requires_grad_(True)
            V = x[2].detach().requires_grad_(True)
            O, _, _, _ = flash_sinkhorn(Q, K, V, None, None, None, eps, None, lm, lm, K_iter=c["K_iter"],
                                        lam=float("inf"), cg_opts=cg)
            gq, gk, gv = torch.autograd.grad(O, (Q, K, V), grad_outputs=x[3])
            ev_done[b].record(stream)
            base = gq._base
            fused = (base is not None and tuple(base.shape) == gshape and base.dtype == torch.bfloat16
                     and gq.data_ptr() == base.data_ptr() and gk.data_ptr() == base[1].data_ptr()
                     and gv.data_ptr() == base[2].data_ptr())
            with torch.cuda.stream(side_out):
                side_out.wait_event(ev_done[b])
                if fused:
                    base.record_stream(side_out)
                    gout[b].copy_(base, non_blocking=True)
                else:
                    for k, t in enumerate((gq, gk, gv)):
                        t.record_stream(side_out)
                        gout[b][k].copy_(t, non_blocking=True)
        stream.wait_stream(side_out)
        stream.wait_stream(side_in)

    e2e_loop(max(args.warmup, 2))
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ee0.record(stream)
    e2e_loop(args.steps)
    ee1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ee0.elapsed_time(ee1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    clocks = sampler.stop() if sampler else None

    if rank == 0:
        peak, _, peak_src = load_peaks()
        f_fwd, f_bwd, useful = flops_per_call(n_cg)
        mf, mb = statistics.mean(fwd_ms), statistics.mean(bwd_ms)
        dom_name, dom_ms, dom_flops = ("resident_bwd_kernel", mb, f_bwd) if mb >= mf else \
            ("resident_fwd_kernel", mf, f_fwd)
        achieved = dom_flops / (dom_ms * 1e-3) / 1e12
        calls = world * args.steps
        value = calls / (total_ms * 1e-3)
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) Q/K/V/dO; B=2 H=8 N=384 d=32)",
            "config": {"workload": workload_name(), "global_batch": CFG["B"] * world,
                       "heads": CFG["H"], "seq_len": CFG["N"], "head_dim": CFG["d"],
                       "parallelism": f"(batch,head)-shard x{world}",
                       "l2": "flushed between timed steps (256 MB write, outside the step events)"},
            "tflops": {"algorithmic_per_call": round((f_fwd + f_bwd) / 1e12, 6),
                       "achieved": round((f_fwd + f_bwd) * calls / (total_ms * 1e-3) / 1e12, 3),
                       "useful_flops_per_call": useful, "cg_iters_mean": n_cg,
                       "frac_of_bf16_peak": round((f_fwd + f_bwd) * calls / (total_ms * 1e-3) / 1e12 / peak, 5)},
            "kernels_ms": {"resident_fwd_kernel": round(mf, 5), "resident_bwd_kernel": round(mb, 5)},
            "roofline": {"bound": "tensor", "kernel": dom_name, "achieved": round(achieved, 3),
                         "peak": peak, "peak_source": peak_src, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 5), "traffic": profile_traffic()},
            "e2e": {"value": round(world * args.steps / (e2e_ms * 1e-3), 3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": 2 * args.steps,
            "device_status": status,
            "clocks": clocks,
        }
        if world == 1 and not args.no_config4:
            line["config4_1gpu"] = config4_single_gpu(dev)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(2, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------- configs 3 and 4
BIG = {
    3: dict(B=8, H=16, N=1024, d=64, eps=0.5, K_iter=50, lam=float("inf"), cg_rtol=1e-6, cg_max_iter=50,
            varlen=True),
    4: dict(B=1, H=16, N=8192, d=64, eps=1.0, K_iter=30, lam=float("inf"), cg_rtol=1e-5, cg_max_iter=40,
            varlen=False),
}


def config4_single_gpu(dev, steps=5, warmup=3):
    """The long-sequence workload (B=1 H=16 N=8192 d=64, fwd + bwd) on this one GPU
    through the public op: the N = 1 point of the row-sharded strong-scaling runs
    (bench.py --gpus N > 1).  Inputs resident, CUDA events around `steps` calls."""
    from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn, last_cg_report
    c = BIG[4]
    host, _, _, lmu, lnu = big_inputs(c)
    inp = {k: v.to(dev) for k, v in host.items()}
    eps = torch.full((c["H"],), c["eps"], device=dev)
    lmu, lnu = lmu.to(dev), lnu.to(dev)
    cg = dict(rtol=c["cg_rtol"], atol=0.0, max_iter=c["cg_max_iter"])

    def step():
        leaves = [inp[k].requires_grad_(True) for k in ("Q", "K", "V")]
        O, _, _, _ = flash_sinkhorn(*leaves, None, None, None, eps, None, lmu, lnu, K_iter=c["K_iter"], lam=c["lam"],
                                    cg_opts=cg)
        torch.autograd.grad(O, leaves, grad_outputs=inp["dO"].float())

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    quiet_gc()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    rep = last_cg_report()
    return {"workload": big_workload_name(4), "value": round(1e3 / ms, 4), "unit": UNIT,
            "ms_per_step": round(ms, 4), "steps": steps, "warmup": warmup,
            "cg_iters_mean": float(rep["cg_iters"].float().mean()) if rep else None}


def big_workload_name(cfg_id):
    c = BIG[cfg_id]
    return (f"config{cfg_id}: flash-Sinkhorn fwd+IFT-bwd B={c['B']} H={c['H']} N={c['N']} d={c['d']} bf16 "
            f"eps={c['eps']} K={c['K_iter']} " +
            ("padded var-len, softmax marginals, balanced" if c["varlen"] else "uniform marginals, balanced") +
            f", CG tol {c['cg_rtol']} max {c['cg_max_iter']}")


def big_inputs(c, seed=0):
    """Seeded host inputs of config 3 / 4 (identical on every rank)."""
    g = torch.Generator().manual_seed(seed)
    B, H, N, d = c["B"], c["H"], c["N"], c["d"]
    host = {k: torch.randn(B, H, N, d, generator=g).to(torch.bfloat16) for k in ("Q", "K", "V", "dO")}
    if c["varlen"]:
        lengths = torch.randint(64, N + 1, (B,), generator=g)
        mask = (torch.arange(N)[None, :] < lengths[:, None]).float()
        lms = []
        for _ in range(2):
            z = torch.randn(B, H, N, generator=g)
            z = torch.where(mask[:, None, :] > 0, z, torch.full_like(z, -1e30))
            lms.append(torch.where(mask[:, None, :] > 0, torch.log_softmax(z, -1), torch.full_like(z, -1e9)))
        lmu, lnu = lms
    else:
        lengths = torch.full((B,), N)
        mask = None
        lmu = torch.full((B, H, N), -math.log(N))
        lnu = lmu.clone()
    return host, [int(x) for x in lengths], mask, lmu, lnu


def run_big(args):
    from deepfold.model.kernels.sinkhorn_bhshard import bh_sharded_flash_sinkhorn
    from deepfold.model.kernels.sinkhorn_kernel import last_cg_report
    from deepfold.model.kernels.sinkhorn_rowshard import last_rowshard_report, row_range, \
        row_sharded_flash_sinkhorn

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    c = BIG[args.config]
    B, H, N, d = c["B"], c["H"], c["N"], c["d"]
    host, lengths, mask, lmu, lnu = big_inputs(c)
    host = {k: v.pin_memory() for k, v in host.items()}
    eps = torch.full((H,), c["eps"], device=dev)
    mask_d = None if mask is None else mask.to(dev)
    lmu_d, lnu_d = lmu.to(dev), lnu.to(dev)
    cg = dict(rtol=c["cg_rtol"], atol=0.0, max_iter=c["cg_max_iter"])
    r0, r1, _ = row_range(N, world, rank)

    def step(inp):
        leaves = [inp[k].requires_grad_(True) for k in ("Q", "K", "V")]
        if args.config == 4:
            O, _, _, _ = row_sharded_flash_sinkhorn(*leaves, eps, lmu_d, lnu_d, K_iter=c["K_iter"], lam=c["lam"],
                                                    mask=mask_d, cg_opts=cg)
            grads = torch.autograd.grad(O, leaves, grad_outputs=inp["dO"].float())
            return [g[:, :, r0:r1] for g in grads]   # this rank's rows (all ranks hold all)
        order, res = bh_sharded_flash_sinkhorn(*leaves, eps, lmu_d, lnu_d, c["K_iter"], c["lam"], lengths, world,
                                               rank, mask=mask_d, cg_opts=cg)
        if not res:
            return []
        dOs = inp["dO"].index_select(0, torch.tensor(order, device=dev)).float()
        outs = [r[4] for r in res]
        gos = [dOs[s0:s1, h0:h1] for s0, s1, h0, h1, *_ in res]
        grads = torch.autograd.grad(outs, leaves, grad_outputs=gos)
        return [g.index_select(0, torch.tensor([order[i] for i in range(s0, s1)], device=dev))[:, h0:h1]
                for g in grads for s0, s1, h0, h1, *_ in res]

    dev_in = {k: v.to(dev) for k, v in host.items()}
    # the clock sampler starts before the warm-up: nvidia-smi's start-up queries
    # every GPU of the host, which must not fall into the timed steps
    sampler = ClockSampler(dev) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(args.warmup):
        step(dev_in)
    torch.cuda.synchronize()
    quiet_gc()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step(dev_in)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # e2e: host inputs copied in and this rank's gradients copied out every step
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = 0
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    pipe = CopyPipeline(host, dev, stream)  # buffers (pinned read-back ones included) made once, outside timing

    def run_e2e(n):
        nbytes = 0
        pipe.start()
        for i in range(n):
            if i + 1 < n:
                pipe.prefetch(i + 1)
            inp = {k: v.detach() for k, v in pipe.inputs(i).items()}
            nbytes = pipe.finish_step(i, step(inp))
        pipe.end()
        return nbytes

    run_e2e(2)  # both buffer sets allocated and used once
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e2.record(stream)
    d2h = run_e2e(args.steps)
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e2.elapsed_time(e3)
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    clocks = sampler.stop() if sampler else None
    rep = last_rowshard_report() if args.config == 4 else last_cg_report()
    n_cg = float(rep["cg_iters"].float().mean()) if rep else 0.0
    status = (int(rep["status"].item()) | int(rep["fwd_status"].item())) if rep else 0
    if rank == 0:
        peak, _, peak_src = load_peaks()
        per = sum(L * L for L in lengths) * d * H   # valid points only: padding is skipped, not counted
        f_call = ((4 * c["K_iter"] + 4) + (14 + 2 * n_cg)) * per
        value = args.steps / (ms * 1e-3)
        per_gpu_tf = f_call * value / world / 1e12
        name = big_workload_name(args.config)
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": f"synthetic (seeded N(0,1); B={B} H={H} N={N} d={d})",
            "config": {"workload": name, "global_batch": B, "heads": H, "seq_len": N, "head_dim": d,
                       "parallelism": (f"(batch,head)-shard x{world}, length^2-balanced" if args.config == 3
                                       else f"row-shard x{world}, peer-memory exchange over NVLink (no "
                                            "collective on the data path)"),
                       "l2": "inputs and per-call working set exceed L2 (streamed N x N recompute)"},
            "tflops": {"algorithmic_per_call": round(f_call / 1e12, 4), "counted_on": "sum_b L_b^2 (true lengths)",
                       "cg_iters_mean": n_cg,
                       "achieved_per_gpu": round(per_gpu_tf, 3), "frac_of_bf16_peak": round(per_gpu_tf / peak, 5)},
            "roofline": {"bound": "tensor", "kernel": "streamed passes (whole fwd+bwd step)",
                         "achieved": round(per_gpu_tf, 3), "peak": peak, "peak_source": peak_src,
                         "unit": "TFLOP/s", "frac": round(per_gpu_tf / peak, 5), "traffic": None},
            "e2e": {"value": round(args.steps / (e2e_ms * 1e-3), 4), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "device_status": status,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.config, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _ref_threads() -> int:
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


def _ref_problem(B, H, N, d, K_iter, lam, eps, seed, mask=None, lmu=None, lnu=None):
    """Seeded inputs of one reference-path call (bf16-rounded values in fp32,
    as the GPU arm sees them)."""
    g = torch.Generator().manual_seed(seed)
    Q, K, V, dO = (torch.randn(B, H, N, d, generator=g).to(torch.bfloat16).float() for _ in range(4))
    lm = torch.full((B, H, N), -math.log(N))
    # the reference's compute_transport_output always gates (sigmoid(G) * O_avg); G = 0 gates by 1/2
    return dict(Q=Q, K=K, V=V, dO=dO, eps=torch.full((H,), float(eps)), log_mu=lm if lmu is None else lmu,
                log_nu=lm if lnu is None else lnu, K_iter=K_iter, lam=1e6 if math.isinf(lam) else lam, mask=mask,
                G=torch.zeros(B, H, N, d), dO_flat=dO.permute(0, 2, 1, 3).reshape(B, N, H * d).contiguous(),
                kind="reference" if _REF_ACTIVE else "port")


REF_DIR = os.path.join(ROOT, "baseline", "_ref")   # the reference, pip-installed (git-ignored, travels)


def _reference_installed() -> bool:
    return os.path.isfile(os.path.join(REF_DIR, "deepfold", "model", "sinkhorn.py"))


_REF_ACTIVE = False


def _use_reference_package():
    """Put the installed reference first on sys.path (only in processes that never
    import this build's ``deepfold``: the --impl reference / triton arms)."""
    global _REF_ACTIVE
    if "deepfold" in sys.modules:
        raise RuntimeError("the reference package must be imported before this build's deepfold")
    sys.path.insert(0, REF_DIR)
    _REF_ACTIVE = True


def _ref_call(prob):
    """One forward + autograd backward of the reference's CPU path in float32:
    C = -Q K^T / sqrt(d) (the cost of sinkhorn_kernel.py:59-129 without the
    optional terms), the reference's own sinkhorn_solve (sinkhorn.py:17) and
    compute_transport_output (sinkhorn.py:115) from the installed package, torch
    autograd of sum(o * dO).  Without the installed package the same computation
    restated in oracle/sinkhorn_torch.py runs instead."""
    if prob.get("kind") == "reference":
        from deepfold.model.sinkhorn import compute_transport_output, sinkhorn_solve
        Q, K, V = (prob[k].detach().clone().requires_grad_(True) for k in ("Q", "K", "V"))
        d = Q.shape[-1]
        C = -(Q @ K.transpose(-1, -2)) / math.sqrt(d)
        lam = prob["lam"]
        lu, lv = sinkhorn_solve(C, prob["log_mu"], prob["log_nu"], prob["eps"], lam=lam, K=prob["K_iter"],
                                mask=prob["mask"])
        o, _, _ = compute_transport_output(V, prob["G"], lu, lv, C, prob["eps"], mask=prob["mask"])
        torch.autograd.grad(o, (Q, K, V), grad_outputs=prob["dO_flat"])
        return
    from oracle import sinkhorn_torch as ort
    ort.attn_fwd_bwd(prob["Q"], prob["K"], prob["V"], prob["eps"], prob["log_mu"], prob["log_nu"], prob["K_iter"],
                     prob["lam"], prob["dO"], dtype=torch.float32, mask=prob["mask"])


def _ref_sample(cfg_id):
    """(problem, calls of the whole configuration one sample call stands for, text).
    Config 2 is timed whole.  For configs 3 and 4 (dense N x N autograd state of
    up to ~20 GB per head) one problem of a smaller length L is timed and the
    time scaled by sum over the configuration's problems of (L_bh / L)^2."""
    if cfg_id == 2:
        c = CFG
        prob = _ref_problem(c["B"], c["H"], c["N"], c["d"], c["K_iter"], float("inf"), c["eps"], 7)
        return prob, 1.0, f"whole config-2 calls (B={c['B']} H={c['H']} N={c['N']} d={c['d']})"
    c = BIG[cfg_id]
    L = 512 if cfg_id == 3 else 2048
    prob = _ref_problem(1, 1, L, c["d"], c["K_iter"], c["lam"], c["eps"], 3)
    _, lengths, _, _, _ = big_inputs(c)
    scale = sum(c["H"] * (Lb / L) ** 2 for Lb in lengths)
    return prob, 1.0 / scale, (f"one (batch, head) problem of N={L}, d={c['d']}, K={c['K_iter']}, scaled by "
                               f"sum over the config's problems of (L_bh/{L})^2 = {scale:.1f}")


def _ref_text(kind, n, what):
    where = ("the installed reference package" if kind == "reference"
             else "restated in oracle/sinkhorn_torch.py")
    return (f"{n} calls of the reference's torch CPU path (dense cost + sinkhorn_solve + compute_transport_output "
            f"+ autograd, float32, {where}): {what}")


def _time_reference(cfg_id, warmup, steps=None, seconds=None):
    """(seconds per sample call, calls made, problem, per_call, what)."""
    prob, per_call, what = _ref_sample(cfg_id)
    for _ in range(max(1, warmup)):
        _ref_call(prob)
    t0 = time.perf_counter()
    n = 0
    while True:
        _ref_call(prob)
        n += 1
        if (steps is not None and n >= steps) or (seconds is not None and time.perf_counter() - t0 > seconds):
            break
    return (time.perf_counter() - t0) / n, n, prob, per_call, what


def cpu_baseline(cfg_id=2, seconds=15.0):
    """The reference's CPU path timed on a bounded sample (~`seconds` of work): the
    installed reference package in a child process (this process has already
    imported this build's ``deepfold``), else the restatement in this process."""
    if _reference_installed():
        env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--config",
                            str(cfg_id), "--warmup", "1", "--ref-seconds", str(seconds)],
                           env=env, capture_output=True, text=True, timeout=600)
        for ln in reversed(r.stdout.splitlines()):
            if ln.startswith("{"):
                return json.loads(ln)["cpu_baseline"]
        print(f"cpu_baseline: reference child failed ({r.returncode}): {r.stderr[-500:]}", file=sys.stderr)
    cores = _ref_threads()
    dt, n, prob, per_call, what = _time_reference(cfg_id, 1, seconds=seconds)
    return {"value": round(per_call / dt, 6), "unit": UNIT, "cores": cores, "kind": prob["kind"],
            "sample": _ref_text(prob["kind"], n, what), "cpu": _cpu_model()}


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cores = _ref_threads()
    if args.ref_seconds:
        dt, n, prob, per_call, what = _time_reference(args.config, args.warmup, seconds=args.ref_seconds)
    else:
        dt, n, prob, per_call, what = _time_reference(args.config, args.warmup, steps=args.steps)
    value = per_call / dt
    if args.config == 2:
        c = CFG
        workload, shape = workload_name(), dict(global_batch=c["B"], heads=c["H"], seq_len=c["N"], head_dim=c["d"])
    else:
        c = BIG[args.config]
        workload, shape = big_workload_name(args.config), dict(global_batch=c["B"], heads=c["H"], seq_len=c["N"],
                                                               head_dim=c["d"])
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": UNIT, "n_gpus": world,
            "steps": n, "warmup": args.warmup, "ms_per_step": round(1e3 / value, 3),
            "higher_is_better": True, "scaling": "weak" if args.config == 2 else "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,1), bf16-rounded values in float32)",
            "config": dict(workload=workload, parallelism="cpu", **shape),
            "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": cores, "kind": prob["kind"],
                             "sample": _ref_text(prob["kind"], n, what), "cpu": _cpu_model()},
            "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_triton(args):
    """The reference's own GPU path on this GPU: ``flash_sinkhorn``
    (sinkhorn_kernel.py:2385; Triton forward, Triton unrolled backward) from the
    installed reference package, unmodified, on the same seeded workload as this
    build's arm (config 2, or config 3 with its masks and marginals).  The
    reference computes in float32 (it casts its inputs); its cost always carries
    the position and geometry terms, given zero weights here.  CUDA events around
    each fwd + bwd, L2 flushed between steps.  Not one of the driver's arms: a
    measurement of the GPU bar."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if not _REF_ACTIVE:
        print(json.dumps({"impl": "triton-reference", "unavailable": "reference package not installed in "
                          "baseline/_ref"}))
        return
    from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn as ref_flash_sinkhorn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.config == 2:
        c = dict(CFG, lam=float("inf"), varlen=False)
        g = torch.Generator().manual_seed(0)
        B, H, N, d = c["B"], c["H"], c["N"], c["d"]
        host = {k: torch.randn(B, H, N, d, generator=g).to(torch.bfloat16) for k in ("Q", "K", "V", "dO")}
        mask = None
        lmu = torch.full((B, H, N), -math.log(N))
        lnu = lmu.clone()
        workload = workload_name()
    else:
        c = BIG[args.config]
        B, H, N, d = c["B"], c["H"], c["N"], c["d"]
        host, _, mask, lmu, lnu = big_inputs(c)
        workload = big_workload_name(args.config)
    lam = 1e6 if math.isinf(c["lam"]) else c["lam"]
    inp = {k: v.float().to(dev) for k, v in host.items()}
    x_res = torch.zeros(B, N, 3, device=dev)
    pos_weight = torch.zeros(H, 68, device=dev)
    pos_bins = torch.zeros(B, N, N, device=dev, dtype=torch.int32)
    w_dist = torch.zeros(H, device=dev)
    eps = torch.full((H,), float(c["eps"]), device=dev)
    lmu, lnu = lmu.to(dev), lnu.to(dev)
    mask_d = None if mask is None else mask.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        leaves = [inp[k].detach().requires_grad_(True) for k in ("Q", "K", "V")]
        O, _, _, _ = ref_flash_sinkhorn(*leaves, x_res, pos_weight, pos_bins, eps, w_dist, lmu, lnu,
                                        K_iter=c["K_iter"], lam=lam, mask=mask_d)
        torch.autograd.grad(O, leaves, grad_outputs=inp["dO"])

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    fwd_only = []
    evs = []
    for _ in range(args.steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        evs.append((e0, e1))
    for _ in range(args.steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.no_grad():
            ref_flash_sinkhorn(inp["Q"], inp["K"], inp["V"], x_res, pos_weight, pos_bins, eps, w_dist, lmu, lnu,
                               K_iter=c["K_iter"], lam=lam, mask=mask_d)
        e1.record(stream)
        fwd_only.append((e0, e1))
    torch.cuda.synchronize()
    t = sorted(a.elapsed_time(b) for a, b in evs)
    tf = sorted(a.elapsed_time(b) for a, b in fwd_only)
    med, medf = t[len(t) // 2], tf[len(tf) // 2]
    line = {"impl": "triton-reference", "metric": METRIC, "value": round(1e3 / med, 4), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(med, 4),
            "fwd_ms": round(medf, 4), "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded N(0,1), bf16-rounded values in float32)",
            "config": {"workload": workload, "l2": "flushed between timed steps",
                       "path": "reference flash_sinkhorn (Triton fwd + unrolled Triton bwd), lam=1e6 for balanced"},
            "gpu": torch.cuda.get_device_name(dev)}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- balanced transport
# The reference's published timing of its balanced transport (Triton forward +
# unrolled Triton backward, x_centroid only), B=1 H=16 d_h=32 K=20, on an
# unnamed GPU: ms per fwd+bwd by N.
TRANSPORT_PUBLISHED_MS = {64: 1.6, 256: 4.5, 512: 8.3, 768: 21.4}


def run_transport(args):
    """fwd+bwd of balanced_sinkhorn_transport (the trunk block's call) through the
    public API at the shapes the reference publishes, fp32 unit-norm Q/K,
    x ~ 4 N(0,1), per-head eps 0.5/1/2/4, alpha ~ N(0,1), r_h = 10, full mask;
    CUDA events around each step, L2 flushed between steps."""
    import torch.nn.functional as F
    from deepfold import _native as nat
    from deepfold.model.kernels.flash_sinkhorn_transport import balanced_sinkhorn_transport

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nat.lib()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    B, H, d, K_iter = 1, 16, 32, 20
    per_n = {}
    sampler = ClockSampler(dev)
    sampler.start()
    time.sleep(0.3)
    for N, pub in TRANSPORT_PUBLISHED_MS.items():
        g = torch.Generator().manual_seed(N)
        Q = F.normalize(torch.randn(B, H, N, d, generator=g), dim=-1).to(dev).requires_grad_(True)
        K = F.normalize(torch.randn(B, H, N, d, generator=g), dim=-1).to(dev).requires_grad_(True)
        x = (torch.randn(B, N, 3, generator=g) * 4.0).to(dev).requires_grad_(True)
        eps = torch.tensor([0.5] * 4 + [1.0] * 4 + [2.0] * 4 + [4.0] * 4, device=dev)
        alpha = torch.randn(H, generator=g).to(dev).requires_grad_(True)
        r_h = torch.full((H,), 10.0, device=dev, requires_grad=True)
        mask = torch.ones(B, N, device=dev)
        gxc = torch.randn(B, H, N, 3, generator=g).to(dev)

        def step():
            xc = balanced_sinkhorn_transport(Q, K, x, eps, alpha, r_h, K_iter=K_iter, mask=mask)
            torch.autograd.backward(xc, gxc)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        ms = []
        for _ in range(args.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            ms.append((e0, e1))
        torch.cuda.synchronize()
        t = sorted(a.elapsed_time(b) for a, b in ms)
        med = t[len(t) // 2]
        per_n[N] = {"ms_median": round(med, 4), "ms_mean": round(sum(t) / len(t), 4),
                    "reference_published_ms": pub, "speedup_vs_published": round(pub / med, 1)}
    clocks = sampler.stop()
    line = {"metric": "balanced transport fwd+bwd ms (B=1 H=16 d_h=32 K=20, fp32)", "value": per_n[768]["ms_median"],
            "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "vs_baseline": round(per_n[768]["ms_median"] / TRANSPORT_PUBLISHED_MS[768], 5), "dtype": "f32",
            "data": "synthetic (seeded unit-norm Q/K, N(0,1) x, alpha)",
            "config": {"workload": "balanced_sinkhorn_transport fwd+bwd, x_centroid only, N=64/256/512/768",
                       "l2": "flushed between timed steps"},
            "per_N": per_n, "clocks": clocks}
    print(json.dumps(line), flush=True)


DENSE = dict(B=1, H=16, N=4096, d=64, eps=1.0, K_iter=20)


def run_dense(args):
    """The dense-cost entry points beyond the resident range: sinkhorn_solve +
    compute_transport_output on a given fp32 cost C (B=1 H=16 N=4096: 1 GiB),
    V head dim 64, K=20, uniform marginals, balanced.  Each iteration streams C
    once (4 bytes per pair: the row and column updates share one read), the
    transport pass twice and writes T_norm; the roofline is those bytes at the
    measured HBM bandwidth.  The line's value is the forward; "fwd_bwd" times
    the same call with a loss on o backpropagated to C and V (the unrolled
    K-step adjoint and the T_norm backward), as the reference's users run it
    under autograd."""
    from deepfold.model.sinkhorn import compute_transport_output, sinkhorn_solve

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = dict(DENSE, H=args.dense_heads or DENSE["H"])
    B, H, N, d = c["B"], c["H"], c["N"], c["d"]
    g = torch.Generator().manual_seed(0)
    C = torch.rand(B, H, N, N, generator=g).to(dev)
    lm = torch.full((B, H, N), -math.log(N), device=dev)
    eps = torch.full((H,), c["eps"], device=dev)
    V = torch.randn(B, H, N, d, generator=g).to(dev)
    G = torch.zeros(B, H, N, d, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        lu, lv = sinkhorn_solve(C, lm, lm, eps, lam=float("inf"), K=c["K_iter"])
        return compute_transport_output(V, G, lu, lv, C, eps)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    quiet_gc()
    sampler = ClockSampler(dev)
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # forward + backward through the public autograd surface
    Cg, Vg = C.clone().requires_grad_(True), V.clone().requires_grad_(True)
    go = torch.randn(B, N, H * d, generator=g).to(dev)

    def grad_step():
        lu, lv = sinkhorn_solve(Cg, lm, lm, eps, lam=float("inf"), K=c["K_iter"])
        o = compute_transport_output(Vg, G, lu, lv, Cg, eps)[0]
        Cg.grad = Vg.grad = None
        (o * go).sum().backward()

    for _ in range(3):
        grad_step()
    torch.cuda.synchronize()
    e0.record(stream)
    gsteps = max(1, min(args.steps, 10))
    for _ in range(gsteps):
        grad_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_fb = e0.elapsed_time(e1) / gsteps
    clocks = sampler.stop()
    pairs = B * H * N * N
    # bytes per call: K iterations reading C once each (N <= 8192: row and column update in one read),
    # the transport pass reading C twice and writing T_norm
    nbytes = (c["K_iter"] + 3) * 4 * pairs
    _, peak, peak_src = load_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    line = {"metric": "dense-cost sinkhorn_solve + compute_transport_output calls/s", "value": round(1e3 / ms, 4),
            "unit": "calls/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "f32",
            "data": f"synthetic (uniform C in [0,1), N(0,1) V; B={B} H={H} N={N} d={d})",
            "config": {"workload": f"dense sinkhorn_solve K={c['K_iter']} + compute_transport_output, B={B} H={H} "
                                   f"N={N} d={d}, balanced", "l2": f"C ({pairs * 4 / 2**30:.2f} GiB) exceeds L2"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "peak_source": peak_src,
                         "unit": "GB/s", "frac": round(gbs / peak, 4), "bytes_per_call": nbytes},
            "fwd_bwd": {"ms_per_step": round(ms_fb, 4), "steps": gsteps, "warmup": 3},
            "clocks": clocks}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "triton"], default="ours")
    ap.add_argument("--ref-seconds", type=float, default=None, help=argparse.SUPPRESS)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--dense-heads", type=int, default=0,
                    help="heads of the --config dense workload (default 16; fewer for small profiling captures)")
    ap.add_argument("--no-config4", action="store_true", help="skip the single-GPU long-sequence point")
    ap.add_argument("--config", choices=["2", "3", "4", "transport", "dense"], default=None,
                    help="default: 2 on one GPU, 4 (long-sequence row shards) on several; 'transport': the "
                         "balanced transport at the reference's published shapes (one GPU)")
    args = ap.parse_args()
    if args.impl in ("reference", "triton") and _reference_installed():
        _use_reference_package()
    if args.config == "transport":
        if args.impl != "ours":
            print(json.dumps({"impl": "reference", "unavailable": "the transport mode times this build only; "
                              "the reference's published timings are printed beside it"}))
            return
        if args.warmup < 3:
            args.warmup = 3
        run_transport(args)
        return
    if args.config == "dense":
        if args.impl != "ours":
            print(json.dumps({"impl": "reference", "unavailable": "the dense mode times this build only"}))
            return
        run_dense(args)
        return
    if args.config is not None:
        args.config = int(args.config)
    if args.config is None:
        args.config = 4 if int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.gpus > 1 else 2
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "triton":
        run_triton(args)
    elif args.config in BIG:
        run_big(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
