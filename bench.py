#!/usr/bin/env python
"""Benchmark: HP/BE co-scheduling on the kx kernels through the drop-in
interposer: HP VGG16 inference against BE GPT training.

Workload (one "step" = one HP request):
  HP  = VGG16 inference, fp32, batch 32 x 3x224x224 N(0,1), Kaiming-normal init
  BE  = training steps of a GPT (6 layers, d_model 512, 8 heads,
        FFN 2048, vocab 32000), batch 16 x seq 256, AdamW lr 1e-4,
        cross-entropy against uniform random targets
Both run as PyTorch models in one process under
LD_PRELOAD=kernel_intercept_b200/libgpu_scheduler.so; client 0 (HP) and client
1 (BE) are registered threads, every captured GEMM / convolution runs on the
kx sm_100a kernels (bench.py re-executes itself with the preload when needed).

Phases (same models and inputs): HP alone, BE alone, HP + BE together (HP
back to back: the timed region), HP paced at a duty cycle of --hp-load
against BE (the Orion setting: HP p99 vs solo and BE retention), and the
end-to-end repeat.  The timed region is the K HP steps of the contended phase,
bracketed by a barrier and a device synchronize, timed with CUDA events on
the HP stream (max over ranks).  `value` = HP images/s under contention
(whole job: sum over ranks).
`e2e` repeats the contended phase (over max(K, 200) HP steps, like the
latency phases) with the HP input copied from pinned host memory and the
logits copied back inside every step.  `roofline` is the
dominant captured kernel class (HP convolutions) from CUDA events recorded
around each captured op during the timed region.  `cpu_baseline` is the CPU
oracle's VGG16 forward on a bounded sample, timed on this host.

--impl reference prints the same line for the reference's CPU path of the
captured ops (the oracle restatement of cuBLAS / cuDNN semantics, all host
threads), on a bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HP_BATCH = 32
BE_BATCH, BE_SEQ = 16, 256
METRIC = "HP p99 latency vs solo + BE iters/s; captured GEMM/conv % of B200 peak"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kx", choices=["kx", "reference"])
    ap.add_argument("--be-seconds", type=float, default=4.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--be-keep-sms", type=int, default=-1,
                    help="SMs a BE op keeps while HP runs (default: the scheduler's)")
    ap.add_argument("--gil-switch-ms", type=float, default=0.5,
                    help="sys.setswitchinterval of the process (HP and BE are Python threads; "
                         "0: Python's default of 5 ms)")
    ap.add_argument("--gc-freeze", type=int, default=0,
                    help="1: freeze the warm-up's objects and pause Python's cyclic garbage "
                         "collector while the clients run (collections stop every thread)")
    ap.add_argument("--trace", default="",
                    help="write a Chrome trace of the interposer's activity in the paced phase "
                         "(client issues and waits, worker execution, HP flag) to this path; "
                         "a .gz path is compressed")
    ap.add_argument("--hp-load", type=float, default=1.0 / 3.0,
                    help="HP duty cycle of the paced phase (request period = solo p50 / load)")
    return ap.parse_args()


def dist_info():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------- CPU baseline ----

def oracle_vgg16_images_per_s(sample_images=1, threads=None):
    """VGG16 forward of `sample_images` images through the oracle (conv and FC
    restatements; ReLU / max-pool in numpy).  Returns (images/s, cores)."""
    import numpy as np

    from oracle import oracle as o
    if threads:
        o.set_num_threads(threads)
    cores = o.num_threads()
    rng = np.random.default_rng(0)
    cfg = [64, 64, "M", 128, 128, "M", 256, 256, 256, "M", 512, 512, 512, "M", 512, 512, 512, "M"]
    x = rng.standard_normal((sample_images, 3, 224, 224)).astype(np.float32)
    c_in = 3
    weights = []
    for v in cfg:
        if v == "M":
            continue
        std = (2.0 / (v * 9)) ** 0.5
        weights.append((rng.standard_normal((v, c_in, 3, 3)).astype(np.float32) * std,
                        np.zeros(v, np.float32)))
        c_in = v
    fcs = [(25088, 4096), (4096, 4096), (4096, 1000)]
    fcw = [(rng.standard_normal((o_, i_)).astype(np.float32) * 0.01, np.zeros(o_, np.float32))
           for i_, o_ in fcs]
    t0 = time.perf_counter()
    h = x
    wi = 0
    for v in cfg:
        if v == "M":
            n, c, hh, ww = h.shape
            h = h.reshape(n, c, hh // 2, 2, ww // 2, 2).max(axis=(3, 5))
            continue
        w, b = weights[wi]
        wi += 1
        n, c, hh, ww = h.shape
        d = o.conv_desc(n, c, hh, ww, w.shape[0], 3, 3, pad=(1, 1))
        h = o.conv_fwd(d, 1.0, h, w) + b[None, :, None, None]
        h = np.maximum(h, 0.0, dtype=np.float32)
    h = h.reshape(h.shape[0], -1)
    for i, (w, b) in enumerate(fcw):
        n = h.shape[0]
        out = np.zeros((n, w.shape[0]), np.float32)
        # y^T (out x n) = W (out x in) . h^T: cuBLAS view transa = T, transb = N
        o.gemm_ex(1, 0, w.shape[0], n, w.shape[1], 1.0, np.ascontiguousarray(w), o.R_32F,
                  w.shape[1], np.ascontiguousarray(h), o.R_32F, w.shape[1], 0.0, None, o.R_32F,
                  w.shape[0], D=out, Dtype=o.R_32F, ldd=w.shape[0], epilogue=4, bias=b)
        h = np.maximum(out, 0.0) if i < 2 else out
    dt = time.perf_counter() - t0
    return sample_images / dt, cores


def run_reference(args):
    rank, world, _ = dist_info()
    if rank != 0:
        return 0  # rank 0 alone runs the CPU path
    cores = os.cpu_count() or 1
    vals = []
    for _ in range(max(0, args.warmup)):
        pass  # the oracle has no warm-up state; warm-up steps are not timed
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, used = oracle_vgg16_images_per_s(1, threads=cores)
        vals.append(v)
    total = time.perf_counter() - t0
    value = args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "images/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64-accumulate",
        "data": "synthetic", "config": {"workload": "VGG16 inference fp32 (the HP model), CPU "
                                        "path of the captured ops, 1-image sample per step",
                                        "batch": 1},
        "cpu_baseline": {"value": round(value, 4), "unit": "images/s", "cores": used,
                         "kind": "port", "sample": "1 image of the batch-32 VGG16 forward per step"},
        "e2e": {"value": round(value, 4), "unit": "images/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- kx arm ------

class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index=0):
        self.path = tempfile.mktemp(prefix="kx_clocks_", suffix=".csv")
        self.proc = None
        self.index = index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 7:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        sm = sorted(float(r[0]) for r in rows if r[0].replace(".", "").isdigit())
        mx = max(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons}


def run_kx(args):
    import torch
    import torch.nn.functional as F

    if args.gil_switch_ms > 0:
        # HP and BE are Python threads of one process (as in the reference's
        # drivers): the interval bounds how long one waits for the other's GIL
        sys.setswitchinterval(args.gil_switch_ms / 1e3)

    from kernel_intercept_b200 import harness, kx

    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
        pg = dist

    orion = harness.Orion()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.benchmark = False
    torch.manual_seed(0)

    # ---- models and resident inputs
    vgg = harness.make_vgg16(dev).eval()
    gpt = harness.make_gpt(device=dev)
    opt = torch.optim.AdamW(gpt.parameters(), lr=1e-4)
    img = torch.randn(HP_BATCH, 3, 224, 224, device=dev)
    img_host = img.cpu().pin_memory()
    out_host = torch.empty(HP_BATCH, 1000).pin_memory()
    tok = torch.randint(0, 32000, (BE_BATCH, BE_SEQ), device=dev)
    tgt = torch.randint(0, 32000, (BE_BATCH, BE_SEQ), device=dev)

    def hp_step():
        with torch.no_grad():
            vgg(img)

    def hp_step_e2e():
        with torch.no_grad():
            img.copy_(img_host, non_blocking=True)
            out = vgg(img)
            out_host.copy_(out, non_blocking=True)

    def be_step():
        logits = gpt(tok)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]), tgt.view(-1))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()

    # native warm-up with capture off (allocator, cuDNN plans), like the reference drivers
    assert orion.orion_init_scheduler(2) == 0, "orion_init_scheduler failed"
    orion.orion_set_capture(0)
    hp_step()
    be_step()
    torch.cuda.synchronize()
    if args.be_keep_sms >= 0:
        orion.orion_set_be_keep_sms(args.be_keep_sms)
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    if args.gc_freeze:
        import gc
        gc.collect()
        gc.freeze()
        gc.disable()

    def barrier():
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()

    kxlib = kx.lib()

    def profiled(tag, run):
        """Runs run(on_start); the profiling session opens in on_start (after
        both clients' warm-up, so warm-up launches are not in the records) and
        closes when run returns.  Returns (run's result, records)."""
        path = tempfile.mktemp(prefix="kx_prof_", suffix=".json")
        opened = []

        def on_start():
            orion.orion_start_profiling(tag.encode())
            opened.append(True)

        try:
            res = run(on_start)
        finally:
            if opened:
                orion.orion_end_profiling(path.encode())
        recs = []
        if opened:
            with open(path) as f:
                recs = json.load(f).get("kernels", [])
            os.unlink(path)
        return res, recs

    # phase 1: HP alone (per-op timing for the solo roofline)
    barrier()
    # latency phases run at least 200 HP steps so that p99 is a percentile
    lat_steps = max(args.steps, 200)
    (hp_solo, _), solo_recs = profiled("hp_solo", lambda on_start: harness.run_clients(
        orion, hp_step, be_step, lat_steps, args.warmup, with_be=False, on_start=on_start))
    # phase 2: BE alone
    _, be_solo = harness.run_clients(orion, hp_step, be_step, 0, 0, with_hp=False,
                                     be_seconds=args.be_seconds)
    # phase 3 (timed): HP + BE, per-op timing, clocks, launch count
    clocks = Clocks(local)
    barrier()
    launches0 = kxlib.kx_launch_count()
    clocks.start()
    (hp_c, be_c), cont_recs = profiled("contended", lambda on_start: harness.run_clients(
        orion, hp_step, be_step, args.steps, args.warmup, on_start=on_start))
    clk = clocks.stop()
    launches = kxlib.kx_launch_count() - launches0
    barrier()
    # phase 4: paced HP (requests every solo_p50 / hp_load ms) against BE, the
    # Orion setting in which HP latency vs solo and BE retention are judged
    s50_now = harness.percentile(hp_solo.latencies_ms, 0.5)
    period = s50_now / max(args.hp_load, 1e-3)
    paced_steps = lat_steps
    for c in (0, 1):
        orion.waits(c, reset=True)
    if args.trace:
        orion.orion_trace_start()
    hp_p, be_p = harness.run_clients(orion, hp_step, be_step, paced_steps, args.warmup,
                                     hp_period_ms=period)
    if args.trace:
        harness.write_trace(orion, args.trace)
    paced_waits = {("hp", "be")[c]: orion.waits(c) for c in (0, 1)}
    # phase 5: e2e (host buffers in every HP step), contended, over as many
    # steps as the latency phases so that one host-side stall on one rank does
    # not stand for the whole run
    hp_e2e = None
    e2e_steps = lat_steps
    if not args.no_e2e:
        hp_e2e, _ = harness.run_clients(orion, hp_step_e2e, be_step, e2e_steps, args.warmup)
    stats = {c: orion.stats(c) for c in (0, 1)}
    orion.orion_set_capture(0)
    orion.orion_stop_scheduler()

    peaks, peak_src = measured_peaks()
    tf32 = measure_tf32_peak(dev)  # capture is off: this runs cuBLAS itself
    roof = roofline(cont_recs, peaks, peak_src, tf32, sustained=True)
    roof_solo = roofline(solo_recs, peaks, peak_src, tf32, sustained=False)

    # ---- aggregate over ranks
    hp_ms = hp_c.elapsed_ms
    imgs = HP_BATCH * args.steps
    e2e_ms = hp_e2e.elapsed_ms if hp_e2e else 0.0
    per_rank = [[hp_ms, e2e_ms]]
    if pg is not None:
        t = torch.tensor([hp_ms, e2e_ms], device=dev)
        parts = [torch.zeros_like(t) for _ in range(world)]
        pg.all_gather(parts, t)
        per_rank = [[float(v) for v in x.tolist()] for x in parts]
        hp_ms = max(r[0] for r in per_rank)
        e2e_ms = max(r[1] for r in per_rank)
    value = world * imgs / (hp_ms / 1e3)
    p50 = harness.percentile(hp_c.latencies_ms, 0.5)
    p99 = harness.percentile(hp_c.latencies_ms, 0.99)
    s50 = harness.percentile(hp_solo.latencies_ms, 0.5)
    s99 = harness.percentile(hp_solo.latencies_ms, 0.99)
    be_solo_ips = be_solo.iters / (be_solo.elapsed_ms / 1e3) if be_solo.elapsed_ms else 0.0
    be_c_ips = be_c.iters / (be_c.elapsed_ms / 1e3) if be_c.elapsed_ms else 0.0
    # HP latency against its own solo run, per rank: the line's hp / paced
    # blocks are rank 0's; at N > 1 the worst rank's ratios are added
    pp99 = harness.percentile(hp_p.latencies_ms, 0.99)
    be_p_ips = be_p.iters / (be_p.elapsed_ms / 1e3) if be_p.elapsed_ms else 0.0
    ratios = [p99 / s99 if s99 else 0.0, pp99 / s99 if s99 else 0.0,
              be_p_ips / be_solo_ips if be_solo_ips else 0.0]
    rank_ratios = [ratios]
    if pg is not None:
        t = torch.tensor(ratios, device=dev, dtype=torch.float64)
        parts = [torch.zeros_like(t) for _ in range(world)]
        pg.all_gather(parts, t)
        rank_ratios = [[float(v) for v in x.tolist()] for x in parts]

    cpu = None
    if rank == 0:
        v, cores = oracle_vgg16_images_per_s(1, threads=os.cpu_count())
        cpu = {"value": round(v, 4), "unit": "images/s", "cores": cores, "kind": "port",
               "sample": "1 image of the batch-32 VGG16 forward (oracle conv + GEMM "
                         "restatement, float64 accumulation)"}
        tv, tcores = torch_cpu_vgg16_images_per_s(2)
        cpu["torch_cpu_forward"] = {"value": round(tv, 4), "unit": "images/s",
                                    "cores": tcores, "sample": "2 images, torch fp32 CPU"}
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(hp_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "HP VGG16 inference fp32 b32 3x224x224 + BE GPT (6L, d512, "
                               "8 heads, vocab 32000) training fp32 b16 s256 AdamW, through "
                               "the LD_PRELOAD interposer",
                   "hp_batch": HP_BATCH, "be_batch": BE_BATCH, "be_seq": BE_SEQ,
                   "parallelism": f"placement x{world} (one HP+BE group per GPU, no collective)",
                   "l2": "inputs larger than L2 (VGG16 first-block activations 411 MB)",
                   "gil_switch_ms": round(sys.getswitchinterval() * 1e3, 3),
                   "gc_frozen": bool(args.gc_freeze)},
        "hp": {"p50_ms": round(p50, 3), "p99_ms": round(p99, 3), "solo_p50_ms": round(s50, 3),
               "solo_p99_ms": round(s99, 3), "p99_vs_solo": round(p99 / s99, 4) if s99 else None,
               "steps": args.steps, "solo_steps": lat_steps},
        "paced": {"hp_load": round(args.hp_load, 3), "period_ms": round(period, 3),
                  "hp_steps": paced_steps,
                  "hp_p50_ms": round(harness.percentile(hp_p.latencies_ms, 0.5), 3),
                  "hp_p99_ms": round(harness.percentile(hp_p.latencies_ms, 0.99), 3),
                  "hp_p99_vs_solo": round(harness.percentile(hp_p.latencies_ms, 0.99) / s99, 4)
                  if s99 else None,
                  "hp_issue_p50_ms": round(harness.percentile(hp_p.issue_ms, 0.5), 3),
                  "hp_issue_p99_ms": round(harness.percentile(hp_p.issue_ms, 0.99), 3),
                  "be_iters_per_s": round(be_p.iters / (be_p.elapsed_ms / 1e3), 3)
                  if be_p.elapsed_ms else None,
                  "be_retention": round(be_p.iters / (be_p.elapsed_ms / 1e3) / be_solo_ips, 4)
                  if be_p.elapsed_ms and be_solo_ips else None,
                  "client_waits": {k: {kk: round(vv, 3) if isinstance(vv, float) else vv
                                       for kk, vv in w.items()}
                                   for k, w in paced_waits.items()}},
        "be": {"iters_per_s": round(be_c_ips, 3), "solo_iters_per_s": round(be_solo_ips, 3),
               "retention": round(be_c_ips / be_solo_ips, 4) if be_solo_ips else None,
               "tokens_per_s": round(be_c_ips * BE_BATCH * BE_SEQ, 1)},
        "roofline": roof, "roofline_hp_solo": roof_solo, "ops": op_table(cont_recs),
        "cpu_baseline": cpu, "clocks": clk, "gpu_launches": int(launches),
        "captured": stats,
    }
    if world > 1:
        line["ms_per_step_per_rank"] = [round(r[0] / args.steps, 3) for r in per_rank]
        line["worst_rank"] = {
            "hp_p99_vs_solo": round(max(r[0] for r in rank_ratios), 4),
            "paced_hp_p99_vs_solo": round(max(r[1] for r in rank_ratios), 4),
            "paced_be_retention": round(min(r[2] for r in rank_ratios), 4)}
    if e2e_ms:
        h2d = HP_BATCH * 3 * 224 * 224 * 4
        d2h = HP_BATCH * 1000 * 4
        line["e2e"] = {"value": round(world * HP_BATCH * e2e_steps / (e2e_ms / 1e3), 3),
                       "unit": "images/s", "steps": e2e_steps,
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        if world > 1:
            line["e2e"]["ms_per_step_per_rank"] = [round(r[1] / e2e_steps, 3) for r in per_rank]
    print(json.dumps(line), flush=True)
    return 0


def group_ops(recs):
    by_op = {}
    for r in recs:
        key = ("HP" if r.get("client") == 0 else "BE", r.get("op_type", "?"))
        agg = by_op.setdefault(key, {"n": 0, "ms": 0.0, "work": 0.0, "kernels": {}})
        agg["n"] += 1
        agg["ms"] += float(r["duration_ms"])
        agg["work"] += float(r.get("work", 0.0))
        k = r["kernel_id"]
        agg["kernels"][k] = agg["kernels"].get(k, 0) + 1
    return by_op


def op_table(recs):
    out = {}
    for (client, op), v in sorted(group_ops(recs).items()):
        rate = v["work"] / (v["ms"] * 1e-3) / 1e12 if v["ms"] > 0 else None
        out[f"{client}:{op}"] = {"launches": v["n"], "ms": round(v["ms"], 3),
                                 "rate": round(rate, 2) if rate is not None else None,
                                 "rate_unit": "TB/s" if "BATCHNORM" in op else "TFLOP/s"}
    return out


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# dominant op class, from one ncu capture of a batch-32 VGG16 HP step: the mean
# over its 13 convolution launches (profiles/vgg16_hp_step_launches.md).
NCU_TRAFFIC_PER_LAUNCH = {"HP:CUDNN_CONV_FWD": 324059668}


def roofline(recs, peaks, peak_src, tf32, sustained):
    """Dominant captured op class of the HP client in a profiled phase (the
    client `value` measures; BE ops are throttled to the SMs HP leaves them,
    so their rate measures the scheduler, not the kernel): algorithmic FLOPs
    per launch (2mnk per GEMM, 2*N*K*C*R*S*P*Q per convolution) over the mean
    launch duration (CUDA events on the worker's dispatch stream)."""
    by_op = group_ops(recs)
    dense = {k: v for k, v in by_op.items()
             if k[0] == "HP" and "BATCHNORM" not in k[1] and v["work"] > 0}
    if not dense:
        return None
    (client, op), agg = max(dense.items(), key=lambda kv: kv[1]["ms"])
    avg_ms = agg["ms"] / agg["n"]
    achieved = agg["work"] / agg["n"] / (avg_ms * 1e-3) / 1e12
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    peak = float(peaks.get(key, peaks.get("bf16_tflops")))
    # fp32 runs as 3xTF32 (three TF32 products per MAC): its ceiling is the TF32 rate / 3
    ceiling = tf32 / 3.0
    top = max(agg["kernels"].items(), key=lambda kv: kv[1])[0]
    return {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1),
            "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "traffic": NCU_TRAFFIC_PER_LAUNCH.get(f"{client}:{op}"),
            "peak_source": f"{key} of {peak_src}",
            "tf32_cublas_tflops": round(tf32, 1),
            "fp32_3xtf32_ceiling": round(ceiling, 1),
            "frac_of_3xtf32_ceiling": round(achieved / ceiling, 4),
            "ffma_ceiling": round(peaks.get("sm_max_mhz", 1965.0) * 148 * 256 / 1e6, 1),
            "op": f"{client}:{op}", "kernel": top, "launches": agg["n"],
            "avg_ms": round(avg_ms, 4), "share_of_captured_ms":
            round(agg["ms"] / sum(v["ms"] for v in by_op.values()), 4)}


def measure_tf32_peak(dev):
    """cuBLAS TF32 rate on 8192^3 (burst, best of 5), the denominator of the
    3xTF32 ceiling.  Called with capture off, so cuBLAS itself runs."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device=dev)
    b = torch.randn(8192, 8192, device=dev)
    c = torch.empty(8192, 8192, device=dev)
    for _ in range(2):
        torch.matmul(a, b, out=c)
    best = 1e9
    for _ in range(5):
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        torch.matmul(a, b, out=c)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def torch_cpu_vgg16_images_per_s(sample_images=2):
    """The reference's CPU-runnable form: the same VGG16 as plain PyTorch on
    the host cores (no interception), fp32."""
    import torch

    from kernel_intercept_b200 import harness
    m = harness.make_vgg16("cpu").eval()
    x = torch.randn(sample_images, 3, 224, 224)
    with torch.no_grad():
        m(x[:1])
        t0 = time.perf_counter()
        m(x)
        dt = time.perf_counter() - t0
    return sample_images / dt, torch.get_num_threads()


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    from kernel_intercept_b200 import harness
    if not harness.preloaded():
        env = harness.preload_env({"ORION_LOG_LEVEL": os.environ.get("ORION_LOG_LEVEL", "WARN")})
        os.execve(sys.executable, [sys.executable] + sys.argv, env)
    return run_kx(args)


if __name__ == "__main__":
    sys.exit(main())
