#!/usr/bin/env python3
"""HP/BE job launcher with one client group per GPU.

Same command line and Python surface as the reference's
python/launch_jobs.py (``OrionScheduler`` 32-127, ``client_worker`` 130-208,
``MODEL_REGISTRY`` 211-267, ``run_with_scheduler`` 270-366, ``run_baseline``
369-416, ``main`` 419-452), with the placement the reference lacks: with
``--gpus N`` the launcher starts N processes, process g owns GPU g
(``CUDA_VISIBLE_DEVICES=g``) and hosts one HP client and its BE clients under
its own interposer instance (own queues, HP flag, SM quotas).  The groups are
independent; nothing crosses GPUs.  Results come back to rank 0 over a gloo
process group on the host (``all_gather_object``), which reports per-group
numbers and the aggregate: HP p99 over every group's HP iterations and the
summed BE throughput.

    python -m kernel_intercept_b200.launch --hp-model vgg16 --be-models gpt --gpus 8

The reference's ``block(phase)`` after every HP iteration is kept (the
interposer exports ``block``; it synchronizes the client's stream).
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import math
import os
import socket
import subprocess
import sys
import threading
import time
from typing import Callable

from . import LIBSHIM


class OrionScheduler:
    """ctypes wrapper of libgpu_scheduler.so, as python/launch_jobs.py 32-127."""

    def __init__(self, lib_path: str | None = None):
        self.lib_path = lib_path or os.environ.get("ORION_LIB_PATH", LIBSHIM)
        self.lib = None
        self.initialized = False

    def load_library(self) -> bool:
        if not os.path.exists(self.lib_path):
            print(f"Error: Library not found at {self.lib_path}")
            return False
        self.lib = ctypes.CDLL(self.lib_path, mode=ctypes.RTLD_GLOBAL)
        L, I = self.lib, ctypes.c_int
        for name, args, res in (("orion_init", [I], I), ("orion_shutdown", [], None),
                                ("orion_set_client_idx", [I], None),
                                ("orion_get_client_idx", [], I),
                                ("orion_set_enabled", [I], None),
                                ("orion_start_scheduler", [I], I),
                                ("orion_stop_scheduler", [], None), ("block", [I], None)):
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        return True

    def init(self, num_clients: int) -> bool:
        if not self.lib and not self.load_library():
            return False
        if self.lib.orion_start_scheduler(num_clients) != 0:
            print("Failed to initialize Orion scheduler")
            return False
        self.initialized = True
        return True

    def shutdown(self):
        if self.lib and self.initialized:
            self.lib.orion_stop_scheduler()
            self.initialized = False

    def set_client_idx(self, idx: int):
        if self.lib:
            self.lib.orion_set_client_idx(idx)

    def get_client_idx(self) -> int:
        return self.lib.orion_get_client_idx() if self.lib else -1

    def set_enabled(self, enabled: bool):
        if self.lib:
            self.lib.orion_set_enabled(1 if enabled else 0)

    def block(self, phase: int = 0):
        if self.lib:
            self.lib.block(phase)


# ------------------------------------------------------------------ models ---

def _vgg16():
    from torchvision.models import vgg16
    return vgg16(weights=None)


def _resnet50():
    from torchvision.models import resnet50
    return resnet50(weights=None)


def _simple():
    import torch.nn as nn
    return nn.Sequential(nn.Conv2d(3, 32, 3, padding=1), nn.BatchNorm2d(32), nn.ReLU(),
                         nn.Conv2d(32, 64, 3, padding=1), nn.BatchNorm2d(64), nn.ReLU(),
                         nn.AdaptiveAvgPool2d((1, 1)), nn.Flatten(), nn.Linear(64, 10))


MODEL_REGISTRY: dict[str, Callable] = {"resnet50": _resnet50, "vgg16": _vgg16, "simple": _simple}


def image_step(model_name: str, batch_size: int, device: str):
    """Returns a step function running inference of an image model."""
    import torch
    model = MODEL_REGISTRY.get(model_name, _simple)().to(device).eval()
    x = torch.randn(batch_size, 3, 224, 224, device=device)

    def step():
        with torch.no_grad():
            model(x)
    return step, batch_size


def gpt_train_step(batch_size: int, device: str):
    """Training step of the decoder used as BE load (batch x 256 tokens)."""
    import torch
    import torch.nn.functional as F

    from .harness import make_gpt
    model = make_gpt(device=device)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4)
    tok = torch.randint(0, 32000, (batch_size, 256), device=device)
    tgt = torch.randint(0, 32000, (batch_size, 256), device=device)

    def step():
        logits = model(tok)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]), tgt.view(-1))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
    return step, batch_size * 256


def make_step(name: str, batch_size: int, device: str):
    if name == "gpt":
        return gpt_train_step(batch_size, device)
    return image_step(name, batch_size, device)


# ----------------------------------------------------------- one GPU group ---

def percentile(xs, q):
    if not xs:
        return float("nan")
    s = sorted(xs)
    k = (len(s) - 1) * q
    f = math.floor(k)
    c = min(f + 1, len(s) - 1)
    return s[f] + (s[c] - s[f]) * (k - f)


def client_worker(scheduler: OrionScheduler | None, client_idx: int, step: Callable,
                  units_per_iter: int, num_iters: int, sync: Callable, start_barrier,
                  stop_event: threading.Event, results: dict):
    """One client thread (python/launch_jobs.py 130-208): warm-up, then
    ``num_iters`` timed iterations for HP, or iterations until HP finishes
    for BE.  Latency per HP iteration is taken after ``block`` + sync."""
    try:
        if scheduler:
            scheduler.set_client_idx(client_idx)
        for _ in range(2):
            step()
        sync()
        start_barrier.wait()
        lat = []
        t0 = time.perf_counter()
        n = 0
        while True:
            ti = time.perf_counter()
            step()
            if scheduler:
                scheduler.block(client_idx)
            sync()
            lat.append((time.perf_counter() - ti) * 1e3)
            n += 1
            if client_idx == 0 and n >= num_iters:
                break
            if client_idx != 0 and (stop_event.is_set() or (num_iters and n >= 100 * num_iters)):
                break
        elapsed = time.perf_counter() - t0
        if client_idx == 0:
            stop_event.set()
        results[client_idx] = {"client_idx": client_idx,
                               "client_type": "HP" if client_idx == 0 else "BE",
                               "num_iters": n, "elapsed_time": elapsed,
                               "throughput": n / elapsed, "units_per_s": n * units_per_iter / elapsed,
                               "latencies_ms": lat}
    except BaseException as e:  # noqa: BLE001 - reported in the results
        stop_event.set()
        results[client_idx] = {"client_idx": client_idx, "error": repr(e)}
    finally:
        if scheduler:
            scheduler.set_client_idx(-1)


def run_group(steps: list[tuple[Callable, int]], num_iters: int, scheduler=None,
              sync: Callable = lambda: None) -> dict:
    """Runs client 0 (HP) and clients 1.. (BE) of one GPU as threads."""
    num_clients = len(steps)
    barrier = threading.Barrier(num_clients)
    stop = threading.Event()
    results: dict = {}
    threads = [threading.Thread(target=client_worker,
                                args=(scheduler, i, st, units, num_iters, sync, barrier, stop,
                                      results), name=f"client{i}")
               for i, (st, units) in enumerate(steps)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    return {"clients": [results[i] for i in range(num_clients)]}


def aggregate(groups: list[dict]) -> dict:
    """Aggregate of per-GPU groups: HP p99 over all HP iterations of all
    groups, BE throughput summed (units: images or tokens per second)."""
    hp_lat = []
    be_units = 0.0
    hp_units = 0.0
    errors = []
    for g in groups:
        for c in g["clients"]:
            if "error" in c:
                errors.append((g.get("rank"), c["client_idx"], c["error"]))
                continue
            if c["client_idx"] == 0:
                hp_lat.extend(c["latencies_ms"])
                hp_units += c["units_per_s"]
            else:
                be_units += c["units_per_s"]
    return {"groups": len(groups), "hp_p50_ms": percentile(hp_lat, 0.5),
            "hp_p99_ms": percentile(hp_lat, 0.99), "hp_units_per_s": hp_units,
            "be_units_per_s": be_units, "errors": errors}


def placement(rank: int, world: int, visible: int) -> int:
    """GPU index of group `rank`: one group per GPU, never two on one GPU."""
    if world > visible:
        raise ValueError(f"{world} client groups need {world} GPUs, {visible} visible")
    return rank


def gather(result: dict, rank: int, world: int) -> list[dict] | None:
    """Collects every group's result on rank 0 over a host-side gloo group."""
    if world == 1:
        return [result]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, result)
    return out if rank == 0 else None


# ------------------------------------------------------------------ driver ---

def run_with_scheduler(hp_model_name: str, be_model_names: list[str], num_iters: int = 100,
                       batch_size: int = 1, device: str = "cuda:0") -> dict:
    import torch
    steps = [make_step(hp_model_name, batch_size, device)]
    steps += [make_step(n, batch_size, device) for n in be_model_names]
    scheduler = OrionScheduler()
    if not scheduler.init(len(steps)):
        raise RuntimeError("Failed to initialize scheduler")
    try:
        return run_group(steps, num_iters, scheduler, sync=torch.cuda.current_stream().synchronize)
    finally:
        scheduler.shutdown()


def run_baseline(model_name: str, num_iters: int = 100, batch_size: int = 1,
                 device: str = "cuda:0") -> dict:
    import torch
    step, units = make_step(model_name, batch_size, device)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(num_iters):
        step()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return {"throughput": num_iters / dt, "avg_latency_ms": dt / num_iters * 1e3}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def group_main(args) -> int:
    """Body of one placed process (rank = GPU index)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=600))
    res = run_with_scheduler(args.hp_model, args.be_models, args.num_iters, args.batch_size,
                             "cuda:0")
    res["rank"] = rank
    res["gpu"] = os.environ.get("CUDA_VISIBLE_DEVICES", "0")
    groups = gather(res, rank, world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(report(groups)), flush=True)
    return 0


def report(groups: list[dict]) -> dict:
    """Aggregate plus per-group numbers (latency lists dropped)."""
    summary = aggregate(groups)
    slim = [{**g, "clients": [{k: v for k, v in c.items() if k != "latencies_ms"}
                              for c in g["clients"]]} for g in groups]
    return {"aggregate": summary, "groups": slim}


def spawn_groups(args) -> int:
    """Starts one process per GPU with the interposer preloaded."""
    port = _free_port()
    procs = []
    for g in range(args.gpus):
        env = dict(os.environ)
        env.update({"RANK": str(g), "WORLD_SIZE": str(args.gpus), "MASTER_ADDR": "127.0.0.1",
                    "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": str(g),
                    "KX_LAUNCH_CHILD": "1"})
        pre = env.get("LD_PRELOAD", "")
        if os.path.basename(LIBSHIM) not in pre:
            env["LD_PRELOAD"] = LIBSHIM + (":" + pre if pre else "")
        cmd = [sys.executable, "-m", "kernel_intercept_b200.launch"] + sys.argv[1:]
        procs.append(subprocess.Popen(cmd, env=env))
    rc = 0
    for p in procs:
        rc |= p.wait()
    return rc


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Orion GPU Scheduler Launcher")
    ap.add_argument("--hp-model", type=str, default="simple")
    ap.add_argument("--be-models", type=str, nargs="+", default=["simple"])
    ap.add_argument("--num-iters", type=int, default=100)
    ap.add_argument("--batch-size", type=int, default=1)
    ap.add_argument("--device", type=str, default="cuda:0")
    ap.add_argument("--baseline", action="store_true")
    ap.add_argument("--list-models", action="store_true")
    ap.add_argument("--gpus", type=int, default=1, help="client groups, one per GPU")
    ap.add_argument("--gil-switch-ms", type=float, default=0.5,
                    help="sys.setswitchinterval of each group process: its HP and BE clients "
                         "are Python threads, and at Python's default of 5 ms a BE thread "
                         "can hold the GIL for 5 ms while HP waits to issue (0: default)")
    args = ap.parse_args(argv)
    if args.gil_switch_ms > 0:
        sys.setswitchinterval(args.gil_switch_ms / 1e3)
    if args.list_models:
        print("\n".join(list(MODEL_REGISTRY) + ["gpt"]))
        return 0
    if args.baseline:
        print(json.dumps(run_baseline(args.hp_model, args.num_iters, args.batch_size,
                                      args.device)))
        return 0
    if os.environ.get("KX_LAUNCH_CHILD") == "1" or args.gpus == 1 and \
            os.path.basename(LIBSHIM) in os.environ.get("LD_PRELOAD", ""):
        return group_main(args)
    return spawn_groups(args)


if __name__ == "__main__":
    sys.exit(main())
