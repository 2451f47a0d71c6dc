"""Per-client kernel tables for the Orion admission gate, from the kx kernels.

The reference builds ``kernel_info.csv`` offline from ncu captures of the
closed cuBLAS / cuDNN kernels (profile_gpt_vgg16.sh:73-286,
profiling/generate_file.py:47-179) and loads one table per client
(orion_load_kernel_info, parsed at src/scheduler.cpp:84-153); the gate at
src/scheduler.cpp:997-1034 admits a BE kernel when the HP client's next kernel
and this one fit in the GPU's SMs together (or when HP has nothing queued).
Rows are the client's kernels in execution order, one per captured op,
indexed cyclically by how many kernel ops the client has executed.

Here the table is measured in-process, through the interposer's own
profiler: each client runs one step alone with capture on, and every kernel
op its worker executes is recorded in order:
* captured dense ops (kx GEMMs, convolutions, batch norm): the kx kernel
  name, the SMs the persistent launch occupies (min(work tiles, quota, SM
  count)), the op's device time (CUDA events around the dispatch);
* kernels the interposer re-issues (PyTorch's own elementwise, softmax,
  normalisation kernels): the function name, the SMs its grid fills at the
  occupancy it reaches (blocks / resident blocks per SM), its device time.
Columns follow the reference's CSV: ``Name,Profile,Memory_footprint,
SM_usage,Duration`` with Profile 1 = compute-bound (GEMM / convolution),
0 = memory-bound (batch norm), -1 = not classified, Memory_footprint 0 and
Duration in nanoseconds.

    python -m kernel_intercept_b200.profile_tables --config 4 --out DIR

writes DIR/client0.csv (HP), DIR/client1.csv, ... for that configuration's
clients (the command re-executes itself under the interposer).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import tempfile
import threading

HEADER = "Name,Profile,Memory_footprint,SM_usage,Duration"


def _profile_class(rec: dict) -> int:
    op = rec.get("op_type", "")
    if "BATCHNORM" in op:
        return 0
    if float(rec.get("work", 0.0)) > 0:
        return 1
    return -1


def rows_from_records(recs: list[dict], client: int) -> list[tuple]:
    """(name, profile, memory, sm_usage, duration_ns) of one client's records,
    in execution order."""
    out = []
    for r in recs:
        if int(r.get("client", -1)) != client:
            continue
        name = str(r.get("kernel_id", "kernel")).replace("\n", " ")
        out.append((name, _profile_class(r), 0, int(r.get("sm_needed", 0)),
                    float(r.get("duration_ms", 0.0)) * 1e6))
    return out


def write_csv(path: str, rows: list[tuple]) -> None:
    with open(path, "w") as f:
        f.write(HEADER + "\n")
        for name, prof, mem, sm, dur in rows:
            f.write(f"{name},{prof},{mem},{sm},{dur:.1f}\n")


def read_csv(path: str) -> list[tuple]:
    """Rows of a table, parsed like the scheduler does (the last four fields
    are numeric, the name is everything before them)."""
    rows = []
    with open(path) as f:
        next(f)
        for line in f:
            line = line.rstrip("\r\n")
            if not line:
                continue
            parts = line.rsplit(",", 4)
            rows.append((parts[0], int(parts[1]), int(parts[2]), int(parts[3]), float(parts[4])))
    return rows


def _run_on_client(orion, client: int, fn) -> None:
    """Runs fn() on a thread registered as `client`, on its own stream."""
    import torch

    from .harness import client_stream
    err = []
    dev = torch.cuda.current_device()

    def body():
        try:
            torch.cuda.set_device(dev)
            s = client_stream(dev, client)
            orion.orion_set_client_idx(client)
            orion.orion_register_client_stream(client, ctypes.c_void_p(s.cuda_stream))
            with torch.cuda.stream(s):
                fn()
            s.synchronize()
        except BaseException as e:  # noqa: BLE001 - re-raised below
            err.append(e)
        finally:
            orion.orion_set_client_idx(-1)

    t = threading.Thread(target=body)
    t.start()
    t.join()
    if err:
        raise err[0]


def generate(orion, steps: list, out_dir: str) -> list[str]:
    """Profiles one step of each client alone (client i runs steps[i]) and
    writes out_dir/client<i>.csv.  Needs the scheduler running and capture
    on; each step should have been run once before (warm-up), so the
    profiled step issues the steady-state sequence of kernels."""
    os.makedirs(out_dir, exist_ok=True)
    paths = []
    orion.orion_set_profile_launches(1)
    for c, step in enumerate(steps):
        fd, tmp = tempfile.mkstemp(suffix=".json")
        os.close(fd)
        orion.orion_start_profiling(f"client{c}".encode())
        try:
            _run_on_client(orion, c, step)
        finally:
            orion.orion_end_profiling(tmp.encode())
        with open(tmp) as f:
            recs = json.load(f).get("kernels", [])
        os.unlink(tmp)
        path = os.path.join(out_dir, f"client{c}.csv")
        write_csv(path, rows_from_records(recs, c))
        paths.append(path)
    orion.orion_set_profile_launches(0)
    return paths


def load(orion, paths: list[str]) -> list[int]:
    """Loads client<i>.csv into the scheduler (fresh kernel counters first)."""
    orion.orion_reset_state()
    return [orion.orion_load_kernel_info(c, p.encode()) for c, p in enumerate(paths)]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=4, choices=[0, 1, 2, 4])
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    from . import harness
    if not harness.preloaded():
        env = harness.preload_env({"ORION_LOG_LEVEL": os.environ.get("ORION_LOG_LEVEL", "WARN")})
        os.execve(sys.executable, [sys.executable, "-m", "kernel_intercept_b200.profile_tables"] +
                  sys.argv[1:], env)
    import torch

    from . import configs
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hp, bes = configs.build(args.config, dev)
    clients = [hp] + bes
    orion = harness.Orion()
    assert orion.orion_init_scheduler(len(clients)) == 0
    orion.orion_set_capture(0)
    for c in clients:
        c.step()
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    for i, c in enumerate(clients):  # one captured warm-up step per client
        _run_on_client(orion, i, c.step)
    paths = generate(orion, [c.step for c in clients], args.out)
    orion.orion_set_capture(0)
    orion.orion_stop_scheduler()
    for p in paths:
        rows = read_csv(p)
        print(f"{p}: {len(rows)} kernels, {sum(r[4] for r in rows) / 1e6:.3f} ms")
    return 0


if __name__ == "__main__":
    sys.exit(main())
