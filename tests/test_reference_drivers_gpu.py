"""The reference's own Python drivers, unmodified, against this build's interposer.

The drop-in claim: a user of the kernel_intercept project keeps running its
scripts (python/test_orion_blocking.py ``run_test``, python/launch_jobs.py
``run_with_scheduler``) with this build's ``libgpu_scheduler.so`` in place of
theirs.  The drivers find the library at ``<project>/build/libgpu_scheduler.so``
(test_orion_blocking.py:143-150) or through ORION_LIB_PATH
(launch_jobs.py:33-37) and import their models from their own directory, so
the test lays out such a project in a temporary directory: ``python/`` holds
links to the unmodified driver files and ``build/libgpu_scheduler.so`` links
to this build's interposer.  Both run under LD_PRELOAD, as the reference's
run.sh does; ORION_STATS_FILE makes the interposer write its per-client
counters when the driver stops the scheduler.  Every dense op the drivers'
models issue must run on kx (no pass-through to cuBLAS / cuDNN, no error).

The driver files come from baseline/_ref/python (copied there unmodified by
``make -C oracle ref-drivers REF=<reference checkout>``; the reference has no
installable package); the test is skipped when they are absent.
"""
import json
import os
import subprocess
import sys

import pytest

from kernel_intercept_b200 import LIBSHIM

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVERS = os.path.join(ROOT, "baseline", "_ref", "python")

pytestmark = pytest.mark.gpu


def _project(tmp_path):
    if not os.path.exists(os.path.join(DRIVERS, "test_orion_blocking.py")):
        pytest.skip("reference drivers not staged (make -C oracle ref-drivers REF=...)")
    proj = tmp_path / "project"
    (proj / "python").mkdir(parents=True)
    (proj / "build").mkdir()
    (proj / "profiles").mkdir()
    for name in os.listdir(DRIVERS):
        if name.endswith(".py"):
            os.symlink(os.path.join(DRIVERS, name), proj / "python" / name)
    os.symlink(LIBSHIM, proj / "build" / "libgpu_scheduler.so")
    return proj


def _run(proj, args, stats, timeout=900):
    env = dict(os.environ)
    env["LD_PRELOAD"] = LIBSHIM
    env["ORION_LIB_PATH"] = str(proj / "build" / "libgpu_scheduler.so")
    env["ORION_STATS_FILE"] = str(stats)
    env.setdefault("ORION_LOG_LEVEL", "WARN")
    p = subprocess.run([sys.executable] + args, cwd=proj / "python", env=env,
                       capture_output=True, text=True, timeout=timeout)
    assert p.returncode == 0, f"rc={p.returncode}\n{p.stdout[-3000:]}\n{p.stderr[-3000:]}"
    assert stats.exists(), p.stdout[-2000:] + p.stderr[-2000:]
    return json.loads(stats.read_text())["clients"], p.stdout


def _check(clients):
    assert sum(c["kx_ops"] for c in clients) > 0, clients
    for c in clients:
        assert c["passthrough_ops"] == 0 and c["errors"] == 0, clients


def test_orion_blocking_driver_unchanged(tmp_path):
    """python/test_orion_blocking.py: HP GPT + 1 BE client, 2 iterations."""
    proj = _project(tmp_path)
    clients, out = _run(proj, ["test_orion_blocking.py", "--num-be", "1", "--num-iters", "2"],
                        tmp_path / "stats_blocking.json")
    assert len(clients) == 2, clients
    _check(clients)
    assert "TEST COMPLETE" in out, out[-2000:]


def test_launch_jobs_driver_unchanged(tmp_path):
    """python/launch_jobs.py: HP VGG16 + BE simple CNN, one GPU."""
    proj = _project(tmp_path)
    clients, _ = _run(proj, ["launch_jobs.py", "--hp-model", "vgg16", "--be-models", "simple",
                             "--num-iters", "5", "--batch-size", "2"],
                      tmp_path / "stats_launch.json")
    _check(clients)
