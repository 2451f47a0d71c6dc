"""Interposer (libgpu_scheduler.so) parity on the GPU.

Each test starts tests/shim_child.py under LD_PRELOAD, the way the
reference's drivers run (run.sh under LD_PRELOAD; python/test_orion_blocking.py
``run_test``), so PyTorch's own cuBLAS / cuBLASLt / cuDNN calls are the ones
intercepted.  The child compares each captured op (executed by the worker on
the kx kernels) with the same op through the real libraries with capture off
and TF32 disabled.  Tolerances: fp32 max normwise relative error 1e-5; bf16
1e-2 against the real library's fp32-accumulated result.
"""
import json
import os
import subprocess
import sys

import pytest

from kernel_intercept_b200 import LIBKX, LIBSHIM

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHILD = os.path.join(ROOT, "tests", "shim_child.py")

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 1e-2


def run_child(scenario, timeout=400, extra_env=None):
    if not (os.path.exists(LIBSHIM) and os.path.exists(LIBKX)):
        pytest.fail("libgpu_scheduler.so / libkx.so not built")
    env = dict(os.environ)
    env["LD_PRELOAD"] = LIBSHIM
    env.setdefault("ORION_LOG_LEVEL", "WARN")
    if extra_env:
        env.update(extra_env)
    p = subprocess.run([sys.executable, CHILD, scenario], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=timeout)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert p.returncode == 0 and lines, (
        f"child {scenario} rc={p.returncode}\nstdout:\n{p.stdout[-3000:]}\n"
        f"stderr:\n{p.stderr[-3000:]}")
    return json.loads(lines[-1])


def test_gemm_ops_through_interposer():
    res = run_child("gemm")
    st = res["stats"]
    assert st["errors"] == 0, st
    assert st["kx_ops"] >= len(res["errors"]), st
    for name, err in res["errors"].items():
        tol = BF16_TOL if res["dtypes"][name] == "bf16" else F32_TOL
        assert err <= tol, (name, err)


def test_conv_fwd_dgrad_wgrad_through_interposer():
    res = run_child("conv")
    st = res["stats"]
    assert st["errors"] == 0, st
    assert st["kx_ops"] >= 15, st  # 5 shapes x (fwd, dgrad, wgrad)
    for name, err in res["errors"].items():
        assert err <= F32_TOL, (name, err)


def test_batchnorm_through_interposer():
    res = run_child("bn")
    st = res["stats"]
    assert st["errors"] == 0, st
    assert st["kx_ops"] >= 9, st  # 3 shapes x (training fwd, bwd, inference)
    for name, err in res["errors"].items():
        assert err <= F32_TOL, (name, err)


def test_fp16_and_sgemmex_through_interposer():
    """cublasHgemm / cublasHgemmStridedBatched (fp16, kx accumulates in fp32)
    and cublasSgemmEx run on kx when captured, none of them on the real
    cuBLAS; results within the 16-bit tolerance of a float64 product, as the
    real library's are."""
    res = run_child("hgemm")
    st = res["stats"]
    assert st["errors"] == 0 and st["passthrough_ops"] == 0, st
    assert st["kx_ops"] == 4, st
    for name, (st_real, st_cap) in res["status"].items():
        assert st_real == 0 and st_cap == 0, (name, st_real, st_cap)
    for name, err in res["errors"].items():
        assert err <= BF16_TOL, (name, err, res["real_errors"][name])


def test_gpt_forward_through_interposer():
    res = run_child("gpt")
    st = res["stats"]
    assert st["errors"] == 0, st
    assert st["kx_ops"] > 200, st  # 144 per-head GEMMs + 96 batched + Lt per forward
    assert res["errors"]["logits"] <= F32_TOL, res


def test_vgg16_forward_through_interposer():
    """The HP model of the VGG16 configuration, batch 32, end to end: every
    convolution and classifier GEMM on kx, within 1e-5 of a float64 forward
    (cuDNN's own fp32 forward is reported beside it)."""
    res = run_child("vgg16", timeout=600)
    st = res["stats"]
    assert st["errors"] == 0 and st["passthrough_ops"] == 0, st
    assert st["kx_ops"] >= 16, st  # 13 convolutions + 3 classifier GEMMs
    e = res["errors"]
    assert e["kx_vs_f64"] <= F32_TOL, e
    assert e["kx_vs_lib"] <= e["lib_vs_f64"] + F32_TOL, e


def test_llama_bf16_forward_through_interposer():
    """The HP model of the LLaMA configuration (bf16, batch 4 x 1024) end to
    end on kx: no further from an fp32 copy of the model than cuBLAS's own
    bf16 forward is, within the bf16 tolerance."""
    res = run_child("llama", timeout=600)
    st = res["stats"]
    assert st["errors"] == 0 and st["passthrough_ops"] == 0, st
    assert st["kx_ops"] >= 12 * 9 + 1, st  # per layer 7 projections + 2 attention bmm; head
    e = res["errors"]
    assert e["kx_vs_f32"] <= max(BF16_TOL, 1.25 * e["lib_vs_f32"]), e
    assert e["kx_vs_lib"] <= BF16_TOL + e["lib_vs_f32"], e


def test_gpt_training_step_through_interposer():
    """One BE training step of the GPT configuration (batch 16 x 256): loss
    and weight gradients on kx no further from a float64 step than the real
    libraries' fp32 step is, plus 1e-5."""
    res = run_child("gpt_train", timeout=600)
    st = res["stats"]
    assert st["errors"] == 0 and st["passthrough_ops"] == 0, st
    for name, e in res["errors"].items():
        assert e["kx_vs_f64"] <= e["lib_vs_f64"] + F32_TOL, (name, e)


def test_gpt_loss_curve_through_interposer():
    """20 AdamW steps of a two-layer GPT from one seed: at every step the loss
    on kx is no further from the float64 run than the real libraries' fp32
    loss is, plus 1e-5, and so are the parameters after the last step."""
    res = run_child("gpt_curve", timeout=900)
    st = res["stats"]
    assert st["errors"] == 0 and st["passthrough_ops"] == 0, st
    assert res["curve64"][-1] < res["curve64"][0], res["curve64"]  # it trains
    for i, (ek, el) in enumerate(zip(res["loss_err_kx"], res["loss_err_lib"])):
        assert ek <= el + F32_TOL, (i, ek, el)
    assert res["param_err_kx"] <= res["param_err_lib"] + F32_TOL, res


def test_hp_be_clients_contend():
    res = run_child("hpbe")
    for c in ("0", "1"):
        assert res["stats"][c]["errors"] == 0, res
    assert res["errors"]["hp"] <= F32_TOL and res["errors"]["be"] <= F32_TOL, res
    assert res["be_iters"] >= 1


def test_be_clients_stop_and_resume_under_hp():
    """Two BE clients whose GEMMs and convolutions stop entirely while HP works
    (KX_BE_KEEP_SMS=0) and are relaunched from their tile queues: every
    result exact, batch norm (which cannot stop) applied once per call."""
    res = run_child("hpbe2", extra_env={"KX_BE_KEEP_SMS": "0"})
    for c in ("0", "1", "2"):
        assert res["stats"][c]["errors"] == 0, res
    for name, err in res["errors"].items():
        assert err <= F32_TOL, (name, err, res)
    assert min(res["be_iters"]) >= 1, res


def test_capture_keeps_op_order_and_counts():
    """The interposer's op log: a GPT training step through the real
    libraries and the same step captured on the kx kernels issue the same
    calls (type, shape, transposes, dtype) in the same order; the worker runs
    the captured ops in that order; under HP + BE contention each client's
    sequence is its solo sequence, step after step."""
    res = run_child("oplog")
    assert res["n_real"] > 50 and res["n_real"] == res["n_cap"], res
    assert res["same_sequence"], res
    assert res["real_routes"] == ["real"], res
    assert res["cap_routes"] == ["capture"], res
    assert res["clients"] == [0], res
    assert res["dispatch_order_same"], res
    assert res["hp_matches_solo"] and res["hp_steps_logged"] == 4, res
    assert res["be_matches_solo"] and res["be_steps_logged"] >= 1, res
    for c in ("0", "1"):
        assert res["stats"][c]["errors"] == 0, res



def test_capture_trace():
    """orion_trace_start / orion_trace_end: a Chrome trace of an HP + BE run
    holds every captured op as an issue instant on its client's track and an
    execution span on its worker's track (same op id, issued before it ran),
    the HP client's blocking waits, and the HP flag being raised."""
    res = run_child("trace")
    assert res["events"] > 0 and res["json_events"] > res["events"], res
    for t in ("HP-Client", "HP-Worker", "BE1-Client", "BE1-Worker", "Scheduler"):
        assert t in res["names"], res
    assert res["hp_gemms"] >= 22 and res["be_gemms"] >= 1, res
    assert res["spans_matched"] and res["nonneg"], res
    assert "hp_flag_raise" in res["flag_markers"], res
    assert any(w.startswith("wait ") for w in res["hp_waits"]), res
    assert res["waits"]["0"]["waits"] >= 1, res


def test_kernel_tables_and_admission_gate():
    """Kernel tables from the interposer's profiler: one row per kernel op of
    a step (captured GEMMs classed compute-bound, re-issued kernels with the
    SMs their grid fills), loadable by orion_load_kernel_info; with them the
    Orion gate holds BE's long re-issued kernel back while HP is active."""
    res = run_child("tables")
    # every captured dense op and every re-issued kernel of the step; other
    # executed ops (copies, allocations) have no row
    for rows, ops, kx_ops in zip(res["rows"], res["step_ops"], res["step_kx_ops"]):
        assert kx_ops <= rows <= ops, res
    assert res["step_kx_ops"][1] == 1 and res["rows"][1] == 2, res
    assert res["loaded"] == res["rows"], res
    assert res["sm_ok"] and res["dur_ok"] and res["names_ok"], res
    assert res["hp_gemm_rows"] > 0 and 1 in res["hp_profiles"], res
    assert res["be_blocked"] > 0, res
    for c in ("0", "1"):
        assert res["stats"][c]["errors"] == 0, res
