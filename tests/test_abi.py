"""C-ABI surface checks (CPU only, no compute calls).

* libkx.so loads and exports every function include/kx.h declares, and
  nothing else.
* libgpu_scheduler.so exports the reference interposer's symbol set (the
  exported names of the reference's src/*.cpp: the CUDA runtime / driver,
  cuBLAS / cuBLASLt and cuDNN wrappers and the orion_* API), plus the
  additions (block, the batch-norm and backend-graph cuDNN entry points,
  event wrappers) — except dlsym, which this interposer deliberately does not
  replace.
* The host-only parts of the orion_* API behave as the reference's drivers
  expect (test/test_basic.py 34-52 calls them the same way).
"""
import ctypes
import os
import re
import subprocess
import sys

import pytest

from kernel_intercept_b200 import LIBKX, LIBSHIM

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REFERENCE_EXPORTS = """
cudaMalloc cudaFree cudaMemcpy cudaMemcpyAsync cudaMemset cudaMemsetAsync cudaLaunchKernel
__cudaLaunchKernel cudaLaunchKernelExC cuLaunchKernel cudaDeviceSynchronize cudaStreamSynchronize
cudaStreamGetCaptureInfo_v2 cudaStreamIsCapturing
cublasSgemm_v2 cublasSgemmBatched cublasSgemmStridedBatched cublasGemmEx cublasGemmStridedBatchedEx
cublasHgemm cublasHgemmStridedBatched cublasSgemmEx cublasSetStream_v2 cublasLtMatmul
cudnnConvolutionForward cudnnConvolutionBackwardData cudnnConvolutionBackwardFilter
cudnnBatchNormalizationForwardTraining cudnnSetStream
orion_init orion_shutdown orion_set_client_idx orion_get_client_idx orion_set_enabled
orion_is_enabled orion_set_capture orion_register_client_stream orion_register_client_handle
orion_resolve_client_idx orion_init_scheduler orion_start_scheduler_thread orion_start_scheduler
orion_stop_scheduler orion_load_kernel_info orion_set_client_kernels orion_set_sm_threshold
orion_get_sm_threshold orion_sync_client_stream orion_reset_state orion_autotune_green_ctx
orion_set_async_mode orion_get_async_mode orion_load_profile orion_start_profiling
orion_end_profiling
""".split()

ADDED_EXPORTS = """
block cudnnBatchNormalizationForwardInference cudnnBatchNormalizationBackward
cudnnBatchNormalizationForwardTrainingEx cudnnBatchNormalizationBackwardEx cudnnBackendExecute
cudnnBackendDestroyDescriptor cudnnBackendCreateDescriptor cudnnBackendSetAttribute
cudnnBackendGetAttribute cudnnBackendFinalize cudaEventRecord cudaEventRecordWithFlags cudaStreamWaitEvent
cudaEventSynchronize cudaEventQuery cudaStreamQuery orion_set_be_keep_sms orion_get_be_keep_sms
orion_set_sm_budgets orion_get_client_stats orion_op_log_start orion_op_log_end
orion_get_client_waits orion_trace_start orion_trace_end orion_set_profile_launches
orion_set_be_host_hold_us orion_get_be_host_hold_us orion_get_client_host_holds
orion_set_profile_every
""".split()


def _ensure_built():
    if not (os.path.exists(LIBKX) and os.path.exists(LIBSHIM)):
        from kernel_intercept_b200 import build
        build.build_all()


def dynamic_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], check=True, capture_output=True,
                         text=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if ln.strip()}


def declared_kx_functions():
    text = open(os.path.join(ROOT, "include", "kx.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(kx_[a-z0-9_]+)\s*\(", text))


def test_kx_exports_match_header():
    _ensure_built()
    declared = declared_kx_functions()
    assert len(declared) >= 20
    syms = dynamic_symbols(LIBKX)
    exported = {s for s in syms if s.startswith("kx_")}
    assert declared - exported == set(), declared - exported
    assert exported - declared == set(), exported - declared
    # nothing else leaks (static cudart, C++ internals stay local)
    others = {s for s in syms if not s.startswith("kx_")}
    assert others == set(), sorted(others)[:20]


def test_kx_loads_without_gpu():
    _ensure_built()
    lib = ctypes.CDLL(LIBKX)
    for name in declared_kx_functions():
        assert getattr(lib, name) is not None
    lib.kx_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.kx_version()


def test_interposer_exports_reference_symbols():
    _ensure_built()
    syms = dynamic_symbols(LIBSHIM)
    missing = [s for s in REFERENCE_EXPORTS if s not in syms]
    assert missing == [], missing
    missing = [s for s in ADDED_EXPORTS if s not in syms]
    assert missing == [], missing
    # dlsym is not replaced: lookups by name keep libdl's behaviour
    assert "dlsym" not in syms


def test_headers_compile_as_cxx():
    src = "\n".join(f'#include "{h}"' for h in
                    ("common.h", "gpu_capture.h", "kernel_profile.h", "scheduler.h", "kx.h"))
    src += "\nint main() { return 0; }\n"
    p = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-x", "c++", "-",
                        "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include"],
                       input=src, capture_output=True, text=True)
    assert p.returncode == 0, p.stderr


def test_kx_header_compiles_as_c():
    p = subprocess.run(["gcc", "-std=c99", "-fsyntax-only", "-x", "c", "-",
                        "-I", os.path.join(ROOT, "include")],
                       input='#include "kx.h"\nint main(void) { return 0; }\n',
                       capture_output=True, text=True)
    assert p.returncode == 0, p.stderr


HOST_API_SCRIPT = r"""
import ctypes, sys
L = ctypes.CDLL(sys.argv[1])
assert L.orion_init(2) == 0
L.orion_set_client_idx(1); assert L.orion_get_client_idx() == 1
L.orion_set_client_idx(-1)
L.orion_register_client_stream(0, ctypes.c_void_p(0xabc0))
assert L.orion_resolve_client_idx(ctypes.c_void_p(0xabc0), None) == 0
assert L.orion_set_capture(0) == 0 and L.orion_is_enabled() == 0
L.orion_set_enabled(1); assert L.orion_is_enabled() == 1
L.orion_set_async_mode(0); assert L.orion_get_async_mode() == 0
L.orion_set_be_keep_sms(24); assert L.orion_get_be_keep_sms() == 24
L.orion_set_be_host_hold_us(300); assert L.orion_get_be_host_hold_us() == 300
L.orion_set_be_host_hold_us(0); assert L.orion_get_be_host_hold_us() == 0
L.orion_set_profile_every(4); L.orion_set_profile_every(1)
L.orion_get_client_host_holds.restype = ctypes.c_ulonglong
assert L.orion_get_client_host_holds(1) == 0 and L.orion_get_client_host_holds(99) == 0
out = (ctypes.c_ulonglong * 6)()
assert L.orion_get_client_stats(1, out) == 0 and list(out) == [0] * 6
assert L.orion_get_client_stats(99, out) != 0
w = (ctypes.c_ulonglong * 8)()
assert L.orion_get_client_waits(0, w, 1) == 0 and list(w) == [0] * 8
assert L.orion_get_client_waits(99, w, 0) != 0
# capture trace: an empty trace is valid Chrome-trace JSON naming every track
import json, os, tempfile
path = os.path.join(tempfile.mkdtemp(), "t.json")
L.orion_trace_start()
assert L.orion_trace_end(path.encode()) == 0
ev = json.load(open(path))["traceEvents"]
names = {e["args"]["name"] for e in ev if e["ph"] == "M"}
assert {"HP-Client", "HP-Worker", "BE1-Client", "BE1-Worker", "Scheduler"} <= names, names
L.orion_shutdown()
print("ok")
"""


def test_orion_host_api_without_gpu():
    _ensure_built()
    p = subprocess.run([sys.executable, "-c", HOST_API_SCRIPT, LIBSHIM], capture_output=True,
                       text=True, timeout=120, env=dict(os.environ, ORION_LOG_LEVEL="ERROR"))
    assert p.returncode == 0 and "ok" in p.stdout, p.stdout + p.stderr


@pytest.mark.parametrize("name", ["kx_gemm_tc_f32x3", "kx_gemm_tc_bf16", "kx_conv", "kx_bn"])
def test_cuda_sources_target_sm100a(name):
    """Every CUDA translation unit is built for sm_100a only (build flags)."""
    from kernel_intercept_b200 import build
    flags = " ".join(build.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert os.path.exists(os.path.join(ROOT, "kernel_intercept_b200", "csrc", name + ".cu"))
