"""Generates the golden fixtures that pin the CPU oracle to the reference.

Run on a GPU machine from the repository root:

    make -C oracle ref           # (where the reference tree exists) builds
                                 # oracle/_ref/libgpu_scheduler.so from the
                                 # reference's own sources
    python tests/golden/make_golden.py

The script re-executes itself with ``LD_PRELOAD=oracle/_ref/libgpu_scheduler.so``
(the unmodified reference shim) and drives its public API exactly like the
reference drivers do (``orion_init_scheduler``, ``orion_set_client_idx``,
``orion_start_scheduler_thread``, ``orion_set_capture``; cf. the reference's
python/test_orion_blocking.py:209-380).  GEMMs are issued as
``cublasSgemm_v2`` / ``cublasSgemmStridedBatched`` / ``cublasGemmEx`` calls
resolved through the global symbol scope, so they enter the shim's wrappers
(src/cublas_intercept.cpp:576, 763, 886), are queued to its worker and executed
by the real cuBLAS (src/cublas_intercept.cpp:455-491).  ORION_ASYNC_MODE=0 makes
the client wait for the worker.

PyTorch reaches cuDNN convolutions through cuDNN's backend API rather than the
legacy entry points the shim wraps, so convolution fixtures are produced by
``torch.nn.functional.conv2d`` and its autograd (cuDNN, TF32 disabled) on the
same B200; they pin the oracle to cuDNN's results, not to the shim.

Batch-norm fixtures come from cuDNN's batch norm (``aten::cudnn_batch_norm``
and its backward, the calls behind PyTorch's ``batch_norm`` on CUDA) at
VGG-like shapes (N = 64, C in {64, 512}, H = W in {14, 56}).  Their inputs are
too large to store, so the fixture holds the seed they are regenerated from
(``bn_inputs``), the per-channel outputs in full and two images x three
channels of y and dx.

Each fixture is a small ``.npz`` with the seeded inputs (or their seed), the
call's arguments and the library's output.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF_SHIM = os.path.join(ROOT, "oracle", "_ref", "libgpu_scheduler.so")
# where fixtures are written (default: next to this script)
OUT = os.environ.get("KX_GOLDEN_DIR", HERE)


def _parent() -> int:
    if not os.path.exists(REF_SHIM):
        print(f"missing {REF_SHIM}; build it with make -C oracle ref", file=sys.stderr)
        return 2
    env = dict(os.environ)
    env["LD_PRELOAD"] = REF_SHIM
    env["ORION_ASYNC_MODE"] = "0"
    env["ORION_LOG_LEVEL"] = "WARN"
    env["KX_GOLDEN_CHILD"] = "gemm"
    rc = subprocess.run([sys.executable, os.path.abspath(__file__)], env=env,
                        timeout=300).returncode
    # convolutions do not pass through the shim: run them without the preload
    env = dict(os.environ)
    env.pop("LD_PRELOAD", None)
    env["KX_GOLDEN_CHILD"] = "conv"
    rc2 = subprocess.run([sys.executable, os.path.abspath(__file__)], env=env,
                         timeout=300).returncode
    return rc or rc2


def _child_gemm() -> int:
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.zeros(1, device="cuda")
    g = ctypes.CDLL(None)  # global scope: the preloaded reference shim comes first
    for name in ("orion_init_scheduler", "orion_start_scheduler_thread", "orion_set_capture",
                 "orion_set_client_idx", "orion_sync_client_stream", "orion_register_client_handle"):
        assert hasattr(g, name), f"reference shim does not export {name}"
    handle = ctypes.c_void_p(torch.cuda.current_blas_handle())
    P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    fp = ctypes.POINTER(ctypes.c_float)
    g.cublasSgemm_v2.argtypes = [P, I, I, I, I, I, fp, P, I, P, I, fp, P, I]
    g.cublasSgemmStridedBatched.argtypes = [P, I, I, I, I, I, fp, P, I, LL, P, I, LL, fp, P, I,
                                            LL, I]
    g.cublasGemmEx.argtypes = [P, I, I, I, I, I, P, P, I, I, P, I, I, P, P, I, I, I, I]
    for f in (g.cublasSgemm_v2, g.cublasSgemmStridedBatched, g.cublasGemmEx):
        f.restype = I

    assert g.orion_init_scheduler(1) == 0
    g.orion_set_capture(0)
    g.orion_start_scheduler_thread()

    def captured(fn, *args):
        g.orion_set_capture(1)
        g.orion_set_client_idx(0)
        st = fn(*args)
        g.orion_set_client_idx(-1)
        g.orion_set_capture(0)
        g.orion_sync_client_stream(0)
        torch.cuda.synchronize()
        assert st == 0, f"reference call returned {st}"

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    a_ = lambda x: ctypes.byref(ctypes.c_float(x))  # noqa: E731
    written = []

    # ---- cublasSgemm_v2 through the shim's queue + worker ------------------
    cases = [(0, 0, 77, 65, 93, (3, 5, 2), 1.5, 0.5), (0, 1, 77, 65, 93, (0, 4, 0), 1.5, 0.5),
             (1, 0, 77, 65, 93, (1, 0, 7), 1.5, 0.5), (1, 1, 77, 65, 93, (2, 2, 2), -1.0, 2.0),
             (1, 0, 128, 128, 128, (0, 0, 0), 1.0, 0.0), (1, 0, 64, 192, 512, (0, 0, 0), 1.0, 0.0)]
    for i, (ta, tb, m, n, k, pads, alpha, beta) in enumerate(cases):
        rng = np.random.default_rng(100 + i)
        lda = (m if ta == 0 else k) + pads[0]
        ldb = (k if tb == 0 else n) + pads[1]
        ldc = m + pads[2]
        A = rng.standard_normal(lda * (k if ta == 0 else m)).astype(np.float32)
        B = rng.standard_normal(ldb * (n if tb == 0 else k)).astype(np.float32)
        C = rng.standard_normal(ldc * n).astype(np.float32)
        dA, dB, dC = dev(A), dev(B), dev(C)
        captured(g.cublasSgemm_v2, handle, ta, tb, m, n, k, a_(alpha), dA.data_ptr(), lda,
                 dB.data_ptr(), ldb, a_(beta), dC.data_ptr(), ldc)
        path = os.path.join(HERE, f"sgemm_{i}.npz")
        np.savez_compressed(path, kind="sgemm", dims=np.array([ta, tb, m, n, k, lda, ldb, ldc]),
                            scalars=np.array([alpha, beta]), A=A, B=B, C_in=C,
                            C_out=dC.cpu().numpy())
        written.append(path)

    # ---- cublasSgemmStridedBatched ------------------------------------------
    rng = np.random.default_rng(200)
    ta, tb, m, n, k, batch = 1, 0, 64, 48, 32, 4
    lda, ldb, ldc = k, k, m
    sA, sB, sC = k * m + 8, k * n + 4, m * n
    A = rng.standard_normal(sA * batch).astype(np.float32)
    B = rng.standard_normal(sB * batch).astype(np.float32)
    C = rng.standard_normal(sC * batch).astype(np.float32)
    dA, dB, dC = dev(A), dev(B), dev(C)
    captured(g.cublasSgemmStridedBatched, handle, ta, tb, m, n, k, a_(0.5), dA.data_ptr(), lda,
             sA, dB.data_ptr(), ldb, sB, a_(1.0), dC.data_ptr(), ldc, sC, batch)
    path = os.path.join(HERE, "sgemm_strided_batched_0.npz")
    np.savez_compressed(path, kind="sgemm_strided_batched",
                        dims=np.array([ta, tb, m, n, k, lda, ldb, ldc, sA, sB, sC, batch]),
                        scalars=np.array([0.5, 1.0]), A=A, B=B, C_in=C, C_out=dC.cpu().numpy())
    written.append(path)

    # ---- cublasGemmEx, bf16 in / bf16 out, fp32 compute (inline in the shim) --
    for i, (ta, tb, m, n, k) in enumerate([(0, 0, 96, 80, 64), (1, 0, 128, 128, 256)]):
        rng = np.random.default_rng(300 + i)
        lda = m if ta == 0 else k
        ldb = k if tb == 0 else n
        At = torch.from_numpy(rng.standard_normal(lda * (k if ta == 0 else m)).astype(np.float32))
        Bt = torch.from_numpy(rng.standard_normal(ldb * (n if tb == 0 else k)).astype(np.float32))
        dA = At.to(torch.bfloat16).cuda()
        dB = Bt.to(torch.bfloat16).cuda()
        dC = torch.zeros(m * n, dtype=torch.bfloat16, device="cuda")
        one, zero = ctypes.c_float(1.0), ctypes.c_float(0.0)
        captured(g.cublasGemmEx, handle, ta, tb, m, n, k, ctypes.byref(one), dA.data_ptr(), 14,
                 lda, dB.data_ptr(), 14, ldb, ctypes.byref(zero), dC.data_ptr(), 14, m, 68, -1)
        bits = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        path = os.path.join(HERE, f"gemm_ex_bf16_{i}.npz")
        np.savez_compressed(path, kind="gemm_ex_bf16", dims=np.array([ta, tb, m, n, k, lda, ldb, m]),
                            A=bits(dA), B=bits(dB), C_out=bits(dC))
        written.append(path)

    for p in written:
        print(os.path.relpath(p, ROOT), os.path.getsize(p), flush=True)
    # The reference's orion_stop_scheduler can block in its worker join; the
    # fixtures are written, so leave without tearing the shim down.
    sys.stdout.flush()
    os._exit(0)


def bn_inputs(shape, seed):
    """Inputs of a batch-norm fixture, regenerated from its seed:
    x, scale, bias, running mean, running var, dy (float32)."""
    n, c, h, w = shape
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(shape, dtype=np.float32) * 3 + 2).astype(np.float32)
    scale = (rng.random(c) + 0.5).astype(np.float32)
    bias = rng.standard_normal(c).astype(np.float32)
    rm = rng.standard_normal(c).astype(np.float32)
    rv = (rng.random(c) + 0.5).astype(np.float32)
    dy = rng.standard_normal(shape, dtype=np.float32)
    return x, scale, bias, rm, rv, dy


BN_SHAPES = [(64, 64, 56, 56), (64, 64, 14, 14), (64, 512, 56, 56), (64, 512, 14, 14)]
BN_FACTOR, BN_EPS = 0.1, 1e-5


def bn_sample(shape):
    """Images and channels of y / dx stored in a batch-norm fixture."""
    n, c = shape[0], shape[1]
    return np.array([0, n - 1]), np.array([0, c // 2, c - 1])


def _child_bn() -> list:
    import torch
    written = []
    for i, shape in enumerate(BN_SHAPES):
        seed = 500 + i
        x, scale, bias, rm, rv, dy = bn_inputs(shape, seed)
        t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        rmt, rvt = t(rm), t(rv)
        y, smean, sinv, reserve = torch.ops.aten.cudnn_batch_norm(
            t(x), t(scale), t(bias), rmt, rvt, True, BN_FACTOR, BN_EPS)
        dx, dscale, dbias = torch.ops.aten.cudnn_batch_norm_backward(
            t(x), t(dy), t(scale), rmt, rvt, smean, sinv, BN_EPS, reserve)
        torch.cuda.synchronize()
        ni, ci = bn_sample(shape)
        sl = lambda a: a.cpu().numpy()[ni][:, ci]  # noqa: E731
        os.makedirs(OUT, exist_ok=True)
        path = os.path.join(OUT, f"bn_spatial_{i}.npz")
        np.savez_compressed(path, kind="bn_spatial", dims=np.array(shape), seed=seed,
                            scalars=np.array([BN_FACTOR, BN_EPS]), y=sl(y), dx=sl(dx),
                            running_mean=rmt.cpu().numpy(), running_var=rvt.cpu().numpy(),
                            save_mean=smean.cpu().numpy(), save_inv_std=sinv.cpu().numpy(),
                            dscale=dscale.cpu().numpy(), dbias=dbias.cpu().numpy())
        written.append(path)
        del x, dy, y, dx, reserve
    return written


def _child_conv() -> int:
    import torch

    torch.backends.cudnn.allow_tf32 = False
    written = []
    # ---- cuDNN convolutions (via PyTorch, TF32 off) ---------------------------
    conv_cases = [(2, 8, 12, 12, 16, 3, 3, (1, 1), (1, 1), (1, 1)),
                  (2, 5, 13, 11, 7, 3, 3, (0, 1), (2, 1), (1, 1))]
    for i, (n, c, h, w, k, r, s, pad, stride, dil) in enumerate(conv_cases):
        rng = np.random.default_rng(400 + i)
        x = rng.standard_normal((n, c, h, w)).astype(np.float32)
        wt = rng.standard_normal((k, c, r, s)).astype(np.float32)
        xt = torch.from_numpy(x).cuda().requires_grad_()
        wtt = torch.from_numpy(wt).cuda().requires_grad_()
        y = torch.nn.functional.conv2d(xt, wtt, stride=stride, padding=pad, dilation=dil)
        dy = torch.from_numpy(rng.standard_normal(tuple(y.shape)).astype(np.float32)).cuda()
        y.backward(dy)
        dims = np.array([n, c, h, w, k, r, s, pad[0], pad[1], stride[0], stride[1], dil[0], dil[1]])
        for kind, out, extra in (("conv_fwd", y.detach(), {"x": x, "w": wt}),
                                 ("conv_bwd_data", xt.grad, {"w": wt, "dy": dy.cpu().numpy()}),
                                 ("conv_bwd_filter", wtt.grad, {"x": x, "dy": dy.cpu().numpy()})):
            path = os.path.join(HERE, f"{kind}_{i}.npz")
            np.savez_compressed(path, kind=kind, dims=dims, out=out.cpu().numpy(), **extra)
            written.append(path)
    written += _child_bn()
    for p in written:
        print(os.path.relpath(p, ROOT), os.path.getsize(p))
    return 0


if __name__ == "__main__":
    mode = os.environ.get("KX_GOLDEN_CHILD")
    if mode == "gemm":
        sys.exit(_child_gemm())
    if mode == "conv":
        sys.exit(_child_conv())
    if mode == "bn":  # batch-norm fixtures alone (no preload needed)
        for p in _child_bn():
            print(p, os.path.getsize(p))
        sys.exit(0)
    sys.exit(_parent())
