"""numpy front end of the CPU oracle (``libkx_oracle.so``, built from kx_oracle.c).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this module, and only as the checker.
The product path never calls it.

Every function restates the semantics of one closed-library call the
kernel_intercept shim captures (citations are to the reference project):

* ``sgemm``                  cublasSgemm_v2            src/cublas_intercept.cpp:461-471
* ``sgemm_strided_batched``  cublasSgemmStridedBatched src/cublas_intercept.cpp:478-490
* ``gemm_ex``                cublasGemm(StridedBatched)Ex / cublasLtMatmul
                             src/cublas_intercept.cpp:886-1029, 1319-1500
* ``conv_fwd`` / ``conv_bwd_data`` / ``conv_bwd_filter``
                             cudnnConvolution*         src/cudnn_intercept.cpp:433-627
* ``bn_fwd_training`` / ``bn_fwd_inference`` / ``bn_bwd``
                             cudnnBatchNormalization*  src/cudnn_intercept.cpp:659-716

Matrices are passed as flat column-major buffers with explicit leading
dimensions, exactly as the cuBLAS call receives them.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libkx_oracle.so")
_lib = None
_lock = threading.Lock()

R_32F, R_16F, R_16BF = 0, 2, 14


class ConvDesc(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int) for name in (
        "n", "c", "h", "w", "k", "r", "s", "pad_h", "pad_w", "stride_h", "stride_w",
        "dil_h", "dil_w", "xcorr")]


def build(force: bool = False) -> str:
    """Compile libkx_oracle.so with the Makefile next to this file."""
    if force or not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "kx_oracle.c"))):
        subprocess.run(["make", "-s", "-C", _HERE, "libkx_oracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            f, i, d, p, ll = (ctypes.c_float, ctypes.c_int, ctypes.c_double, ctypes.c_void_p,
                              ctypes.c_longlong)
            L.kxo_sgemm.argtypes = [i, i, i, i, i, f, p, i, p, i, f, p, i]
            L.kxo_sgemm_strided_batched.argtypes = [i, i, i, i, i, f, p, i, ll, p, i, ll, f, p, i,
                                                    ll, i]
            L.kxo_gemm_ex.argtypes = [i, i, i, i, i, f, p, i, i, ll, p, i, i, ll, f, p, i, i, ll,
                                      p, i, i, ll, i, i, p, i]
            cd = ctypes.POINTER(ConvDesc)
            L.kxo_conv_fwd.argtypes = [cd, f, p, p, f, p]
            L.kxo_conv_bwd_data.argtypes = [cd, f, p, p, f, p]
            L.kxo_conv_bwd_filter.argtypes = [cd, f, p, p, f, p]
            L.kxo_bn_fwd_training.argtypes = [i, f, f, i, i, i, i, p, p, p, p, d, p, p, d, p, p]
            L.kxo_bn_fwd_inference.argtypes = [i, f, f, i, i, i, i, p, p, p, p, p, p, d]
            L.kxo_bn_bwd.argtypes = [i, f, f, f, f, i, i, i, i, p, p, p, p, p, p, d, p, p]
            L.kxo_num_threads.restype = i
            L.kxo_set_num_threads.argtypes = [i]
            L.kxo_f32_to_bf16.restype = ctypes.c_uint16
            L.kxo_f32_to_bf16.argtypes = [f]
            L.kxo_bf16_to_f32.restype = f
            L.kxo_bf16_to_f32.argtypes = [ctypes.c_uint16]
            _lib = L
    return _lib


def _ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"] or a.ndim == 1
    return a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return lib().kxo_num_threads()


def set_num_threads(n: int) -> None:
    lib().kxo_set_num_threads(int(n))


# ------------------------------------------------------------------ GEMM ---

def sgemm(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc):
    """cublasSgemm_v2 on flat float32 column-major buffers; C updated in place."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    assert C.dtype == np.float32 and C.flags["C_CONTIGUOUS"]
    lib().kxo_sgemm(transa, transb, m, n, k, alpha, _ptr(A), lda, _ptr(B), ldb, beta, _ptr(C),
                    ldc)
    return C


def sgemm_strided_batched(transa, transb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc,
                          sC, batch):
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    assert C.dtype == np.float32 and C.flags["C_CONTIGUOUS"]
    lib().kxo_sgemm_strided_batched(transa, transb, m, n, k, alpha, _ptr(A), lda, sA, _ptr(B),
                                    ldb, sB, beta, _ptr(C), ldc, sC, batch)
    return C


def gemm_ex(transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C, Ctype, ldc,
            D=None, Dtype=None, ldd=None, batch=1, sA=0, sB=0, sC=0, sD=0, epilogue=1,
            bias=None, bias_type=R_32F):
    """Typed GEMM / Lt matmul.  16-bit buffers are np.uint16 bit patterns."""
    if D is None:
        D, Dtype, ldd, sD = C, Ctype, ldc, sC
    lib().kxo_gemm_ex(transa, transb, m, n, k, alpha, _ptr(A), Atype, lda, sA, _ptr(B), Btype,
                      ldb, sB, beta, _ptr(C) if C is not None else None, Ctype, ldc, sC, _ptr(D),
                      Dtype, ldd, sD, batch, epilogue, _ptr(bias), bias_type)
    return D


# ------------------------------------------------------------- conversions --

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (np.uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7F800000) == 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = (u[nan] >> 16).astype(np.uint16) | np.where((u[nan] & 0x7FFFFF) != 0, 0x40, 0)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------- convolution ---

def conv_desc(n, c, h, w, k, r, s, pad=(0, 0), stride=(1, 1), dil=(1, 1), xcorr=True):
    return ConvDesc(n, c, h, w, k, r, s, pad[0], pad[1], stride[0], stride[1], dil[0], dil[1],
                    1 if xcorr else 0)


def conv_out_dims(d: ConvDesc):
    p = (d.h + 2 * d.pad_h - ((d.r - 1) * d.dil_h + 1)) // d.stride_h + 1
    q = (d.w + 2 * d.pad_w - ((d.s - 1) * d.dil_w + 1)) // d.stride_w + 1
    return p, q


def conv_fwd(d: ConvDesc, alpha, x, w, beta=0.0, y=None):
    p, q = conv_out_dims(d)
    if y is None:
        y = np.zeros((d.n, d.k, p, q), np.float32)
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    lib().kxo_conv_fwd(ctypes.byref(d), alpha, _ptr(x), _ptr(w), beta, _ptr(y))
    return y


def conv_bwd_data(d: ConvDesc, alpha, w, dy, beta=0.0, dx=None):
    if dx is None:
        dx = np.zeros((d.n, d.c, d.h, d.w), np.float32)
    w = np.ascontiguousarray(w, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    lib().kxo_conv_bwd_data(ctypes.byref(d), alpha, _ptr(w), _ptr(dy), beta, _ptr(dx))
    return dx


def conv_bwd_filter(d: ConvDesc, alpha, x, dy, beta=0.0, dw=None):
    if dw is None:
        dw = np.zeros((d.k, d.c, d.r, d.s), np.float32)
    x = np.ascontiguousarray(x, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    lib().kxo_conv_bwd_filter(ctypes.byref(d), alpha, _ptr(x), _ptr(dy), beta, _ptr(dw))
    return dw


# ------------------------------------------------------------ batch norm ---

def bn_fwd_training(mode, alpha, beta, x, y, scale, bias, factor, rmean, rvar, eps, smean,
                    sinv):
    n, c, h, w = x.shape
    lib().kxo_bn_fwd_training(mode, alpha, beta, n, c, h, w, _ptr(x), _ptr(y), _ptr(scale),
                              _ptr(bias), factor, _ptr(rmean), _ptr(rvar), eps, _ptr(smean),
                              _ptr(sinv))
    return y


def bn_fwd_inference(mode, alpha, beta, x, y, scale, bias, mean, var, eps):
    n, c, h, w = x.shape
    lib().kxo_bn_fwd_inference(mode, alpha, beta, n, c, h, w, _ptr(x), _ptr(y), _ptr(scale),
                               _ptr(bias), _ptr(mean), _ptr(var), eps)
    return y


def bn_bwd(mode, alpha_d, beta_d, alpha_p, beta_p, x, dy, dx, scale, dscale, dbias, eps, smean,
           sinv):
    n, c, h, w = x.shape
    lib().kxo_bn_bwd(mode, alpha_d, beta_d, alpha_p, beta_p, n, c, h, w, _ptr(x), _ptr(dy),
                     _ptr(dx), _ptr(scale), _ptr(dscale), _ptr(dbias), eps, _ptr(smean),
                     _ptr(sinv))
    return dx


# ---------------------------------------------------------------- metrics --

def normwise_rel_err(got, ref) -> float:
    """max |got-ref| / max |ref| over one output tensor (the fp32 parity metric)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.max(np.abs(ref)) if ref.size else 0.0
    num = np.max(np.abs(got - ref)) if ref.size else 0.0
    return float(num / den) if den > 0 else float(num)
