"""ctypes front end of ``libkx.so`` (the kx C ABI in include/kx.h).

The functions here take raw device pointers (ints) exactly like the C ABI, plus
thin torch conveniences (``mm``, ``conv2d``...) used by tests and the harness.
There is no host or library fallback: if ``libkx.so`` is missing, or CUDA is
unavailable, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIBKX_PATH = os.path.join(PKG, "libkx.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_DEVICE, ERR_NOMEM, YIELDED = range(7)
OP_N, OP_T = 0, 1
R_32F, R_16F, R_16BF = 0, 2, 14
FP32_3XTF32, FP32_TF32, FP32_FFMA = 0, 1, 2
EPI_DEFAULT, EPI_RELU, EPI_BIAS, EPI_RELU_BIAS, EPI_GELU, EPI_GELU_BIAS = 1, 2, 4, 6, 32, 36

STATUS_NAMES = {0: "KX_OK", 1: "KX_ERR_INVALID", 2: "KX_ERR_UNSUPPORTED", 3: "KX_ERR_TIMEOUT",
                4: "KX_ERR_DEVICE", 5: "KX_ERR_NOMEM", 6: "KX_YIELDED"}


class KxError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} returned {STATUS_NAMES.get(status, status)}")
        self.status = status


class Exec(ctypes.Structure):
    """Mirror of ``kx_exec``."""
    _fields_ = [
        ("stream", ctypes.c_void_p),
        ("sm_quota", ctypes.c_int),
        ("yield_flag", ctypes.c_void_p),
        ("done_flag", ctypes.c_void_p),
        ("max_tiles", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("fp32_mode", ctypes.c_int),
        ("err_word", ctypes.c_void_p),
        ("scalars_on_device", ctypes.c_int),
    ]


class ConvDesc(ctypes.Structure):
    """Mirror of ``kx_conv_desc``."""
    _fields_ = [(f, ctypes.c_int) for f in (
        "n", "c", "h", "w", "k", "r", "s", "pad_h", "pad_w", "stride_h", "stride_w", "dil_h",
        "dil_w", "cross_correlation")]


_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_D = ctypes.c_double
_FP = ctypes.POINTER(ctypes.c_float)
_EP = ctypes.POINTER(Exec)
_CD = ctypes.POINTER(ConvDesc)

_SIGNATURES = {
    "kx_sgemm": [_EP, _I, _I, _I, _I, _I, _P, _P, _I, _P, _I, _P, _P, _I],
    "kx_sgemm_strided_batched": [_EP, _I, _I, _I, _I, _I, _P, _P, _I, _LL, _P, _I, _LL, _P, _P,
                                 _I, _LL, _I],
    "kx_sgemm_batched": [_EP, _I, _I, _I, _I, _I, _P, _P, _I, _P, _I, _P, _P, _I, _I],
    "kx_gemm_ex": [_EP, _I, _I, _I, _I, _I, _P, _P, _I, _I, _P, _I, _I, _P, _P, _I, _I],
    "kx_gemm_strided_batched_ex": [_EP, _I, _I, _I, _I, _I, _P, _P, _I, _I, _LL, _P, _I, _I, _LL,
                                   _P, _P, _I, _I, _LL, _I],
    "kx_matmul": [_EP, _I, _I, _I, _I, _I, _P, _P, _I, _I, _LL, _P, _I, _I, _LL, _P, _P, _I, _I,
                  _LL, _P, _I, _I, _LL, _I, _I, _P, _I],
    "kx_conv_out_dims": [_CD, ctypes.POINTER(_I), ctypes.POINTER(_I)],
    "kx_conv_fwd": [_EP, _CD, _P, _P, _P, _P, _P],
    "kx_conv_bwd_data": [_EP, _CD, _P, _P, _P, _P, _P],
    "kx_conv_bwd_filter": [_EP, _CD, _P, _P, _P, _P, _P],
    "kx_bn_fwd_training": [_EP, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _D, _P, _P, _D, _P,
                           _P],
    "kx_bn_fwd_training_noalloc": [_EP, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _D, _P, _P,
                                   _D, _P, _P],
    "kx_bn_fwd_inference": [_EP, _I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _D],
    "kx_bn_bwd": [_EP, _I, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _D, _P, _P],
    "kx_host_flags_alloc": [_I, ctypes.POINTER(_P), ctypes.POINTER(_P)],
    "kx_host_flags_free": [_P],
    "kx_wait_flag": [_P, _P, ctypes.c_ulonglong, _P],
    "kx_num_sms": [],
    "kx_last_kernel_name": [],
    "kx_last_grid": [],
    "kx_last_cuda_error": [],
    "kx_version": [],
}


def lib() -> ctypes.CDLL:
    """Load libkx.so (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIBKX_PATH):
                raise RuntimeError(
                    f"{LIBKX_PATH} is missing; build it with python -m kernel_intercept_b200.build")
            L = ctypes.CDLL(LIBKX_PATH)
            for name, args in _SIGNATURES.items():
                fn = getattr(L, name, None)
                if fn is None:
                    continue
                fn.argtypes = args
                fn.restype = _I
            L.kx_last_kernel_name.restype = ctypes.c_char_p
            L.kx_version.restype = ctypes.c_char_p
            L.kx_launch_count.argtypes = []
            L.kx_launch_count.restype = ctypes.c_ulonglong
            L.kx_device_alloc_count.argtypes = []
            L.kx_device_alloc_count.restype = ctypes.c_ulonglong
            _lib = L
    return _lib


def _check(name: str, status: int) -> int:
    if status not in (OK,):
        raise KxError(name, status)
    return status


def _f(x: float):
    return ctypes.byref(ctypes.c_float(float(x)))


def make_exec(stream=None, sm_quota=0, yield_flag=None, done_flag=None, max_tiles=0,
              timeout_ns=0, fp32_mode=FP32_3XTF32, err_word=None, scalars_on_device=0):
    """Build a kx_exec.  ``stream`` may be a torch.cuda.Stream, an int handle or None."""
    if stream is not None and hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    return Exec(stream or None, sm_quota, yield_flag, done_flag, max_tiles, timeout_ns, fp32_mode,
                err_word, scalars_on_device)


def current_exec(**kw) -> Exec:
    import torch
    return make_exec(stream=torch.cuda.current_stream().cuda_stream, **kw)


# ----------------------------------------------------------- raw C ABI ---

def sgemm(ex, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, check=True):
    s = lib().kx_sgemm(ctypes.byref(ex) if ex is not None else None, transa, transb, m, n, k,
                       _f(alpha), A, lda, B, ldb, _f(beta), C, ldc)
    return _check("kx_sgemm", s) if check else s


def sgemm_strided_batched(ex, transa, transb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, C,
                          ldc, sC, batch, check=True):
    s = lib().kx_sgemm_strided_batched(ctypes.byref(ex) if ex is not None else None, transa,
                                       transb, m, n, k, _f(alpha), A, lda, sA, B, ldb, sB,
                                       _f(beta), C, ldc, sC, batch)
    return _check("kx_sgemm_strided_batched", s) if check else s


def sgemm_batched(ex, transa, transb, m, n, k, alpha, Aarr, lda, Barr, ldb, beta, Carr, ldc,
                  batch, check=True):
    s = lib().kx_sgemm_batched(ctypes.byref(ex) if ex is not None else None, transa, transb, m,
                               n, k, _f(alpha), Aarr, lda, Barr, ldb, _f(beta), Carr, ldc, batch)
    return _check("kx_sgemm_batched", s) if check else s


def gemm_ex(ex, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C, Ctype,
            ldc, check=True):
    s = lib().kx_gemm_ex(ctypes.byref(ex) if ex is not None else None, transa, transb, m, n, k,
                         _f(alpha), A, Atype, lda, B, Btype, ldb, _f(beta), C, Ctype, ldc)
    return _check("kx_gemm_ex", s) if check else s


def gemm_strided_batched_ex(ex, transa, transb, m, n, k, alpha, A, Atype, lda, sA, B, Btype, ldb,
                            sB, beta, C, Ctype, ldc, sC, batch, check=True):
    s = lib().kx_gemm_strided_batched_ex(ctypes.byref(ex) if ex is not None else None, transa,
                                         transb, m, n, k, _f(alpha), A, Atype, lda, sA, B, Btype,
                                         ldb, sB, _f(beta), C, Ctype, ldc, sC, batch)
    return _check("kx_gemm_strided_batched_ex", s) if check else s


def matmul(ex, transa, transb, m, n, k, alpha, A, Atype, lda, sA, B, Btype, ldb, sB, beta, C,
           Ctype, ldc, sC, D, Dtype, ldd, sD, batch=1, epilogue=EPI_DEFAULT, bias=None,
           bias_type=R_32F, check=True):
    s = lib().kx_matmul(ctypes.byref(ex) if ex is not None else None, transa, transb, m, n, k,
                        _f(alpha), A, Atype, lda, sA, B, Btype, ldb, sB, _f(beta), C, Ctype, ldc,
                        sC, D, Dtype, ldd, sD, batch, epilogue, bias, bias_type)
    return _check("kx_matmul", s) if check else s


def conv_out_dims(d: ConvDesc):
    p, q = _I(0), _I(0)
    _check("kx_conv_out_dims", lib().kx_conv_out_dims(ctypes.byref(d), ctypes.byref(p),
                                                       ctypes.byref(q)))
    return p.value, q.value


def conv_fwd(ex, d, alpha, x, w, beta, y, check=True):
    s = lib().kx_conv_fwd(ctypes.byref(ex) if ex is not None else None, ctypes.byref(d), _f(alpha),
                          x, w, _f(beta), y)
    return _check("kx_conv_fwd", s) if check else s


def conv_bwd_data(ex, d, alpha, w, dy, beta, dx, check=True):
    s = lib().kx_conv_bwd_data(ctypes.byref(ex) if ex is not None else None, ctypes.byref(d),
                               _f(alpha), w, dy, _f(beta), dx)
    return _check("kx_conv_bwd_data", s) if check else s


def conv_bwd_filter(ex, d, alpha, x, dy, beta, dw, check=True):
    s = lib().kx_conv_bwd_filter(ctypes.byref(ex) if ex is not None else None, ctypes.byref(d),
                                 _f(alpha), x, dy, _f(beta), dw)
    return _check("kx_conv_bwd_filter", s) if check else s


def bn_fwd_training(ex, mode, alpha, beta, n, c, h, w, x, y, scale, bias, factor, rmean, rvar,
                    eps, smean, sinv, check=True):
    s = lib().kx_bn_fwd_training(ctypes.byref(ex) if ex is not None else None, mode, _f(alpha),
                                 _f(beta), n, c, h, w, x, y, scale, bias, factor, rmean, rvar,
                                 eps, smean, sinv)
    return _check("kx_bn_fwd_training", s) if check else s


def bn_fwd_inference(ex, mode, alpha, beta, n, c, h, w, x, y, scale, bias, mean, var, eps,
                     check=True):
    s = lib().kx_bn_fwd_inference(ctypes.byref(ex) if ex is not None else None, mode, _f(alpha),
                                  _f(beta), n, c, h, w, x, y, scale, bias, mean, var, eps)
    return _check("kx_bn_fwd_inference", s) if check else s


def bn_bwd(ex, mode, alpha_d, beta_d, alpha_p, beta_p, n, c, h, w, x, dy, dx, scale, dscale,
           dbias, eps, smean, sinv, check=True):
    s = lib().kx_bn_bwd(ctypes.byref(ex) if ex is not None else None, mode, _f(alpha_d),
                        _f(beta_d), _f(alpha_p), _f(beta_p), n, c, h, w, x, dy, dx, scale, dscale,
                        dbias, eps, smean, sinv)
    return _check("kx_bn_bwd", s) if check else s


class HostFlags:
    """``count`` pinned, device-mapped ints (kx_host_flags_alloc)."""

    def __init__(self, count: int = 1):
        h, d = _P(), _P()
        _check("kx_host_flags_alloc", lib().kx_host_flags_alloc(count, ctypes.byref(h),
                                                                ctypes.byref(d)))
        self.count = count
        self.host_ptr = h.value
        self.dev_ptr = d.value
        self._arr = (ctypes.c_int * count).from_address(self.host_ptr)

    def __getitem__(self, i):
        return self._arr[i]

    def __setitem__(self, i, v):
        self._arr[i] = int(v)

    def dev(self, i=0) -> int:
        return self.dev_ptr + 4 * i

    def close(self):
        if self.host_ptr:
            lib().kx_host_flags_free(self.host_ptr)
            self.host_ptr = None


def wait_flag(stream, flag_dev_ptr, timeout_ns, status_dev_ptr):
    return _check("kx_wait_flag", lib().kx_wait_flag(stream, flag_dev_ptr, timeout_ns,
                                                     status_dev_ptr))


def num_sms() -> int:
    return lib().kx_num_sms()


def last_kernel_name() -> str:
    return lib().kx_last_kernel_name().decode()


# ------------------------------------------------------ torch helpers ---

def _dtype_code(t):
    import torch
    return {torch.float32: R_32F, torch.bfloat16: R_16BF, torch.float16: R_16F}[t.dtype]


def mm(a, b, out=None, alpha=1.0, beta=0.0, ex=None):
    """Row-major ``out = alpha * a @ b + beta * out`` for 2-D CUDA tensors via the
    column-major C ABI (computes out^T = b^T a^T).  fp32 -> kx_sgemm,
    bf16/fp16 -> kx_gemm_ex."""
    import torch
    assert a.is_cuda and b.is_cuda and a.dim() == 2 and b.dim() == 2
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    a = a.contiguous()
    b = b.contiguous()
    if out is None:
        out = torch.zeros(M, N, device=a.device, dtype=a.dtype)
    ex = ex if ex is not None else current_exec()
    if a.dtype == torch.float32:
        sgemm(ex, OP_N, OP_N, N, M, K, alpha, b.data_ptr(), N, a.data_ptr(), K, beta,
              out.data_ptr(), N)
    else:
        t = _dtype_code(a)
        gemm_ex(ex, OP_N, OP_N, N, M, K, alpha, b.data_ptr(), t, N, a.data_ptr(), t, K, beta,
                out.data_ptr(), _dtype_code(out), N)
    return out
