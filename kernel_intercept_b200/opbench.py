"""Op-level timings of the kx kernels against the libraries they replace.

    python -m kernel_intercept_b200.opbench vgg  [--batch 32] [--check]
    python -m kernel_intercept_b200.opbench gemm [--check]
    python -m kernel_intercept_b200.opbench vggbwd [--batch 32] [--check]

One JSON line per operation.  Every time is the mean of R back-to-back calls
on one stream measured with CUDA events after 3 warm-up calls (operands stay
resident; at these sizes most of them fit in the 126 MB L2, so the figures
are warm-cache rates).  The library arm is PyTorch's own call into cuDNN /
cuBLAS with TF32 off (`allow_tf32 = False`, cuDNN `benchmark = True`), i.e.
the fp32 kernels an unmodified PyTorch program reaches.  `host_us` is the
wall time of one kx C-ABI call (enqueue only).  `--check` adds the normwise
error max|kx - ref| / max|ref| against a float64 evaluation on the GPU.

vgg : the 13 VGG16 3x3 convolutions (pad 1) at batch 32, forward.
vggbwd: the same layers' backward data (dx) and backward filter (dw); the
      library arm is aten::convolution_backward with one output each.
gemm: the GEMM shapes of the benchmark's models in the transposes PyTorch
      issues (column-major, cuBLAS notation), fp32 through 3xTF32 and bf16.
"""
from __future__ import annotations

import argparse
import json
import sys
import time

VGG16_CONVS = [(3, 64, 224), (64, 64, 224), (64, 128, 112), (128, 128, 112),
               (128, 256, 56), (256, 256, 56), (256, 256, 56), (256, 512, 28),
               (512, 512, 28), (512, 512, 28), (512, 512, 14), (512, 512, 14),
               (512, 512, 14)]

# name, transa, transb, m, n, k, batch, dtype ("f32" | "bf16")
GEMMS = [
    ("gpt_head_fwd", 1, 0, 64, 4096, 512, 1, "f32"),
    ("gpt_head_dgrad", 0, 0, 512, 4096, 64, 1, "f32"),
    ("gpt_head_wgrad", 0, 1, 512, 64, 4096, 1, "f32"),
    ("gpt_qk", 1, 0, 256, 256, 64, 16, "f32"),
    ("gpt_pv", 0, 0, 64, 256, 256, 16, "f32"),
    ("gpt_l1_fwd", 1, 0, 2048, 4096, 512, 1, "f32"),
    ("gpt_l1_wgrad", 0, 1, 512, 2048, 4096, 1, "f32"),
    ("gpt_lm_head", 1, 0, 32000, 4096, 512, 1, "f32"),
    ("vgg_fc6", 1, 0, 4096, 32, 25088, 1, "f32"),
    ("vgg_fc7", 1, 0, 4096, 32, 4096, 1, "f32"),
    ("big_f32", 1, 0, 8192, 8192, 8192, 1, "f32"),
    ("llama_wq_bf16", 1, 0, 2048, 4096, 2048, 1, "bf16"),
    ("llama_up_bf16", 1, 0, 5504, 4096, 2048, 1, "bf16"),
    ("llama_down_bf16", 1, 0, 2048, 4096, 5504, 1, "bf16"),
    ("llama_lm_head_bf16", 1, 0, 32000, 4096, 2048, 1, "bf16"),
    ("llama_scores_bf16", 1, 0, 1024, 1024, 128, 64, "bf16"),
    ("llama_context_bf16", 0, 0, 128, 1024, 1024, 64, "bf16"),
    ("gpt_l1_wgrad_bf16", 0, 1, 512, 2048, 4096, 1, "bf16"),
    ("big_bf16", 1, 0, 8192, 8192, 8192, 1, "bf16"),
]


def _time(fn, min_ms=20.0):
    """Mean milliseconds of fn() over enough back-to-back calls to fill
    about min_ms, after 3 warm-up calls."""
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    fn()
    e.record()
    e.synchronize()
    one = max(s.elapsed_time(e), 1e-3)
    reps = max(3, min(200, int(min_ms / one)))
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / reps


def _host_us(fn, n=50):
    import torch
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        fn()
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    return (t1 - t0) / n * 1e6


def _err(a, ref):
    d = (a.double() - ref).abs().max().item()
    r = ref.abs().max().item()
    return d / r if r else d


def run_vgg(batch, check):
    import torch
    import torch.nn.functional as F

    from . import kx
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.benchmark = True
    torch.manual_seed(0)
    ex = kx.current_exec()
    tot_kx = tot_lib = 0.0
    for li, (c, k, hw) in enumerate(VGG16_CONVS):
        x = torch.randn(batch, c, hw, hw, device="cuda")
        w = torch.randn(k, c, 3, 3, device="cuda") * (2.0 / (c * 9)) ** 0.5
        y = torch.empty(batch, k, hw, hw, device="cuda")
        d = kx.ConvDesc(batch, c, hw, hw, k, 3, 3, 1, 1, 1, 1, 1, 1, 1)

        def f_kx():
            kx.conv_fwd(ex, d, 1.0, x.data_ptr(), w.data_ptr(), 0.0, y.data_ptr())

        def f_lib():
            F.conv2d(x, w, padding=1)

        t_kx = _time(f_kx)
        name = kx.last_kernel_name()
        t_lib = _time(f_lib)
        fl = 2.0 * batch * k * c * 9 * hw * hw
        rec = {"layer": li, "c": c, "k": k, "hw": hw, "batch": batch, "kx_ms": round(t_kx, 4),
               "kx_tflops": round(fl / (t_kx * 1e-3) / 1e12, 1), "cudnn_ms": round(t_lib, 4),
               "cudnn_tflops": round(fl / (t_lib * 1e-3) / 1e12, 1), "kernel": name,
               "host_us": round(_host_us(f_kx, 10), 1)}
        if check:
            f_kx()
            ref = F.conv2d(x.double(), w.double(), padding=1)
            rec["err_kx"] = float(f"{_err(y, ref):.2e}")
            rec["err_cudnn"] = float(f"{_err(F.conv2d(x, w, padding=1), ref):.2e}")
            del ref
        tot_kx += t_kx
        tot_lib += t_lib
        print(json.dumps(rec), flush=True)
        del x, w, y
        torch.cuda.empty_cache()
    print(json.dumps({"total_kx_ms": round(tot_kx, 3), "total_cudnn_ms": round(tot_lib, 3)}),
          flush=True)


def run_vgg_bwd(batch, check):
    import torch

    from . import kx
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.benchmark = True
    torch.manual_seed(0)
    ex = kx.current_exec()
    tot = {"dgrad_kx": 0.0, "dgrad_lib": 0.0, "wgrad_kx": 0.0, "wgrad_lib": 0.0}
    for li, (c, k, hw) in enumerate(VGG16_CONVS):
        x = torch.randn(batch, c, hw, hw, device="cuda")
        w = torch.randn(k, c, 3, 3, device="cuda") * (2.0 / (c * 9)) ** 0.5
        dy = torch.randn(batch, k, hw, hw, device="cuda")
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        d = kx.ConvDesc(batch, c, hw, hw, k, 3, 3, 1, 1, 1, 1, 1, 1, 1)
        fl = 2.0 * batch * k * c * 9 * hw * hw
        rec = {"layer": li, "c": c, "k": k, "hw": hw, "batch": batch}

        def lib(mask):
            return torch.ops.aten.convolution_backward(dy, x, w, None, [1, 1], [1, 1], [1, 1],
                                                       False, [0, 0], 1, mask)

        for name, f_kx, mask in (
                ("dgrad", lambda: kx.conv_bwd_data(ex, d, 1.0, w.data_ptr(), dy.data_ptr(), 0.0,
                                                   dx.data_ptr()), [True, False, False]),
                ("wgrad", lambda: kx.conv_bwd_filter(ex, d, 1.0, x.data_ptr(), dy.data_ptr(),
                                                     0.0, dw.data_ptr()), [False, True, False])):
            if li == 0 and name == "dgrad":
                continue  # the first layer's input gradient is never needed
            t_kx = _time(f_kx)
            kname = kx.last_kernel_name()
            t_lib = _time(lambda: lib(mask))
            rec[f"{name}_kx_ms"] = round(t_kx, 4)
            rec[f"{name}_kx_tflops"] = round(fl / (t_kx * 1e-3) / 1e12, 1)
            rec[f"{name}_cudnn_ms"] = round(t_lib, 4)
            rec[f"{name}_cudnn_tflops"] = round(fl / (t_lib * 1e-3) / 1e12, 1)
            rec[f"{name}_kernel"] = kname
            tot[f"{name}_kx"] += t_kx
            tot[f"{name}_lib"] += t_lib
            if check:
                f_kx()
                ref = torch.ops.aten.convolution_backward(
                    dy.double(), x.double(), w.double(), None, [1, 1], [1, 1], [1, 1], False,
                    [0, 0], 1, mask)
                got = dx if name == "dgrad" else dw
                rec[f"{name}_err_kx"] = float(f"{_err(got, ref[0 if name == 'dgrad' else 1]):.2e}")
                del ref
        print(json.dumps(rec), flush=True)
        del x, w, dy, dx, dw
        torch.cuda.empty_cache()
    print(json.dumps({k: round(v, 3) for k, v in tot.items()}), flush=True)


def run_gemm(check, only="", fp32_mode="3xtf32"):
    import torch

    from . import kx
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    ex = kx.current_exec(fp32_mode=kx.FP32_FFMA if fp32_mode == "ffma" else kx.FP32_3XTF32)
    for name, ta, tb, m, n, k, batch, dt in GEMMS:
        if only and only not in name:
            continue
        tdt = torch.float32 if dt == "f32" else torch.bfloat16
        # row-major storage of the column-major operands (cuBLAS view)
        a_shape = (m, k) if ta else (k, m)
        b_shape = (k, n) if tb else (n, k)
        A = torch.randn(batch, *a_shape, device="cuda").to(tdt)
        B = torch.randn(batch, *b_shape, device="cuda").to(tdt)
        C = torch.empty(batch, n, m, device="cuda", dtype=tdt)
        lda, ldb, ldc = a_shape[1], b_shape[1], m
        opa = A.transpose(1, 2) if ta else A   # C_rm = op(B)^T . op(A)^T
        opb = B.transpose(1, 2) if tb else B
        code = kx.R_32F if dt == "f32" else kx.R_16BF

        def f_kx():
            if batch > 1:
                if dt == "f32":
                    kx.sgemm_strided_batched(ex, ta, tb, m, n, k, 1.0, A.data_ptr(), lda,
                                             A[0].numel(), B.data_ptr(), ldb, B[0].numel(), 0.0,
                                             C.data_ptr(), ldc, C[0].numel(), batch)
                else:
                    kx.gemm_strided_batched_ex(ex, ta, tb, m, n, k, 1.0, A.data_ptr(), code, lda,
                                               A[0].numel(), B.data_ptr(), code, ldb,
                                               B[0].numel(), 0.0, C.data_ptr(), code, ldc,
                                               C[0].numel(), batch)
            elif dt == "f32":
                kx.sgemm(ex, ta, tb, m, n, k, 1.0, A.data_ptr(), lda, B.data_ptr(), ldb, 0.0,
                         C.data_ptr(), ldc)
            else:
                kx.gemm_ex(ex, ta, tb, m, n, k, 1.0, A.data_ptr(), code, lda, B.data_ptr(), code,
                           ldb, 0.0, C.data_ptr(), code, ldc)

        def f_lib():
            torch.matmul(opb, opa, out=C)

        t_kx = _time(f_kx)
        kname = kx.last_kernel_name()
        t_lib = _time(f_lib)
        fl = 2.0 * m * n * k * batch
        rec = {"name": name, "trans": ("T" if ta else "N") + ("T" if tb else "N"), "m": m, "n": n,
               "k": k, "batch": batch, "dt": dt, "kx_ms": round(t_kx, 4),
               "kx_tflops": round(fl / (t_kx * 1e-3) / 1e12, 1), "cublas_ms": round(t_lib, 4),
               "cublas_tflops": round(fl / (t_lib * 1e-3) / 1e12, 1), "kernel": kname,
               "host_us": round(_host_us(f_kx), 1)}
        if check and m * n * k * batch <= 2 ** 36:
            f_kx()
            ref = torch.matmul(opb.double(), opa.double())
            rec["err_kx"] = float(f"{_err(C, ref):.2e}")
            del ref
        print(json.dumps(rec), flush=True)
        del A, B, C
        torch.cuda.empty_cache()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("what", choices=["vgg", "vggbwd", "gemm"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--only", default="", help="gemm: run the shapes whose name contains this")
    ap.add_argument("--fp32-mode", default="3xtf32", choices=["3xtf32", "ffma"],
                    help="gemm: arithmetic of the fp32 shapes on kx")
    args = ap.parse_args(argv)
    if args.what == "vgg":
        run_vgg(args.batch, args.check)
    elif args.what == "vggbwd":
        run_vgg_bwd(args.batch, args.check)
    else:
        run_gemm(args.check, args.only, args.fp32_mode)
    return 0


if __name__ == "__main__":
    sys.exit(main())
