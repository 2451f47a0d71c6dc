"""Single-workload runners for device profiling of the kx kernels.

    python -m kernel_intercept_b200.cases CASE [--reps R]

Each case allocates its inputs once (seeded N(0,1) data), runs one untimed
launch, then R more (default 1), synchronizes and prints the kernel name the
last call ran.  The shapes are the ones the HP/BE co-scheduling benchmark
exercises, chosen so every input is larger than the 126 MB L2 where the
workload allows it, while the whole case stays within a few GB of device
memory (small enough for a multi-pass profiler capture):

  conv3_2     VGG16 conv3_2 forward, batch 32, 256 -> 256 channels, 56x56, 3x3
              pad 1 (x and y 103 MB each)
  conv1_2     VGG16 conv1_2 forward, batch 32, 64 -> 64 channels, 224x224
              (x and y 411 MB each; the 64-column tile shape)
  dgrad3_2    the same layer's backward data (dx from dy and w)
  wgrad3_2    the same layer's backward filter (dw from x and dy)
  vgg16_convs the 13 VGG16 convolution layers, batch 32, forward, in order
  gemm_f32    4096^3 fp32 SGEMM (3xTF32 with pre-split operands)
  gemm_bf16   2048 x 4096 x 2048 bf16 GemmEx (the hidden-2048 LLaMA's query
              projection at 4096 tokens)
  gemm_scores the same model's attention scores: 64 x (1024 x 1024 x 128) bf16
              GemmStridedBatchedEx (q k^T, K = head width)
  gemm_fc6    VGG16 fc6 at batch 32: 4096 x 32 x 25088 fp32 SGEMM (TN), weights
              411 MB
  bn_train    batch-norm training forward, spatial, 32 x 256 x 56 x 56
  hp_step     one batch-32 VGG16 inference step (the HP client of
              configuration 1) through the LD_PRELOAD interposer and the scheduler
  hp_step_llama one batch-4 x 1024 LLaMA-style bf16 inference step (the HP
              client of configuration 4), the same way
"""
from __future__ import annotations

import argparse
import os
import sys

CASES = ("conv3_2", "conv1_2", "dgrad3_2", "wgrad3_2", "vgg16_convs", "gemm_f32", "gemm_bf16",
         "gemm_scores", "gemm_fc6", "bn_train", "hp_step", "hp_step_llama")

# VGG16 convolution stack: (in channels, out channels, spatial size)
VGG16_CONVS = [(3, 64, 224), (64, 64, 224), (64, 128, 112), (128, 128, 112),
               (128, 256, 56), (256, 256, 56), (256, 256, 56), (256, 512, 28),
               (512, 512, 28), (512, 512, 28), (512, 512, 14), (512, 512, 14),
               (512, 512, 14)]


def _direct(case, reps):
    """Cases that call the C-ABI directly (no interposer)."""
    import torch

    from . import kx
    torch.manual_seed(0)
    ex = kx.current_exec()
    dev = "cuda"
    calls = []
    if case in ("conv3_2", "conv1_2", "vgg16_convs"):
        layers = {"conv3_2": [(256, 256, 56)], "conv1_2": [(64, 64, 224)]}.get(case, VGG16_CONVS)
        n = 32
        for c, k, hw in layers:
            x = torch.randn(n, c, hw, hw, device=dev)
            w = torch.randn(k, c, 3, 3, device=dev) * (2.0 / (c * 9)) ** 0.5
            y = torch.empty(n, k, hw, hw, device=dev)
            d = kx.ConvDesc(n, c, hw, hw, k, 3, 3, 1, 1, 1, 1, 1, 1, 1)
            calls.append(lambda d=d, x=x, w=w, y=y: kx.conv_fwd(
                ex, d, 1.0, x.data_ptr(), w.data_ptr(), 0.0, y.data_ptr()))
    elif case in ("dgrad3_2", "wgrad3_2"):
        n, c, k, hw = 32, 256, 256, 56
        x = torch.randn(n, c, hw, hw, device=dev)
        w = torch.randn(k, c, 3, 3, device=dev) * (2.0 / (c * 9)) ** 0.5
        dy = torch.randn(n, k, hw, hw, device=dev)
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        d = kx.ConvDesc(n, c, hw, hw, k, 3, 3, 1, 1, 1, 1, 1, 1, 1)
        if case == "dgrad3_2":
            calls.append(lambda: kx.conv_bwd_data(ex, d, 1.0, w.data_ptr(), dy.data_ptr(), 0.0,
                                                  dx.data_ptr()))
        else:
            calls.append(lambda: kx.conv_bwd_filter(ex, d, 1.0, x.data_ptr(), dy.data_ptr(), 0.0,
                                                    dw.data_ptr()))
    elif case == "gemm_fc6":
        m, n_, k = 4096, 32, 25088
        w = torch.randn(m, k, device=dev) * 0.01
        xin = torch.randn(n_, k, device=dev)
        c_ = torch.empty(n_, m, device=dev)
        calls.append(lambda: kx.sgemm(ex, 1, 0, m, n_, k, 1.0, w.data_ptr(), k, xin.data_ptr(), k,
                                      0.0, c_.data_ptr(), m))
    elif case == "gemm_f32":
        s = 4096
        a = torch.randn(s, s, device=dev)
        b = torch.randn(s, s, device=dev)
        c_ = torch.empty(s, s, device=dev)
        calls.append(lambda: kx.sgemm(ex, 1, 0, s, s, s, 1.0, a.data_ptr(), s, b.data_ptr(), s,
                                      0.0, c_.data_ptr(), s))
    elif case == "gemm_bf16":
        m, n_, k = 2048, 4096, 2048
        a = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
        b = torch.randn(n_, k, device=dev, dtype=torch.bfloat16)
        c_ = torch.empty(n_, m, device=dev, dtype=torch.bfloat16)
        calls.append(lambda: kx.gemm_ex(ex, 1, 0, m, n_, k, 1.0, a.data_ptr(), kx.R_16BF, k,
                                        b.data_ptr(), kx.R_16BF, k, 0.0, c_.data_ptr(),
                                        kx.R_16BF, m))
    elif case == "gemm_scores":
        batch, t, hd = 64, 1024, 128
        q = torch.randn(batch, t, hd, device=dev, dtype=torch.bfloat16)
        k_ = torch.randn(batch, t, hd, device=dev, dtype=torch.bfloat16)
        s_ = torch.empty(batch, t, t, device=dev, dtype=torch.bfloat16)
        calls.append(lambda: kx.gemm_strided_batched_ex(
            ex, 1, 0, t, t, hd, 1.0, k_.data_ptr(), kx.R_16BF, hd, t * hd, q.data_ptr(),
            kx.R_16BF, hd, t * hd, 0.0, s_.data_ptr(), kx.R_16BF, t, t * t, batch))
    elif case == "bn_train":
        n, c, h, w_ = 32, 256, 56, 56
        x = torch.randn(n, c, h, w_, device=dev)
        y = torch.empty_like(x)
        sc = torch.ones(c, device=dev)
        bi = torch.zeros(c, device=dev)
        rm = torch.zeros(c, device=dev)
        rv = torch.ones(c, device=dev)
        sm = torch.empty(c, device=dev)
        si = torch.empty(c, device=dev)
        calls.append(lambda: kx.bn_fwd_training(
            ex, 1, 1.0, 0.0, n, c, h, w_, x.data_ptr(), y.data_ptr(), sc.data_ptr(),
            bi.data_ptr(), 0.1, rm.data_ptr(), rv.data_ptr(), 1e-5, sm.data_ptr(), si.data_ptr()))
    for _ in range(1 + reps):
        for f in calls:
            f()
    torch.cuda.synchronize()
    return kx.last_kernel_name()


def _hp_step(reps, model="vgg16"):
    """One untimed and `reps` more HP inference steps (batch-32 VGG16, or the
    batch-4 x 1024 bf16 LLaMA-style decoder) as the HP client of the
    scheduler, with every convolution and GEMM captured."""
    import torch

    from . import harness, kx
    dev = torch.device("cuda", 0)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.benchmark = False
    torch.manual_seed(0)
    orion = harness.Orion()
    if model == "vgg16":
        net = harness.make_vgg16(dev).eval()
        inp = torch.randn(32, 3, 224, 224, device=dev)
    else:
        net = harness.make_llama(device=dev, dtype=torch.bfloat16).eval()
        inp = torch.randint(0, 32000, (4, 1024), device=dev)

    def step():
        with torch.no_grad():
            net(inp)

    assert orion.orion_init_scheduler(2) == 0, "orion_init_scheduler failed"
    orion.orion_set_capture(0)
    step()
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    hp, _ = harness.run_clients(orion, step, None, reps, 1, with_be=False)
    if hp.error is not None:
        raise hp.error
    stats = orion.stats(0)
    orion.orion_set_capture(0)
    orion.orion_stop_scheduler()
    if stats["kx_ops"] == 0 or stats["errors"]:
        raise RuntimeError(f"HP step not captured by the kx kernels: {stats}")
    return kx.last_kernel_name()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("case", choices=CASES)
    ap.add_argument("--reps", type=int, default=1)
    args = ap.parse_args(argv)
    if args.case in ("hp_step", "hp_step_llama"):
        from . import harness
        if not harness.preloaded():
            env = harness.preload_env({"ORION_LOG_LEVEL": os.environ.get("ORION_LOG_LEVEL",
                                                                          "WARN")})
            os.execve(sys.executable, [sys.executable, "-m", "kernel_intercept_b200.cases"]
                      + sys.argv[1:], env)
        name = _hp_step(args.reps, "vgg16" if args.case == "hp_step" else "llama")
    else:
        name = _direct(args.case, args.reps)
    print("ok", args.case, name, flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
