"""The five HP/BE configurations the co-scheduler is benchmarked on.

Each configuration is one GPU's client group: an HP client (client 0) and
one or more BE clients (1, 2, ...), all PyTorch models whose dense ops the
interposer captures.  Shapes and optimisers follow the benchmark
configurations of the kernel_intercept project (its models:
python/GPT.py:42-149 CharGPT, python/VGG16.py torchvision vgg16,
python/LLaMA.py:78-98 / 163-208 CharLLaMA; its drivers run HP and BE as
threads of one process, python/test_orion_blocking.py:192-423):

* 0: HP GPT inference fp32 (6 layers, d512, 8 heads, FFN 2048, vocab 32000)
     at batch 8 x 256; BE the same GPT inference (own weights).
* 1: HP VGG16 inference fp32, batch 32 x 3x224x224; BE GPT training fp32,
     batch 16 x 256, AdamW lr 1e-4, cross-entropy vs uniform random targets.
* 2: HP LLaMA-style decoder inference bf16 (12 layers, d2048, 16 heads,
     SwiGLU 5504, RMSNorm 1e-6, RoPE 1e4, vocab 32000), batch 4 x 1024; BE two
     clients each training the GPT in bf16 (batch 16 x 256, AdamW).
* 3: GEMM contention microbench (bench.py runs it separately: small HP GEMMs
     every 200 us against back-to-back 8192^3 BE GEMMs, BE SM quota sweep).
* 4: the per-GPU group of the placement sweep: HP LLaMA bf16 inference; BE1
     VGG16 training fp32 at batch 64 (SGD momentum 0.9, labels uniform in
     [0, 1000)); BE2 GPT training fp32 (batch 16 x 256, AdamW).

Weights are random-init as the configurations state (N(0, 0.02) for the
decoders, torchvision's Kaiming-normal for VGG16); inputs are seeded synthetic
tensors of the stated shapes and distributions.
"""
from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field
from typing import Callable

from . import harness

GPT_SEQ, LLAMA_SEQ = 256, 1024


@dataclass
class Client:
    """One client of a configuration: its step, what a step processes, and
    (HP only) the end-to-end step with host buffers."""
    name: str
    step: Callable[[], None]
    units: int                   # items one step processes (tokens or images)
    unit: str                    # "tokens" or "images"
    dtype: str
    flops: float                 # captured dense-op FLOPs of one step
    e2e_step: Callable[[], None] | None = None
    h2d_bytes: int = 0
    d2h_bytes: int = 0
    extra: dict = field(default_factory=dict)


def gpt_train_flops(batch, seq=GPT_SEQ):
    # forward + backward (data and weight gradients) of every captured GEMM
    return 3 * harness.gpt_flops_forward(batch, seq)


def llama_flops_forward(batch, seq=LLAMA_SEQ, hidden=2048, inter=5504, layers=12, vocab=32000):
    tok = batch * seq
    per_layer = (2 * tok * hidden * hidden * 4          # wq, wk, wv, wo
                 + 2 * tok * hidden * inter * 3         # gate, up, down
                 + 2 * 2 * batch * seq * seq * hidden)  # scores + context (all heads)
    return layers * per_layer + 2 * tok * hidden * vocab


def vgg16_train_flops(batch):
    # forward, backward data (all but the first convolution) and backward filter
    first = 2 * batch * 3 * 64 * 9 * 224 * 224
    fwd = harness.vgg16_flops_forward(batch)
    return 3 * fwd - first


def _gpt_infer(dev, batch, seed, name, e2e=False):
    import torch
    torch.manual_seed(seed)
    m = harness.make_gpt(device=dev).eval()
    tok = torch.randint(0, 32000, (batch, GPT_SEQ), device=dev)

    def step():
        with torch.no_grad():
            m(tok)

    c = Client(name, step, batch * GPT_SEQ, "tokens", "f32", harness.gpt_flops_forward(batch))
    if e2e:
        tok_host = tok.cpu().pin_memory()
        out_host = torch.empty(batch, 32000).pin_memory()

        def step_e2e():
            with torch.no_grad():
                tok.copy_(tok_host, non_blocking=True)
                out = m(tok)
                # next-token logits of every sequence back to the host
                out_host.copy_(out[:, -1], non_blocking=True)

        c.e2e_step, c.h2d_bytes, c.d2h_bytes = step_e2e, tok.numel() * 8, batch * 32000 * 4
    return c


def _gpt_train(dev, batch, seed, name, dtype=None):
    import torch
    import torch.nn.functional as F
    torch.manual_seed(seed)
    m = harness.make_gpt(device=dev, dtype=dtype)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-4)
    tok = torch.randint(0, 32000, (batch, GPT_SEQ), device=dev)
    tgt = torch.randint(0, 32000, (batch, GPT_SEQ), device=dev)

    def step():
        logits = m(tok)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]).float(), tgt.view(-1))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()

    return Client(name, step, batch * GPT_SEQ, "tokens", "bf16" if dtype is not None else "f32",
                  gpt_train_flops(batch))


def _vgg16_infer(dev, batch, seed, name):
    import torch
    torch.manual_seed(seed)
    m = harness.make_vgg16(dev).eval()
    img = torch.randn(batch, 3, 224, 224, device=dev)
    img_host = img.cpu().pin_memory()
    out_host = torch.empty(batch, 1000).pin_memory()

    def step():
        with torch.no_grad():
            m(img)

    def step_e2e():
        with torch.no_grad():
            img.copy_(img_host, non_blocking=True)
            out = m(img)
            out_host.copy_(out, non_blocking=True)

    return Client(name, step, batch, "images", "f32", harness.vgg16_flops_forward(batch),
                  e2e_step=step_e2e, h2d_bytes=img.numel() * 4, d2h_bytes=batch * 1000 * 4)


def _vgg16_train(dev, batch, seed, name):
    import torch
    import torch.nn.functional as F
    torch.manual_seed(seed)
    m = harness.make_vgg16(dev).train()
    opt = torch.optim.SGD(m.parameters(), lr=0.01, momentum=0.9)
    img = torch.randn(batch, 3, 224, 224, device=dev)
    lbl = torch.randint(0, 1000, (batch,), device=dev)

    def step():
        loss = F.cross_entropy(m(img), lbl)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()

    return Client(name, step, batch, "images", "f32", vgg16_train_flops(batch))


def _llama_infer(dev, batch, seed, name):
    import torch
    torch.manual_seed(seed)
    m = harness.make_llama(device=dev, dtype=torch.bfloat16).eval()
    tok = torch.randint(0, 32000, (batch, LLAMA_SEQ), device=dev)
    tok_host = tok.cpu().pin_memory()
    out_host = torch.empty(batch, 32000, dtype=torch.bfloat16).pin_memory()

    def step():
        with torch.no_grad():
            m(tok)

    def step_e2e():
        with torch.no_grad():
            tok.copy_(tok_host, non_blocking=True)
            out = m(tok)
            # next-token logits of every sequence back to the host
            out_host.copy_(out[:, -1], non_blocking=True)

    return Client(name, step, batch * LLAMA_SEQ, "tokens", "bf16", llama_flops_forward(batch),
                  e2e_step=step_e2e, h2d_bytes=tok.numel() * 8, d2h_bytes=batch * 32000 * 2)


DESCRIPTIONS = {
    0: "HP GPT inference fp32 b8 s256 + BE GPT inference fp32 b8 s256 (6L, d512, 8 heads, "
       "vocab 32000)",
    1: "HP VGG16 inference fp32 b32 3x224x224 + BE GPT training fp32 b16 s256 AdamW",
    2: "HP LLaMA-style decoder inference bf16 b4 s1024 (12L, d2048, 16 heads, SwiGLU 5504, "
       "vocab 32000) + 2 BE GPT training bf16 b16 s256 AdamW",
    3: "GEMM contention microbench: HP M x N=K GEMMs (M in 64/128/256, N=K in 1024/4096) every "
       "200 us vs BE back-to-back 8192^3, BE SM quota 16/32/64/148, fp32 and bf16",
    4: "per-GPU group of the placement sweep: HP LLaMA-style decoder inference bf16 b4 s1024 + "
       "BE1 VGG16 training fp32 b64 SGD momentum 0.9 + BE2 GPT training fp32 b16 s256 AdamW",
}


def build(cfg: int, dev) -> tuple[Client, list[Client]]:
    """HP and BE clients of configuration cfg (0, 1, 2 or 4) on device dev."""
    if cfg == 0:
        return (_gpt_infer(dev, 8, 0, "gpt_infer_b8", e2e=True),
                [_gpt_infer(dev, 8, 1, "gpt_infer_b8")])
    if cfg == 1:
        return _vgg16_infer(dev, 32, 0, "vgg16_infer_b32"), [_gpt_train(dev, 16, 1, "gpt_train_b16")]
    if cfg == 2:
        import torch
        return (_llama_infer(dev, 4, 0, "llama_bf16_infer_b4"),
                [_gpt_train(dev, 16, 1 + i, "gpt_train_bf16_b16", dtype=torch.bfloat16)
                 for i in range(2)])
    if cfg == 4:
        return (_llama_infer(dev, 4, 0, "llama_bf16_infer_b4"),
                [_vgg16_train(dev, 64, 1, "vgg16_train_b64"), _gpt_train(dev, 16, 2, "gpt_train_b16")])
    raise ValueError(f"no client group for configuration {cfg}")


# ----------------------------------------------------------- CPU forward ---

def cpu_forward_rate(cfg: int, threads: int | None = None, sample: int = 1):
    """The HP model's plain PyTorch CPU forward on this host (no interception),
    the configurations' CPU-runnable form: returns (units/s, unit, threads
    used, sample description, dtype).  `sample` images or sequences per
    timed forward after one untimed forward."""
    import torch
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    used = torch.get_num_threads()
    torch.manual_seed(0)
    if cfg == 0:
        m = harness.make_gpt(device="cpu").eval()
        x = torch.randint(0, 32000, (sample, GPT_SEQ))
        units, unit, dtype, what = sample * GPT_SEQ, "tokens", "f32", f"{sample} x {GPT_SEQ} tokens"
    elif cfg in (1, 3):
        m = harness.make_vgg16("cpu").eval()
        x = torch.randn(sample, 3, 224, 224)
        units, unit, dtype, what = sample, "images", "f32", f"{sample} images"
    else:
        # the bf16 decoder; CPU bf16 matmul speed varies by host, so the CPU
        # forward runs the same weights in fp32 (stated in the sample)
        m = harness.make_llama(device="cpu").eval()
        x = torch.randint(0, 32000, (sample, LLAMA_SEQ))
        units, unit, dtype, what = (sample * LLAMA_SEQ, "tokens", "f32",
                                    f"{sample} x {LLAMA_SEQ} tokens, fp32 weights")
    with torch.no_grad():
        m(x[:1])
        t0 = time.perf_counter()
        m(x)
        dt = time.perf_counter() - t0
    return units / dt, unit, used, what, dtype


def peak_note(flops: float, ms: float) -> float:
    """TFLOP/s of `flops` done in `ms` milliseconds."""
    return flops / (ms * 1e-3) / 1e12 if ms > 0 else math.nan
