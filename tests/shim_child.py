"""Child process for the interposer GPU tests.

Runs under LD_PRELOAD=libgpu_scheduler.so (the parent test sets it) and
prints one JSON object on its last stdout line.  Each scenario computes the
same PyTorch ops twice on the same inputs: once with capture off (the real
cuBLAS / cuDNN behind the interposer, TF32 disabled, i.e. the reference
shim's own path) and once captured on client 0 (queued to the worker and run
on the kx kernels), and reports the normwise relative error of every output.

Usage: python tests/shim_child.py <scenario>
"""
from __future__ import annotations

import ctypes
import json
import os
import sys
import threading

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def rel(got, ref):
    import torch
    got = got.double()
    ref = ref.double()
    den = ref.abs().max().item()
    return (got - ref).abs().max().item() / (den if den > 0 else 1.0)


def run_on_client(orion, client, fn):
    """Runs fn() on a thread registered as `client`, on its own stream."""
    import torch
    out = {}

    def body():
        try:
            s = torch.cuda.Stream()
            orion.orion_set_client_idx(client)
            orion.orion_register_client_stream(client, ctypes.c_void_p(s.cuda_stream))
            with torch.cuda.stream(s):
                out["v"] = fn()
            s.synchronize()
        except BaseException as e:  # noqa: BLE001 - reported to the parent
            out["e"] = e
        finally:
            orion.orion_set_client_idx(-1)

    t = threading.Thread(target=body)
    t.start()
    t.join()
    if "e" in out:
        raise out["e"]
    return out["v"]


def gemm_cases(torch):
    """(name, fn, dtype) triples; fn(inputs) -> output tensor."""
    g = torch.Generator(device="cuda").manual_seed(0)

    def r(*shape, dtype=torch.float32):
        return torch.randn(*shape, device="cuda", generator=g).to(dtype)

    F = torch.nn.functional
    bf = torch.bfloat16
    cases = []
    a, b = r(256, 512), r(512, 384)
    cases.append(("mm_256x512x384", lambda: a @ b, "f32"))
    at = r(512, 256)
    cases.append(("mm_tn", lambda: at.t() @ b, "f32"))
    bt = r(384, 512)
    cases.append(("mm_nt", lambda: a @ bt.t(), "f32"))
    x, w = r(2048, 512), r(64, 512)  # GPT per-head projection: m=64, n=2048, k=512
    cases.append(("linear_head", lambda: F.linear(x, w), "f32"))
    w2, bias = r(2048, 512), r(2048)
    cases.append(("linear_bias_lt", lambda: F.linear(x, w2, bias), "f32"))
    q, k = r(8, 256, 64), r(8, 256, 64)
    cases.append(("bmm_qk", lambda: q @ k.transpose(-2, -1), "f32"))
    p, v = r(8, 256, 256), r(8, 256, 64)
    cases.append(("bmm_pv", lambda: p @ v, "f32"))
    o1, o2 = r(33, 70), r(70, 45)
    cases.append(("mm_odd", lambda: o1 @ o2, "f32"))
    xb, wb, bb = r(1024, 2048, dtype=bf), r(2048, 2048, dtype=bf), r(2048, dtype=bf)
    cases.append(("bf16_linear", lambda: F.linear(xb, wb), "bf16"))
    cases.append(("bf16_linear_bias", lambda: F.linear(xb, wb, bb), "bf16"))
    qb, kb = r(16, 512, 128, dtype=bf), r(16, 512, 128, dtype=bf)
    cases.append(("bf16_bmm", lambda: qb @ kb.transpose(-2, -1), "bf16"))
    return cases


def scenario_gemm(orion):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    cases = gemm_cases(torch)
    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    refs = {n: fn().float() for n, fn, _ in cases}
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    outs = run_on_client(orion, 0, lambda: {n: fn().float() for n, fn, _ in cases})
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    errs = {n: rel(outs[n], refs[n]) for n, _, _ in cases}
    kinds = {n: d for n, _, d in cases}
    return {"errors": errs, "dtypes": kinds, "stats": stats}


def conv_cases():
    # (N, C, H, W, K, R, S, pad, stride, dil)
    return [(4, 16, 32, 32, 32, 3, 3, 1, 1, 1),
            (2, 3, 64, 64, 64, 3, 3, 1, 1, 1),
            (2, 32, 28, 28, 48, 3, 3, 1, 2, 1),
            (2, 64, 14, 14, 64, 1, 1, 0, 1, 1),
            (1, 8, 20, 20, 16, 3, 3, 2, 1, 2)]


def scenario_conv(orion):
    import torch
    F = torch.nn.functional
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.benchmark = False
    g = torch.Generator(device="cuda").manual_seed(1)
    inputs = []
    for (n, c, h, w, k, r, s, pad, stride, dil) in conv_cases():
        x = torch.randn(n, c, h, w, device="cuda", generator=g)
        wt = torch.randn(k, c, r, s, device="cuda", generator=g) * (2.0 / (c * r * s)) ** 0.5
        bias = torch.randn(k, device="cuda", generator=g)
        inputs.append((x, wt, bias, pad, stride, dil))

    def run():
        res = []
        for x, wt, bias, pad, stride, dil in inputs:
            xx = x.clone().requires_grad_(True)
            ww = wt.clone().requires_grad_(True)
            y = F.conv2d(xx, ww, bias, stride=stride, padding=pad, dilation=dil)
            gy = torch.ones_like(y) + 0.01 * torch.arange(y.numel(), device=y.device).view_as(y) % 7
            y.backward(gy)
            res.append((y.detach(), xx.grad.detach(), ww.grad.detach()))
        return res

    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    refs = run()
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    outs = run_on_client(orion, 0, run)
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    errs = {}
    for i, ((y, dx, dw), (ry, rdx, rdw)) in enumerate(zip(outs, refs)):
        errs[f"fwd_{i}"] = rel(y, ry)
        errs[f"dgrad_{i}"] = rel(dx, rdx)
        errs[f"wgrad_{i}"] = rel(dw, rdw)
    return {"errors": errs, "stats": stats}


def scenario_bn(orion):
    import torch
    F = torch.nn.functional
    g = torch.Generator(device="cuda").manual_seed(2)
    shapes = [(8, 64, 28, 28), (4, 128, 14, 14), (16, 32, 7, 7)]
    inputs = [(torch.randn(*s, device="cuda", generator=g) * 2 + 0.5,
               torch.rand(s[1], device="cuda", generator=g) + 0.5,
               torch.randn(s[1], device="cuda", generator=g)) for s in shapes]

    def run():
        res = []
        for x, wgt, b in inputs:
            xx = x.clone().requires_grad_(True)
            ww = wgt.clone().requires_grad_(True)
            bb = b.clone().requires_grad_(True)
            rm = torch.zeros(x.shape[1], device="cuda")
            rv = torch.ones(x.shape[1], device="cuda")
            y = F.batch_norm(xx, rm, rv, ww, bb, training=True, momentum=0.1, eps=1e-5)
            y.backward(torch.cos(y.detach()))
            yi = F.batch_norm(x, rm, rv, wgt, b, training=False, eps=1e-5)
            res.append((y.detach(), xx.grad, ww.grad, bb.grad, rm, rv, yi))
        return res

    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    refs = run()
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    outs = run_on_client(orion, 0, run)
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    names = ("y", "dx", "dscale", "dbias", "running_mean", "running_var", "y_inference")
    errs = {}
    for i, (o, r) in enumerate(zip(outs, refs)):
        for nm, a, b in zip(names, o, r):
            errs[f"{nm}_{i}"] = rel(a, b)
    return {"errors": errs, "stats": stats}


def scenario_gpt(orion):
    """End-to-end: the GPT decoder forward (fp32, batch 2 x seq 256) captured
    on client 0 vs the same forward through the real libraries."""
    import torch

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    m = harness.make_gpt(device="cuda").eval()
    tok = torch.randint(0, 32000, (2, 256), device="cuda")
    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    with torch.no_grad():
        ref = m(tok)
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)

    def fwd():
        with torch.no_grad():
            return m(tok)

    out = run_on_client(orion, 0, fwd)
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    return {"errors": {"logits": rel(out, ref)}, "stats": stats}


def scenario_hpbe(orion):
    """HP (small GEMMs) and BE (large GEMMs) clients at once: both finish,
    results stay exact, the BE client saw yields or blocking."""
    import torch

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(256, 1024, device="cuda", generator=g)
    b = torch.randn(1024, 1024, device="cuda", generator=g)
    A = torch.randn(4096, 4096, device="cuda", generator=g)
    B = torch.randn(4096, 4096, device="cuda", generator=g)
    assert orion.orion_init_scheduler(2) == 0
    orion.orion_set_capture(0)
    ref_hp = a @ b
    ref_be = A @ B
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    hp_out, be_out = [], []

    def hp_step():
        hp_out.append(a @ b)

    def be_step():
        be_out.append(A @ B)

    hp, be = harness.run_clients(orion, hp_step, be_step, hp_steps=40, hp_warmup=2)
    orion.orion_set_capture(0)
    stats = {c: orion.stats(c) for c in (0, 1)}
    orion.orion_stop_scheduler()
    torch.cuda.synchronize()
    err_hp = max(rel(o, ref_hp) for o in hp_out)
    err_be = max(rel(o, ref_be) for o in be_out)
    return {"errors": {"hp": err_hp, "be": err_be}, "stats": stats,
            "hp_p50_ms": harness.percentile(hp.latencies_ms, 0.5), "be_iters": be.iters}


def scenario_hpbe2(orion):
    """HP (small GEMMs) against two BE clients (a large GEMM; a convolution
    with batch norm in training) with BE keeping no SMs under HP load
    (KX_BE_KEEP_SMS=0, set by the parent): BE GEMMs and convolutions stop at
    tile boundaries while HP works and are relaunched by their own worker
    (each BE client has its own done flag); results stay exact."""
    import torch
    import torch.nn.functional as F

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn(256, 1024, device="cuda", generator=g)
    b = torch.randn(1024, 1024, device="cuda", generator=g)
    A = torch.randn(4096, 4096, device="cuda", generator=g)
    x = torch.randn(16, 64, 56, 56, device="cuda", generator=g)
    w = torch.randn(128, 64, 3, 3, device="cuda", generator=g) * 0.05
    gamma = torch.rand(128, device="cuda", generator=g) + 0.5
    beta_ = torch.randn(128, device="cuda", generator=g)

    def conv_bn():
        rm, rv = torch.zeros(128, device="cuda"), torch.ones(128, device="cuda")
        y = F.conv2d(x, w, padding=1)
        return F.batch_norm(y, rm, rv, gamma, beta_, training=True, momentum=0.1), rm, rv

    assert orion.orion_init_scheduler(3) == 0
    orion.orion_set_capture(0)
    ref_hp, ref_be1, ref_be2 = a @ b, A @ A, conv_bn()
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    outs = {"hp": [], "be1": [], "be2": []}
    harness.run_clients(orion, lambda: outs["hp"].append(a @ b),
                        [lambda: outs["be1"].append(A @ A),
                         lambda: outs["be2"].append(conv_bn())],
                        hp_steps=60, hp_warmup=2)
    orion.orion_set_capture(0)
    stats = {c: orion.stats(c) for c in (0, 1, 2)}
    orion.orion_stop_scheduler()
    torch.cuda.synchronize()
    errs = {"hp": max(rel(o, ref_hp) for o in outs["hp"]),
            "be1": max(rel(o, ref_be1) for o in outs["be1"]),
            "be2_y": max(rel(o[0], ref_be2[0]) for o in outs["be2"]),
            "be2_rm": max(rel(o[1], ref_be2[1]) for o in outs["be2"]),
            "be2_rv": max(rel(o[2], ref_be2[2]) for o in outs["be2"])}
    return {"errors": errs, "stats": stats, "be_iters": [len(outs["be1"]), len(outs["be2"])]}


def scenario_trace(orion):
    """Capture trace of an HP + BE run: per-client issue instants, worker
    execution spans, blocking waits and HP-flag markers, as Chrome-trace JSON;
    plus the per-client wait counters."""
    import tempfile

    import torch

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(256, 1024, device="cuda", generator=g)
    b = torch.randn(1024, 1024, device="cuda", generator=g)
    A = torch.randn(2048, 2048, device="cuda", generator=g)
    assert orion.orion_init_scheduler(2) == 0
    orion.orion_set_capture(0)
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    for c in (0, 1):
        orion.waits(c, reset=True)
    orion.orion_trace_start()
    hp, be = harness.run_clients(orion, lambda: a @ b, lambda: A @ A, hp_steps=20, hp_warmup=2)
    path = os.path.join(tempfile.mkdtemp(), "trace.json.gz")
    n = harness.write_trace(orion, path)
    waits = {c: orion.waits(c) for c in (0, 1)}
    orion.orion_set_capture(0)
    orion.orion_stop_scheduler()
    torch.cuda.synchronize()
    import gzip
    ev = json.load(gzip.open(path))["traceEvents"]
    names = sorted({e["args"]["name"] for e in ev if e["ph"] == "M" and "name" in e["args"]})
    spans = [e for e in ev if e["ph"] == "X" and e["tid"] >= 100 and e["tid"] < 200]
    issues = {(e["tid"], e["args"]["op_id"]): e["ts"] for e in ev if e["ph"] == "i" and e["tid"] < 100}
    hp_gemms = [e for e in spans if e["tid"] == 100 and "GEMM" in e["name"] or
                e["tid"] == 100 and "MATMUL" in e["name"]]
    be_gemms = [e for e in spans if e["tid"] == 101 and ("GEMM" in e["name"] or "MATMUL" in e["name"])]
    matched = all((e["tid"] - 99, e["args"]["op_id"]) in issues and
                  issues[(e["tid"] - 99, e["args"]["op_id"])] <= e["ts"] + 1e-3 for e in spans)
    return {"events": n, "json_events": len(ev), "names": names, "hp_gemms": len(hp_gemms),
            "be_gemms": len(be_gemms), "spans_matched": matched,
            "nonneg": all(e["dur"] >= 0 and e["args"]["queued_us"] >= 0 for e in spans),
            "flag_markers": sorted({e["name"] for e in ev if e.get("tid") == 200 and e["ph"] == "i"}),
            "hp_waits": [e["name"] for e in ev if e["ph"] == "X" and e["tid"] == 1],
            "waits": waits, "hp_iters": hp.iters, "be_iters": be.iters}


def scenario_hgemm(orion):
    """cublasHgemm, cublasHgemmStridedBatched and cublasSgemmEx called
    directly (PyTorch issues none of them): captured on client 0 they run on
    the kx kernels; the same calls with capture off run on the real cuBLAS.
    Both are compared with a float64 product of the same operands."""
    import torch
    g = ctypes.CDLL(None)  # global scope: the preloaded interposer comes first
    P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    g.cublasHgemm.argtypes = [P, I, I, I, I, I, P, P, I, P, I, P, P, I]
    g.cublasHgemmStridedBatched.argtypes = [P, I, I, I, I, I, P, P, I, LL, P, I, LL, P, P, I,
                                            LL, I]
    g.cublasSgemmEx.argtypes = [P, I, I, I, I, I, P, P, I, I, P, I, I, P, P, I, I]
    for f in (g.cublasHgemm, g.cublasHgemmStridedBatched, g.cublasSgemmEx):
        f.restype = I
    gen = torch.Generator(device="cuda").manual_seed(7)

    def r(*shape, dtype):
        return torch.randn(*shape, device="cuda", generator=gen).to(dtype)

    def half(v):
        return ctypes.byref(ctypes.c_uint16(
            int(torch.tensor([v], dtype=torch.float16).view(torch.int16).item()) & 0xFFFF))

    def f32(v):
        return ctypes.byref(ctypes.c_float(v))

    h, bf = torch.float16, torch.bfloat16
    # column-major views: y^T (m x n) = W (m x k, stored k-major: transa = T) . x^T
    m, n, k = 384, 256, 320
    A, B = r(m, k, dtype=h), r(n, k, dtype=h)
    C0 = r(n, m, dtype=h)
    batch, sA, sB, sC = 3, m * k, n * k, n * m
    Ab, Bb, Cb0 = r(batch, m, k, dtype=h), r(batch, n, k, dtype=h), r(batch, n, m, dtype=h)
    Abf, Bbf = r(m, k, dtype=bf), r(n, k, dtype=bf)

    def ref64(a, b, alpha=1.0, beta=0.0, c=None):
        out = alpha * (b.double() @ a.double().t())
        if c is not None and beta != 0.0:
            out = out + beta * c.double()
        return out

    refs = {"hgemm": ref64(A, B, 1.5, 0.5, C0),
            "hgemm_strided_batched": torch.stack([ref64(Ab[i], Bb[i], 0.75, -1.0, Cb0[i])
                                                  for i in range(batch)]),
            "sgemmex_bf16_f32": ref64(Abf, Bbf),
            "sgemmex_f16_f16": ref64(A, B, 2.0, 0.0)}

    def run():
        handle = ctypes.c_void_p(torch.cuda.current_blas_handle())
        out = {}
        C = C0.clone()
        st = g.cublasHgemm(handle, 1, 0, m, n, k, half(1.5), A.data_ptr(), k, B.data_ptr(), k,
                           half(0.5), C.data_ptr(), m)
        out["hgemm"] = (st, C)
        Cb = Cb0.clone()
        st = g.cublasHgemmStridedBatched(handle, 1, 0, m, n, k, half(0.75), Ab.data_ptr(), k, sA,
                                         Bb.data_ptr(), k, sB, half(-1.0), Cb.data_ptr(), m, sC,
                                         batch)
        out["hgemm_strided_batched"] = (st, Cb)
        D = torch.zeros(n, m, device="cuda")
        st = g.cublasSgemmEx(handle, 1, 0, m, n, k, f32(1.0), Abf.data_ptr(), 14, k,
                             Bbf.data_ptr(), 14, k, f32(0.0), D.data_ptr(), 0, m)
        out["sgemmex_bf16_f32"] = (st, D)
        E = torch.zeros(n, m, device="cuda", dtype=h)
        st = g.cublasSgemmEx(handle, 1, 0, m, n, k, f32(2.0), A.data_ptr(), 2, k, B.data_ptr(),
                             2, k, f32(0.0), E.data_ptr(), 2, m)
        out["sgemmex_f16_f16"] = (st, E)
        torch.cuda.current_stream().synchronize()
        return out

    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    real = run_on_client(orion, 0, run)
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    cap = run_on_client(orion, 0, run)
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    res = {"stats": stats, "status": {}, "errors": {}, "real_errors": {}}
    for name, ref in refs.items():
        res["status"][name] = [real[name][0], cap[name][0]]
        res["errors"][name] = rel(cap[name][1], ref)
        res["real_errors"][name] = rel(real[name][1], ref)
    return res


def scenario_vgg16(orion):
    """End-to-end: the VGG16 forward of the HP client (fp32, batch 32 x
    3x224x224) captured on the kx kernels vs the same forward through the
    real cuDNN / cuBLAS (TF32 off), both against a float64 forward of two of
    the images (samples are independent in eval mode)."""
    import copy

    import torch

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.manual_seed(0)
    m = harness.make_vgg16("cuda").eval()
    x = torch.randn(32, 3, 224, 224, device="cuda")
    pick = [0, 31]
    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    with torch.no_grad():
        ref = m(x)
        ref64 = copy.deepcopy(m).double()(x[pick].double())
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)

    def fwd():
        with torch.no_grad():
            return m(x)

    out = run_on_client(orion, 0, fwd)
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    return {"errors": {"kx_vs_f64": rel(out[pick], ref64), "lib_vs_f64": rel(ref[pick], ref64),
                       "kx_vs_lib": rel(out, ref)}, "stats": stats}


def scenario_llama(orion):
    """End-to-end: the LLaMA-style decoder forward of the bf16 HP client
    (12 layers, d_model 2048, batch 4 x seq 1024) captured on the kx kernels
    vs the same forward through the real cuBLAS (bf16 in / out, fp32
    accumulation), both against an fp32 copy of the model (TF32 off) on one
    of the sequences."""
    import copy

    import torch

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    m = harness.make_llama(device="cuda", dtype=torch.bfloat16).eval()
    tok = torch.randint(0, 32000, (4, 1024), device="cuda")
    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    with torch.no_grad():
        ref = m(tok)
        m32 = copy.deepcopy(m).float()
        ref32 = m32(tok[:1])
        del m32
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)

    def fwd():
        with torch.no_grad():
            return m(tok)

    out = run_on_client(orion, 0, fwd)
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    return {"errors": {"kx_vs_f32": rel(out[:1], ref32), "lib_vs_f32": rel(ref[:1], ref32),
                       "kx_vs_lib": rel(out, ref)}, "stats": stats}


def scenario_gpt_train(orion):
    """End-to-end: one BE training step of the GPT decoder (fp32, batch 16 x
    256, cross-entropy against random targets): loss and gradients captured
    on the kx kernels vs the real libraries (TF32 off), both against a
    float64 copy of the model."""
    import copy

    import torch
    import torch.nn.functional as F

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    # dropout off: the three steps compared must see the same masks
    m = harness.make_gpt(device="cuda", dropout=0.0)
    tok = torch.randint(0, 32000, (16, 256), device="cuda")
    tgt = torch.randint(0, 32000, (16, 256), device="cuda")
    names = ["lm_head.weight", "blocks.0.mha.heads.0.query.weight", "blocks.5.ff.l1.weight",
             "token_embedding.weight"]

    def step(model):
        model.zero_grad(set_to_none=True)
        logits = model(tok)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]), tgt.view(-1))
        loss.backward()
        params = dict(model.named_parameters())
        return loss.detach().clone(), {n: params[n].grad.detach().clone() for n in names}

    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    loss_ref, g_ref = step(m)
    loss64, g64 = step(copy.deepcopy(m).double())
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    loss_kx, g_kx = run_on_client(orion, 0, lambda: step(m))
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    errs = {"loss": {"kx_vs_f64": rel(loss_kx, loss64), "lib_vs_f64": rel(loss_ref, loss64)}}
    for n in names:
        errs[n] = {"kx_vs_f64": rel(g_kx[n], g64[n]), "lib_vs_f64": rel(g_ref[n], g64[n]),
                   "kx_vs_lib": rel(g_kx[n], g_ref[n])}
    return {"errors": errs, "stats": stats, "loss": float(loss_kx)}


def scenario_gpt_curve(orion):
    """End-to-end: 20 AdamW steps of a two-layer GPT decoder (fp32, batch 8 x
    256, cross-entropy against fixed random targets) from one seed, three
    times: captured on the kx kernels, on the real libraries (TF32 off), and
    as a float64 copy.  Returns the three loss curves and the parameters'
    normwise distance to the float64 run after the last step."""
    import copy

    import torch
    import torch.nn.functional as F

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    base = harness.make_gpt(layers=2, device="cuda", dropout=0.0)
    tok = torch.randint(0, 32000, (8, 256), device="cuda")
    tgt = torch.randint(0, 32000, (8, 256), device="cuda")
    steps = 20

    def train(model):
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4)
        losses = []
        for _ in range(steps):
            opt.zero_grad(set_to_none=True)
            logits = model(tok)
            loss = F.cross_entropy(logits.view(-1, logits.shape[-1]), tgt.view(-1))
            loss.backward()
            opt.step()
            losses.append(loss.detach().double())
        return torch.stack(losses), model

    m_lib, m_kx, m64 = copy.deepcopy(base), copy.deepcopy(base), copy.deepcopy(base).double()
    assert orion.orion_init_scheduler(1) == 0
    orion.orion_set_capture(0)
    curve_lib, m_lib = train(m_lib)
    curve64, m64 = train(m64)
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    curve_kx, m_kx = run_on_client(orion, 0, lambda: train(m_kx))
    orion.orion_set_capture(0)
    stats = orion.stats(0)
    orion.orion_stop_scheduler()
    p64 = dict(m64.named_parameters())

    def param_err(m):
        return max(rel(p.detach(), p64[n].detach()) for n, p in m.named_parameters())

    return {"stats": stats,
            "curve_kx": curve_kx.tolist(), "curve_lib": curve_lib.tolist(),
            "curve64": curve64.tolist(),
            "loss_err_kx": [abs(a - b) / abs(b) for a, b in zip(curve_kx.tolist(),
                                                               curve64.tolist())],
            "loss_err_lib": [abs(a - b) / abs(b) for a, b in zip(curve_lib.tolist(),
                                                                curve64.tolist())],
            "param_err_kx": param_err(m_kx), "param_err_lib": param_err(m_lib)}


def scenario_tables(orion):
    """Per-client kernel tables measured through the interposer's profiler
    (kernel_intercept_b200.profile_tables): one row per kernel op the worker
    executes in a step, in order; then, with the tables loaded, an HP + BE
    run in which the Orion admission gate holds BE ops back."""
    import tempfile

    import torch

    from kernel_intercept_b200 import harness, profile_tables
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    m = harness.make_gpt(layers=2, device="cuda").eval()
    tok = torch.randint(0, 32000, (2, 256), device="cuda")
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(4096, 4096, device="cuda", generator=g)
    Bbig = torch.randn(64 << 20, device="cuda", generator=g)

    def hp_step():
        with torch.no_grad():
            m(tok)

    def be_step():
        # one captured GEMM (yields to HP at tile boundaries) and one long
        # re-issued elementwise kernel (cannot yield: the gate holds it back)
        A @ A
        Bbig.mul_(1.0000001)

    assert orion.orion_init_scheduler(2) == 0
    orion.orion_set_capture(0)
    hp_step()
    be_step()
    torch.cuda.synchronize()
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    for i, f in enumerate((hp_step, be_step)):
        profile_tables._run_on_client(orion, i, f)
    st0 = [orion.stats(c) for c in (0, 1)]
    d = tempfile.mkdtemp()
    paths = profile_tables.generate(orion, [hp_step, be_step], d)
    st1 = [orion.stats(c) for c in (0, 1)]
    rows = [profile_tables.read_csv(p) for p in paths]
    loaded = profile_tables.load(orion, paths)
    blocked0 = orion.stats(1)["be_blocked"]

    def be_gate_step():
        # the long re-issued kernel alone: a BE GEMM stopped by HP would hold
        # the BE worker until HP is idle, and the gate would see no BE op
        # while HP is active
        Bbig.mul_(1.0000001)

    harness.run_clients(orion, hp_step, be_gate_step, hp_steps=20, hp_warmup=1)
    stats = {c: orion.stats(c) for c in (0, 1)}
    orion.orion_set_capture(0)
    orion.orion_stop_scheduler()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return {"rows": [len(r) for r in rows], "loaded": loaded,
            "step_ops": [b["ops"] - a["ops"] for a, b in zip(st0, st1)],
            "step_kx_ops": [b["kx_ops"] - a["kx_ops"] for a, b in zip(st0, st1)],
            "hp_profiles": sorted({r[1] for r in rows[0]}),
            "sm_ok": all(1 <= r[3] <= sms for rs in rows for r in rs),
            "dur_ok": all(r[4] > 0 for rs in rows for r in rs),
            "names_ok": all(r[0] for rs in rows for r in rs),
            "hp_gemm_rows": sum(1 for r in rows[0] if r[1] == 1),
            "be_blocked": stats[1]["be_blocked"] - blocked0, "stats": stats}


def read_op_log(path):
    """Entries of an op log: (client, op type, route, shape integers)."""
    out = []
    with open(path) as f:
        for line in f:
            parts = line.rstrip("\n").split("\t")
            out.append((int(parts[0]), parts[1], parts[2], tuple(int(v) for v in parts[3:])))
    return out


def scenario_oplog(orion):
    """Op order and counts: one GPT training step (2 layers, batch 2 x 256)
    issued by client 0 through the real libraries (capture off) and then
    captured on the kx kernels must produce the same sequence of intercepted
    calls (type, shape, transposes, dtype); the worker must execute the
    captured ops in that order; and with an HP client (forward) and a BE
    client (training steps) running at once, each client's sequence must be
    its solo sequence (repeated per step)."""
    import tempfile

    import torch
    import torch.nn.functional as F

    from kernel_intercept_b200 import harness
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    m = harness.make_gpt(layers=2, device="cuda")
    opt = torch.optim.SGD(m.parameters(), lr=1e-3)
    tok = torch.randint(0, 32000, (2, 256), device="cuda")
    tgt = torch.randint(0, 32000, (2, 256), device="cuda")

    def train_step():
        logits = m(tok)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]), tgt.view(-1))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()

    def fwd_step():
        with torch.no_grad():
            m(tok)

    tmp = tempfile.mkdtemp()
    assert orion.orion_init_scheduler(2) == 0
    orion.orion_set_capture(0)
    train_step()  # warm-up: allocator, library handles
    torch.cuda.synchronize()

    def logged(path, fn):
        orion.orion_op_log_start()
        fn()
        torch.cuda.synchronize()
        n = orion.orion_op_log_end(path.encode())
        return read_op_log(path) if n >= 0 else None

    real = logged(os.path.join(tmp, "real.tsv"), lambda: run_on_client(orion, 0, train_step))
    real_fwd = logged(os.path.join(tmp, "real_fwd.tsv"), lambda: run_on_client(orion, 0, fwd_step))
    orion.orion_start_scheduler_thread()
    orion.orion_set_capture(1)
    prof = os.path.join(tmp, "prof.json")
    orion.orion_start_profiling(b"oplog")
    cap = logged(os.path.join(tmp, "cap.tsv"), lambda: run_on_client(orion, 0, train_step))
    orion.orion_end_profiling(prof.encode())
    with open(prof) as f:
        recs = json.load(f).get("kernels", [])
    both = logged(os.path.join(tmp, "both.tsv"), lambda: harness.run_clients(
        orion, fwd_step, train_step, hp_steps=4, hp_warmup=0, be_warmup=0))
    orion.orion_set_capture(0)
    stats = {c: orion.stats(c) for c in (0, 1)}
    orion.orion_stop_scheduler()

    def key(e):
        return (e[1], e[3])

    res = {"stats": stats, "n_real": len(real), "n_cap": len(cap)}
    res["same_sequence"] = [key(e) for e in real] == [key(e) for e in cap]
    res["real_routes"] = sorted({e[2] for e in real})
    res["cap_routes"] = sorted({e[2] for e in cap})
    res["clients"] = sorted({e[0] for e in real + cap})
    captured = [e[1] for e in cap if e[2] == "capture"]
    res["dispatch_order_same"] = [r.get("op_type") for r in recs if r.get("client") == 0] == captured
    hp = [key(e) for e in both if e[0] == 0]
    be = [key(e) for e in both if e[0] == 1]
    step_fwd = [key(e) for e in real_fwd]
    step_train = [key(e) for e in real]
    res["hp_steps_logged"] = len(hp) / max(1, len(step_fwd))
    res["be_steps_logged"] = len(be) / max(1, len(step_train))
    res["hp_matches_solo"] = len(hp) > 0 and hp == step_fwd * (len(hp) // max(1, len(step_fwd)))
    res["be_matches_solo"] = (len(be) % max(1, len(step_train)) == 0 and
                              be == step_train * (len(be) // max(1, len(step_train))))
    res["op_types"] = sorted({e[1] for e in real})
    return res


def main():
    scenario = sys.argv[1]
    from kernel_intercept_b200 import harness
    if not harness.preloaded():
        print(json.dumps({"error": "not preloaded"}))
        return 2
    orion = harness.Orion()
    res = globals()["scenario_" + scenario](orion)
    print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    rc = main()
    sys.stdout.flush()
    os._exit(rc)
