"""Allocation-free batch-norm training entry point (kx_bn_fwd_training_noalloc).

Called through the C ABI twice in a row on different inputs; each result is
compared with the regular kx_bn_fwd_training on the same inputs (tolerance of
the fp32 parity tests: normwise relative error <= 1e-5).  Collected last so
that it runs both alone in a fresh process and after every other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5


def _run(fn_name, mode, x, scale, bias, rmean, rvar, y0):
    import torch

    from kernel_intercept_b200 import kx
    n, c, h, w = x.shape
    d = {k: v.clone() for k, v in dict(x=x, y=y0, scale=scale, bias=bias, rm=rmean,
                                         rv=rvar).items()}
    G = d["scale"].numel()
    d["sm"] = torch.zeros(G, device="cuda")
    d["si"] = torch.zeros(G, device="cuda")
    alpha, beta = ctypes.c_float(1.0), ctypes.c_float(0.5)
    fn = getattr(kx.lib(), fn_name)
    ex = kx.current_exec()
    st = fn(ctypes.byref(ex), mode, ctypes.byref(alpha), ctypes.byref(beta), n, c, h, w,
            d["x"].data_ptr(), d["y"].data_ptr(), d["scale"].data_ptr(), d["bias"].data_ptr(),
            0.1, d["rm"].data_ptr(), d["rv"].data_ptr(), 1e-5, d["sm"].data_ptr(),
            d["si"].data_ptr())
    torch.cuda.synchronize()
    return st, {k: d[k].cpu().numpy() for k in ("y", "rm", "rv", "sm", "si")}


def _inputs(mode, shape, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    n, c, h, w = shape
    G = c if mode != 0 else c * h * w
    x = torch.randn(*shape, device="cuda", generator=g) * 3 + 1
    return (x, torch.rand(G, device="cuda", generator=g) + 0.5,
            torch.randn(G, device="cuda", generator=g),
            torch.randn(G, device="cuda", generator=g),
            torch.rand(G, device="cuda", generator=g) + 0.5,
            torch.randn(*shape, device="cuda", generator=g))


def _err(a, b):
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / (den if den > 0 else 1.0))


@pytest.mark.parametrize("mode,shape", [(1, (8, 64, 28, 28)), (2, (4, 32, 15, 17)),
                                        (0, (16, 8, 7, 7))])
def test_no_alloc_matches_regular_entry_point(cuda, mode, shape):
    for call, seed in enumerate((11, 12)):  # two calls in a row share the scratch array
        args = _inputs(mode, shape, seed + 10 * mode)
        st_ref, ref = _run("kx_bn_fwd_training", mode, *args)
        st, got = _run("kx_bn_fwd_training_noalloc", mode, *args)
        assert st_ref == 0 and st == 0, (st_ref, st)
        for k in ref:
            assert _err(got[k], ref[k]) <= TOL_F32, (call, k)


def test_no_alloc_rejects_oversize(cuda):
    import torch
    from kernel_intercept_b200 import kx
    # per-activation statistics of 1 Mi features need 8 MiB of scratch > 4 MiB
    shape = (2, 1, 1024, 1024)
    args = _inputs(0, shape, 5)
    y_before = args[5].clone()
    st, got = _run("kx_bn_fwd_training_noalloc", 0, *args)
    assert st == kx.ERR_INVALID
    assert np.array_equal(got["y"], y_before.cpu().numpy())
    torch.cuda.synchronize()
