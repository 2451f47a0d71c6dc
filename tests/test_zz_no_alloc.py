"""Allocation-free batch-norm training entry point (kx_bn_fwd_training_noalloc).

Some callers cannot allocate device memory while they run an op: a CUDA graph
being captured, or a host that hands every device byte to its own allocator.
For them kx_bn_fwd_training_noalloc keeps its statistics scratch in a static
device array instead of the stream's scratch buffer.  These tests call it
through the C ABI twice in a row on different inputs (the two calls share the
array) and check each result against the CPU oracle and against the regular
kx_bn_fwd_training on the same inputs, at the fp32 parity tolerance
(normwise relative error <= 1e-5).  They also check the property the entry
point exists for: the library's device-allocation count does not move across
its calls, including the first call on a fresh stream.  Collected last so that
it runs both alone in a fresh process and after every other test.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
ALPHA, BETA, FACTOR, EPS = 1.0, 0.5, 0.1, 1e-5


def _run(fn_name, mode, host, stream=None):
    """Runs one entry point on device copies of the host arrays; returns the
    status and the outputs (y, running mean / var, saved mean / inv std)."""
    import torch

    from kernel_intercept_b200 import kx
    n, c, h, w = host["x"].shape
    d = {k: torch.from_numpy(v.copy()).cuda() for k, v in host.items()}
    G = host["scale"].size
    d["sm"] = torch.zeros(G, device="cuda")
    d["si"] = torch.zeros(G, device="cuda")
    alpha, beta = ctypes.c_float(ALPHA), ctypes.c_float(BETA)
    fn = getattr(kx.lib(), fn_name)
    ex = kx.make_exec(stream=stream) if stream is not None else kx.current_exec()
    torch.cuda.synchronize()
    st = fn(ctypes.byref(ex), mode, ctypes.byref(alpha), ctypes.byref(beta), n, c, h, w,
            d["x"].data_ptr(), d["y"].data_ptr(), d["scale"].data_ptr(), d["bias"].data_ptr(),
            FACTOR, d["rm"].data_ptr(), d["rv"].data_ptr(), EPS, d["sm"].data_ptr(),
            d["si"].data_ptr())
    torch.cuda.synchronize()
    return st, {k: d[k].cpu().numpy() for k in ("y", "rm", "rv", "sm", "si")}


def _inputs(mode, shape, seed):
    rng = np.random.default_rng(seed)
    n, c, h, w = shape
    G = c if mode != 0 else c * h * w
    f = np.float32
    return {"x": (rng.standard_normal(shape) * 3 + 1).astype(f),
            "scale": (rng.random(G) + 0.5).astype(f),
            "bias": rng.standard_normal(G).astype(f),
            "rm": rng.standard_normal(G).astype(f),
            "rv": (rng.random(G) + 0.5).astype(f),
            "y": rng.standard_normal(shape).astype(f)}


def _oracle(mode, host):
    G = host["scale"].size
    out = {"y": host["y"].copy(), "rm": host["rm"].copy(), "rv": host["rv"].copy(),
           "sm": np.zeros(G, np.float32), "si": np.zeros(G, np.float32)}
    o.bn_fwd_training(mode, ALPHA, BETA, host["x"], out["y"], host["scale"], host["bias"],
                      FACTOR, out["rm"], out["rv"], EPS, out["sm"], out["si"])
    return out


@pytest.mark.parametrize("mode,shape", [(1, (8, 64, 28, 28)), (2, (4, 32, 15, 17)),
                                        (0, (16, 8, 7, 7)), (1, (64, 64, 14, 14))])
def test_no_alloc_matches_oracle_and_regular_entry_point(cuda, mode, shape):
    from kernel_intercept_b200 import kx
    for call, seed in enumerate((11, 12)):  # two calls in a row share the scratch array
        host = _inputs(mode, shape, seed + 10 * mode)
        ref = _oracle(mode, host)
        st_reg, reg = _run("kx_bn_fwd_training", mode, host)
        allocs = kx.lib().kx_device_alloc_count()
        st, got = _run("kx_bn_fwd_training_noalloc", mode, host)
        assert kx.lib().kx_device_alloc_count() == allocs, "the no-alloc call allocated"
        assert st_reg == 0 and st == 0, (st_reg, st)
        for k in ref:
            assert o.normwise_rel_err(got[k], ref[k]) <= TOL_F32, (call, k, "vs oracle")
            assert o.normwise_rel_err(got[k], reg[k]) <= TOL_F32, (call, k, "vs regular")


def test_no_alloc_on_a_fresh_stream_allocates_nothing(cuda):
    import torch

    from kernel_intercept_b200 import kx
    host = _inputs(1, (4, 16, 10, 12), 3)
    ref = _oracle(1, host)
    stream = torch.cuda.Stream()
    allocs = kx.lib().kx_device_alloc_count()
    for _ in range(2):
        st, got = _run("kx_bn_fwd_training_noalloc", 1, host, stream=stream)
        assert st == 0
        assert o.normwise_rel_err(got["y"], ref["y"]) <= TOL_F32
    assert kx.lib().kx_device_alloc_count() == allocs
    # the counter does see allocations: the regular entry point's first call on
    # a new stream creates that stream's scratch buffer
    st, _ = _run("kx_bn_fwd_training", 1, host, stream=torch.cuda.Stream())
    assert st == 0 and kx.lib().kx_device_alloc_count() > allocs


def test_no_alloc_rejects_oversize(cuda):
    from kernel_intercept_b200 import kx
    # per-activation statistics of 1 Mi features need 8 MiB of scratch > 4 MiB
    host = _inputs(0, (2, 1, 1024, 1024), 5)
    st, got = _run("kx_bn_fwd_training_noalloc", 0, host)
    assert st == kx.ERR_INVALID
    assert np.array_equal(got["y"], host["y"])
