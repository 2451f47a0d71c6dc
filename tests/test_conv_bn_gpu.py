"""GPU parity of the kx convolution and batch-norm entry points against the
CPU oracle (fp32: normwise relative error <= 1e-5)."""
import os

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5

CONV_CASES = [
    # n, c, h, w, k, r, s, pad, stride, dil, xcorr
    (2, 8, 12, 12, 16, 3, 3, (1, 1), (1, 1), (1, 1), True),     # VGG-style 3x3 same
    (2, 3, 20, 20, 8, 3, 3, (1, 1), (1, 1), (1, 1), True),      # first layer, CRS = 27
    (2, 5, 13, 11, 7, 3, 3, (0, 1), (2, 1), (1, 1), True),      # strided, ragged
    (1, 4, 9, 10, 6, 3, 2, (2, 1), (1, 2), (2, 1), True),       # dilated
    (3, 6, 8, 8, 4, 3, 3, (1, 1), (1, 1), (1, 1), False),       # true convolution (flip)
    (2, 64, 14, 14, 64, 3, 3, (1, 1), (1, 1), (1, 1), True),    # VGG conv5-like shape
]


def _kx():
    from kernel_intercept_b200 import kx
    return kx


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _desc(case):
    kx = _kx()
    n, c, h, w, k, r, s, pad, stride, dil, xc = case
    return (kx.ConvDesc(n, c, h, w, k, r, s, pad[0], pad[1], stride[0], stride[1], dil[0], dil[1],
                        1 if xc else 0),
            o.conv_desc(n, c, h, w, k, r, s, pad=pad, stride=stride, dil=dil, xcorr=xc))


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_fwd(cuda, case):
    kx = _kx()
    import torch
    kd, od = _desc(case)
    rng = np.random.default_rng(sum(case[:7]))
    x = rng.standard_normal((od.n, od.c, od.h, od.w)).astype(np.float32)
    w = rng.standard_normal((od.k, od.c, od.r, od.s)).astype(np.float32)
    p, q = kx.conv_out_dims(kd)
    assert (p, q) == o.conv_out_dims(od)
    y0 = rng.standard_normal((od.n, od.k, p, q)).astype(np.float32)
    ref = o.conv_fwd(od, 1.5, x, w, beta=0.5, y=y0.copy())
    dx, dw, dy = _dev(x), _dev(w), _dev(y0)
    kx.conv_fwd(kx.current_exec(), kd, 1.5, dx.data_ptr(), dw.data_ptr(), 0.5, dy.data_ptr())
    torch.cuda.synchronize()
    assert o.normwise_rel_err(dy.cpu().numpy(), ref) <= TOL_F32


IMPLICIT_CASES = [
    (8, 32, 56, 56, 128, 3, 3, (1, 1), (1, 1), (1, 1), True),   # 128-wide channel tiles
    (2, 40, 17, 19, 72, 3, 3, (1, 1), (1, 1), (1, 1), True),    # partial channel block, ragged K
    (2, 96, 15, 15, 64, 1, 1, (0, 0), (1, 1), (1, 1), True),    # 1x1
    (2, 16, 30, 30, 32, 5, 5, (2, 2), (2, 2), (1, 1), False),   # 5x5 strided, flipped
    (2, 64, 28, 28, 128, 3, 3, (1, 1), (2, 2), (1, 1), True),   # stride 2 (TMA element strides)
    (2, 32, 20, 22, 64, 3, 3, (2, 2), (1, 1), (2, 2), True),    # dilated taps
    (4, 3, 64, 64, 64, 3, 3, (1, 1), (1, 1), (1, 1), True),     # C = 3: taps folded into K
    (3, 64, 14, 14, 128, 3, 3, (1, 1), (1, 1), (1, 1), True),   # 128-pixel tiles across images
    (4, 32, 7, 7, 64, 3, 3, (1, 1), (1, 1), (1, 1), True),      # P*Q = 49: per-element stores
    (2, 48, 21, 26, 96, 3, 5, (1, 2), (1, 2), (1, 1), True),    # R != S, pad_h != pad_w
    (8, 256, 14, 14, 256, 3, 3, (1, 1), (1, 1), (1, 1), True),  # split K (4 slices)
]


@pytest.mark.parametrize("case", IMPLICIT_CASES)
def test_conv_fwd_implicit_gemm(cuda, case):
    """Forward convolution on the implicit-GEMM kernel (A tiles by 4-D TMA
    from the NHWC staging copy; folded taps for small C*R*S)."""
    kx = _kx()
    import torch
    kd, od = _desc(case)
    rng = np.random.default_rng(3 + sum(case[:7]))
    x = rng.standard_normal((od.n, od.c, od.h, od.w)).astype(np.float32)
    w = rng.standard_normal((od.k, od.c, od.r, od.s)).astype(np.float32)
    p, q = o.conv_out_dims(od)
    y0 = rng.standard_normal((od.n, od.k, p, q)).astype(np.float32)
    ref = o.conv_fwd(od, 0.5, x, w, beta=-0.25, y=y0.copy())
    dx, dw, dy = _dev(x), _dev(w), _dev(y0)
    kx.conv_fwd(kx.current_exec(), kd, 0.5, dx.data_ptr(), dw.data_ptr(), -0.25, dy.data_ptr())
    torch.cuda.synchronize()
    name = kx.last_kernel_name()
    assert name.startswith("kx_conv_fwd_tc<")
    mode = os.environ.get("KX_CONV_IM2COL")
    if mode is not None:
        assert ("box" if mode == "0" else "im2col") in name
    pair = os.environ.get("KX_CTA_PAIR")
    if pair is not None:
        assert (",pair>" in name) == (pair == "1")
    assert o.normwise_rel_err(dy.cpu().numpy(), ref) <= TOL_F32


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("mode", ["0", "1"])
@pytest.mark.parametrize("case", IMPLICIT_CASES)
def test_conv_fwd_tile_modes(cuda, case, mode, pair, monkeypatch):
    """Every A-tile form of the kernel on every case: 4-D TMA boxes of whole
    output rows (KX_CONV_IM2COL=0) or im2col-mode loads of 128 consecutive
    output pixels (KX_CONV_IM2COL=1), on one CTA per 128-row tile
    (KX_CTA_PAIR=0) or on 2-CTA clusters with cta_group::2 MMAs over
    256-row tiles (KX_CTA_PAIR=1)."""
    monkeypatch.setenv("KX_CONV_IM2COL", mode)
    monkeypatch.setenv("KX_CTA_PAIR", pair)
    test_conv_fwd_implicit_gemm(cuda, case)


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_bwd_data(cuda, case):
    kx = _kx()
    import torch
    kd, od = _desc(case)
    rng = np.random.default_rng(7 + sum(case[:7]))
    p, q = o.conv_out_dims(od)
    w = rng.standard_normal((od.k, od.c, od.r, od.s)).astype(np.float32)
    gy = rng.standard_normal((od.n, od.k, p, q)).astype(np.float32)
    dx0 = rng.standard_normal((od.n, od.c, od.h, od.w)).astype(np.float32)
    ref = o.conv_bwd_data(od, 0.75, w, gy, beta=-1.0, dx=dx0.copy())
    dw_, dgy, ddx = _dev(w), _dev(gy), _dev(dx0)
    kx.conv_bwd_data(kx.current_exec(), kd, 0.75, dw_.data_ptr(), dgy.data_ptr(), -1.0,
                     ddx.data_ptr())
    torch.cuda.synchronize()
    assert o.normwise_rel_err(ddx.cpu().numpy(), ref) <= TOL_F32


# stride-1 cases: backward data runs as a forward implicit-GEMM convolution of
# dy with the transposed, flipped filter
DGRAD_IMPLICIT_CASES = [
    (8, 32, 56, 56, 128, 3, 3, (1, 1), (1, 1), (1, 1), True),
    (2, 32, 20, 22, 64, 3, 3, (2, 2), (1, 1), (2, 2), True),    # dilated
    (2, 48, 21, 26, 96, 3, 5, (1, 2), (1, 1), (1, 1), True),    # R != S, pad_h != pad_w
    (2, 16, 30, 30, 32, 5, 5, (2, 2), (1, 1), (1, 1), False),   # true convolution
    (4, 3, 32, 32, 64, 3, 3, (1, 1), (1, 1), (1, 1), True),     # 3 input channels
    (3, 64, 14, 14, 128, 3, 3, (1, 1), (1, 1), (1, 1), True),
]


@pytest.mark.parametrize("case", DGRAD_IMPLICIT_CASES)
def test_conv_bwd_data_implicit(cuda, case):
    """Backward data on the implicit-GEMM kernel (stride 1)."""
    kx = _kx()
    test_conv_bwd_data(cuda, case)
    assert kx.last_kernel_name().startswith("kx_conv_fwd_tc<")


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_bwd_filter(cuda, case):
    kx = _kx()
    import torch
    kd, od = _desc(case)
    rng = np.random.default_rng(11 + sum(case[:7]))
    p, q = o.conv_out_dims(od)
    x = rng.standard_normal((od.n, od.c, od.h, od.w)).astype(np.float32)
    gy = rng.standard_normal((od.n, od.k, p, q)).astype(np.float32)
    dw0 = rng.standard_normal((od.k, od.c, od.r, od.s)).astype(np.float32)
    ref = o.conv_bwd_filter(od, 2.0, x, gy, beta=0.25, dw=dw0.copy())
    dx_, dgy, ddw = _dev(x), _dev(gy), _dev(dw0)
    kx.conv_bwd_filter(kx.current_exec(), kd, 2.0, dx_.data_ptr(), dgy.data_ptr(), 0.25,
                       ddw.data_ptr())
    torch.cuda.synchronize()
    assert o.normwise_rel_err(ddw.cpu().numpy(), ref) <= TOL_F32


# backward filter on the implicit-GEMM kernel (>= 64 channels, P*Q % 4 == 0):
# dy as the A operand, im2col-mode loads of x as B, split over the pixel sum
WGRAD_IMPLICIT_CASES = [
    (8, 64, 56, 56, 128, 3, 3, (1, 1), (1, 1), (1, 1), True),
    (2, 128, 20, 22, 64, 3, 3, (2, 2), (1, 1), (2, 2), True),   # dilated
    (2, 128, 20, 28, 96, 3, 5, (1, 2), (1, 2), (1, 1), True),   # R != S, stride 2 in W
    (2, 64, 16, 16, 32, 5, 5, (2, 2), (1, 1), (1, 1), False),   # true convolution
    (3, 512, 14, 14, 128, 3, 3, (1, 1), (1, 1), (1, 1), True),  # P*Q = 196: partial block
    (4, 3, 32, 32, 64, 3, 3, (1, 1), (1, 1), (1, 1), True),     # C = 3: taps folded
]


@pytest.mark.parametrize("case", WGRAD_IMPLICIT_CASES)
def test_conv_bwd_filter_implicit(cuda, case):
    kx = _kx()
    test_conv_bwd_filter(cuda, case)
    assert kx.last_kernel_name().startswith("kx_conv_wgrad_tc<")


def test_conv_invalid(cuda):
    kx = _kx()
    bad = kx.ConvDesc(1, 1, 2, 2, 1, 5, 5, 0, 0, 1, 1, 1, 1, 1)  # filter larger than input
    assert kx.lib().kx_conv_out_dims(bad, None, None) == kx.ERR_INVALID


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("shape", [(4, 3, 5, 6), (8, 16, 14, 14), (2, 4, 7, 9)])
def test_batchnorm_fwd_bwd(cuda, mode, shape):
    kx = _kx()
    import torch
    n, c, h, w = shape
    rng = np.random.default_rng(mode * 100 + sum(shape))
    G = c if mode == 1 else c * h * w
    x = (rng.standard_normal(shape) * 3 + 2).astype(np.float32)
    scale = rng.standard_normal(G).astype(np.float32)
    bias = rng.standard_normal(G).astype(np.float32)
    rmean = rng.standard_normal(G).astype(np.float32)
    rvar = (rng.random(G) + 0.5).astype(np.float32)
    y0 = rng.standard_normal(shape).astype(np.float32)
    # oracle
    o_y, o_rm, o_rv = y0.copy(), rmean.copy(), rvar.copy()
    o_sm, o_si = np.zeros(G, np.float32), np.zeros(G, np.float32)
    o.bn_fwd_training(mode, 1.0, 0.5, x, o_y, scale, bias, 0.1, o_rm, o_rv, 1e-5, o_sm, o_si)
    # kx
    d = {k_: _dev(v) for k_, v in dict(x=x, y=y0, scale=scale, bias=bias, rm=rmean, rv=rvar,
                                       sm=np.zeros(G, np.float32),
                                       si=np.zeros(G, np.float32)).items()}
    kx.bn_fwd_training(kx.current_exec(), mode, 1.0, 0.5, n, c, h, w, d["x"].data_ptr(),
                       d["y"].data_ptr(), d["scale"].data_ptr(), d["bias"].data_ptr(), 0.1,
                       d["rm"].data_ptr(), d["rv"].data_ptr(), 1e-5, d["sm"].data_ptr(),
                       d["si"].data_ptr())
    torch.cuda.synchronize()
    assert o.normwise_rel_err(d["y"].cpu().numpy(), o_y) <= TOL_F32
    assert o.normwise_rel_err(d["rm"].cpu().numpy(), o_rm) <= TOL_F32
    assert o.normwise_rel_err(d["rv"].cpu().numpy(), o_rv) <= TOL_F32
    assert o.normwise_rel_err(d["sm"].cpu().numpy(), o_sm) <= TOL_F32
    assert o.normwise_rel_err(d["si"].cpu().numpy(), o_si) <= TOL_F32
    # inference with the running statistics
    o_yi = np.zeros(shape, np.float32)
    o.bn_fwd_inference(mode, 1.0, 0.0, x, o_yi, scale, bias, o_rm, o_rv, 1e-5)
    yi = torch.zeros(shape, device="cuda")
    kx.bn_fwd_inference(kx.current_exec(), mode, 1.0, 0.0, n, c, h, w, d["x"].data_ptr(),
                        yi.data_ptr(), d["scale"].data_ptr(), d["bias"].data_ptr(),
                        d["rm"].data_ptr(), d["rv"].data_ptr(), 1e-5)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(yi.cpu().numpy(), o_yi) <= TOL_F32
    # backward with saved statistics, and with recomputed ones
    gy = rng.standard_normal(shape).astype(np.float32)
    for use_saved in (True, False):
        o_dx = np.zeros(shape, np.float32)
        o_ds = np.ones(G, np.float32)
        o_db = np.ones(G, np.float32)
        o.bn_bwd(mode, 1.0, 0.0, 1.0, 0.5, x, gy, o_dx, scale, o_ds, o_db, 1e-5, o_sm, o_si)
        ddx = torch.zeros(shape, device="cuda")
        dds = torch.ones(G, device="cuda")
        ddb = torch.ones(G, device="cuda")
        dgy = _dev(gy)
        kx.bn_bwd(kx.current_exec(), mode, 1.0, 0.0, 1.0, 0.5, n, c, h, w, d["x"].data_ptr(),
                  dgy.data_ptr(), ddx.data_ptr(), d["scale"].data_ptr(), dds.data_ptr(),
                  ddb.data_ptr(), 1e-5, d["sm"].data_ptr() if use_saved else None,
                  d["si"].data_ptr() if use_saved else None)
        torch.cuda.synchronize()
        assert o.normwise_rel_err(ddx.cpu().numpy(), o_dx) <= TOL_F32
        assert o.normwise_rel_err(dds.cpu().numpy(), o_ds) <= TOL_F32
        assert o.normwise_rel_err(ddb.cpu().numpy(), o_db) <= TOL_F32
