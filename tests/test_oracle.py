"""CPU checks of the oracle itself (no GPU).

The oracle restates cuBLAS / cuDNN semantics; here it is checked against
independent fp64 formulations (numpy matmul, torch CPU conv2d / autograd /
batch_norm) and, when present, against the golden fixtures captured from the
reference shim on a B200 (tests/golden/*.npz, made by tests/golden/make_golden.py).
"""
import glob
import sys
import os

import numpy as np
import pytest
import torch

from oracle import oracle as o

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _colmajor(buf, rows, cols, ld):
    return buf.reshape(cols, ld).T[:rows, :cols]


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_sgemm_matches_numpy(ta, tb):
    rng = np.random.default_rng(ta * 2 + tb)
    m, n, k = 45, 37, 29
    lda = (m if ta == 0 else k) + 3
    ldb = (k if tb == 0 else n) + 1
    ldc = m + 2
    A = rng.standard_normal(lda * (k if ta == 0 else m)).astype(np.float32)
    B = rng.standard_normal(ldb * (n if tb == 0 else k)).astype(np.float32)
    C = rng.standard_normal(ldc * n).astype(np.float32)
    C0 = C.copy()
    o.sgemm(ta, tb, m, n, k, 1.25, A, lda, B, ldb, -0.5, C, ldc)
    Am = _colmajor(A, m, k, lda) if ta == 0 else _colmajor(A, k, m, lda).T
    Bm = _colmajor(B, k, n, ldb) if tb == 0 else _colmajor(B, n, k, ldb).T
    ref = 1.25 * (Am.astype(np.float64) @ Bm.astype(np.float64)) - 0.5 * _colmajor(C0, m, n, ldc)
    assert o.normwise_rel_err(_colmajor(C, m, n, ldc), ref) < 1e-6
    # padding rows untouched
    assert np.array_equal(C.reshape(n, ldc)[:, m:], C0.reshape(n, ldc)[:, m:])


def test_sgemm_beta_zero_ignores_nan():
    A = np.ones(4, np.float32)
    B = np.ones(4, np.float32)
    C = np.full(4, np.nan, np.float32)
    o.sgemm(0, 0, 2, 2, 2, 1.0, A, 2, B, 2, 0.0, C, 2)
    assert np.all(C == 2.0)


def test_strided_batched_and_typed():
    rng = np.random.default_rng(5)
    b, m, n, k = 3, 8, 6, 5
    A = rng.standard_normal(b * m * k).astype(np.float32)
    B = rng.standard_normal(b * k * n).astype(np.float32)
    C = np.zeros(b * m * n, np.float32)
    o.sgemm_strided_batched(0, 0, m, n, k, 1.0, A, m, m * k, B, k, k * n, 0.0, C, m, m * n, b)
    for i in range(b):
        Ai = A[i * m * k:(i + 1) * m * k]
        Bi = B[i * k * n:(i + 1) * k * n]
        Ci = C[i * m * n:(i + 1) * m * n]
        ref = _colmajor(Ai, m, k, m).astype(np.float64) @ _colmajor(Bi, k, n, k)
        assert o.normwise_rel_err(_colmajor(Ci, m, n, m), ref) < 1e-6
    # bf16 operands, bf16 result, bias + ReLU epilogue
    Ab = o.f32_to_bf16_bits(A[:m * k])
    Bb = o.f32_to_bf16_bits(B[:k * n])
    bias = rng.standard_normal(m).astype(np.float32)
    D = np.zeros(m * n, np.uint16)
    o.gemm_ex(0, 0, m, n, k, 1.0, Ab, o.R_16BF, m, Bb, o.R_16BF, k, 0.0, None, o.R_16BF, m, D=D,
              Dtype=o.R_16BF, ldd=m, epilogue=6, bias=bias)
    ref = _colmajor(o.bf16_bits_to_f32(Ab), m, k, m).astype(np.float64) @ _colmajor(
        o.bf16_bits_to_f32(Bb), k, n, k) + bias[:, None]
    ref = np.maximum(ref, 0)
    assert o.normwise_rel_err(_colmajor(o.bf16_bits_to_f32(D), m, n, m), ref) < 1e-2


def test_bf16_rounding_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 1e3
    ours = o.bf16_bits_to_f32(o.f32_to_bf16_bits(x))
    theirs = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours, theirs)


@pytest.mark.parametrize("pad,stride,dil", [((1, 1), (1, 1), (1, 1)), ((0, 2), (2, 1), (1, 2)),
                                            ((2, 0), (1, 3), (2, 1))])
def test_conv_matches_torch(pad, stride, dil):
    rng = np.random.default_rng(sum(pad) + sum(stride))
    n, c, h, w, k, r, s = 2, 3, 11, 13, 4, 3, 3
    d = o.conv_desc(n, c, h, w, k, r, s, pad=pad, stride=stride, dil=dil)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = rng.standard_normal((k, c, r, s)).astype(np.float32)
    xt = torch.from_numpy(x).double().requires_grad_()
    wtt = torch.from_numpy(wt).double().requires_grad_()
    yt = torch.nn.functional.conv2d(xt, wtt, stride=stride, padding=pad, dilation=dil)
    y = o.conv_fwd(d, 1.0, x, wt)
    assert o.normwise_rel_err(y, yt.detach().numpy()) < 1e-6
    g = torch.from_numpy(rng.standard_normal(yt.shape).astype(np.float32)).double()
    yt.backward(g)
    dx = o.conv_bwd_data(d, 1.0, wt, g.float().numpy())
    dw = o.conv_bwd_filter(d, 1.0, x, g.float().numpy())
    assert o.normwise_rel_err(dx, xt.grad.numpy()) < 1e-6
    assert o.normwise_rel_err(dw, wtt.grad.numpy()) < 1e-6


def test_conv_alpha_beta_and_flip():
    rng = np.random.default_rng(9)
    d = o.conv_desc(1, 2, 6, 6, 3, 3, 3, pad=(1, 1))
    x = rng.standard_normal((1, 2, 6, 6)).astype(np.float32)
    w = rng.standard_normal((3, 2, 3, 3)).astype(np.float32)
    y0 = rng.standard_normal((1, 3, 6, 6)).astype(np.float32)
    y = o.conv_fwd(d, 2.0, x, w, beta=0.5, y=y0.copy())
    ref = 2.0 * torch.nn.functional.conv2d(torch.from_numpy(x).double(),
                                           torch.from_numpy(w).double(), padding=1).numpy()
    assert o.normwise_rel_err(y, ref + 0.5 * y0) < 1e-6
    # CUDNN_CONVOLUTION (true convolution) == cross-correlation with a flipped filter
    dc = o.conv_desc(1, 2, 6, 6, 3, 3, 3, pad=(1, 1), xcorr=False)
    yc = o.conv_fwd(dc, 1.0, x, w)
    yf = o.conv_fwd(d, 1.0, x, np.ascontiguousarray(w[:, :, ::-1, ::-1]))
    assert o.normwise_rel_err(yc, yf) < 1e-6


@pytest.mark.parametrize("mode", [0, 1])
def test_batchnorm_matches_torch(mode):
    rng = np.random.default_rng(mode)
    n, c, h, w = 4, 3, 5, 6
    x = rng.standard_normal((n, c, h, w)).astype(np.float32) * 2 + 1
    G = c if mode == 1 else c * h * w
    scale = rng.standard_normal(G).astype(np.float32)
    bias = rng.standard_normal(G).astype(np.float32)
    rmean = np.zeros(G, np.float32)
    rvar = np.ones(G, np.float32)
    smean = np.zeros(G, np.float32)
    sinv = np.zeros(G, np.float32)
    y = np.zeros_like(x)
    o.bn_fwd_training(mode, 1.0, 0.0, x, y, scale, bias, 0.1, rmean, rvar, 1e-5, smean, sinv)
    xt = torch.from_numpy(x).double()
    if mode == 1:
        rm = torch.zeros(c, dtype=torch.float64)
        rv = torch.ones(c, dtype=torch.float64)
        xr = xt.clone().requires_grad_()
        st = torch.from_numpy(scale).double().requires_grad_()
        bt = torch.from_numpy(bias).double().requires_grad_()
        yt = torch.nn.functional.batch_norm(xr, rm, rv, st, bt, training=True, momentum=0.1,
                                            eps=1e-5)
    else:
        flat = xt.reshape(n, -1)
        rm = torch.zeros(G, dtype=torch.float64)
        rv = torch.ones(G, dtype=torch.float64)
        xr = flat.clone().requires_grad_()
        st = torch.from_numpy(scale).double().requires_grad_()
        bt = torch.from_numpy(bias).double().requires_grad_()
        yt = torch.nn.functional.batch_norm(xr, rm, rv, st, bt, training=True, momentum=0.1,
                                            eps=1e-5)
    assert o.normwise_rel_err(y.reshape(yt.shape), yt.detach().numpy()) < 1e-6
    assert o.normwise_rel_err(rmean, rm.numpy()) < 1e-6
    assert o.normwise_rel_err(rvar, rv.numpy()) < 1e-6
    g = rng.standard_normal(yt.shape)
    yt.backward(torch.from_numpy(g))
    dx = np.zeros_like(x)
    ds = np.zeros(G, np.float32)
    db = np.zeros(G, np.float32)
    o.bn_bwd(mode, 1.0, 0.0, 1.0, 0.0, x, g.reshape(x.shape).astype(np.float32), dx, scale, ds,
             db, 1e-5, smean, sinv)
    assert o.normwise_rel_err(dx.reshape(yt.shape), xr.grad.numpy()) < 1e-5
    assert o.normwise_rel_err(ds, st.grad.numpy()) < 1e-5
    assert o.normwise_rel_err(db, bt.grad.numpy()) < 1e-5
    # inference with the running statistics
    yi = np.zeros_like(x)
    o.bn_fwd_inference(mode, 1.0, 0.0, x, yi, scale, bias, rmean, rvar, 1e-5)
    ti = torch.nn.functional.batch_norm(xt.reshape(yt.shape), rm, rv,
                                        torch.from_numpy(scale).double(),
                                        torch.from_numpy(bias).double(), training=False, eps=1e-5)
    assert o.normwise_rel_err(yi.reshape(ti.shape), ti.numpy()) < 1e-6


# ------------------------------------------------------ golden fixtures ---

def _check_bn_golden(z, path):
    """cuDNN spatial batch norm (training forward + backward) at a VGG-like
    shape: inputs regenerated from the fixture's seed, the oracle's outputs
    against cuDNN's per-channel results and sampled y / dx."""
    sys.path.insert(0, GOLDEN)
    import make_golden as mg
    shape = tuple(int(v) for v in z["dims"])
    factor, eps = (float(v) for v in z["scalars"])
    x, scale, bias, rm, rv, dy = mg.bn_inputs(shape, int(z["seed"]))
    c = shape[1]
    y = np.zeros(shape, np.float32)
    sm, si = np.zeros(c, np.float32), np.zeros(c, np.float32)
    o.bn_fwd_training(1, 1.0, 0.0, x, y, scale, bias, factor, rm, rv, eps, sm, si)
    dx = np.zeros(shape, np.float32)
    ds, db = np.zeros(c, np.float32), np.zeros(c, np.float32)
    o.bn_bwd(1, 1.0, 0.0, 1.0, 0.0, x, dy, dx, scale, ds, db, eps, sm, si)
    ni, ci = mg.bn_sample(shape)
    for name, got in (("y", y[ni][:, ci]), ("dx", dx[ni][:, ci]), ("running_mean", rm),
                      ("running_var", rv), ("save_mean", sm), ("save_inv_std", si),
                      ("dscale", ds), ("dbias", db)):
        assert o.normwise_rel_err(got, z[name]) < 1e-5, (path, name)


def _golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


@pytest.mark.skipif(not _golden_files(), reason="no golden fixtures captured yet")
def test_oracle_pinned_to_reference_goldens():
    """Pins the oracle to outputs of the reference shim (real cuBLAS / cuDNN on B200)."""
    checked = 0
    for path in _golden_files():
        z = np.load(path, allow_pickle=False)
        kind = str(z["kind"])
        if kind == "sgemm":
            ta, tb, m, n, k, lda, ldb, ldc = (int(v) for v in z["dims"])
            alpha, beta = (float(v) for v in z["scalars"])
            C = z["C_in"].copy()
            o.sgemm(ta, tb, m, n, k, alpha, z["A"], lda, z["B"], ldb, beta, C, ldc)
            got = C.reshape(n, ldc)[:, :m]
            ref = z["C_out"].reshape(n, ldc)[:, :m]
            assert o.normwise_rel_err(got, ref) < 1e-5, path
        elif kind == "sgemm_strided_batched":
            ta, tb, m, n, k, lda, ldb, ldc, sA, sB, sC, batch = (int(v) for v in z["dims"])
            alpha, beta = (float(v) for v in z["scalars"])
            C = z["C_in"].copy()
            o.sgemm_strided_batched(ta, tb, m, n, k, alpha, z["A"], lda, sA, z["B"], ldb, sB, beta,
                                    C, ldc, sC, batch)
            assert o.normwise_rel_err(C, z["C_out"]) < 1e-5, path
        elif kind == "gemm_ex_bf16":
            ta, tb, m, n, k, lda, ldb, ldc = (int(v) for v in z["dims"])
            D = np.zeros(m * n, np.float32)
            o.gemm_ex(ta, tb, m, n, k, 1.0, z["A"], o.R_16BF, lda, z["B"], o.R_16BF, ldb, 0.0,
                      None, o.R_32F, ldc, D=D, Dtype=o.R_32F, ldd=ldc)
            ref = o.bf16_bits_to_f32(z["C_out"])
            assert o.normwise_rel_err(D, ref) < 1e-2, path
        elif kind in ("conv_fwd", "conv_bwd_data", "conv_bwd_filter"):
            dims = [int(v) for v in z["dims"]]
            d = o.conv_desc(*dims[:7], pad=tuple(dims[7:9]), stride=tuple(dims[9:11]),
                            dil=tuple(dims[11:13]))
            if kind == "conv_fwd":
                got = o.conv_fwd(d, 1.0, z["x"], z["w"])
            elif kind == "conv_bwd_data":
                got = o.conv_bwd_data(d, 1.0, z["w"], z["dy"])
            else:
                got = o.conv_bwd_filter(d, 1.0, z["x"], z["dy"])
            assert o.normwise_rel_err(got, z["out"]) < 1e-5, path
        elif kind == "bn_spatial":
            _check_bn_golden(z, path)
        else:
            continue
        checked += 1
    assert checked > 0


def test_bn_spatial_persistent_mode_is_spatial():
    """cuDNN's SPATIAL_PERSISTENT mode (2) normalises per channel like
    SPATIAL (1): the oracle gives identical results and writes only C
    per-channel statistics."""
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((4, 6, 5, 7)) * 2 + 1).astype(np.float32)
    outs = []
    for mode in (1, 2):
        c = 6
        y = np.zeros_like(x)
        stats = [np.zeros(c + 8, np.float32) for _ in range(4)]  # 8 guard entries
        sc, b = np.linspace(0.5, 1.5, c).astype(np.float32), np.zeros(c, np.float32)
        o.bn_fwd_training(mode, 1.0, 0.0, x, y, sc, b, 0.1, stats[0], stats[1], 1e-5,
                          stats[2], stats[3])
        assert all(np.all(s[c:] == 0) for s in stats), mode
        outs.append((y, [s[:c] for s in stats]))
    assert np.array_equal(outs[0][0], outs[1][0])
    for a, b_ in zip(outs[0][1], outs[1][1]):
        assert np.array_equal(a, b_)
