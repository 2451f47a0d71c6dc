"""GPU parity at the shapes of the benchmark configurations.

The kx C ABI is called at full size; the CPU oracle (float64 accumulation)
checks a sample of the output, which is exact because every op here is
separable along the sampled axis:
* GEMM columns (tokens) are independent: the oracle computes sampled columns;
* convolution outputs are independent per image and per output channel
  (forward), per image and per input channel (backward data), and per
  (output, input) channel pair over the whole batch (backward filter).

Tolerances: fp32 ops <= 1e-5 max normwise relative error against float64
(3xTF32 on the tensor cores); bf16 ops <= 1e-2 against an fp32/float64-
accumulated product.  For the VGG16 convolutions cuDNN's own fp32 result
(TF32 off) is also measured against float64: kx must be within 1e-5 of
float64 and no further from it than cuDNN is plus 1e-5.  With KX_PARITY_LOG
set, each case appends its errors as one JSON line to that file.

Shapes: LLaMA projections and attention of the bf16 configuration (the
reference's python/LLaMA.py:78-98, 163-208 at hidden 2048, FFN 5504, 16
heads, batch 4 x 1024 tokens); the 13 VGG16 convolutions at batch 32
(python/VGG16.py, torchvision vgg16); batch norm at VGG-like shapes.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_BF16 = 1e-2


def _kx():
    from kernel_intercept_b200 import kx
    return kx


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _log(case, **errs):
    path = os.environ.get("KX_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": case, **{k: float(v) for k, v in errs.items()}}) + "\n")


def _bf16_dev(bits):
    import torch
    return _dev(bits.view(np.int16)).view(torch.bfloat16)


# ------------------------------------------------------------ bf16 GEMM ---

# nn.Linear y = x W^T in cuBLAS's column-major view: transa = T, transb = N,
# m = out_features, n = tokens (4 x 1024), k = in_features
LLAMA_LINEAR = [
    ("wq_wk_wv_wo", 2048, 4096, 2048),
    ("gate_up", 5504, 4096, 2048),
    ("down", 2048, 4096, 5504),
    ("lm_head", 32000, 4096, 2048),
]


def _gemm_bf16_sampled(ta, tb, m, n, k, cols, seed, scale_a=1.0, scale_b=1.0):
    kx = _kx()
    import torch
    rng = np.random.default_rng(seed)
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else n
    A = o.f32_to_bf16_bits(rng.standard_normal(lda * (k if ta == 0 else m),
                                               dtype=np.float32) * scale_a)
    B = o.f32_to_bf16_bits(rng.standard_normal(ldb * (n if tb == 0 else k),
                                               dtype=np.float32) * scale_b)
    dA, dB = _bf16_dev(A), _bf16_dev(B)
    dC = torch.empty(m * n, dtype=torch.bfloat16, device="cuda")
    kx.gemm_ex(kx.current_exec(), ta, tb, m, n, k, 1.0, dA.data_ptr(), kx.R_16BF, lda,
               dB.data_ptr(), kx.R_16BF, ldb, 0.0, dC.data_ptr(), kx.R_16BF, m)
    torch.cuda.synchronize()
    name = kx.last_kernel_name()
    got = dC.float().cpu().numpy().reshape(n, m)[cols]
    Bm = B.reshape(-1, ldb)
    if tb == 0:
        Bsub, ldb_sub = np.ascontiguousarray(Bm[cols]).reshape(-1), ldb
    else:
        Bsub, ldb_sub = np.ascontiguousarray(Bm[:, cols]).reshape(-1), len(cols)
    ref = np.zeros(m * len(cols), np.float32)
    o.gemm_ex(ta, tb, m, len(cols), k, 1.0, A, o.R_16BF, lda, Bsub, o.R_16BF, ldb_sub, 0.0,
              None, o.R_32F, m, D=ref, Dtype=o.R_32F, ldd=m)
    return o.normwise_rel_err(got, ref.reshape(len(cols), m)), name


@pytest.mark.parametrize("name,m,n,k", LLAMA_LINEAR)
def test_llama_linear_bf16(cuda, name, m, n, k):
    cols = np.sort(np.random.default_rng(m + k).choice(n, 64, replace=False))
    err, kernel = _gemm_bf16_sampled(1, 0, m, n, k, cols, seed=m * 3 + k, scale_b=0.5)
    _log(f"llama_{name}_{m}x{n}x{k}", kx_vs_oracle=err)
    assert kernel.startswith("kx_gemm_tc<"), kernel
    assert err <= TOL_BF16, err


# weight and input gradients of the same projections (the bf16 training
# clients): dW = dy^T x is NT in the column-major view, dx = dy W is NN
@pytest.mark.parametrize("ta,tb,m,n,k", [(0, 1, 2048, 2048, 4096), (0, 0, 2048, 4096, 5504),
                                         (0, 1, 512, 2048, 4096), (0, 0, 512, 4096, 2048)])
def test_linear_backward_bf16(cuda, ta, tb, m, n, k):
    cols = np.sort(np.random.default_rng(n + k).choice(n, 48, replace=False))
    err, kernel = _gemm_bf16_sampled(ta, tb, m, n, k, cols, seed=m + n + k)
    _log(f"linear_bwd_bf16_{'NT'[ta]}{'NT'[tb]}_{m}x{n}x{k}", kx_vs_oracle=err)
    assert err <= TOL_BF16, err


@pytest.mark.parametrize("which", ["scores", "context"])
def test_llama_attention_bf16(cuda, which):
    """Attention of 4 sequences x 16 heads (batch 64) at seq 1024, head 128:
    scores = q k^T (T x T, K = 128) and context = att v (128 x T, K = T)."""
    kx = _kx()
    import torch
    rng = np.random.default_rng(5 if which == "scores" else 6)
    batch, T, hd = 64, 1024, 128
    if which == "scores":  # column-major: S^T (T x T) = k (T x hd, k-major) . q^T
        ta, tb, m, n, k, lda, ldb = 1, 0, T, T, hd, hd, hd
        a_len, b_len = T * hd, T * hd
    else:                  # C^T (hd x T) = v^T (hd x T) . att^T (T x T)
        ta, tb, m, n, k, lda, ldb = 0, 0, hd, T, T, hd, T
        a_len, b_len = T * hd, T * T
    A = o.f32_to_bf16_bits(rng.standard_normal(batch * a_len, dtype=np.float32))
    B = o.f32_to_bf16_bits(rng.standard_normal(batch * b_len, dtype=np.float32) *
                           (1.0 if which == "scores" else 0.03))
    dA, dB = _bf16_dev(A), _bf16_dev(B)
    dC = torch.empty(batch * m * n, dtype=torch.bfloat16, device="cuda")
    kx.gemm_strided_batched_ex(kx.current_exec(), ta, tb, m, n, k, 1.0, dA.data_ptr(),
                               kx.R_16BF, lda, a_len, dB.data_ptr(), kx.R_16BF, ldb, b_len, 0.0,
                               dC.data_ptr(), kx.R_16BF, m, m * n, batch)
    torch.cuda.synchronize()
    got = dC.float().cpu().numpy()
    worst = 0.0
    for b in (0, 17, batch - 1):
        ref = np.zeros(m * n, np.float32)
        o.gemm_ex(ta, tb, m, n, k, 1.0, A[b * a_len:(b + 1) * a_len], o.R_16BF, lda,
                  B[b * b_len:(b + 1) * b_len], o.R_16BF, ldb, 0.0, None, o.R_32F, m, D=ref,
                  Dtype=o.R_32F, ldd=m)
        worst = max(worst, o.normwise_rel_err(got[b * m * n:(b + 1) * m * n], ref))
    _log(f"llama_attention_{which}", kx_vs_oracle=worst)
    assert worst <= TOL_BF16, worst


# ------------------------------------------------------ VGG16 convolutions ---

# (C, K, H=W) of the 13 convolutions, 3x3, pad 1, stride 1, batch 32
VGG16_CONVS = [(3, 64, 224), (64, 64, 224), (64, 128, 112), (128, 128, 112), (128, 256, 56),
               (256, 256, 56), (256, 256, 56), (256, 512, 28), (512, 512, 28), (512, 512, 28),
               (512, 512, 14), (512, 512, 14), (512, 512, 14)]


def _pick(count, total, rng):
    return np.sort(rng.choice(total, min(count, total), replace=False))


@pytest.mark.parametrize("layer", range(len(VGG16_CONVS)))
def test_vgg16_conv_b32(cuda, layer):
    """Forward, backward data and backward filter of one VGG16 layer at batch
    32 on kx; the oracle checks 2 images x 4 channels (forward, backward data)
    and 4 x 4 channel pairs over the whole batch (backward filter); cuDNN
    (TF32 off) on the same tensors is measured against the same oracle."""
    kx = _kx()
    import torch
    import torch.nn.functional as F
    torch.backends.cudnn.allow_tf32 = False
    C, K, HW = VGG16_CONVS[layer]
    N = 32
    rng = np.random.default_rng(1000 + layer)
    x = rng.standard_normal((N, C, HW, HW), dtype=np.float32)
    w = (rng.standard_normal((K, C, 3, 3), dtype=np.float32) *
         np.float32((2.0 / (C * 9)) ** 0.5))
    dy = rng.standard_normal((N, K, HW, HW), dtype=np.float32)
    kd = kx.ConvDesc(N, C, HW, HW, K, 3, 3, 1, 1, 1, 1, 1, 1, 1)
    dx_, dw_, ddy = _dev(x), _dev(w), _dev(dy)
    y = torch.empty(N, K, HW, HW, device="cuda")
    gx = torch.empty(N, C, HW, HW, device="cuda")
    gw = torch.empty(K, C, 3, 3, device="cuda")
    ex = kx.current_exec()
    kx.conv_fwd(ex, kd, 1.0, dx_.data_ptr(), dw_.data_ptr(), 0.0, y.data_ptr())
    kx.conv_bwd_data(ex, kd, 1.0, dw_.data_ptr(), ddy.data_ptr(), 0.0, gx.data_ptr())
    kx.conv_bwd_filter(ex, kd, 1.0, dx_.data_ptr(), ddy.data_ptr(), 0.0, gw.data_ptr())
    # cuDNN on the same device tensors
    lib_y = F.conv2d(dx_, dw_, padding=1)
    lib_gx = torch.nn.grad.conv2d_input(dx_.shape, dw_, ddy, padding=1)
    lib_gw = torch.nn.grad.conv2d_weight(dx_, dw_.shape, ddy, padding=1)
    torch.cuda.synchronize()
    ns, ks, cs = _pick(2, N, rng), _pick(4, K, rng), _pick(4, C, rng)
    ns[0], ns[-1] = 0, N - 1
    # forward: y[ns][:, ks]
    d = o.conv_desc(len(ns), C, HW, HW, len(ks), 3, 3, pad=(1, 1))
    ref = o.conv_fwd(d, 1.0, x[ns], w[ks])
    sl = (torch.as_tensor(ns).cuda()[:, None], torch.as_tensor(ks).cuda()[None, :])
    e_fwd = o.normwise_rel_err(y[sl].cpu().numpy(), ref)
    l_fwd = o.normwise_rel_err(lib_y[sl].cpu().numpy(), ref)
    # backward data: dx[ns][:, cs]
    d = o.conv_desc(len(ns), len(cs), HW, HW, K, 3, 3, pad=(1, 1))
    ref = o.conv_bwd_data(d, 1.0, np.ascontiguousarray(w[:, cs]), dy[ns])
    sl = (torch.as_tensor(ns).cuda()[:, None], torch.as_tensor(cs).cuda()[None, :])
    e_dgrad = o.normwise_rel_err(gx[sl].cpu().numpy(), ref)
    l_dgrad = o.normwise_rel_err(lib_gx[sl].cpu().numpy(), ref)
    # backward filter: dw[ks][:, cs] over the whole batch
    d = o.conv_desc(N, len(cs), HW, HW, len(ks), 3, 3, pad=(1, 1))
    ref = o.conv_bwd_filter(d, 1.0, np.ascontiguousarray(x[:, cs]),
                            np.ascontiguousarray(dy[:, ks]))
    sl = (torch.as_tensor(ks).cuda()[:, None], torch.as_tensor(cs).cuda()[None, :])
    e_wgrad = o.normwise_rel_err(gw[sl].cpu().numpy(), ref)
    l_wgrad = o.normwise_rel_err(lib_gw[sl].cpu().numpy(), ref)
    _log(f"vgg16_conv{layer}_b32", kx_fwd=e_fwd, cudnn_fwd=l_fwd, kx_dgrad=e_dgrad,
         cudnn_dgrad=l_dgrad, kx_wgrad=e_wgrad, cudnn_wgrad=l_wgrad)
    for kxe, libe, what in ((e_fwd, l_fwd, "fwd"), (e_dgrad, l_dgrad, "dgrad"),
                            (e_wgrad, l_wgrad, "wgrad")):
        assert kxe <= TOL_F32, (what, kxe, libe)
        assert kxe <= libe + TOL_F32, (what, kxe, libe)


# ------------------------------------------------------------- batch norm ---

def _bn_case(shape, seed, offset=0):
    """Spatial batch norm training forward + backward on kx vs the oracle.
    offset > 0 starts every device tensor that many floats into its buffer
    (4-byte aligned pointers that are not 16-byte aligned)."""
    kx = _kx()
    import torch
    n, c, h, w = shape
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(shape, dtype=np.float32) * 3 + 2).astype(np.float32)
    scale = (rng.random(c) + 0.5).astype(np.float32)
    bias = rng.standard_normal(c).astype(np.float32)
    rm = rng.standard_normal(c).astype(np.float32)
    rv = (rng.random(c) + 0.5).astype(np.float32)
    dy = rng.standard_normal(shape, dtype=np.float32)
    o_y, o_rm, o_rv = np.zeros(shape, np.float32), rm.copy(), rv.copy()
    o_sm, o_si = np.zeros(c, np.float32), np.zeros(c, np.float32)
    o.bn_fwd_training(1, 1.0, 0.0, x, o_y, scale, bias, 0.1, o_rm, o_rv, 1e-5, o_sm, o_si)
    o_dx = np.zeros(shape, np.float32)
    o_ds, o_db = np.zeros(c, np.float32), np.zeros(c, np.float32)
    o.bn_bwd(1, 1.0, 0.0, 1.0, 0.0, x, dy, o_dx, scale, o_ds, o_db, 1e-5, o_sm, o_si)

    def place(a):
        buf = torch.zeros(a.size + offset, device="cuda")
        t = buf[offset:]
        t.copy_(torch.from_numpy(np.ascontiguousarray(a).reshape(-1)))
        return t

    d = {k_: place(v) for k_, v in dict(x=x, y=np.zeros(shape, np.float32), scale=scale,
                                        bias=bias, rm=rm, rv=rv, sm=np.zeros(c, np.float32),
                                        si=np.zeros(c, np.float32), dy=dy,
                                        dx=np.zeros(shape, np.float32),
                                        ds=np.zeros(c, np.float32),
                                        db=np.zeros(c, np.float32)).items()}
    ex = kx.current_exec()
    kx.bn_fwd_training(ex, 1, 1.0, 0.0, n, c, h, w, d["x"].data_ptr(), d["y"].data_ptr(),
                       d["scale"].data_ptr(), d["bias"].data_ptr(), 0.1, d["rm"].data_ptr(),
                       d["rv"].data_ptr(), 1e-5, d["sm"].data_ptr(), d["si"].data_ptr())
    kx.bn_bwd(ex, 1, 1.0, 0.0, 1.0, 0.0, n, c, h, w, d["x"].data_ptr(), d["dy"].data_ptr(),
              d["dx"].data_ptr(), d["scale"].data_ptr(), d["ds"].data_ptr(),
              d["db"].data_ptr(), 1e-5, d["sm"].data_ptr(), d["si"].data_ptr())
    torch.cuda.synchronize()
    got = {k_: d[k_].cpu().numpy().reshape(v.shape) for k_, v in
           dict(y=o_y, rm=o_rm, rv=o_rv, sm=o_sm, si=o_si, dx=o_dx, ds=o_ds, db=o_db).items()}
    refs = dict(y=o_y, rm=o_rm, rv=o_rv, sm=o_sm, si=o_si, dx=o_dx, ds=o_ds, db=o_db)
    return {k_: o.normwise_rel_err(got[k_], refs[k_]) for k_ in refs}


@pytest.mark.parametrize("shape", [(64, 64, 56, 56), (64, 64, 14, 14), (64, 512, 56, 56),
                                   (64, 512, 14, 14)])
def test_batchnorm_vgg_shapes(cuda, shape):
    errs = _bn_case(shape, seed=sum(shape))
    _log("bn_%dx%dx%dx%d" % shape, **errs)
    for k_, e in errs.items():
        assert e <= TOL_F32, (k_, e)


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_batchnorm_unaligned_pointers(cuda, offset):
    """Tensors that start 4, 8 or 12 bytes past a 16-byte boundary (as views
    with a storage offset reach cuDNN) take the scalar path, with the same
    results."""
    errs = _bn_case((4, 8, 8, 8), seed=offset, offset=offset)
    for k_, e in errs.items():
        assert e <= TOL_F32, (k_, e)
