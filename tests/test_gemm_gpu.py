"""GPU parity of the kx GEMM entry points against the CPU oracle.

Every case calls the C ABI (libkx.so) on seeded inputs laid out exactly as the
cuBLAS call receives them (column-major, explicit leading dimensions) and
compares with the oracle's restatement of the same call.

Tolerances (from the parity contract):
* fp32 ops: max normwise relative error ||got - ref||_inf / ||ref||_inf <= 1e-5
  (3xTF32 on the tensor cores; never plain TF32 by default);
* bf16 ops: <= 1e-2 relative to an fp32/fp64-accumulated result.
"""
import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_BF16 = 1e-2


def _kx():
    from kernel_intercept_b200 import kx
    return kx


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _sgemm_case(ta, tb, m, n, k, pads=(0, 0, 0), alpha=1.0, beta=0.0, seed=0, mode=None,
                quota=0, col_subset=None):
    kx = _kx()
    import torch
    rng = np.random.default_rng(seed)
    lda = (m if ta == 0 else k) + pads[0]
    ldb = (k if tb == 0 else n) + pads[1]
    ldc = m + pads[2]
    A = rng.standard_normal(lda * (k if ta == 0 else m)).astype(np.float32)
    B = rng.standard_normal(ldb * (n if tb == 0 else k)).astype(np.float32)
    if beta != 0.0:
        C = rng.standard_normal(ldc * n).astype(np.float32)
    else:
        C = np.full(ldc * n, np.nan, np.float32)  # must never be read when beta == 0
    dA, dB, dC = _dev(A), _dev(B), _dev(C)
    ex = kx.current_exec(fp32_mode=kx.FP32_3XTF32 if mode is None else mode, sm_quota=quota)
    kx.sgemm(ex, ta, tb, m, n, k, alpha, dA.data_ptr(), lda, dB.data_ptr(), ldb, beta,
             dC.data_ptr(), ldc)
    torch.cuda.synchronize()
    got = dC.cpu().numpy().reshape(n, ldc)
    cols = np.arange(n) if col_subset is None else np.asarray(col_subset)
    # oracle on the selected columns only (a GEMM is column-separable)
    Bm = B.reshape(-1, ldb)
    if tb == 0:
        Bsub = np.ascontiguousarray(Bm[cols]).reshape(-1)
    else:
        Bsub = np.ascontiguousarray(Bm[:, cols]).reshape(-1)
        ldb_sub = len(cols)
    ref = np.ascontiguousarray(C.reshape(n, ldc)[cols]).reshape(-1).copy()
    o.sgemm(ta, tb, m, len(cols), k, alpha, A, lda, Bsub, ldb if tb == 0 else ldb_sub, beta, ref,
            ldc)
    ref = ref.reshape(len(cols), ldc)
    err = o.normwise_rel_err(got[cols, :m], ref[:, :m])
    # rows beyond m (padding) must be untouched
    assert np.array_equal(got[:, m:], C.reshape(n, ldc)[:, m:], equal_nan=True)
    return err


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 300, 100), (1, 1, 1), (130, 70, 33),
                                   (257, 129, 300), (64, 2048, 512)])
def test_sgemm_parity(cuda, ta, tb, m, n, k):
    err = _sgemm_case(ta, tb, m, n, k)
    assert err <= TOL_F32, err


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1)])
def test_sgemm_padded_ld_alpha_beta(cuda, ta, tb):
    err = _sgemm_case(ta, tb, 190, 170, 150, pads=(4, 8, 12), alpha=1.5, beta=-0.5, seed=3)
    assert err <= TOL_F32, err


def test_sgemm_unaligned_ld_uses_cuda_cores(cuda):
    # lda*4 bytes not a multiple of 16: not TMA-addressable, served by the SIMT kernel
    err = _sgemm_case(0, 0, 67, 45, 23, pads=(2, 1, 3), alpha=0.75, beta=0.25, seed=5)
    assert err <= TOL_F32, err
    assert _kx().last_kernel_name() == "kx_gemm_simt"


@pytest.mark.parametrize("m,n,k", [(512, 2048, 512), (2048, 2048, 512), (512, 2048, 2048)])
def test_sgemm_gpt_shapes(cuda, m, n, k):
    # y = x W^T of the GPT blocks: transa = T, transb = N (cuBLAS view of nn.Linear)
    err = _sgemm_case(1, 0, m, n, k, seed=m + n + k)
    assert err <= TOL_F32, err
    assert _kx().last_kernel_name().startswith("kx_gemm_tc<")


@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 0), (0, 1), (1, 1)])
def test_sgemm_long_k_accuracy(cuda, ta, tb):
    # the tensor core's fp32 accumulation is not round-to-nearest; segment
    # promotion keeps long reductions (VGG FC: K = 25088) within 1e-5
    err = _sgemm_case(ta, tb, 256, 128, 8192, seed=17)
    assert err <= TOL_F32, err


def test_sgemm_vgg_fc(cuda):
    # VGG16 fc6 at batch 32: m = 4096 outputs, n = 32 images, k = 25088
    err = _sgemm_case(1, 0, 4096, 32, 25088, seed=19)
    assert err <= TOL_F32, err


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k,alpha,beta,pads", [
    (512, 64, 4096, 1.0, 0.0, (0, 0, 0)),      # GPT per-head weight gradient: split-K
    (100, 50, 3000, 0.75, 0.5, (3, 5, 7)),     # ragged K and tiles, padded ld, beta
    (27, 64, 20000, 1.0, 1.0, (0, 0, 0)),      # first-layer conv weight gradient shape
])
def test_sgemm_split_k(cuda, ta, tb, m, n, k, alpha, beta, pads):
    # few output tiles, long K: partials of K slices are reduced in a second kernel
    err = _sgemm_case(ta, tb, m, n, k, pads=pads, alpha=alpha, beta=beta, seed=m + n)
    assert err <= TOL_F32, err


def test_split_k_epilogue_and_batch(cuda):
    """Split-K with the Lt bias+GELU epilogue, and a strided batch whose
    per-matrix tile count is small."""
    kx = _kx()
    import torch
    rng = np.random.default_rng(31)
    m, n, k = 256, 48, 6144
    A = rng.standard_normal(k * m).astype(np.float32)
    B = rng.standard_normal(k * n).astype(np.float32)
    bias = rng.standard_normal(m).astype(np.float32)
    ref = np.zeros(m * n, np.float32)
    o.gemm_ex(1, 0, m, n, k, 0.5, A, o.R_32F, k, B, o.R_32F, k, 0.0, None, o.R_32F, m, D=ref,
              Dtype=o.R_32F, ldd=m, epilogue=36, bias=bias)
    dA, dB, db = _dev(A), _dev(B), _dev(bias)
    dD = torch.zeros(m * n, device="cuda")
    kx.matmul(kx.current_exec(), 1, 0, m, n, k, 0.5, dA.data_ptr(), kx.R_32F, k, 0,
              dB.data_ptr(), kx.R_32F, k, 0, 0.0, None, kx.R_32F, m, 0, dD.data_ptr(), kx.R_32F,
              m, 0, 1, 36, db.data_ptr(), kx.R_32F)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(dD.cpu().numpy(), ref) <= TOL_F32

    batch, m, n, k = 3, 96, 80, 2048
    sA, sB, sC = m * k, k * n, m * n
    A = rng.standard_normal(sA * batch).astype(np.float32)
    B = rng.standard_normal(sB * batch).astype(np.float32)
    C = rng.standard_normal(sC * batch).astype(np.float32)
    ref = C.copy()
    o.sgemm_strided_batched(0, 0, m, n, k, 1.0, A, m, sA, B, k, sB, -1.0, ref, m, sC, batch)
    dA, dB, dC = _dev(A), _dev(B), _dev(C)
    kx.sgemm_strided_batched(kx.current_exec(), 0, 0, m, n, k, 1.0, dA.data_ptr(), m, sA,
                             dB.data_ptr(), k, sB, -1.0, dC.data_ptr(), m, sC, batch)
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    for b in range(batch):
        seg = slice(b * sC, (b + 1) * sC)
        assert o.normwise_rel_err(got[seg], ref[seg]) <= TOL_F32, b


def test_sgemm_lm_head(cuda):
    # vocab 32000 x tokens 2048 x emb 512; oracle on 48 sampled token columns
    cols = np.random.default_rng(1).choice(2048, 48, replace=False)
    err = _sgemm_case(1, 0, 32000, 2048, 512, seed=11, col_subset=np.sort(cols))
    assert err <= TOL_F32, err


def test_sgemm_k_zero_and_alpha_zero(cuda):
    # cuBLAS requires ldb >= max(1, k): pad ldb to 1 for k == 0
    assert _sgemm_case(0, 0, 100, 50, 0, pads=(0, 1, 0), alpha=1.0, beta=0.5, seed=2) <= TOL_F32
    assert _sgemm_case(1, 0, 100, 50, 20, alpha=0.0, beta=2.0, seed=2) <= TOL_F32


def test_sgemm_modes(cuda):
    kx = _kx()
    assert _sgemm_case(1, 0, 256, 256, 256, mode=kx.FP32_FFMA, seed=7) <= TOL_F32
    # plain TF32 is what cuBLAS does under TF32 math mode: ~1e-3, far from fp32
    e = _sgemm_case(1, 0, 256, 256, 256, mode=kx.FP32_TF32, seed=7)
    assert 1e-5 < e < 5e-3, e


def test_sgemm_quota(cuda):
    assert _sgemm_case(1, 0, 1024, 1024, 256, quota=8, seed=9) <= TOL_F32


def test_sgemm_strided_batched(cuda):
    kx = _kx()
    import torch
    rng = np.random.default_rng(4)
    batch, m, n, k = 8, 256, 256, 64
    for ta, tb in [(1, 0), (0, 0), (0, 1)]:
        lda = m if ta == 0 else k
        ldb = k if tb == 0 else n
        sA, sB, sC = lda * (k if ta == 0 else m) + 16, ldb * (n if tb == 0 else k) + 32, m * n + 8
        A = rng.standard_normal(sA * batch).astype(np.float32)
        B = rng.standard_normal(sB * batch).astype(np.float32)
        C = rng.standard_normal(sC * batch).astype(np.float32)
        ref = C.copy()
        o.sgemm_strided_batched(ta, tb, m, n, k, 0.125, A, lda, sA, B, ldb, sB, 1.0, ref, m, sC,
                                batch)
        dA, dB, dC = _dev(A), _dev(B), _dev(C)
        kx.sgemm_strided_batched(kx.current_exec(), ta, tb, m, n, k, 0.125, dA.data_ptr(), lda, sA,
                                 dB.data_ptr(), ldb, sB, 1.0, dC.data_ptr(), m, sC, batch)
        torch.cuda.synchronize()
        got = dC.cpu().numpy()
        for b in range(batch):
            seg = slice(b * sC, b * sC + m * n)
            err = o.normwise_rel_err(got[seg], ref[seg])
            assert err <= TOL_F32, (ta, tb, b, err)


def test_sgemm_batched_pointer_arrays(cuda):
    kx = _kx()
    import torch
    rng = np.random.default_rng(8)
    batch, m, n, k = 3, 70, 50, 40
    As = [_dev(rng.standard_normal(m * k).astype(np.float32)) for _ in range(batch)]
    Bs = [_dev(rng.standard_normal(k * n).astype(np.float32)) for _ in range(batch)]
    Cs = [_dev(np.zeros(m * n, np.float32)) for _ in range(batch)]
    pa = torch.tensor([t.data_ptr() for t in As], dtype=torch.int64, device="cuda")
    pb = torch.tensor([t.data_ptr() for t in Bs], dtype=torch.int64, device="cuda")
    pc = torch.tensor([t.data_ptr() for t in Cs], dtype=torch.int64, device="cuda")
    kx.sgemm_batched(kx.current_exec(), 0, 0, m, n, k, 1.0, pa.data_ptr(), m, pb.data_ptr(), k,
                     0.0, pc.data_ptr(), m, batch)
    torch.cuda.synchronize()
    for b in range(batch):
        ref = np.zeros(m * n, np.float32)
        o.sgemm(0, 0, m, n, k, 1.0, As[b].cpu().numpy(), m, Bs[b].cpu().numpy(), k, 0.0, ref, m)
        assert o.normwise_rel_err(Cs[b].cpu().numpy(), ref) <= TOL_F32


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(512, 384, 256), (300, 200, 72), (2048, 1024, 2048)])
def test_gemm_ex_bf16(cuda, ta, tb, m, n, k):
    kx = _kx()
    import torch
    rng = np.random.default_rng(m * 7 + n + k + ta * 2 + tb)
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else n
    A = o.f32_to_bf16_bits(rng.standard_normal(lda * (k if ta == 0 else m)).astype(np.float32))
    B = o.f32_to_bf16_bits(rng.standard_normal(ldb * (n if tb == 0 else k)).astype(np.float32))
    C = np.zeros(m * n, np.uint16)
    ref = np.zeros(m * n, np.float32)
    o.gemm_ex(ta, tb, m, n, k, 1.0, A, o.R_16BF, lda, B, o.R_16BF, ldb, 0.0, None, o.R_32F, m,
              D=ref, Dtype=o.R_32F, ldd=m)
    dA = _dev(A.view(np.int16)).view(torch.bfloat16)
    dB = _dev(B.view(np.int16)).view(torch.bfloat16)
    dC = _dev(C.view(np.int16)).view(torch.bfloat16)
    kx.gemm_ex(kx.current_exec(), ta, tb, m, n, k, 1.0, dA.data_ptr(), kx.R_16BF, lda,
               dB.data_ptr(), kx.R_16BF, ldb, 0.0, dC.data_ptr(), kx.R_16BF, m)
    torch.cuda.synchronize()
    got = dC.float().cpu().numpy()
    assert o.normwise_rel_err(got, ref) <= TOL_BF16
    if (lda * 2) % 16 == 0 and (ldb * 2) % 16 == 0:  # TMA-addressable
        assert _kx().last_kernel_name().startswith("kx_gemm_tc<")


@pytest.mark.parametrize("m,n,k", [(512, 384, 256), (300, 200, 72), (2048, 1024, 2048),
                                   (2048, 4096, 512), (1000, 520, 136)])
def test_gemm_ex_bf16_cta_pair(cuda, m, n, k, monkeypatch):
    """16-bit GEMM with K-major A and B on 2-CTA clusters (KX_GEMM_PAIR=1):
    256-row tiles of cta_group::2 MMAs, each CTA loading half of the B tile;
    odd numbers of 128-row blocks leave the second half of the last pair
    tile past the end of M."""
    monkeypatch.setenv("KX_GEMM_PAIR", "1")
    test_gemm_ex_bf16(cuda, 1, 0, m, n, k)
    assert ",pair" in _kx().last_kernel_name(), _kx().last_kernel_name()


@pytest.mark.parametrize("pair", ["0", "1"])
def test_gemm_strided_batched_ex_bf16_attention(cuda, pair, monkeypatch):
    # LLaMA attention scores: batch 64, 1024 x 1024 x 128 (q k^T), bf16; one
    # CTA per tile or 2-CTA clusters
    monkeypatch.setenv("KX_GEMM_PAIR", pair)
    kx = _kx()
    import torch
    rng = np.random.default_rng(21)
    batch, m, n, k = 4, 1024, 1024, 128
    A = o.f32_to_bf16_bits(rng.standard_normal(batch * k * m).astype(np.float32))
    B = o.f32_to_bf16_bits(rng.standard_normal(batch * k * n).astype(np.float32))
    dA = _dev(A.view(np.int16)).view(torch.bfloat16)
    dB = _dev(B.view(np.int16)).view(torch.bfloat16)
    dC = torch.zeros(batch * m * n, dtype=torch.bfloat16, device="cuda")
    kx.gemm_strided_batched_ex(kx.current_exec(), 1, 0, m, n, k, 1.0, dA.data_ptr(), kx.R_16BF,
                               k, k * m, dB.data_ptr(), kx.R_16BF, k, k * n, 0.0, dC.data_ptr(),
                               kx.R_16BF, m, m * n, batch)
    torch.cuda.synchronize()
    got = dC.float().cpu().numpy()
    for b in (0, batch - 1):
        ref = np.zeros(m * n, np.float32)
        o.gemm_ex(1, 0, m, n, k, 1.0, A[b * k * m:(b + 1) * k * m], o.R_16BF, k,
                  B[b * k * n:(b + 1) * k * n], o.R_16BF, k, 0.0, None, o.R_32F, m, D=ref,
                  Dtype=o.R_32F, ldd=m)
        assert o.normwise_rel_err(got[b * m * n:(b + 1) * m * n], ref) <= TOL_BF16


@pytest.mark.parametrize("epi", [1, 4, 6, 36])
def test_matmul_epilogues_fp32(cuda, epi):
    # cublasLtMatmul as PyTorch issues it for nn.Linear with bias (addmm)
    kx = _kx()
    import torch
    rng = np.random.default_rng(epi)
    m, n, k = 384, 256, 200
    A = rng.standard_normal(k * m).astype(np.float32)      # transa = T, lda = k
    B = rng.standard_normal(k * n).astype(np.float32)      # transb = N, ldb = k
    bias = rng.standard_normal(m).astype(np.float32)
    D = np.zeros(m * n, np.float32)
    ref = np.zeros(m * n, np.float32)
    o.gemm_ex(1, 0, m, n, k, 1.0, A, o.R_32F, k, B, o.R_32F, k, 0.0, None, o.R_32F, m, D=ref,
              Dtype=o.R_32F, ldd=m, epilogue=epi, bias=bias)
    dA, dB, dD, db = _dev(A), _dev(B), _dev(D), _dev(bias)
    kx.matmul(kx.current_exec(), 1, 0, m, n, k, 1.0, dA.data_ptr(), kx.R_32F, k, 0,
              dB.data_ptr(), kx.R_32F, k, 0, 0.0, None, kx.R_32F, m, 0, dD.data_ptr(), kx.R_32F,
              m, 0, 1, epi, db.data_ptr(), kx.R_32F)
    torch.cuda.synchronize()
    assert o.normwise_rel_err(dD.cpu().numpy(), ref) <= TOL_F32


def _bf16_matmul_case(m, n, k, epi=1, beta=0.0, batch=1, quota=0, seed=0, ta=1, tb=0):
    """cublasLtMatmul with bf16 A, B, C, D (fp32 accumulation), an optional
    bias / activation epilogue and beta, as PyTorch issues it for a bf16
    nn.Linear; returns the normwise error against the oracle and the kernel
    name."""
    kx = _kx()
    import torch
    rng = np.random.default_rng(seed)
    lda = m if ta == 0 else k
    ldb = k if tb == 0 else n
    sA, sB, sD = lda * (k if ta == 0 else m), ldb * (n if tb == 0 else k), m * n
    A = o.f32_to_bf16_bits(rng.standard_normal(sA * batch).astype(np.float32))
    B = o.f32_to_bf16_bits(rng.standard_normal(sB * batch).astype(np.float32))
    C = o.f32_to_bf16_bits(rng.standard_normal(sD * batch).astype(np.float32))
    bias = o.f32_to_bf16_bits(rng.standard_normal(m).astype(np.float32))
    ref = np.zeros(sD * batch, np.float32)
    o.gemm_ex(ta, tb, m, n, k, 1.0, A, o.R_16BF, lda, B, o.R_16BF, ldb, beta, C, o.R_16BF, m,
              D=ref, Dtype=o.R_32F, ldd=m, batch=batch, sA=sA, sB=sB, sC=sD, sD=sD,
              epilogue=epi, bias=bias, bias_type=o.R_16BF)
    bf = torch.bfloat16
    dA = _dev(A.view(np.int16)).view(bf)
    dB = _dev(B.view(np.int16)).view(bf)
    dC = _dev(C.view(np.int16)).view(bf)
    dbias = _dev(bias.view(np.int16)).view(bf)
    dD = torch.full((sD * batch,), float("nan"), dtype=bf, device="cuda")
    kx.matmul(kx.current_exec(sm_quota=quota), ta, tb, m, n, k, 1.0, dA.data_ptr(), kx.R_16BF,
              lda, sA, dB.data_ptr(), kx.R_16BF, ldb, sB, beta, dC.data_ptr(), kx.R_16BF, m, sD,
              dD.data_ptr(), kx.R_16BF, m, sD, batch, epi, dbias.data_ptr(), kx.R_16BF)
    torch.cuda.synchronize()
    got = dD.float().cpu().numpy()
    return o.normwise_rel_err(got, ref), _kx().last_kernel_name()


@pytest.mark.parametrize("epi,beta", [(1, 0.0), (1, 0.5), (4, 0.0), (6, 0.0), (36, 0.0)])
def test_matmul_epilogues_bf16_wide_tiles(cuda, epi, beta, monkeypatch):
    """bf16 Lt matmuls on 256-wide tiles: the plain epilogue stores 64-column
    boxes, every other (beta, bias, ReLU, GELU) 32-column ones."""
    monkeypatch.setenv("KX_GEMM_BN", "256")
    err, name = _bf16_matmul_case(384, 640, 200, epi=epi, beta=beta, seed=epi)
    assert name.startswith("kx_gemm_tc<bn256,bf16"), name
    assert err <= TOL_BF16, err


@pytest.mark.parametrize("arith", ["f32", "bf16_pair"])
def test_yield_and_continuation(cuda, arith, monkeypatch):
    """A BE launch that stops at tile boundaries resumes exactly where it left
    off: 3xTF32 on single CTAs, and bf16 on 2-CTA clusters (the leader takes
    the tiles and the follower follows its stops)."""
    kx = _kx()
    import torch
    rng = np.random.default_rng(31)
    m, n, k = 512, 1024, 256
    A = rng.standard_normal(k * m).astype(np.float32)
    B = rng.standard_normal(k * n).astype(np.float32)
    ref = np.zeros(m * n, np.float32)
    if arith == "f32":
        o.sgemm(1, 0, m, n, k, 1.0, A, k, B, k, 0.0, ref, m)
        dA, dB = _dev(A), _dev(B)
        dC = torch.zeros(m * n, device="cuda")
        tol = TOL_F32

        def op(ex):
            kx.sgemm(ex, 1, 0, m, n, k, 1.0, dA.data_ptr(), k, dB.data_ptr(), k, 0.0,
                     dC.data_ptr(), m)
    else:
        monkeypatch.setenv("KX_GEMM_PAIR", "1")
        A16, B16 = o.f32_to_bf16_bits(A), o.f32_to_bf16_bits(B)
        o.gemm_ex(1, 0, m, n, k, 1.0, A16, o.R_16BF, k, B16, o.R_16BF, k, 0.0, None, o.R_32F,
                  m, D=ref, Dtype=o.R_32F, ldd=m)
        dA = _dev(A16.view(np.int16)).view(torch.bfloat16)
        dB = _dev(B16.view(np.int16)).view(torch.bfloat16)
        dC = torch.zeros(m * n, device="cuda")
        tol = TOL_BF16

        def op(ex):
            kx.gemm_ex(ex, 1, 0, m, n, k, 1.0, dA.data_ptr(), kx.R_16BF, k, dB.data_ptr(),
                       kx.R_16BF, k, 0.0, dC.data_ptr(), kx.R_32F, m)
    flags = kx.HostFlags(2)  # [0] = yield flag, [1] = done flag
    stream = torch.cuda.Stream()
    try:
        # 1) flag < 0 before launch: no CTA takes a tile, op reports "not done"
        flags[0] = -1
        flags[1] = -1
        op(kx.make_exec(stream=stream, sm_quota=4, yield_flag=flags.dev(0),
                        done_flag=flags.dev(1)))
        stream.synchronize()
        assert flags[1] == 0
        assert float(dC.abs().max()) == 0.0
        if arith != "f32":
            assert ",pair>" in kx.last_kernel_name(), kx.last_kernel_name()
        # 2) flag lowered; per-launch budget of one tile per CTA forces many relaunches
        flags[0] = 0
        ex = kx.make_exec(stream=stream, sm_quota=4, yield_flag=flags.dev(0),
                          done_flag=flags.dev(1), max_tiles=1)
        launches = 0
        while True:
            flags[1] = -1
            op(ex)
            stream.synchronize()
            launches += 1
            if flags[1] == 1:
                break
            assert flags[1] == 0 and launches < 1000
        assert launches > 2
        assert o.normwise_rel_err(dC.cpu().numpy(), ref) <= tol
        # 3) flag > 0: CTAs at or above the budget retire, the rest finish the op
        dC.zero_()
        flags[0] = 2
        flags[1] = -1
        op(kx.make_exec(stream=stream, sm_quota=16, yield_flag=flags.dev(0),
                        done_flag=flags.dev(1)))
        stream.synchronize()
        assert flags[1] == 1
        assert o.normwise_rel_err(dC.cpu().numpy(), ref) <= tol
        flags[0] = 0
        # 4) the slot was reset: a plain follow-up op on the same stream is complete
        dC.zero_()
        flags[1] = -1
        op(kx.make_exec(stream=stream, done_flag=flags.dev(1)))
        stream.synchronize()
        assert flags[1] == 1
        assert o.normwise_rel_err(dC.cpu().numpy(), ref) <= tol
    finally:
        flags.close()


def test_invalid_arguments(cuda):
    kx = _kx()
    import torch
    buf = torch.zeros(64, device="cuda")
    p = buf.data_ptr()
    assert kx.sgemm(None, 0, 0, -1, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4, check=False) == kx.ERR_INVALID
    assert kx.sgemm(None, 0, 0, 8, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 8, check=False) == kx.ERR_INVALID
    assert kx.sgemm(None, 5, 0, 4, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4, check=False) == kx.ERR_INVALID
    assert kx.sgemm(None, 0, 0, 0, 4, 4, 1.0, p, 4, p, 4, 0.0, p, 4, check=False) == kx.OK


def test_bounded_wait_gives_up(cuda):
    """The device-side bounded wait returns KX_ERR_TIMEOUT when nothing sets the flag."""
    kx = _kx()
    import torch
    flags = kx.HostFlags(1)
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    try:
        s = torch.cuda.current_stream().cuda_stream
        kx.wait_flag(s, flags.dev(0), 50_000_000, status.data_ptr())
        torch.cuda.synchronize()
        assert int(status.item()) == kx.ERR_TIMEOUT
        flags[0] = 1
        kx.wait_flag(s, flags.dev(0), 50_000_000, status.data_ptr())
        torch.cuda.synchronize()
        assert int(status.item()) == kx.OK
    finally:
        flags.close()
