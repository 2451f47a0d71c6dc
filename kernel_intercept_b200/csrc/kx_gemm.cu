// kx_gemm.cu — GEMM entry points of the kx C ABI (cuBLAS column-major
// semantics) and the CUDA-core fallback kernel.
//
// Dispatch: fp32 operands go to the tcgen05 kernel in 3xTF32 (default),
// 1xTF32 or CUDA-core FFMA mode (kx_exec.fp32_mode); bf16 / fp16 operands go
// to the tcgen05 kind::f16 kernel.  The CUDA-core kernel serves what TMA
// cannot address (unaligned pointers or leading dimensions, pointer-array
// batches, mixed operand types, k == 0 / alpha == 0 scaling) — it is part of
// the product, not a CPU fallback: no entry point ever computes on the host.
#include <cstdlib>
#include <cstring>

#include "kx_gemm_launch.cuh"

namespace kx {

struct SimtGemmParams {
  int transa, transb, m, n, k;
  const void* A;
  int a_type;
  long long lda, strideA;
  const void* B;
  int b_type;
  long long ldb, strideB;
  const void* const* Aarr;  // pointer-array batch (nullable)
  const void* const* Barr;
  void* const* Darr;
  float alpha, beta;
  const float* alpha_dev;
  const float* beta_dev;
  void* D;
  int d_type;
  long long ldd, strideD;
  const void* C;
  int c_type;
  long long ldc, strideC;
  int relu, gelu;
  const void* bias;
  int bias_type;
  volatile int* done_flag;
};

// 64x64 output tile per block, 256 threads each owning a 4x4 register tile.
// Thread (tx, ty) owns rows i0 + tx + 16r and columns j0 + ty + 16c, so warp
// stores along the contiguous (row) dimension of column-major D coalesce.
__global__ void __launch_bounds__(256) kx_gemm_simt_kernel(const SimtGemmParams p) {
  __shared__ float As[16][65];
  __shared__ float Bs[16][65];
  const int b = blockIdx.z;
  const int i0 = blockIdx.x * 64, j0 = blockIdx.y * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const void* A = p.Aarr ? p.Aarr[b] : static_cast<const char*>(p.A) + (size_t)b * p.strideA * (p.a_type == DT_F32 ? 4 : 2);
  const void* B = p.Barr ? p.Barr[b] : static_cast<const char*>(p.B) + (size_t)b * p.strideB * (p.b_type == DT_F32 ? 4 : 2);
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;

  for (int k0 = 0; k0 < p.k; k0 += 16) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = threadIdx.x + e * 256;
      const int ii = idx & 63, pp = idx >> 6;
      const int i = i0 + ii, kk = k0 + pp;
      float av = 0.f;
      if (i < p.m && kk < p.k) {
        size_t off = p.transa == 0 ? (size_t)i + (size_t)kk * p.lda : (size_t)kk + (size_t)i * p.lda;
        av = load_scalar(A, p.a_type, off);
      }
      As[pp][ii] = av;
      const int j = j0 + ii;
      float bv = 0.f;
      if (j < p.n && kk < p.k) {
        size_t off = p.transb == 0 ? (size_t)kk + (size_t)j * p.ldb : (size_t)j + (size_t)kk * p.ldb;
        bv = load_scalar(B, p.b_type, off);
      }
      Bs[pp][ii] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int pp = 0; pp < 16; ++pp) {
      float a[4], bb[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r] = As[pp][tx + 16 * r];
#pragma unroll
      for (int c = 0; c < 4; ++c) bb[c] = Bs[pp][ty + 16 * c];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r], bb[c], acc[r][c]);
    }
    __syncthreads();
  }
  const float alpha = p.alpha_dev ? *p.alpha_dev : p.alpha;
  const float beta = p.beta_dev ? *p.beta_dev : p.beta;
  void* D = p.Darr ? p.Darr[b] : static_cast<char*>(p.D) + (size_t)b * p.strideD * (p.d_type == DT_F32 ? 4 : 2);
  const void* C = p.Darr ? static_cast<const void*>(p.Darr[b])
                         : static_cast<const char*>(p.C) + (size_t)b * p.strideC * (p.c_type == DT_F32 ? 4 : 2);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = i0 + tx + 16 * r;
    if (i >= p.m) continue;
    const float bias_v = p.bias ? load_scalar(p.bias, p.bias_type, i) : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = j0 + ty + 16 * c;
      if (j >= p.n) continue;
      float o = alpha * acc[r][c];
      if (beta != 0.f) o += beta * load_scalar(C, p.c_type, (size_t)i + (size_t)j * p.ldc);
      o += bias_v;
      if (p.relu) o = fmaxf(o, 0.f);
      if (p.gelu) o = gelu_tanh(o);
      store_scalar(D, p.d_type, (size_t)i + (size_t)j * p.ldd, o);
    }
  }
  if (p.done_flag != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 &&
      threadIdx.x == 0) {
    *p.done_flag = 1;
    __threadfence_system();
  }
}

// lo[i] = src[i] - trunc_tf32(src[i]) over two spans (the 3xTF32 low parts
// of both GEMM operands in one launch).
__global__ void __launch_bounds__(256) tf32_split_lo(const float* __restrict__ a, float* __restrict__ alo,
                                                     size_t na, const float* __restrict__ b,
                                                     float* __restrict__ blo, size_t nb) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t t0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  // both spans start 16-byte aligned (TMA-addressable operands)
  const size_t na4 = na / 4, nb4 = nb / 4;
  for (size_t i = t0; i < na4 + nb4; i += stride) {
    const bool in_a = i < na4;
    const float4 x = in_a ? reinterpret_cast<const float4*>(a)[i]
                          : reinterpret_cast<const float4*>(b)[i - na4];
    const float4 l = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
    if (in_a)
      reinterpret_cast<float4*>(alo)[i] = l;
    else
      reinterpret_cast<float4*>(blo)[i - na4] = l;
  }
  if (t0 < na - na4 * 4) alo[na4 * 4 + t0] = tf32_lo(a[na4 * 4 + t0]);
  if (t0 < nb - nb4 * 4) blo[nb4 * 4 + t0] = tf32_lo(b[nb4 * 4 + t0]);
}

namespace {

// KX_PRESPLIT=0 keeps the 3xTF32 split inside the GEMM kernel.
bool presplit_disabled() {
  static const bool off = [] {
    const char* s = std::getenv("KX_PRESPLIT");
    return s != nullptr && s[0] == '0';
  }();
  return off;
}

// Elements from the first to the last one a (possibly batched, padded)
// column-major operand touches.
size_t operand_span(long long rows, long long cols, long long ld, long long stride, int batch) {
  long long span = (cols - 1) * ld + rows;
  if (batch > 1 && stride > 0) span += (batch - 1) * stride;
  return span > 0 ? static_cast<size_t>(span) : 0;
}

struct GemmCall {
  int transa, transb, m, n, k, batch;
  const float* alpha;
  const float* beta;
  const void* A;
  int a_type;
  long long lda, strideA;
  const void* B;
  int b_type;
  long long ldb, strideB;
  const void* C;
  int c_type;
  long long ldc, strideC;
  void* D;
  int d_type;
  long long ldd, strideD;
  int epilogue;
  const void* bias;
  int bias_type;
  const void* const* Aarr = nullptr;
  const void* const* Barr = nullptr;
  void* const* Darr = nullptr;
};

bool valid_type(int t) { return t == DT_F32 || t == DT_BF16 || t == DT_F16; }
int esize(int t) { return t == DT_F32 ? 4 : 2; }

int launch_simt(const Exec& e, const GemmCall& g, bool dev_scalars) {
  SimtGemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.transa = g.transa;
  p.transb = g.transb;
  p.m = g.m;
  p.n = g.n;
  p.k = g.k;
  p.A = g.A;
  p.a_type = g.a_type;
  p.lda = g.lda;
  p.strideA = g.strideA;
  p.B = g.B;
  p.b_type = g.b_type;
  p.ldb = g.ldb;
  p.strideB = g.strideB;
  p.Aarr = g.Aarr;
  p.Barr = g.Barr;
  p.Darr = g.Darr;
  if (dev_scalars) {
    p.alpha_dev = g.alpha;
    p.beta_dev = g.beta;
  } else {
    p.alpha = *g.alpha;
    p.beta = *g.beta;
  }
  p.D = g.D;
  p.d_type = g.d_type;
  p.ldd = g.ldd;
  p.strideD = g.strideD;
  p.C = g.C;
  p.c_type = g.c_type;
  p.ldc = g.ldc;
  p.strideC = g.strideC;
  p.relu = (g.epilogue == KX_EPI_RELU || g.epilogue == KX_EPI_RELU_BIAS);
  p.gelu = (g.epilogue == KX_EPI_GELU || g.epilogue == KX_EPI_GELU_BIAS);
  const bool has_bias = (g.epilogue == KX_EPI_BIAS || g.epilogue == KX_EPI_RELU_BIAS ||
                         g.epilogue == KX_EPI_GELU_BIAS);
  p.bias = has_bias ? g.bias : nullptr;
  p.bias_type = g.bias_type;
  p.done_flag = e.done_flag;
  dim3 grid((g.m + 63) / 64, (g.n + 63) / 64, g.batch);
  if (grid.y > 65535 || grid.z > 65535) return KX_ERR_UNSUPPORTED;
  note_launch();
  kx_gemm_simt_kernel<<<grid, 256, 0, e.stream>>>(p);
  set_last_kernel_name("kx_gemm_simt");
  return launch_status();
}

bool tma_ok(const void* ptr, long long ld, long long stride, int batch, int es) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return false;
  if ((ld * es) % 16 != 0) return false;
  if (batch > 1 && stride != 0 && (stride * es) % 16 != 0) return false;
  return true;
}

// Widest N tile that still gives every SM a tile; 3xTF32 tiles stop at 128
// (the epilogue keeps a BN-wide fp32 accumulator per thread).
int choose_bn(int m, int n, int batch, int sms, int max_bn) {
  if (const char* f = std::getenv("KX_GEMM_BN")) {
    int v = std::atoi(f);
    if ((v == 64 || v == 128 || v == 256) && v <= max_bn) return v;
  }
  const long long mb = (m + 127) / 128;
  auto tiles = [&](int bn) { return mb * ((n + bn - 1) / bn) * batch; };
  // share of a tile row that falls beyond n (computed, then thrown away)
  auto waste = [&](int bn) {
    const long long padded = (static_cast<long long>(n) + bn - 1) / bn * bn;
    return static_cast<double>(padded - n) / static_cast<double>(padded);
  };
  if (max_bn >= 256 && tiles(256) >= sms && waste(256) <= 0.125) return 256;
  if (tiles(128) >= sms && waste(128) <= 0.125) return 128;
  // N <= 32 (a classifier at batch 32): a 32-wide tile halves the B side of
  // the in-kernel 3xTF32 split and the MMA width that would only multiply
  // zero rows (fp32 only; max_bn 128 marks it)
  if (max_bn == 128 && n <= 32) return 32;
  return 64;
}

int run_gemm(const kx_exec* ex, const GemmCall& g) {
  if (g.m < 0 || g.n < 0 || g.k < 0 || g.batch < 0) return KX_ERR_INVALID;
  if (g.transa < 0 || g.transa > 2 || g.transb < 0 || g.transb > 2) return KX_ERR_INVALID;
  if (!valid_type(g.a_type) || !valid_type(g.b_type) || !valid_type(g.d_type) ||
      !valid_type(g.c_type))
    return KX_ERR_UNSUPPORTED;
  if (g.alpha == nullptr || g.beta == nullptr) return KX_ERR_INVALID;
  const int ta = g.transa == 0 ? 0 : 1, tb = g.transb == 0 ? 0 : 1;
  const long long a_rows = ta == 0 ? g.m : g.k;
  const long long b_rows = tb == 0 ? g.k : g.n;
  if (g.lda < (a_rows > 1 ? a_rows : 1) || g.ldb < (b_rows > 1 ? b_rows : 1) ||
      g.ldd < (g.m > 1 ? g.m : 1))
    return KX_ERR_INVALID;
  if (g.m == 0 || g.n == 0 || g.batch == 0) return KX_OK;
  Exec e = resolve_exec(ex);
  const bool dev_scalars = ex != nullptr && ex->scalars_on_device != 0;
  GemmCall gc = g;
  gc.transa = ta;
  gc.transb = tb;

  // Pointer arrays, k == 0, alpha == 0 (host mode): CUDA-core kernel.
  const bool zero_k = g.k == 0 || (!dev_scalars && *g.alpha == 0.f);
  if (g.Aarr != nullptr || zero_k) {
    if (zero_k) gc.k = 0;
    return launch_simt(e, gc, dev_scalars);
  }
  Arith ar;
  if (g.a_type == DT_F32 && g.b_type == DT_F32) {
    if (e.fp32_mode == KX_FP32_FFMA) return launch_simt(e, gc, dev_scalars);
    ar = e.fp32_mode == KX_FP32_TF32 ? Arith::TF32 : Arith::F32x3;
  } else if (g.a_type == DT_BF16 && g.b_type == DT_BF16) {
    ar = Arith::BF16;
  } else if (g.a_type == DT_F16 && g.b_type == DT_F16) {
    ar = Arith::F16;
  } else {
    return launch_simt(e, gc, dev_scalars);
  }
  const int es = esize(g.a_type);
  if (!tma_ok(g.A, g.lda, g.strideA, g.batch, es) || !tma_ok(g.B, g.ldb, g.strideB, g.batch, es))
    return launch_simt(e, gc, dev_scalars);

  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = g.m;
  p.n = g.n;
  p.k = g.k;
  if (dev_scalars) {
    p.alpha_dev = g.alpha;
    p.beta_dev = g.beta;
  } else {
    p.alpha = *g.alpha;
    p.beta = *g.beta;
  }
  p.D = g.D;
  p.ldd = g.ldd;
  p.strideD = g.strideD;
  p.d_type = g.d_type;
  p.C = g.C;
  p.ldc = g.ldc;
  p.strideC = g.strideC;
  p.c_type = g.c_type;
  p.relu = (g.epilogue == KX_EPI_RELU || g.epilogue == KX_EPI_RELU_BIAS);
  p.gelu = (g.epilogue == KX_EPI_GELU || g.epilogue == KX_EPI_GELU_BIAS);
  const bool has_bias = (g.epilogue == KX_EPI_BIAS || g.epilogue == KX_EPI_RELU_BIAS ||
                         g.epilogue == KX_EPI_GELU_BIAS);
  p.bias = has_bias ? g.bias : nullptr;
  p.bias_type = g.bias_type;
  p.work = work_slot_for(e.stream);
  if (p.work == nullptr) return KX_ERR_NOMEM;
  p.yield_flag = e.yield_flag;
  p.done_flag = e.done_flag;
  p.max_tiles = e.max_tiles;
  p.timeout_ns = e.timeout_ns;
  p.err_word = e.err_word ? e.err_word : &p.work->err;

  TcProblem pr{g.m, g.n, g.k, g.batch, g.A, g.lda, g.strideA, g.B, g.ldb, g.strideB,
               nullptr, nullptr};
  // 3xTF32 low parts: split off in global memory when every operand element
  // is reused by enough output tiles to amortise the extra pass; skinny
  // problems (m or n small: few reuses, large operand) split in the kernel.
  p.presplit = (ar == Arith::F32x3 && g.m >= 256 && g.n >= 256 &&
                static_cast<long long>(g.m) * g.n >= (1LL << 20) && !presplit_disabled())
                   ? 1
                   : 0;
  if (p.presplit) {
    // low parts of both operands, laid out exactly like the operands
    const size_t na = operand_span(ta == 0 ? g.m : g.k, ta == 0 ? g.k : g.m, g.lda, g.strideA,
                                   g.batch);
    const size_t nb = operand_span(tb == 0 ? g.k : g.n, tb == 0 ? g.n : g.k, g.ldb, g.strideB,
                                   g.batch);
    const size_t na_pad = (na + 63) & ~static_cast<size_t>(63);
    float* lo = static_cast<float*>(scratch_for(e.stream, (na_pad + nb) * sizeof(float), 2));
    if (lo == nullptr) return KX_ERR_NOMEM;
    size_t blocks = (na / 4 + nb / 4 + 255) / 256;
    const size_t cap = 8ull * device_info().num_sms;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    note_launch();
    tf32_split_lo<<<static_cast<int>(blocks), 256, 0, e.stream>>>(
        static_cast<const float*>(g.A), lo, na, static_cast<const float*>(g.B), lo + na_pad, nb);
    pr.Alo = lo;
    pr.Blo = lo + na_pad;
  }
  const int sms = persistent_grid(e, 1 << 30);
  const int bn = choose_bn(g.m, g.n, g.batch, sms, ar == Arith::F32x3 ? 128 : 256);
  const bool amn = ta == 0, bmn = tb == 1;
  int rc;
  switch (ar) {
    case Arith::F32x3: rc = dispatch_gemm_tc_f32x3(bn, amn, bmn, e, pr, p); break;
    case Arith::TF32: rc = dispatch_gemm_tc_tf32(bn, amn, bmn, e, pr, p); break;
    case Arith::BF16: rc = dispatch_gemm_tc_bf16(bn, amn, bmn, e, pr, p); break;
    default: rc = dispatch_gemm_tc_f16(bn, amn, bmn, e, pr, p); break;
  }
  if (rc == KX_ERR_UNSUPPORTED) return launch_simt(e, gc, dev_scalars);
  return rc;
}

}  // namespace
}  // namespace kx

using kx::GemmCall;

extern "C" int kx_sgemm(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                        const float* alpha, const float* A, int lda, const float* B, int ldb,
                        const float* beta, float* C, int ldc) {
  GemmCall g{};
  g.transa = transa; g.transb = transb; g.m = m; g.n = n; g.k = k; g.batch = 1;
  g.alpha = alpha; g.beta = beta;
  g.A = A; g.a_type = kx::DT_F32; g.lda = lda; g.strideA = 0;
  g.B = B; g.b_type = kx::DT_F32; g.ldb = ldb; g.strideB = 0;
  g.C = C; g.c_type = kx::DT_F32; g.ldc = ldc; g.strideC = 0;
  g.D = C; g.d_type = kx::DT_F32; g.ldd = ldc; g.strideD = 0;
  g.epilogue = KX_EPI_DEFAULT;
  return kx::run_gemm(ex, g);
}

extern "C" int kx_sgemm_strided_batched(const kx_exec* ex, int transa, int transb, int m, int n,
                                        int k, const float* alpha, const float* A, int lda,
                                        long long strideA, const float* B, int ldb,
                                        long long strideB, const float* beta, float* C, int ldc,
                                        long long strideC, int batch) {
  GemmCall g{};
  g.transa = transa; g.transb = transb; g.m = m; g.n = n; g.k = k; g.batch = batch;
  g.alpha = alpha; g.beta = beta;
  g.A = A; g.a_type = kx::DT_F32; g.lda = lda; g.strideA = strideA;
  g.B = B; g.b_type = kx::DT_F32; g.ldb = ldb; g.strideB = strideB;
  g.C = C; g.c_type = kx::DT_F32; g.ldc = ldc; g.strideC = strideC;
  g.D = C; g.d_type = kx::DT_F32; g.ldd = ldc; g.strideD = strideC;
  g.epilogue = KX_EPI_DEFAULT;
  return kx::run_gemm(ex, g);
}

extern "C" int kx_sgemm_batched(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                                const float* alpha, const float* const* Aarray, int lda,
                                const float* const* Barray, int ldb, const float* beta,
                                float* const* Carray, int ldc, int batch) {
  if (batch > 0 && (Aarray == nullptr || Barray == nullptr || Carray == nullptr))
    return KX_ERR_INVALID;
  GemmCall g{};
  g.transa = transa; g.transb = transb; g.m = m; g.n = n; g.k = k; g.batch = batch;
  g.alpha = alpha; g.beta = beta;
  g.a_type = kx::DT_F32; g.lda = lda;
  g.b_type = kx::DT_F32; g.ldb = ldb;
  g.c_type = kx::DT_F32; g.ldc = ldc;
  g.d_type = kx::DT_F32; g.ldd = ldc;
  g.epilogue = KX_EPI_DEFAULT;
  g.Aarr = reinterpret_cast<const void* const*>(Aarray);
  g.Barr = reinterpret_cast<const void* const*>(Barray);
  g.Darr = reinterpret_cast<void* const*>(Carray);
  return kx::run_gemm(ex, g);
}

extern "C" int kx_gemm_ex(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                          const float* alpha, const void* A, int Atype, int lda, const void* B,
                          int Btype, int ldb, const float* beta, void* C, int Ctype, int ldc) {
  GemmCall g{};
  g.transa = transa; g.transb = transb; g.m = m; g.n = n; g.k = k; g.batch = 1;
  g.alpha = alpha; g.beta = beta;
  g.A = A; g.a_type = Atype; g.lda = lda;
  g.B = B; g.b_type = Btype; g.ldb = ldb;
  g.C = C; g.c_type = Ctype; g.ldc = ldc;
  g.D = C; g.d_type = Ctype; g.ldd = ldc;
  g.epilogue = KX_EPI_DEFAULT;
  return kx::run_gemm(ex, g);
}

extern "C" int kx_gemm_strided_batched_ex(const kx_exec* ex, int transa, int transb, int m,
                                          int n, int k, const float* alpha, const void* A,
                                          int Atype, int lda, long long strideA, const void* B,
                                          int Btype, int ldb, long long strideB,
                                          const float* beta, void* C, int Ctype, int ldc,
                                          long long strideC, int batch) {
  GemmCall g{};
  g.transa = transa; g.transb = transb; g.m = m; g.n = n; g.k = k; g.batch = batch;
  g.alpha = alpha; g.beta = beta;
  g.A = A; g.a_type = Atype; g.lda = lda; g.strideA = strideA;
  g.B = B; g.b_type = Btype; g.ldb = ldb; g.strideB = strideB;
  g.C = C; g.c_type = Ctype; g.ldc = ldc; g.strideC = strideC;
  g.D = C; g.d_type = Ctype; g.ldd = ldc; g.strideD = strideC;
  g.epilogue = KX_EPI_DEFAULT;
  return kx::run_gemm(ex, g);
}

extern "C" int kx_matmul(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                         const float* alpha, const void* A, int Atype, int lda,
                         long long strideA, const void* B, int Btype, int ldb,
                         long long strideB, const float* beta, const void* C, int Ctype, int ldc,
                         long long strideC, void* D, int Dtype, int ldd, long long strideD,
                         int batch, int epilogue, const void* bias, int bias_type) {
  switch (epilogue) {
    case KX_EPI_DEFAULT: case KX_EPI_RELU: case KX_EPI_BIAS: case KX_EPI_RELU_BIAS:
    case KX_EPI_GELU: case KX_EPI_GELU_BIAS: break;
    default: return KX_ERR_UNSUPPORTED;
  }
  GemmCall g{};
  g.transa = transa; g.transb = transb; g.m = m; g.n = n; g.k = k; g.batch = batch;
  g.alpha = alpha; g.beta = beta;
  g.A = A; g.a_type = Atype; g.lda = lda; g.strideA = strideA;
  g.B = B; g.b_type = Btype; g.ldb = ldb; g.strideB = strideB;
  g.C = C != nullptr ? C : D; g.c_type = C != nullptr ? Ctype : Dtype;
  g.ldc = C != nullptr ? ldc : ldd; g.strideC = C != nullptr ? strideC : strideD;
  g.D = D; g.d_type = Dtype; g.ldd = ldd; g.strideD = strideD;
  g.epilogue = epilogue;
  g.bias = bias;
  g.bias_type = bias_type;
  return kx::run_gemm(ex, g);
}
