// cublas_intercept.cpp — exported cuBLAS / cuBLASLt entry points.
//
// Same symbols and signatures as the reference's src/cublas_intercept.cpp
// (cublasSgemm_v2 576-683, cublasSgemmBatched 691-755,
// cublasSgemmStridedBatched 763-879, cublasGemmEx 886-952,
// cublasGemmStridedBatchedEx 959-1029, cublasHgemm / HgemmStridedBatched /
// SgemmEx 1036-1235, cublasSetStream_v2 1248-1309, cublasLtMatmul 1319-1443).
// What the call does differs:
//
//  * Route.  A call from a registered client thread while capture is on is
//    captured: it becomes an OperationRecord (decoded arguments, scalar values
//    copied, the handle's current stream recorded) in the client's queue and
//    the worker runs it on the kx kernels.  ORION_ASYNC_MODE=1 (default)
//    returns at once, 0 waits for the worker, 2 runs kx on the calling thread.
//    Uncaptured calls go to the real library unless KX_DISPATCH=all, which
//    runs them on kx on the calling thread as well.
//  * Captured cublasLtMatmul descriptors are decoded on the calling thread
//    (cublasLt attribute getters), so the op no longer has to block until the
//    worker ran it.
//  * Operand combinations kx does not implement (e.g. fp16 compute, int8)
//    are outside the captured dense-op contract: the client's queue is drained
//    first (to keep its order) and the real library runs them.
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "dispatch.h"
#include "gpu_capture.h"
#include "real_libs.h"
#include "scheduler.h"

namespace {

using namespace orion;

typedef int cublasStatus_t;
constexpr int kStatusOk = 0;
constexpr int kStatusInternal = 6;
constexpr int kStatusExecFailed = 13;  // CUBLAS_STATUS_EXECUTION_FAILED

enum class Route { kReal, kDirect, kCapture };

bool dispatch_all() {
  static const bool all = [] {
    const char* s = std::getenv("KX_DISPATCH");
    return s != nullptr && std::strcmp(s, "all") == 0;
  }();
  return all;
}

Route route_for(void* handle, cudaStream_t stream, int* client) {
  *client = -1;
  if (tl_is_scheduler_thread || tl_in_scheduler_execution) return Route::kReal;
  if (!is_capture_enabled()) return dispatch_all() ? Route::kDirect : Route::kReal;
  const int c = resolve_client_idx(stream, handle);
  if (c < 0) return dispatch_all() ? Route::kDirect : Route::kReal;
  *client = c;
  if (get_async_mode_internal() == 2) return Route::kDirect;
  return Route::kCapture;
}

// Waits until the worker emptied the client's queue (used before an op that
// must run on the calling thread, so the client's order is kept).
void drain_client(int client) {
  if (client < 0 || client >= g_capture_state.num_clients) return;
  auto& q = g_capture_state.client_queues[client];
  const int64_t limit = wait_timeout_ns() / 1000;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(limit);
  while (q && !q->empty() && std::chrono::steady_clock::now() < deadline)
    std::this_thread::yield();  // a sleep would oversleep by the timer slack
}

cudaStream_t real_handle_stream(void* handle) {
  using Fn = int (*)(void*, cudaStream_t*);
  static Fn fn = reinterpret_cast<Fn>(real::cublas("cublasGetStream_v2"));
  cudaStream_t s = nullptr;
  if (fn && fn(handle, &s) == 0) return s;
  return handle_stream(handle);
}

bool device_pointer_mode(void* handle) {
  using Fn = int (*)(void*, int*);
  static Fn fn = reinterpret_cast<Fn>(real::cublas("cublasGetPointerMode_v2"));
  int mode = 0;
  if (fn && fn(handle, &mode) == 0) return mode == 1;
  return false;
}

int math_mode(void* handle) {
  using Fn = int (*)(void*, int*);
  static Fn fn = reinterpret_cast<Fn>(real::cublas("cublasGetMathMode"));
  int mode = 0;
  if (fn) fn(handle, &mode);
  return mode;
}

bool kx_type(int t) { return t == KX_R_32F || t == KX_R_16F || t == KX_R_16BF; }

bool fp32_compute(int compute) {
  // cublasComputeType_t with fp32 accumulation (or the legacy CUDA_R_32F)
  return compute == 0 || compute == 68 || compute == 69 || compute == 74 || compute == 75 ||
         compute == 77;
}

// Fills the shared fields of a GEMM record.
CublasGemmParams make_gemm(void* handle, int ta, int tb, int m, int n, int k, const void* alpha,
                           const void* A, int lda, const void* B, int ldb, const void* beta,
                           void* C, int ldc) {
  CublasGemmParams p;
  p.handle = handle;
  p.transa = ta;
  p.transb = tb;
  p.m = m;
  p.n = n;
  p.k = k;
  p.A = A;
  p.lda = lda;
  p.B = B;
  p.ldb = ldb;
  p.C = C;
  p.ldc = ldc;
  p.stream = real_handle_stream(handle);
  p.scalars_on_device = device_pointer_mode(handle);
  p.math_mode = math_mode(handle);
  p.Atype = p.Btype = p.Ctype = KX_R_32F;
  if (p.scalars_on_device) {
    p.alpha = alpha;
    p.beta = beta;
    p.use_stored_scalars = false;
  } else {
    p.alpha_value = alpha ? *static_cast<const float*>(alpha) : 1.f;
    p.beta_value = beta ? *static_cast<const float*>(beta) : 0.f;
    p.alpha = &p.alpha_value;
    p.beta = &p.beta_value;
    p.use_stored_scalars = true;
  }
  return p;
}

// Runs / captures a decoded GEMM record.  `real` performs the call on the
// real library when the op is not captured (or not supported).
const char* route_name(Route r, bool supported) {
  if (!supported || r == Route::kReal) return "real";
  return r == Route::kDirect ? "direct" : "capture";
}

template <class RealFn>
cublasStatus_t submit_gemm(OperationType type, CublasGemmParams p, bool supported, RealFn real) {
  int client = -1;
  const Route r = route_for(p.handle, p.stream, &client);
  if (op_log_enabled()) {
    const long long d[7] = {p.m, p.n, p.k, p.transa, p.transb, p.Atype,
                            p.batchCount > 0 ? p.batchCount : 1};
    op_log_record(client >= 0 ? client : resolve_client_idx(p.stream, p.handle), type, d, 7,
                  route_name(r, supported));
  }
  if (r == Route::kReal) return real();
  if (!supported) {
    drain_client(client);
    g_scheduler.stats(client < 0 ? 0 : client).passthrough_ops.fetch_add(1);
    return real();
  }
  if (r == Route::kDirect) {
    OperationRecord op;
    op.type = type;
    op.client_idx = client;
    op.params = p;
    auto& stored = std::get<CublasGemmParams>(op.params);
    if (stored.use_stored_scalars) {
      stored.alpha = &stored.alpha_value;
      stored.beta = &stored.beta_value;
    }
    ExecPolicy pol;
    pol.stream = p.stream;
    return dispatch_dense(op, pol) == KX_OK ? kStatusOk : kStatusExecFailed;
  }
  auto op = create_operation(client, type);
  if (!op) return real();
  op->params = p;
  auto& stored = std::get<CublasGemmParams>(op->params);
  if (stored.use_stored_scalars) {  // re-point at the record's own copies
    stored.alpha = &stored.alpha_value;
    stored.beta = &stored.beta_value;
  }
  if (!enqueue_operation(op)) return kStatusExecFailed;
  if (get_async_mode_internal() == 1) return kStatusOk;
  return wait_operation(op) == cudaSuccess ? kStatusOk : kStatusExecFailed;
}

}  // namespace

extern "C" {

cublasStatus_t cublasSgemm_v2(void* handle, int transa, int transb, int m, int n, int k,
                              const float* alpha, const float* A, int lda, const float* B,
                              int ldb, const float* beta, float* C, int ldc) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const float*, const float*, int,
                                const float*, int, const float*, float*, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasSgemm_v2"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CublasGemmParams p = make_gemm(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta,
                                 C, ldc);
  return submit_gemm(OperationType::CUBLAS_SGEMM, p, true, call_real);
}

cublasStatus_t cublasSgemmStridedBatched(void* handle, int transa, int transb, int m, int n,
                                         int k, const float* alpha, const float* A, int lda,
                                         long long strideA, const float* B, int ldb,
                                         long long strideB, const float* beta, float* C, int ldc,
                                         long long strideC, int batchCount) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const float*, const float*, int,
                                long long, const float*, int, long long, const float*, float*,
                                int, long long, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasSgemmStridedBatched"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, lda, strideA, B, ldb, strideB, beta, C,
                ldc, strideC, batchCount);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CublasGemmParams p = make_gemm(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta,
                                 C, ldc);
  p.strideA = strideA;
  p.strideB = strideB;
  p.strideC = strideC;
  p.batchCount = batchCount;
  p.is_strided = true;
  return submit_gemm(OperationType::CUBLAS_SGEMM_STRIDED_BATCHED, p, true, call_real);
}

cublasStatus_t cublasSgemmBatched(void* handle, int transa, int transb, int m, int n, int k,
                                  const float* alpha, const float* const Aarray[], int lda,
                                  const float* const Barray[], int ldb, const float* beta,
                                  float* const Carray[], int ldc, int batchCount) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const float*,
                                const float* const*, int, const float* const*, int, const float*,
                                float* const*, int, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasSgemmBatched"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, Aarray, lda, Barray, ldb, beta, Carray,
                ldc, batchCount);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CublasGemmParams p = make_gemm(handle, transa, transb, m, n, k, alpha, Aarray, lda, Barray,
                                 ldb, beta, const_cast<float**>(Carray), ldc);
  p.batchCount = batchCount;
  p.is_batched = true;
  return submit_gemm(OperationType::CUBLAS_SGEMM_BATCHED, p, true, call_real);
}

cublasStatus_t cublasGemmEx(void* handle, int transa, int transb, int m, int n, int k,
                            const void* alpha, const void* A, int Atype, int lda, const void* B,
                            int Btype, int ldb, const void* beta, void* C, int Ctype, int ldc,
                            int computeType, int algo) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const void*, const void*, int,
                                int, const void*, int, int, const void*, void*, int, int, int,
                                int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasGemmEx"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C,
                Ctype, ldc, computeType, algo);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  const bool ok = kx_type(Atype) && Atype == Btype && kx_type(Ctype) && fp32_compute(computeType);
  CublasGemmParams p = make_gemm(handle, transa, transb, m, n, k, ok ? alpha : nullptr, A, lda, B,
                                 ldb, ok ? beta : nullptr, C, ldc);
  p.Atype = Atype;
  p.Btype = Btype;
  p.Ctype = Ctype;
  return submit_gemm(OperationType::CUBLAS_GEMM_EX, p, ok, call_real);
}

cublasStatus_t cublasGemmStridedBatchedEx(void* handle, int transa, int transb, int m, int n,
                                          int k, const void* alpha, const void* A, int Atype,
                                          int lda, long long strideA, const void* B, int Btype,
                                          int ldb, long long strideB, const void* beta, void* C,
                                          int Ctype, int ldc, long long strideC, int batchCount,
                                          int computeType, int algo) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const void*, const void*, int,
                                int, long long, const void*, int, int, long long, const void*,
                                void*, int, int, long long, int, int, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasGemmStridedBatchedEx"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, Atype, lda, strideA, B, Btype, ldb,
                strideB, beta, C, Ctype, ldc, strideC, batchCount, computeType, algo);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  const bool ok = kx_type(Atype) && Atype == Btype && kx_type(Ctype) && fp32_compute(computeType);
  CublasGemmParams p = make_gemm(handle, transa, transb, m, n, k, ok ? alpha : nullptr, A, lda, B,
                                 ldb, ok ? beta : nullptr, C, ldc);
  p.Atype = Atype;
  p.Btype = Btype;
  p.Ctype = Ctype;
  p.strideA = strideA;
  p.strideB = strideB;
  p.strideC = strideC;
  p.batchCount = batchCount;
  p.is_strided = true;
  return submit_gemm(OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX, p, ok, call_real);
}

}  // extern "C"

namespace {

// cublasHgemm / cublasHgemmStridedBatched: fp16 A, B, C with __half
// alpha / beta.  kx runs them on the kind::f16 tensor-core kernel with fp32
// accumulation and one rounding of the result to fp16 (cuBLAS's
// CUBLAS_COMPUTE_16F may accumulate in fp16; fp32 accumulation is at least as
// accurate).  Host-mode scalars are converted to fp32 on the calling thread;
// __half scalars in device memory (CUBLAS_POINTER_MODE_DEVICE) are not
// decoded and such calls run on the real library (counted as passthrough).
float half_bits_to_float(const void* p) {
  uint16_t h = 0;
  std::memcpy(&h, p, sizeof(h));
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0x1fu) {
    bits = sign | 0x7f800000u | (man << 13);          // inf / nan
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);  // normal: rebias 15 -> 127
  } else if (man == 0) {
    bits = sign;                                        // signed zero
  } else {                                              // subnormal: normalise
    int e = -1;
    do {
      man <<= 1;
      ++e;
    } while ((man & 0x400u) == 0);
    bits = sign | (static_cast<uint32_t>(112 - e) << 23) | ((man & 0x3ffu) << 13);
  }
  float f;
  std::memcpy(&f, &bits, sizeof(f));
  return f;
}

CublasGemmParams make_hgemm(void* handle, int ta, int tb, int m, int n, int k, const void* alpha,
                            const void* A, int lda, const void* B, int ldb, const void* beta,
                            void* C, int ldc, bool* supported) {
  CublasGemmParams p = make_gemm(handle, ta, tb, m, n, k, nullptr, A, lda, B, ldb, nullptr, C,
                                 ldc);
  p.Atype = p.Btype = p.Ctype = KX_R_16F;
  *supported = !p.scalars_on_device && alpha != nullptr && beta != nullptr;
  if (*supported) {
    p.alpha_value = half_bits_to_float(alpha);
    p.beta_value = half_bits_to_float(beta);
    p.alpha = &p.alpha_value;
    p.beta = &p.beta_value;
    p.use_stored_scalars = true;
  }
  return p;
}

}  // namespace

extern "C" {

cublasStatus_t cublasHgemm(void* handle, int transa, int transb, int m, int n, int k,
                           const void* alpha, const void* A, int lda, const void* B, int ldb,
                           const void* beta, void* C, int ldc) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const void*, const void*, int,
                                const void*, int, const void*, void*, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasHgemm"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  bool ok = false;
  CublasGemmParams p = make_hgemm(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta,
                                  C, ldc, &ok);
  return submit_gemm(OperationType::CUBLAS_GEMM_EX, p, ok, call_real);
}

cublasStatus_t cublasHgemmStridedBatched(void* handle, int transa, int transb, int m, int n, int k,
                                         const void* alpha, const void* A, int lda,
                                         long long strideA, const void* B, int ldb,
                                         long long strideB, const void* beta, void* C, int ldc,
                                         long long strideC, int batchCount) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const void*, const void*, int,
                                long long, const void*, int, long long, const void*, void*, int,
                                long long, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasHgemmStridedBatched"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, lda, strideA, B, ldb, strideB, beta, C,
                ldc, strideC, batchCount);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  bool ok = false;
  CublasGemmParams p = make_hgemm(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta,
                                  C, ldc, &ok);
  p.strideA = strideA;
  p.strideB = strideB;
  p.strideC = strideC;
  p.batchCount = batchCount;
  p.is_strided = true;
  return submit_gemm(OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX, p, ok, call_real);
}

cublasStatus_t cublasSgemmEx(void* handle, int transa, int transb, int m, int n, int k,
                             const float* alpha, const void* A, int Atype, int lda,
                             const void* B, int Btype, int ldb, const float* beta, void* C,
                             int Ctype, int ldc) {
  using Fn = cublasStatus_t (*)(void*, int, int, int, int, int, const float*, const void*, int,
                                int, const void*, int, int, const float*, void*, int, int);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasSgemmEx"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C,
                Ctype, ldc);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  const bool ok = kx_type(Atype) && Atype == Btype && kx_type(Ctype);
  CublasGemmParams p = make_gemm(handle, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C,
                                 ldc);
  p.Atype = Atype;
  p.Btype = Btype;
  p.Ctype = Ctype;
  return submit_gemm(OperationType::CUBLAS_GEMM_EX, p, ok, call_real);
}

cublasStatus_t cublasSetStream_v2(void* handle, cudaStream_t streamId) {
  using Fn = cublasStatus_t (*)(void*, cudaStream_t);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublas("cublasSetStream_v2"));
  orion::remember_handle_stream(handle, streamId);
  if (!orion::tl_is_scheduler_thread && orion::is_capture_enabled()) {
    const int c = orion::resolve_client_idx(streamId, handle);
    if (c >= 0) {
      orion::register_client_handle(c, handle);
      if (streamId) orion::register_client_stream(c, streamId);
    }
  }
  return real ? real(handle, streamId) : kStatusInternal;
}

}  // extern "C"

// ---------------------------------------------------------------- cuBLASLt --

namespace {

using GetDescAttr = int (*)(void*, int, void*, size_t, size_t*);

template <class T>
bool get_desc(GetDescAttr fn, void* d, int attr, T* out) {
  size_t written = 0;
  return fn && fn(d, attr, out, sizeof(T), &written) == 0;
}

struct Layout {
  uint32_t type = 0;
  int32_t order = 0;
  uint64_t rows = 0, cols = 0;
  int64_t ld = 0;
  int32_t batch = 1;
  int64_t stride = 0;
};

bool read_layout(void* desc, Layout& l) {
  static GetDescAttr fn =
      reinterpret_cast<GetDescAttr>(orion::real::cublaslt("cublasLtMatrixLayoutGetAttribute"));
  if (desc == nullptr || fn == nullptr) return false;
  bool ok = get_desc(fn, desc, 0, &l.type) && get_desc(fn, desc, 2, &l.rows) &&
            get_desc(fn, desc, 3, &l.cols) && get_desc(fn, desc, 4, &l.ld);
  get_desc(fn, desc, 1, &l.order);
  get_desc(fn, desc, 5, &l.batch);
  get_desc(fn, desc, 6, &l.stride);
  return ok;
}

// Decodes a cublasLtMatmul call into LtDecoded; `supported` says whether kx
// implements it (column-major, fp32 compute and scale, host/device scalars,
// DEFAULT/RELU/BIAS/GELU epilogues, matching batch counts).
LtDecoded decode_lt(void* computeDesc, void* Adesc, void* Bdesc, void* Cdesc, void* Ddesc) {
  static GetDescAttr gd =
      reinterpret_cast<GetDescAttr>(orion::real::cublaslt("cublasLtMatmulDescGetAttribute"));
  LtDecoded d;
  std::memset(&d, 0, sizeof(d));
  int32_t compute = 0, scale = 0, pmode = 0, ta = 0, tb = 0, tc = 0, bias_type = -1;
  uint32_t epi = 1;
  const void* bias = nullptr;
  const void* ptr_attr = nullptr;
  bool ok = gd != nullptr && get_desc(gd, computeDesc, 0, &compute) &&
            get_desc(gd, computeDesc, 1, &scale) && get_desc(gd, computeDesc, 3, &ta) &&
            get_desc(gd, computeDesc, 4, &tb);
  get_desc(gd, computeDesc, 2, &pmode);
  get_desc(gd, computeDesc, 5, &tc);
  get_desc(gd, computeDesc, 7, &epi);
  get_desc(gd, computeDesc, 8, &bias);
  get_desc(gd, computeDesc, 26, &bias_type);
  // fp8 scaling pointers (A/B/C/D scale, amax) must be unset
  for (int attr : {17, 18, 19, 20, 21}) {
    ptr_attr = nullptr;
    get_desc(gd, computeDesc, attr, &ptr_attr);
    if (ptr_attr != nullptr) ok = false;
  }
  Layout A, B, C, D;
  ok = ok && read_layout(Adesc, A) && read_layout(Bdesc, B) && read_layout(Ddesc, D);
  if (Cdesc != nullptr) ok = ok && read_layout(Cdesc, C);
  else C = D;
  d.transa = ta == 0 ? 0 : 1;
  d.transb = tb == 0 ? 0 : 1;
  d.m = static_cast<int>(D.rows);
  d.n = static_cast<int>(D.cols);
  d.k = static_cast<int>(d.transa == 0 ? A.cols : A.rows);
  d.Atype = static_cast<int>(A.type);
  d.Btype = static_cast<int>(B.type);
  d.Ctype = static_cast<int>(C.type);
  d.Dtype = static_cast<int>(D.type);
  d.lda = A.ld;
  d.ldb = B.ld;
  d.ldc = C.ld;
  d.ldd = D.ld;
  d.batch = D.batch;
  d.strideA = A.batch > 1 ? A.stride : 0;
  d.strideB = B.batch > 1 ? B.stride : 0;
  d.strideC = C.batch > 1 ? C.stride : 0;
  d.strideD = D.batch > 1 ? D.stride : 0;
  d.epilogue = static_cast<int>(epi);
  d.bias = bias;
  d.bias_type = bias_type < 0 ? d.Dtype : bias_type;
  d.compute_type = compute;
  d.scale_type = scale;
  d.scalars_on_device = pmode == 1;
  const bool epi_ok = epi == KX_EPI_DEFAULT || epi == KX_EPI_RELU || epi == KX_EPI_BIAS ||
                      epi == KX_EPI_RELU_BIAS || epi == KX_EPI_GELU || epi == KX_EPI_GELU_BIAS;
  const int rows_a = d.transa == 0 ? d.m : d.k;
  const int rows_b = d.transb == 0 ? d.k : d.n;
  ok = ok && A.order == 0 && B.order == 0 && C.order == 0 && D.order == 0 && tc == 0 &&
       (pmode == 0 || pmode == 1) && epi_ok && fp32_compute(compute) && scale == KX_R_32F &&
       kx_type(d.Atype) && d.Atype == d.Btype && kx_type(d.Ctype) && kx_type(d.Dtype) &&
       static_cast<int>(A.rows) == rows_a && static_cast<int>(B.rows) == rows_b &&
       static_cast<int>(d.transb == 0 ? B.cols : B.rows) == d.n &&
       (A.batch == D.batch || A.batch == 1) && (B.batch == D.batch || B.batch == 1) &&
       (d.bias == nullptr || kx_type(d.bias_type));
  d.supported = ok;
  return d;
}

}  // namespace

extern "C" cublasStatus_t cublasLtMatmul(void* lightHandle, void* computeDesc, const void* alpha,
                                         const void* A, void* Adesc, const void* B, void* Bdesc,
                                         const void* beta, const void* C, void* Cdesc, void* D,
                                         void* Ddesc, const void* algo, void* workspace,
                                         size_t workspaceSizeInBytes, cudaStream_t stream) {
  using Fn = cublasStatus_t (*)(void*, void*, const void*, const void*, void*, const void*,
                                void*, const void*, const void*, void*, void*, void*, const void*,
                                void*, size_t, cudaStream_t);
  static Fn real = reinterpret_cast<Fn>(orion::real::cublaslt("cublasLtMatmul"));
  auto call_real = [&]() -> cublasStatus_t {
    if (!real) return kStatusInternal;
    return real(lightHandle, computeDesc, alpha, A, Adesc, B, Bdesc, beta, C, Cdesc, D, Ddesc,
                algo, workspace, workspaceSizeInBytes, stream);
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  int client = -1;
  const Route r = route_for(lightHandle, stream, &client);
  if (orion::op_log_enabled()) {
    const LtDecoded dec = decode_lt(computeDesc, Adesc, Bdesc, Cdesc, Ddesc);
    const long long d[8] = {dec.m, dec.n, dec.k, dec.transa, dec.transb, dec.Atype,
                            dec.batch > 0 ? dec.batch : 1, dec.epilogue};
    orion::op_log_record(client >= 0 ? client : orion::resolve_client_idx(stream, lightHandle),
                         orion::OperationType::CUBLASLT_MATMUL, d, 8,
                         route_name(r, dec.supported));
  }
  if (r == Route::kReal) return call_real();
  CublasLtMatmulParams p;
  p.lightHandle = lightHandle;
  p.A = A;
  p.B = B;
  p.C = C;
  p.D = D;
  p.stream = stream;
  p.dec = decode_lt(computeDesc, Adesc, Bdesc, Cdesc, Ddesc);
  if (!p.dec.supported) {
    drain_client(client);
    orion::g_scheduler.stats(client < 0 ? 0 : client).passthrough_ops.fetch_add(1);
    return call_real();
  }
  if (p.dec.scalars_on_device) {
    p.alpha = alpha;
    p.beta = beta;
  } else {
    p.alpha_value = *static_cast<const float*>(alpha);
    p.beta_value = *static_cast<const float*>(beta);
    p.use_stored_scalars = true;
  }
  if (r == Route::kDirect) {
    orion::OperationRecord op;
    op.type = orion::OperationType::CUBLASLT_MATMUL;
    op.client_idx = client;
    op.params = p;
    orion::ExecPolicy pol;
    pol.stream = stream;
    return orion::dispatch_dense(op, pol) == KX_OK ? kStatusOk : kStatusExecFailed;
  }
  auto op = orion::create_operation(client, orion::OperationType::CUBLASLT_MATMUL);
  if (!op) return call_real();
  op->params = p;
  if (!orion::enqueue_operation(op)) return kStatusExecFailed;
  if (orion::get_async_mode_internal() == 1) return kStatusOk;
  return orion::wait_operation(op) == cudaSuccess ? kStatusOk : kStatusExecFailed;
}
