// cudnn_intercept.cpp — exported cuDNN entry points.
//
// Same symbols and signatures as the reference's src/cudnn_intercept.cpp
// (cudnnConvolutionForward 433-489, BackwardData 512-558, BackwardFilter
// 581-627, cudnnBatchNormalizationForwardTraining 659-716, cudnnSetStream
// 730-747), plus the batch-norm inference / backward entry points whose types
// the reference declares (112-143) but does not wrap.
//
// Differences from the reference:
//  * descriptors are decoded on the calling thread with cuDNN's own getters
//    (cudnnGetTensor4dDescriptor / cudnnGetFilter4dDescriptor /
//    cudnnGetConvolution2dDescriptor / cudnnGetConvolutionGroupCount) and the
//    record is filled before it is enqueued (the reference enqueues first and
//    fills afterwards, src/cudnn_intercept.cpp:461/485);
//  * all three convolutions and batch norm execute under capture (the
//    reference's worker only executes CONV_FWD, src/cudnn_intercept.cpp:286-299);
//  * they run on the cuDNN handle's stream on the kx kernels.
// Calls kx does not implement (non-float data, grouped or 3-D convolutions,
// non-packed NCHW tensors) go to the real cuDNN after the client's queue has
// drained.
#include <algorithm>
#include <atomic>
#include <vector>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>

#include "dispatch.h"
#include "gpu_capture.h"
#include "real_libs.h"
#include "scheduler.h"

namespace {

using namespace orion;

typedef int cudnnStatus_t;
constexpr int kOk = 0;
constexpr int kExecFailed = 8;  // CUDNN_STATUS_EXECUTION_FAILED

enum class Route { kReal, kDirect, kCapture };

bool dispatch_all() {
  static const bool all = [] {
    const char* s = std::getenv("KX_DISPATCH");
    return s != nullptr && std::strcmp(s, "all") == 0;
  }();
  return all;
}

cudaStream_t cudnn_stream(void* handle) {
  using Fn = int (*)(void*, cudaStream_t*);
  static Fn fn = reinterpret_cast<Fn>(real::cudnn("cudnnGetStream"));
  cudaStream_t s = nullptr;
  if (fn && fn(handle, &s) == 0) return s;
  return handle_stream(handle);
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

void drain_client(int client) {
  if (client < 0 || client >= g_capture_state.num_clients) return;
  auto& q = g_capture_state.client_queues[client];
  const int64_t limit = wait_timeout_ns() / 1000;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(limit);
  while (q && !q->empty() && std::chrono::steady_clock::now() < deadline)
    std::this_thread::yield();  // a sleep would oversleep by the timer slack
}

struct Tensor4 {
  int type = -1, n = 0, c = 0, h = 0, w = 0, ns = 0, cs = 0, hs = 0, ws = 0;
  bool packed_float() const {
    return type == 0 && ws == 1 && hs == w && cs == h * w && ns == c * h * w;
  }
};

bool read_tensor(void* desc, Tensor4& t) {
  using Fn = int (*)(void*, int*, int*, int*, int*, int*, int*, int*, int*, int*);
  static Fn fn = reinterpret_cast<Fn>(real::cudnn("cudnnGetTensor4dDescriptor"));
  return desc && fn && fn(desc, &t.type, &t.n, &t.c, &t.h, &t.w, &t.ns, &t.cs, &t.hs, &t.ws) == 0;
}

bool read_filter(void* desc, int* type, int* format, int* k, int* c, int* r, int* s) {
  using Fn = int (*)(void*, int*, int*, int*, int*, int*, int*);
  static Fn fn = reinterpret_cast<Fn>(real::cudnn("cudnnGetFilter4dDescriptor"));
  return desc && fn && fn(desc, type, format, k, c, r, s) == 0;
}

bool read_conv(void* desc, ConvGeometry& g) {
  using Fn = int (*)(void*, int*, int*, int*, int*, int*, int*, int*, int*);
  using Gc = int (*)(void*, int*);
  static Fn fn = reinterpret_cast<Fn>(real::cudnn("cudnnGetConvolution2dDescriptor"));
  static Gc gc = reinterpret_cast<Gc>(real::cudnn("cudnnGetConvolutionGroupCount"));
  int mode = 0, compute = 0, groups = 1;
  if (!desc || !fn ||
      fn(desc, &g.pad_h, &g.pad_w, &g.stride_h, &g.stride_w, &g.dil_h, &g.dil_w, &mode,
         &compute) != 0)
    return false;
  if (gc) gc(desc, &groups);
  g.cross_correlation = mode == 1 ? 1 : 0;
  return groups == 1;
}

// Geometry of a convolution from (input, filter, output) descriptors.
bool conv_geometry(void* xDesc, void* wDesc, void* convDesc, void* yDesc, ConvGeometry& g) {
  std::memset(&g, 0, sizeof(g));
  Tensor4 x, y;
  int wtype = -1, wfmt = -1;
  if (!read_tensor(xDesc, x) || !read_tensor(yDesc, y) ||
      !read_filter(wDesc, &wtype, &wfmt, &g.k, &g.c, &g.r, &g.s) || !read_conv(convDesc, g))
    return false;
  g.n = x.n;
  g.h = x.h;
  g.w = x.w;
  g.data_type = x.type;
  g.packed_nchw = x.packed_float() && y.packed_float() && wtype == 0 && wfmt == 0 &&
                  x.c == g.c && y.c == g.k && y.n == x.n;
  return g.packed_nchw != 0;
}

// Shape integers of an intercepted call for the op log.
int log_dims(const CudnnConvParams& p, long long* d) {
  const ConvGeometry& g = p.geom;
  const long long v[8] = {g.n, g.c, g.h, g.w, g.k, g.r, g.s, g.stride_h * 100 + g.pad_h};
  for (int i = 0; i < 8; ++i) d[i] = v[i];
  return 8;
}
int log_dims(const CudnnBatchNormParams& p, long long* d) {
  const long long v[5] = {p.n, p.c, p.h, p.w, p.mode};
  for (int i = 0; i < 5; ++i) d[i] = v[i];
  return 5;
}

template <class Params, class RealFn>
cudnnStatus_t submit_op(OperationType type, void* handle, Params p, bool supported, RealFn real) {
  int client = -1;
  const Route r = route_for(handle, p.stream, &client);
  if (op_log_enabled()) {
    long long d[8];
    const int nd = log_dims(p, d);
    op_log_record(client >= 0 ? client : resolve_client_idx(p.stream, handle), type, d, nd,
                  (!supported || r == Route::kReal) ? "real"
                  : r == Route::kDirect            ? "direct"
                                                   : "capture");
  }
  if (r == Route::kReal) return real();
  if (!supported) {
    static std::atomic<int> reported{0};
    if (reported.fetch_add(1) < 8)
      LOG_WARN("%s: arguments not handled by kx; running on cuDNN", op_type_name(type));
    drain_client(client);
    g_scheduler.stats(client < 0 ? 0 : client).passthrough_ops.fetch_add(1);
    return real();
  }
  if (r == Route::kDirect) {
    OperationRecord op;
    op.type = type;
    op.client_idx = client;
    op.params = p;
    ExecPolicy pol;
    pol.stream = p.stream;
    return dispatch_dense(op, pol) == KX_OK ? kOk : kExecFailed;
  }
  auto op = create_operation(client, type);
  if (!op) return real();
  op->params = p;  // filled before the worker can see it
  if (!enqueue_operation(op)) return kExecFailed;
  if (get_async_mode_internal() == 1) return kOk;
  return wait_operation(op) == cudaSuccess ? kOk : kExecFailed;
}

float scalar(const void* p, float dflt) { return p ? *static_cast<const float*>(p) : dflt; }

}  // namespace

extern "C" {

cudnnStatus_t cudnnConvolutionForward(void* handle, const void* alpha, void* xDesc, const void* x,
                                      void* wDesc, const void* w, void* convDesc, int algo,
                                      void* workSpace, size_t workSpaceSizeInBytes,
                                      const void* beta, void* yDesc, void* y) {
  using Fn = cudnnStatus_t (*)(void*, const void*, void*, const void*, void*, const void*, void*,
                               int, void*, size_t, const void*, void*, void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnConvolutionForward"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, alpha, xDesc, x, wDesc, w, convDesc, algo, workSpace,
                       workSpaceSizeInBytes, beta, yDesc, y)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnConvParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.xDesc = xDesc;
  p.x = x;
  p.wDesc = wDesc;
  p.w = w;
  p.convDesc = convDesc;
  p.algo = algo;
  p.workSpace = workSpace;
  p.workSpaceSizeInBytes = workSpaceSizeInBytes;
  p.alpha = alpha;
  p.beta = beta;
  p.yDesc = yDesc;
  p.y = y;
  p.stream = cudnn_stream(handle);
  const bool ok = conv_geometry(xDesc, wDesc, convDesc, yDesc, p.geom);
  p.alpha_value = scalar(alpha, 1.f);
  p.beta_value = scalar(beta, 0.f);
  return submit_op(OperationType::CUDNN_CONV_FWD, handle, p, ok, call_real);
}

cudnnStatus_t cudnnConvolutionBackwardData(void* handle, const void* alpha, void* wDesc,
                                           const void* w, void* dyDesc, const void* dy,
                                           void* convDesc, int algo, void* workSpace,
                                           size_t workSpaceSizeInBytes, const void* beta,
                                           void* dxDesc, void* dx) {
  using Fn = cudnnStatus_t (*)(void*, const void*, void*, const void*, void*, const void*, void*,
                               int, void*, size_t, const void*, void*, void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnConvolutionBackwardData"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, alpha, wDesc, w, dyDesc, dy, convDesc, algo, workSpace,
                       workSpaceSizeInBytes, beta, dxDesc, dx)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnConvParams p;
  std::memset(&p, 0, sizeof(p));
  // field use of the reference's wrapper: x = dy, w = w, y = dx
  p.handle = handle;
  p.wDesc = wDesc;
  p.w = w;
  p.xDesc = dyDesc;
  p.x = dy;
  p.convDesc = convDesc;
  p.algo = algo;
  p.workSpace = workSpace;
  p.workSpaceSizeInBytes = workSpaceSizeInBytes;
  p.alpha = alpha;
  p.beta = beta;
  p.yDesc = dxDesc;
  p.y = dx;
  p.stream = cudnn_stream(handle);
  // geometry is that of the forward problem: input = dx, output = dy
  const bool ok = conv_geometry(dxDesc, wDesc, convDesc, dyDesc, p.geom);
  p.alpha_value = scalar(alpha, 1.f);
  p.beta_value = scalar(beta, 0.f);
  return submit_op(OperationType::CUDNN_CONV_BWD_DATA, handle, p, ok, call_real);
}

cudnnStatus_t cudnnConvolutionBackwardFilter(void* handle, const void* alpha, void* xDesc,
                                             const void* x, void* dyDesc, const void* dy,
                                             void* convDesc, int algo, void* workSpace,
                                             size_t workSpaceSizeInBytes, const void* beta,
                                             void* dwDesc, void* dw) {
  using Fn = cudnnStatus_t (*)(void*, const void*, void*, const void*, void*, const void*, void*,
                               int, void*, size_t, const void*, void*, void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnConvolutionBackwardFilter"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, alpha, xDesc, x, dyDesc, dy, convDesc, algo, workSpace,
                       workSpaceSizeInBytes, beta, dwDesc, dw)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnConvParams p;
  std::memset(&p, 0, sizeof(p));
  // field use of the reference's wrapper: x = x, y = dy, w = dw
  p.handle = handle;
  p.xDesc = xDesc;
  p.x = x;
  p.yDesc = dyDesc;
  p.y = const_cast<void*>(dy);
  p.convDesc = convDesc;
  p.algo = algo;
  p.workSpace = workSpace;
  p.workSpaceSizeInBytes = workSpaceSizeInBytes;
  p.alpha = alpha;
  p.beta = beta;
  p.wDesc = dwDesc;
  p.w = dw;
  p.stream = cudnn_stream(handle);
  const bool ok = conv_geometry(xDesc, dwDesc, convDesc, dyDesc, p.geom);
  p.alpha_value = scalar(alpha, 1.f);
  p.beta_value = scalar(beta, 0.f);
  return submit_op(OperationType::CUDNN_CONV_BWD_FILTER, handle, p, ok, call_real);
}

cudnnStatus_t cudnnBatchNormalizationForwardTraining(
    void* handle, int mode, const void* alpha, const void* beta, void* xDesc, const void* x,
    void* yDesc, void* y, void* bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    double exponentialAverageFactor, void* resultRunningMean, void* resultRunningVariance,
    double epsilon, void* resultSaveMean, void* resultSaveInvVariance) {
  using Fn = cudnnStatus_t (*)(void*, int, const void*, const void*, void*, const void*, void*,
                               void*, void*, const void*, const void*, double, void*, void*,
                               double, void*, void*);
  static Fn real =
      reinterpret_cast<Fn>(orion::real::cudnn("cudnnBatchNormalizationForwardTraining"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, mode, alpha, beta, xDesc, x, yDesc, y, bnScaleBiasMeanVarDesc,
                       bnScale, bnBias, exponentialAverageFactor, resultRunningMean,
                       resultRunningVariance, epsilon, resultSaveMean, resultSaveInvVariance)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnBatchNormParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.mode = mode;
  p.alpha = alpha;
  p.beta = beta;
  p.xDesc = xDesc;
  p.x = x;
  p.yDesc = yDesc;
  p.y = y;
  p.bnScaleBiasMeanVarDesc = bnScaleBiasMeanVarDesc;
  p.bnScale = bnScale;
  p.bnBias = bnBias;
  p.exponentialAverageFactor = exponentialAverageFactor;
  p.resultRunningMean = resultRunningMean;
  p.resultRunningVariance = resultRunningVariance;
  p.epsilon = epsilon;
  p.resultSaveMean = resultSaveMean;
  p.resultSaveInvVariance = resultSaveInvVariance;
  p.stream = cudnn_stream(handle);
  Tensor4 tx, ty;
  const bool ok = read_tensor(xDesc, tx) && read_tensor(yDesc, ty) && tx.packed_float() &&
                  ty.packed_float() && mode >= 0 && mode <= 2;
  p.n = tx.n;
  p.c = tx.c;
  p.h = tx.h;
  p.w = tx.w;
  p.alpha_value = scalar(alpha, 1.f);
  p.beta_value = scalar(beta, 0.f);
  return submit_op(OperationType::CUDNN_BATCHNORM_FWD, handle, p, ok, call_real);
}

cudnnStatus_t cudnnBatchNormalizationForwardInference(
    void* handle, int mode, const void* alpha, const void* beta, void* xDesc, const void* x,
    void* yDesc, void* y, void* bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    const void* estimatedMean, const void* estimatedVariance, double epsilon) {
  using Fn = cudnnStatus_t (*)(void*, int, const void*, const void*, void*, const void*, void*,
                               void*, void*, const void*, const void*, const void*, const void*,
                               double);
  static Fn real =
      reinterpret_cast<Fn>(orion::real::cudnn("cudnnBatchNormalizationForwardInference"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, mode, alpha, beta, xDesc, x, yDesc, y, bnScaleBiasMeanVarDesc,
                       bnScale, bnBias, estimatedMean, estimatedVariance, epsilon)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnBatchNormParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.mode = mode;
  p.x = x;
  p.y = y;
  p.xDesc = xDesc;
  p.yDesc = yDesc;
  p.bnScaleBiasMeanVarDesc = bnScaleBiasMeanVarDesc;
  p.bnScale = bnScale;
  p.bnBias = bnBias;
  p.estimatedMean = estimatedMean;
  p.estimatedVariance = estimatedVariance;
  p.epsilon = epsilon;
  p.stream = cudnn_stream(handle);
  Tensor4 tx, ty;
  const bool ok = read_tensor(xDesc, tx) && read_tensor(yDesc, ty) && tx.packed_float() &&
                  ty.packed_float() && mode >= 0 && mode <= 2;
  p.n = tx.n;
  p.c = tx.c;
  p.h = tx.h;
  p.w = tx.w;
  p.alpha_value = scalar(alpha, 1.f);
  p.beta_value = scalar(beta, 0.f);
  return submit_op(OperationType::CUDNN_BATCHNORM_INF, handle, p, ok, call_real);
}

cudnnStatus_t cudnnBatchNormalizationBackward(
    void* handle, int mode, const void* alphaDataDiff, const void* betaDataDiff,
    const void* alphaParamDiff, const void* betaParamDiff, void* xDesc, const void* x,
    void* dyDesc, const void* dy, void* dxDesc, void* dx, void* dBnScaleBiasDesc,
    const void* bnScale, void* dBnScaleResult, void* dBnBiasResult, double epsilon,
    const void* savedMean, const void* savedInvVariance) {
  using Fn = cudnnStatus_t (*)(void*, int, const void*, const void*, const void*, const void*,
                               void*, const void*, void*, const void*, void*, void*, void*,
                               const void*, void*, void*, double, const void*, const void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBatchNormalizationBackward"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, mode, alphaDataDiff, betaDataDiff, alphaParamDiff, betaParamDiff,
                       xDesc, x, dyDesc, dy, dxDesc, dx, dBnScaleBiasDesc, bnScale,
                       dBnScaleResult, dBnBiasResult, epsilon, savedMean, savedInvVariance)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnBatchNormParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.mode = mode;
  p.xDesc = xDesc;
  p.x = x;
  p.dy = dy;
  p.dx = dx;
  p.bnScale = bnScale;
  p.dBnScaleResult = dBnScaleResult;
  p.dBnBiasResult = dBnBiasResult;
  p.epsilon = epsilon;
  p.resultSaveMean = const_cast<void*>(savedMean);
  p.resultSaveInvVariance = const_cast<void*>(savedInvVariance);
  p.stream = cudnn_stream(handle);
  Tensor4 tx, tdy, tdx;
  const bool ok = read_tensor(xDesc, tx) && read_tensor(dyDesc, tdy) &&
                  read_tensor(dxDesc, tdx) && tx.packed_float() && tdy.packed_float() &&
                  tdx.packed_float() && mode >= 0 && mode <= 2;
  p.n = tx.n;
  p.c = tx.c;
  p.h = tx.h;
  p.w = tx.w;
  p.alpha_value = scalar(alphaDataDiff, 1.f);
  p.beta_value = scalar(betaDataDiff, 0.f);
  p.alpha_param = scalar(alphaParamDiff, 1.f);
  p.beta_param = scalar(betaParamDiff, 0.f);
  return submit_op(OperationType::CUDNN_BATCHNORM_BWD, handle, p, ok, call_real);
}

// The *Ex forms are what PyTorch's cuDNN batch norm calls.  With bnOps ==
// CUDNN_BATCHNORM_OPS_BN (0), no z input and no activation they compute the
// same thing as the plain forms and take the same kx path; the fused
// add / activation forms go to the real cuDNN.  The kx kernels neither read
// nor write the reserve space, so a forward and its backward must take the
// same route (both captured or both real), as they do when the capture flag
// is not toggled between them.
cudnnStatus_t cudnnBatchNormalizationForwardTrainingEx(
    void* handle, int mode, int bnOps, const void* alpha, const void* beta, void* xDesc,
    const void* x, void* zDesc, const void* z, void* yDesc, void* y,
    void* bnScaleBiasMeanVarDesc, const void* bnScale, const void* bnBias,
    double exponentialAverageFactor, void* resultRunningMean, void* resultRunningVariance,
    double epsilon, void* resultSaveMean, void* resultSaveInvVariance, void* activationDesc,
    void* workspace, size_t workSpaceSizeInBytes, void* reserveSpace,
    size_t reserveSpaceSizeInBytes) {
  using Fn = cudnnStatus_t (*)(void*, int, int, const void*, const void*, void*, const void*,
                               void*, const void*, void*, void*, void*, const void*, const void*,
                               double, void*, void*, double, void*, void*, void*, void*, size_t,
                               void*, size_t);
  static Fn real =
      reinterpret_cast<Fn>(orion::real::cudnn("cudnnBatchNormalizationForwardTrainingEx"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, mode, bnOps, alpha, beta, xDesc, x, zDesc, z, yDesc, y,
                       bnScaleBiasMeanVarDesc, bnScale, bnBias, exponentialAverageFactor,
                       resultRunningMean, resultRunningVariance, epsilon, resultSaveMean,
                       resultSaveInvVariance, activationDesc, workspace, workSpaceSizeInBytes,
                       reserveSpace, reserveSpaceSizeInBytes)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnBatchNormParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.mode = mode;
  p.alpha = alpha;
  p.beta = beta;
  p.xDesc = xDesc;
  p.x = x;
  p.yDesc = yDesc;
  p.y = y;
  p.bnScaleBiasMeanVarDesc = bnScaleBiasMeanVarDesc;
  p.bnScale = bnScale;
  p.bnBias = bnBias;
  p.exponentialAverageFactor = exponentialAverageFactor;
  p.resultRunningMean = resultRunningMean;
  p.resultRunningVariance = resultRunningVariance;
  p.epsilon = epsilon;
  p.resultSaveMean = resultSaveMean;
  p.resultSaveInvVariance = resultSaveInvVariance;
  p.stream = cudnn_stream(handle);
  Tensor4 tx, ty;
  const bool ok = bnOps == 0 && z == nullptr && activationDesc == nullptr &&
                  read_tensor(xDesc, tx) && read_tensor(yDesc, ty) && tx.packed_float() &&
                  ty.packed_float() && mode >= 0 && mode <= 2;
  p.n = tx.n;
  p.c = tx.c;
  p.h = tx.h;
  p.w = tx.w;
  p.alpha_value = scalar(alpha, 1.f);
  p.beta_value = scalar(beta, 0.f);
  return submit_op(OperationType::CUDNN_BATCHNORM_FWD, handle, p, ok, call_real);
}

cudnnStatus_t cudnnBatchNormalizationBackwardEx(
    void* handle, int mode, int bnOps, const void* alphaDataDiff, const void* betaDataDiff,
    const void* alphaParamDiff, const void* betaParamDiff, void* xDesc, const void* x,
    void* yDesc, const void* y, void* dyDesc, const void* dy, void* dzDesc, void* dz,
    void* dxDesc, void* dx, void* dBnScaleBiasDesc, const void* bnScale, const void* bnBias,
    void* dBnScaleResult, void* dBnBiasResult, double epsilon, const void* savedMean,
    const void* savedInvVariance, void* activationDesc, void* workSpace,
    size_t workSpaceSizeInBytes, void* reserveSpace, size_t reserveSpaceSizeInBytes) {
  using Fn = cudnnStatus_t (*)(void*, int, int, const void*, const void*, const void*,
                               const void*, void*, const void*, void*, const void*, void*,
                               const void*, void*, void*, void*, void*, void*, const void*,
                               const void*, void*, void*, double, const void*, const void*,
                               void*, void*, size_t, void*, size_t);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBatchNormalizationBackwardEx"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, mode, bnOps, alphaDataDiff, betaDataDiff, alphaParamDiff,
                       betaParamDiff, xDesc, x, yDesc, y, dyDesc, dy, dzDesc, dz, dxDesc, dx,
                       dBnScaleBiasDesc, bnScale, bnBias, dBnScaleResult, dBnBiasResult, epsilon,
                       savedMean, savedInvVariance, activationDesc, workSpace,
                       workSpaceSizeInBytes, reserveSpace, reserveSpaceSizeInBytes)
                : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  CudnnBatchNormParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.mode = mode;
  p.xDesc = xDesc;
  p.x = x;
  p.dy = dy;
  p.dx = dx;
  p.bnScale = bnScale;
  p.dBnScaleResult = dBnScaleResult;
  p.dBnBiasResult = dBnBiasResult;
  p.epsilon = epsilon;
  p.resultSaveMean = const_cast<void*>(savedMean);
  p.resultSaveInvVariance = const_cast<void*>(savedInvVariance);
  p.stream = cudnn_stream(handle);
  Tensor4 tx, tdy, tdx;
  const bool ok = bnOps == 0 && dz == nullptr && activationDesc == nullptr &&
                  read_tensor(xDesc, tx) && read_tensor(dyDesc, tdy) &&
                  read_tensor(dxDesc, tdx) && tx.packed_float() && tdy.packed_float() &&
                  tdx.packed_float() && mode >= 0 && mode <= 2;
  p.n = tx.n;
  p.c = tx.c;
  p.h = tx.h;
  p.w = tx.w;
  p.alpha_value = scalar(alphaDataDiff, 1.f);
  p.beta_value = scalar(betaDataDiff, 0.f);
  p.alpha_param = scalar(alphaParamDiff, 1.f);
  p.beta_param = scalar(betaParamDiff, 0.f);
  return submit_op(OperationType::CUDNN_BATCHNORM_BWD, handle, p, ok, call_real);
}

cudnnStatus_t cudnnSetStream(void* handle, cudaStream_t streamId) {
  using Fn = cudnnStatus_t (*)(void*, cudaStream_t);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnSetStream"));
  orion::remember_handle_stream(handle, streamId);
  if (orion::g_capture_state.initialized.load() && !orion::tl_is_scheduler_thread) {
    const int c = orion::resolve_client_idx(streamId, handle);
    if (c >= 0) {
      orion::register_client_handle(c, handle);
      if (streamId) orion::register_client_stream(c, streamId);
    }
  }
  return real ? real(handle, streamId) : 1;
}

}  // extern "C"

// ------------------------------------------------------- backend graph API --
//
// PyTorch 2.x reaches cuDNN convolutions only through the graph API: it
// builds a one-operation graph, finalizes an execution plan for it and calls
// cudnnBackendExecute(handle, plan, variantPack).  cuDNN does not hand the
// operations of a finalized graph back (getting CUDNN_ATTR_OPERATIONGRAPH_OPS
// answers CUDNN_STATUS_NOT_SUPPORTED), so the interposer keeps a shadow of
// the descriptors as the caller builds them: cudnnBackendCreateDescriptor
// records each descriptor's type, cudnnBackendSetAttribute the attributes
// that describe a convolution (tensor dims / strides / UID / type, the
// convolution descriptor, the operation's tensors and scalars, graph ops,
// engine -> graph, engine config -> engine, plan -> engine config) and
// cudnnBackendGetAttribute the engine configs that heuristics return for a
// graph.  When a plan is finalized its chain is resolved (all descriptors are
// still alive then) and the decoded convolution is cached per plan;
// cudnnBackendDestroyDescriptor drops shadows and cached plans.  Data
// pointers come from the variant pack by tensor UID.  A plan that does not
// decode to a single packed-NCHW fp32 2-D convolution runs on the real cuDNN.

namespace {

using BDesc = void*;
using GetAttr = int (*)(BDesc, int, int, int64_t, int64_t*, void*);

constexpr int kTypeDataType = 1, kTypeInt64 = 3, kTypeFloat = 4, kTypeDouble = 5,
              kTypeVoidPtr = 6, kTypeConvMode = 7, kTypeBackendDesc = 15;
constexpr int kDescPlan = 5, kDescConvFwd = 10, kDescConvBwdFilter = 11, kDescConvBwdData = 12,
              kDescOpGraph = 15;
// attribute names (cudnnBackendAttributeName_t)
constexpr int kAttrConvCompType = 100, kAttrConvMode = 101, kAttrConvDilations = 102,
              kAttrConvStrides = 103, kAttrConvPostPad = 104, kAttrConvPrePad = 105,
              kAttrConvSpatialDims = 106, kAttrHeurGraph = 201, kAttrHeurResults = 202,
              kAttrCfgEngine = 300, kAttrPlanCfg = 401, kAttrGraphOps = 801,
              kAttrTensorType = 901, kAttrTensorDims = 902, kAttrTensorStrides = 903,
              kAttrTensorUid = 906, kAttrPackUids = 1000, kAttrPackPtrs = 1001,
              kAttrEngineGraph = 1300;
constexpr int kSynthCfgGraph = -1;  // graph of the heuristics query a config came from

bool recorded_attr(int a) {
  return (a >= kAttrConvCompType && a <= kAttrConvSpatialDims) || a == kAttrHeurGraph ||
         a == kAttrCfgEngine || a == kAttrPlanCfg || (a >= 700 && a <= 717) ||
         a == kAttrGraphOps || a == kAttrTensorType || a == kAttrTensorDims ||
         a == kAttrTensorStrides || a == kAttrTensorUid || a == kAttrEngineGraph ||
         a == kAttrPackUids || a == kAttrPackPtrs;
}

struct PlanInfo;

struct Shadow {
  int type = -1;
  std::unordered_map<int, std::vector<int64_t>> ints;  // INT64 and enum attributes
  std::unordered_map<int, std::vector<BDesc>> descs;   // descriptor attributes
  std::unordered_map<int, double> scalars;             // FLOAT / DOUBLE attributes
  // Heuristics, engine and engine-config descriptors: the convolution their
  // operation graph holds, decoded while that graph was alive (callers may
  // destroy the graph before they finalize the plan).
  std::shared_ptr<const PlanInfo> conv;
};

std::shared_ptr<const PlanInfo> decode_graph_shared(BDesc graph);

std::mutex g_shadow_mu;
std::unordered_map<BDesc, Shadow> g_shadow;

void record_set(BDesc d, int attr, int type, int64_t count, const void* elems) {
  if (!recorded_attr(attr) || elems == nullptr || count < 0 || count > 64) return;
  std::lock_guard<std::mutex> lk(g_shadow_mu);
  Shadow& s = g_shadow[d];
  switch (type) {
    case kTypeInt64: {
      const int64_t* v = static_cast<const int64_t*>(elems);
      s.ints[attr].assign(v, v + count);
      break;
    }
    case kTypeDataType:
    case kTypeConvMode: {
      const int* v = static_cast<const int*>(elems);
      s.ints[attr].assign(v, v + count);
      break;
    }
    case kTypeVoidPtr: {
      const BDesc* v = static_cast<const BDesc*>(elems);
      s.descs[attr].assign(v, v + count);
      break;
    }
    case kTypeBackendDesc: {
      const BDesc* v = static_cast<const BDesc*>(elems);
      s.descs[attr].assign(v, v + count);
      if (count == 1 && (attr == kAttrHeurGraph || attr == kAttrEngineGraph)) {
        s.conv = decode_graph_shared(v[0]);
      } else if (count == 1 && attr == kAttrCfgEngine) {
        auto it = g_shadow.find(v[0]);
        s.conv = it == g_shadow.end() ? nullptr : it->second.conv;
      }
      break;
    }
    case kTypeFloat:
      if (count == 1) s.scalars[attr] = *static_cast<const float*>(elems);
      break;
    case kTypeDouble:
      if (count == 1) s.scalars[attr] = *static_cast<const double*>(elems);
      break;
    default:
      break;
  }
}

// Reads from the shadow map (caller holds g_shadow_mu).
const Shadow* shadow_of(BDesc d) {
  auto it = g_shadow.find(d);
  return it == g_shadow.end() ? nullptr : &it->second;
}

BDesc first_desc(const Shadow* s, int attr) {
  if (s == nullptr) return nullptr;
  auto it = s->descs.find(attr);
  return it == s->descs.end() || it->second.empty() ? nullptr : it->second[0];
}

const std::vector<int64_t>* ints_of(const Shadow* s, int attr) {
  if (s == nullptr) return nullptr;
  auto it = s->ints.find(attr);
  return it == s->ints.end() ? nullptr : &it->second;
}

struct TensorInfo {
  int64_t uid = -1;
  int64_t dims[4] = {0};
  int64_t strides[4] = {0};
  int dtype = -1;
};

bool shadow_tensor(BDesc t, TensorInfo& ti) {
  const Shadow* s = shadow_of(t);
  const auto* dims = ints_of(s, kAttrTensorDims);
  const auto* str = ints_of(s, kAttrTensorStrides);
  const auto* uid = ints_of(s, kAttrTensorUid);
  const auto* dt = ints_of(s, kAttrTensorType);
  if (!dims || !str || !uid || !dt || dims->size() != 4 || str->size() != 4 || uid->empty() ||
      dt->empty())
    return false;
  for (int i = 0; i < 4; ++i) {
    ti.dims[i] = (*dims)[i];
    ti.strides[i] = (*str)[i];
  }
  ti.uid = (*uid)[0];
  ti.dtype = static_cast<int>((*dt)[0]);
  return true;
}

bool packed_nchw(const TensorInfo& t) {
  return t.strides[3] == 1 && t.strides[2] == t.dims[3] && t.strides[1] == t.dims[2] * t.dims[3] &&
         t.strides[0] == t.dims[1] * t.dims[2] * t.dims[3];
}

// Decoded plan: which convolution, geometry, the three UIDs and the scalars.
struct PlanInfo {
  bool ok = false;
  const char* why = "not decoded";  // first check that failed
  OperationType type = OperationType::UNKNOWN;
  ConvGeometry geom;
  int64_t uid_x = -1, uid_w = -1, uid_y = -1;  // forward roles: input, filter, output
  float alpha = 1.f, beta = 0.f;
};

// Decodes the single convolution of an operation graph from the shadow
// records.  Caller holds g_shadow_mu.
PlanInfo decode_op(BDesc op_desc);

PlanInfo decode_graph(BDesc graph) {
  PlanInfo info;
  const Shadow* sg = shadow_of(graph);
  if (sg && sg->conv) return *sg->conv;  // decoded when the graph was finalized
  if (!sg || !sg->descs.count(kAttrGraphOps)) {
    info.why = "graph without recorded operations";
    return info;
  }
  const auto& ops = sg->descs.at(kAttrGraphOps);
  if (ops.size() != 1) {
    info.why = "graph is not a single operation";
    return info;
  }
  const Shadow* op = shadow_of(ops[0]);
  if (op && op->conv) return *op->conv;  // decoded when the operation was finalized
  return decode_op(ops[0]);
}

// Decodes one convolution operation descriptor (its tensors and convolution
// descriptor must still be recorded).  Caller holds g_shadow_mu.
PlanInfo decode_op(BDesc op_desc) {
  PlanInfo info;
  auto fail = [&info](const char* why) {
    info.why = why;
    return info;
  };
  const Shadow* op = shadow_of(op_desc);
  if (!op) return fail("operation not recorded");
  struct Kind { int desc; OperationType t; int alpha, beta, conv, in, filt, out; };
  // attribute numbers in forward roles: input, filter, output
  static const Kind kinds[] = {
      {kDescConvFwd, OperationType::CUDNN_CONV_FWD, 700, 701, 702, 704, 703, 705},
      {kDescConvBwdData, OperationType::CUDNN_CONV_BWD_DATA, 706, 707, 708, 710, 709, 711},
      {kDescConvBwdFilter, OperationType::CUDNN_CONV_BWD_FILTER, 712, 713, 714, 716, 715, 717},
  };
  const Kind* k = nullptr;
  for (const auto& c : kinds)
    if (op->type == c.desc) k = &c;
  if (!k) return fail("operation is not a convolution");
  TensorInfo in, filt, out;
  if (!shadow_tensor(first_desc(op, k->in), in) || !shadow_tensor(first_desc(op, k->filt), filt) ||
      !shadow_tensor(first_desc(op, k->out), out)) {
    if (std::getenv("KX_CUDNN_DEBUG") != nullptr) {
      for (int a : {k->in, k->filt, k->out}) {
        BDesc t = first_desc(op, a);
        const Shadow* st = shadow_of(t);
        std::string d = "tensor attr " + std::to_string(a) + " desc " +
                        std::to_string(reinterpret_cast<uintptr_t>(t)) +
                        (st ? " type " + std::to_string(st->type) : std::string(" unrecorded"));
        if (st)
          for (const auto& kv : st->ints) {
            d += " [" + std::to_string(kv.first) + ":";
            for (int64_t v : kv.second) d += " " + std::to_string(v);
            d += "]";
          }
        LOG_WARN("%s", d.c_str());
      }
    }
    return fail("convolution tensors are not 4-D or not recorded");
  }
  const Shadow* cd = shadow_of(first_desc(op, k->conv));
  const auto* sd = ints_of(cd, kAttrConvSpatialDims);
  const auto* pre = ints_of(cd, kAttrConvPrePad);
  const auto* post = ints_of(cd, kAttrConvPostPad);
  const auto* dil = ints_of(cd, kAttrConvDilations);
  const auto* str = ints_of(cd, kAttrConvStrides);
  const auto* mode = ints_of(cd, kAttrConvMode);
  const auto* comp = ints_of(cd, kAttrConvCompType);
  if (!sd || sd->empty() || (*sd)[0] != 2 || !pre || pre->size() != 2 || !post ||
      post->size() != 2 || !dil || dil->size() != 2 || !str || str->size() != 2)
    return fail("convolution descriptor is not 2-D");
  ConvGeometry& G = info.geom;
  std::memset(&G, 0, sizeof(G));
  G.n = static_cast<int>(in.dims[0]);
  G.c = static_cast<int>(in.dims[1]);
  G.h = static_cast<int>(in.dims[2]);
  G.w = static_cast<int>(in.dims[3]);
  G.k = static_cast<int>(filt.dims[0]);
  G.r = static_cast<int>(filt.dims[2]);
  G.s = static_cast<int>(filt.dims[3]);
  G.pad_h = static_cast<int>((*pre)[0]);
  G.pad_w = static_cast<int>((*pre)[1]);
  G.dil_h = static_cast<int>((*dil)[0]);
  G.dil_w = static_cast<int>((*dil)[1]);
  G.stride_h = static_cast<int>((*str)[0]);
  G.stride_w = static_cast<int>((*str)[1]);
  G.cross_correlation = (mode && !mode->empty() && (*mode)[0] == 0) ? 0 : 1;
  G.data_type = in.dtype;
  const bool float_math = !comp || comp->empty() || (*comp)[0] == 0;
  const bool geom_ok = (*pre)[0] == (*post)[0] && (*pre)[1] == (*post)[1] &&
                       filt.dims[1] == in.dims[1] && out.dims[0] == in.dims[0] &&
                       out.dims[1] == filt.dims[0] && in.dtype == 0 && filt.dtype == 0 &&
                       out.dtype == 0 && float_math && packed_nchw(in) && packed_nchw(filt) &&
                       packed_nchw(out) && G.stride_h > 0 && G.stride_w > 0 && G.dil_h > 0 &&
                       G.dil_w > 0;
  if (!geom_ok) return fail("data type / grouping / layout not handled by kx");
  G.packed_nchw = 1;
  info.type = k->t;
  info.uid_x = in.uid;
  info.uid_w = filt.uid;
  info.uid_y = out.uid;
  auto sa = op->scalars.find(k->alpha);
  auto sb = op->scalars.find(k->beta);
  info.alpha = sa == op->scalars.end() ? 1.f : static_cast<float>(sa->second);
  info.beta = sb == op->scalars.end() ? 0.f : static_cast<float>(sb->second);
  info.ok = true;
  info.why = "";
  return info;
}

std::shared_ptr<const PlanInfo> decode_graph_shared(BDesc graph) {
  return std::make_shared<const PlanInfo>(decode_graph(graph));
}

// Resolves plan -> engine config -> decoded convolution (recorded when the
// config came from heuristics or was built on an engine).  Caller holds
// g_shadow_mu.
PlanInfo decode_shadow(BDesc plan) {
  PlanInfo info;
  BDesc cfg = first_desc(shadow_of(plan), kAttrPlanCfg);
  if (!cfg) {
    info.why = "plan has no recorded engine config";
    return info;
  }
  const Shadow* scfg = shadow_of(cfg);
  if (scfg && scfg->conv) return *scfg->conv;
  info.why = "engine config without a recorded operation graph";
  return info;
}

std::mutex g_plan_mu;
std::unordered_map<BDesc, PlanInfo> g_plans;

// Calls seen per attribute name (diagnostics for undecodable plans).
std::atomic<int> g_set_calls[2048], g_get_calls[2048];

std::string describe(BDesc d) {
  const Shadow* s = shadow_of(d);
  if (!s) return "unrecorded";
  std::string out = "type " + std::to_string(s->type) + " attrs";
  for (const auto& kv : s->ints) out += " " + std::to_string(kv.first);
  for (const auto& kv : s->descs) out += " " + std::to_string(kv.first) + "(d" + std::to_string(kv.second.size()) + ")";
  for (const auto& kv : s->scalars) out += " " + std::to_string(kv.first) + "(f)";
  return out;
}

void dump_chain(BDesc plan) {
  std::string msg;
  {
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    BDesc cfg = first_desc(shadow_of(plan), kAttrPlanCfg);
    BDesc synth = first_desc(shadow_of(cfg), kSynthCfgGraph);
    BDesc eng = first_desc(shadow_of(cfg), kAttrCfgEngine);
    BDesc eg = first_desc(shadow_of(eng), kAttrEngineGraph);
    char buf[160];
    snprintf(buf, sizeof(buf), "plan %p cfg %p synth-graph %p engine %p engine-graph %p; ", plan,
             cfg, synth, eng, eg);
    msg = buf;
    msg += "plan: " + describe(plan) + "; cfg: " + describe(cfg) + "; graph: " +
           describe(synth ? synth : eg) + "; set calls:";
  }
  for (int a = 0; a < 2048; ++a)
    if (g_set_calls[a].load()) msg += " " + std::to_string(a) + "x" + std::to_string(g_set_calls[a].load());
  msg += "; get calls:";
  for (int a = 0; a < 2048; ++a)
    if (g_get_calls[a].load()) msg += " " + std::to_string(a) + "x" + std::to_string(g_get_calls[a].load());
  LOG_WARN("%s", msg.c_str());
}

void note_plan(BDesc plan, const PlanInfo& info) {
  static std::atomic<int> reported{0};
  const int nrep = reported.fetch_add(1);
  if (!info.ok && nrep < 8) LOG_WARN("cudnn plan %p will run on cuDNN (%s)", plan, info.why);
  if (!info.ok && nrep < 2 && std::getenv("KX_CUDNN_DEBUG") != nullptr) dump_chain(plan);
  std::lock_guard<std::mutex> lk(g_plan_mu);
  g_plans[plan] = info;
}

PlanInfo plan_info(BDesc plan) {
  {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto it = g_plans.find(plan);
    if (it != g_plans.end()) return it->second;
  }
  // finalized before the interposer saw it (not expected under LD_PRELOAD)
  PlanInfo info;
  {
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    info = decode_shadow(plan);
  }
  note_plan(plan, info);
  return info;
}

// Data pointers of the plan's three tensors, by UID, from the variant pack
// (recorded as the caller set it; cuDNN's getter as a fallback).
bool variant_pointers(BDesc vp, const PlanInfo& info, void** px, void** pw, void** py) {
  int64_t uids[16], n = 0, np = 0;
  void* ptrs[16];
  {
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    const Shadow* s = shadow_of(vp);
    const auto* u = ints_of(s, kAttrPackUids);
    auto pit = s ? s->descs.find(kAttrPackPtrs) : decltype(s->descs.end()){};
    if (u && s && pit != s->descs.end() && u->size() == pit->second.size() && u->size() <= 16) {
      n = np = static_cast<int64_t>(u->size());
      for (int64_t i = 0; i < n; ++i) {
        uids[i] = (*u)[i];
        ptrs[i] = pit->second[i];
      }
    }
  }
  if (n == 0) {
    static GetAttr get = reinterpret_cast<GetAttr>(real::cudnn("cudnnBackendGetAttribute"));
    if (!get) return false;
    if (get(vp, kAttrPackUids, kTypeInt64, 16, &n, uids) != 0) return false;
    if (get(vp, kAttrPackPtrs, kTypeVoidPtr, 16, &np, ptrs) != 0 || np != n) return false;
  }
  *px = *pw = *py = nullptr;
  for (int64_t i = 0; i < n && i < 16; ++i) {
    if (uids[i] == info.uid_x) *px = ptrs[i];
    if (uids[i] == info.uid_w) *pw = ptrs[i];
    if (uids[i] == info.uid_y) *py = ptrs[i];
  }
  return *px && *pw && *py;
}

}  // namespace

extern "C" {

cudnnStatus_t cudnnBackendCreateDescriptor(int descriptorType, void** descriptor) {
  using Fn = cudnnStatus_t (*)(int, void**);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBackendCreateDescriptor"));
  if (!real) return 1;
  const cudnnStatus_t st = real(descriptorType, descriptor);
  if (st == 0 && descriptor && *descriptor) {
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    Shadow& s = g_shadow[*descriptor];
    s = Shadow();
    s.type = descriptorType;
  }
  return st;
}

cudnnStatus_t cudnnBackendSetAttribute(void* descriptor, int attributeName, int attributeType,
                                       int64_t elementCount, const void* arrayOfElements) {
  using Fn = cudnnStatus_t (*)(void*, int, int, int64_t, const void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBackendSetAttribute"));
  if (!real) return 1;
  const cudnnStatus_t st = real(descriptor, attributeName, attributeType, elementCount,
                                arrayOfElements);
  if (attributeName >= 0 && attributeName < 2048) g_set_calls[attributeName].fetch_add(1);
  if (st == 0) record_set(descriptor, attributeName, attributeType, elementCount, arrayOfElements);
  return st;
}

cudnnStatus_t cudnnBackendGetAttribute(void* descriptor, int attributeName, int attributeType,
                                       int64_t requestedElementCount, int64_t* elementCount,
                                       void* arrayOfElements) {
  using Fn = cudnnStatus_t (*)(void*, int, int, int64_t, int64_t*, void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBackendGetAttribute"));
  if (!real) return 1;
  const cudnnStatus_t st = real(descriptor, attributeName, attributeType, requestedElementCount,
                                elementCount, arrayOfElements);
  if (attributeName >= 0 && attributeName < 2048) g_get_calls[attributeName].fetch_add(1);
  if (st == 0 && attributeName == kAttrHeurResults && attributeType == kTypeBackendDesc &&
      arrayOfElements && elementCount) {
    // engine configs returned by heuristics belong to the heuristics' graph
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    const Shadow* heur = shadow_of(descriptor);
    BDesc graph = first_desc(heur, kAttrHeurGraph);
    std::shared_ptr<const PlanInfo> conv = heur ? heur->conv : nullptr;
    const int64_t n = std::min<int64_t>(*elementCount, requestedElementCount);
    BDesc* cfgs = static_cast<BDesc*>(arrayOfElements);
    if (graph) {
      for (int64_t i = 0; i < n; ++i) {
        Shadow& c = g_shadow[cfgs[i]];
        c.descs[kSynthCfgGraph] = {graph};
        c.conv = conv;
      }
    }
  }
  return st;
}

cudnnStatus_t cudnnBackendFinalize(void* descriptor) {
  using Fn = cudnnStatus_t (*)(void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBackendFinalize"));
  if (!real) return 1;
  const cudnnStatus_t st = real(descriptor);
  if (st != 0) return st;
  // Decode as early as possible: callers may destroy tensors once the
  // operation is finalized, and operations once the graph is.
  PlanInfo info;
  bool is_plan = false;
  {
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    auto it = g_shadow.find(descriptor);
    if (it != g_shadow.end()) {
      Shadow& sd = it->second;
      if (sd.type == kDescConvFwd || sd.type == kDescConvBwdData || sd.type == kDescConvBwdFilter) {
        sd.conv = std::make_shared<const PlanInfo>(decode_op(descriptor));
      } else if (sd.type == kDescOpGraph) {
        sd.conv = std::make_shared<const PlanInfo>(decode_graph(descriptor));
      } else if (sd.type == kDescPlan) {
        is_plan = true;
        info = decode_shadow(descriptor);
      }
    }
  }
  if (is_plan) note_plan(descriptor, info);
  return st;
}

cudnnStatus_t cudnnBackendExecute(void* handle, void* executionPlan, void* variantPack) {
  using Fn = cudnnStatus_t (*)(void*, void*, void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBackendExecute"));
  auto call_real = [&]() -> cudnnStatus_t {
    return real ? real(handle, executionPlan, variantPack) : 1;
  };
  if (orion::tl_is_scheduler_thread || orion::tl_in_scheduler_execution) return call_real();
  const cudaStream_t stream = cudnn_stream(handle);
  int client = -1;
  const Route r = route_for(handle, stream, &client);
  // with the op log on, decode anyway: submit_op logs the call, then runs it
  // on cuDNN (route "real")
  if (r == Route::kReal && !orion::op_log_enabled()) return call_real();
  const PlanInfo info = plan_info(executionPlan);
  void *px = nullptr, *pw = nullptr, *py = nullptr;
  const bool ok = info.ok && variant_pointers(variantPack, info, &px, &pw, &py);
  if (info.ok && !ok) LOG_WARN("cudnnBackendExecute: variant pack lacks the plan's tensor UIDs");
  CudnnConvParams p;
  std::memset(&p, 0, sizeof(p));
  p.handle = handle;
  p.stream = stream;
  p.geom = info.geom;
  p.alpha_value = info.alpha;
  p.beta_value = info.beta;
  // record fields follow the legacy wrappers' use (see dispatch.cpp)
  switch (info.type) {
    case OperationType::CUDNN_CONV_FWD:  // x, w -> y
      p.x = px;
      p.w = pw;
      p.y = py;
      break;
    case OperationType::CUDNN_CONV_BWD_DATA:  // w, dy -> dx: x = dy, y = dx
      p.x = py;
      p.w = pw;
      p.y = px;
      break;
    case OperationType::CUDNN_CONV_BWD_FILTER:  // x, dy -> dw: y = dy, w = dw
      p.x = px;
      p.y = py;
      p.w = pw;
      break;
    default:
      break;
  }
  return submit_op(ok ? info.type : orion::OperationType::CUDNN_CONV_FWD, handle, p, ok,
                   call_real);
}

cudnnStatus_t cudnnBackendDestroyDescriptor(void* descriptor) {
  using Fn = cudnnStatus_t (*)(void*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudnn("cudnnBackendDestroyDescriptor"));
  {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    g_plans.erase(descriptor);
  }
  {
    std::lock_guard<std::mutex> lk(g_shadow_mu);
    g_shadow.erase(descriptor);
  }
  return real ? real(descriptor) : 1;
}

}  // extern "C"
