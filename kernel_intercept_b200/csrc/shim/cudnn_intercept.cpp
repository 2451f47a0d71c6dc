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
#include <cstdlib>
#include <cstring>
#include <mutex>
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
  int64_t waited = 0;
  while (q && !q->empty() && waited < limit) {
    std::this_thread::sleep_for(std::chrono::microseconds(2));
    waited += 2;
  }
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

template <class Params, class RealFn>
cudnnStatus_t submit_op(OperationType type, void* handle, Params p, bool supported, RealFn real) {
  int client = -1;
  const Route r = route_for(handle, p.stream, &client);
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
    ExecPolicy pol;
    pol.stream = p.stream;
    return dispatch_dense(op, pol) == KX_OK ? kOk : kExecFailed;
  }
  auto op = create_operation(client, type);
  if (!op) return real();
  op->params = p;  // filled before the worker can see it
  enqueue_operation(op);
  if (get_async_mode_internal() == 1) return kOk;
  wait_operation(op);
  return op->result == cudaSuccess ? kOk : kExecFailed;
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
// finalizes an execution plan for a one-operation graph and calls
// cudnnBackendExecute(handle, plan, variantPack).  The plan is decoded with
// cuDNN's public getters (plan -> engine config -> engine -> operation graph
// -> convolution operation -> X/W/Y tensors + convolution descriptor) and
// cached per plan (cudnnBackendDestroyDescriptor evicts).  Data pointers come
// from the variant pack by tensor UID.  Anything that does not decode to a
// single packed-NCHW fp32 2-D convolution runs on the real cuDNN.

namespace {

using BDesc = void*;
using GetAttr = int (*)(BDesc, int, int, int64_t, int64_t*, void*);
using CreateDesc = int (*)(int, BDesc*);
using DestroyDesc = int (*)(BDesc);

constexpr int kTypeDataType = 1, kTypeInt64 = 3, kTypeFloat = 4, kTypeDouble = 5,
              kTypeVoidPtr = 6, kTypeConvMode = 7, kTypeBackendDesc = 15;
constexpr int kDescConvolution = 1, kDescEngine = 2, kDescEngineCfg = 3,
              kDescConvFwd = 10, kDescConvBwdFilter = 11, kDescConvBwdData = 12,
              kDescOpGraph = 15, kDescTensor = 17;

struct Getters {
  GetAttr get = reinterpret_cast<GetAttr>(real::cudnn("cudnnBackendGetAttribute"));
  CreateDesc create = reinterpret_cast<CreateDesc>(real::cudnn("cudnnBackendCreateDescriptor"));
  DestroyDesc destroy = reinterpret_cast<DestroyDesc>(real::cudnn("cudnnBackendDestroyDescriptor"));
  bool ok() const { return get && create && destroy; }
};

const Getters& getters() {
  static Getters g;
  return g;
}

// RAII for descriptors created to receive attribute copies.
struct Owned {
  BDesc d = nullptr;
  explicit Owned(int type) { getters().create(type, &d); }
  ~Owned() {
    if (d) getters().destroy(d);
  }
};

bool get_desc_attr(BDesc from, int attr, BDesc into) {
  int64_t n = 0;
  return into && getters().get(from, attr, kTypeBackendDesc, 1, &n, &into) == 0 && n == 1;
}

struct TensorInfo {
  int64_t uid = -1;
  int64_t dims[8] = {0};
  int64_t strides[8] = {0};
  int64_t nd = 0;
  int dtype = -1;
};

bool read_backend_tensor(BDesc t, TensorInfo& ti) {
  const Getters& g = getters();
  int64_t n = 0;
  if (g.get(t, 906, kTypeInt64, 1, &n, &ti.uid) != 0) return false;
  if (g.get(t, 902, kTypeInt64, 8, &ti.nd, ti.dims) != 0) return false;
  int64_t ns = 0;
  if (g.get(t, 903, kTypeInt64, 8, &ns, ti.strides) != 0 || ns != ti.nd) return false;
  g.get(t, 901, kTypeDataType, 1, &n, &ti.dtype);
  return ti.nd == 4;
}

bool packed_nchw(const TensorInfo& t) {
  return t.strides[3] == 1 && t.strides[2] == t.dims[3] && t.strides[1] == t.dims[2] * t.dims[3] &&
         t.strides[0] == t.dims[1] * t.dims[2] * t.dims[3];
}

// Decoded plan: which convolution, geometry, the three UIDs and the scalars.
struct PlanInfo {
  bool ok = false;
  OperationType type = OperationType::UNKNOWN;
  ConvGeometry geom;
  int64_t uid_x = -1, uid_w = -1, uid_y = -1;  // forward roles: x (input), w, y (output)
  float alpha = 1.f, beta = 0.f;
};

float read_scalar(BDesc op, int attr, float dflt) {
  const Getters& g = getters();
  int64_t n = 0;
  float f = 0.f;
  if (g.get(op, attr, kTypeFloat, 1, &n, &f) == 0 && n == 1) return f;
  double d = 0.0;
  if (g.get(op, attr, kTypeDouble, 1, &n, &d) == 0 && n == 1) return static_cast<float>(d);
  return dflt;
}

PlanInfo decode_plan(BDesc plan) {
  PlanInfo info;
  const Getters& g = getters();
  if (!g.ok()) return info;
  Owned cfg(kDescEngineCfg), eng(kDescEngine), graph(kDescOpGraph);
  if (!get_desc_attr(plan, 401, cfg.d) || !get_desc_attr(cfg.d, 300, eng.d) ||
      !get_desc_attr(eng.d, 1300, graph.d))
    return info;
  int64_t nops = 0;
  // one-operation graphs only; try each convolution flavour for the op's type
  const struct { int desc; OperationType t; int x, w, y, conv, alpha, beta; } kinds[] = {
      {kDescConvFwd, OperationType::CUDNN_CONV_FWD, 704, 703, 705, 702, 700, 701},
      {kDescConvBwdData, OperationType::CUDNN_CONV_BWD_DATA, 710, 709, 711, 708, 706, 707},
      {kDescConvBwdFilter, OperationType::CUDNN_CONV_BWD_FILTER, 716, 715, 717, 714, 712, 713},
  };
  for (const auto& k : kinds) {
    Owned op(k.desc);
    BDesc arr[1] = {op.d};
    if (g.get(graph.d, 801, kTypeBackendDesc, 1, &nops, arr) != 0 || nops != 1) continue;
    Owned tx(kDescTensor), tw(kDescTensor), ty(kDescTensor), cd(kDescConvolution);
    if (!get_desc_attr(op.d, k.x, tx.d) || !get_desc_attr(op.d, k.w, tw.d) ||
        !get_desc_attr(op.d, k.y, ty.d) || !get_desc_attr(op.d, k.conv, cd.d))
      continue;
    // For bwd-data the attributes are (dx, w, dy); for bwd-filter (x, dw, dy):
    // map them to the forward roles input / filter / output.
    TensorInfo a, b, c;
    if (!read_backend_tensor(tx.d, a) || !read_backend_tensor(tw.d, b) ||
        !read_backend_tensor(ty.d, c))
      return info;
    TensorInfo in = a, filt = b, out = c;
    if (k.t == OperationType::CUDNN_CONV_BWD_FILTER) {  // (x, dw, dy): a = x, b = dw, c = dy
      in = a;
      filt = b;
      out = c;
    }
    int64_t n = 0, sd = 0;
    int64_t pre[4] = {0}, post[4] = {0}, dil[4] = {0}, str[4] = {0};
    int mode = 1, ctype = -1;
    if (g.get(cd.d, 106, kTypeInt64, 1, &n, &sd) != 0 || sd != 2) return info;
    if (g.get(cd.d, 105, kTypeInt64, 4, &n, pre) != 0 || n != 2) return info;
    if (g.get(cd.d, 104, kTypeInt64, 4, &n, post) != 0 || n != 2) return info;
    if (g.get(cd.d, 102, kTypeInt64, 4, &n, dil) != 0 || n != 2) return info;
    if (g.get(cd.d, 103, kTypeInt64, 4, &n, str) != 0 || n != 2) return info;
    g.get(cd.d, 101, kTypeConvMode, 1, &n, &mode);
    g.get(cd.d, 100, kTypeDataType, 1, &n, &ctype);
    ConvGeometry& G = info.geom;
    std::memset(&G, 0, sizeof(G));
    G.n = static_cast<int>(in.dims[0]);
    G.c = static_cast<int>(in.dims[1]);
    G.h = static_cast<int>(in.dims[2]);
    G.w = static_cast<int>(in.dims[3]);
    G.k = static_cast<int>(filt.dims[0]);
    G.r = static_cast<int>(filt.dims[2]);
    G.s = static_cast<int>(filt.dims[3]);
    G.pad_h = static_cast<int>(pre[0]);
    G.pad_w = static_cast<int>(pre[1]);
    G.stride_h = static_cast<int>(str[0]);
    G.stride_w = static_cast<int>(str[1]);
    G.dil_h = static_cast<int>(dil[0]);
    G.dil_w = static_cast<int>(dil[1]);
    G.cross_correlation = mode == 1 ? 1 : 0;
    G.data_type = in.dtype;
    const bool geom_ok =
        pre[0] == post[0] && pre[1] == post[1] && filt.dims[1] == in.dims[1] &&
        out.dims[0] == in.dims[0] && out.dims[1] == filt.dims[0] && in.dtype == 0 &&
        filt.dtype == 0 && out.dtype == 0 && (ctype == 0 || ctype == -1) && packed_nchw(in) &&
        packed_nchw(filt) && packed_nchw(out) && G.stride_h > 0 && G.stride_w > 0;
    if (!geom_ok) return info;
    G.packed_nchw = 1;
    info.type = k.t;
    info.uid_x = in.uid;
    info.uid_w = filt.uid;
    info.uid_y = out.uid;
    info.alpha = read_scalar(op.d, k.alpha, 1.f);
    info.beta = read_scalar(op.d, k.beta, 0.f);
    info.ok = true;
    return info;
  }
  return info;
}

std::mutex g_plan_mu;
std::unordered_map<BDesc, PlanInfo> g_plans;

PlanInfo plan_info(BDesc plan) {
  {
    std::lock_guard<std::mutex> lk(g_plan_mu);
    auto it = g_plans.find(plan);
    if (it != g_plans.end()) return it->second;
  }
  PlanInfo info = decode_plan(plan);
  std::lock_guard<std::mutex> lk(g_plan_mu);
  g_plans[plan] = info;
  return info;
}

bool variant_pointers(BDesc vp, const PlanInfo& info, void** px, void** pw, void** py) {
  const Getters& g = getters();
  int64_t uids[16], n = 0, np = 0;
  void* ptrs[16];
  if (g.get(vp, 1000, kTypeInt64, 16, &n, uids) != 0) return false;
  if (g.get(vp, 1001, kTypeVoidPtr, 16, &np, ptrs) != 0 || np != n) return false;
  *px = *pw = *py = nullptr;
  for (int64_t i = 0; i < n; ++i) {
    if (uids[i] == info.uid_x) *px = ptrs[i];
    if (uids[i] == info.uid_w) *pw = ptrs[i];
    if (uids[i] == info.uid_y) *py = ptrs[i];
  }
  return *px && *pw && *py;
}

}  // namespace

extern "C" {

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
  if (r == Route::kReal) return call_real();
  const PlanInfo info = plan_info(executionPlan);
  void *px = nullptr, *pw = nullptr, *py = nullptr;
  const bool ok = info.ok && variant_pointers(variantPack, info, &px, &pw, &py);
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
  return real ? real(descriptor) : 1;
}

}  // extern "C"
