// cuda_intercept.cpp — exported CUDA runtime / driver entry points.
//
// Same symbols as the reference's src/cuda_intercept.cpp (cudaMalloc,
// cudaFree, cudaMemcpy(Async), cudaMemset(Async) 726-900, cudaLaunchKernel /
// __cudaLaunchKernel 920-985, cudaLaunchKernelExC 995-1039, cuLaunchKernel
// 1049-1109, cudaDeviceSynchronize / cudaStreamSynchronize 1120-1186,
// cudaStreamGetCaptureInfo_v2 / cudaStreamIsCapturing 1206-1243).  These ops
// are not replaced by kx kernels: they are captured so a client's work runs
// on the worker in its original order, and otherwise passed through.
//
// Differences from the reference:
//  * kernel arguments are deep-copied when the runtime can describe the
//    kernel's parameters (cudaFuncGetParamInfo / cuFuncGetParamInfo, layouts
//    cached per function), so a captured launch no longer has to block until
//    the worker issued it; launches the runtime cannot describe still wait;
//  * the capture-status queries are passed through unchanged (the reference
//    always answers "not capturing"; ORION_SPOOF_CAPTURE=1 restores that);
//  * dlsym is not interposed: a dlsym wrapper resolves RTLD_NEXT relative to
//    itself instead of its caller, and its only purpose in the reference was
//    to feed that capture-status answer to cuBLAS, whose math is no longer
//    called for captured ops.
#include <cuda.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <shared_mutex>
#include <unordered_map>
#include <vector>

#include "dispatch.h"
#include "gpu_capture.h"
#include "real_libs.h"
#include "scheduler.h"

namespace {

using namespace orion;

bool passthrough_thread() { return tl_is_scheduler_thread || tl_in_scheduler_execution; }

int capture_client(void* stream) {
  if (passthrough_thread() || !is_capture_enabled()) return -1;
  return resolve_client_idx(stream, nullptr);
}

// --------------------------------------------------- parameter layouts ----

struct ParamLayout {
  std::vector<size_t> off, size;
  size_t total = 0;
  bool known = false;
};

std::shared_mutex g_layout_mu;
std::unordered_map<const void*, ParamLayout> g_layouts;

const ParamLayout& layout_for(const void* func, bool driver) {
  {
    std::shared_lock<std::shared_mutex> lk(g_layout_mu);
    auto it = g_layouts.find(func);
    if (it != g_layouts.end()) return it->second;
  }
  ParamLayout L;
  if (!driver) {
    using Fn = cudaError_t (*)(const void*, size_t, size_t*, size_t*);
    static Fn fn = reinterpret_cast<Fn>(real::cudart("cudaFuncGetParamInfo"));
    if (fn) {
      L.known = true;
      for (size_t i = 0; i < MAX_KERNEL_ARGS_COUNT; ++i) {
        size_t o = 0, s = 0;
        if (fn(func, i, &o, &s) != cudaSuccess) break;
        L.off.push_back(o);
        L.size.push_back(s);
        L.total = std::max(L.total, o + s);
      }
      ORION_REAL(cudart, cudaGetLastError)();  // clear the out-of-range error
    }
  } else {
    using Fn = CUresult (*)(CUfunction, size_t, size_t*, size_t*);
    static Fn fn = reinterpret_cast<Fn>(real::cudadrv("cuFuncGetParamInfo"));
    if (fn) {
      L.known = true;
      for (size_t i = 0; i < MAX_KERNEL_ARGS_COUNT; ++i) {
        size_t o = 0, s = 0;
        if (fn(reinterpret_cast<CUfunction>(const_cast<void*>(func)), i, &o, &s) != CUDA_SUCCESS)
          break;
        L.off.push_back(o);
        L.size.push_back(s);
        L.total = std::max(L.total, o + s);
      }
    }
  }
  if (L.total > MAX_KERNEL_ARGS_SIZE) L.known = false;
  std::unique_lock<std::shared_mutex> lk(g_layout_mu);
  return g_layouts.emplace(func, std::move(L)).first->second;
}

// Copies the argument values into the record; false when not describable.
bool deep_copy_args(KernelLaunchParams& kp, void** args, const void* func, bool driver) {
  if (args == nullptr) return false;
  const ParamLayout& L = layout_for(func, driver);
  if (!L.known) return false;
  kp.num_args = L.off.size();
  kp.args_buffer.assign(L.total ? L.total : 1, 0);
  kp.args_offsets = L.off;
  kp.args_sizes = L.size;
  for (size_t i = 0; i < kp.num_args; ++i)
    std::memcpy(kp.args_buffer.data() + L.off[i], args[i], L.size[i]);
  kp.use_deep_copy = true;
  return true;
}

// A copy of a cudaLaunchConfig_t that outlives the caller's frame.
struct OwnedConfig {
  cudaLaunchConfig_t cfg;
  std::vector<cudaLaunchAttribute> attrs;
};

// Queues a captured runtime call.  must_wait: the record refers to memory of
// the calling thread (launch arguments on its stack, an out-pointer, a host
// buffer), so the call returns only once the worker ran it; otherwise, in
// async mode, at once.  A record whose arguments were copied is detachable: a
// timed-out client may stop waiting for it even while it runs.
cudaError_t run_captured(OperationPtr op, bool must_wait) {
  op->detachable = !must_wait;
  if (!enqueue_operation(op)) return cudaErrorTimeout;
  if (!must_wait && get_async_mode_internal() == 1) return cudaSuccess;
  return wait_operation(op);
}

}  // namespace

extern "C" {

cudaError_t cudaMalloc(void** devPtr, size_t size) {
  auto real = ORION_REAL(cudart, cudaMalloc);
  const int c = capture_client(nullptr);
  if (c < 0) return real(devPtr, size);
  auto op = create_operation(c, OperationType::MALLOC);
  if (!op) return real(devPtr, size);
  op->params = MallocParams{devPtr, size};
  return run_captured(op, true);
}

cudaError_t cudaFree(void* devPtr) {
  auto real = ORION_REAL(cudart, cudaFree);
  const int c = capture_client(nullptr);
  if (c < 0) return real(devPtr);
  auto op = create_operation(c, OperationType::FREE);
  if (!op) return real(devPtr);
  op->params = FreeParams{devPtr};
  return run_captured(op, true);
}

cudaError_t cudaMemcpy(void* dst, const void* src, size_t count, cudaMemcpyKind kind) {
  auto real = ORION_REAL(cudart, cudaMemcpy);
  const int c = capture_client(nullptr);
  if (c < 0) return real(dst, src, count, kind);
  auto op = create_operation(c, OperationType::MEMCPY);
  if (!op) return real(dst, src, count, kind);
  op->params = MemcpyParams{dst, src, count, kind, nullptr, false};
  return run_captured(op, true);
}

cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t count, cudaMemcpyKind kind,
                            cudaStream_t stream) {
  auto real = ORION_REAL(cudart, cudaMemcpyAsync);
  const int c = capture_client(stream);
  if (c < 0) return real(dst, src, count, kind, stream);
  auto op = create_operation(c, OperationType::MEMCPY_ASYNC);
  if (!op) return real(dst, src, count, kind, stream);
  op->params = MemcpyParams{dst, src, count, kind, stream, true};
  // host buffers may be pageable and reused at once: wait until issued
  return run_captured(op, true);
}

cudaError_t cudaMemset(void* devPtr, int value, size_t count) {
  auto real = ORION_REAL(cudart, cudaMemset);
  const int c = capture_client(nullptr);
  if (c < 0) return real(devPtr, value, count);
  auto op = create_operation(c, OperationType::MEMSET);
  if (!op) return real(devPtr, value, count);
  op->params = MemsetParams{devPtr, value, count, nullptr, false};
  return run_captured(op, true);
}

cudaError_t cudaMemsetAsync(void* devPtr, int value, size_t count, cudaStream_t stream) {
  auto real = ORION_REAL(cudart, cudaMemsetAsync);
  const int c = capture_client(stream);
  if (c < 0) return real(devPtr, value, count, stream);
  auto op = create_operation(c, OperationType::MEMSET_ASYNC);
  if (!op) return real(devPtr, value, count, stream);
  op->params = MemsetParams{devPtr, value, count, stream, true};
  return run_captured(op, false);
}

cudaError_t cudaLaunchKernel(const void* func, dim3 gridDim, dim3 blockDim, void** args,
                             size_t sharedMem, cudaStream_t stream) {
  auto real = ORION_REAL(cudart, cudaLaunchKernel);
  const int c = capture_client(stream);
  if (c < 0) return real(func, gridDim, blockDim, args, sharedMem, stream);
  auto op = create_operation(c, OperationType::KERNEL_LAUNCH);
  if (!op) return real(func, gridDim, blockDim, args, sharedMem, stream);
  KernelLaunchParams kp;
  kp.func = func;
  kp.gridDim = gridDim;
  kp.blockDim = blockDim;
  kp.sharedMem = sharedMem;
  kp.stream = stream;
  kp.original_args = args;
  const bool copied = deep_copy_args(kp, args, func, false);
  op->params = std::move(kp);
  return run_captured(op, !copied);
}

// Internal runtime symbol some libtorch builds call instead of cudaLaunchKernel.
cudaError_t __cudaLaunchKernel(const void* func, dim3 gridDim, dim3 blockDim, void** args,
                               size_t sharedMem, cudaStream_t stream) {
  return cudaLaunchKernel(func, gridDim, blockDim, args, sharedMem, stream);
}

cudaError_t cudaLaunchKernelExC(const cudaLaunchConfig_t* config, const void* func, void** args) {
  auto real = ORION_REAL(cudart, cudaLaunchKernelExC);
  const int c = config ? capture_client(config->stream) : -1;
  if (c < 0) return real(config, func, args);
  auto op = create_operation(c, OperationType::KERNEL_LAUNCH_EX);
  if (!op) return real(config, func, args);
  auto owned = std::make_shared<OwnedConfig>();
  owned->cfg = *config;
  if (config->attrs && config->numAttrs) {
    owned->attrs.assign(config->attrs, config->attrs + config->numAttrs);
    owned->cfg.attrs = owned->attrs.data();
  }
  KernelLaunchParams kp;
  kp.api = 1;
  kp.func = func;
  kp.gridDim = config->gridDim;
  kp.blockDim = config->blockDim;
  kp.sharedMem = config->dynamicSmemBytes;
  kp.stream = config->stream;
  kp.original_args = args;
  kp.ex_config = &owned->cfg;
  kp.ex_owned = owned;  // the config and its attributes live as long as the record
  const bool copied = deep_copy_args(kp, args, func, false);
  op->params = std::move(kp);
  return run_captured(op, !copied);
}

CUresult cuLaunchKernel(CUfunction f, unsigned int gridDimX, unsigned int gridDimY,
                        unsigned int gridDimZ, unsigned int blockDimX, unsigned int blockDimY,
                        unsigned int blockDimZ, unsigned int sharedMemBytes, CUstream hStream,
                        void** kernelParams, void** extra) {
  auto real = ORION_REAL(cudadrv, cuLaunchKernel);
  const int c = capture_client(reinterpret_cast<void*>(hStream));
  if (c < 0)
    return real(f, gridDimX, gridDimY, gridDimZ, blockDimX, blockDimY, blockDimZ, sharedMemBytes,
                hStream, kernelParams, extra);
  auto op = create_operation(c, OperationType::KERNEL_LAUNCH_DRV);
  if (!op)
    return real(f, gridDimX, gridDimY, gridDimZ, blockDimX, blockDimY, blockDimZ, sharedMemBytes,
                hStream, kernelParams, extra);
  KernelLaunchParams kp;
  kp.api = 2;
  kp.func = reinterpret_cast<const void*>(f);
  kp.gridDim = dim3(gridDimX, gridDimY, gridDimZ);
  kp.blockDim = dim3(blockDimX, blockDimY, blockDimZ);
  kp.sharedMem = sharedMemBytes;
  kp.stream = reinterpret_cast<cudaStream_t>(hStream);
  kp.original_args = kernelParams;
  kp.extra = extra;
  const bool copied = extra == nullptr && deep_copy_args(kp, kernelParams, kp.func, true);
  op->params = std::move(kp);
  cudaError_t r = run_captured(op, !copied);
  return r == cudaSuccess ? CUDA_SUCCESS : CUDA_ERROR_LAUNCH_FAILED;
}

cudaError_t cudaDeviceSynchronize(void) {
  auto real = ORION_REAL(cudart, cudaDeviceSynchronize);
  const int c = capture_client(nullptr);
  if (c < 0) return real();
  auto op = create_operation(c, OperationType::DEVICE_SYNC);
  if (!op) return real();
  op->params = SyncParams{nullptr, nullptr};
  cudaError_t r = run_captured(op, true);
  cudaError_t latched = get_and_clear_last_error(c);
  return latched != cudaSuccess ? latched : r;
}

cudaError_t cudaStreamSynchronize(cudaStream_t stream) {
  auto real = ORION_REAL(cudart, cudaStreamSynchronize);
  const int c = capture_client(stream);
  if (c < 0) return real(stream);
  auto op = create_operation(c, OperationType::STREAM_SYNC);
  if (!op) return real(stream);
  op->params = SyncParams{stream, nullptr};
  cudaError_t r = run_captured(op, true);
  cudaError_t latched = get_and_clear_last_error(c);
  return latched != cudaSuccess ? latched : r;
}

// Events and cross-stream waits issued by a client thread must keep their
// place among the client's captured ops (the worker issues those later), so
// under capture they are queued too; queries that would observe them first
// wait for the client's queue to drain.
cudaError_t cudaEventRecordWithFlags(cudaEvent_t event, cudaStream_t stream, unsigned int flags) {
  auto real = ORION_REAL(cudart, cudaEventRecordWithFlags);
  const int c = capture_client(stream);
  if (c < 0) return real(event, stream, flags);
  auto op = create_operation(c, OperationType::EVENT_RECORD);
  if (!op) return real(event, stream, flags);
  op->params = SyncParams{stream, event, flags};
  return run_captured(op, false);
}

cudaError_t cudaEventRecord(cudaEvent_t event, cudaStream_t stream) {
  return cudaEventRecordWithFlags(event, stream, 0);
}

cudaError_t cudaStreamWaitEvent(cudaStream_t stream, cudaEvent_t event, unsigned int flags) {
  auto real = ORION_REAL(cudart, cudaStreamWaitEvent);
  const int c = capture_client(stream);
  if (c < 0) return real(stream, event, flags);
  auto op = create_operation(c, OperationType::STREAM_WAIT_EVENT);
  if (!op) return real(stream, event, flags);
  op->params = SyncParams{stream, event, flags};
  return run_captured(op, false);
}

static void drain_own_queue() {
  const int c = capture_client(nullptr);
  if (c < 0) return;
  auto& q = g_capture_state.client_queues[c];
  const int64_t limit_us = wait_timeout_ns() / 1000;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(limit_us);
  while (q && !q->empty() && std::chrono::steady_clock::now() < deadline)
    std::this_thread::yield();  // a sleep would oversleep by the timer slack
}

cudaError_t cudaEventSynchronize(cudaEvent_t event) {
  drain_own_queue();
  return ORION_REAL(cudart, cudaEventSynchronize)(event);
}

cudaError_t cudaEventQuery(cudaEvent_t event) {
  const int c = capture_client(nullptr);
  if (c >= 0 && !g_capture_state.client_queues[c]->empty()) return cudaErrorNotReady;
  return ORION_REAL(cudart, cudaEventQuery)(event);
}

cudaError_t cudaStreamQuery(cudaStream_t stream) {
  const int c = capture_client(stream);
  if (c >= 0 && !g_capture_state.client_queues[c]->empty()) return cudaErrorNotReady;
  return ORION_REAL(cudart, cudaStreamQuery)(stream);
}

static bool spoof_capture() {
  static const bool s = [] {
    const char* v = std::getenv("ORION_SPOOF_CAPTURE");
    return v != nullptr && std::strcmp(v, "1") == 0;
  }();
  return s;
}

cudaError_t cudaStreamGetCaptureInfo_v2(cudaStream_t stream,
                                        cudaStreamCaptureStatus* captureStatus_out,
                                        unsigned long long* id_out, cudaGraph_t* graph_out,
                                        const cudaGraphNode_t** dependencies_out,
                                        size_t* numDependencies_out) {
  if (spoof_capture()) {
    if (captureStatus_out) *captureStatus_out = cudaStreamCaptureStatusNone;
    if (id_out) *id_out = 0;
    if (graph_out) *graph_out = nullptr;
    if (dependencies_out) *dependencies_out = nullptr;
    if (numDependencies_out) *numDependencies_out = 0;
    return cudaSuccess;
  }
  using Fn = cudaError_t (*)(cudaStream_t, cudaStreamCaptureStatus*, unsigned long long*,
                             cudaGraph_t*, const cudaGraphNode_t**, size_t*);
  static Fn real = reinterpret_cast<Fn>(orion::real::cudart("cudaStreamGetCaptureInfo_v2"));
  if (!real) return cudaErrorNotSupported;
  return real(stream, captureStatus_out, id_out, graph_out, dependencies_out, numDependencies_out);
}

cudaError_t cudaStreamIsCapturing(cudaStream_t stream, cudaStreamCaptureStatus* pCaptureStatus) {
  if (spoof_capture()) {
    if (pCaptureStatus) *pCaptureStatus = cudaStreamCaptureStatusNone;
    return cudaSuccess;
  }
  return ORION_REAL(cudart, cudaStreamIsCapturing)(stream, pCaptureStatus);
}

}  // extern "C"
