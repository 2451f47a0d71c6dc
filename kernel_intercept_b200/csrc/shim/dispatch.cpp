// dispatch.cpp — runs captured operations: dense ops through the kx C ABI,
// runtime ops through the real CUDA runtime (see dispatch.h).
#include "dispatch.h"

#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "real_libs.h"

namespace orion {

int fp32_mode() {
  static const int mode = [] {
    const char* s = std::getenv("KX_FP32_MODE");
    if (s == nullptr) return static_cast<int>(KX_FP32_3XTF32);
    if (std::strcmp(s, "ffma") == 0) return static_cast<int>(KX_FP32_FFMA);
    if (std::strcmp(s, "tf32") == 0) return static_cast<int>(KX_FP32_TF32);
    return static_cast<int>(KX_FP32_3XTF32);
  }();
  return mode;
}

kx_exec make_kx_exec(const ExecPolicy& pol) {
  kx_exec e;
  std::memset(&e, 0, sizeof(e));
  e.stream = pol.stream;
  e.sm_quota = pol.sm_quota;
  e.yield_flag = pol.yield_flag;
  e.done_flag = pol.done_flag;
  e.fp32_mode = fp32_mode();
  return e;
}

bool is_dense_op(OperationType t) {
  switch (t) {
    case OperationType::CUBLAS_SGEMM:
    case OperationType::CUBLAS_SGEMM_BATCHED:
    case OperationType::CUBLAS_SGEMM_STRIDED_BATCHED:
    case OperationType::CUBLASLT_MATMUL:
    case OperationType::CUBLAS_GEMM_EX:
    case OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX:
    case OperationType::CUDNN_CONV_FWD:
    case OperationType::CUDNN_CONV_BWD_DATA:
    case OperationType::CUDNN_CONV_BWD_FILTER:
    case OperationType::CUDNN_BATCHNORM_FWD:
    case OperationType::CUDNN_BATCHNORM_BWD:
    case OperationType::CUDNN_BATCHNORM_INF:
      return true;
    default:
      return false;
  }
}

cudaError_t kx_to_cuda(int status) {
  switch (status) {
    case KX_OK: return cudaSuccess;
    case KX_ERR_INVALID: return cudaErrorInvalidValue;
    case KX_ERR_UNSUPPORTED: return cudaErrorNotSupported;
    case KX_ERR_TIMEOUT: return cudaErrorTimeout;
    case KX_ERR_NOMEM: return cudaErrorMemoryAllocation;
    default: return cudaErrorLaunchFailure;
  }
}

static kx_conv_desc to_kx(const ConvGeometry& g) {
  kx_conv_desc d;
  d.n = g.n; d.c = g.c; d.h = g.h; d.w = g.w;
  d.k = g.k; d.r = g.r; d.s = g.s;
  d.pad_h = g.pad_h; d.pad_w = g.pad_w;
  d.stride_h = g.stride_h; d.stride_w = g.stride_w;
  d.dil_h = g.dil_h; d.dil_w = g.dil_w;
  d.cross_correlation = g.cross_correlation;
  return d;
}

int dispatch_dense(OperationRecord& op, const ExecPolicy& pol) {
  kx_exec ex = make_kx_exec(pol);
  switch (op.type) {
    case OperationType::CUBLAS_SGEMM:
    case OperationType::CUBLAS_SGEMM_STRIDED_BATCHED:
    case OperationType::CUBLAS_SGEMM_BATCHED:
    case OperationType::CUBLAS_GEMM_EX:
    case OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX: {
      auto& p = std::get<CublasGemmParams>(op.params);
      ex.scalars_on_device = p.scalars_on_device ? 1 : 0;
      const float* al = p.use_stored_scalars ? &p.alpha_value : static_cast<const float*>(p.alpha);
      const float* be = p.use_stored_scalars ? &p.beta_value : static_cast<const float*>(p.beta);
      switch (op.type) {
        case OperationType::CUBLAS_SGEMM:
          return kx_sgemm(&ex, p.transa, p.transb, p.m, p.n, p.k, al,
                          static_cast<const float*>(p.A), p.lda, static_cast<const float*>(p.B),
                          p.ldb, be, static_cast<float*>(p.C), p.ldc);
        case OperationType::CUBLAS_SGEMM_STRIDED_BATCHED:
          return kx_sgemm_strided_batched(&ex, p.transa, p.transb, p.m, p.n, p.k, al,
                                          static_cast<const float*>(p.A), p.lda, p.strideA,
                                          static_cast<const float*>(p.B), p.ldb, p.strideB, be,
                                          static_cast<float*>(p.C), p.ldc, p.strideC,
                                          p.batchCount);
        case OperationType::CUBLAS_SGEMM_BATCHED:
          return kx_sgemm_batched(&ex, p.transa, p.transb, p.m, p.n, p.k, al,
                                  static_cast<const float* const*>(p.A), p.lda,
                                  static_cast<const float* const*>(p.B), p.ldb, be,
                                  static_cast<float* const*>(p.C), p.ldc, p.batchCount);
        case OperationType::CUBLAS_GEMM_EX:
          return kx_gemm_ex(&ex, p.transa, p.transb, p.m, p.n, p.k, al, p.A, p.Atype, p.lda, p.B,
                            p.Btype, p.ldb, be, p.C, p.Ctype, p.ldc);
        default:
          return kx_gemm_strided_batched_ex(&ex, p.transa, p.transb, p.m, p.n, p.k, al, p.A,
                                            p.Atype, p.lda, p.strideA, p.B, p.Btype, p.ldb,
                                            p.strideB, be, p.C, p.Ctype, p.ldc, p.strideC,
                                            p.batchCount);
      }
    }
    case OperationType::CUBLASLT_MATMUL: {
      auto& p = std::get<CublasLtMatmulParams>(op.params);
      const LtDecoded& d = p.dec;
      ex.scalars_on_device = d.scalars_on_device ? 1 : 0;
      const float* al = p.use_stored_scalars ? &p.alpha_value : static_cast<const float*>(p.alpha);
      const float* be = p.use_stored_scalars ? &p.beta_value : static_cast<const float*>(p.beta);
      return kx_matmul(&ex, d.transa, d.transb, d.m, d.n, d.k, al, p.A, d.Atype,
                       static_cast<int>(d.lda), d.strideA, p.B, d.Btype, static_cast<int>(d.ldb),
                       d.strideB, be, p.C, d.Ctype, static_cast<int>(d.ldc), d.strideC, p.D,
                       d.Dtype, static_cast<int>(d.ldd), d.strideD, d.batch, d.epilogue, d.bias,
                       d.bias_type);
    }
    case OperationType::CUDNN_CONV_FWD: {
      auto& p = std::get<CudnnConvParams>(op.params);
      kx_conv_desc d = to_kx(p.geom);
      return kx_conv_fwd(&ex, &d, &p.alpha_value, static_cast<const float*>(p.x),
                         static_cast<const float*>(p.w), &p.beta_value, static_cast<float*>(p.y));
    }
    case OperationType::CUDNN_CONV_BWD_DATA: {
      // field use follows the reference's wrapper: x = dy, w = w, y = dx
      auto& p = std::get<CudnnConvParams>(op.params);
      kx_conv_desc d = to_kx(p.geom);
      return kx_conv_bwd_data(&ex, &d, &p.alpha_value, static_cast<const float*>(p.w),
                              static_cast<const float*>(p.x), &p.beta_value,
                              static_cast<float*>(p.y));
    }
    case OperationType::CUDNN_CONV_BWD_FILTER: {
      // x = x, y = dy, w = dw
      auto& p = std::get<CudnnConvParams>(op.params);
      kx_conv_desc d = to_kx(p.geom);
      return kx_conv_bwd_filter(&ex, &d, &p.alpha_value, static_cast<const float*>(p.x),
                                static_cast<const float*>(p.y), &p.beta_value,
                                static_cast<float*>(const_cast<void*>(p.w)));
    }
    case OperationType::CUDNN_BATCHNORM_FWD: {
      auto& p = std::get<CudnnBatchNormParams>(op.params);
      return kx_bn_fwd_training(&ex, p.mode, &p.alpha_value, &p.beta_value, p.n, p.c, p.h, p.w,
                                static_cast<const float*>(p.x), static_cast<float*>(p.y),
                                static_cast<const float*>(p.bnScale),
                                static_cast<const float*>(p.bnBias), p.exponentialAverageFactor,
                                static_cast<float*>(p.resultRunningMean),
                                static_cast<float*>(p.resultRunningVariance), p.epsilon,
                                static_cast<float*>(p.resultSaveMean),
                                static_cast<float*>(p.resultSaveInvVariance));
    }
    case OperationType::CUDNN_BATCHNORM_INF: {
      auto& p = std::get<CudnnBatchNormParams>(op.params);
      return kx_bn_fwd_inference(&ex, p.mode, &p.alpha_value, &p.beta_value, p.n, p.c, p.h, p.w,
                                 static_cast<const float*>(p.x), static_cast<float*>(p.y),
                                 static_cast<const float*>(p.bnScale),
                                 static_cast<const float*>(p.bnBias),
                                 static_cast<const float*>(p.estimatedMean),
                                 static_cast<const float*>(p.estimatedVariance), p.epsilon);
    }
    case OperationType::CUDNN_BATCHNORM_BWD: {
      auto& p = std::get<CudnnBatchNormParams>(op.params);
      return kx_bn_bwd(&ex, p.mode, &p.alpha_value, &p.beta_value, &p.alpha_param, &p.beta_param,
                       p.n, p.c, p.h, p.w, static_cast<const float*>(p.x),
                       static_cast<const float*>(p.dy), static_cast<float*>(p.dx),
                       static_cast<const float*>(p.bnScale),
                       static_cast<float*>(p.dBnScaleResult), static_cast<float*>(p.dBnBiasResult),
                       p.epsilon, static_cast<const float*>(p.resultSaveMean),
                       static_cast<const float*>(p.resultSaveInvVariance));
    }
    default:
      return KX_ERR_UNSUPPORTED;
  }
}

cudaError_t dispatch_runtime(OperationRecord& op, cudaStream_t fallback) {
  switch (op.type) {
    case OperationType::KERNEL_LAUNCH: {
      auto& p = std::get<KernelLaunchParams>(op.params);
      cudaStream_t st = p.stream ? p.stream : fallback;
      if (p.api == 1) {
        cudaLaunchConfig_t cfg = *static_cast<const cudaLaunchConfig_t*>(p.ex_config);
        cfg.stream = st;
        return ORION_REAL(cudart, cudaLaunchKernelExC)(&cfg, p.func, p.get_args());
      }
      return ORION_REAL(cudart, cudaLaunchKernel)(p.func, p.gridDim, p.blockDim, p.get_args(),
                                                  p.sharedMem, st);
    }
    case OperationType::KERNEL_LAUNCH_EX: {
      auto& p = std::get<KernelLaunchParams>(op.params);
      cudaLaunchConfig_t cfg = *static_cast<const cudaLaunchConfig_t*>(p.ex_config);
      if (cfg.stream == nullptr) cfg.stream = fallback;
      return ORION_REAL(cudart, cudaLaunchKernelExC)(&cfg, p.func, p.get_args());
    }
    case OperationType::KERNEL_LAUNCH_DRV: {
      auto& p = std::get<KernelLaunchParams>(op.params);
      CUresult r = ORION_REAL(cudadrv, cuLaunchKernel)(
          reinterpret_cast<CUfunction>(const_cast<void*>(p.func)), p.gridDim.x, p.gridDim.y,
          p.gridDim.z, p.blockDim.x, p.blockDim.y, p.blockDim.z,
          static_cast<unsigned int>(p.sharedMem), reinterpret_cast<CUstream>(p.stream),
          p.get_args(), p.extra);
      return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorLaunchFailure;
    }
    case OperationType::MALLOC: {
      auto& p = std::get<MallocParams>(op.params);
      return ORION_REAL(cudart, cudaMalloc)(p.devPtr, p.size);
    }
    case OperationType::FREE: {
      auto& p = std::get<FreeParams>(op.params);
      return ORION_REAL(cudart, cudaFree)(p.devPtr);
    }
    case OperationType::MEMCPY: {
      auto& p = std::get<MemcpyParams>(op.params);
      return ORION_REAL(cudart, cudaMemcpy)(p.dst, p.src, p.count, p.kind);
    }
    case OperationType::MEMCPY_ASYNC: {
      auto& p = std::get<MemcpyParams>(op.params);
      return ORION_REAL(cudart, cudaMemcpyAsync)(p.dst, p.src, p.count, p.kind,
                                                 p.stream ? p.stream : fallback);
    }
    case OperationType::MEMSET: {
      auto& p = std::get<MemsetParams>(op.params);
      return ORION_REAL(cudart, cudaMemset)(p.devPtr, p.value, p.count);
    }
    case OperationType::MEMSET_ASYNC: {
      auto& p = std::get<MemsetParams>(op.params);
      return ORION_REAL(cudart, cudaMemsetAsync)(p.devPtr, p.value, p.count,
                                                 p.stream ? p.stream : fallback);
    }
    case OperationType::DEVICE_SYNC:
      return ORION_REAL(cudart, cudaDeviceSynchronize)();
    case OperationType::STREAM_SYNC: {
      auto& p = std::get<SyncParams>(op.params);
      return ORION_REAL(cudart, cudaStreamSynchronize)(p.stream);
    }
    case OperationType::EVENT_RECORD: {
      auto& p = std::get<SyncParams>(op.params);
      return ORION_REAL(cudart, cudaEventRecordWithFlags)(p.event, p.stream, p.flags);
    }
    case OperationType::STREAM_WAIT_EVENT: {
      auto& p = std::get<SyncParams>(op.params);
      return ORION_REAL(cudart, cudaStreamWaitEvent)(p.stream, p.event, p.flags);
    }
    default:
      return cudaErrorNotSupported;
  }
}

}  // namespace orion
