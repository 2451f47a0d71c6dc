// dispatch.h — executes captured operations: dense ops on the kx kernels
// (libkx.so, include/kx.h), runtime ops on the real CUDA runtime.
#pragma once

#include <cuda_runtime_api.h>

#include "gpu_capture.h"
#include "kx.h"

namespace orion {

/** How one captured dense op is run. */
struct ExecPolicy {
    cudaStream_t stream = nullptr;      // op's own stream (client order)
    int sm_quota = 0;                   // 0 = all SMs
    const volatile int* yield_flag = nullptr;  // device view of the HP flag (BE ops)
    volatile int* done_flag = nullptr;         // device view of a per-worker done word
};

/** True for op types served by the kx kernels. */
bool is_dense_op(OperationType t);

/** Runs a captured dense op through the kx C ABI.  Returns the kx status. */
int dispatch_dense(OperationRecord& op, const ExecPolicy& pol);

/** Runs a captured runtime op (launch / memcpy / memset / malloc / free / sync)
 *  with the real CUDA runtime. */
cudaError_t dispatch_runtime(OperationRecord& op, cudaStream_t fallback);

/** Maps a kx status to a cudaError_t for the worker's error latch. */
cudaError_t kx_to_cuda(int status);

/** kx_exec for a policy. */
kx_exec make_kx_exec(const ExecPolicy& pol);

/** fp32 arithmetic used for captured fp32 ops (KX_FP32_MODE: 3xtf32 | ffma | tf32;
 *  default 3xtf32 — plain TF32 only when explicitly requested). */
int fp32_mode();

}  // namespace orion
