// kx_runtime.cuh — host-side runtime shared by the kx entry points:
// device properties, the per-stream work-slot pool used by persistent
// launches, tensor-map encoding through the driver entry point, and the
// execution-control defaults.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "kx.h"
#include "kx_gemm.cuh"

namespace kx {

struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int max_smem_optin = 0;
};

// Properties of the current device (cached per device).
const DeviceInfo& device_info();

// A WorkSlot reserved for `stream` on the current device.  Slots live in one
// device allocation per device (made on first use, zero-initialised) and are
// reused by every op enqueued on the same stream: a persistent launch resets
// its slot when it completes, and stream order serialises ops on one stream.
WorkSlot* work_slot_for(cudaStream_t stream);

// Scratch device memory reserved for `stream` on the current device, at least
// `bytes` long.  Growing it frees the previous buffer (cudaFree waits for the
// device), so ops on one stream may reuse it back to back; ops on different
// streams get different buffers.  The buffers of one device stay within a
// budget (KX_SCRATCH_BUDGET_MB, default a quarter of device memory, at most
// 24 GiB): a growing buffer first frees the buffers of streams that have not
// asked for theirs in the last second, oldest first; on an allocation
// failure every other stream's buffer idle for 100 ms is freed and the
// allocation retried.  Returns nullptr on allocation failure.
// Slot 0 serves the operator entry points (im2col buffers, batch-norm
// statistics); slot 1 is the GEMM's own split-K workspace and slot 2 holds
// the 3xTF32 low parts of its operands, so a GEMM issued by an operator never
// overwrites the operator's buffer.
void* scratch_for(cudaStream_t stream, size_t bytes, int slot = 0);

// KX_TMA_STORE=0 makes the tcgen05 epilogues store D with one st.global per
// element instead of staging it through shared memory for TMA stores.
inline bool tma_store_disabled() {
  static const bool off = [] {
    const char* s = std::getenv("KX_TMA_STORE");
    return s != nullptr && s[0] == '0';
  }();
  return off;
}

// 3xTF32 accumulator segment length in k-blocks (KX_SEG_KB, default 4 =
// 128 of K for tf32 k-blocks of 32): the tensor core's fp32 accumulation
// truncates, and the bias of one accumulator grows with its K length; it has
// the same sign in every layer of a network, so it compounds.  Measured on a
// VGG16 batch-32 forward through the interposer (max normwise error of the
// logits against a float64 forward): 1.20e-5 at 8, 8.06e-6 at 4, 6.28e-6 at
// 2; the 13 convolutions take 4.2 % longer at 4 than at 8 and 12 % at 2.
inline int seg_kb_default() {
  static const int v = [] {
    const char* s = std::getenv("KX_SEG_KB");
    const int x = s != nullptr ? std::atoi(s) : 4;
    return x >= 1 && x <= 64 ? x : 4;
  }();
  return v;
}

// KX_SPLITK=0 turns split-K off (every output tile then runs its whole K).
inline bool split_k_disabled() {
  static const bool off = [] {
    const char* s = std::getenv("KX_SPLITK");
    return s != nullptr && s[0] == '0';
  }();
  return off;
}

// Resolved execution controls.
struct Exec {
  cudaStream_t stream = nullptr;
  int sm_quota = 0;
  const volatile int* yield_flag = nullptr;
  volatile int* done_flag = nullptr;
  int max_tiles = 0;
  unsigned long long timeout_ns = 2000000000ull;
  int fp32_mode = KX_FP32_3XTF32;
  int* err_word = nullptr;
};

Exec resolve_exec(const kx_exec* ex);

// Grid size for a persistent launch with `tiles` work items.
int persistent_grid(const Exec& e, int tiles);

// Convolution problem in the form the implicit-GEMM kernel takes.
struct ConvShape {
  int N, C, H, W, K, R, S, ph, pw, sh, sw, dh, dw, P, Q;
  bool flip;  // CUDNN_CONVOLUTION (true convolution) rather than cross-correlation
  // the filter is stored [C][K][R][S] (the transpose of this convolution's
  // [K][C][R][S]): backward data run as a forward convolution of dy
  bool transposed = false;
};

// Forward convolution on the implicit-GEMM tcgen05 kernel (3xTF32):
// y = alpha * conv(x, w) + beta * y.  Returns KX_ERR_UNSUPPORTED when the
// shape is outside what the kernel addresses (the caller then lowers
// through im2col).  Defined in kx_conv_tc.cu.
int conv_fwd_implicit(const Exec& e, const ConvShape& g, const float* x, const float* w, float* y,
                      float alpha, float beta);

// Backward filter on the implicit-GEMM tcgen05 kernel (3xTF32):
// dw = alpha * dL/dw + beta * dw.  KX_ERR_UNSUPPORTED outside its reach
// (P*Q not a multiple of 4, fewer than 64 padded channels, ...): the caller
// then lowers through im2col.  Defined in kx_conv_tc.cu.
int conv_bwd_filter_implicit(const Exec& e, const ConvShape& g, const float* x, const float* dy,
                             float* dw, float alpha, float beta);


// cuTensorMapEncodeTiled through cudaGetDriverEntryPoint (no libcuda link).
// 3-D map {inner, outer, batch} with 128-byte swizzle.  Returns false when the
// driver rejects the geometry (caller falls back to the SIMT kernel).
bool encode_map_3d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t batch, uint64_t ld_elems,
                   uint64_t batch_stride_elems, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);

// Generic tiled map of rank 2..5 (dims/strides in elements / bytes as the
// driver expects), 128-byte swizzle, zero OOB fill.
// elem_strides (nullable): traversal stride per dimension (a box of b
// elements with stride t loads b / t of them).
bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B,
                const uint32_t* elem_strides = nullptr);

// im2col map of a 4-D NHWC tensor {C, W, H, N} (dims in elements, strides in
// bytes) for cp.async.bulk.tensor ... .im2col: each load brings `pixels`
// consecutive filter-window positions x `channels` channels.  lower / upper:
// bounding-box corner offsets {w, h} (lower = -pad, upper = pad - dil*(taps-1)),
// each within [-128, 127]; elem_strides {1, stride_w, stride_h, 1}.  128-byte
// swizzle, zero OOB fill.  Returns false when the driver rejects the geometry.
bool encode_im2col_map(CUtensorMap* map, const void* base, const uint64_t* dims,
                       const uint64_t* strides_bytes, const int* lower, const int* upper,
                       uint32_t channels, uint32_t pixels, const uint32_t* elem_strides,
                       CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B);

void set_last_kernel_name(const char* name);

// KX_SINGLE_BOX=0: M/N-major GEMM tiles as one TMA load per 128-byte chunk.
bool single_box_disabled();

// Pipeline diagnostics of the tcgen05 kernels (KX_PIPE_STATS=1): a zeroed
// device buffer for GemmParams::pipe_stats (nullptr when off), and a report of
// the per-role wait fractions to stderr after the launch (synchronises).
unsigned long long* pipe_stats_begin();
void pipe_stats_end(unsigned long long* buf, const char* kernel, cudaStream_t stream, int grid);

// Counts one kernel launch of this library (process-wide, read back by
// kx_launch_count).  Every `<<<...>>>` site calls it just before launching.
void note_launch();

// Counts one device-memory allocation or free by this library (cudaMalloc /
// cudaFree of scratch, work slots and diagnostics), read back by
// kx_device_alloc_count.  Every cudaMalloc / cudaFree site calls it.
void note_device_alloc();

// Records the CUDA error behind a KX_ERR_DEVICE status of this thread's last
// call (read back by kx_last_cuda_error).
void note_cuda_error(cudaError_t e);

// Status mapping helper.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return KX_OK;
  note_cuda_error(e);
  return KX_ERR_DEVICE;
}

// KX_ERR_DEVICE for a failed runtime call, with its error recorded.
inline int device_error(cudaError_t e) {
  note_cuda_error(e);
  return KX_ERR_DEVICE;
}

}  // namespace kx
