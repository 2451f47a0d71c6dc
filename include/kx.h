/*
 * kx.h — C ABI of the B200 (sm_100a) dense-operator kernels behind the
 * interposer (libgpu_scheduler.so).  These are the functions the captured
 * cuBLAS / cuBLASLt / cuDNN calls are dispatched to instead of the closed
 * libraries.  Plain pointers, sizes and ints only; no torch or CUDA types in
 * the signatures (streams are `void*` holding a cudaStream_t).
 *
 * Reference interfaces each entry point replaces (paths within the
 * kernel_intercept project):
 *   kx_sgemm                      <- cublasSgemm_v2 wrapper, src/cublas_intercept.cpp:576-683,
 *                                    executed at src/cublas_intercept.cpp:455-471
 *   kx_sgemm_strided_batched      <- cublasSgemmStridedBatched, src/cublas_intercept.cpp:763-879,
 *                                    executed at src/cublas_intercept.cpp:474-491
 *   kx_sgemm_batched              <- cublasSgemmBatched, src/cublas_intercept.cpp:691-755
 *   kx_gemm_ex                    <- cublasGemmEx / cublasSgemmEx / cublasHgemm,
 *                                    src/cublas_intercept.cpp:886-952, 1036-1235
 *   kx_gemm_strided_batched_ex    <- cublasGemmStridedBatchedEx / cublasHgemmStridedBatched,
 *                                    src/cublas_intercept.cpp:959-1029, 1100-1166
 *   kx_matmul                     <- cublasLtMatmul, src/cublas_intercept.cpp:1319-1443,
 *                                    executed at src/cublas_intercept.cpp:1453-1500
 *   kx_conv_fwd                   <- cudnnConvolutionForward, src/cudnn_intercept.cpp:433-489
 *   kx_conv_bwd_data              <- cudnnConvolutionBackwardData, src/cudnn_intercept.cpp:512-558
 *   kx_conv_bwd_filter            <- cudnnConvolutionBackwardFilter, src/cudnn_intercept.cpp:581-627
 *   kx_bn_fwd_training            <- cudnnBatchNormalizationForwardTraining, src/cudnn_intercept.cpp:659-716
 *   kx_bn_fwd_inference           <- cudnnBatchNormalizationForwardInference (declared at
 *                                    src/cudnn_intercept.cpp:125-129)
 *   kx_bn_bwd                     <- cudnnBatchNormalizationBackward (declared at
 *                                    src/cudnn_intercept.cpp:138-143)
 *
 * Status: every entry point returns a kx_status.  The interposer maps it to
 * the library's own status type (cuBLAS: 0 ok, 1 failure, 6 internal error;
 * cuDNN: 0 ok, 1 failure), matching src/cublas_intercept.cpp:288-295,682 and
 * src/cudnn_intercept.cpp:239-246,488.
 *
 * Layout conventions follow the libraries they replace: GEMMs are
 * column-major (C is m x n with leading dimension ldc; op(A) is m x k;
 * op(B) is k x n), convolutions and batch norm are NCHW / KCRS fp32.
 */
#ifndef KX_H
#define KX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum kx_status {
    KX_OK = 0,
    KX_ERR_INVALID = 1,     /* bad argument (negative size, bad ld, null pointer) */
    KX_ERR_UNSUPPORTED = 2, /* type / mode combination not implemented */
    KX_ERR_TIMEOUT = 3,     /* a bounded device-side wait gave up */
    KX_ERR_DEVICE = 4,      /* CUDA runtime error at launch */
    KX_ERR_NOMEM = 5,       /* scratch allocation failed */
    KX_YIELDED = 6          /* best-effort op stopped at a tile boundary; relaunch to continue */
} kx_status;

/* cuBLAS operation codes (cublasOperation_t values). */
enum { KX_OP_N = 0, KX_OP_T = 1, KX_OP_C = 2 };

/* cudaDataType_t values accepted by the *_ex entry points. */
enum { KX_R_32F = 0, KX_R_16F = 2, KX_R_16BF = 14 };

/* fp32 arithmetic used by fp32 GEMMs / convolutions. */
enum {
    KX_FP32_3XTF32 = 0,  /* hi/lo split on the TF32 tensor path, ~fp32 accuracy (default) */
    KX_FP32_TF32 = 1,    /* single TF32 pass (what cuBLAS does under TF32 tensor-op math) */
    KX_FP32_FFMA = 2     /* CUDA-core FFMA (no tensor cores) */
};

/* cublasLt epilogues understood by kx_matmul (cublasLtEpilogue_t values). */
enum {
    KX_EPI_DEFAULT = 1,
    KX_EPI_RELU = 2,
    KX_EPI_BIAS = 4,
    KX_EPI_RELU_BIAS = 6,
    KX_EPI_GELU = 32,
    KX_EPI_GELU_BIAS = 36
};

/*
 * Per-launch execution controls.  A NULL kx_exec means: default stream, all
 * SMs, no yielding, fp32 via 3xTF32.
 *
 *  stream       cudaStream_t the kernels are enqueued on.
 *  sm_quota     upper bound on the number of SMs (persistent CTAs) the op may
 *               occupy; 0 = all SMs.  This is how the HP/BE scheduler shares
 *               the GPU (it replaces the green-context SM split of
 *               src/scheduler.cpp:244-446).
 *  yield_flag   host-mapped int (pinned memory).  When non-NULL, persistent
 *               CTAs read it before taking each new tile: 0 = keep going;
 *               f > 0 = only CTAs with index < f keep taking tiles (the op
 *               still completes, on fewer SMs); f < 0 = every CTA stops.  A
 *               stopped op keeps its progress in its work slot, so calling the
 *               same entry point again with identical arguments continues where
 *               it stopped.  Ops that may stop should pass done_flag.
 *  done_flag    host-mapped int.  When non-NULL the last CTA of the launch
 *               writes 1 (all tiles finished) or 0 (yielded) to it.
 *  max_tiles    >0: each CTA takes at most this many tiles per launch (a
 *               deterministic way to exercise continuation); 0 = unlimited.
 *  timeout_ns   limit for each bounded device-side wait; 0 = 2 s.
 *  fp32_mode    KX_FP32_* for fp32 operands.
 *  err_word     optional device int; a bounded wait that gives up writes
 *               KX_ERR_TIMEOUT there (first error wins).
 *  scalars_on_device  non-zero: alpha/beta are device pointers
 *               (CUBLAS_POINTER_MODE_DEVICE); otherwise host pointers.
 */
typedef struct kx_exec {
    void* stream;
    int sm_quota;
    const volatile int* yield_flag;
    volatile int* done_flag;
    int max_tiles;
    unsigned long long timeout_ns;
    int fp32_mode;
    int* err_word;
    int scalars_on_device;
} kx_exec;

/* ---------------------------------------------------------------- GEMM --- */

int kx_sgemm(const kx_exec* ex, int transa, int transb, int m, int n, int k,
             const float* alpha, const float* A, int lda, const float* B, int ldb,
             const float* beta, float* C, int ldc);

int kx_sgemm_strided_batched(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                             const float* alpha, const float* A, int lda, long long strideA,
                             const float* B, int ldb, long long strideB, const float* beta,
                             float* C, int ldc, long long strideC, int batch);

/* Pointer-array batch (cublasSgemmBatched).  Aarray/Barray/Carray are DEVICE
 * arrays of device pointers, as in cuBLAS. */
int kx_sgemm_batched(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                     const float* alpha, const float* const* Aarray, int lda,
                     const float* const* Barray, int ldb, const float* beta,
                     float* const* Carray, int ldc, int batch);

/* Mixed precision: A/B/C types are KX_R_*; alpha/beta are fp32 host values
 * (compute type CUBLAS_COMPUTE_32F / 32F_FAST_*). */
int kx_gemm_ex(const kx_exec* ex, int transa, int transb, int m, int n, int k,
               const float* alpha, const void* A, int Atype, int lda,
               const void* B, int Btype, int ldb, const float* beta,
               void* C, int Ctype, int ldc);

int kx_gemm_strided_batched_ex(const kx_exec* ex, int transa, int transb, int m, int n, int k,
                               const float* alpha, const void* A, int Atype, int lda,
                               long long strideA, const void* B, int Btype, int ldb,
                               long long strideB, const float* beta, void* C, int Ctype,
                               int ldc, long long strideC, int batch);

/* cublasLtMatmul as decoded by the interposer: D = epi(alpha*op(A)op(B) + beta*C + bias).
 * C and D may alias.  bias (length m, type bias_type) is used by *_BIAS
 * epilogues.  All matrices column-major. */
int kx_matmul(const kx_exec* ex, int transa, int transb, int m, int n, int k,
              const float* alpha, const void* A, int Atype, int lda, long long strideA,
              const void* B, int Btype, int ldb, long long strideB, const float* beta,
              const void* C, int Ctype, int ldc, long long strideC,
              void* D, int Dtype, int ldd, long long strideD, int batch,
              int epilogue, const void* bias, int bias_type);

/* ------------------------------------------------------- convolution --- */

/* NCHW x (n,c,h,w), KCRS filter (k,c,r,s), NCHW y (n,k,p,q); cross-correlation
 * (CUDNN_CROSS_CORRELATION) or convolution (mode 0, filter flipped);
 * y = alpha*conv(x,w) + beta*y.  groups = 1. */
typedef struct kx_conv_desc {
    int n, c, h, w;      /* input */
    int k, r, s;         /* filter */
    int pad_h, pad_w;
    int stride_h, stride_w;
    int dil_h, dil_w;
    int cross_correlation; /* 1 = CUDNN_CROSS_CORRELATION, 0 = CUDNN_CONVOLUTION */
} kx_conv_desc;

/* Output spatial size of a convolution descriptor. */
int kx_conv_out_dims(const kx_conv_desc* d, int* p, int* q);

int kx_conv_fwd(const kx_exec* ex, const kx_conv_desc* d, const float* alpha,
                const float* x, const float* w, const float* beta, float* y);

/* dx = alpha*conv^T(w, dy) + beta*dx */
int kx_conv_bwd_data(const kx_exec* ex, const kx_conv_desc* d, const float* alpha,
                     const float* w, const float* dy, const float* beta, float* dx);

/* dw = alpha*corr(x, dy) + beta*dw */
int kx_conv_bwd_filter(const kx_exec* ex, const kx_conv_desc* d, const float* alpha,
                       const float* x, const float* dy, const float* beta, float* dw);

/* -------------------------------------------------------- batch norm --- */

/* mode: 0 = CUDNN_BATCHNORM_PER_ACTIVATION, 1 = CUDNN_BATCHNORM_SPATIAL.
 * y = alpha*BN(x) + beta*y; running stats updated with
 * running = (1-f)*running + f*batch (unbiased variance for the running value);
 * save_mean / save_inv_var hold batch mean and 1/sqrt(var_biased + eps). */
int kx_bn_fwd_training(const kx_exec* ex, int mode, const float* alpha, const float* beta,
                       int n, int c, int h, int w, const float* x, float* y,
                       const float* scale, const float* bias, double exp_avg_factor,
                       float* running_mean, float* running_var, double eps,
                       float* save_mean, float* save_inv_var);

/* Allocation-free kx_bn_fwd_training (no counterpart in the reference: an
 * addition for callers that cannot allocate device memory, such as code that
 * runs while a CUDA graph is being captured or under an allocator that owns
 * every device byte).  Same arguments and results; its statistics scratch is
 * one file-scope device array of 4 MiB per device, so it calls no
 * cudaMalloc / cudaFree.  Returns KX_ERR_INVALID when the call needs more
 * scratch than that (16 bytes per channel-split partial plus 8 bytes per
 * channel in modes 1 and 2; 8 bytes per activation c*h*w in mode 0), or when
 * ex->stream belongs to another device than the current one.  The first call
 * on a device looks up the array's device address; make it before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race and
 * must be serialised by the caller. */
int kx_bn_fwd_training_noalloc(const kx_exec* ex, int mode, const float* alpha,
                               const float* beta, int n, int c, int h, int w, const float* x,
                               float* y, const float* scale, const float* bias,
                               double exp_avg_factor, float* running_mean, float* running_var,
                               double eps, float* save_mean, float* save_inv_var);

int kx_bn_fwd_inference(const kx_exec* ex, int mode, const float* alpha, const float* beta,
                        int n, int c, int h, int w, const float* x, float* y,
                        const float* scale, const float* bias, const float* est_mean,
                        const float* est_var, double eps);

int kx_bn_bwd(const kx_exec* ex, int mode, const float* alpha_data, const float* beta_data,
              const float* alpha_param, const float* beta_param, int n, int c, int h, int w,
              const float* x, const float* dy, float* dx, const float* scale,
              float* dscale, float* dbias, double eps, const float* save_mean,
              const float* save_inv_var);

/* --------------------------------------------------------- utilities --- */

/* Pinned, device-mapped host ints (zeroed) for yield / done flags: *host and
 * *dev receive the host and the device address of the same `count` ints. */
int kx_host_flags_alloc(int count, int** host, int** dev);
int kx_host_flags_free(int* host);

/* Waits (bounded by timeout_ns) until the host-mapped *flag becomes non-zero,
 * on `stream`.  Writes KX_OK or KX_ERR_TIMEOUT to the device int *status.
 * This is the same bounded-wait path the persistent kernels use, exposed so
 * the give-up behaviour can be exercised without faulting or hanging a GPU. */
int kx_wait_flag(void* stream, const volatile int* flag, unsigned long long timeout_ns,
                 int* status);

/* Number of SMs on the current device (cached). */
int kx_num_sms(void);

/* Human-readable name of the kernel configuration the last GEMM call on this
 * thread selected (for profile tables); never NULL. */
const char* kx_last_kernel_name(void);

/* Grid (persistent CTAs, i.e. SMs occupied) of the last persistent GEMM /
 * convolution launch this thread made: min(work tiles, SM quota, SM count).
 * For profile tables; 0 before the first such launch. */
int kx_last_grid(void);

/* cudaError_t (as int) behind the last KX_ERR_DEVICE status this thread got
 * from the library; 0 before the first.  Diagnostics only. */
int kx_last_cuda_error(void);

/* Version string of the library. */
const char* kx_version(void);

/* Number of kernels this library has launched in this process (all devices,
 * all threads; the count is taken on the host just before each launch). */
unsigned long long kx_launch_count(void);

/* Number of device-memory allocations and frees (cudaMalloc / cudaFree) this
 * library has made in this process, all devices.  Scratch buffers grow on
 * demand; a call that leaves this count unchanged allocated nothing. */
unsigned long long kx_device_alloc_count(void);

#ifdef __cplusplus
}
#endif

#endif /* KX_H */
