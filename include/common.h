/**
 * @file common.h
 * @brief Shared definitions of the interposer (libgpu_scheduler.so).
 *
 * Same public declarations as the reference's include/common.h (op-type and
 * profile-type enums, logging macros, the scheduler thread-locals), so code
 * written against the reference headers compiles unchanged.  The op-type enum
 * keeps the reference enumerators in their order (include/common.h:60-93 of
 * the reference) and appends the ops this build captures in addition
 * (cuBLAS *Ex GEMMs, batch-norm inference/backward) before UNKNOWN.
 */
#ifndef ORION_COMMON_H
#define ORION_COMMON_H

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>

namespace orion {

/** Maximum number of clients (1 HP + up to 15 BE). */
constexpr int MAX_CLIENTS = 16;

/** Operations the interposer can capture. */
enum class OperationType : uint8_t {
    KERNEL_LAUNCH = 0,
    KERNEL_LAUNCH_EX,
    KERNEL_LAUNCH_DRV,
    MALLOC,
    FREE,
    MEMCPY,
    MEMCPY_ASYNC,
    MEMSET,
    MEMSET_ASYNC,
    DEVICE_SYNC,
    STREAM_SYNC,
    EVENT_SYNC,
    CUDNN_CONV_FWD,
    CUDNN_CONV_BWD_DATA,
    CUDNN_CONV_BWD_FILTER,
    CUDNN_BATCHNORM_FWD,
    CUDNN_BATCHNORM_BWD,
    CUBLAS_SGEMM,
    CUBLAS_SGEMM_BATCHED,
    CUBLAS_SGEMM_STRIDED_BATCHED,
    CUBLASLT_MATMUL,
    CUBLAS_GEMM_EX,                  // cublasGemmEx / cublasSgemmEx / cublasHgemm
    CUBLAS_GEMM_STRIDED_BATCHED_EX,  // cublasGemmStridedBatchedEx / cublasHgemmStridedBatched
    CUDNN_BATCHNORM_INF,             // cudnnBatchNormalizationForwardInference
    EVENT_RECORD,                    // cudaEventRecord(WithFlags): kept in client order
    STREAM_WAIT_EVENT,               // cudaStreamWaitEvent: kept in client order
    UNKNOWN
};

/** Compute- vs memory-bound classification used by the profile tables. */
enum class ProfileType : uint8_t {
    COMPUTE_BOUND = 0,
    MEMORY_BOUND,
    UNKNOWN
};

inline const char* op_type_name(OperationType type) {
    switch (type) {
        case OperationType::KERNEL_LAUNCH: return "KERNEL_LAUNCH";
        case OperationType::KERNEL_LAUNCH_EX: return "KERNEL_LAUNCH_EX";
        case OperationType::KERNEL_LAUNCH_DRV: return "KERNEL_LAUNCH_DRV";
        case OperationType::MALLOC: return "MALLOC";
        case OperationType::FREE: return "FREE";
        case OperationType::MEMCPY: return "MEMCPY";
        case OperationType::MEMCPY_ASYNC: return "MEMCPY_ASYNC";
        case OperationType::MEMSET: return "MEMSET";
        case OperationType::MEMSET_ASYNC: return "MEMSET_ASYNC";
        case OperationType::DEVICE_SYNC: return "DEVICE_SYNC";
        case OperationType::STREAM_SYNC: return "STREAM_SYNC";
        case OperationType::EVENT_SYNC: return "EVENT_SYNC";
        case OperationType::CUDNN_CONV_FWD: return "CUDNN_CONV_FWD";
        case OperationType::CUDNN_CONV_BWD_DATA: return "CUDNN_CONV_BWD_DATA";
        case OperationType::CUDNN_CONV_BWD_FILTER: return "CUDNN_CONV_BWD_FILTER";
        case OperationType::CUDNN_BATCHNORM_FWD: return "CUDNN_BATCHNORM_FWD";
        case OperationType::CUDNN_BATCHNORM_BWD: return "CUDNN_BATCHNORM_BWD";
        case OperationType::CUBLAS_SGEMM: return "CUBLAS_SGEMM";
        case OperationType::CUBLAS_SGEMM_BATCHED: return "CUBLAS_SGEMM_BATCHED";
        case OperationType::CUBLAS_SGEMM_STRIDED_BATCHED: return "CUBLAS_SGEMM_STRIDED_BATCHED";
        case OperationType::CUBLASLT_MATMUL: return "CUBLASLT_MATMUL";
        case OperationType::CUBLAS_GEMM_EX: return "CUBLAS_GEMM_EX";
        case OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX: return "CUBLAS_GEMM_STRIDED_BATCHED_EX";
        case OperationType::CUDNN_BATCHNORM_INF: return "CUDNN_BATCHNORM_INF";
        case OperationType::EVENT_RECORD: return "EVENT_RECORD";
        case OperationType::STREAM_WAIT_EVENT: return "STREAM_WAIT_EVENT";
        default: return "UNKNOWN";
    }
}

/** Log levels (ORION_LOG_LEVEL = NONE|ERROR|WARN|INFO|DEBUG|TRACE or 0-5). */
enum class LogLevel : uint8_t {
    NONE = 0,
    ERROR,
    WARN,
    INFO,
    DEBUG,
    TRACE
};

extern LogLevel g_log_level;

/** Reads ORION_LOG_LEVEL. */
void init_log_level();

#define ORION_LOG(level, fmt, ...)                                                     \
    do {                                                                               \
        if (static_cast<uint8_t>(level) <= static_cast<uint8_t>(orion::g_log_level)) { \
            fprintf(stderr, "[ORION][%s] " fmt "\n", #level, ##__VA_ARGS__);          \
            fflush(stderr);                                                            \
        }                                                                              \
    } while (0)

#define LOG_ERROR(fmt, ...) ORION_LOG(orion::LogLevel::ERROR, fmt, ##__VA_ARGS__)
#define LOG_WARN(fmt, ...) ORION_LOG(orion::LogLevel::WARN, fmt, ##__VA_ARGS__)
#define LOG_INFO(fmt, ...) ORION_LOG(orion::LogLevel::INFO, fmt, ##__VA_ARGS__)
#define LOG_DEBUG(fmt, ...) ORION_LOG(orion::LogLevel::DEBUG, fmt, ##__VA_ARGS__)
#define LOG_TRACE(fmt, ...) ORION_LOG(orion::LogLevel::TRACE, fmt, ##__VA_ARGS__)

/** True on scheduler worker threads (their CUDA calls are never captured). */
extern thread_local bool tl_is_scheduler_thread;

/** True while a worker executes a captured op (re-entrancy guard). */
extern thread_local bool tl_in_scheduler_execution;

/** Client index served by the current worker thread (-1 elsewhere). */
extern thread_local int tl_worker_idx;

}  // namespace orion

#endif  // ORION_COMMON_H
