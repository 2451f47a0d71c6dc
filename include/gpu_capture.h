/**
 * @file gpu_capture.h
 * @brief Capture layer of the interposer: operation records, per-client
 *        queues, client identity and the orion_* capture C API.
 *
 * Public declarations follow the reference's include/gpu_capture.h (param
 * structs 38-199, OperationRecord 205-252, ClientQueue 260-305, API 327-383)
 * so drivers and C++ code written against it keep working.  Differences of
 * this build, all additive:
 *  - ClientQueue is a lock-free bounded multi-producer ring (Vyukov style)
 *    instead of a mutex-guarded std::queue; push/try_pop/peek/empty/size keep
 *    their meaning (peek is for the queue's single consumer, the worker).
 *  - OperationRecord::wait_completion() is bounded by a deadline
 *    (ORION_WAIT_TIMEOUT_MS, default 60000) and records cudaErrorTimeout
 *    instead of spinning forever.
 *  - cuBLAS / cuBLASLt / cuDNN params carry the decoded call (types, layout,
 *    epilogue, descriptor contents, scalar values) so the worker can dispatch
 *    to the kx kernels after the caller's descriptors are gone.
 */
#ifndef ORION_GPU_CAPTURE_H
#define ORION_GPU_CAPTURE_H

#include <cuda_runtime_api.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <variant>
#include <vector>

#include "common.h"

namespace orion {

constexpr size_t MAX_KERNEL_ARGS_SIZE = 4096;
constexpr size_t MAX_KERNEL_ARGS_COUNT = 64;

struct KernelLaunchParams {
    const void* func;
    dim3 gridDim;
    dim3 blockDim;
    size_t sharedMem;
    cudaStream_t stream;
    void** original_args;

    std::vector<uint8_t> args_buffer;
    std::vector<size_t> args_offsets;
    std::vector<size_t> args_sizes;
    size_t num_args;
    std::vector<void*> args_ptrs;
    bool use_deep_copy;

    // launch flavour: 0 = cudaLaunchKernel, 1 = cudaLaunchKernelExC, 2 = cuLaunchKernel
    int api;
    const void* ex_config;   // cudaLaunchConfig_t* (api 1)
    void** extra;            // cuLaunchKernel extra (api 2)
    std::shared_ptr<void> ex_owned;  // keeps *ex_config and its attributes alive (api 1)

    KernelLaunchParams()
        : func(nullptr), sharedMem(0), stream(nullptr), original_args(nullptr), num_args(0),
          use_deep_copy(false), api(0), ex_config(nullptr), extra(nullptr) {
        gridDim = {1, 1, 1};
        blockDim = {1, 1, 1};
    }

    void** get_args() {
        if (use_deep_copy && num_args > 0) {
            args_ptrs.resize(num_args);
            for (size_t i = 0; i < num_args; i++) args_ptrs[i] = args_buffer.data() + args_offsets[i];
            return args_ptrs.data();
        }
        return original_args;
    }
};

struct MallocParams {
    void** devPtr;
    size_t size;
};

struct FreeParams {
    void* devPtr;
};

struct MemcpyParams {
    void* dst;
    const void* src;
    size_t count;
    cudaMemcpyKind kind;
    cudaStream_t stream;
    bool is_async;
};

struct MemsetParams {
    void* devPtr;
    int value;
    size_t count;
    cudaStream_t stream;
    bool is_async;
};

struct SyncParams {
    cudaStream_t stream;
    cudaEvent_t event;
    unsigned int flags;
};

/** Decoded convolution geometry (NCHW / KCRS, 2-D, groups = 1). */
struct ConvGeometry {
    int n, c, h, w;
    int k, r, s;
    int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
    int cross_correlation;
    int data_type;       // cudnnDataType_t of x / w / y
    int packed_nchw;     // 1 when all three tensors are fully packed NCHW
};

struct CudnnConvParams {
    void* handle;
    void* xDesc;
    const void* x;
    void* wDesc;
    const void* w;
    void* convDesc;
    int algo;
    void* workSpace;
    size_t workSpaceSizeInBytes;
    const void* alpha;
    const void* beta;
    void* yDesc;
    void* y;
    // decoded at capture time
    ConvGeometry geom;
    float alpha_value;
    float beta_value;
    cudaStream_t stream;
};

struct CudnnBatchNormParams {
    void* handle;
    int mode;
    const void* alpha;
    const void* beta;
    void* xDesc;
    const void* x;
    void* yDesc;
    void* y;
    void* bnScaleBiasMeanVarDesc;
    const void* bnScale;
    const void* bnBias;
    double exponentialAverageFactor;
    void* resultRunningMean;
    void* resultRunningVariance;
    double epsilon;
    void* resultSaveMean;
    void* resultSaveInvVariance;
    // decoded at capture time
    int n, c, h, w;
    float alpha_value, beta_value;
    // backward / inference extras
    const void* dy;
    void* dx;
    void* dBnScaleResult;
    void* dBnBiasResult;
    float alpha_param, beta_param;
    const void* estimatedMean;
    const void* estimatedVariance;
    cudaStream_t stream;
};

struct CublasGemmParams {
    void* handle;
    int transa;
    int transb;
    int m, n, k;
    const void* alpha;
    const void* A;
    int lda;
    const void* B;
    int ldb;
    const void* beta;
    void* C;
    int ldc;
    int batchCount;
    long long strideA, strideB, strideC;
    bool is_batched;
    bool is_strided;
    float alpha_value;
    float beta_value;
    bool use_stored_scalars;
    cudaStream_t stream;
    // additions: operand types (cudaDataType_t), scalar residency, math mode
    int Atype, Btype, Ctype;
    bool scalars_on_device;
    int math_mode;  // cublasMath_t of the handle at capture time

    CublasGemmParams()
        : handle(nullptr), transa(0), transb(0), m(0), n(0), k(0), alpha(nullptr), A(nullptr),
          lda(0), B(nullptr), ldb(0), beta(nullptr), C(nullptr), ldc(0), batchCount(0),
          strideA(0), strideB(0), strideC(0), is_batched(false), is_strided(false),
          alpha_value(1.0f), beta_value(0.0f), use_stored_scalars(false), stream(nullptr),
          Atype(0), Btype(0), Ctype(0), scalars_on_device(false), math_mode(0) {}
};

/** cublasLtMatmul call decoded from its (caller-owned) descriptors. */
struct LtDecoded {
    int transa, transb;
    int m, n, k;
    int Atype, Btype, Ctype, Dtype;
    long long lda, ldb, ldc, ldd;
    long long strideA, strideB, strideC, strideD;
    int batch;
    int epilogue;
    const void* bias;
    int bias_type;
    int compute_type;
    int scale_type;
    bool scalars_on_device;
    bool supported;
};

struct CublasLtMatmulParams {
    void* lightHandle;
    void* computeDesc;
    const void* alpha;
    const void* A;
    void* Adesc;
    const void* B;
    void* Bdesc;
    const void* beta;
    const void* C;
    void* Cdesc;
    void* D;
    void* Ddesc;
    const void* algo;
    void* workspace;
    size_t workspaceSizeInBytes;
    cudaStream_t stream;
    float alpha_value;
    float beta_value;
    bool use_stored_scalars;
    LtDecoded dec;

    CublasLtMatmulParams()
        : lightHandle(nullptr), computeDesc(nullptr), alpha(nullptr), A(nullptr), Adesc(nullptr),
          B(nullptr), Bdesc(nullptr), beta(nullptr), C(nullptr), Cdesc(nullptr), D(nullptr),
          Ddesc(nullptr), algo(nullptr), workspace(nullptr), workspaceSizeInBytes(0),
          stream(nullptr), alpha_value(1.0f), beta_value(0.0f), use_stored_scalars(false) {
        std::memset(&dec, 0, sizeof(dec));
    }
};

// ============================================================================
// OperationRecord
// ============================================================================

/** Deadline for client-side waits (ORION_WAIT_TIMEOUT_MS, default 60 s). */
int64_t wait_timeout_ns();

struct OperationRecord {
    OperationType type;
    uint64_t op_id;
    int client_idx;

    std::variant<KernelLaunchParams, MallocParams, FreeParams, MemcpyParams, MemsetParams,
                 SyncParams, CudnnConvParams, CudnnBatchNormParams, CublasGemmParams,
                 CublasLtMatmulParams>
        params;

    std::atomic<bool> completed{false};
    std::atomic<bool> started{false};
    /** Life cycle: kQueued -> kClaimed (the worker took it and will run it)
     *  or kQueued -> kCancelled (the client gave up waiting first; the
     *  worker then skips it).  Exactly one of the two transitions wins. */
    enum : int { kQueued = 0, kClaimed = 1, kCancelled = 2 };
    std::atomic<int> state{kQueued};
    /** True when running the record later touches nothing the issuing
     *  thread owns (its arguments were copied into the record): the client
     *  may stop waiting for it even after the worker claimed it. */
    bool detachable{false};
    /** Written by the worker only, before `completed` is released. */
    cudaError_t result{cudaSuccess};
    void* result_ptr{nullptr};
    int64_t enqueue_ns{0};
    int64_t start_ns{0};  // worker began executing it
    int64_t end_ns{0};    // worker finished executing it

    OperationRecord()
        : type(OperationType::UNKNOWN), op_id(0), client_idx(-1), params(MallocParams{}) {}
    ~OperationRecord() = default;
    OperationRecord(const OperationRecord&) = delete;
    OperationRecord& operator=(const OperationRecord&) = delete;
    OperationRecord(OperationRecord&&) = delete;
    OperationRecord& operator=(OperationRecord&&) = delete;

    /** Waits for the worker and returns the op's result.  After
     *  wait_timeout_ns() a record the worker has not claimed is cancelled
     *  (it never runs) and cudaErrorTimeout is returned; a detachable
     *  record is abandoned the same way; any other claimed record is
     *  running on the worker and is waited for to the end, because it still
     *  reads or writes memory of the issuing thread. */
    cudaError_t wait_completion();

    /** Worker side: claims a queued record; false when it was cancelled. */
    bool claim() {
        int expect = kQueued;
        return state.compare_exchange_strong(expect, kClaimed, std::memory_order_acq_rel);
    }
    /** Client side: cancels a record the worker has not claimed. */
    bool cancel() {
        int expect = kQueued;
        return state.compare_exchange_strong(expect, kCancelled, std::memory_order_acq_rel);
    }

    void mark_completed(cudaError_t res) {
        result = res;
        completed.store(true, std::memory_order_release);
    }
};

using OperationPtr = std::shared_ptr<OperationRecord>;

// ============================================================================
// ClientQueue — lock-free bounded ring, many producers, one consumer (worker)
// ============================================================================

class ClientQueue {
public:
    static constexpr size_t kCapacity = 8192;  // power of two

    ClientQueue();
    ~ClientQueue();

    /** Enqueue; spins (yielding) while the ring is full, for at most
     *  wait_timeout_ns(); false when the ring stayed full that long. */
    bool push(OperationPtr op);
    /** Non-blocking enqueue; false when full. */
    bool try_push(OperationPtr op);
    /** Dequeue or nullptr when empty. */
    OperationPtr try_pop();
    /** Head without removing it (consumer thread only). */
    OperationPtr peek();
    bool empty();
    size_t size();
    void shutdown() { shutdown_.store(true); }
    bool is_shutdown() const { return shutdown_.load(); }

private:
    struct Cell {
        std::atomic<size_t> seq;
        OperationPtr op;
    };
    Cell* cells_;
    alignas(64) std::atomic<size_t> head_;  // next to dequeue
    alignas(64) std::atomic<size_t> tail_;  // next to enqueue
    std::atomic<bool> shutdown_;
};

// ============================================================================
// CaptureLayerState
// ============================================================================

struct CaptureLayerState {
    std::atomic<bool> initialized{false};
    std::atomic<bool> enabled{false};
    int num_clients{0};

    std::vector<std::unique_ptr<ClientQueue>> client_queues;
    std::atomic<uint64_t> next_op_id{0};
    std::atomic<bool> shutdown{false};
};

extern CaptureLayerState g_capture_state;

int init_capture_layer(int num_clients);
void shutdown_capture_layer();

int get_current_client_idx();
void set_current_client_idx(int idx);

OperationPtr create_operation(int client_idx, OperationType type);
/** Queues the record for its client's worker.  False when the queue stayed
 *  full for wait_timeout_ns(): the record is then completed with
 *  cudaErrorTimeout, never runs, and the client's error latch is set. */
bool enqueue_operation(OperationPtr op);
/** BE client threads pass here before queueing an op (see
 *  Scheduler::be_issue_gate); a no-op for the HP client and for ops other
 *  than kernel launches and captured dense ops. */
void be_issue_gate(int client_idx, OperationType type);
/** The HP client queued an op (see be_issue_gate). */
void note_hp_issue();
/** Bounded wait for the worker (see OperationRecord::wait_completion);
 *  returns the op's result, cudaErrorTimeout when the client gave up. */
cudaError_t wait_operation(OperationPtr op);

/** create + enqueue in one step (the record must be filled before the
 *  worker can see it: callers fill params on the returned record only when
 *  they created it with create_operation; this helper enqueues last). */
OperationPtr submit_operation(int client_idx, OperationType type);

bool is_managed_thread();
bool is_capture_enabled();
void set_capture_enabled(bool enabled);

void register_client_stream(int client_idx, void* stream);
void register_client_handle(int client_idx, void* handle);
int resolve_client_idx(void* stream = nullptr, void* handle = nullptr);
void clear_client_maps();

/** Stream a library handle was bound to by cublasSetStream / cudnnSetStream. */
void remember_handle_stream(void* handle, cudaStream_t stream);
cudaStream_t handle_stream(void* handle);

void set_async_mode_internal(int mode);
int get_async_mode_internal();
void set_last_error(int client_idx, cudaError_t error);
cudaError_t get_and_clear_last_error(int client_idx);

/** Time client threads spent blocked in wait_operation (see
 *  orion_get_client_waits). */
void get_wait_stats(int client_idx, unsigned long long* out8, bool reset);

/** Capture trace (addition of this build; see orion_trace_start). */
bool trace_enabled();
/** The worker executed `op` (start_ns .. end_ns set). */
void trace_executed(const OperationRecord& op);
/** A client thread waited for `op` from t0 to t1 (CLOCK_MONOTONIC ns). */
void trace_client_wait(const OperationRecord& op, int64_t t0, int64_t t1);
/** A scheduler event without duration (e.g. the HP flag changing). */
void trace_marker(const char* name, int value);

/** Op log (addition of this build; see orion_op_log_start). */
bool op_log_enabled();
/** One intercepted dense call: client (resolved even with capture off), op
 *  type, up to 8 shape / layout integers, and its route ("capture", "direct",
 *  "real"). */
void op_log_record(int client_idx, OperationType type, const long long* dims, int ndims,
                   const char* route);

}  // namespace orion

extern "C" {

int orion_init(int num_clients);
void orion_shutdown();
void orion_set_client_idx(int idx);
int orion_get_client_idx();
void orion_set_enabled(int enabled);
int orion_is_enabled();

int orion_set_capture(int enabled);
void orion_register_client_stream(int client_idx, void* stream);
void orion_register_client_handle(int client_idx, void* handle);
int orion_resolve_client_idx(void* stream, void* handle);

/* Op log (addition of this build, no counterpart in the reference): records
 * every dense library call the interposer intercepts (cuBLAS GEMMs, cuBLASLt
 * matmul, cuDNN convolutions and batch norm), in the order the calling
 * threads made them and whether it was captured, passed through, or made with
 * capture off.  Comparing the log of a run through the real libraries with
 * the log of the same program captured shows that capture keeps each
 * client's op sequence (types, shapes, counts) unchanged.
 * orion_op_log_end writes one tab-separated line per call (client, op type,
 * route, shape integers) and returns the number of lines, or -1. */
void orion_op_log_start(void);
int orion_op_log_end(const char* path);

/* Client-thread blocking (addition of this build): how often and how long a
 * client's threads waited for its worker inside intercepted calls (those that
 * must complete before returning: copies from pageable memory, allocations,
 * launches whose arguments could not be copied, ...).  out8 = {waits,
 * total ns, longest ns, and for the longest: OperationType, ns queued before
 * the worker took it, ns the worker spent executing it, bytes (allocation or
 * copy size, else 0), 0}; reset != 0 clears. */
int orion_get_client_waits(int client_idx, unsigned long long* out8, int reset);

/* Capture trace (addition of this build): a Chrome trace (JSON, chrome://tracing
 * or Perfetto) of the interposer's own activity between orion_trace_start and
 * orion_trace_end: per client, one track for the client thread (each captured
 * call as an instant at the moment it was issued, and the calls that blocked
 * as spans), one for its worker (each op's execution span with op id, time
 * queued and size as args), and a scheduler track with the HP-flag changes.
 * Timestamps are CLOCK_MONOTONIC microseconds.  At most 4 M events are kept;
 * orion_trace_end writes the file and returns the number of events, or -1. */
void orion_trace_start(void);
int orion_trace_end(const char* path);
}

#endif  // ORION_GPU_CAPTURE_H
