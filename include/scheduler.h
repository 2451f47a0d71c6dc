/**
 * @file scheduler.h
 * @brief Orion-style HP/BE scheduler of the interposer.
 *
 * Public declarations follow the reference's include/scheduler.h (profile
 * info, execution modes, SchedulerConfig, OrionSchedulingState, the Scheduler
 * class surface and the C API).  What changes is how SMs are shared:
 *
 *  - The reference splits the GPU with CUDA green contexts
 *    (src/scheduler.cpp:244-446 of the reference).  Here every captured dense
 *    op runs as a persistent kx kernel whose grid is bounded by an SM quota,
 *    and best-effort (BE) kernels poll a host-mapped HP flag at tile
 *    boundaries.  "ISOLATED" mode therefore means disjoint SM budgets
 *    (hp_sm_count / be_sm_count) enforced by the kernels themselves, and
 *    init_green_contexts() / autotune_green_ctx() choose those budgets.
 *  - In DEFAULT mode BE kernels may use every SM while the HP client is idle;
 *    when HP work is in flight the HP worker raises the flag to the number of
 *    SMs BE may keep (be_keep_sms), CTAs above it retire at their next tile
 *    boundary and the rest finish the op.
 *  - Captured ops execute on the stream the client issued them on, in the
 *    client's FIFO order, so ordering with the client's other work is kept.
 */
#ifndef ORION_SCHEDULER_H
#define ORION_SCHEDULER_H

#include <cuda_runtime_api.h>

#include <atomic>
#include <chrono>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include "gpu_capture.h"
#include "kernel_profile.h"

namespace orion {

/** One row of kernel_info.csv (Name,Profile,Memory_footprint,SM_usage,Duration). */
struct KernelProfileInfo {
    std::string name;
    int profile;     // 1 compute-bound, 0 memory-bound, -1 unclear
    int mem;
    int sm_used;
    float duration;  // ns

    KernelProfileInfo() : profile(-1), mem(0), sm_used(0), duration(0.0f) {}
    KernelProfileInfo(const std::string& n, int p, int m, int sm, float dur)
        : name(n), profile(p), mem(m), sm_used(sm), duration(dur) {}
};

enum class ExecutionMode {
    DEFAULT = 0,   // BE may use all SMs while HP is idle; shrinks when HP runs
    ISOLATED = 1,  // fixed disjoint SM budgets for HP and BE
};

struct SchedulerConfig {
    int device_id = 0;
    int num_sms = 0;
    int sm_threshold = 0;
};

struct OrionSchedulingState {
    std::vector<std::vector<KernelProfileInfo>> op_info_vector;
    std::vector<int> seen;
    std::vector<int> num_client_kernels;
    int sm_threshold = 0;
    std::mutex mutex;

    void init(int num_clients, int num_sms) {
        op_info_vector.assign(num_clients, {});
        seen.assign(num_clients, 0);
        num_client_kernels.assign(num_clients, 0);
        sm_threshold = num_sms / 2;
    }

    void reset() {
        for (auto& v : op_info_vector) v.clear();
        std::fill(seen.begin(), seen.end(), 0);
        std::fill(num_client_kernels.begin(), num_client_kernels.end(), 0);
    }
};

extern OrionSchedulingState g_orion_state;

/** Per-client counters (exported through orion_get_client_stats). */
struct ClientStats {
    std::atomic<uint64_t> ops{0};
    std::atomic<uint64_t> kx_ops{0};
    std::atomic<uint64_t> passthrough_ops{0};
    std::atomic<uint64_t> be_blocked{0};
    std::atomic<uint64_t> yields{0};
    std::atomic<uint64_t> errors{0};
    std::atomic<uint64_t> host_holds{0};  // ops this BE client's threads waited before queueing
};

class Scheduler {
public:
    Scheduler();
    ~Scheduler();

    /** SM budgets of ISOLATED mode (kept under the reference's name). */
    struct GreenCtxConfig {
        unsigned int hp_sm_count = 56;
        unsigned int be_sm_count = 56;
        bool enabled = false;
        bool auto_tune = true;
    };

    bool init(int num_clients, const SchedulerConfig& config = SchedulerConfig());
    void start();
    void stop();
    void join();
    void reset();
    int autotune_green_ctx();

    const SchedulerConfig& get_config() const { return config_; }
    SchedulerConfig& get_mutable_config() { return config_; }
    int get_num_clients() const { return num_clients_; }

    bool is_green_ctx_enabled() const { return isolated_; }
    ExecutionMode get_current_mode() const { return isolated_ ? ExecutionMode::ISOLATED : ExecutionMode::DEFAULT; }

    /** Applies fixed HP/BE SM budgets (ISOLATED mode). */
    bool init_green_contexts(const GreenCtxConfig& gc_config);
    /** Returns to DEFAULT mode (shared SMs, HP flag). */
    void clear_budgets() { isolated_ = false; }
    /** Wave-model choice of budgets from the loaded kernel_info profiles. */
    GreenCtxConfig choose_best_green_ctx_config_from_profiles() const;

    void sync_client_stream(int client_idx);

    // SM budget policy
    int hp_quota() const;
    int be_quota() const;
    void set_be_keep_sms(int sms) { be_keep_sms_.store(sms); }
    /** Profiling sessions also time the kernels the interposer re-issues. */
    void set_profile_launches(bool on) { profile_launches_.store(on); }
    int be_keep_sms() const { return be_keep_sms_.load(); }
    /** A BE client thread about to queue a kernel while the HP client is
     *  issuing (it queued an op within the last KX_BE_HOST_WINDOW_US, default
     *  500) waits until HP stops issuing, at most KX_BE_HOST_HOLD_US per op
     *  (default 3000; 0 turns the gate off), unless it holds the Python
     *  interpreter lock.  PyTorch releases that lock around every operator,
     *  so a BE thread held here leaves the interpreter to the HP client's
     *  thread while it issues; once HP waits for its results, BE issues
     *  again. */
    void be_issue_gate(int client_idx);
    /** The HP client queued an op (the issue gate's clock). */
    void note_hp_issue();
    void set_be_host_hold_us(int us) { be_host_hold_ns_.store(us < 0 ? 0 : 1000LL * us); }
    /** Profiling sessions time one in n dense ops of each client (n >= 1). */
    void set_profile_every(int n) { profile_every_.store(n < 1 ? 1 : n); }
    int be_host_hold_us() const { return static_cast<int>(be_host_hold_ns_.load() / 1000); }
    volatile int* hp_flag_host() const { return hp_flag_host_; }
    int* hp_flag_device() const { return hp_flag_dev_; }

    ClientStats& stats(int client_idx) { return stats_[client_idx < 0 ? 0 : client_idx % MAX_CLIENTS]; }

    /** Resolves the CUDA events recorded around profiled ops into g_profiler. */
    void flush_profile();
    /** Creates n timing events for profiled ops up front: creating a CUDA event
     *  can block the calling thread for milliseconds while other clients'
     *  work is in flight, so workers take events from this pool. */
    void reserve_profile_events(int n);

    std::atomic<bool> running_{false};

    // Streams the workers fall back to when an op carries no stream.
    cudaStream_t hp_stream_{nullptr};
    std::vector<cudaStream_t> be_streams_;

private:
    void run_worker(int client_idx);
    cudaError_t execute_operation(OperationPtr op, cudaStream_t fallback_stream);
    bool orion_should_schedule(OperationPtr op, int client_idx);
    bool create_streams();
    void destroy_streams();
    int peek_sm_requirement(int client_idx, int offset = 0);
    /** Table duration (ns) of the client's next kernel; 0 without a table. */
    float peek_duration(int client_idx);
    double estimate_client_time_ns(int client_idx, unsigned int allocated_sms) const;
    void hp_activity_begin();
    void hp_activity_poll();

    SchedulerConfig config_;
    std::vector<std::thread> workers_;
    std::atomic<bool> initialized_{false};
    int num_clients_{0};
    bool isolated_{false};
    GreenCtxConfig gc_config_;

    // HP flag in pinned, device-mapped host memory (read by BE kernels).
    volatile int* hp_flag_host_{nullptr};
    int* hp_flag_dev_{nullptr};
    // Copy of hp_flag_host_[0] in device memory: the flag BE kernels poll.
    // Device reads of pinned host memory cross PCIe and serialise when many
    // CTAs poll at once, so the kernels read this copy, which the scheduler
    // updates with an async copy on flag_stream_ whenever the flag changes.
    int* hp_flag_devmem_{nullptr};
    // HP idle hysteresis: the flag drops only after HP has been idle this long
    int64_t hp_idle_since_ns_{0};
    int64_t hp_hold_ns_{1000000};
    // Longest table duration of a BE kernel that may share SMs with an active
    // HP client (KX_BE_MAX_US, default 50 us); longer ones wait for HP to idle.
    float be_max_ns_{50000.0f};
    std::atomic<long long> be_host_hold_ns_{3000000};
    long long be_host_window_ns_{500000};
    std::atomic<int> profile_every_{1};            // see execute_operation
    std::atomic<uint64_t> prof_seq_[MAX_CLIENTS];  // dense ops per client
    std::atomic<long long> hp_last_issue_ns_{-(1LL << 60)};
    cudaStream_t flag_stream_{nullptr};
    void publish_hp_flag(int value);
    std::atomic<int> be_keep_sms_{0};
    cudaEvent_t hp_last_event_{nullptr};
    std::atomic<bool> hp_event_pending_{false};
    std::mutex hp_mu_;

    ClientStats stats_[MAX_CLIENTS];

    struct PendingProfile {
        cudaEvent_t start, end;
        KernelProfile rec;
    };
    std::mutex prof_mu_;
    std::vector<PendingProfile> pending_prof_;
    std::atomic<bool> profile_launches_{false};
    std::vector<cudaEvent_t> prof_events_;  // free timing events (guarded by prof_mu_)
    cudaEvent_t take_profile_event();
};

extern Scheduler g_scheduler;

bool start_scheduler(int num_clients, const SchedulerConfig& config = SchedulerConfig());
void stop_scheduler();

}  // namespace orion

extern "C" {

int orion_start_scheduler(int num_clients);
void orion_stop_scheduler();
int orion_load_kernel_info(int client_idx, const char* file_path);
void orion_set_client_kernels(int client_idx, int num_kernels);
void orion_set_sm_threshold(int threshold);
int orion_get_sm_threshold();
void orion_sync_client_stream(int client_idx);
void orion_reset_state();
int orion_autotune_green_ctx();

// Exported by the reference without a header declaration (src/scheduler.cpp:1382-1398).
int orion_init_scheduler(int num_clients);
int orion_start_scheduler_thread();

// Additions of this build.
/** SMs BE kernels keep while HP work is in flight (DEFAULT mode). */
void orion_set_be_keep_sms(int sms);
/** Addition: 1 = profiling sessions (orion_start_profiling) also record every
 *  kernel the interposer re-issues (name, SMs its grid fills, device time),
 *  for per-client kernel tables; 0 (default) = captured dense ops only. */
void orion_set_profile_launches(int on);
int orion_get_be_keep_sms();
/** Fixed HP / BE SM budgets (ISOLATED mode); 0,0 returns to DEFAULT. */
int orion_set_sm_budgets(int hp_sms, int be_sms);
/** Counters of one client: ops, kx_ops, passthrough_ops, be_blocked, yields, errors. */
int orion_get_client_stats(int client_idx, unsigned long long* out6);
/** Longest time (us) a BE client thread waits before queueing an op while the
 *  HP client is issuing (Scheduler::be_issue_gate); 0 = never waits. */
void orion_set_be_host_hold_us(int us);
int orion_get_be_host_hold_us();
/** Ops of one BE client whose thread waited at the issue gate. */
unsigned long long orion_get_client_host_holds(int client_idx);
/** Addition: profiling sessions time one in n captured dense ops of each
 *  client, picked by a hash of the op's sequence number (default 1: every op;
 *  ORION_PROFILE_EVERY sets the initial value). */
void orion_set_profile_every(int n);
/** Called by the reference's launch_jobs.py; synchronises the client's stream. */
void block(int client_idx);
}

#endif  // ORION_SCHEDULER_H
