/**
 * @file kernel_profile.h
 * @brief Kernel profile tables (JSON / YAML) and the in-process profiler.
 *
 * Same declarations as the reference's include/kernel_profile.h.  The live
 * scheduling format remains kernel_info.csv (Name,Profile,Memory_footprint,
 * SM_usage,Duration), read by orion_load_kernel_info (scheduler.h); these
 * tables serve orion_load_profile / orion_start_profiling /
 * orion_end_profiling.  In this build KernelProfiler::record_kernel is fed by
 * the workers: every kx dispatch records its kernel name, measured duration
 * (CUDA events, when profiling is on) and SM quota.
 */
#ifndef ORION_KERNEL_PROFILE_H
#define ORION_KERNEL_PROFILE_H

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace orion {

struct KernelProfile {
    std::string kernel_id;
    float duration_ms;
    int sm_needed;
    ProfileType profile_type;
    int grid_size;
    int block_size;
    size_t shared_mem_bytes;
    // additions: client, captured op type and its algorithmic work (FLOPs or bytes)
    int client_idx;
    std::string op_type;
    double work;

    KernelProfile()
        : duration_ms(0.0f), sm_needed(0), profile_type(ProfileType::UNKNOWN), grid_size(0),
          block_size(0), shared_mem_bytes(0), client_idx(-1), work(0.0) {}
};

class KernelProfileTable {
public:
    KernelProfileTable();
    ~KernelProfileTable() = default;

    bool load_from_json(const std::string& filepath);
    bool load_from_yaml(const std::string& filepath);
    const KernelProfile* find(const std::string& kernel_id) const;
    void add(const KernelProfile& profile);
    void clear();
    const std::unordered_map<std::string, KernelProfile>& get_all() const { return profiles_; }
    float compute_average_duration() const;
    float compute_recommended_dur_threshold(float target_ratio = 0.025f) const;
    size_t size() const { return profiles_.size(); }

private:
    std::unordered_map<std::string, KernelProfile> profiles_;
    mutable std::mutex mutex_;
};

class KernelProfiler {
public:
    KernelProfiler();
    ~KernelProfiler();

    void start_session(const std::string& model_name);
    void end_session(const std::string& output_path);
    void record_kernel(const std::string& kernel_id, float duration_ms, int sm_needed,
                       ProfileType profile_type);
    void record(const KernelProfile& p);
    void get_profile_table(KernelProfileTable& table) const;
    bool active() const { return session_active_; }

private:
    std::string model_name_;
    std::vector<KernelProfile> recorded_profiles_;
    bool session_active_;
    mutable std::mutex mutex_;
};

extern KernelProfiler g_profiler;

}  // namespace orion

extern "C" {
int orion_load_profile(const char* filepath);
void orion_start_profiling(const char* model_name);
void orion_end_profiling(const char* output_path);
}

#endif  // ORION_KERNEL_PROFILE_H
