// kernel_profile.cpp — JSON / YAML kernel profile tables and the in-process
// profiler (orion_load_profile / orion_start_profiling / orion_end_profiling).
//
// File formats follow the reference (include/kernel_profile.h:95-123 and
// src/kernel_profile.cpp:152-340 of the reference): a "kernels" array of
// objects with kernel_id, duration_ms, sm_needed, profile_type
// ("compute" | "memory"), grid_size, block_size.  The parser here is a small
// tokenizer of its own.
#include "kernel_profile.h"

#include "scheduler.h"

#include <algorithm>
#include <cctype>
#include <cstdlib>
#include <fstream>
#include <sstream>

namespace orion {

KernelProfiler g_profiler;

namespace {

ProfileType parse_profile_type(const std::string& v) {
  if (v == "compute" || v == "compute_bound" || v == "1") return ProfileType::COMPUTE_BOUND;
  if (v == "memory" || v == "memory_bound" || v == "0") return ProfileType::MEMORY_BOUND;
  return ProfileType::UNKNOWN;
}

const char* profile_type_str(ProfileType t) {
  switch (t) {
    case ProfileType::COMPUTE_BOUND: return "compute";
    case ProfileType::MEMORY_BOUND: return "memory";
    default: return "unknown";
  }
}

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && (std::isspace(static_cast<unsigned char>(s[a])) || s[a] == '"' || s[a] == '\''))
    ++a;
  while (b > a &&
         (std::isspace(static_cast<unsigned char>(s[b - 1])) || s[b - 1] == '"' ||
          s[b - 1] == '\'' || s[b - 1] == ','))
    --b;
  return s.substr(a, b - a);
}

void assign_field(KernelProfile& p, const std::string& key, const std::string& val) {
  if (key == "kernel_id") p.kernel_id = val;
  else if (key == "duration_ms") p.duration_ms = std::strtof(val.c_str(), nullptr);
  else if (key == "sm_needed") p.sm_needed = std::atoi(val.c_str());
  else if (key == "profile_type") p.profile_type = parse_profile_type(val);
  else if (key == "grid_size") p.grid_size = std::atoi(val.c_str());
  else if (key == "block_size") p.block_size = std::atoi(val.c_str());
  else if (key == "shared_mem_bytes") p.shared_mem_bytes = std::strtoull(val.c_str(), nullptr, 10);
}

// Splits a flat JSON object body `"k": v, "k2": "v2"` into key/value pairs.
void parse_json_object(const std::string& body, KernelProfile& p) {
  size_t i = 0;
  while (i < body.size()) {
    size_t k0 = body.find('"', i);
    if (k0 == std::string::npos) break;
    size_t k1 = body.find('"', k0 + 1);
    if (k1 == std::string::npos) break;
    const std::string key = body.substr(k0 + 1, k1 - k0 - 1);
    size_t colon = body.find(':', k1);
    if (colon == std::string::npos) break;
    size_t v0 = colon + 1;
    while (v0 < body.size() && std::isspace(static_cast<unsigned char>(body[v0]))) ++v0;
    size_t v1;
    if (v0 < body.size() && body[v0] == '"') {
      v1 = body.find('"', v0 + 1);
      if (v1 == std::string::npos) break;
      assign_field(p, key, body.substr(v0 + 1, v1 - v0 - 1));
      i = v1 + 1;
    } else {
      v1 = body.find_first_of(",}", v0);
      if (v1 == std::string::npos) v1 = body.size();
      assign_field(p, key, trim(body.substr(v0, v1 - v0)));
      i = v1 + 1;
    }
  }
}

}  // namespace

KernelProfileTable::KernelProfileTable() = default;

bool KernelProfileTable::load_from_json(const std::string& filepath) {
  std::ifstream f(filepath);
  if (!f.is_open()) {
    LOG_ERROR("failed to open profile file %s", filepath.c_str());
    return false;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  const std::string text = ss.str();
  size_t at = text.find("\"kernels\"");
  if (at == std::string::npos) {
    LOG_ERROR("no \"kernels\" array in %s", filepath.c_str());
    return false;
  }
  at = text.find('[', at);
  if (at == std::string::npos) return false;
  std::lock_guard<std::mutex> lk(mutex_);
  size_t pos = at + 1;
  while (pos < text.size()) {
    size_t ob = text.find_first_of("{]", pos);
    if (ob == std::string::npos || text[ob] == ']') break;
    size_t cb = text.find('}', ob);
    if (cb == std::string::npos) break;
    KernelProfile p;
    parse_json_object(text.substr(ob + 1, cb - ob - 1), p);
    if (!p.kernel_id.empty()) profiles_[p.kernel_id] = p;
    pos = cb + 1;
  }
  return true;
}

bool KernelProfileTable::load_from_yaml(const std::string& filepath) {
  std::ifstream f(filepath);
  if (!f.is_open()) {
    LOG_ERROR("failed to open profile file %s", filepath.c_str());
    return false;
  }
  std::lock_guard<std::mutex> lk(mutex_);
  std::string line;
  bool in_kernels = false;
  KernelProfile cur;
  bool have = false;
  auto flush = [&] {
    if (have && !cur.kernel_id.empty()) profiles_[cur.kernel_id] = cur;
    cur = KernelProfile();
    have = false;
  };
  while (std::getline(f, line)) {
    const size_t hash = line.find('#');
    if (hash != std::string::npos) line = line.substr(0, hash);
    if (trim(line).empty()) continue;
    if (line.find("kernels:") != std::string::npos) {
      in_kernels = true;
      continue;
    }
    if (!in_kernels) continue;
    std::string t = line;
    const size_t dash = t.find_first_not_of(" \t");
    if (dash != std::string::npos && t[dash] == '-') {
      flush();
      have = true;
      t = t.substr(dash + 1);
    }
    const size_t colon = t.find(':');
    if (colon == std::string::npos) continue;
    assign_field(cur, trim(t.substr(0, colon)), trim(t.substr(colon + 1)));
    have = true;
  }
  flush();
  return true;
}

const KernelProfile* KernelProfileTable::find(const std::string& kernel_id) const {
  std::lock_guard<std::mutex> lk(mutex_);
  auto it = profiles_.find(kernel_id);
  return it == profiles_.end() ? nullptr : &it->second;
}

void KernelProfileTable::add(const KernelProfile& profile) {
  std::lock_guard<std::mutex> lk(mutex_);
  profiles_[profile.kernel_id] = profile;
}

void KernelProfileTable::clear() {
  std::lock_guard<std::mutex> lk(mutex_);
  profiles_.clear();
}

float KernelProfileTable::compute_average_duration() const {
  std::lock_guard<std::mutex> lk(mutex_);
  if (profiles_.empty()) return 0.f;
  double s = 0.0;
  for (const auto& kv : profiles_) s += kv.second.duration_ms;
  return static_cast<float>(s / profiles_.size());
}

float KernelProfileTable::compute_recommended_dur_threshold(float target_ratio) const {
  // Orion's rule: BE kernels may run while their expected duration stays
  // within a small fraction of the HP request latency (sum of HP kernels).
  std::lock_guard<std::mutex> lk(mutex_);
  double total = 0.0;
  for (const auto& kv : profiles_) total += kv.second.duration_ms;
  return static_cast<float>(total * target_ratio);
}

KernelProfiler::KernelProfiler() : session_active_(false) {}

KernelProfiler::~KernelProfiler() = default;

void KernelProfiler::start_session(const std::string& model_name) {
  std::lock_guard<std::mutex> lk(mutex_);
  model_name_ = model_name;
  recorded_profiles_.clear();
  session_active_ = true;
}

void KernelProfiler::end_session(const std::string& output_path) {
  std::lock_guard<std::mutex> lk(mutex_);
  session_active_ = false;
  if (output_path.empty()) return;
  std::ofstream f(output_path);
  if (!f.is_open()) {
    LOG_ERROR("failed to open %s", output_path.c_str());
    return;
  }
  f << "{\n  \"model_name\": \"" << model_name_ << "\",\n  \"kernels\": [\n";
  for (size_t i = 0; i < recorded_profiles_.size(); ++i) {
    const KernelProfile& p = recorded_profiles_[i];
    std::string id;  // JSON string escaping of the kernel name
    for (char ch : p.kernel_id) {
      if (ch == '"' || ch == '\\') id.push_back('\\');
      if (static_cast<unsigned char>(ch) >= 0x20) id.push_back(ch);
    }
    f << "    {\"kernel_id\": \"" << id << "\", \"duration_ms\": " << p.duration_ms
      << ", \"sm_needed\": " << p.sm_needed << ", \"profile_type\": \""
      << profile_type_str(p.profile_type) << "\", \"grid_size\": " << p.grid_size
      << ", \"block_size\": " << p.block_size << ", \"client\": " << p.client_idx
      << ", \"op_type\": \"" << p.op_type << "\", \"work\": " << p.work << "}"
      << (i + 1 < recorded_profiles_.size() ? "," : "") << "\n";
  }
  f << "  ]\n}\n";
}

void KernelProfiler::record_kernel(const std::string& kernel_id, float duration_ms,
                                   int sm_needed, ProfileType profile_type) {
  std::lock_guard<std::mutex> lk(mutex_);
  if (!session_active_) return;
  KernelProfile p;
  p.kernel_id = kernel_id;
  p.duration_ms = duration_ms;
  p.sm_needed = sm_needed;
  p.profile_type = profile_type;
  p.grid_size = sm_needed;
  p.block_size = 256;
  recorded_profiles_.push_back(p);
}

void KernelProfiler::record(const KernelProfile& p) {
  std::lock_guard<std::mutex> lk(mutex_);
  if (session_active_) recorded_profiles_.push_back(p);
}

void KernelProfiler::get_profile_table(KernelProfileTable& table) const {
  std::lock_guard<std::mutex> lk(mutex_);
  table.clear();
  for (const auto& p : recorded_profiles_) table.add(p);
}

}  // namespace orion

extern "C" {

int orion_load_profile(const char* filepath) {
  static orion::KernelProfileTable table;
  if (filepath == nullptr) return -1;
  const std::string path(filepath);
  if (path.find(".yaml") != std::string::npos || path.find(".yml") != std::string::npos)
    return table.load_from_yaml(path) ? 0 : -1;
  return table.load_from_json(path) ? 0 : -1;
}

void orion_start_profiling(const char* model_name) {
  // timing events for the profiled ops, made here rather than by the workers
  if (orion::g_scheduler.running_.load()) orion::g_scheduler.reserve_profile_events(16384);
  orion::g_profiler.start_session(model_name ? model_name : "unnamed");
}

void orion_end_profiling(const char* output_path) {
  orion::g_scheduler.flush_profile();
  orion::g_profiler.end_session(output_path ? output_path : "");
}

}  // extern "C"
