// scheduler.cpp — Orion-style HP/BE scheduler on SM-quota-aware kx kernels.
//
// One worker thread per client pops that client's captured operations in
// FIFO order and runs them on the stream the client issued them on.  Client 0
// is high priority (HP); clients 1.. are best effort (BE).
//
//  * Admission (orion_should_schedule) keeps the reference's profile-table
//    rule (src/scheduler.cpp:997-1034 of the reference): a BE kernel op runs
//    when HP's next kernel plus this BE kernel fit in the GPU's SMs according
//    to kernel_info.csv, or when the HP queue is empty; otherwise it waits.
//  * Sharing (replaces the green-context split, src/scheduler.cpp:244-446):
//    dense BE ops run as persistent kx kernels that read the HP flag before
//    every tile (a device-memory copy of the pinned host flag, updated by an
//    async copy whenever the flag changes).  The HP worker raises the flag to
//    be_keep_sms while HP work is queued or in flight; BE CTAs whose index is
//    at or above it retire at their next tile boundary and the lower ones
//    finish the op.  With be_keep_sms = 0 the flag is -1: every BE CTA stops
//    and the BE worker relaunches the op (same arguments, continuing from its
//    tile queue) once HP is idle.  ISOLATED mode instead gives HP and BE fixed
//    disjoint SM budgets (hp_sm_count / be_sm_count).
//  * kernel_info.csv rows are parsed right-to-left (Name may contain commas),
//    as in the reference (src/scheduler.cpp:84-153).
#include "scheduler.h"

#include <cuda.h>
#include <dlfcn.h>

#include <sys/prctl.h>
#include <time.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "dispatch.h"
#include "real_libs.h"

namespace orion {

Scheduler g_scheduler;
OrionSchedulingState g_orion_state;

namespace {

bool is_memory_op(OperationType t) {
  return t == OperationType::MALLOC || t == OperationType::FREE ||
         t == OperationType::MEMCPY || t == OperationType::MEMCPY_ASYNC ||
         t == OperationType::MEMSET || t == OperationType::MEMSET_ASYNC;
}

bool is_kernel_op(OperationType t) {
  return t == OperationType::KERNEL_LAUNCH || t == OperationType::KERNEL_LAUNCH_EX ||
         t == OperationType::KERNEL_LAUNCH_DRV || is_dense_op(t);
}

int64_t mono_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return static_cast<int64_t>(ts.tv_sec) * 1000000000LL + ts.tv_nsec;
}

cudaStream_t op_stream(const OperationRecord& op) {
  switch (op.type) {
    case OperationType::KERNEL_LAUNCH:
    case OperationType::KERNEL_LAUNCH_EX:
    case OperationType::KERNEL_LAUNCH_DRV:
      return std::get<KernelLaunchParams>(op.params).stream;
    case OperationType::MEMCPY_ASYNC:
      return std::get<MemcpyParams>(op.params).stream;
    case OperationType::MEMSET_ASYNC:
      return std::get<MemsetParams>(op.params).stream;
    case OperationType::CUBLAS_SGEMM:
    case OperationType::CUBLAS_SGEMM_BATCHED:
    case OperationType::CUBLAS_SGEMM_STRIDED_BATCHED:
    case OperationType::CUBLAS_GEMM_EX:
    case OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX:
      return std::get<CublasGemmParams>(op.params).stream;
    case OperationType::CUBLASLT_MATMUL:
      return std::get<CublasLtMatmulParams>(op.params).stream;
    case OperationType::CUDNN_CONV_FWD:
    case OperationType::CUDNN_CONV_BWD_DATA:
    case OperationType::CUDNN_CONV_BWD_FILTER:
      return std::get<CudnnConvParams>(op.params).stream;
    case OperationType::CUDNN_BATCHNORM_FWD:
    case OperationType::CUDNN_BATCHNORM_BWD:
    case OperationType::CUDNN_BATCHNORM_INF:
      return std::get<CudnnBatchNormParams>(op.params).stream;
    default:
      return nullptr;
  }
}

// Algorithmic work of a captured dense op: FLOPs for GEMMs / convolutions,
// HBM bytes for batch norm (the units its roofline uses).
double op_work(const OperationRecord& op) {
  switch (op.type) {
    case OperationType::CUBLAS_SGEMM:
    case OperationType::CUBLAS_GEMM_EX: {
      const auto& p = std::get<CublasGemmParams>(op.params);
      return 2.0 * p.m * p.n * p.k;
    }
    case OperationType::CUBLAS_SGEMM_BATCHED:
    case OperationType::CUBLAS_SGEMM_STRIDED_BATCHED:
    case OperationType::CUBLAS_GEMM_STRIDED_BATCHED_EX: {
      const auto& p = std::get<CublasGemmParams>(op.params);
      return 2.0 * p.m * p.n * p.k * p.batchCount;
    }
    case OperationType::CUBLASLT_MATMUL: {
      const auto& d = std::get<CublasLtMatmulParams>(op.params).dec;
      return 2.0 * d.m * d.n * d.k * (d.batch > 0 ? d.batch : 1);
    }
    case OperationType::CUDNN_CONV_FWD:
    case OperationType::CUDNN_CONV_BWD_DATA:
    case OperationType::CUDNN_CONV_BWD_FILTER: {
      const ConvGeometry& g = std::get<CudnnConvParams>(op.params).geom;
      const int P = (g.h + 2 * g.pad_h - ((g.r - 1) * g.dil_h + 1)) / g.stride_h + 1;
      const int Q = (g.w + 2 * g.pad_w - ((g.s - 1) * g.dil_w + 1)) / g.stride_w + 1;
      return 2.0 * g.n * g.k * g.c * g.r * g.s * P * Q;
    }
    case OperationType::CUDNN_BATCHNORM_FWD:
    case OperationType::CUDNN_BATCHNORM_INF:
    case OperationType::CUDNN_BATCHNORM_BWD: {
      const auto& p = std::get<CudnnBatchNormParams>(op.params);
      const double elems = static_cast<double>(p.n) * p.c * p.h * p.w;
      const double passes = op.type == OperationType::CUDNN_BATCHNORM_INF ? 2.0
                            : op.type == OperationType::CUDNN_BATCHNORM_FWD ? 3.0 : 5.0;
      return passes * elems * 4.0;
    }
    default:
      return 0.0;
  }
}

int populate_kernel_info(int client_idx, const std::string& path) {
  std::ifstream f(path);
  if (!f.is_open()) {
    LOG_ERROR("failed to open kernel_info file %s", path.c_str());
    return -1;
  }
  std::vector<KernelProfileInfo> rows;
  std::string line;
  bool header = true;
  while (std::getline(f, line)) {
    if (header) {
      header = false;
      continue;
    }
    if (!line.empty() && line.back() == '\r') line.pop_back();
    if (line.empty()) continue;
    // last four comma-separated fields are numeric; the name is the rest
    size_t cut[4];
    size_t pos = line.size();
    bool ok = true;
    for (int i = 3; i >= 0; --i) {
      size_t c = line.rfind(',', pos == 0 ? std::string::npos : pos - 1);
      if (c == std::string::npos) {
        ok = false;
        break;
      }
      cut[i] = c;
      pos = c;
    }
    if (!ok) continue;
    try {
      KernelProfileInfo info;
      info.name = line.substr(0, cut[0]);
      info.profile = std::stoi(line.substr(cut[0] + 1, cut[1] - cut[0] - 1));
      info.mem = std::stoi(line.substr(cut[1] + 1, cut[2] - cut[1] - 1));
      info.sm_used = std::stoi(line.substr(cut[2] + 1, cut[3] - cut[2] - 1));
      info.duration = std::stof(line.substr(cut[3] + 1));
      rows.push_back(info);
    } catch (...) {
      continue;
    }
  }
  std::lock_guard<std::mutex> lk(g_orion_state.mutex);
  if (client_idx < 0 || client_idx >= static_cast<int>(g_orion_state.op_info_vector.size()))
    return -1;
  g_orion_state.op_info_vector[client_idx] = std::move(rows);
  return static_cast<int>(g_orion_state.op_info_vector[client_idx].size());
}

}  // namespace

Scheduler::Scheduler() = default;

Scheduler::~Scheduler() {
  stop();
  join();
}

bool Scheduler::init(int num_clients, const SchedulerConfig& config) {
  if (initialized_.load()) return true;
  num_clients_ = num_clients;
  config_ = config;
  int dev = config_.device_id;
  ORION_REAL(cudart, cudaGetDevice)(&dev);
  config_.device_id = dev;
  int sms = 0;
  if (ORION_REAL(cudart, cudaDeviceGetAttribute)(&sms, cudaDevAttrMultiProcessorCount, dev) !=
      cudaSuccess) {
    LOG_ERROR("cannot query the device's SM count");
    return false;
  }
  config_.num_sms = sms;
  if (config_.sm_threshold == 0) config_.sm_threshold = sms / 2;
  if (!create_streams()) return false;
  // HP flag shared with BE kernels (pinned, device-mapped)
  int* h = nullptr;
  int* d = nullptr;
  // [0] = HP flag; [c] = done flag of BE client c's stoppable op (one per
  // client: BE workers relaunch their own ops independently)
  if (kx_host_flags_alloc(1 + MAX_CLIENTS, &h, &d) != KX_OK) {
    LOG_ERROR("cannot allocate the HP flag");
    return false;
  }
  hp_flag_host_ = h;
  hp_flag_dev_ = d;
  if (ORION_REAL(cudart, cudaMalloc)(reinterpret_cast<void**>(&hp_flag_devmem_), sizeof(int)) !=
          cudaSuccess ||
      ORION_REAL(cudart, cudaMemset)(hp_flag_devmem_, 0, sizeof(int)) != cudaSuccess) {
    LOG_ERROR("cannot allocate the device copy of the HP flag");
    return false;
  }
  {
    int lo = 0, hi = 0;
    ORION_REAL(cudart, cudaDeviceGetStreamPriorityRange)(&lo, &hi);
    ORION_REAL(cudart, cudaStreamCreateWithPriority)(&flag_stream_, cudaStreamNonBlocking, hi);
  }
  // 0: BE GEMMs / convolutions stop at their next tile boundary while HP
  // works and are relaunched from their tile queues once it idles.  Measured
  // on the LLaMA-HP / VGG16 + GPT-BE group: paced HP p99 1.07x solo with BE
  // keeping 0.72 / 0.66 of its rate, against 1.00x and 0.49 / 2.3 with 4 SMs
  // kept per BE client (an op caught by HP then finishes on those 4 SMs).
  int keep = 0;
  if (const char* s = std::getenv("KX_BE_KEEP_SMS")) keep = std::atoi(s);
  be_keep_sms_.store(std::max(0, std::min(keep, sms)));
  if (const char* s = std::getenv("KX_HP_HOLD_US")) hp_hold_ns_ = std::max(0LL, std::atoll(s)) * 1000;
  if (const char* s = std::getenv("KX_BE_MAX_US")) be_max_ns_ = std::max(0.0f, std::strtof(s, nullptr)) * 1000.f;
  if (const char* s = std::getenv("KX_BE_HOST_HOLD_US"))
    be_host_hold_ns_.store(std::max(0LL, std::atoll(s)) * 1000);
  if (const char* s = std::getenv("KX_BE_HOST_WINDOW_US"))
    be_host_window_ns_ = std::max(0LL, std::atoll(s)) * 1000;
  if (const char* s = std::getenv("ORION_PROFILE_EVERY")) set_profile_every(std::atoi(s));
  ORION_REAL(cudart, cudaEventCreateWithFlags)(&hp_last_event_, cudaEventDisableTiming);
  g_orion_state.init(num_clients, sms);
  g_orion_state.sm_threshold = config_.sm_threshold;
  const char* hp = std::getenv("ORION_HP_SMS");
  const char* be = std::getenv("ORION_BE_SMS");
  if (hp && be) {
    GreenCtxConfig gc;
    gc.hp_sm_count = static_cast<unsigned>(std::atoi(hp));
    gc.be_sm_count = static_cast<unsigned>(std::atoi(be));
    gc.enabled = gc.hp_sm_count > 0 && gc.be_sm_count > 0;
    if (gc.enabled) init_green_contexts(gc);
  }
  initialized_.store(true);
  LOG_INFO("scheduler initialized: %d clients, %d SMs, BE keeps %d SMs under HP load",
           num_clients, sms, be_keep_sms_.load());
  return true;
}

bool Scheduler::create_streams() {
  int lo = 0, hi = 0;
  ORION_REAL(cudart, cudaDeviceGetStreamPriorityRange)(&lo, &hi);
  auto create = ORION_REAL(cudart, cudaStreamCreateWithPriority);
  if (create(&hp_stream_, cudaStreamNonBlocking, hi) != cudaSuccess) return false;
  be_streams_.assign(std::max(0, num_clients_ - 1), nullptr);
  for (size_t i = 0; i < be_streams_.size(); ++i)
    if (create(&be_streams_[i], cudaStreamNonBlocking, lo) != cudaSuccess) return false;
  return true;
}

void Scheduler::destroy_streams() {
  auto destroy = ORION_REAL(cudart, cudaStreamDestroy);
  if (hp_stream_) destroy(hp_stream_);
  hp_stream_ = nullptr;
  for (auto s : be_streams_)
    if (s) destroy(s);
  be_streams_.clear();
}

bool Scheduler::init_green_contexts(const GreenCtxConfig& gc) {
  const unsigned total = static_cast<unsigned>(config_.num_sms);
  if (!gc.enabled || gc.hp_sm_count == 0 || gc.be_sm_count == 0 ||
      gc.hp_sm_count + gc.be_sm_count > total) {
    LOG_ERROR("invalid SM budgets HP=%u BE=%u (GPU has %u SMs)", gc.hp_sm_count,
              gc.be_sm_count, total);
    return false;
  }
  gc_config_ = gc;
  isolated_ = true;
  LOG_INFO("ISOLATED mode: HP budget %u SMs, BE budget %u SMs", gc.hp_sm_count, gc.be_sm_count);
  return true;
}

int Scheduler::hp_quota() const { return isolated_ ? static_cast<int>(gc_config_.hp_sm_count) : 0; }

int Scheduler::be_quota() const { return isolated_ ? static_cast<int>(gc_config_.be_sm_count) : 0; }

double Scheduler::estimate_client_time_ns(int client_idx, unsigned int allocated_sms) const {
  // Wave model: a kernel needing S SMs run on A < S SMs takes ceil(S/A) waves.
  auto& rows = g_orion_state.op_info_vector[client_idx];
  double t = 0.0;
  const unsigned a = std::max(1u, allocated_sms);
  for (const auto& r : rows) {
    const unsigned need = static_cast<unsigned>(std::max(1, r.sm_used));
    const double waves = std::ceil(static_cast<double>(need) / a);
    t += r.duration * (need > a ? waves : 1.0);
  }
  return t;
}

Scheduler::GreenCtxConfig Scheduler::choose_best_green_ctx_config_from_profiles() const {
  // Minimise the slower of HP and the slowest BE client over budgets in steps
  // of 8 SMs (the granularity the reference's green contexts used).
  GreenCtxConfig best;
  best.enabled = false;
  const unsigned total = static_cast<unsigned>(config_.num_sms);
  double best_t = 1e300;
  for (unsigned hp = 8; hp + 8 <= total; hp += 8) {
    const unsigned be = total - hp;
    double t_hp = estimate_client_time_ns(0, hp);
    double t_be = 0.0;
    for (int c = 1; c < num_clients_; ++c) t_be = std::max(t_be, estimate_client_time_ns(c, be));
    const double t = std::max(t_hp, t_be);
    if (t < best_t) {
      best_t = t;
      best.hp_sm_count = hp;
      best.be_sm_count = be;
      best.enabled = true;
    }
  }
  return best;
}

int Scheduler::autotune_green_ctx() {
  GreenCtxConfig gc = choose_best_green_ctx_config_from_profiles();
  if (!gc.enabled) return -1;
  return init_green_contexts(gc) ? 0 : -1;
}

int Scheduler::peek_sm_requirement(int client_idx, int offset) {
  std::lock_guard<std::mutex> lk(g_orion_state.mutex);
  if (client_idx < 0 || client_idx >= static_cast<int>(g_orion_state.op_info_vector.size()))
    return 0;
  auto& rows = g_orion_state.op_info_vector[client_idx];
  if (rows.empty()) return 0;
  const int n = static_cast<int>(rows.size());
  const int idx = ((g_orion_state.seen[client_idx] + offset) % n + n) % n;
  return rows[idx].sm_used;
}

float Scheduler::peek_duration(int client_idx) {
  std::lock_guard<std::mutex> lk(g_orion_state.mutex);
  if (client_idx < 0 || client_idx >= static_cast<int>(g_orion_state.op_info_vector.size()))
    return 0.f;
  auto& rows = g_orion_state.op_info_vector[client_idx];
  if (rows.empty()) return 0.f;
  const int n = static_cast<int>(rows.size());
  const int idx = ((g_orion_state.seen[client_idx]) % n + n) % n;
  return rows[idx].duration;
}

// Admission of a BE kernel op (the reference's rule, src/scheduler.cpp:997-1034:
// run when HP's next kernel and this one fit in the SMs together, or when HP
// has nothing queued), with two changes for kernels that cannot yield:
//  * HP counts as active while its flag is raised, not only while its queue
//    holds ops: a request's ops reach the queue one at a time, and a BE
//    kernel admitted into such a gap holds the SMs HP's next kernel needs;
//  * a BE kernel that does not fit beside HP's next one may still run when its
//    table duration is at most be_max_ns_ (it delays HP by that much at most).
// Captured dense BE ops are always admitted: they run as persistent kx kernels
// that leave the SMs above the HP flag at their next tile boundary.
bool Scheduler::orion_should_schedule(OperationPtr op, int client_idx) {
  if (is_memory_op(op->type) || !is_kernel_op(op->type)) return true;
  if (isolated_) return true;  // disjoint budgets: no interference to arbitrate
  if (is_dense_op(op->type)) return true;
  auto& q = g_capture_state.client_queues[0];
  const bool hp_active =
      (q && !q->empty()) || (hp_flag_host_ != nullptr && hp_flag_host_[0] != 0);
  if (!hp_active) return true;
  const int hp = peek_sm_requirement(0);
  const int be = peek_sm_requirement(client_idx);
  if (hp + be <= config_.num_sms) return true;
  const float dur = peek_duration(client_idx);
  return dur > 0.f && dur <= be_max_ns_;
}

namespace {
// splitmix64's finaliser (Steele, Lea, Flood 2014) over a sequence number,
// reduced to a 1-in-n pick that has no period of its own
bool sampled(uint64_t seq, int n) {
  uint64_t z = seq + 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z % static_cast<uint64_t>(n) == 0;
}

// PyGILState_Check of the interpreter hosting the process, if there is one
int (*gil_check_fn())() {
  static int (*fn)() = reinterpret_cast<int (*)()>(dlsym(RTLD_DEFAULT, "PyGILState_Check"));
  return fn;
}
}  // namespace

void Scheduler::be_issue_gate(int client_idx) {
  const long long hold = be_host_hold_ns_.load(std::memory_order_relaxed);
  if (client_idx <= 0 || hold <= 0 || isolated_) return;
  // HP is issuing while its client queued an op within the window
  const long long window = be_host_window_ns_;
  auto hp_issuing = [&] {
    return mono_ns() - hp_last_issue_ns_.load(std::memory_order_relaxed) < window;
  };
  if (!hp_issuing() || !running_.load()) return;
  // a thread that holds the interpreter lock (or a process without one)
  // never waits here: the HP thread would wait for it in turn
  auto chk = gil_check_fn();
  if (chk == nullptr || chk() != 0) return;
  stats(client_idx).host_holds.fetch_add(1);
  const int64_t deadline = mono_ns() + hold;
  while (hp_issuing() && running_.load() && mono_ns() < deadline)
    std::this_thread::sleep_for(std::chrono::microseconds(20));
}

void be_issue_gate(int client_idx, OperationType type) {
  // kernels only: allocations and copies may be issued under a lock (the
  // caching allocator's) that the HP thread also needs
  if (is_kernel_op(type)) g_scheduler.be_issue_gate(client_idx);
}

void Scheduler::note_hp_issue() {
  hp_last_issue_ns_.store(mono_ns(), std::memory_order_relaxed);
}

void note_hp_issue() { g_scheduler.note_hp_issue(); }

void Scheduler::publish_hp_flag(int value) {
  trace_marker(value != 0 ? "hp_flag_raise" : "hp_flag_clear", value);
  hp_flag_host_[0] = value;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  // the copy reads the pinned host value when it executes, so the latest
  // value always reaches the device copy
  if (hp_flag_devmem_ != nullptr && flag_stream_ != nullptr)
    ORION_REAL(cudart, cudaMemcpyAsync)(hp_flag_devmem_, const_cast<int*>(&hp_flag_host_[0]),
                                        sizeof(int), cudaMemcpyHostToDevice, flag_stream_);
}

void Scheduler::hp_activity_begin() {
  if (isolated_ || hp_flag_host_ == nullptr) return;
  hp_idle_since_ns_ = 0;
  // be_keep_sms is what all BE clients together keep: each BE op's CTAs
  // below its share stay, the others retire at their next tile boundary
  const int keep = be_keep_sms_.load();
  const int n_be = num_clients_ > 1 ? num_clients_ - 1 : 1;
  const int v = keep > 0 ? std::max(1, keep / n_be) : -1;
  if (hp_flag_host_[0] != v) publish_hp_flag(v);
}

void Scheduler::hp_activity_poll() {
  // Lower the flag once the HP queue is drained and HP's last op finished.
  if (hp_flag_host_ == nullptr || hp_flag_host_[0] == 0) return;
  auto& q = g_capture_state.client_queues[0];
  if (q && !q->empty()) return;
  std::lock_guard<std::mutex> lk(hp_mu_);
  if (hp_event_pending_.load()) {
    if (ORION_REAL(cudart, cudaEventQuery)(hp_last_event_) != cudaSuccess) return;
    hp_event_pending_.store(false);
  }
  // hold the flag a little longer: HP requests issue kernels with host gaps
  // between them, and a flag that drops in every gap lets BE retake the SMs
  const int64_t now = mono_ns();
  if (hp_idle_since_ns_ == 0) hp_idle_since_ns_ = now;
  if (now - hp_idle_since_ns_ < hp_hold_ns_) return;
  publish_hp_flag(0);
}

// Name and SM need of a kernel the interposer re-issues (profile tables):
// the function's name from the runtime / driver, and the SMs its grid fills
// at the occupancy the function reaches with its block and shared memory
// (total blocks / resident blocks per SM, at most every SM).
static void describe_launch(const KernelLaunchParams& p, int num_sms, std::string* name,
                            int* sm_needed, int* blocks, int* threads) {
  const long long b = static_cast<long long>(p.gridDim.x) * p.gridDim.y * p.gridDim.z;
  const int t = static_cast<int>(p.blockDim.x * p.blockDim.y * p.blockDim.z);
  int per_sm = 0;
  const char* nm = nullptr;
  size_t smem = p.sharedMem;
  if (p.api == 1 && p.ex_config != nullptr)
    smem = static_cast<const cudaLaunchConfig_t*>(p.ex_config)->dynamicSmemBytes;
  if (p.api == 2) {
    using NameFn = CUresult (*)(const char**, CUfunction);
    using OccFn = CUresult (*)(int*, CUfunction, int, size_t);
    auto fn = reinterpret_cast<CUfunction>(const_cast<void*>(p.func));
    if (auto get = ORION_REAL_T(cudadrv, NameFn, "cuFuncGetName")) get(&nm, fn);
    if (auto occ = ORION_REAL_T(cudadrv, OccFn, "cuOccupancyMaxActiveBlocksPerMultiprocessor"))
      occ(&per_sm, fn, t, smem);
  } else {
    using NameFn = cudaError_t (*)(const char**, const void*);
    using OccFn = cudaError_t (*)(int*, const void*, int, size_t);
    if (auto get = ORION_REAL_T(cudart, NameFn, "cudaFuncGetName"))
      if (get(&nm, p.func) != cudaSuccess) nm = nullptr;
    if (auto occ = ORION_REAL_T(cudart, OccFn, "cudaOccupancyMaxActiveBlocksPerMultiprocessor"))
      if (occ(&per_sm, p.func, t, smem) != cudaSuccess) per_sm = 0;
    ORION_REAL(cudart, cudaGetLastError)();
  }
  *name = nm != nullptr ? nm : "kernel";
  if (per_sm < 1) per_sm = 1;
  const long long need = (b + per_sm - 1) / per_sm;
  *sm_needed = static_cast<int>(need < num_sms ? (need < 1 ? 1 : need) : num_sms);
  *blocks = static_cast<int>(b < 0x7fffffffLL ? b : 0x7fffffffLL);
  *threads = t;
}

static bool is_launch_op(OperationType t) {
  return t == OperationType::KERNEL_LAUNCH || t == OperationType::KERNEL_LAUNCH_EX ||
         t == OperationType::KERNEL_LAUNCH_DRV;
}

cudaError_t Scheduler::execute_operation(OperationPtr op, cudaStream_t fallback) {
  op->started.store(true);
  const int c = op->client_idx;
  ClientStats& st = stats(c);
  st.ops.fetch_add(1);
  if (!is_dense_op(op->type)) {
    if (!(g_profiler.active() && profile_launches_.load() && is_launch_op(op->type)))
      return dispatch_runtime(*op, fallback);
    // profiled re-issued kernel: timed on its stream like the dense ops
    auto& kp = std::get<KernelLaunchParams>(op->params);
    cudaStream_t s = kp.stream ? kp.stream : fallback;
    if (op->type == OperationType::KERNEL_LAUNCH_EX && kp.ex_config != nullptr) {
      cudaStream_t cs = static_cast<const cudaLaunchConfig_t*>(kp.ex_config)->stream;
      s = cs ? cs : fallback;
    }
    PendingProfile pp;
    pp.start = take_profile_event();
    pp.end = take_profile_event();
    ORION_REAL(cudart, cudaEventRecord)(pp.start, s);
    const cudaError_t err = dispatch_runtime(*op, fallback);
    ORION_REAL(cudart, cudaEventRecord)(pp.end, s);
    describe_launch(kp, config_.num_sms, &pp.rec.kernel_id, &pp.rec.sm_needed, &pp.rec.grid_size,
                    &pp.rec.block_size);
    pp.rec.profile_type = ProfileType::UNKNOWN;
    pp.rec.client_idx = c;
    pp.rec.op_type = op_type_name(op->type);
    pp.rec.work = 0.0;
    std::lock_guard<std::mutex> lk(prof_mu_);
    pending_prof_.push_back(pp);
    return err;
  }

  ExecPolicy pol;
  pol.stream = op_stream(*op);
  if (pol.stream == nullptr) pol.stream = nullptr;  // legacy default stream of the client
  const bool be = c > 0;
  pol.sm_quota = be ? be_quota() : hp_quota();
  // DEFAULT mode with BE keeping k SMs under HP load: HP kernels take the
  // other SMs only, so an HP launch never queues behind BE CTAs that are
  // allowed to finish their op.
  const int keep = be_keep_sms_.load();
  if (!be && !isolated_ && keep > 0 && keep < config_.num_sms) pol.sm_quota = config_.num_sms - keep;
  // BE ops stop entirely under HP load when BE keeps no SMs; only the
  // persistent GEMM / convolution kernels report through the done flag
  // whether they finished or stopped (batch norm runs to completion)
  const bool persistent = op->type != OperationType::CUDNN_BATCHNORM_FWD &&
                          op->type != OperationType::CUDNN_BATCHNORM_BWD &&
                          op->type != OperationType::CUDNN_BATCHNORM_INF;
  const bool can_stop = be && !isolated_ && be_keep_sms_.load() <= 0 && persistent;
  if (be && !isolated_) pol.yield_flag = hp_flag_devmem_ ? hp_flag_devmem_ : hp_flag_dev_;
  if (can_stop) {
    hp_flag_host_[c] = -1;
    pol.done_flag = hp_flag_dev_ + c;
  }
  cudaEvent_t ev_start = nullptr, ev_end = nullptr;
  // a profiling session times one in n dense ops of each client (two events
  // around it), so a session over a timed region costs that region 1/n of
  // the event records (orion_set_profile_every, ORION_PROFILE_EVERY).  The
  // choice hashes the op's sequence number: a plain "every n-th op" aliases
  // with a step whose dense-op count is a multiple of n and then times the
  // same few layers of every step
  const int every = profile_every_.load(std::memory_order_relaxed);
  const bool profiling =
      g_profiler.active() && (every <= 1 || sampled(prof_seq_[c].fetch_add(1), every));
  if (profiling) {
    ev_start = take_profile_event();
    ev_end = take_profile_event();
    ORION_REAL(cudart, cudaEventRecord)(ev_start, pol.stream);
  }
  tl_in_scheduler_execution = true;
  int rc = dispatch_dense(*op, pol);
  while (rc == KX_OK && can_stop) {
    // BE op that may have stopped entirely: wait for it, then resume once HP is idle.
    ORION_REAL(cudart, cudaStreamSynchronize)(pol.stream);
    if (hp_flag_host_[c] == 1) break;
    st.yields.fetch_add(1);
    const int64_t deadline = mono_ns() + wait_timeout_ns();
    while (hp_flag_host_[0] != 0 && running_.load() && mono_ns() < deadline)
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    hp_flag_host_[c] = -1;
    rc = dispatch_dense(*op, pol);
  }
  tl_in_scheduler_execution = false;
  if (c == 0 && rc == KX_OK && !isolated_) {
    std::lock_guard<std::mutex> lk(hp_mu_);
    ORION_REAL(cudart, cudaEventRecord)(hp_last_event_, pol.stream);
    hp_event_pending_.store(true);
  }
  if (profiling) {
    // resolved without blocking the worker; see flush_profile()
    ORION_REAL(cudart, cudaEventRecord)(ev_end, pol.stream);
    PendingProfile pp;
    pp.start = ev_start;
    pp.end = ev_end;
    pp.rec.kernel_id = kx_last_kernel_name();
    pp.rec.sm_needed = pol.sm_quota > 0 ? pol.sm_quota : config_.num_sms;
    if (op->type != OperationType::CUDNN_BATCHNORM_FWD &&
        op->type != OperationType::CUDNN_BATCHNORM_BWD &&
        op->type != OperationType::CUDNN_BATCHNORM_INF) {
      // GEMMs and convolutions: the persistent grid min(work tiles, quota)
      const int g = kx_last_grid();
      if (g > 0 && g < pp.rec.sm_needed) pp.rec.sm_needed = g;
    }
    pp.rec.grid_size = pp.rec.sm_needed;
    pp.rec.block_size = 256;
    pp.rec.profile_type = (op->type == OperationType::CUDNN_BATCHNORM_FWD ||
                           op->type == OperationType::CUDNN_BATCHNORM_BWD ||
                           op->type == OperationType::CUDNN_BATCHNORM_INF)
                              ? ProfileType::MEMORY_BOUND
                              : ProfileType::COMPUTE_BOUND;
    pp.rec.client_idx = c;
    pp.rec.op_type = op_type_name(op->type);
    pp.rec.work = op_work(*op);
    std::lock_guard<std::mutex> lk(prof_mu_);
    pending_prof_.push_back(pp);
  }
  if (rc == KX_OK) {
    st.kx_ops.fetch_add(1);
    return cudaSuccess;
  }
  // the first 16 failures of a client, then every 1024th
  const uint64_t nerr = st.errors.fetch_add(1);
  if (nerr < 16 || (nerr & 1023) == 0) {
    auto err_name = ORION_REAL(cudart, cudaGetErrorName);
    const char* why = rc == KX_ERR_DEVICE && err_name != nullptr
                          ? err_name(static_cast<cudaError_t>(kx_last_cuda_error()))
                          : "";
    LOG_ERROR("client %d: %s failed in kx (status %d%s%s; %llu failures so far)", c,
              op_type_name(op->type), rc, rc == KX_ERR_DEVICE ? ", " : "", why,
              static_cast<unsigned long long>(nerr + 1));
  }
  return kx_to_cuda(rc);
}

void Scheduler::run_worker(int client_idx) {
  tl_is_scheduler_thread = true;
  tl_worker_idx = client_idx;
  // Linux lets a sleeping thread oversleep by its timer slack (50 us by
  // default): a 5 us idle sleep of a worker then costs 55 us of latency for
  // the next op it is handed.  1 us slack keeps idle BE workers cheap and
  // responsive.
  prctl(PR_SET_TIMERSLACK, 1000UL, 0UL, 0UL, 0UL);
  ORION_REAL(cudart, cudaSetDevice)(config_.device_id);
  cudaStream_t fallback = client_idx == 0 ? hp_stream_ : be_streams_[client_idx - 1];
  ClientQueue* q = g_capture_state.client_queues[client_idx].get();
  uint32_t idle = 0;
  while (running_.load()) {
    OperationPtr op = q->peek();
    if (!op) {
      if (client_idx == 0) hp_activity_poll();
      // the HP worker never sleeps (an HP op must start at once); BE workers
      // sleep briefly once idle for a while
      if (client_idx > 0 && ++idle > 64) std::this_thread::sleep_for(std::chrono::microseconds(5));
      else std::this_thread::yield();
      continue;
    }
    idle = 0;
    if (client_idx == 0 && is_kernel_op(op->type)) hp_activity_begin();
    if (client_idx > 0 && !orion_should_schedule(op, client_idx)) {
      // FIFO order is kept: the op stays at the head until admitted
      stats(client_idx).be_blocked.fetch_add(1);
      std::this_thread::yield();
      continue;
    }
    op = q->try_pop();
    if (!op) continue;
    if (!op->claim()) {
      // the client gave up waiting before the op started: it must not run
      op->mark_completed(cudaErrorTimeout);
      continue;
    }
    op->start_ns = mono_ns();
    cudaError_t err = execute_operation(op, fallback);
    op->end_ns = mono_ns();
    if (trace_enabled()) trace_executed(*op);
    if (err != cudaSuccess) set_last_error(client_idx, err);
    if (client_idx == 0 && !isolated_ && is_kernel_op(op->type) && !is_dense_op(op->type) &&
        q->empty()) {
      // HP kernels the interposer only re-issues count as HP activity too;
      // the event goes after the last HP op queued so far (a later op records
      // its own), one record per burst instead of one per kernel
      cudaStream_t s = op_stream(*op);
      std::lock_guard<std::mutex> lk(hp_mu_);
      ORION_REAL(cudart, cudaEventRecord)(hp_last_event_, s ? s : fallback);
      hp_event_pending_.store(true);
    }
    if (is_kernel_op(op->type)) {
      std::lock_guard<std::mutex> lk(g_orion_state.mutex);
      if (client_idx < static_cast<int>(g_orion_state.seen.size())) g_orion_state.seen[client_idx]++;
    }
    op->mark_completed(err);
  }
  // drain what is left so no client waits forever
  while (OperationPtr op = q->try_pop()) {
    if (!op->claim()) {
      op->mark_completed(cudaErrorTimeout);
      continue;
    }
    cudaError_t err = execute_operation(op, fallback);
    op->mark_completed(err);
  }
  ORION_REAL(cudart, cudaStreamSynchronize)(fallback);
}

void Scheduler::start() {
  if (!initialized_.load() || running_.load()) return;
  running_.store(true);
  workers_.clear();
  for (int i = 0; i < num_clients_; ++i) workers_.emplace_back(&Scheduler::run_worker, this, i);
}

void Scheduler::stop() {
  if (!running_.load()) return;
  running_.store(false);
  for (auto& q : g_capture_state.client_queues)
    if (q) q->shutdown();
}

void Scheduler::join() {
  for (auto& w : workers_)
    if (w.joinable()) w.join();
  workers_.clear();
  // host copy only: join() also runs from the destructor at process exit,
  // when CUDA calls may no longer be made
  if (hp_flag_host_) hp_flag_host_[0] = 0;
}

void Scheduler::reset() {
  if (running_.load()) return;
  destroy_streams();
  if (hp_last_event_) {
    ORION_REAL(cudart, cudaEventDestroy)(hp_last_event_);
    hp_last_event_ = nullptr;
  }
  {
    std::lock_guard<std::mutex> lk(prof_mu_);
    for (cudaEvent_t e : prof_events_) ORION_REAL(cudart, cudaEventDestroy)(e);
    prof_events_.clear();
  }
  if (flag_stream_) {
    ORION_REAL(cudart, cudaStreamSynchronize)(flag_stream_);
    ORION_REAL(cudart, cudaStreamDestroy)(flag_stream_);
    flag_stream_ = nullptr;
  }
  if (hp_flag_devmem_) {
    ORION_REAL(cudart, cudaFree)(hp_flag_devmem_);
    hp_flag_devmem_ = nullptr;
  }
  if (hp_flag_host_) {
    kx_host_flags_free(const_cast<int*>(hp_flag_host_));
    hp_flag_host_ = nullptr;
    hp_flag_dev_ = nullptr;
  }
  isolated_ = false;
  initialized_.store(false);
  num_clients_ = 0;
  g_orion_state.reset();
}

void Scheduler::sync_client_stream(int client_idx) {
  // wait until the client's queue has been executed, then for its work on the GPU
  if (client_idx >= 0 && client_idx < g_capture_state.num_clients) {
    auto& q = g_capture_state.client_queues[client_idx];
    const int64_t deadline = mono_ns() + wait_timeout_ns();
    while (q && !q->empty() && running_.load() && mono_ns() < deadline) std::this_thread::yield();
  }
  ORION_REAL(cudart, cudaDeviceSynchronize)();
}

void Scheduler::flush_profile() {
  std::vector<PendingProfile> pend;
  {
    std::lock_guard<std::mutex> lk(prof_mu_);
    pend.swap(pending_prof_);
  }
  for (auto& pp : pend) {
    ORION_REAL(cudart, cudaEventSynchronize)(pp.end);
    float ms = 0.f;
    ORION_REAL(cudart, cudaEventElapsedTime)(&ms, pp.start, pp.end);
    pp.rec.duration_ms = ms;
    g_profiler.record(pp.rec);
  }
  std::lock_guard<std::mutex> lk(prof_mu_);
  for (auto& pp : pend) {
    prof_events_.push_back(pp.start);
    prof_events_.push_back(pp.end);
  }
}

cudaEvent_t Scheduler::take_profile_event() {
  {
    std::lock_guard<std::mutex> lk(prof_mu_);
    if (!prof_events_.empty()) {
      cudaEvent_t e = prof_events_.back();
      prof_events_.pop_back();
      return e;
    }
  }
  cudaEvent_t e = nullptr;
  ORION_REAL(cudart, cudaEventCreate)(&e);
  return e;
}

void Scheduler::reserve_profile_events(int n) {
  std::vector<cudaEvent_t> made;
  {
    std::lock_guard<std::mutex> lk(prof_mu_);
    n -= static_cast<int>(prof_events_.size());
  }
  for (int i = 0; i < n; ++i) {
    cudaEvent_t e = nullptr;
    if (ORION_REAL(cudart, cudaEventCreate)(&e) != cudaSuccess) break;
    made.push_back(e);
  }
  std::lock_guard<std::mutex> lk(prof_mu_);
  prof_events_.insert(prof_events_.end(), made.begin(), made.end());
}

bool start_scheduler(int num_clients, const SchedulerConfig& config) {
  if (init_capture_layer(num_clients) != 0) return false;
  if (!g_scheduler.init(num_clients, config)) return false;
  g_scheduler.start();
  return true;
}

void stop_scheduler() {
  g_scheduler.stop();
  g_scheduler.join();
  g_scheduler.reset();
  shutdown_capture_layer();
}

}  // namespace orion

extern "C" {

int orion_init_scheduler(int num_clients) {
  if (orion::init_capture_layer(num_clients) != 0) return -1;
  return orion::g_scheduler.init(num_clients) ? 0 : -1;
}

int orion_start_scheduler_thread() {
  orion::g_scheduler.start();
  return 0;
}

int orion_start_scheduler(int num_clients) {
  return orion::start_scheduler(num_clients) ? 0 : -1;
}

// ORION_STATS_FILE=<path>: orion_stop_scheduler writes the per-client
// counters (orion_get_client_stats) there as JSON, so runs of drivers that do
// not read them (the reference's own scripts) can still be checked.
static void write_stats_file() {
  const char* path = std::getenv("ORION_STATS_FILE");
  if (path == nullptr || path[0] == '\0') return;
  FILE* f = std::fopen(path, "w");
  if (f == nullptr) return;
  const int n = orion::g_capture_state.num_clients;
  std::fprintf(f, "{\"clients\": [");
  for (int c = 0; c < n; ++c) {
    orion::ClientStats& s = orion::g_scheduler.stats(c);
    std::fprintf(f,
                 "%s{\"client\": %d, \"ops\": %llu, \"kx_ops\": %llu, \"passthrough_ops\": %llu, "
                 "\"be_blocked\": %llu, \"yields\": %llu, \"errors\": %llu}",
                 c ? ", " : "", c, (unsigned long long)s.ops.load(),
                 (unsigned long long)s.kx_ops.load(), (unsigned long long)s.passthrough_ops.load(),
                 (unsigned long long)s.be_blocked.load(), (unsigned long long)s.yields.load(),
                 (unsigned long long)s.errors.load());
  }
  std::fprintf(f, "]}\n");
  std::fclose(f);
}

void orion_stop_scheduler() {
  orion::stop_scheduler();
  write_stats_file();
}

int orion_load_kernel_info(int client_idx, const char* file_path) {
  if (file_path == nullptr) return -1;
  return orion::populate_kernel_info(client_idx, file_path);
}

void orion_set_client_kernels(int client_idx, int num_kernels) {
  std::lock_guard<std::mutex> lk(orion::g_orion_state.mutex);
  if (client_idx < 0 || client_idx >= static_cast<int>(orion::g_orion_state.num_client_kernels.size()))
    return;
  orion::g_orion_state.num_client_kernels[client_idx] = num_kernels;
}

void orion_set_sm_threshold(int threshold) {
  std::lock_guard<std::mutex> lk(orion::g_orion_state.mutex);
  orion::g_orion_state.sm_threshold = threshold;
  orion::g_scheduler.get_mutable_config().sm_threshold = threshold;
}

int orion_get_sm_threshold() {
  std::lock_guard<std::mutex> lk(orion::g_orion_state.mutex);
  return orion::g_orion_state.sm_threshold;
}

void orion_sync_client_stream(int client_idx) { orion::g_scheduler.sync_client_stream(client_idx); }

void orion_reset_state() { orion::g_orion_state.reset(); }

int orion_autotune_green_ctx() { return orion::g_scheduler.autotune_green_ctx(); }

void orion_set_profile_launches(int on) { orion::g_scheduler.set_profile_launches(on != 0); }

void orion_set_be_keep_sms(int sms) { orion::g_scheduler.set_be_keep_sms(sms < 0 ? 0 : sms); }

int orion_get_be_keep_sms() { return orion::g_scheduler.be_keep_sms(); }

int orion_set_sm_budgets(int hp_sms, int be_sms) {
  if (hp_sms == 0 && be_sms == 0) {
    orion::g_scheduler.clear_budgets();
    return 0;
  }
  orion::Scheduler::GreenCtxConfig gc;
  gc.hp_sm_count = static_cast<unsigned>(hp_sms);
  gc.be_sm_count = static_cast<unsigned>(be_sms);
  gc.enabled = true;
  return orion::g_scheduler.init_green_contexts(gc) ? 0 : -1;
}

void orion_set_be_host_hold_us(int us) { orion::g_scheduler.set_be_host_hold_us(us); }

int orion_get_be_host_hold_us() { return orion::g_scheduler.be_host_hold_us(); }

void orion_set_profile_every(int n) { orion::g_scheduler.set_profile_every(n); }

unsigned long long orion_get_client_host_holds(int client_idx) {
  if (client_idx < 0 || client_idx >= orion::MAX_CLIENTS) return 0;
  return orion::g_scheduler.stats(client_idx).host_holds.load();
}

int orion_get_client_stats(int client_idx, unsigned long long* out6) {
  if (out6 == nullptr || client_idx < 0 || client_idx >= orion::MAX_CLIENTS) return -1;
  orion::ClientStats& s = orion::g_scheduler.stats(client_idx);
  out6[0] = s.ops.load();
  out6[1] = s.kx_ops.load();
  out6[2] = s.passthrough_ops.load();
  out6[3] = s.be_blocked.load();
  out6[4] = s.yields.load();
  out6[5] = s.errors.load();
  return 0;
}

void block(int client_idx) { orion::g_scheduler.sync_client_stream(client_idx); }

}  // extern "C"
