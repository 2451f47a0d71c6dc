// gpu_capture.cpp — capture layer: lock-free client queues, client identity
// (thread-local, then stream / handle maps), async-mode switch, first-error
// latch per client, and the orion_* capture C API.
//
// Behaviour follows the reference's src/gpu_capture.cpp (init 107-146,
// create/enqueue/wait 200-241, async mode 244, error latch 247-271, C API
// 281-322); the queue, the bounded waits and the handle -> stream map are this
// build's.
#include <vector>
#include <cstdio>
#include <pthread.h>
#include <time.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <shared_mutex>
#include <thread>
#include <unordered_map>

#include "gpu_capture.h"

namespace orion {

CaptureLayerState g_capture_state;
LogLevel g_log_level = LogLevel::WARN;

static thread_local int tl_client_idx = -1;
thread_local bool tl_is_scheduler_thread = false;
thread_local bool tl_in_scheduler_execution = false;
thread_local int tl_worker_idx = -1;

static std::unordered_map<void*, int> g_stream_to_client;
static std::unordered_map<void*, int> g_handle_to_client;
static std::unordered_map<void*, cudaStream_t> g_handle_to_stream;
static std::shared_mutex g_map_mu;

static std::atomic<int> g_async_mode{1};
static std::atomic<int> g_last_error[MAX_CLIENTS];

static int64_t now_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return static_cast<int64_t>(ts.tv_sec) * 1000000000LL + ts.tv_nsec;
}

int64_t wait_timeout_ns() {
  static int64_t t = [] {
    const char* s = std::getenv("ORION_WAIT_TIMEOUT_MS");
    long long ms = s ? std::atoll(s) : 60000;
    if (ms <= 0) ms = 60000;
    return static_cast<int64_t>(ms) * 1000000LL;
  }();
  return t;
}

cudaError_t OperationRecord::wait_completion() {
  if (completed.load(std::memory_order_acquire)) return result;
  int64_t deadline = now_ns() + wait_timeout_ns();
  uint32_t spins = 0;
  while (!completed.load(std::memory_order_acquire)) {
    if (++spins > 2048) {
      std::this_thread::yield();
      if ((spins & 1023) == 0 && now_ns() > deadline) {
        if (cancel()) {
          LOG_ERROR("op %lu (%s) not started within %lld ms; cancelled", (unsigned long)op_id,
                    op_type_name(type), (long long)(wait_timeout_ns() / 1000000));
          return cudaErrorTimeout;
        }
        if (detachable) {
          LOG_ERROR("op %lu (%s) not completed within %lld ms; no longer waited for",
                    (unsigned long)op_id, op_type_name(type),
                    (long long)(wait_timeout_ns() / 1000000));
          return cudaErrorTimeout;
        }
        // running on the worker with the caller's memory: wait it out
        LOG_ERROR("op %lu (%s) still running after %lld ms; waiting for it", (unsigned long)op_id,
                  op_type_name(type), (long long)(wait_timeout_ns() / 1000000));
        deadline = now_ns() + wait_timeout_ns();
      }
    }
  }
  return result;
}

// ---------------------------------------------------------------- queue ----

ClientQueue::ClientQueue() : cells_(new Cell[kCapacity]), head_(0), tail_(0), shutdown_(false) {
  for (size_t i = 0; i < kCapacity; ++i) cells_[i].seq.store(i, std::memory_order_relaxed);
}

ClientQueue::~ClientQueue() { delete[] cells_; }

bool ClientQueue::try_push(OperationPtr op) {
  size_t pos = tail_.load(std::memory_order_relaxed);
  for (;;) {
    Cell& c = cells_[pos & (kCapacity - 1)];
    const size_t seq = c.seq.load(std::memory_order_acquire);
    const intptr_t diff = static_cast<intptr_t>(seq) - static_cast<intptr_t>(pos);
    if (diff == 0) {
      if (tail_.compare_exchange_weak(pos, pos + 1, std::memory_order_relaxed)) {
        c.op = std::move(op);
        c.seq.store(pos + 1, std::memory_order_release);
        return true;
      }
    } else if (diff < 0) {
      return false;  // full
    } else {
      pos = tail_.load(std::memory_order_relaxed);
    }
  }
}

bool ClientQueue::push(OperationPtr op) {
  if (try_push(op)) return true;
  const int64_t deadline = now_ns() + wait_timeout_ns();
  while (!try_push(op)) {
    if (now_ns() > deadline) return false;
    std::this_thread::yield();
  }
  return true;
}

OperationPtr ClientQueue::try_pop() {
  size_t pos = head_.load(std::memory_order_relaxed);
  for (;;) {
    Cell& c = cells_[pos & (kCapacity - 1)];
    const size_t seq = c.seq.load(std::memory_order_acquire);
    const intptr_t diff = static_cast<intptr_t>(seq) - static_cast<intptr_t>(pos + 1);
    if (diff == 0) {
      if (head_.compare_exchange_weak(pos, pos + 1, std::memory_order_relaxed)) {
        OperationPtr op = std::move(c.op);
        c.seq.store(pos + kCapacity, std::memory_order_release);
        return op;
      }
    } else if (diff < 0) {
      return nullptr;  // empty
    } else {
      pos = head_.load(std::memory_order_relaxed);
    }
  }
}

OperationPtr ClientQueue::peek() {
  const size_t pos = head_.load(std::memory_order_acquire);
  Cell& c = cells_[pos & (kCapacity - 1)];
  if (c.seq.load(std::memory_order_acquire) == pos + 1) return c.op;
  return nullptr;
}

bool ClientQueue::empty() { return size() == 0; }

size_t ClientQueue::size() {
  const size_t t = tail_.load(std::memory_order_acquire);
  const size_t h = head_.load(std::memory_order_acquire);
  return t > h ? t - h : 0;
}

// ------------------------------------------------------------ identity -----

void register_client_stream(int client_idx, void* stream) {
  if (client_idx < 0 || stream == nullptr) return;
  std::unique_lock<std::shared_mutex> lk(g_map_mu);
  g_stream_to_client[stream] = client_idx;
}

void register_client_handle(int client_idx, void* handle) {
  if (client_idx < 0 || handle == nullptr) return;
  std::unique_lock<std::shared_mutex> lk(g_map_mu);
  g_handle_to_client[handle] = client_idx;
}

int resolve_client_idx(void* stream, void* handle) {
  if (tl_client_idx >= 0) return tl_client_idx;
  std::shared_lock<std::shared_mutex> lk(g_map_mu);
  if (stream) {
    auto it = g_stream_to_client.find(stream);
    if (it != g_stream_to_client.end()) return it->second;
  }
  if (handle) {
    auto it = g_handle_to_client.find(handle);
    if (it != g_handle_to_client.end()) return it->second;
  }
  return -1;
}

void clear_client_maps() {
  std::unique_lock<std::shared_mutex> lk(g_map_mu);
  g_stream_to_client.clear();
  g_handle_to_client.clear();
}

void remember_handle_stream(void* handle, cudaStream_t stream) {
  if (handle == nullptr) return;
  std::unique_lock<std::shared_mutex> lk(g_map_mu);
  g_handle_to_stream[handle] = stream;
}

cudaStream_t handle_stream(void* handle) {
  std::shared_lock<std::shared_mutex> lk(g_map_mu);
  auto it = g_handle_to_stream.find(handle);
  return it == g_handle_to_stream.end() ? nullptr : it->second;
}

// ------------------------------------------------------------- logging -----

void init_log_level() {
  const char* s = std::getenv("ORION_LOG_LEVEL");
  if (!s) return;
  struct { const char* name; LogLevel lvl; } table[] = {
      {"NONE", LogLevel::NONE}, {"0", LogLevel::NONE},   {"ERROR", LogLevel::ERROR},
      {"1", LogLevel::ERROR},   {"WARN", LogLevel::WARN}, {"2", LogLevel::WARN},
      {"INFO", LogLevel::INFO}, {"3", LogLevel::INFO},   {"DEBUG", LogLevel::DEBUG},
      {"4", LogLevel::DEBUG},   {"TRACE", LogLevel::TRACE}, {"5", LogLevel::TRACE}};
  for (auto& t : table)
    if (std::strcmp(s, t.name) == 0) g_log_level = t.lvl;
}

// ---------------------------------------------------------- lifecycle ------

int init_capture_layer(int num_clients) {
  if (g_capture_state.initialized.load()) {
    LOG_WARN("capture layer already initialized");
    return 0;
  }
  if (num_clients <= 0 || num_clients > MAX_CLIENTS) {
    LOG_ERROR("invalid num_clients %d (1-%d)", num_clients, MAX_CLIENTS);
    return -1;
  }
  init_log_level();
  if (const char* m = std::getenv("ORION_ASYNC_MODE")) {
    const int mode = std::atoi(m);
    if (mode >= 0 && mode <= 2) set_async_mode_internal(mode);
  }
  g_capture_state.num_clients = num_clients;
  g_capture_state.client_queues.clear();
  for (int i = 0; i < num_clients; ++i)
    g_capture_state.client_queues.emplace_back(std::make_unique<ClientQueue>());
  for (int i = 0; i < MAX_CLIENTS; ++i) g_last_error[i].store(cudaSuccess);
  g_capture_state.shutdown.store(false);
  g_capture_state.initialized.store(true);
  g_capture_state.enabled.store(true);
  LOG_INFO("capture layer initialized with %d clients", num_clients);
  return 0;
}

void shutdown_capture_layer() {
  if (!g_capture_state.initialized.load()) return;
  g_capture_state.shutdown.store(true);
  g_capture_state.enabled.store(false);
  for (auto& q : g_capture_state.client_queues) q->shutdown();
  g_capture_state.initialized.store(false);
}

int get_current_client_idx() { return tl_client_idx; }

void set_current_client_idx(int idx) {
  if (idx < -1 || idx >= MAX_CLIENTS ||
      (g_capture_state.initialized.load() && idx >= g_capture_state.num_clients)) {
    LOG_ERROR("invalid client index %d", idx);
    return;
  }
  tl_client_idx = idx;
}

bool is_managed_thread() { return tl_client_idx >= 0 && g_capture_state.enabled.load(); }

bool is_capture_enabled() {
  return g_capture_state.initialized.load() && g_capture_state.enabled.load();
}

void set_capture_enabled(bool enabled) { g_capture_state.enabled.store(enabled); }

OperationPtr create_operation(int client_idx, OperationType type) {
  if (client_idx < 0 || client_idx >= g_capture_state.num_clients) return nullptr;
  auto op = std::make_shared<OperationRecord>();
  op->type = type;
  op->client_idx = client_idx;
  op->op_id = g_capture_state.next_op_id.fetch_add(1);
  op->enqueue_ns = now_ns();
  return op;
}

bool enqueue_operation(OperationPtr op) {
  if (!op) return false;
  if (op->client_idx > 0)
    be_issue_gate(op->client_idx, op->type);
  else
    note_hp_issue();
  if (g_capture_state.client_queues[op->client_idx]->push(op)) return true;
  LOG_ERROR("client %d: queue full for %lld ms; op %lu (%s) dropped", op->client_idx,
            (long long)(wait_timeout_ns() / 1000000), (unsigned long)op->op_id,
            op_type_name(op->type));
  op->state.store(OperationRecord::kCancelled, std::memory_order_release);
  op->mark_completed(cudaErrorTimeout);
  set_last_error(op->client_idx, cudaErrorTimeout);
  return false;
}

namespace {
// How long client threads block in wait_operation, per client.
struct WaitStats {
  std::atomic<unsigned long long> count{0}, total_ns{0}, max_ns{0};
  std::mutex mu;  // guards the description of the longest wait
  unsigned long long max_desc[5] = {0, 0, 0, 0, 0};
};

unsigned long long op_bytes(const OperationRecord& op) {
  if (auto* m = std::get_if<MallocParams>(&op.params)) return m->size;
  if (auto* c = std::get_if<MemcpyParams>(&op.params)) return c->count;
  return 0;
}
WaitStats g_wait_stats[MAX_CLIENTS];
}  // namespace

cudaError_t wait_operation(OperationPtr op) {
  if (!op) return cudaErrorInvalidValue;
  if (op->completed.load(std::memory_order_acquire)) return op->result;
  const int64_t t0 = now_ns();
  const cudaError_t res = op->wait_completion();
  const int64_t t1 = now_ns();
  if (trace_enabled()) trace_client_wait(*op, t0, t1);
  const unsigned long long dt = static_cast<unsigned long long>(t1 - t0);
  if (op->client_idx < 0 || op->client_idx >= MAX_CLIENTS) return res;
  WaitStats& w = g_wait_stats[op->client_idx];
  w.count.fetch_add(1, std::memory_order_relaxed);
  w.total_ns.fetch_add(dt, std::memory_order_relaxed);
  unsigned long long prev = w.max_ns.load(std::memory_order_relaxed);
  while (dt > prev && !w.max_ns.compare_exchange_weak(prev, dt)) {
  }
  if (dt > prev) {
    auto span = [](int64_t a, int64_t b) {
      return b > a && a > 0 ? static_cast<unsigned long long>(b - a) : 0ULL;
    };
    std::lock_guard<std::mutex> lk(w.mu);
    w.max_desc[0] = static_cast<unsigned long long>(op->type);
    w.max_desc[1] = span(op->enqueue_ns, op->start_ns);
    w.max_desc[2] = span(op->start_ns, op->end_ns);
    w.max_desc[3] = op_bytes(*op);
    w.max_desc[4] = 0;
  }
  return res;
}

void get_wait_stats(int client_idx, unsigned long long* out8, bool reset) {
  if (client_idx < 0 || client_idx >= MAX_CLIENTS) return;
  WaitStats& w = g_wait_stats[client_idx];
  out8[0] = reset ? w.count.exchange(0) : w.count.load();
  out8[1] = reset ? w.total_ns.exchange(0) : w.total_ns.load();
  out8[2] = reset ? w.max_ns.exchange(0) : w.max_ns.load();
  std::lock_guard<std::mutex> lk(w.mu);
  for (int i = 0; i < 5; ++i) {
    out8[3 + i] = w.max_desc[i];
    if (reset) w.max_desc[i] = 0;
  }
}

OperationPtr submit_operation(int client_idx, OperationType type) {
  // The record is returned un-enqueued would be the safe form; to keep the
  // reference's contract (returned op already queued) callers that still
  // need to fill params must use create_operation + enqueue_operation.
  auto op = create_operation(client_idx, type);
  if (op) enqueue_operation(op);
  return op;
}

void set_async_mode_internal(int mode) { g_async_mode.store(mode); }
int get_async_mode_internal() { return g_async_mode.load(); }

void set_last_error(int client_idx, cudaError_t error) {
  if (client_idx < 0 || client_idx >= MAX_CLIENTS) return;
  int expected = cudaSuccess;
  g_last_error[client_idx].compare_exchange_strong(expected, static_cast<int>(error));
}

cudaError_t get_and_clear_last_error(int client_idx) {
  if (client_idx < 0 || client_idx >= MAX_CLIENTS) return cudaSuccess;
  return static_cast<cudaError_t>(g_last_error[client_idx].exchange(cudaSuccess));
}

namespace {
struct OpLogEntry {
  int client;
  OperationType type;
  const char* route;
  int ndims;
  long long dims[8];
};
std::mutex g_oplog_mu;
std::vector<OpLogEntry> g_oplog;
std::atomic<bool> g_oplog_on{false};
}  // namespace

bool op_log_enabled() { return g_oplog_on.load(std::memory_order_relaxed); }

namespace {
// kind 0: worker execution span; 1: client wait span; 2: scheduler marker
struct TraceEvent {
  int kind;
  int client;
  OperationType type;
  uint64_t op_id;
  int64_t enq, t0, t1;
  unsigned long long bytes;
  const char* name;
  int value;
};
constexpr size_t kTraceMax = size_t(4) << 20;
std::mutex g_trace_mu;
std::vector<TraceEvent> g_trace;
std::atomic<bool> g_trace_on{false};

void trace_push(const TraceEvent& e) {
  std::lock_guard<std::mutex> lk(g_trace_mu);
  if (g_trace.size() < kTraceMax) g_trace.push_back(e);
}
}  // namespace

bool trace_enabled() { return g_trace_on.load(std::memory_order_relaxed); }

void trace_executed(const OperationRecord& op) {
  if (!trace_enabled()) return;
  trace_push({0, op.client_idx, op.type, op.op_id, op.enqueue_ns, op.start_ns, op.end_ns,
              op_bytes(op), nullptr, 0});
}

void trace_client_wait(const OperationRecord& op, int64_t t0, int64_t t1) {
  trace_push({1, op.client_idx, op.type, op.op_id, op.enqueue_ns, t0, t1, op_bytes(op), nullptr,
              0});
}

void trace_marker(const char* name, int value) {
  if (!trace_enabled()) return;
  const int64_t t = now_ns();
  trace_push({2, -1, OperationType::UNKNOWN, 0, t, t, t, 0, name, value});
}

void op_log_record(int client_idx, OperationType type, const long long* dims, int ndims,
                   const char* route) {
  if (!op_log_enabled()) return;
  OpLogEntry e;
  e.client = client_idx;
  e.type = type;
  e.route = route;
  e.ndims = ndims < 0 ? 0 : (ndims > 8 ? 8 : ndims);
  for (int i = 0; i < e.ndims; ++i) e.dims[i] = dims[i];
  std::lock_guard<std::mutex> lk(g_oplog_mu);
  g_oplog.push_back(e);
}

}  // namespace orion

extern "C" {

int orion_get_client_waits(int client_idx, unsigned long long* out8, int reset) {
  if (out8 == nullptr || client_idx < 0 || client_idx >= orion::MAX_CLIENTS) return -1;
  orion::get_wait_stats(client_idx, out8, reset != 0);
  return 0;
}

void orion_op_log_start(void) {
  std::lock_guard<std::mutex> lk(orion::g_oplog_mu);
  orion::g_oplog.clear();
  orion::g_oplog_on.store(true);
}

void orion_trace_start(void) {
  std::lock_guard<std::mutex> lk(orion::g_trace_mu);
  orion::g_trace.clear();
  orion::g_trace.reserve(size_t(1) << 16);
  orion::g_trace_on.store(true);
}

int orion_trace_end(const char* path) {
  orion::g_trace_on.store(false);
  std::lock_guard<std::mutex> lk(orion::g_trace_mu);
  if (path == nullptr) return -1;
  FILE* f = std::fopen(path, "w");
  if (f == nullptr) return -1;
  auto track_name = [](int client, bool worker) {
    static thread_local char buf[32];
    if (client == 0) std::snprintf(buf, sizeof(buf), "HP-%s", worker ? "Worker" : "Client");
    else std::snprintf(buf, sizeof(buf), "BE%d-%s", client, worker ? "Worker" : "Client");
    return buf;
  };
  std::fprintf(f, "{\"displayTimeUnit\": \"ms\", \"traceEvents\": [\n");
  std::fprintf(f, "{\"ph\": \"M\", \"pid\": 1, \"tid\": 0, \"name\": \"process_name\", "
                  "\"args\": {\"name\": \"orion capture\"}}");
  const int nclients = orion::g_capture_state.num_clients;
  for (int c = 0; c < nclients; ++c)
    for (int w = 0; w < 2; ++w)
      std::fprintf(f, ",\n{\"ph\": \"M\", \"pid\": 1, \"tid\": %d, \"name\": \"thread_name\", "
                      "\"args\": {\"name\": \"%s\"}}",
                   (w ? 100 : 1) + c, track_name(c, w != 0));
  std::fprintf(f, ",\n{\"ph\": \"M\", \"pid\": 1, \"tid\": 200, \"name\": \"thread_name\", "
                  "\"args\": {\"name\": \"Scheduler\"}}");
  for (const auto& e : orion::g_trace) {
    const double us0 = e.t0 / 1e3, dur = (e.t1 - e.t0) / 1e3;
    if (e.kind == 2) {
      std::fprintf(f, ",\n{\"ph\": \"i\", \"s\": \"t\", \"pid\": 1, \"tid\": 200, "
                      "\"ts\": %.3f, \"name\": \"%s\", \"args\": {\"value\": %d}}",
                   us0, e.name, e.value);
      continue;
    }
    const char* tn = orion::op_type_name(e.type);
    if (e.kind == 0) {
      // the issue instant on the client track, then the execution span
      std::fprintf(f, ",\n{\"ph\": \"i\", \"s\": \"t\", \"pid\": 1, \"tid\": %d, "
                      "\"ts\": %.3f, \"name\": \"%s\", \"args\": {\"op_id\": %llu}}",
                   1 + e.client, e.enq / 1e3, tn, static_cast<unsigned long long>(e.op_id));
      std::fprintf(f, ",\n{\"ph\": \"X\", \"pid\": 1, \"tid\": %d, \"ts\": %.3f, "
                      "\"dur\": %.3f, \"name\": \"%s\", \"args\": {\"op_id\": %llu, "
                      "\"queued_us\": %.3f, \"bytes\": %llu}}",
                   100 + e.client, us0, dur, tn, static_cast<unsigned long long>(e.op_id),
                   (e.t0 - e.enq) / 1e3, e.bytes);
    } else {
      std::fprintf(f, ",\n{\"ph\": \"X\", \"pid\": 1, \"tid\": %d, \"ts\": %.3f, "
                      "\"dur\": %.3f, \"name\": \"wait %s\", \"args\": {\"op_id\": %llu, "
                      "\"bytes\": %llu}}",
                   1 + e.client, us0, dur, tn, static_cast<unsigned long long>(e.op_id), e.bytes);
    }
  }
  std::fprintf(f, "\n]}\n");
  std::fclose(f);
  const int n = static_cast<int>(orion::g_trace.size());
  orion::g_trace.clear();
  orion::g_trace.shrink_to_fit();
  return n;
}

int orion_op_log_end(const char* path) {
  orion::g_oplog_on.store(false);
  std::lock_guard<std::mutex> lk(orion::g_oplog_mu);
  if (path == nullptr) return -1;
  FILE* f = std::fopen(path, "w");
  if (f == nullptr) return -1;
  for (const auto& e : orion::g_oplog) {
    std::fprintf(f, "%d\t%s\t%s", e.client, orion::op_type_name(e.type), e.route);
    for (int i = 0; i < e.ndims; ++i) std::fprintf(f, "\t%lld", e.dims[i]);
    std::fprintf(f, "\n");
  }
  std::fclose(f);
  const int n = static_cast<int>(orion::g_oplog.size());
  orion::g_oplog.clear();
  return n;
}

int orion_init(int num_clients) { return orion::init_capture_layer(num_clients); }
void orion_shutdown() { orion::shutdown_capture_layer(); }
void orion_set_client_idx(int idx) { orion::set_current_client_idx(idx); }
int orion_get_client_idx() { return orion::get_current_client_idx(); }
void orion_set_enabled(int enabled) { orion::set_capture_enabled(enabled != 0); }
int orion_is_enabled() { return orion::is_capture_enabled() ? 1 : 0; }
int orion_set_capture(int enabled) {
  orion::set_capture_enabled(enabled != 0);
  return 0;
}
void orion_register_client_stream(int client_idx, void* stream) {
  orion::register_client_stream(client_idx, stream);
}
void orion_register_client_handle(int client_idx, void* handle) {
  orion::register_client_handle(client_idx, handle);
}
int orion_resolve_client_idx(void* stream, void* handle) {
  return orion::resolve_client_idx(stream, handle);
}

}  // extern "C"

extern "C" {

// Async mode: 0 = client waits for the worker, 1 = worker-async (default),
// 2 = run on the calling thread.  Same C API as the reference
// (src/cuda_intercept.cpp:1299-1311).
void orion_set_async_mode(int mode) {
  if (mode >= 0 && mode <= 2) orion::set_async_mode_internal(mode);
}

int orion_get_async_mode() { return orion::get_async_mode_internal(); }

}  // extern "C"
