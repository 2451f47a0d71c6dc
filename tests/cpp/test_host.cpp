// Host-side unit tests of the interposer (no GPU, no worker thread).
//
// Follows the idea of the reference's test/test_main.cpp (capture init,
// client index, submit, profile load, scheduling decision, concurrency; the
// ops are completed by the test itself, 236-276) with real assertions.
// Built and run by tests/test_host_cpp.py against libgpu_scheduler.so.
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#define private public  // reach the scheduler's decision functions
#include "gpu_capture.h"
#include "kernel_profile.h"
#include "scheduler.h"
#undef private

// Exported but declared in no header (as in the reference).
extern "C" void orion_set_async_mode(int mode);
extern "C" int orion_get_async_mode();

static int g_failures = 0;
#define CHECK(cond)                                                       \
  do {                                                                    \
    if (!(cond)) {                                                        \
      std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
      ++g_failures;                                                       \
    }                                                                     \
  } while (0)

using namespace orion;

static void test_capture_init() {
  CHECK(orion_init(0) == -1);
  CHECK(orion_init(MAX_CLIENTS + 1) == -1);
  CHECK(orion_init(3) == 0);
  CHECK(orion_init(3) == 0);  // second init is a warning, not an error
  CHECK(g_capture_state.num_clients == 3);
  CHECK(orion_is_enabled() == 1);
  orion_set_enabled(0);
  CHECK(orion_is_enabled() == 0);
  CHECK(orion_set_capture(1) == 0);
  CHECK(orion_is_enabled() == 1);
}

static void test_client_index_thread_local() {
  orion_set_client_idx(2);
  int other = -7;
  std::thread t([&] { other = orion_get_client_idx(); });
  t.join();
  CHECK(orion_get_client_idx() == 2);
  CHECK(other == -1);  // a new thread has no client
  orion_set_client_idx(5);  // out of range for 3 clients: rejected
  CHECK(orion_get_client_idx() == 2);
  orion_set_client_idx(-1);
  CHECK(orion_get_client_idx() == -1);
}

static void test_stream_handle_maps() {
  void* s1 = reinterpret_cast<void*>(0x1000);
  void* s2 = reinterpret_cast<void*>(0x2000);
  void* h1 = reinterpret_cast<void*>(0x3000);
  orion_register_client_stream(1, s1);
  orion_register_client_handle(2, h1);
  CHECK(orion_resolve_client_idx(s1, nullptr) == 1);
  CHECK(orion_resolve_client_idx(nullptr, h1) == 2);
  CHECK(orion_resolve_client_idx(s2, nullptr) == -1);
  orion_set_client_idx(0);  // the thread's own identity wins
  CHECK(orion_resolve_client_idx(s1, h1) == 0);
  orion_set_client_idx(-1);
  clear_client_maps();
  CHECK(orion_resolve_client_idx(s1, nullptr) == -1);
}

static void test_submit_and_complete() {
  auto op = create_operation(1, OperationType::CUBLAS_SGEMM);
  CHECK(op != nullptr);
  CHECK(op->client_idx == 1);
  enqueue_operation(op);
  auto& q = g_capture_state.client_queues[1];
  CHECK(q->size() == 1);
  auto head = q->peek();
  CHECK(head.get() == op.get());
  auto got = q->try_pop();
  CHECK(got.get() == op.get());
  CHECK(q->empty());
  CHECK(got->claim());
  std::thread worker([got] { got->mark_completed(cudaSuccess); });
  CHECK(op->wait_completion() == cudaSuccess);
  worker.join();
  CHECK(op->completed.load());
  CHECK(op->result == cudaSuccess);
  // op ids increase
  auto a = create_operation(0, OperationType::MALLOC);
  auto b = create_operation(0, OperationType::MALLOC);
  CHECK(b->op_id > a->op_id);
}

static int64_t ms_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration_cast<std::chrono::milliseconds>(
             std::chrono::steady_clock::now() - t0).count();
}

static void test_bounded_wait() {
  // ORION_WAIT_TIMEOUT_MS=200 is set by the driver: an op nobody starts is
  // cancelled after the deadline and reports cudaErrorTimeout.
  auto op = create_operation(0, OperationType::KERNEL_LAUNCH);
  CHECK(op->wait_completion() == cudaErrorTimeout);
  CHECK(!op->completed.load());
  CHECK(op->state.load() == OperationRecord::kCancelled);
  // a stalled worker that reaches the record later must skip it
  CHECK(!op->claim());
}

static void test_timeout_paths_with_stalled_worker() {
  // 1) queued, the worker stalls: the client cancels it, the worker skips it
  auto& q = g_capture_state.client_queues[0];
  while (!q->empty()) q->try_pop();
  auto op = create_operation(0, OperationType::CUBLAS_SGEMM);
  CHECK(enqueue_operation(op));
  auto t0 = std::chrono::steady_clock::now();
  CHECK(wait_operation(op) == cudaErrorTimeout);
  CHECK(ms_since(t0) >= 150);
  auto popped = q->try_pop();
  CHECK(popped.get() == op.get());
  CHECK(!popped->claim());  // never executed
  // 2) claimed by a slow worker, ordinary record (reads the caller's memory):
  //    the client waits past the deadline until the worker finishes
  auto slow = create_operation(0, OperationType::MALLOC);
  CHECK(slow->claim());
  std::thread w1([slow] {
    std::this_thread::sleep_for(std::chrono::milliseconds(450));
    slow->mark_completed(cudaSuccess);
  });
  t0 = std::chrono::steady_clock::now();
  CHECK(slow->wait_completion() == cudaSuccess);
  CHECK(ms_since(t0) >= 400);
  w1.join();
  // 3) claimed, detachable (arguments copied into the record): the client
  //    stops waiting at the deadline; the worker finishes later on its own
  auto det = create_operation(0, OperationType::KERNEL_LAUNCH);
  det->detachable = true;
  CHECK(det->claim());
  std::thread w2([det] {
    std::this_thread::sleep_for(std::chrono::milliseconds(500));
    det->mark_completed(cudaSuccess);
  });
  t0 = std::chrono::steady_clock::now();
  CHECK(det->wait_completion() == cudaErrorTimeout);
  CHECK(ms_since(t0) < 450);
  w2.join();
  CHECK(det->completed.load());
}

static void test_bounded_push() {
  // a full ring: push gives up after the deadline instead of spinning forever
  ClientQueue q;
  for (size_t i = 0; i < ClientQueue::kCapacity; ++i)
    CHECK(q.try_push(std::make_shared<OperationRecord>()));
  auto t0 = std::chrono::steady_clock::now();
  CHECK(!q.push(std::make_shared<OperationRecord>()));
  CHECK(ms_since(t0) >= 150);
  // enqueue_operation on a full client queue: the record completes with a
  // timeout, is marked cancelled and the client's error latch is set
  auto& cq = g_capture_state.client_queues[2];
  while (!cq->empty()) cq->try_pop();
  for (size_t i = 0; i < ClientQueue::kCapacity; ++i)
    CHECK(cq->try_push(create_operation(2, OperationType::MEMSET)));
  auto op = create_operation(2, OperationType::CUBLAS_SGEMM);
  CHECK(!enqueue_operation(op));
  CHECK(op->completed.load() && op->result == cudaErrorTimeout);
  CHECK(!op->claim());
  CHECK(get_and_clear_last_error(2) == cudaErrorTimeout);
  while (!cq->empty()) cq->try_pop();
}

static void test_queue_fifo_concurrent() {
  ClientQueue q;
  constexpr int kProducers = 4, kPer = 20000;
  std::atomic<int> done{0};
  std::vector<std::thread> ps;
  for (int p = 0; p < kProducers; ++p) {
    ps.emplace_back([&, p] {
      for (int i = 0; i < kPer; ++i) {
        auto op = std::make_shared<OperationRecord>();
        op->client_idx = p;
        op->op_id = static_cast<uint64_t>(i);
        q.push(op);  // spins while the 8192-slot ring is full
      }
      done.fetch_add(1);
    });
  }
  std::vector<long> last(kProducers, -1);
  long popped = 0;
  bool ordered = true;
  while (popped < static_cast<long>(kProducers) * kPer) {
    auto op = q.try_pop();
    if (!op) {
      std::this_thread::yield();
      continue;
    }
    if (static_cast<long>(op->op_id) != last[op->client_idx] + 1) ordered = false;
    last[op->client_idx] = static_cast<long>(op->op_id);
    ++popped;
  }
  for (auto& t : ps) t.join();
  CHECK(ordered);  // each producer's ops come out in its order
  CHECK(q.empty());
  CHECK(q.try_pop() == nullptr);
  // try_push reports a full ring
  ClientQueue small;
  size_t pushed = 0;
  while (small.try_push(std::make_shared<OperationRecord>())) ++pushed;
  CHECK(pushed == ClientQueue::kCapacity);
}

static void write_file(const char* path, const char* text) {
  std::ofstream f(path);
  f << text;
}

static void test_kernel_info_and_decision(const std::string& dir) {
  g_orion_state.init(2, 148);
  const std::string hp = dir + "/hp_kernel_info.csv";
  const std::string be = dir + "/be_kernel_info.csv";
  // Name may contain commas (template arguments); parsed right to left.
  write_file(hp.c_str(),
             "Name,Profile,Memory_footprint,SM_usage,Duration\r\n"
             "void gemm<float, 128, 64>(Params),1,0,100,5000\r\n"
             "elementwise,0,0,20,800\r\n"
             "broken row\r\n");
  write_file(be.c_str(),
             "Name,Profile,Memory_footprint,SM_usage,Duration\n"
             "conv_fwd,1,0,60,90000\n"
             "bias_relu,0,0,40,3000\n"
             "short_wide,0,0,148,2000\n");
  CHECK(orion_load_kernel_info(0, hp.c_str()) == 2);
  CHECK(orion_load_kernel_info(1, be.c_str()) == 3);
  CHECK(orion_load_kernel_info(2, be.c_str()) == -1);
  CHECK(orion_load_kernel_info(0, (dir + "/missing.csv").c_str()) == -1);
  CHECK(g_orion_state.op_info_vector[0][0].name == "void gemm<float, 128, 64>(Params)");
  CHECK(g_orion_state.op_info_vector[0][0].sm_used == 100);
  CHECK(g_orion_state.op_info_vector[1][1].duration == 3000.0f);

  Scheduler& s = g_scheduler;
  s.config_.num_sms = 148;
  s.num_clients_ = 2;
  CHECK(s.peek_sm_requirement(0) == 100);
  CHECK(s.peek_sm_requirement(1) == 60);
  CHECK(s.peek_sm_requirement(1, 1) == 40);
  CHECK(s.peek_sm_requirement(1, 3) == 60);  // wraps around the table

  // an opaque BE kernel (re-issued as it is, cannot yield)
  auto be_op = std::make_shared<OperationRecord>();
  be_op->type = OperationType::KERNEL_LAUNCH;
  be_op->client_idx = 1;
  auto& hpq = g_capture_state.client_queues[0];
  while (!hpq->empty()) hpq->try_pop();
  // 100 + 60 > 148 SMs but the HP queue is empty: BE may run
  CHECK(s.orion_should_schedule(be_op, 1));
  // HP work waiting: BE must wait
  hpq->push(create_operation(0, OperationType::CUBLAS_SGEMM));
  CHECK(!s.orion_should_schedule(be_op, 1));
  // next BE kernel needs 40 SMs: 100 + 40 fits
  g_orion_state.seen[1] = 1;
  CHECK(s.orion_should_schedule(be_op, 1));
  // 100 + 148 does not fit, but the BE kernel is short (2 us <= 50 us)
  g_orion_state.seen[1] = 2;
  CHECK(s.peek_duration(1) == 2000.0f);
  CHECK(s.orion_should_schedule(be_op, 1));
  g_orion_state.seen[1] = 0;
  // captured dense BE ops yield at tile boundaries: always admitted
  auto be_dense = std::make_shared<OperationRecord>();
  be_dense->type = OperationType::CUDNN_CONV_FWD;
  be_dense->client_idx = 1;
  CHECK(s.orion_should_schedule(be_dense, 1));
  // HP queue empty but its flag raised (a request in progress): still held
  hpq->try_pop();
  CHECK(s.orion_should_schedule(be_op, 1));
  int flag[2] = {4, 0};
  s.hp_flag_host_ = flag;
  CHECK(!s.orion_should_schedule(be_op, 1));
  flag[0] = 0;
  CHECK(s.orion_should_schedule(be_op, 1));
  s.hp_flag_host_ = nullptr;
  hpq->push(create_operation(0, OperationType::CUBLAS_SGEMM));
  // memory ops are never held back
  auto mem = std::make_shared<OperationRecord>();
  mem->type = OperationType::MEMCPY_ASYNC;
  CHECK(s.orion_should_schedule(mem, 1));
  // ISOLATED budgets: nothing to arbitrate
  Scheduler::GreenCtxConfig gc;
  gc.enabled = true;
  gc.hp_sm_count = 96;
  gc.be_sm_count = 52;
  CHECK(s.init_green_contexts(gc));
  CHECK(s.hp_quota() == 96 && s.be_quota() == 52);
  CHECK(s.orion_should_schedule(be_op, 1));
  gc.be_sm_count = 60;  // 96 + 60 > 148
  CHECK(!s.init_green_contexts(gc));
  s.clear_budgets();
  CHECK(s.hp_quota() == 0);
  hpq->try_pop();

  // wave-model budget choice: HP (100 SMs, 5 us) vs BE (60 SMs, 90 us)
  auto best = s.choose_best_green_ctx_config_from_profiles();
  CHECK(best.enabled);
  CHECK(best.hp_sm_count + best.be_sm_count == 148);
  CHECK(best.hp_sm_count % 8 == 0);
  CHECK(best.be_sm_count >= 60);  // BE dominates: it keeps at least one full wave

  orion_set_sm_threshold(74);
  CHECK(orion_get_sm_threshold() == 74);
  orion_set_client_kernels(1, 12);
  CHECK(g_orion_state.num_client_kernels[1] == 12);
  orion_reset_state();
  CHECK(g_orion_state.op_info_vector[0].empty());
}

static void test_profile_tables(const std::string& dir) {
  const std::string js = dir + "/profile.json";
  const std::string ym = dir + "/profile.yaml";
  write_file(js.c_str(),
             "{\"model_name\": \"m\", \"kernels\": [\n"
             " {\"kernel_id\": \"k1\", \"duration_ms\": 0.5, \"sm_needed\": 64, "
             "\"profile_type\": \"compute\", \"grid_size\": 128, \"block_size\": 256},\n"
             " {\"kernel_id\": \"k2\", \"duration_ms\": 1.5, \"sm_needed\": 8, "
             "\"profile_type\": \"memory\", \"grid_size\": 8, \"block_size\": 128}\n]}\n");
  write_file(ym.c_str(),
             "model_name: m\nkernels:\n"
             "  - kernel_id: k1  # comment\n    duration_ms: 0.25\n    sm_needed: 32\n"
             "    profile_type: compute\n"
             "  - kernel_id: k3\n    duration_ms: 2.0\n    sm_needed: 4\n"
             "    profile_type: memory\n");
  KernelProfileTable t;
  CHECK(t.load_from_json(js));
  CHECK(t.size() == 2);
  const KernelProfile* k2 = t.find("k2");
  CHECK(k2 && k2->sm_needed == 8 && k2->profile_type == ProfileType::MEMORY_BOUND);
  CHECK(t.compute_average_duration() == 1.0f);
  CHECK(t.load_from_yaml(ym));
  CHECK(t.size() == 3);  // k1 replaced, k3 added
  CHECK(t.find("k1")->duration_ms == 0.25f);
  CHECK(t.find("k3")->profile_type == ProfileType::MEMORY_BOUND);
  CHECK(orion_load_profile(js.c_str()) == 0);
  CHECK(orion_load_profile((dir + "/nope.json").c_str()) == -1);

  // profiler session round trip
  const std::string out = dir + "/recorded.json";
  orion_start_profiling("unit");
  KernelProfile p;
  p.kernel_id = "kx_gemm_tc<f32x3,128>";
  p.duration_ms = 0.125f;
  p.sm_needed = 148;
  p.profile_type = ProfileType::COMPUTE_BOUND;
  p.client_idx = 1;
  p.op_type = "CUBLAS_SGEMM";
  p.work = 2.0e9;
  g_profiler.record(p);
  orion_end_profiling(out.c_str());
  KernelProfileTable back;
  CHECK(back.load_from_json(out));
  const KernelProfile* r = back.find("kx_gemm_tc<f32x3,128>");
  CHECK(r && r->sm_needed == 148 && r->duration_ms == 0.125f);
  g_profiler.record(p);  // outside a session: dropped
  KernelProfileTable empty;
  g_profiler.get_profile_table(empty);
  CHECK(empty.size() == 1);
}

static void test_async_mode() {
  orion_set_async_mode(1);
  CHECK(orion_get_async_mode() == 1);
  orion_set_async_mode(7);  // invalid: ignored
  CHECK(orion_get_async_mode() == 1);
  orion_set_async_mode(0);
  CHECK(orion_get_async_mode() == 0);
}

static void test_error_latch() {
  set_last_error(1, cudaErrorInvalidValue);
  set_last_error(1, cudaErrorMemoryAllocation);  // first error is kept
  CHECK(get_and_clear_last_error(1) == cudaErrorInvalidValue);
  CHECK(get_and_clear_last_error(1) == cudaSuccess);
}

int main(int argc, char** argv) {
  const std::string dir = argc > 1 ? argv[1] : ".";
  test_capture_init();
  test_client_index_thread_local();
  test_stream_handle_maps();
  test_submit_and_complete();
  test_bounded_wait();
  test_timeout_paths_with_stalled_worker();
  test_bounded_push();
  test_queue_fifo_concurrent();
  test_kernel_info_and_decision(dir);
  test_profile_tables(dir);
  test_async_mode();
  test_error_latch();
  orion_shutdown();
  if (g_failures == 0) std::printf("ALL PASSED\n");
  return g_failures == 0 ? 0 : 1;
}
