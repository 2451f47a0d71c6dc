// kx_runtime.cu — device info, work-slot pool, tensor-map encoding.
#include "kx_runtime.cuh"

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <unordered_map>
#include <vector>

namespace kx {

static std::atomic<unsigned long long> g_device_allocs{0};

void note_device_alloc() { g_device_allocs.fetch_add(1, std::memory_order_relaxed); }

namespace {

std::mutex g_mu;
DeviceInfo g_dev[64];

struct SlotPool {
  WorkSlot* base = nullptr;
  int capacity = 0;
  int used = 0;
  std::unordered_map<cudaStream_t, int> by_stream;
};
SlotPool g_pools[64];

constexpr int kSlotsPerDevice = 4096;

thread_local const char* tl_kernel_name = "none";
thread_local int tl_last_grid = 0;
thread_local int tl_last_cuda_error = 0;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
bool g_encode_looked_up = false;

EncodeTiledFn encode_fn() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode_looked_up) {
    g_encode_looked_up = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  return g_encode;
}

using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const int*,
                                    const int*, cuuint32_t, cuuint32_t, const cuuint32_t*,
                                    CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeIm2colFn g_encode_im2col = nullptr;
bool g_encode_im2col_looked_up = false;

EncodeIm2colFn encode_im2col_fn() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode_im2col_looked_up) {
    g_encode_im2col_looked_up = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode_im2col = reinterpret_cast<EncodeIm2colFn>(fn);
    }
  }
  return g_encode_im2col;
}

}  // namespace

const DeviceInfo& device_info() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.device < 0) {
    cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.device = dev;
  }
  return d;
}

WorkSlot* work_slot_for(cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lk(g_mu);
  SlotPool& pool = g_pools[dev];
  if (pool.base == nullptr) {
    void* p = nullptr;
    note_device_alloc();
    if (cudaMalloc(&p, sizeof(WorkSlot) * kSlotsPerDevice) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(WorkSlot) * kSlotsPerDevice) != cudaSuccess) return nullptr;
    if (cudaDeviceSynchronize() != cudaSuccess) return nullptr;
    pool.base = static_cast<WorkSlot*>(p);
    pool.capacity = kSlotsPerDevice;
  }
  auto it = pool.by_stream.find(stream);
  if (it != pool.by_stream.end()) return pool.base + it->second;
  if (pool.used >= pool.capacity) return nullptr;
  int idx = pool.used++;
  pool.by_stream.emplace(stream, idx);
  return pool.base + idx;
}

namespace {
struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
  int64_t last_use_ns = 0;
};
std::unordered_map<cudaStream_t, Scratch> g_scratch[64][3];
size_t g_scratch_total[64] = {0};

int64_t now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

// Budget for the scratch buffers of one device: KX_SCRATCH_BUDGET_MB, else a
// quarter of the device's memory (at most 24 GiB).
size_t scratch_budget(int dev) {
  static size_t budget[64] = {0};
  if (budget[dev] == 0) {
    size_t b = 0;
    if (const char* s = std::getenv("KX_SCRATCH_BUDGET_MB")) b = std::strtoull(s, nullptr, 10) << 20;
    if (b == 0) {
      size_t free_b = 0, total_b = 0;
      cudaMemGetInfo(&free_b, &total_b);
      b = total_b / 4;
      if (b > (24ull << 30)) b = 24ull << 30;
      if (b < (1ull << 30)) b = 1ull << 30;
    }
    budget[dev] = b;
  }
  return budget[dev];
}

// Frees the buffers of streams other than `keep` that no op has asked for in
// the last `idle_ns`, oldest first, until `need` more bytes fit the budget
// (need = SIZE_MAX: every such buffer).  A buffer idle that long belongs to a
// stream whose ops were enqueued long ago; cudaFree waits for the device, so
// none of them is still running.  Caller holds g_mu.
void evict_idle(int dev, cudaStream_t keep, size_t need, int64_t idle_ns) {
  const int64_t now = now_ns();
  const size_t budget = scratch_budget(dev);
  while (need == SIZE_MAX || g_scratch_total[dev] + need > budget) {
    Scratch* oldest = nullptr;
    for (int slot = 0; slot < 3; ++slot)
      for (auto& kv : g_scratch[dev][slot]) {
        Scratch& s = kv.second;
        if (kv.first == keep || s.ptr == nullptr || now - s.last_use_ns < idle_ns) continue;
        if (oldest == nullptr || s.last_use_ns < oldest->last_use_ns) oldest = &s;
      }
    if (oldest == nullptr) return;
    note_device_alloc();
    cudaFree(oldest->ptr);
    g_scratch_total[dev] -= oldest->bytes;
    oldest->ptr = nullptr;
    oldest->bytes = 0;
  }
}
}  // namespace

void* scratch_for(cudaStream_t stream, size_t bytes, int slot) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (slot < 0 || slot > 2) return nullptr;
  if (bytes == 0) bytes = 256;
  std::lock_guard<std::mutex> lk(g_mu);
  Scratch& s = g_scratch[dev][slot][stream];
  s.last_use_ns = now_ns();
  if (s.bytes >= bytes) return s.ptr;
  if (s.ptr != nullptr) {
    note_device_alloc();
    cudaFree(s.ptr);
    g_scratch_total[dev] -= s.bytes;
    s.ptr = nullptr;
    s.bytes = 0;
  }
  size_t want = bytes + bytes / 8;  // headroom against repeated small growth
  want = (want + 255) & ~static_cast<size_t>(255);
  // streams come and go (a client may run each phase on a new stream): keep
  // the buffers of streams idle for a second within the budget
  evict_idle(dev, stream, want, 1000000000LL);
  note_device_alloc();
  if (cudaMalloc(&s.ptr, want) != cudaSuccess) {
    cudaGetLastError();
    // out of memory: give back every other stream's idle buffer and retry
    evict_idle(dev, stream, SIZE_MAX, 100000000LL);
    note_device_alloc();
    if (cudaMalloc(&s.ptr, want) != cudaSuccess) {
      cudaGetLastError();
      s.ptr = nullptr;
      return nullptr;
    }
  }
  s.bytes = want;
  g_scratch_total[dev] += want;
  return s.ptr;
}

Exec resolve_exec(const kx_exec* ex) {
  Exec e;
  if (ex != nullptr) {
    e.stream = static_cast<cudaStream_t>(ex->stream);
    e.sm_quota = ex->sm_quota;
    e.yield_flag = ex->yield_flag;
    e.done_flag = ex->done_flag;
    e.max_tiles = ex->max_tiles;
    if (ex->timeout_ns != 0) e.timeout_ns = ex->timeout_ns;
    e.fp32_mode = ex->fp32_mode;
    e.err_word = ex->err_word;
  }
  return e;
}

int persistent_grid(const Exec& e, int tiles) {
  int sms = device_info().num_sms;
  int cap = (e.sm_quota > 0 && e.sm_quota < sms) ? e.sm_quota : sms;
  if (tiles < cap) cap = tiles;
  tl_last_grid = cap < 1 ? 1 : cap;
  return tl_last_grid;
}

namespace {
// Tensor maps by their complete description.  An encoded map is a pure
// function of these arguments, and a model step's activations and weights
// come back at the same addresses step after step, so most encodes repeat
// (a GEMM launch encodes up to five maps, a microsecond or more each on the
// dispatching thread).  Per thread, so no lock; cleared when it grows large.
struct MapKey {
  uint64_t w[24];
  int n;
  bool operator==(const MapKey& o) const {
    return n == o.n && std::memcmp(w, o.w, sizeof(uint64_t) * n) == 0;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    for (int i = 0; i < k.n; ++i) h = (h ^ k.w[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};
thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> tl_map_cache;
constexpr size_t kMapCacheMax = 8192;
}  // namespace

bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swz, const uint32_t* elem_strides) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  if (rank < 1 || rank > 5) return false;
  MapKey key;
  key.n = 0;
  key.w[key.n++] = reinterpret_cast<uintptr_t>(base);
  key.w[key.n++] = (static_cast<uint64_t>(dt) << 32) | (static_cast<uint64_t>(swz) << 8) |
                   static_cast<uint64_t>(rank);
  for (int i = 0; i < rank; ++i) key.w[key.n++] = dims[i];
  for (int i = 0; i + 1 < rank; ++i) key.w[key.n++] = strides_bytes[i];
  for (int i = 0; i < rank; ++i)
    key.w[key.n++] = (static_cast<uint64_t>(box[i]) << 32) |
                     (elem_strides != nullptr ? elem_strides[i] : 1u);
  auto hit = tl_map_cache.find(key);
  if (hit != tl_map_cache.end()) {
    std::memcpy(map, &hit->second, sizeof(CUtensorMap));
    return true;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || dims[i] > (1ull << 32)) return false;
    if (box[i] == 0 || box[i] > 256) return false;
    d[i] = dims[i];
    b[i] = box[i];
    if (elem_strides != nullptr) {
      if (elem_strides[i] == 0 || elem_strides[i] > 8) return false;
      es[i] = elem_strides[i];
    }
  }
  for (int i = 0; i + 1 < rank; ++i) {
    if ((strides_bytes[i] & 15u) != 0 || strides_bytes[i] >= (1ull << 40)) return false;
    s[i] = strides_bytes[i];
  }
  std::memset(map, 0, sizeof(CUtensorMap));
  CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (tl_map_cache.size() >= kMapCacheMax) tl_map_cache.clear();
  tl_map_cache.emplace(key, *map);
  return true;
}

bool encode_im2col_map(CUtensorMap* map, const void* base, const uint64_t* dims,
                       const uint64_t* strides_bytes, const int* lower, const int* upper,
                       uint32_t channels, uint32_t pixels, const uint32_t* elem_strides,
                       CUtensorMapSwizzle swz) {
  EncodeIm2colFn fn = encode_im2col_fn();
  if (fn == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if (channels == 0 || channels * 4 > 128 || pixels == 0 || pixels > 1024) return false;
  cuuint64_t d[4];
  cuuint64_t s[3];
  cuuint32_t es[4];
  for (int i = 0; i < 4; ++i) {
    if (dims[i] == 0 || dims[i] > (1ull << 32)) return false;
    if (elem_strides[i] == 0 || elem_strides[i] > 8) return false;
    d[i] = dims[i];
    es[i] = elem_strides[i];
  }
  for (int i = 0; i < 3; ++i) {
    if ((strides_bytes[i] & 15u) != 0 || strides_bytes[i] >= (1ull << 40)) return false;
    s[i] = strides_bytes[i];
  }
  for (int i = 0; i < 2; ++i)
    if (lower[i] < -128 || lower[i] > 127 || upper[i] < -128 || upper[i] > 127) return false;
  std::memset(map, 0, sizeof(CUtensorMap));
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), d, s, lower,
                  upper, channels, pixels, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_map_3d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t batch, uint64_t ld_elems,
                   uint64_t batch_stride_elems, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swz) {
  uint64_t dims[3] = {inner, outer, batch};
  uint32_t box[3] = {box_inner, box_outer, 1};
  if (batch <= 1 || batch_stride_elems == 0) {
    uint64_t strides[1] = {ld_elems * static_cast<uint64_t>(esize)};
    dims[2] = 1;
    // rank-2 map; the kernel's third coordinate is then always 0
    uint64_t d3[3] = {inner, outer, 1};
    uint64_t s3[2] = {strides[0], strides[0] * outer};
    // keep the rank at 3 so kernels issue one instruction form
    if ((s3[1] & 15u) != 0) s3[1] = (s3[1] + 15u) & ~static_cast<uint64_t>(15u);
    return encode_map(map, dt, 3, base, d3, s3, box, swz);
  }
  uint64_t strides[2] = {ld_elems * static_cast<uint64_t>(esize),
                         batch_stride_elems * static_cast<uint64_t>(esize)};
  return encode_map(map, dt, 3, base, dims, strides, box, swz);
}

void set_last_kernel_name(const char* name) { tl_kernel_name = name; }

bool single_box_disabled() {
  static const bool off = [] {
    const char* v = std::getenv("KX_SINGLE_BOX");
    return v != nullptr && v[0] == '0';
  }();
  return off;
}

unsigned long long* pipe_stats_begin() {
  static const bool on = [] {
    const char* s = std::getenv("KX_PIPE_STATS");
    return s != nullptr && s[0] == '1';
  }();
  if (!on) return nullptr;
  static unsigned long long* buf = nullptr;
  const size_t bytes = sizeof(unsigned long long) * kPipeStats * 1024;
  if (buf == nullptr) note_device_alloc();
  if (buf == nullptr && cudaMalloc(&buf, bytes) != cudaSuccess) {
    buf = nullptr;
    return nullptr;
  }
  cudaMemset(buf, 0, bytes);
  return buf;
}

void pipe_stats_end(unsigned long long* buf, const char* kernel, cudaStream_t stream, int grid) {
  if (buf == nullptr || grid <= 0 || grid > 1024) return;
  std::vector<unsigned long long> h(static_cast<size_t>(grid) * kPipeStats);
  cudaStreamSynchronize(stream);
  cudaMemcpy(h.data(), buf, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  double sum[kPipeStats] = {0};
  for (int c = 0; c < grid; ++c)
    for (int i = 0; i < kPipeStats; ++i) sum[i] += static_cast<double>(h[c * kPipeStats + i]);
  const double tot = sum[PS_TOTAL] > 0 ? sum[PS_TOTAL] : 1.0;
  std::fprintf(stderr,
               "[kx pipe] %s grid %d cycles/CTA %.0f | share: prologue %.3f prod-empty %.3f "
               "prod-ring %.3f prod-issue %.3f mma-data %.3f mma-tmem %.3f mma-ring %.3f "
               "mma-issue %.3f mma-loop %.3f mma-kloop %.3f epi-tfull %.3f epi-fold %.3f "
               "epi-emit %.3f (proxy fences %.3f)\n",
               kernel, grid, tot / grid, sum[PS_PROLOGUE] / tot, sum[PS_PROD_EMPTY] / tot,
               sum[PS_PROD_RING] / tot, sum[PS_PROD_ISSUE] / tot, sum[PS_MMA_DATA] / tot,
               sum[PS_MMA_TMEM] / tot,
               sum[PS_MMA_RING] / tot, sum[PS_MMA_ISSUE] / tot, sum[PS_MMA_LOOP] / tot,
               sum[PS_MMA_KLOOP] / tot,
               sum[PS_EPI_TFULL] / tot,
               sum[PS_EPI_FOLD] / tot, sum[PS_EPI_EMIT] / tot, sum[PS_EPI_STWAIT] / tot);
}

static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void note_cuda_error(cudaError_t e) { tl_last_cuda_error = static_cast<int>(e); }

}  // namespace kx

extern "C" unsigned long long kx_launch_count(void) {
  return kx::g_launches.load(std::memory_order_relaxed);
}

extern "C" unsigned long long kx_device_alloc_count(void) {
  return kx::g_device_allocs.load(std::memory_order_relaxed);
}

extern "C" int kx_num_sms(void) { return kx::device_info().num_sms; }

extern "C" const char* kx_last_kernel_name(void) { return kx::tl_kernel_name; }

extern "C" int kx_last_grid(void) { return kx::tl_last_grid; }

extern "C" int kx_last_cuda_error(void) { return kx::tl_last_cuda_error; }

extern "C" const char* kx_version(void) { return "kx 0.1 sm_100a"; }

extern "C" int kx_host_flags_alloc(int count, int** host, int** dev) {
  if (count <= 0 || host == nullptr || dev == nullptr) return KX_ERR_INVALID;
  void* h = nullptr;
  if (cudaHostAlloc(&h, sizeof(int) * count, cudaHostAllocMapped | cudaHostAllocPortable) !=
      cudaSuccess)
    return KX_ERR_NOMEM;
  std::memset(h, 0, sizeof(int) * count);
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
    cudaFreeHost(h);
    return KX_ERR_DEVICE;
  }
  *host = static_cast<int*>(h);
  *dev = static_cast<int*>(d);
  return KX_OK;
}

extern "C" int kx_host_flags_free(int* host) {
  if (host == nullptr) return KX_OK;
  return cudaFreeHost(host) == cudaSuccess ? KX_OK : KX_ERR_DEVICE;
}

namespace kx {
// One thread polls the flag with the same give-up rule as the persistent
// kernels' bounded waits: re-check a deadline every 256 polls.
__global__ void kx_wait_flag_kernel(const volatile int* flag, unsigned long long timeout_ns,
                                    int* status) {
  uint64_t t0 = globaltimer();
  uint32_t polls = 0;
  while (*flag == 0) {
    if ((++polls & 255u) == 0 && globaltimer() - t0 > timeout_ns) {
      *status = KX_ERR_TIMEOUT;
      return;
    }
  }
  *status = KX_OK;
}
}  // namespace kx

extern "C" int kx_wait_flag(void* stream, const volatile int* flag,
                            unsigned long long timeout_ns, int* status) {
  if (flag == nullptr || status == nullptr) return KX_ERR_INVALID;
  kx::note_launch();
  kx::kx_wait_flag_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, timeout_ns,
                                                                         status);
  return kx::launch_status();
}
