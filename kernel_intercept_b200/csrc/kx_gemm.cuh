// kx_gemm.cuh — persistent, SM-quota-aware tcgen05 GEMM for sm_100a.
//
// Computes the cuBLAS column-major contract
//     D[b] = epi(alpha * op(A[b]) * op(B[b]) + beta * C[b] + bias)
// for the ops the kernel_intercept shim captures (cublasSgemm_v2,
// cublasSgemmStridedBatched, cublasGemmEx, cublasGemmStridedBatchedEx,
// cublasLtMatmul; see src/cublas_intercept.cpp:455-491 and 1453-1500 of the
// reference for the calls this replaces).
//
// Mapping onto the tensor core.  GEMM rows i (M) become UMMA M (TMEM lanes),
// GEMM columns j (N) become UMMA N (TMEM columns).  Because C is column-major,
// the TMEM lane -> row mapping makes every epilogue store a coalesced
// 32-row column segment.  op(A) is K-major in memory when transa = T and
// M-major when transa = N; op(B) is K-major when transb = N and N-major when
// transb = T.  Both majors are native UMMA operand layouts, so no transpose
// pass is ever needed.
//
// Warp roles (256 threads, one CTA per SM):
//   warp 0      TMA producer: takes tiles from the global tile queue,
//               publishes them to the other roles, streams A/B k-blocks.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma.
//   warps 2-3   3xTF32 with in-kernel split only: compute the low parts.
//   warps 4-7   epilogue: TMEM -> registers -> alpha/beta/bias/act -> HBM.
// fp32 (3xTF32): each operand x is used as hi (a kind::tf32 MMA reads only
// its top 19 bits, i.e. trunc_tf32(x)) and lo = x - trunc_tf32(x); three
// MMAs per k-step accumulate lo*hi + hi*lo + hi*hi.  When both operands are
// reused enough, a split kernel writes lo to global memory before the launch
// and TMA brings it beside hi; otherwise warps 2-3 compute it per k-block.
// The accumulator is double-buffered in TMEM so the epilogue of tile t
// overlaps the MMAs of tile t+1.
//
// Scheduling controls (replacing the reference's green-context SM split,
// src/scheduler.cpp:244-446): the grid is bounded by the caller's SM quota;
// tiles come from an atomic queue in a per-stream work slot, so a launch
// that yields (host-mapped flag raised, or per-launch tile budget used up)
// can be continued by relaunching the same call.
#pragma once
#include <mutex>
#include <unordered_map>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kx_ptx.cuh"

namespace kx {

enum class Arith : int { F32x3 = 0, TF32 = 1, BF16 = 2, F16 = 3 };

// Per-stream bookkeeping for persistent launches (device memory).
struct WorkSlot {
  unsigned int next_tile;  // head of the tile queue
  unsigned int exited;     // CTAs of the running launch that have retired
  int status;              // last launch: 1 = op complete, 0 = yielded
  int err;                 // first device-side error (KX_ERR_TIMEOUT)
};

enum : int { DT_F32 = 0, DT_F16 = 2, DT_BF16 = 14 };

struct GemmParams {
  int m, n, k;
  int num_mb, num_nb, num_kb;
  int tiles_per_batch, num_tiles;
  int a_bcast, b_bcast;  // batch stride 0: use batch coordinate 0
  float alpha, beta;
  const float* alpha_dev;  // device pointer mode (nullable)
  const float* beta_dev;
  void* D;
  long long ldd, strideD;
  int d_type;
  const void* C;
  long long ldc, strideC;
  int c_type;
  int relu, gelu;
  const void* bias;
  int bias_type;
  WorkSlot* work;
  const volatile int* yield_flag;
  volatile int* done_flag;
  int max_tiles;
  unsigned long long timeout_ns;
  int* err_word;
  // split-K: each output tile is computed as `splits` K slices of
  // `kb_per_split` k-blocks whose fp32 partials go to ws
  // ([batch][splits][n][m], column-major per slice); kx_splitk_reduce then
  // applies alpha / beta / bias / activation.  splits == 1: direct epilogue.
  int splits, kb_per_split;
  float* ws;
  // 3xTF32: 1 = the low parts of A and B were written to global memory
  // before the launch and arrive by TMA (maps tmAlo / tmBlo); 0 = warps 2-3
  // compute them in shared memory from each k-block.
  int presplit;
  // Implicit-GEMM convolution (kernel instantiated with CONV = true).  The A
  // operand is a 4-D TMA box (32 channels x cv_wbox x cv_hbox output pixels
  // of one image) of an NHWC staging copy of x whose channels are padded to
  // cv_cb blocks of 32; K runs over (filter tap, channel block).  An output
  // tile is cv_hbox rows x cv_wbox columns of output pixels (cv_tiles_w tiles
  // across a row); batch = image; D is NCHW (ld = P*Q).
  int cv_p, cv_q, cv_wbox, cv_hbox, cv_tiles_w, cv_s, cv_cb;
  int cv_pad_h, cv_pad_w, cv_str_h, cv_str_w, cv_dil_h, cv_dil_w;
  // cv_im2col = 1: the A operand comes by im2col-mode TMA instead: M runs
  // over all N*P*Q output pixels (batch 1), an A tile is 128 consecutive
  // output pixels whatever row or image they fall in, and output row f is
  // pixel f % cv_pq of image f / cv_pq (D offset image * strideD + pixel).
  int cv_im2col, cv_pq;
  // cv_wgrad = 1: backward filter (kernel instantiated with CONV = true and an
  // MN-major B).  M = output channels, N = (filter tap, input channel) as
  // cv_nb_per_tap channel blocks of BN per tap, K = output pixels of every
  // image in blocks of 32 (cv_pb blocks per image; pixels past P*Q read zero
  // from dy).  A = dy as a {P*Q, K, N} map; B = 32 pixels x 32 channels
  // im2col-mode loads of the NHWC staging of x at the tile's tap.  Partials
  // always go to ws (or to D = ws when splits == 1); a reduce kernel writes
  // dw.
  int cv_wgrad, cv_pb, cv_nb_per_tap;
  // 1: the M/N-major A (B) tile arrives as one 4-D TMA box {CHUNK, BK,
  // chunks, 1} of a map whose third dimension steps CHUNK elements through
  // M (N), instead of one load per 128-byte chunk (M, N multiples of CHUNK).
  int a_single, b_single;
  // Pipeline diagnostics (nullable): per CTA kPipeStats clock64 counters of
  // the time each role spends waiting (see PipeStat).
  unsigned long long* pipe_stats;
  // 1: 16-bit D stored 32 rows x 64 columns per TMA store (map tmD's box is
  // {32, 64}); only with tma_store, for plain GEMMs.
  int wide16;
  // 3xTF32: k-blocks per TMEM accumulator segment (0 = Cfg::SEG)
  int seg_kb;
  // 1: the epilogue writes D through shared memory and TMA stores (map tmD:
  // {m, n, batch} for GEMMs, {Q, P, K, N} for box-tiled convolutions,
  // {P*Q, K, N} for im2col convolutions); 0: one st.global per element
  // (unaligned D, split-K partials).
  int tma_store;
};

enum PipeStat : int {
  PS_PROD_EMPTY = 0,  // producer waits for a free stage
  PS_PROD_RING,       // producer waits for a free tile-ring slot
  PS_MMA_DATA,        // MMA issuer waits for a stage's data
  PS_MMA_TMEM,        // MMA issuer waits for a free accumulator buffer
  PS_MMA_RING,        // MMA issuer waits for the next tile id
  PS_EPI_TFULL,       // epilogue (warp 4) waits for an accumulator
  PS_TOTAL,           // CTA lifetime
  PS_PROLOGUE,        // barrier init + TMEM allocation
  PS_MMA_ISSUE,       // MMA issuer: issuing a k-block's MMAs and its commit
  PS_EPI_FOLD,        // epilogue (warp 4): folding segments from TMEM
  PS_EPI_EMIT,        // epilogue (warp 4): output stores
  PS_EPI_STWAIT,      // epilogue (warp 4): proxy fences before its TMA stores
  PS_PROD_ISSUE,      // producer: coordinates and TMA issue of a k-block's loads
  PS_MMA_LOOP,        // MMA issuer: its whole tile loop
  PS_MMA_KLOOP,       // MMA issuer: inside its k-block loops (waits, issue, bookkeeping)
  kPipeStats = 15
};

KX_DEV bool timed_wait(uint32_t bar, uint32_t parity, const WaitCtl& wc,
                       unsigned long long* acc) {
  if (acc == nullptr) return mbar_wait(bar, parity, wc);
  const long long t0 = clock64();
  const bool ok = mbar_wait(bar, parity, wc);
  *acc += static_cast<unsigned long long>(clock64() - t0);
  return ok;
}

template <int BN_, Arith AR_, bool A_MN_, bool B_MN_, bool PAIR_ = false>
struct GemmCfg {
  static constexpr int BM = 128;  // accumulator rows per CTA
  static constexpr int BN = BN_;
  // PAIR: a 2-CTA cluster computes a 256 x BN tile with cta_group::2 MMAs
  // issued by the leader; each CTA loads its 128 rows of A and BN/2 rows of B
  // (3xTF32 with pre-split low parts only).
  static constexpr bool PAIR = PAIR_;
  static constexpr int MMA_M = PAIR ? 2 * BM : BM;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B in this CTA
  static constexpr Arith AR = AR_;
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr int ESIZE = (AR == Arith::BF16 || AR == Arith::F16) ? 2 : 4;
  static constexpr int BK = 128 / ESIZE;       // elements of K per 128-byte row
  static constexpr int UMMA_K = 32 / ESIZE;    // K per tcgen05.mma (8 tf32 / 16 x 16-bit)
  static constexpr int CHUNK = 128 / ESIZE;    // M/N elements per 128-byte chunk (MN-major)
  static constexpr bool SPLIT = (AR == Arith::F32x3);
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = B_ROWS * 128;
  static constexpr int LOAD_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGE_BYTES = LOAD_BYTES * (SPLIT ? 2 : 1);
  static constexpr int STAGES_RAW = (192 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int STAGE_REGION = STAGES * STAGE_BYTES;
  static constexpr int RING = 4;  // depth of the tile-id broadcast ring
  // TMEM columns of one accumulator buffer.  3xTF32 keeps two BN-wide
  // halves: [0, BN) = hi*hi and [BN, 2BN) = hi*lo + lo*hi (see the MMA
  // issuer).  The tensor core's fp32 accumulate truncates, so each add into
  // the large half costs up to one ulp of the running sum; the small half is
  // 2^-11 of it, and its truncations are negligible.  One CTA issues hi*hi
  // and hi*lo as one MMA over [B_hi; B_lo] (MERGED); a pair issues three.
  static constexpr bool MERGED = SPLIT && !PAIR;
  static constexpr int ACC_COLS = SPLIT ? 2 * BN : BN;
  static constexpr int TMEM_COLS = (2 * ACC_COLS) <= 32 ? 32 : (2 * ACC_COLS) <= 64 ? 64 : (2 * ACC_COLS) <= 128 ? 128 : (2 * ACC_COLS) <= 256 ? 256 : 512;
  static constexpr int THREADS = 256;
  static constexpr int NUM_CONS = 1 + 4;  // ring consumers: MMA issuer + epilogue warps
  // 3xTF32: the tensor core's fp32 accumulation does not round to nearest, so
  // the error of one TMEM accumulator grows linearly with its K length.  The
  // K loop is therefore cut into segments of SEG k-blocks (256 of K); each
  // segment accumulates in its own TMEM buffer and the epilogue warps fold it
  // into round-to-nearest fp32 registers.
  static constexpr bool PROMOTE = (AR == Arith::F32x3);
  static constexpr int SEG = PROMOTE ? 8 : (1 << 30);
  // Descriptor geometry.  K-major: 128-byte swizzle (layout 2), SBO 1024.
  // M/N-major 16-bit: layout 2, 8-row atoms, SBO 1024.  M/N-major tf32:
  // 32-byte-atom swizzle (layout 1), 4-row atoms, SBO 512.
  static constexpr bool A_MN32 = A_MN && ESIZE == 4;
  static constexpr bool B_MN32 = B_MN && ESIZE == 4;
  static constexpr uint32_t A_LBO = A_MN ? BK * 128 : 16;
  static constexpr uint32_t B_LBO = B_MN ? BK * 128 : 16;
  static constexpr uint32_t A_SBO = A_MN32 ? 512 : 1024;
  static constexpr uint32_t B_SBO = B_MN32 ? 512 : 1024;
  static constexpr uint32_t A_LAYOUT = A_MN32 ? 1 : 2;
  static constexpr uint32_t B_LAYOUT = B_MN32 ? 1 : 2;
  static_assert(!PROMOTE || BN <= 128, "3xTF32 keeps a BN-wide fp32 accumulator per thread");
  static_assert(!PAIR || (!A_MN && !B_MN), "CTA pairs load K-major tiles only");
  static constexpr uint32_t FMT = (AR == Arith::BF16) ? 1u : (AR == Arith::F16) ? 0u : 2u;
  static constexpr uint32_t IDESC = make_idesc(FMT, A_MN, B_MN, MMA_M, BN);
  // 3xTF32 on one CTA: A_hi x [B_hi; B_lo] as one N = 2*BN product
  static constexpr uint32_t IDESC2 = make_idesc(FMT, A_MN, B_MN, MMA_M, MERGED ? 2 * BN : BN);
  // epilogue staging (4 warps x 2 buffers of 32 x 32 fp32) after the stages,
  // then the barrier block
  static constexpr int EPI_OFF = STAGE_REGION;
  static constexpr int EPI_BYTES = 4 * 2 * 4096;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + BAR_OFF + 1024 /*barriers*/;
  static_assert(STAGES >= 2, "not enough shared memory for two stages");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "bad BN");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(!PAIR || (BN >= 64 && (SPLIT || (!A_MN && !B_MN && ESIZE == 2))),
                "CTA pairs: 3xTF32, or 16-bit operands with K-major A and B; BN >= 64");
};

struct SmemBars {
  uint64_t full[8], conv[8], empty[8];
  uint64_t tfull[2], tempty[2];
  uint64_t ring_full[4], ring_empty[4];
  uint64_t final_mma;
  int ring[4];
  uint32_t tmem_base;
  int abort_flag;
};

KX_DEV float load_scalar(const void* p, int type, size_t idx) {
  if (type == DT_F32) return static_cast<const float*>(p)[idx];
  unsigned short h = static_cast<const unsigned short*>(p)[idx];
  if (type == DT_BF16) return __uint_as_float(static_cast<uint32_t>(h) << 16);
  return __half2float(__ushort_as_half(h));
}

KX_DEV void store_scalar(void* p, int type, size_t idx, float v) {
  if (type == DT_F32) {
    static_cast<float*>(p)[idx] = v;
  } else if (type == DT_BF16) {
    static_cast<__nv_bfloat16*>(p)[idx] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(p)[idx] = __float2half_rn(v);
  }
}

KX_DEV float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

// Tile id -> (batch, K slice, M block, N block).  Slices are outermost within
// a batch so that concurrently running CTAs share A/B rows in L2.
KX_DEV void decode_tile(int tile, const GemmParams& p, int& b, int& ks, int& mb, int& nb) {
  b = tile / p.tiles_per_batch;
  int t = tile - b * p.tiles_per_batch;
  const int per_split = p.num_mb * p.num_nb;
  ks = t / per_split;
  t -= ks * per_split;
  // grouped raster: 8 M-blocks share each sweep over N for L2 reuse of B
  constexpr int G = 8;
  int group_span = G * p.num_nb;
  int g = t / group_span;
  int first_mb = g * G;
  int gsize = p.num_mb - first_mb < G ? p.num_mb - first_mb : G;
  int r = t - g * group_span;
  mb = first_mb + r % gsize;
  nb = r / gsize;
}

// First k-block and k-block count of a tile's K slice.
KX_DEV void tile_k_range(int tile, const GemmParams& p, int& kb0, int& nkb) {
  const int ks = (tile % p.tiles_per_batch) / (p.num_mb * p.num_nb);
  kb0 = ks * p.kb_per_split;
  const int end = kb0 + p.kb_per_split < p.num_kb ? kb0 + p.kb_per_split : p.num_kb;
  nkb = end - kb0;
}

// Sums the split-K partials of every output element and applies the
// epilogue.  Runs after the GEMM kernel on the same stream; does nothing when
// that launch stopped early (yield or tile budget), in which case the
// relaunch that completes the tiles is followed by another reduce.  One
// thread per output element (column-major: consecutive threads take
// consecutive rows, so partial reads and output writes coalesce); I is the
// index type, 32-bit whenever the batch of planes has fewer than 2^31
// elements (integer division is the costliest part of the index decode).
template <class I>
KX_DEV void splitk_reduce_body(const GemmParams& p, int batch) {
  const float alpha = p.alpha_dev ? *p.alpha_dev : p.alpha;
  const float beta = p.beta_dev ? *p.beta_dev : p.beta;
  const I m = static_cast<I>(p.m);
  const I mn = m * static_cast<I>(p.n);
  const I total = mn * static_cast<I>(batch);
  for (I e = static_cast<I>(blockIdx.x) * 256 + threadIdx.x; e < total;
       e += static_cast<I>(gridDim.x) * 256) {
    const I b = e / mn;
    const I r = e - b * mn;
    const I col = r / m;
    const I row = r - col * m;
    const float* src = p.ws + static_cast<long long>(b) * p.splits * mn + r;
    float acc = 0.f;
    for (int s = 0; s < p.splits; ++s) acc += src[static_cast<long long>(s) * mn];
    float o = alpha * acc;
    // im2col convolution: row = image * P*Q + pixel
    long long cb = static_cast<long long>(b) * p.strideC, db = static_cast<long long>(b) * p.strideD;
    long long pix = row;
    if (p.cv_im2col) {
      const I img = row / static_cast<I>(p.cv_pq);
      pix = row - img * static_cast<I>(p.cv_pq);
      cb = static_cast<long long>(img) * p.strideC;
      db = static_cast<long long>(img) * p.strideD;
    }
    if (beta != 0.f)
      o += beta * load_scalar(p.C, p.c_type, cb + static_cast<long long>(col) * p.ldc + pix);
    if (p.bias != nullptr) o += load_scalar(p.bias, p.bias_type, static_cast<size_t>(row));
    if (p.relu) o = fmaxf(o, 0.f);
    if (p.gelu) o = gelu_tanh(o);
    store_scalar(p.D, p.d_type, db + static_cast<long long>(col) * p.ldd + pix, o);
  }
}

static __global__ void __launch_bounds__(256) kx_splitk_reduce(const GemmParams p, int batch) {
  if (p.work->status != 1) return;
  const long long total = static_cast<long long>(p.m) * p.n * batch;
  if (total + 256LL * gridDim.x < (1LL << 31))
    splitk_reduce_body<int>(p, batch);
  else
    splitk_reduce_body<long long>(p, batch);
}

// Grid of kx_splitk_reduce: one thread per element, at most 8 blocks per SM.
inline int splitk_reduce_grid(int m, int n, int batch, int sms) {
  const long long blocks = (static_cast<long long>(m) * n * batch + 255) / 256;
  const long long cap = 8LL * sms;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// ---------------------------------------------------- CTA-pair launches --

// Largest even grid <= want whose 2-CTA clusters can all be resident at once.
// Tiles come from an atomic queue, so correctness does not depend on it; a
// cluster that only starts after the others finished finds the queue empty.
template <class K>
int pair_grid(K kern, int threads, int smem, int want) {
  static std::mutex mu;
  static std::unordered_map<long long, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const long long key = (static_cast<long long>(reinterpret_cast<uintptr_t>(kern)) << 8) ^ dev;
  int clusters = -1;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) clusters = it->second;
  }
  if (clusters < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = clusters;
  }
  int g = want & ~1;
  if (clusters > 0 && 2 * clusters < g) g = 2 * clusters;
  return clusters > 0 ? g : 0;
}

template <class K, class... Args>
cudaError_t launch_pair(K kern, int grid, int threads, int smem, cudaStream_t stream,
                        const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// CONV = true: implicit-GEMM convolution (see GemmParams::cv_*): the A tile
// of k-block (tap, channel block) is the 4-D box of the NHWC staging copy
// shifted by the tap's offset, so TMA zero-fills the padding border.
template <class Cfg, bool CONV = false>
__global__ void __launch_bounds__(256, 1)
    kx_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmAlo,
                      const __grid_constant__ CUtensorMap tmBlo,
                      const __grid_constant__ CUtensorMap tmD, const GemmParams p) {
  static_assert(!CONV || (Cfg::AR == Arith::F32x3 && !Cfg::A_MN),
                "implicit convolution: 3xTF32 with a K-major A tile");
  const long long t_start = clock64();  // CTA lifetime starts here
  constexpr int S = Cfg::STAGES;
  constexpr int R = Cfg::RING;
  // CTA pair (Cfg::PAIR): rank 0 leads (tile ids, MMAs), rank 1 follows
  constexpr bool PAIR = Cfg::PAIR;
  // pairs: the follower's TMA loads complete on the leader's stage barriers
  // (.cta_group::2 loads), so the leader's MMA thread waits on one barrier
  constexpr bool DIRECT = PAIR;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  // in-kernel 3xTF32 split (warps 2-3) unless the low parts come by TMA
  const bool convert = Cfg::SPLIT && !CONV && !PAIR && p.presplit == 0;
  const bool lo_by_tma = Cfg::SPLIT && !convert;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SmemBars* sb = reinterpret_cast<SmemBars*>(smem + Cfg::BAR_OFF);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  // stage layout [A | B] (one operand set) or [A | A_lo | B | B_lo] (3xTF32:
  // B_lo directly after B, so that B_hi and B_lo read as one 2*BN-row operand)
  auto stageA = [&](uint32_t s) { return smem + s * Cfg::STAGE_BYTES; };
  auto stageAlo = [&](uint32_t s) { return smem + s * Cfg::STAGE_BYTES + Cfg::A_BYTES; };
  auto stageB = [&](uint32_t s) {
    return smem + s * Cfg::STAGE_BYTES + (Cfg::SPLIT ? 2 : 1) * Cfg::A_BYTES;
  };
  auto stageBlo = [&](uint32_t s) {
    return smem + s * Cfg::STAGE_BYTES + 2 * Cfg::A_BYTES + Cfg::B_BYTES;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&sb->full[s]), 1);
      mbar_init(smem_addr(&sb->conv[s]), convert ? 2 : 1);  // one arrival per converter warp
      mbar_init(smem_addr(&sb->empty[s]), 1);
    }
    // pair: the leader's tempty / ring_empty also count the follower's
    // epilogue warps (4) and its producer and forwarder threads (2)
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_addr(&sb->tfull[a]), 1);
      mbar_init(smem_addr(&sb->tempty[a]), PAIR ? 8 : 4);
    }
    for (int r = 0; r < R; ++r) {
      mbar_init(smem_addr(&sb->ring_full[r]), 1);
      mbar_init(smem_addr(&sb->ring_empty[r]), Cfg::NUM_CONS + (convert ? 2 : 0) + (PAIR ? 6 : 0));
    }
    mbar_init(smem_addr(&sb->final_mma), 1);
    sb->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (lo_by_tma) {
      tma_prefetch_desc(&tmAlo);
      tma_prefetch_desc(&tmBlo);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_addr(&sb->tmem_base), Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_addr(&sb->tmem_base), Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // the peer's barriers are initialised before any remote arrival
  else
    __syncthreads();
  tc_fence_after();
  // leader's barriers as seen from this CTA (pair only)
  auto leader_bar = [&](const uint64_t* b) { return mapa_shared(smem_addr(b), 0u); };
  const uint32_t tmem = sb->tmem_base;
  const long long t_ready = clock64();

  WaitCtl wc{&sb->abort_flag, p.err_word, p.timeout_ns};
  // k-blocks per accumulator segment (3xTF32: the tensor core's fp32
  // accumulation rounds toward zero, so each TMEM accumulator covers a short
  // K range and the epilogue folds segments in round-to-nearest registers)
  const int seg = Cfg::PROMOTE ? (p.seg_kb > 0 ? p.seg_kb : Cfg::SEG) : Cfg::SEG;
  unsigned long long st_a = 0, st_b = 0, st_c = 0, st_d = 0, st_e = 0, st_f = 0;  // per role
  const bool stats = p.pipe_stats != nullptr;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      uint32_t it = 0;
      uint32_t prod_s = 0, prod_ph = 0;  // stage and phase of k-block `it`
      int taken = 0;
      for (uint32_t slot = 0;; ++slot) {
        int tile;
        const uint32_t r = slot % R;
        if (leader) {
          // yield flag f: 0 = run; f > 0 = only CTAs below f keep taking tiles
          // (the op still completes on them); f < 0 = every CTA stops.
          const int f = p.yield_flag != nullptr ? *p.yield_flag : 0;
          if (p.max_tiles > 0 && taken >= p.max_tiles) {
            tile = -2;
          } else if (f < 0 || (f > 0 && static_cast<int>(blockIdx.x) >= f)) {
            tile = -2;
          } else {
            tile = static_cast<int>(atomicAdd(&p.work->next_tile, 1u));
            if (tile >= p.num_tiles) tile = -1;
          }
          const uint32_t eb = smem_addr(&sb->ring_empty[r]);
          const uint32_t ep = ((slot / R) & 1) ^ 1;
          if (!(PAIR ? mbar_wait_cluster(eb, ep, wc) : timed_wait(eb, ep, wc, stats ? &st_b : nullptr)))
            break;
          sb->ring[r] = tile;
          mbar_arrive(smem_addr(&sb->ring_full[r]));
          if constexpr (PAIR) {
            // the same tile id into the follower's ring
            st_shared_cluster_u32(mapa_shared(smem_addr(&sb->ring[r]), 1u),
                                  static_cast<uint32_t>(tile));
            mbar_arrive_cluster(mapa_shared(smem_addr(&sb->ring_full[r]), 1u));
          }
        } else {
          if (!mbar_wait_cluster(smem_addr(&sb->ring_full[r]), (slot / R) & 1, wc)) break;
          tile = sb->ring[r];
          mbar_arrive_cluster(leader_bar(&sb->ring_empty[r]));
        }
        if (tile < 0) break;
        ++taken;
        int b, ks, mb, nb, kb0, nkb;
        decode_tile(tile, p, b, ks, mb, nb);
        if constexpr (PAIR) mb = 2 * mb + static_cast<int>(rank);  // this CTA's 128 rows
        tile_k_range(tile, p, kb0, nkb);
        const int ba = p.a_bcast ? 0 : b;
        const int bb = p.b_bcast ? 0 : b;
        // this CTA's rows of B: all BN, or half of them in a pair
        const int n0 = nb * Cfg::BN + static_cast<int>(rank) * Cfg::B_ROWS;
        // Per-tile coordinate state (the single producer thread's issue loop
        // is on the critical path: no divisions per k-block).
        //  conv (forward): the tile's filter-window origin (w0, h0, image) and
        //    a (tap row rr, tap column ss, channel block cb) cursor over K;
        //  backward filter: the B operand's tap / channel block (fixed per
        //    tile) and an (image, pixel f0, output row oh, column ow) cursor.
        int cv_w0 = 0, cv_h0 = 0, cv_img = b, rr = 0, ss = 0, cb = 0;
        int wg_img = 0, wg_f0 = 0, wg_oh = 0, wg_ow = 0, wg_c0 = 0, wg_offw = 0, wg_offh = 0;
        if constexpr (CONV) {
          if (p.cv_wgrad) {
            wg_img = kb0 / p.cv_pb;
            wg_f0 = (kb0 - wg_img * p.cv_pb) * 32;
            wg_oh = wg_f0 / p.cv_q;
            wg_ow = wg_f0 - wg_oh * p.cv_q;
            const int tap = nb / p.cv_nb_per_tap;
            const int tr = tap / p.cv_s;
            wg_c0 = (nb - tap * p.cv_nb_per_tap) * Cfg::BN;
            wg_offw = (tap - tr * p.cv_s) * p.cv_dil_w;
            wg_offh = tr * p.cv_dil_h;
          } else {
            if (p.cv_im2col) {
              const int f0 = mb * Cfg::BM;
              cv_img = f0 / p.cv_pq;
              const int rem = f0 - cv_img * p.cv_pq;
              const int oh = rem / p.cv_q;
              const int ow = rem - oh * p.cv_q;
              cv_w0 = ow * p.cv_str_w - p.cv_pad_w;
              cv_h0 = oh * p.cv_str_h - p.cv_pad_h;
            } else {
              const int th = mb / p.cv_tiles_w;
              const int tw = mb - th * p.cv_tiles_w;
              cv_w0 = tw * p.cv_wbox * p.cv_str_w - p.cv_pad_w;
              cv_h0 = th * p.cv_hbox * p.cv_str_h - p.cv_pad_h;
            }
            const int tap = kb0 / p.cv_cb;
            cb = kb0 - tap * p.cv_cb;
            rr = tap / p.cv_s;
            ss = tap - rr * p.cv_s;
          }
        }
        bool ok = true;
        for (int kb = kb0; kb < kb0 + nkb; ++kb, ++it) {
          const uint32_t s = prod_s;
          const uint32_t ph = prod_ph;
          if (++prod_s == static_cast<uint32_t>(S)) {
            prod_s = 0;
            prod_ph ^= 1u;
          }
          if (!timed_wait(smem_addr(&sb->empty[s]), ph ^ 1u, wc, stats ? &st_a : nullptr)) {
            ok = false;
            break;
          }
          const long long t_iss = stats ? clock64() : 0;
          const uint32_t fb = smem_addr(&sb->full[s]);
          // CTA pair: both CTAs' loads complete on the leader's stage
          // barrier, which expects the bytes of both (the follower arrives on
          // nothing and the leader's MMA waits on one barrier).  3xTF32 with
          // pre-split operands: the low parts arrive by TMA beside the high
          // parts.
          const uint32_t fb_peer = DIRECT ? mapa_shared(fb, 0u) : fb;
          const bool peer_load = DIRECT && !leader;
          if (!peer_load)
            mbar_arrive_expect_tx(fb, Cfg::LOAD_BYTES * (lo_by_tma ? 2 : 1) * (PAIR ? 2 : 1));
          auto load_a = [&](uint32_t sa, const CUtensorMap* map) {
            if constexpr (CONV) {
              if (p.cv_wgrad) {  // dy rows k = mb*128.., 32 pixels
                tma_load_3d(sa, map, fb, wg_f0, mb * Cfg::BM, wg_img);
              } else if (p.cv_im2col) {
                if (peer_load)
                  tma_load_4d_im2col_pair(sa, map, fb_peer, cb * 32, cv_w0, cv_h0, cv_img,
                                          static_cast<uint16_t>(ss * p.cv_dil_w),
                                          static_cast<uint16_t>(rr * p.cv_dil_h));
                else
                  tma_load_4d_im2col(sa, map, fb, cb * 32, cv_w0, cv_h0, cv_img,
                                     static_cast<uint16_t>(ss * p.cv_dil_w),
                                     static_cast<uint16_t>(rr * p.cv_dil_h));
              } else if (peer_load) {
                tma_load_4d_pair(sa, map, fb_peer, cb * 32, cv_w0 + ss * p.cv_dil_w,
                                 cv_h0 + rr * p.cv_dil_h, cv_img);
              } else {
                tma_load_4d(sa, map, fb, cb * 32, cv_w0 + ss * p.cv_dil_w,
                            cv_h0 + rr * p.cv_dil_h, cv_img);
              }
            } else if (!Cfg::A_MN) {
              if (peer_load)
                tma_load_3d_pair(sa, map, fb_peer, kb * Cfg::BK, mb * Cfg::BM, ba);
              else
                tma_load_3d(sa, map, fb, kb * Cfg::BK, mb * Cfg::BM, ba);
            } else if (p.a_single) {
              tma_load_4d(sa, map, fb, 0, kb * Cfg::BK, mb * (Cfg::BM / Cfg::CHUNK), ba);
            } else {
#pragma unroll
              for (int c = 0; c < Cfg::BM / Cfg::CHUNK; ++c)
                tma_load_3d(sa + c * Cfg::BK * 128, map, fb, mb * Cfg::BM + c * Cfg::CHUNK,
                            kb * Cfg::BK, ba);
            }
          };
          auto load_b = [&](uint32_t sbb, const CUtensorMap* map) {
            if constexpr (CONV && Cfg::B_MN) {
              // backward filter: BN/32 im2col loads of 32 pixels x 32 channels
              const int wx = wg_ow * p.cv_str_w - p.cv_pad_w;
              const int hy = wg_oh * p.cv_str_h - p.cv_pad_h;
#pragma unroll
              for (int c = 0; c < Cfg::B_ROWS / 32; ++c)
                tma_load_4d_im2col(sbb + c * Cfg::BK * 128, map, fb, wg_c0 + c * 32, wx, hy,
                                   wg_img, static_cast<uint16_t>(wg_offw),
                                   static_cast<uint16_t>(wg_offh));
            } else if (!Cfg::B_MN) {
              if (peer_load)
                tma_load_3d_pair(sbb, map, fb_peer, kb * Cfg::BK, n0, bb);
              else
                tma_load_3d(sbb, map, fb, kb * Cfg::BK, n0, bb);
            } else if (p.b_single) {
              tma_load_4d(sbb, map, fb, 0, kb * Cfg::BK, n0 / Cfg::CHUNK, bb);
            } else {
#pragma unroll
              for (int c = 0; c < Cfg::B_ROWS / Cfg::CHUNK; ++c)
                tma_load_3d(sbb + c * Cfg::BK * 128, map, fb, n0 + c * Cfg::CHUNK,
                            kb * Cfg::BK, bb);
            }
          };
          load_a(smem_addr(stageA(s)), &tmA);
          load_b(smem_addr(stageB(s)), &tmB);
          if (lo_by_tma) {
            load_a(smem_addr(stageAlo(s)), &tmAlo);
            load_b(smem_addr(stageBlo(s)), &tmBlo);
          }
          // advance the coordinate cursors to the next k-block
          if constexpr (CONV) {
            if (p.cv_wgrad) {
              wg_f0 += 32;
              if (wg_f0 >= p.cv_pb * 32) {
                wg_f0 = 0;
                wg_oh = 0;
                wg_ow = 0;
                ++wg_img;
              } else {
                wg_ow += 32;
                while (wg_ow >= p.cv_q) {
                  wg_ow -= p.cv_q;
                  ++wg_oh;
                }
              }
            } else if (++cb == p.cv_cb) {
              cb = 0;
              if (++ss == p.cv_s) {
                ss = 0;
                ++rr;
              }
            }
          }
          if (stats) st_c += static_cast<unsigned long long>(clock64() - t_iss);
        }
        if (!ok) break;
      }
      // Drain: every issued TMA load must land before the CTA can retire.
      WaitCtl drain{&sb->abort_flag, nullptr, p.timeout_ns};
      int dummy_abort = 0;
      drain.abort_flag = &dummy_abort;
      if (DIRECT && !leader) {
        // the follower's loads complete on the leader's barriers: they have
        // landed once the leader's MMAs consumed them, i.e. once the commit
        // that frees each of the last S stages arrived here
        const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(smem_addr(&sb->empty[j % S]), (j / S) & 1, drain);
      } else {
        const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(smem_addr(&sb->full[j % S]), (j / S) & 1, drain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer ---
    if (lane == 0 && PAIR && !leader) {
      // follower: the leader issues the pair's MMAs and the follower's loads
      // signal the leader themselves; this thread only consumes the tile ids
      for (uint32_t slot = 0;; ++slot) {
        const uint32_t r = slot % R;
        if (!mbar_wait_cluster(smem_addr(&sb->ring_full[r]), (slot / R) & 1, wc)) break;
        const int tile = sb->ring[r];
        mbar_arrive_cluster(leader_bar(&sb->ring_empty[r]));
        if (tile < 0) break;
      }
    } else if (lane == 0) {
      // `sc` counts accumulator segments across tiles; segment sc uses TMEM
      // buffer sc & 1 (one segment per tile unless PROMOTE splits K).
      uint32_t it = 0, sc = 0;
      uint32_t mma_s = 0, mma_ph = 0;  // stage and phase of k-block `it`
      const uint64_t a_desc0 =
          sdesc_sw128(smem_addr(stageA(0)), Cfg::A_LBO, Cfg::A_SBO, Cfg::A_LAYOUT);
      const uint64_t b_desc0 =
          sdesc_sw128(smem_addr(stageB(0)), Cfg::B_LBO, Cfg::B_SBO, Cfg::B_LAYOUT);
      const long long t_loop = stats ? clock64() : 0;
      bool ok = true;
      for (uint32_t slot = 0; ok; ++slot) {
        const uint32_t r = slot % R;
        if (!timed_wait(smem_addr(&sb->ring_full[r]), (slot / R) & 1, wc,
                        stats ? &st_c : nullptr))
          break;
        const int tile = sb->ring[r];
        mbar_arrive(smem_addr(&sb->ring_empty[r]));
        if (tile < 0) break;
        int kb0, nkb;
        tile_k_range(tile, p, kb0, nkb);
        for (int kb = 0; kb < nkb && ok; ++sc) {
          const uint32_t a = sc & 1;
          const bool tfree =
              PAIR ? mbar_wait_cluster(smem_addr(&sb->tempty[a]), ((sc >> 1) & 1) ^ 1, wc)
                   : timed_wait(smem_addr(&sb->tempty[a]), ((sc >> 1) & 1) ^ 1, wc,
                                stats ? &st_b : nullptr);
          if (!tfree) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem + a * Cfg::ACC_COLS;
          const int kend = (nkb - kb > seg) ? kb + seg : nkb;
          const int kfirst = kb;
          const long long t_k = stats ? clock64() : 0;
          for (; kb < kend; ++kb, ++it) {
            // stage and phase of k-block `it`, kept as running counters (the
            // single issuing thread's instruction count per k-block is on the
            // critical path)
            const uint32_t s = mma_s;
            const uint32_t ph = mma_ph;
            if (++mma_s == static_cast<uint32_t>(S)) {
              mma_s = 0;
              mma_ph ^= 1u;
            }
            const uint32_t wb = convert ? smem_addr(&sb->conv[s]) : smem_addr(&sb->full[s]);
            if (!timed_wait(wb, ph, wc, stats ? &st_a : nullptr)) {
              ok = false;
              break;
            }
            const long long t_iss = stats ? clock64() : 0;
            tc_fence_after();
            // descriptors of this stage: the stage-0 descriptors plus the
            // stage offset in the 16-byte address field (no carry: shared
            // memory addresses stay below 2^18)
            const uint32_t soff = s * static_cast<uint32_t>(Cfg::STAGE_BYTES >> 4);
#pragma unroll
            for (int kk = 0; kk < Cfg::BK / Cfg::UMMA_K; ++kk) {
              const uint32_t aoff = Cfg::A_MN ? kk * Cfg::UMMA_K * 128 : kk * 32;
              const uint32_t boff = Cfg::B_MN ? kk * Cfg::UMMA_K * 128 : kk * 32;
              const uint64_t ad = a_desc0 + (soff + (aoff >> 4));
              const uint64_t bd = b_desc0 + (soff + (boff >> 4));
              const uint32_t acc = (kb > kfirst || kk > 0) ? 1u : 0u;
              if constexpr (PAIR && !Cfg::SPLIT) {
                // 16-bit operands: one 256 x BN MMA over the pair's A and B rows
                umma_f16_pair(d_tmem, ad, bd, Cfg::IDESC, acc);
              } else if constexpr (PAIR) {
                // 256 x BN over the pair, A rows and B rows from both CTAs (A_lo
                // right after A, B_lo right after B in the stage): hi*hi into
                // [0, BN), hi*lo and lo*hi into [BN, 2BN)
                const uint64_t adl = ad + (Cfg::A_BYTES >> 4);
                const uint64_t bdl = bd + (Cfg::B_BYTES >> 4);
                umma_tf32_pair(d_tmem, ad, bd, Cfg::IDESC, acc);
                umma_tf32_pair(d_tmem + Cfg::BN, ad, bdl, Cfg::IDESC, acc);
                umma_tf32_pair(d_tmem + Cfg::BN, adl, bd, Cfg::IDESC, 1u);
              } else if constexpr (Cfg::AR == Arith::F32x3) {
                // hi*hi and hi*lo in one N = 2*BN MMA over [B_hi; B_lo]
                // (columns [0, BN) and [BN, 2BN)), then lo*hi into [BN, 2BN):
                // A_hi is read from shared memory once per k-step, not twice,
                // and the large half takes one truncating add per k-step
                const uint64_t adl = ad + (Cfg::A_BYTES >> 4);  // A_lo follows A
                umma_tf32(d_tmem, ad, bd, Cfg::IDESC2, acc);
                umma_tf32(d_tmem + Cfg::BN, adl, bd, Cfg::IDESC, 1u);
              } else if constexpr (Cfg::AR == Arith::TF32) {
                umma_tf32(d_tmem, ad, bd, Cfg::IDESC, acc);
              } else {
                umma_f16(d_tmem, ad, bd, Cfg::IDESC, acc);
              }
            }
            if constexpr (PAIR)
              tc_commit_pair(smem_addr(&sb->empty[s]));  // frees the stage in both CTAs
            else
              tc_commit(smem_addr(&sb->empty[s]));
            if (stats) st_d += static_cast<unsigned long long>(clock64() - t_iss);
          }
          if (stats) st_f += static_cast<unsigned long long>(clock64() - t_k);
          if (!ok) break;
          if constexpr (PAIR)
            tc_commit_pair(smem_addr(&sb->tfull[a]));
          else
            tc_commit(smem_addr(&sb->tfull[a]));
        }
      }
      if (stats) st_e = static_cast<unsigned long long>(clock64() - t_loop);
      // Wait (bounded) for every MMA this thread issued before TMEM is freed.
      if constexpr (PAIR)
        tc_commit_pair(smem_addr(&sb->final_mma));
      else
        tc_commit(smem_addr(&sb->final_mma));
      int dummy_abort = 0;
      WaitCtl drain{&dummy_abort, nullptr, p.timeout_ns};
      mbar_wait(smem_addr(&sb->final_mma), 0, drain);
    }
  } else if (warp < 4) {
    // -------------------------- 3xTF32 low parts in shared memory (warps 2-3) --
    // Only when they were not split off before the launch.  hi is the fp32
    // value itself (a kind::tf32 MMA reads trunc_tf32(x)); lo = x -
    // trunc_tf32(x) is exact in fp32 and goes to the stage's lo buffers.
    if (convert) {
      const int ct = threadIdx.x - 64;  // 0..63
      uint32_t it = 0;
      for (uint32_t slot = 0;; ++slot) {
        const uint32_t r = slot % R;
        bool ok = mbar_wait(smem_addr(&sb->ring_full[r]), (slot / R) & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const int tile = sb->ring[r];
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&sb->ring_empty[r]));
        if (tile < 0) break;
        int kb0, nkb;
        tile_k_range(tile, p, kb0, nkb);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const uint32_t s = it % S;
          ok = mbar_wait(smem_addr(&sb->full[s]), (it / S) & 1, wc);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          // A -> A_lo and B -> B_lo (stage layout [A | A_lo | B | B_lo])
          const float4* ha = reinterpret_cast<const float4*>(stageA(s));
          float4* la = reinterpret_cast<float4*>(stageAlo(s));
          const float4* hb = reinterpret_cast<const float4*>(stageB(s));
          float4* lb = reinterpret_cast<float4*>(stageBlo(s));
          constexpr int NA = Cfg::A_BYTES / 16;
          constexpr int NB = Cfg::B_BYTES / 16;
#pragma unroll 8
          for (int v = ct; v < NA; v += 64) {
            const float4 x = ha[v];
            la[v] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
          }
#pragma unroll 8
          for (int v = ct; v < NB; v += 64) {
            const float4 x = hb[v];
            lb[v] = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
          }
          // every thread orders its own writes before the async proxy reads;
          // then one arrival per warp
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&sb->conv[s]));
        }
        if (!ok) break;
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------- epilogue -----
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const float alpha = p.alpha_dev ? *p.alpha_dev : p.alpha;
    const float beta = p.beta_dev ? *p.beta_dev : p.beta;
    const uint32_t lane_off = (q * 32u) << 16;
    const bool split = p.splits > 1;
    // alpha * acc only (no beta, bias or activation)
    const bool plain_epi = beta == 0.f && p.bias == nullptr && !p.relu && !p.gelu;
    // a 64-column D box (wide16) serves the plain 16-bit epilogue only
    const bool use_tma_store = p.tma_store != 0 && !split && (p.wide16 == 0 || plain_epi);
    uint32_t epi_chunk = 0;
    uint32_t sc = 0;
    for (uint32_t slot = 0;; ++slot) {
      const uint32_t r = slot % R;
      bool ok = leader ? mbar_wait(smem_addr(&sb->ring_full[r]), (slot / R) & 1, wc)
                       : mbar_wait_cluster(smem_addr(&sb->ring_full[r]), (slot / R) & 1, wc);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const int tile = sb->ring[r];
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(smem_addr(&sb->ring_empty[r]));
        else
          mbar_arrive_cluster(leader_bar(&sb->ring_empty[r]));
      }
      if (tile < 0) break;
      int b, ks, mb, nb, kb0, nkb;
      decode_tile(tile, p, b, ks, mb, nb);
      if constexpr (PAIR) mb = 2 * mb + static_cast<int>(rank);  // this CTA's 128 rows
      tile_k_range(tile, p, kb0, nkb);
      const int nseg = Cfg::PROMOTE ? (nkb + seg - 1) / seg : 1;
      int row = mb * Cfg::BM + q * 32 + static_cast<int>(lane);
      bool row_ok = row < p.m;
      size_t d_base = static_cast<size_t>(b) * p.strideD + row;
      size_t c_base = static_cast<size_t>(b) * p.strideC + row;
      // im2col convolution: this warp's TMA store covers one image
      bool warp_tma = use_tma_store;
      int st_img = 0, st_pix = 0;
      if constexpr (CONV) {
        if (p.cv_wgrad) {
          // plain GEMM rows (output channels) into ws / D
        } else if (p.cv_im2col) {
          const int img = row / p.cv_pq;
          const int pix = row - img * p.cv_pq;
          d_base = static_cast<size_t>(img) * p.strideD + pix;
          c_base = static_cast<size_t>(img) * p.strideC + pix;
          const int f0 = mb * Cfg::BM + q * 32;
          st_img = f0 / p.cv_pq;
          st_pix = f0 - st_img * p.cv_pq;
          warp_tma = use_tma_store && f0 < p.m && (f0 + 31) / p.cv_pq == st_img;
        } else {
          // tile row i = output pixel (th*hbox + i / wbox, tw*wbox + i % wbox)
          const int i = q * 32 + static_cast<int>(lane);
          const int th = mb / p.cv_tiles_w;
          const int tw = mb - th * p.cv_tiles_w;
          const int op = th * p.cv_hbox + i / p.cv_wbox;
          const int oq = tw * p.cv_wbox + (i - (i / p.cv_wbox) * p.cv_wbox);
          row_ok = op < p.cv_p && oq < p.cv_q;
          row = op * p.cv_q + oq;
          d_base = static_cast<size_t>(b) * p.strideD + row;
          c_base = static_cast<size_t>(b) * p.strideC + row;
        }
      }
      const float bias_v = (p.bias != nullptr && row_ok && !split) ? load_scalar(p.bias, p.bias_type, row) : 0.f;
      // split-K slice: raw fp32 partial, column-major with ld m
      float* ws_tile = split ? p.ws + (static_cast<size_t>(b) * p.splits + ks) *
                                          static_cast<size_t>(p.m) * p.n + row
                             : nullptr;
      // alpha/beta/bias/activation for 32 consecutive columns of this row
      auto emit = [&](int c0, const float* acc) {
        const int col0 = nb * Cfg::BN + c0;
        if (!row_ok) return;
        if (split) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.n) ws_tile[static_cast<size_t>(col0 + j) * p.m] = acc[j];
          return;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = col0 + j;
          if (col < p.n) {
            float o = alpha * acc[j];
            if (beta != 0.f)
              o += beta * load_scalar(p.C, p.c_type, c_base + static_cast<size_t>(col) * p.ldc);
            o += bias_v;
            if (p.relu) o = fmaxf(o, 0.f);
            if (p.gelu) o = gelu_tanh(o);
            store_scalar(p.D, p.d_type, d_base + static_cast<size_t>(col) * p.ldd, o);
          }
        }
      };
      // Same values through shared memory: the warp writes its 32 rows x 32
      // columns (column-contiguous, as D is) into one of its two staging
      // buffers and lane 0 issues a TMA store, which clips rows / columns
      // outside D.  A buffer is rewritten only after the store issued from it
      // two chunks earlier has read it.
      auto emit_tma = [&](int c0, const float* acc) {
        const int col0 = nb * Cfg::BN + c0;
        uint8_t* buf = smem + Cfg::EPI_OFF + (q * 2 + (epi_chunk & 1u)) * 4096;
        ++epi_chunk;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        // element (column j, row lane) at index j*32 + lane of the buffer
        float* fbuf = reinterpret_cast<float*>(buf);
        if (plain_epi && p.d_type == DT_F32) {
#pragma unroll
          for (int j = 0; j < 32; ++j) fbuf[j * 32 + lane] = alpha * acc[j];
        } else if (plain_epi && p.d_type == DT_BF16) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            reinterpret_cast<__nv_bfloat16*>(buf)[j * 32 + lane] = __float2bfloat16_rn(alpha * acc[j]);
        } else {
          // general epilogue in a second, rolled pass over the staged values
          // (keeps the code small: the epilogue warps share the instruction
          // cache with the producer and MMA loops)
#pragma unroll
          for (int j = 0; j < 32; ++j) fbuf[j * 32 + lane] = alpha * acc[j];
          __syncwarp();
#pragma unroll 1
          for (int j = 0; j < 32; ++j) {
            const int col = col0 + j;
            float o = fbuf[j * 32 + lane];
            if (beta != 0.f && row_ok && col < p.n)
              o += beta * load_scalar(p.C, p.c_type, c_base + static_cast<size_t>(col) * p.ldc);
            o += bias_v;
            if (p.relu) o = fmaxf(o, 0.f);
            if (p.gelu) o = gelu_tanh(o);
            // 16-bit outputs shrink in place: element i is written at byte 2i,
            // below every element a later iteration still reads
            if (p.d_type == DT_F32)
              fbuf[j * 32 + lane] = o;
            else if (p.d_type == DT_BF16)
              reinterpret_cast<__nv_bfloat16*>(buf)[j * 32 + lane] = __float2bfloat16_rn(o);
            else
              reinterpret_cast<__half*>(buf)[j * 32 + lane] = __float2half_rn(o);
            __syncwarp();
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CONV) {
            if (p.cv_im2col) {
              tma_store_3d(&tmD, smem_addr(buf), st_pix, col0, st_img);
            } else {
              // warp q holds tile rows 32q .. 32q+31 = a {min(wbox,32), 32/min(wbox,32)} box
              const int th = mb / p.cv_tiles_w;
              const int tw = mb - th * p.cv_tiles_w;
              const int i0 = q * 32;
              tma_store_4d(&tmD, smem_addr(buf), tw * p.cv_wbox + i0 % p.cv_wbox,
                           th * p.cv_hbox + i0 / p.cv_wbox, col0, b);
            }
          } else {
            tma_store_3d(&tmD, smem_addr(buf), mb * Cfg::BM + q * 32, col0, b);
          }
          bulk_commit_group();
        }
      };
      if constexpr (Cfg::PROMOTE) {
        // fold every segment's TMEM partial into round-to-nearest registers
        float acc[Cfg::BN / 32][32];
#pragma unroll
        for (int c = 0; c < Cfg::BN / 32; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[c][j] = 0.f;
        for (int sg = 0; sg < nseg; ++sg, ++sc) {
          const uint32_t a = sc & 1;
          ok = timed_wait(smem_addr(&sb->tfull[a]), (sc >> 1) & 1, wc,
                          stats && warp == 4 ? &st_a : nullptr);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          const long long t_fold = stats ? clock64() : 0;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < Cfg::BN / 32; ++c) {
            // both accumulator halves of the chunk in flight, one wait
            uint32_t v[32], w[32];
            tmem_ld_32x32b_x32(tmem + a * Cfg::ACC_COLS + c * 32 + lane_off, v);
            if constexpr (Cfg::ACC_COLS == 2 * Cfg::BN)
              tmem_ld_32x32b_x32(tmem + a * Cfg::ACC_COLS + Cfg::BN + c * 32 + lane_off, w);
            tmem_ld_wait();
            tmem_regs_ready(v);
            if constexpr (Cfg::ACC_COLS == 2 * Cfg::BN) {
              // small half first: one rounding of the segment's sum
              tmem_regs_ready(w);
#pragma unroll
              for (int j = 0; j < 32; ++j)
                acc[c][j] += __uint_as_float(v[j]) + __uint_as_float(w[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) acc[c][j] += __uint_as_float(v[j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              mbar_arrive(smem_addr(&sb->tempty[a]));
            else
              mbar_arrive_cluster(leader_bar(&sb->tempty[a]));
          }
          if (stats) st_b += static_cast<unsigned long long>(clock64() - t_fold);
        }
        if (!ok) break;
        const long long t_emit = stats ? clock64() : 0;
        if (warp_tma) {
#pragma unroll
          for (int c = 0; c < Cfg::BN / 32; ++c) emit_tma(c * 32, acc[c]);
        } else {
#pragma unroll
          for (int c = 0; c < Cfg::BN / 32; ++c) emit(c * 32, acc[c]);
        }
        if (stats) st_c += static_cast<unsigned long long>(clock64() - t_emit);
      } else {
        const uint32_t a = sc & 1;
        ok = timed_wait(smem_addr(&sb->tfull[a]), (sc >> 1) & 1, wc,
                        stats && warp == 4 ? &st_a : nullptr);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const long long t_emit = stats ? clock64() : 0;
        // Two 32-column register buffers: the TMEM load of the next chunk is
        // in flight while the current one is converted and stored.
        const uint32_t tbase = tmem + a * Cfg::ACC_COLS + lane_off;
        uint32_t va[32], vb[32];
        auto out = [&](int c0, uint32_t (&v)[32]) {
          tmem_regs_ready(v);
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
          if (warp_tma)
            emit_tma(c0, f);
          else
            emit(c0, f);
        };
        if (p.wide16 && warp_tma && plain_epi && Cfg::BN % 64 == 0) {
          // 16-bit D, alpha only: 64 columns (4 KB) per staging buffer and per
          // TMA store, half the per-store fences, waits and issues
#pragma unroll 1
          for (int c0 = 0; c0 < Cfg::BN; c0 += 64) {
            tmem_ld_32x32b_x32(tbase + c0, va);
            tmem_ld_32x32b_x32(tbase + c0 + 32, vb);
            tmem_ld_wait();
            tmem_regs_ready(va);
            tmem_regs_ready(vb);
            uint8_t* buf = smem + Cfg::EPI_OFF + (q * 2 + (epi_chunk & 1u)) * 4096;
            ++epi_chunk;
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            if (p.d_type == DT_BF16) {
              __nv_bfloat16* hb = reinterpret_cast<__nv_bfloat16*>(buf);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                hb[j * 32 + lane] = __float2bfloat16_rn(alpha * __uint_as_float(va[j]));
                hb[(32 + j) * 32 + lane] = __float2bfloat16_rn(alpha * __uint_as_float(vb[j]));
              }
            } else {
              __half* hh = reinterpret_cast<__half*>(buf);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                hh[j * 32 + lane] = __float2half_rn(alpha * __uint_as_float(va[j]));
                hh[(32 + j) * 32 + lane] = __float2half_rn(alpha * __uint_as_float(vb[j]));
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmD, smem_addr(buf), mb * Cfg::BM + q * 32, nb * Cfg::BN + c0, b);
              bulk_commit_group();
            }
          }
        } else {
          tmem_ld_32x32b_x32(tbase, va);
          tmem_ld_wait();
#pragma unroll 1
          for (int c0 = 0; c0 < Cfg::BN; c0 += 64) {
            const bool has_b = c0 + 32 < Cfg::BN;
            if (has_b) tmem_ld_32x32b_x32(tbase + c0 + 32, vb);
            out(c0, va);
            tmem_ld_wait();
            if (c0 + 64 < Cfg::BN) tmem_ld_32x32b_x32(tbase + c0 + 64, va);
            if (has_b) out(c0 + 32, vb);
            tmem_ld_wait();
          }
        }
        if (stats) st_c += static_cast<unsigned long long>(clock64() - t_emit);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(smem_addr(&sb->tempty[a]));
          else
            mbar_arrive_cluster(leader_bar(&sb->tempty[a]));
        }
        ++sc;
      }
    }
  }

  // --------------------------------------------------------- teardown ----
  // the epilogue's TMA stores complete before the CTA counts as retired
  if (warp >= 4 && warp < 8 && lane == 0 && p.tma_store != 0) bulk_wait_group_all();
  if (stats && lane == 0) {
    unsigned long long* ps = p.pipe_stats + static_cast<size_t>(blockIdx.x) * kPipeStats;
    if (warp == 0) {
      ps[PS_PROD_EMPTY] = st_a;
      ps[PS_PROD_RING] = st_b;
      ps[PS_PROD_ISSUE] = st_c;
    } else if (warp == 1) {
      ps[PS_MMA_DATA] = st_a;
      ps[PS_MMA_TMEM] = st_b;
      ps[PS_MMA_RING] = st_c;
      ps[PS_MMA_ISSUE] = st_d;
      ps[PS_MMA_LOOP] = st_e;
      ps[PS_MMA_KLOOP] = st_f;
    } else if (warp == 4) {
      ps[PS_EPI_TFULL] = st_a;
      ps[PS_EPI_FOLD] = st_b;
      ps[PS_EPI_EMIT] = st_c;
      ps[PS_EPI_STWAIT] = st_e;
      ps[PS_TOTAL] = static_cast<unsigned long long>(clock64() - t_start);
      ps[PS_PROLOGUE] = static_cast<unsigned long long>(t_ready - t_start);
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // no remote arrival or MMA into this CTA is still pending
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    const bool aborted = sb->abort_flag != 0;
    __threadfence();
    const unsigned prev = atomicAdd(&p.work->exited, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      const unsigned nt = atomicAdd(&p.work->next_tile, 0u);
      const bool complete = nt >= static_cast<unsigned>(p.num_tiles);
      if (complete || aborted) atomicExch(&p.work->next_tile, 0u);
      atomicExch(&p.work->exited, 0u);
      p.work->status = complete ? 1 : 0;
      if (p.done_flag != nullptr) {
        *p.done_flag = complete ? 1 : 0;
        __threadfence_system();
      }
    }
    if (aborted) atomicCAS(&p.work->err, 0, 3);
  }
}

}  // namespace kx
