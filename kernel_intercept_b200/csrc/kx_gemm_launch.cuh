// kx_gemm_launch.cuh — host launcher for one tcgen05 GEMM configuration.
// Each kx_gemm_tc_<arith>.cu includes this and instantiates the launchers
// for its arithmetic, so the 48 kernel variants compile in parallel.
#pragma once
#include <cstdio>

#include "kx_gemm.cuh"
#include "kx_runtime.cuh"

namespace kx {

struct TcProblem {
  int m, n, k, batch;
  const void* A;
  long long lda, strideA;
  const void* B;
  long long ldb, strideB;
  // 3xTF32 only: x - trunc_tf32(x) of A and B, same layout as A and B
  const void* Alo;
  const void* Blo;
};

template <Arith AR>
constexpr CUtensorMapDataType map_dtype() {
  return AR == Arith::BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
         : AR == Arith::F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

template <Arith AR>
constexpr const char* arith_name() {
  return AR == Arith::F32x3 ? "f32x3" : AR == Arith::TF32 ? "tf32" : AR == Arith::BF16 ? "bf16" : "f16";
}

// KX_GEMM_PAIR: "1" = every 16-bit GEMM with K-major operands runs on 2-CTA
// clusters (256-row tiles, cta_group::2 MMAs, each SM loading half of the B
// tile); "0" = never; unset = where pairs measured faster on B200: K of at
// least 4096 over at least four waves of 128 x 256 tiles (8192^3: 1434-1438
// TFLOP/s against 1287-1340 with one CTA per tile; the K = 2048 GEMMs of the
// LLaMA step lose 3-9% on pairs).
inline int gemm_pair_mode() {
  const char* s = std::getenv("KX_GEMM_PAIR");
  return s == nullptr ? -1 : (s[0] == '1' ? 1 : (s[0] == '0' ? 0 : -1));
}

template <int BN, Arith AR, bool AMN, bool BMN, bool PAIR = false>
int launch_gemm_tc(const Exec& e, const TcProblem& pr, GemmParams p) {
  using Cfg = GemmCfg<BN, AR, AMN, BMN, PAIR>;
  constexpr CUtensorMapDataType dt = map_dtype<AR>();
  CUtensorMap ma, mb, malo, mblo;
  // M/N-major tf32 operands need the 32-byte-atom variant of the 128-byte swizzle
  constexpr CUtensorMapSwizzle swzA =
      Cfg::A_MN32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  constexpr CUtensorMapSwizzle swzB =
      Cfg::B_MN32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  auto map_a = [&](CUtensorMap* m, const void* base) {
    return AMN ? encode_map_3d(m, dt, Cfg::ESIZE, base, pr.m, pr.k, pr.batch, pr.lda, pr.strideA,
                               Cfg::CHUNK, Cfg::BK, swzA)
               : encode_map_3d(m, dt, Cfg::ESIZE, base, pr.k, pr.m, pr.batch, pr.lda, pr.strideA,
                               Cfg::BK, Cfg::BM);
  };
  auto map_b = [&](CUtensorMap* m, const void* base) {
    return BMN ? encode_map_3d(m, dt, Cfg::ESIZE, base, pr.n, pr.k, pr.batch, pr.ldb, pr.strideB,
                               Cfg::CHUNK, Cfg::BK, swzB)
               : encode_map_3d(m, dt, Cfg::ESIZE, base, pr.k, pr.n, pr.batch, pr.ldb, pr.strideB,
                               Cfg::BK, Cfg::B_ROWS);
  };
  // M/N-major tile in one TMA box: {CHUNK, K, rows / CHUNK, batch} with the
  // third dimension stepping CHUNK elements.  Only when the rows are a
  // multiple of CHUNK (the box's inner dimension is a whole chunk, so a
  // partial last chunk would read past the matrix).
  auto map_single = [&](CUtensorMap* m, const void* base, long long rows, long long ld,
                        long long stride, int box_chunks, CUtensorMapSwizzle swz) {
    const bool batched = pr.batch > 1 && stride != 0;
    const uint64_t dims[4] = {static_cast<uint64_t>(Cfg::CHUNK), static_cast<uint64_t>(pr.k),
                              static_cast<uint64_t>(rows / Cfg::CHUNK),
                              static_cast<uint64_t>(batched ? pr.batch : 1)};
    const uint64_t strides[3] = {static_cast<uint64_t>(ld) * Cfg::ESIZE,
                                 static_cast<uint64_t>(Cfg::CHUNK) * Cfg::ESIZE,
                                 static_cast<uint64_t>(batched ? stride : rows * ld) * Cfg::ESIZE};
    const uint32_t box[4] = {static_cast<uint32_t>(Cfg::CHUNK), static_cast<uint32_t>(Cfg::BK),
                             static_cast<uint32_t>(box_chunks), 1u};
    return encode_map(m, dt, 4, base, dims, strides, box, swz);
  };
  p.a_single = 0;
  p.b_single = 0;
  const bool lo_maps = Cfg::SPLIT && p.presplit;
  if (lo_maps && (pr.Alo == nullptr || pr.Blo == nullptr)) return KX_ERR_INVALID;
  if (AMN && pr.m % Cfg::CHUNK == 0 && !single_box_disabled() &&
      map_single(&ma, pr.A, pr.m, pr.lda, pr.strideA, Cfg::BM / Cfg::CHUNK, swzA) &&
      (!lo_maps ||
       map_single(&malo, pr.Alo, pr.m, pr.lda, pr.strideA, Cfg::BM / Cfg::CHUNK, swzA)))
    p.a_single = 1;
  if (BMN && pr.n % Cfg::CHUNK == 0 && !single_box_disabled() &&
      map_single(&mb, pr.B, pr.n, pr.ldb, pr.strideB, Cfg::B_ROWS / Cfg::CHUNK, swzB) &&
      (!lo_maps ||
       map_single(&mblo, pr.Blo, pr.n, pr.ldb, pr.strideB, Cfg::B_ROWS / Cfg::CHUNK, swzB)))
    p.b_single = 1;
  if ((!p.a_single && !map_a(&ma, pr.A)) || (!p.b_single && !map_b(&mb, pr.B)))
    return KX_ERR_UNSUPPORTED;
  if (lo_maps) {
    if ((!p.a_single && !map_a(&malo, pr.Alo)) || (!p.b_single && !map_b(&mblo, pr.Blo)))
      return KX_ERR_UNSUPPORTED;
  } else {
    malo = ma;
    mblo = mb;
  }

  p.num_mb = (pr.m + Cfg::BM - 1) / Cfg::BM;
  // a pair tile covers two consecutive 128-row blocks (the second may lie
  // past the end: its loads read zeros and its rows are not stored)
  if (PAIR) p.num_mb = (p.num_mb + 1) / 2;
  p.num_nb = (pr.n + BN - 1) / BN;
  p.num_kb = (pr.k + Cfg::BK - 1) / Cfg::BK;
  p.tiles_per_batch = p.num_mb * p.num_nb;
  const long long tiles = static_cast<long long>(p.tiles_per_batch) * pr.batch;
  if (tiles <= 0 || tiles > 0x7fffffffLL) return KX_ERR_UNSUPPORTED;
  p.num_tiles = static_cast<int>(tiles);
  p.a_bcast = (pr.batch > 1 && pr.strideA == 0) ? 1 : 0;
  p.b_bcast = (pr.batch > 1 && pr.strideB == 0) ? 1 : 0;

  auto kern = kx_gemm_tc_kernel<Cfg>;
  static bool attr_set[64] = {false};
  const DeviceInfo& di = device_info();
  if (!attr_set[di.device & 63]) {
    const cudaError_t ae = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (ae != cudaSuccess) return device_error(ae);
    attr_set[di.device & 63] = true;
  }
  // Split-K when the output tiles cannot fill the CTAs the launch may use and
  // K is long: slices of at least MIN_KB k-blocks (256 of K), at most 32.
  constexpr int MIN_KB = 256 / Cfg::BK;
  const int cap = persistent_grid(e, 1 << 30);
  p.splits = 1;
  p.kb_per_split = p.num_kb;
  if (!PAIR && tiles * 2 <= cap && p.num_kb >= 2 * MIN_KB && !split_k_disabled()) {
    long long want = cap / tiles;
    const long long by_k = p.num_kb / MIN_KB;
    if (want > by_k) want = by_k;
    if (want > 32) want = 32;
    if (want >= 2) {
      const int kbps = static_cast<int>((p.num_kb + want - 1) / want);
      const int splits = (p.num_kb + kbps - 1) / kbps;
      const size_t ws_bytes = sizeof(float) * static_cast<size_t>(splits) * pr.batch *
                              static_cast<size_t>(pr.m) * pr.n;
      float* ws = static_cast<float*>(scratch_for(e.stream, ws_bytes, 1));
      if (ws != nullptr && tiles * splits <= 0x7fffffffLL) {
        p.splits = splits;
        p.kb_per_split = kbps;
        p.ws = ws;
        p.tiles_per_batch *= splits;
        p.num_tiles = static_cast<int>(tiles * splits);
      }
    }
  }
  // D through TMA stores when D is TMA-addressable (split-K writes partials)
  CUtensorMap md = ma;
  p.tma_store = 0;
  p.wide16 = 0;
  p.seg_kb = seg_kb_default();
  if (p.splits == 1 && !tma_store_disabled()) {
    const int des = p.d_type == DT_F32 ? 4 : 2;
    const CUtensorMapDataType ddt = p.d_type == DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : p.d_type == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const bool aligned = (p.ldd * des) % 16 == 0 &&
                         (pr.batch <= 1 || p.strideD == 0 || (p.strideD * des) % 16 == 0);
    // 16-bit D of a 16-bit GEMM with a plain epilogue (alpha only, beta known
    // to be 0 on the host): boxes of 32 rows x 64 columns (4 KB, one staging
    // buffer); every other epilogue stores 32-column chunks
    const bool plain = p.beta_dev == nullptr && p.beta == 0.f && p.bias == nullptr && !p.relu &&
                       !p.gelu;
    const uint32_t box_cols = (des == 2 && BN % 64 == 0 && !Cfg::PROMOTE && plain) ? 64 : 32;
    if (aligned && encode_map_3d(&md, ddt, des, p.D, pr.m, pr.n, pr.batch, p.ldd, p.strideD, 32,
                                 box_cols, CU_TENSOR_MAP_SWIZZLE_NONE)) {
      p.tma_store = 1;
      p.wide16 = box_cols == 64 ? 1 : 0;
    }
  }
  int grid = persistent_grid(e, p.num_tiles * (PAIR ? 2 : 1));
  if (PAIR) {
    grid = pair_grid(kern, Cfg::THREADS, Cfg::SMEM_BYTES, grid);
    if (grid < 2) return KX_ERR_UNSUPPORTED;
  }
  p.pipe_stats = pipe_stats_begin();
  note_launch();
  if (PAIR) {
    const cudaError_t le = launch_pair(kern, grid, Cfg::THREADS, Cfg::SMEM_BYTES, e.stream, ma,
                                       mb, malo, mblo, md, p);
    if (le != cudaSuccess) return device_error(le);
  } else {
    kern<<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, e.stream>>>(ma, mb, malo, mblo, md, p);
  }
  pipe_stats_end(p.pipe_stats, "kx_gemm_tc", e.stream, grid);
  if (p.splits > 1) {
    note_launch();
    kx_splitk_reduce<<<splitk_reduce_grid(pr.m, pr.n, pr.batch, device_info().num_sms), 256, 0,
                       e.stream>>>(p, pr.batch);
  }
  static char name[96];
  if (name[0] == 0)
    snprintf(name, sizeof(name), "kx_gemm_tc<bn%d,%s,A%s,B%s%s>", BN, arith_name<AR>(),
             AMN ? "mn" : "k", BMN ? "mn" : "k", PAIR ? ",pair" : "");
  set_last_kernel_name(name);
  return launch_status();
}

// Per-arithmetic dispatch over (BN, A major, B major).
template <Arith AR>
int dispatch_gemm_tc(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                     const GemmParams& p) {
#define KX_CASE(BNV)                                                           \
  if (bn == BNV) {                                                              \
    if (!amn && !bmn) return launch_gemm_tc<BNV, AR, false, false>(e, pr, p);   \
    if (!amn && bmn) return launch_gemm_tc<BNV, AR, false, true>(e, pr, p);     \
    if (amn && !bmn) return launch_gemm_tc<BNV, AR, true, false>(e, pr, p);     \
    return launch_gemm_tc<BNV, AR, true, true>(e, pr, p);                       \
  }
  if constexpr (AR == Arith::BF16 || AR == Arith::F16) {
    bool pair = false;
    if (!amn && !bmn) {
      const int pm = gemm_pair_mode();
      const long long tiles = static_cast<long long>((pr.m + 127) / 128) * ((pr.n + 255) / 256) *
                              (pr.batch > 0 ? pr.batch : 1);
      pair = pm == 1 || (pm < 0 && pr.k >= 4096 && tiles >= 4LL * device_info().num_sms);
    }
    if (pair) {
      const int rc = bn == 256   ? launch_gemm_tc<256, AR, false, false, true>(e, pr, p)
                     : bn == 128 ? launch_gemm_tc<128, AR, false, false, true>(e, pr, p)
                                 : launch_gemm_tc<64, AR, false, false, true>(e, pr, p);
      if (rc != KX_ERR_UNSUPPORTED) return rc;
    }
  }
  if constexpr (AR != Arith::F32x3) {
    KX_CASE(256)
  }
  KX_CASE(128)
  KX_CASE(64)
  if constexpr (AR == Arith::F32x3) {
    KX_CASE(32)
  }
#undef KX_CASE
  return KX_ERR_UNSUPPORTED;
}

int dispatch_gemm_tc_f32x3(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                           const GemmParams& p);
int dispatch_gemm_tc_tf32(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                          const GemmParams& p);
int dispatch_gemm_tc_bf16(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                          const GemmParams& p);
int dispatch_gemm_tc_f16(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                         const GemmParams& p);

}  // namespace kx
