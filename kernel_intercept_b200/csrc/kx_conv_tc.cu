// kx_conv_tc.cu — forward convolution as an implicit GEMM on the persistent
// tcgen05 kernel (kx_gemm_tc_kernel with CONV = true), 3xTF32.
//
//   y_n (pixels x K) = A_n (pixels x Kd) * Wp^T (Kd x K)
//
// A is never materialised per tap.  One staging pass copies x to NHWC with
// the channels padded to a multiple of 32 (and writes the 3xTF32 low part
// beside it); the GEMM's producer then loads, for k-block (tap r,s; channel
// block c0), the 4-D TMA box {32 channels, wbox columns, hbox rows, 1 image}
// starting at the tap's offset (q0*sw - pw + s*dw, p0*sh - ph + r*dh).  The
// box lands as 128 rows of 128 bytes, exactly the K-major 128-byte-swizzled
// A tile, and TMA's zero fill supplies the padding border.  Strides use the
// tensor map's element strides.  When C*R*S is small (the first layer of a
// CNN: C = 3), taps are folded into the channel dimension instead: the
// staging holds [N][P][Q][round32(C*R*S)] and the GEMM is a 1x1 convolution.
//
// Wp[k][(r*S + s)*Cp + c] is the filter repacked tap-major (flipped for
// CUDNN_CONVOLUTION), streamed by TMA as a K-major B operand, with its low
// part beside it.  Replaces the im2col lowering for the forward pass
// (cudnnConvolutionForward, src/cudnn_intercept.cpp:433-489 of the reference).
#include <cstdio>
#include <cstring>

#include "kx_gemm_launch.cuh"

namespace kx {
namespace {

// NCHW -> NHWC with channels padded to cp; hi = x, lo = x - trunc_tf32(x).
// 32 channels x 32 pixels per block through shared memory so both the read
// (along pixels) and the write (along channels) coalesce.
__global__ void __launch_bounds__(256) stage_nhwc_split(const float* __restrict__ x,
                                                        float* __restrict__ xh,
                                                        float* __restrict__ xl, int C, int HW,
                                                        int cp) {
  __shared__ float tile[32][33];
  const int n = blockIdx.z;
  const int c0 = blockIdx.y * 32;
  const int p0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const float* xn = x + static_cast<size_t>(n) * C * HW;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = c0 + ty + 8 * j;
    const int px = p0 + tx;
    tile[ty + 8 * j][tx] = (c < C && px < HW) ? __ldg(xn + static_cast<size_t>(c) * HW + px) : 0.f;
  }
  __syncthreads();
  const size_t base = static_cast<size_t>(n) * HW * cp;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int px = p0 + ty + 8 * j;
    if (px < HW) {
      const float v = tile[tx][ty + 8 * j];
      const size_t o = base + static_cast<size_t>(px) * cp + c0 + tx;
      xh[o] = v;
      xl[o] = tf32_lo(v);
    }
  }
}

// Taps folded into channels: st[n][p][q][kk], kk = (c*R + r)*S + s < C*R*S,
// zero up to kf; hi and lo as above.  Block (blockIdx.x, p, n) covers 32
// output pixels q of row p of image n; lane = kk within a 32-wide chunk, so
// every store is one 128-byte row segment, and the (c, r, s) decode runs once
// per chunk instead of once per element.
constexpr int kFoldQ = 32;
__global__ void __launch_bounds__(256) stage_folded_split(const float* __restrict__ x,
                                                          float* __restrict__ xh,
                                                          float* __restrict__ xl, ConvShape g,
                                                          int kf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int p = blockIdx.y, n = blockIdx.z;
  const int q0 = blockIdx.x * kFoldQ;
  const int crs = g.C * g.R * g.S, rs_n = g.R * g.S;
  const float* xn = x + static_cast<size_t>(n) * g.C * g.H * g.W;
  const size_t row0 = (static_cast<size_t>(n) * g.P + p) * g.Q;
  for (int kb = 0; kb < kf; kb += 32) {
    const int kk = kb + lane;
    int c = 0, r = 0, sx = 0;
    bool valid = kk < crs;
    if (valid) {
      c = kk / rs_n;
      const int rs = kk - c * rs_n;
      r = rs / g.S;
      sx = rs - r * g.S;
    }
    const int h = p * g.sh - g.ph + r * g.dh;
    valid = valid && h >= 0 && h < g.H;
    const float* xr = xn + (static_cast<size_t>(c) * g.H + (valid ? h : 0)) * g.W;
    for (int i = warp; i < kFoldQ; i += 8) {
      const int q = q0 + i;
      if (q >= g.Q) break;
      const int w = q * g.sw - g.pw + sx * g.dw;
      const float v = (valid && w >= 0 && w < g.W) ? __ldg(xr + w) : 0.f;
      const size_t o = (row0 + q) * kf + kk;
      xh[o] = v;
      xl[o] = tf32_lo(v);
    }
  }
}

// Filter for the tap-major K order (folded = false: Wp[k][(r*S+s)*cp + c])
// or the folded order (folded = true: Wp[k][(c*R + r)*S + s], padded to cp).
__global__ void pack_filter(const float* __restrict__ w, float* __restrict__ wp,
                            float* __restrict__ wp_lo, int K, int C, int R, int S, int cp,
                            int folded, int flip, int transposed) {
  // 32-bit index math: the caller keeps K * row below 2^31
  const int RS = R * S;
  const int row = folded ? cp : RS * cp;
  const int total = K * row;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int k = i / row;
    const int rem = i - k * row;
    int c, r, s;
    bool valid;
    if (folded) {
      c = rem / RS;
      const int rs = rem - c * RS;
      r = rs / S;
      s = rs - r * S;
      valid = rem < C * RS;
    } else {
      const int tap = rem / cp;
      c = rem - tap * cp;
      r = tap / S;
      s = tap - r * S;
      valid = c < C;
    }
    float v = 0.f;
    if (valid) {
      if (flip) {
        r = R - 1 - r;
        s = S - 1 - s;
      }
      v = transposed ? w[((c * K + k) * R + r) * S + s] : w[((k * C + c) * R + r) * S + s];
    }
    wp[i] = v;
    wp_lo[i] = tf32_lo(v);
  }
}

// Output tile = hbox rows x wbox columns of output pixels (wbox * hbox =
// 128, powers of two), chosen to waste the fewest MMA rows (ties: widest).
void choose_box(int P, int Q, int sw, int sh, int& wbox, int& hbox) {
  long long best = -1;
  wbox = 128;
  hbox = 1;
  for (int wb = 1; wb <= 128; wb *= 2) {
    const int hb = 128 / wb;
    if (wb * sw > 256 || hb * sh > 256) continue;
    const long long tiles = static_cast<long long>((Q + wb - 1) / wb) * ((P + hb - 1) / hb);
    // ties go to the wider box: longer contiguous output rows
    if (best < 0 || tiles <= best) {
      best = tiles;
      wbox = wb;
      hbox = hb;
    }
  }
}

// How one forward convolution runs on the tcgen05 kernel.
struct ConvPlan {
  int bn;      // channel tile width (64 or 128)
  bool im2col; // A tiles by im2col-mode TMA (else wbox x hbox boxes)
  int splits;  // K slices (partials reduced by kx_splitk_reduce)
  int wbox, hbox;
  bool pair;   // 2-CTA clusters: 256-row tiles, cta_group::2 MMAs
};

// KX_CONV_IM2COL: "0" = box tiles; unset or "1" = im2col tiles whenever the
// map can express the geometry (see plan_conv).
int im2col_mode() {
  const char* v = std::getenv("KX_CONV_IM2COL");
  if (v == nullptr || v[0] == 0) return -1;
  return v[0] == '0' ? 0 : 1;
}

// KX_CTA_PAIR: "1" = CTA pairs whenever possible; unset or "0" = one CTA per
// tile.  Pairs load half of B per SM, but each SM's tensor core still reads
// all of B (half from the peer's shared memory) and the three 3xTF32
// products need three instructions instead of the one-CTA kernel's merged
// hi*[hi; lo]; on B200 the 13 VGG16 forward layers at batch 32 took 7.23 ms
// with pairs against 6.03 ms without (conv3_2 0.624 against 0.574 ms), so
// pairs are opt-in.
int pair_mode() {
  const char* v = std::getenv("KX_CTA_PAIR");
  if (v == nullptr || v[0] == 0) return -1;
  return v[0] == '0' ? 0 : 1;
}

// Bounding-box corners {w, h} of the im2col map for geometry t.
void im2col_corners(const ConvShape& t, int lower[2], int upper[2]) {
  lower[0] = -t.pw;
  lower[1] = -t.ph;
  upper[0] = t.pw - t.dw * (t.S - 1);
  upper[1] = t.ph - t.dh * (t.R - 1);
}

ConvPlan plan_conv(const ConvShape& g, const ConvShape& t, int cp, int sms) {
  ConvPlan pl{64, false, 1, 0, 0, false};
  choose_box(g.P, g.Q, t.sw, t.sh, pl.wbox, pl.hbox);
  const long long m = static_cast<long long>(g.N) * g.P * g.Q;
  int lo[2], up[2];
  im2col_corners(t, lo, up);
  bool im2col_ok = m + 128 <= 0x7fffffffLL && t.dw * (t.S - 1) < 65536 &&
                   t.dh * (t.R - 1) < 65536;
  for (int i = 0; i < 2; ++i)
    im2col_ok = im2col_ok && lo[i] >= -128 && up[i] >= -128 && up[i] <= 127;
  const long long box_mt = static_cast<long long>((g.Q + pl.wbox - 1) / pl.wbox) *
                           ((g.P + pl.hbox - 1) / pl.hbox) * g.N;
  // im2col tiles waste no MMA rows; box tiles of whole output rows waste
  // 12.5-23% of them on 28/56/112/14-wide maps.  Measured on VGG16 at batch
  // 32: im2col 5.70 ms over the 13 layers, boxes 5.94 ms (no layer more than
  // 0.7% slower with im2col).
  const int mode = im2col_mode();
  pl.im2col = im2col_ok && mode != 0;
  const long long mt = pl.im2col ? (m + 127) / 128 : box_mt;
  // 128-wide channel tiles when they fill the GPU and waste nothing
  if (g.K % 128 == 0 && mt * (g.K / 128) >= sms) pl.bn = 128;
  // CTA pairs: each CTA loads half of B, so 4 stages fit instead of 3
  const long long pair_tiles = (mt + 1) / 2 * ((g.K + pl.bn - 1) / pl.bn);
  const int pmode = pair_mode();
  pl.pair = sms >= 2 && pmode == 1 && pair_tiles >= 1;
  if (pl.pair) return pl;  // no split-K with pairs
  if (split_k_disabled()) return pl;
  // Split K when the tiles leave the last wave mostly empty: per slice count
  // s, waves x k-blocks per slice (a k-block ~0.55 us per CTA at BN 128),
  // plus writing and reading s fp32 partial planes (~5 TB/s).
  const long long tiles = mt * ((g.K + pl.bn - 1) / pl.bn);
  const int num_kb = t.R * t.S * cp / 32;
  if (tiles >= 4LL * sms) return pl;
  const double t_kb = 0.55e-6 * pl.bn / 128.0;
  double best = -1.0;
  for (int s = 1; s <= 8; ++s) {
    const int kbps = (num_kb + s - 1) / s;
    if (s > 1 && kbps < 8) break;
    const int real = (num_kb + kbps - 1) / kbps;
    if (real != s) continue;
    const long long waves = (tiles * s + sms - 1) / sms;
    double cost = static_cast<double>(waves) * kbps * t_kb;
    if (s > 1) cost += 2.0 * s * static_cast<double>(m) * g.K * 4.0 / 5e12;
    if (best < 0 || cost < best) {
      best = cost;
      pl.splits = s;
    }
  }
  return pl;
}

template <int BN, bool PAIR>
int launch_conv_tc(const Exec& e, const ConvShape& g, const ConvShape& t, const float* xh,
                   const float* xl, int cp, const float* wp, const float* wp_lo, float* y,
                   float alpha, float beta, const ConvPlan& pl) {
  // t: the geometry the kernel sees (g itself, or the folded 1x1 problem)
  using Cfg = GemmCfg<BN, Arith::F32x3, false, false, PAIR>;
  const long long kd = static_cast<long long>(t.R) * t.S * cp;
  const long long pq = static_cast<long long>(g.P) * g.Q;
  const int wbox = pl.wbox, hbox = pl.hbox;
  // A: NHWC staging {cp, W, H, N}
  const uint64_t dims[4] = {static_cast<uint64_t>(cp), static_cast<uint64_t>(t.W),
                            static_cast<uint64_t>(t.H), static_cast<uint64_t>(t.N)};
  const uint64_t strides[3] = {static_cast<uint64_t>(cp) * 4,
                               static_cast<uint64_t>(cp) * t.W * 4,
                               static_cast<uint64_t>(cp) * t.W * t.H * 4};
  const uint32_t es[4] = {1u, static_cast<uint32_t>(t.sw), static_cast<uint32_t>(t.sh), 1u};
  CUtensorMap ma, malo, mb, mblo;
  if (pl.im2col) {
    int lo[2], up[2];
    im2col_corners(t, lo, up);
    if (!encode_im2col_map(&ma, xh, dims, strides, lo, up, 32, Cfg::BM, es) ||
        !encode_im2col_map(&malo, xl, dims, strides, lo, up, 32, Cfg::BM, es))
      return KX_ERR_UNSUPPORTED;
  } else {
    const uint32_t box[4] = {32u, static_cast<uint32_t>(wbox * t.sw),
                             static_cast<uint32_t>(hbox * t.sh), 1u};
    if (!encode_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xh, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B, es) ||
        !encode_map(&malo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xl, dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B, es))
      return KX_ERR_UNSUPPORTED;
  }
  if (!encode_map_3d(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, wp, kd, g.K, 1, kd, 0, Cfg::BK,
                     Cfg::B_ROWS) ||
      !encode_map_3d(&mblo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, wp_lo, kd, g.K, 1, kd, 0, Cfg::BK,
                     Cfg::B_ROWS))
    return KX_ERR_UNSUPPORTED;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = static_cast<int>(pl.im2col ? pq * g.N : pq);
  p.n = g.K;
  p.k = static_cast<int>(kd);
  p.alpha = alpha;
  p.beta = beta;
  p.D = y;
  p.ldd = pq;
  p.strideD = pq * g.K;
  p.d_type = DT_F32;
  p.C = y;
  p.ldc = pq;
  p.strideC = pq * g.K;
  p.c_type = DT_F32;
  p.work = work_slot_for(e.stream);
  if (p.work == nullptr) return KX_ERR_NOMEM;
  p.yield_flag = e.yield_flag;
  p.done_flag = e.done_flag;
  p.max_tiles = e.max_tiles;
  p.timeout_ns = e.timeout_ns;
  p.err_word = e.err_word ? e.err_word : &p.work->err;
  p.presplit = 1;
  p.cv_p = g.P;
  p.cv_q = g.Q;
  p.cv_wbox = wbox;
  p.cv_hbox = hbox;
  p.cv_tiles_w = (g.Q + wbox - 1) / wbox;
  p.cv_s = t.S;
  p.cv_cb = cp / 32;
  p.cv_pad_h = t.ph;
  p.cv_pad_w = t.pw;
  p.cv_str_h = t.sh;
  p.cv_str_w = t.sw;
  p.cv_dil_h = t.dh;
  p.cv_dil_w = t.dw;
  p.cv_im2col = pl.im2col ? 1 : 0;
  p.cv_pq = static_cast<int>(pq);
  p.num_mb = pl.im2col ? (p.m + Cfg::BM - 1) / Cfg::BM
                       : p.cv_tiles_w * ((g.P + hbox - 1) / hbox);
  // a pair tile covers two consecutive 128-row blocks (the second may lie
  // past the end: its loads read zeros and its rows are not stored)
  if (PAIR) p.num_mb = (p.num_mb + 1) / 2;
  p.num_nb = (g.K + BN - 1) / BN;
  p.num_kb = static_cast<int>(kd / Cfg::BK);
  const int batch = pl.im2col ? 1 : g.N;
  p.splits = 1;
  p.kb_per_split = p.num_kb;
  if (pl.splits > 1) {
    const int kbps = (p.num_kb + pl.splits - 1) / pl.splits;
    const int splits = (p.num_kb + kbps - 1) / kbps;
    const size_t ws_bytes = sizeof(float) * static_cast<size_t>(splits) * batch *
                            static_cast<size_t>(p.m) * p.n;
    float* ws = static_cast<float*>(scratch_for(e.stream, ws_bytes, 1));
    if (ws != nullptr) {
      p.splits = splits;
      p.kb_per_split = kbps;
      p.ws = ws;
    }
  }
  p.tiles_per_batch = p.num_mb * p.num_nb * p.splits;
  const long long tiles = static_cast<long long>(p.tiles_per_batch) * batch;
  if (tiles <= 0 || tiles > 0x7fffffffLL) return KX_ERR_UNSUPPORTED;
  p.num_tiles = static_cast<int>(tiles);
  p.a_bcast = 0;
  p.b_bcast = 1;

  auto kern = kx_gemm_tc_kernel<Cfg, true>;
  static bool attr_set[64] = {false};
  const DeviceInfo& di = device_info();
  if (!attr_set[di.device & 63]) {
    const cudaError_t ae = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (ae != cudaSuccess) return device_error(ae);
    attr_set[di.device & 63] = true;
  }
  // y through TMA stores (16-byte rows needed).  im2col: {P*Q, K, N} map, a
  // warp's box {32 pixels, 32 channels, 1} when its rows lie in one image.
  // Boxes: {Q, P, K, N} map, per-warp box {min(wbox,32), 32/min(wbox,32),
  // 32 channels, 1}, at least 16 bytes wide.
  CUtensorMap md = ma;
  p.tma_store = 0;
  p.wide16 = 0;
  p.seg_kb = seg_kb_default();
  if (p.splits == 1 && !tma_store_disabled()) {
    if (pl.im2col) {
      if (pq % 4 == 0 && encode_map_3d(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, pq, g.K, g.N,
                                       pq, pq * g.K, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE))
        p.tma_store = 1;
    } else if (g.Q % 4 == 0 && wbox >= 4) {
      const int ww = wbox < 32 ? wbox : 32;
      const uint64_t ydims[4] = {static_cast<uint64_t>(g.Q), static_cast<uint64_t>(g.P),
                                 static_cast<uint64_t>(g.K), static_cast<uint64_t>(g.N)};
      const uint64_t ystr[3] = {static_cast<uint64_t>(g.Q) * 4, static_cast<uint64_t>(pq) * 4,
                                static_cast<uint64_t>(pq) * g.K * 4};
      const uint32_t ybox[4] = {static_cast<uint32_t>(ww), static_cast<uint32_t>(32 / ww), 32u,
                                1u};
      if (encode_map(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, ydims, ystr, ybox,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        p.tma_store = 1;
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
  pipe_stats_end(p.pipe_stats, "kx_conv_fwd_tc", e.stream, grid);
  if (p.splits > 1) {
    note_launch();
    kx_splitk_reduce<<<splitk_reduce_grid(p.m, p.n, batch, di.num_sms), 256, 0, e.stream>>>(
        p, batch);
  }
  static char names[2][64];
  char* name = names[pl.im2col ? 1 : 0];
  if (name[0] == 0)
    snprintf(name, 64, "kx_conv_fwd_tc<bn%d,f32x3,%s%s>", BN,
             pl.im2col ? "im2col" : "box", PAIR ? ",pair" : "");
  set_last_kernel_name(name);
  return launch_status();
}

size_t round256(size_t elems) { return (elems + 63) & ~static_cast<size_t>(63); }

int grid_for(size_t total) {
  size_t b = (total + 255) / 256;
  const size_t cap = 8ull * device_info().num_sms;
  return static_cast<int>(b < 1 ? 1 : (b > cap ? cap : b));
}

// ------------------------------------------------------- backward filter --

// lo = x - trunc_tf32(x), elementwise (the 3xTF32 low part of dy)
__global__ void __launch_bounds__(256) split_lo(const float* __restrict__ x,
                                                float* __restrict__ lo, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    lo[i] = tf32_lo(x[i]);
}

// dw[k][c][r][s] = alpha * sum over K slices of D[k][(tap, c)] + beta * dw,
// D column-major per slice (ld = K), tap = r*S + s, or (R-1-r)*S + (S-1-s)
// for a true convolution (its forward pass applied the filter flipped); with
// folded taps D's columns are (c, tap) of the folded staging.
// Runs only when the GEMM launch completed all its tiles.
__global__ void __launch_bounds__(256) wgrad_reduce(const float* __restrict__ ws,
                                                    const WorkSlot* work, int splits, int K,
                                                    int C, int R, int S, int cp, int ncols,
                                                    int flip, int folded, float alpha,
                                                    float beta, float* dw) {
  if (work->status != 1) return;
  const int RS = R * S;
  const long long total = static_cast<long long>(K) * C * RS;
  const long long mn = static_cast<long long>(K) * ncols;  // one K slice of D
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * 256) {
    const int k = static_cast<int>(i / (static_cast<long long>(C) * RS));
    const int rem = static_cast<int>(i - static_cast<long long>(k) * C * RS);
    const int c = rem / RS;
    const int rs = rem - c * RS;
    const int r = rs / S;
    const int s = rs - r * S;
    const int tap = flip ? (R - 1 - r) * S + (S - 1 - s) : rs;
    // folded: one column per (c, r, s) of the folded staging ((c*R + r)*S + s)
    const long long col = folded ? static_cast<long long>(c) * RS + tap
                                 : static_cast<long long>(tap) * cp + c;
    float acc = 0.f;
    for (int sl = 0; sl < splits; ++sl) acc += ws[sl * mn + col * K + k];
    float o = alpha * acc;
    if (beta != 0.f) o += beta * dw[i];
    dw[i] = o;
  }
}

// t: the geometry the kernel sees (g itself, or the folded 1x1 problem over
// the [N][P][Q][cp] staging); g: the convolution (for dw's layout)
template <int BN>
int launch_wgrad(const Exec& e, const ConvShape& g, const ConvShape& t, bool folded,
                 const float* xh, const float* xl, int cp, const float* dy, const float* dy_lo,
                 float* dw, float alpha, float beta) {
  using Cfg = GemmCfg<BN, Arith::F32x3, false, true>;
  const long long pq = static_cast<long long>(g.P) * g.Q;
  // A: dy as {P*Q, K, N}, 32 pixels x 128 output channels per box
  CUtensorMap ma, malo, mb, mblo;
  if (!encode_map_3d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dy, pq, g.K, g.N, pq, pq * g.K,
                     Cfg::BK, Cfg::BM) ||
      !encode_map_3d(&malo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dy_lo, pq, g.K, g.N, pq,
                     pq * g.K, Cfg::BK, Cfg::BM))
    return KX_ERR_UNSUPPORTED;
  // B: im2col of the NHWC staging, 32 pixels x 32 channels, M/N-major tf32
  const uint64_t dims[4] = {static_cast<uint64_t>(cp), static_cast<uint64_t>(t.W),
                            static_cast<uint64_t>(t.H), static_cast<uint64_t>(t.N)};
  const uint64_t strides[3] = {static_cast<uint64_t>(cp) * 4,
                               static_cast<uint64_t>(cp) * t.W * 4,
                               static_cast<uint64_t>(cp) * t.W * t.H * 4};
  const uint32_t es[4] = {1u, static_cast<uint32_t>(t.sw), static_cast<uint32_t>(t.sh), 1u};
  int lo[2], up[2];
  im2col_corners(t, lo, up);
  if (!encode_im2col_map(&mb, xh, dims, strides, lo, up, 32, 32, es,
                         CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !encode_im2col_map(&mblo, xl, dims, strides, lo, up, 32, 32, es,
                         CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return KX_ERR_UNSUPPORTED;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  const int pb = static_cast<int>((pq + 31) / 32);
  const long long num_kb = static_cast<long long>(g.N) * pb;
  if (num_kb > 0x7fffffffLL / 32) return KX_ERR_UNSUPPORTED;
  p.m = g.K;
  p.n = t.R * t.S * cp;
  p.k = static_cast<int>(num_kb * 32);
  p.alpha = 1.f;
  p.beta = 0.f;
  p.d_type = DT_F32;
  p.c_type = DT_F32;
  p.work = work_slot_for(e.stream);
  if (p.work == nullptr) return KX_ERR_NOMEM;
  p.yield_flag = e.yield_flag;
  p.done_flag = e.done_flag;
  p.max_tiles = e.max_tiles;
  p.timeout_ns = e.timeout_ns;
  p.err_word = e.err_word ? e.err_word : &p.work->err;
  p.presplit = 1;
  p.cv_wgrad = 1;
  p.cv_pb = pb;
  p.cv_nb_per_tap = cp / BN;
  p.cv_p = g.P;
  p.cv_q = t.Q;
  p.cv_s = t.S;
  p.cv_pad_h = t.ph;
  p.cv_pad_w = t.pw;
  p.cv_str_h = t.sh;
  p.cv_str_w = t.sw;
  p.cv_dil_h = t.dh;
  p.cv_dil_w = t.dw;
  p.num_mb = (g.K + Cfg::BM - 1) / Cfg::BM;
  p.num_nb = t.R * t.S * (cp / BN);
  p.num_kb = static_cast<int>(num_kb);
  // K slices: about 3 waves of work units (measured on the VGG16 layers:
  // 3 waves beat 1 to 2), choosing within +-50% the count whose last wave is
  // fullest; at least 8 k-blocks per slice
  const long long tiles = static_cast<long long>(p.num_mb) * p.num_nb;
  const int sms = persistent_grid(e, 1 << 30);
  long long target = 3LL * sms / tiles;
  if (target < 1) target = 1;
  long long want = 1;
  double best = -1.0;
  for (long long sl = (target + 1) / 2; sl <= target + target / 2; ++sl) {
    if (sl < 1 || (sl > 1 && sl * 8 > num_kb)) continue;
    const long long units = tiles * sl;
    const long long waves = (units + sms - 1) / sms;
    const double fill = static_cast<double>(units) / static_cast<double>(waves * sms);
    const double score = fill - 1e-3 * static_cast<double>(sl > target ? sl - target : target - sl);
    if (score > best) {
      best = score;
      want = sl;
    }
  }
  const int kbps = static_cast<int>((num_kb + want - 1) / want);
  p.splits = static_cast<int>((num_kb + kbps - 1) / kbps);
  p.kb_per_split = kbps;
  const size_t plane = static_cast<size_t>(p.m) * p.n;
  float* ws = static_cast<float*>(scratch_for(e.stream, sizeof(float) * plane * p.splits, 1));
  if (ws == nullptr) return KX_ERR_NOMEM;
  p.ws = ws;
  // one slice: the plain epilogue writes the raw sums (alpha 1, beta 0) to ws
  p.D = ws;
  p.ldd = p.m;
  p.C = ws;
  p.ldc = p.m;
  p.tiles_per_batch = p.num_mb * p.num_nb * p.splits;
  if (static_cast<long long>(p.tiles_per_batch) > 0x7fffffffLL) return KX_ERR_UNSUPPORTED;
  p.num_tiles = p.tiles_per_batch;
  p.tma_store = 0;
  p.wide16 = 0;
  p.seg_kb = seg_kb_default();
  auto kern = kx_gemm_tc_kernel<Cfg, true>;
  static bool attr_set[64] = {false};
  const DeviceInfo& di = device_info();
  if (!attr_set[di.device & 63]) {
    const cudaError_t ae = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (ae != cudaSuccess) return device_error(ae);
    attr_set[di.device & 63] = true;
  }
  CUtensorMap md = ma;  // unused (no TMA stores)
  const int grid = persistent_grid(e, p.num_tiles);
  p.pipe_stats = pipe_stats_begin();
  note_launch();
  kern<<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, e.stream>>>(ma, mb, malo, mblo, md, p);
  pipe_stats_end(p.pipe_stats, "kx_conv_wgrad_tc", e.stream, grid);
  note_launch();
  wgrad_reduce<<<grid_for(static_cast<size_t>(g.K) * g.C * g.R * g.S), 256, 0, e.stream>>>(
      ws, p.work, p.splits, g.K, g.C, g.R, g.S, cp, p.n, g.flip ? 1 : 0, folded ? 1 : 0, alpha,
      beta, dw);
  static char name[64];
  if (name[0] == 0) snprintf(name, sizeof(name), "kx_conv_wgrad_tc<bn%d,f32x3>", BN);
  set_last_kernel_name(name);
  return launch_status();
}

}  // namespace

int conv_fwd_implicit(const Exec& e, const ConvShape& g, const float* x, const float* w, float* y,
                      float alpha, float beta) {
  if (e.fp32_mode != KX_FP32_3XTF32) return KX_ERR_UNSUPPORTED;
  const int crs = g.C * g.R * g.S;
  const int cp_taps = (g.C + 31) / 32 * 32;
  const int kf = (crs + 31) / 32 * 32;
  // fold the taps into channels when that at least halves the K extent
  const bool folded = static_cast<long long>(kf) * 2 <= static_cast<long long>(cp_taps) * g.R * g.S;
  ConvShape t = g;  // geometry seen by the kernel
  int cp = cp_taps;
  if (folded) {
    t.C = kf;
    t.H = g.P;
    t.W = g.Q;
    t.R = t.S = 1;
    t.ph = t.pw = 0;
    t.sh = t.sw = 1;
    t.dh = t.dw = 1;
    cp = kf;
  }
  if (t.sw > 8 || t.sh > 8) return KX_ERR_UNSUPPORTED;
  const size_t stage_elems = static_cast<size_t>(t.N) * t.H * t.W * cp;
  const size_t wp_elems = static_cast<size_t>(g.K) * t.R * t.S * cp;
  if (stage_elems > (1ull << 36) || wp_elems >= (1ull << 31) ||
      static_cast<long long>(g.P) * g.Q * g.K > (1LL << 40))
    return KX_ERR_UNSUPPORTED;
  const size_t s_pad = round256(stage_elems), w_pad = round256(wp_elems);
  float* base = static_cast<float*>(
      scratch_for(e.stream, (2 * s_pad + 2 * w_pad) * sizeof(float)));
  if (base == nullptr) return KX_ERR_NOMEM;
  float* xh = base;
  float* xl = base + s_pad;
  float* wp = base + 2 * s_pad;
  float* wp_lo = wp + w_pad;
  note_launch();
  if (folded) {
    dim3 grid((g.Q + kFoldQ - 1) / kFoldQ, g.P, g.N);
    if (grid.y > 65535 || grid.z > 65535) return KX_ERR_UNSUPPORTED;
    stage_folded_split<<<grid, 256, 0, e.stream>>>(x, xh, xl, g, kf);
  } else {
    const int hw = g.H * g.W;
    dim3 grid((hw + 31) / 32, cp / 32, g.N);
    if (grid.y > 65535 || grid.z > 65535) return KX_ERR_UNSUPPORTED;
    stage_nhwc_split<<<grid, 256, 0, e.stream>>>(x, xh, xl, g.C, hw, cp);
  }
  note_launch();
  pack_filter<<<grid_for(wp_elems), 256, 0, e.stream>>>(w, wp, wp_lo, g.K, g.C, g.R, g.S, cp,
                                                        folded ? 1 : 0, g.flip ? 1 : 0,
                                                        g.transposed ? 1 : 0);
  if (launch_status() != KX_OK) return KX_ERR_DEVICE;
  const ConvPlan pl = plan_conv(g, t, cp, persistent_grid(e, 1 << 30));
  if (pl.pair) {
    const int rc =
        pl.bn == 128 ? launch_conv_tc<128, true>(e, g, t, xh, xl, cp, wp, wp_lo, y, alpha, beta, pl)
                     : launch_conv_tc<64, true>(e, g, t, xh, xl, cp, wp, wp_lo, y, alpha, beta, pl);
    if (rc != KX_ERR_UNSUPPORTED) return rc;
  }
  if (pl.bn == 128)
    return launch_conv_tc<128, false>(e, g, t, xh, xl, cp, wp, wp_lo, y, alpha, beta, pl);
  return launch_conv_tc<64, false>(e, g, t, xh, xl, cp, wp, wp_lo, y, alpha, beta, pl);
}

int conv_bwd_filter_implicit(const Exec& e, const ConvShape& g, const float* x, const float* dy,
                             float* dw, float alpha, float beta) {
  if (e.fp32_mode != KX_FP32_3XTF32) return KX_ERR_UNSUPPORTED;
  const long long pq = static_cast<long long>(g.P) * g.Q;
  const int cp_taps = (g.C + 31) / 32 * 32;
  const int kf = (g.C * g.R * g.S + 31) / 32 * 32;
  // fold the taps into channels when that at least halves the N extent
  // (the first layer: C = 3); the kernel then sees a 1x1 problem over the
  // [N][P][Q][kf] staging
  const bool folded = static_cast<long long>(kf) * 2 <= static_cast<long long>(cp_taps) * g.R * g.S;
  ConvShape t = g;
  int cp = cp_taps;
  if (folded) {
    t.C = kf;
    t.H = g.P;
    t.W = g.Q;
    t.R = t.S = 1;
    t.ph = t.pw = 0;
    t.sh = t.sw = 1;
    t.dh = t.dw = 1;
    cp = kf;
  }
  // 16-byte dy rows for the TMA map
  if (pq % 4 != 0 || t.sw > 8 || t.sh > 8) return KX_ERR_UNSUPPORTED;
  int lo[2], up[2];
  im2col_corners(t, lo, up);
  for (int i = 0; i < 2; ++i)
    if (lo[i] < -128 || up[i] < -128 || up[i] > 127) return KX_ERR_UNSUPPORTED;
  if (t.dw * (t.S - 1) >= 65536 || t.dh * (t.R - 1) >= 65536) return KX_ERR_UNSUPPORTED;
  const size_t stage_elems = static_cast<size_t>(t.N) * t.H * t.W * cp;
  const size_t dy_elems = static_cast<size_t>(g.N) * g.K * pq;
  if (stage_elems > (1ull << 36) || dy_elems > (1ull << 36)) return KX_ERR_UNSUPPORTED;
  const size_t s_pad = round256(stage_elems), d_pad = round256(dy_elems);
  float* base = static_cast<float*>(scratch_for(e.stream, (2 * s_pad + d_pad) * sizeof(float)));
  if (base == nullptr) return KX_ERR_NOMEM;
  float* xh = base;
  float* xl = base + s_pad;
  float* dy_lo = base + 2 * s_pad;
  if (folded) {
    dim3 grid((g.Q + kFoldQ - 1) / kFoldQ, g.P, g.N);
    if (grid.y > 65535 || grid.z > 65535) return KX_ERR_UNSUPPORTED;
    note_launch();
    stage_folded_split<<<grid, 256, 0, e.stream>>>(x, xh, xl, g, kf);
  } else {
    const int hw = g.H * g.W;
    dim3 grid((hw + 31) / 32, cp / 32, g.N);
    if (grid.y > 65535 || grid.z > 65535) return KX_ERR_UNSUPPORTED;
    note_launch();
    stage_nhwc_split<<<grid, 256, 0, e.stream>>>(x, xh, xl, g.C, hw, cp);
  }
  note_launch();
  split_lo<<<grid_for(dy_elems), 256, 0, e.stream>>>(dy, dy_lo, dy_elems);
  if (launch_status() != KX_OK) return KX_ERR_DEVICE;
  if (cp % 128 == 0)
    return launch_wgrad<128>(e, g, t, folded, xh, xl, cp, dy, dy_lo, dw, alpha, beta);
  if (cp % 64 == 0)
    return launch_wgrad<64>(e, g, t, folded, xh, xl, cp, dy, dy_lo, dw, alpha, beta);
  return launch_wgrad<32>(e, g, t, folded, xh, xl, cp, dy, dy_lo, dw, alpha, beta);
}

}  // namespace kx

