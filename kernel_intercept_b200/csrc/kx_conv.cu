// kx_conv.cu — convolution entry points (cudnnConvolutionForward /
// BackwardData / BackwardFilter replacements), NCHW x, KCRS w, NCHW y, fp32.
//
// Each convolution is lowered onto the tcgen05 GEMM (3xTF32 by default):
//   fwd    y_n (PQ x K)    = colT_n^T (PQ x CRS) * W^T (CRS x K)
//   dgrad  colT_n (CRS x PQ) <- dy_n^T (PQ x K) * W (K x CRS), then a
//          gather (col2im) writes dx with alpha/beta
//   wgrad  dW (CRS x K)    = sum_n colT_n (CRS x PQ) * dy_n^T (PQ x K)
// colT_n is the im2col matrix of image n stored tap-major ([CRS][PQ], rows
// padded to a multiple of 4 floats so TMA can address it); it lives in the
// stream's scratch arena and is produced / consumed in chunks of images that
// bound the scratch size.  Tap-major layout keeps both the im2col gather and
// the col2im gather coalesced along the output row (q).
// Reference call sites: src/cudnn_intercept.cpp:433-627.
#include <cstring>

#include "kx_runtime.cuh"

namespace kx {
namespace {

constexpr size_t kScratchBudget = 1ull << 31;  // bytes of im2col staging per chunk

struct ConvGeom {
  int N, C, H, W, K, R, S, ph, pw, sh, sw, dh, dw, xcorr;
  int P, Q, PQ, CRS, ldpq;
};

bool make_geom(const kx_conv_desc* d, ConvGeom& g) {
  if (d == nullptr) return false;
  g.N = d->n; g.C = d->c; g.H = d->h; g.W = d->w; g.K = d->k; g.R = d->r; g.S = d->s;
  g.ph = d->pad_h; g.pw = d->pad_w; g.sh = d->stride_h; g.sw = d->stride_w;
  g.dh = d->dil_h; g.dw = d->dil_w; g.xcorr = d->cross_correlation;
  if (g.N <= 0 || g.C <= 0 || g.H <= 0 || g.W <= 0 || g.K <= 0 || g.R <= 0 || g.S <= 0)
    return false;
  if (g.ph < 0 || g.pw < 0 || g.sh <= 0 || g.sw <= 0 || g.dh <= 0 || g.dw <= 0) return false;
  g.P = (g.H + 2 * g.ph - ((g.R - 1) * g.dh + 1)) / g.sh + 1;
  g.Q = (g.W + 2 * g.pw - ((g.S - 1) * g.dw + 1)) / g.sw + 1;
  if (g.P <= 0 || g.Q <= 0) return false;
  g.PQ = g.P * g.Q;
  g.CRS = g.C * g.R * g.S;
  g.ldpq = (g.PQ + 3) & ~3;
  return true;
}

// colT[i][crs][pq] for images n0 .. n0+nb-1 (i = n - n0).
__global__ void im2col_tap_major(const float* __restrict__ x, float* __restrict__ col, ConvGeom g,
                                 int n0) {
  const int crs = blockIdx.y;
  const int i = blockIdx.z;
  const int c = crs / (g.R * g.S);
  const int rs = crs - c * g.R * g.S;
  const int r = rs / g.S, s = rs - (rs / g.S) * g.S;
  const float* xc = x + (static_cast<size_t>(n0 + i) * g.C + c) * g.H * g.W;
  float* out = col + (static_cast<size_t>(i) * g.CRS + crs) * g.ldpq;
  for (int pq = blockIdx.x * blockDim.x + threadIdx.x; pq < g.PQ; pq += gridDim.x * blockDim.x) {
    const int p = pq / g.Q, q = pq - (pq / g.Q) * g.Q;
    const int h = p * g.sh - g.ph + r * g.dh;
    const int w = q * g.sw - g.pw + s * g.dw;
    float v = 0.f;
    if (h >= 0 && h < g.H && w >= 0 && w < g.W) v = __ldg(xc + static_cast<size_t>(h) * g.W + w);
    out[pq] = v;
  }
}

// dx[n][c][h][w] = alpha * sum_{r,s} colT[i][(c,r,s)][(p,q)] + beta * dx.
__global__ void col2im_gather(const float* __restrict__ col, float* dx, ConvGeom g, int n0,
                              float alpha, float beta) {
  const int c = blockIdx.y, i = blockIdx.z;
  float* out = dx + (static_cast<size_t>(n0 + i) * g.C + c) * g.H * g.W;
  const float* cb = col + (static_cast<size_t>(i) * g.CRS + static_cast<size_t>(c) * g.R * g.S) * g.ldpq;
  for (int hw = blockIdx.x * blockDim.x + threadIdx.x; hw < g.H * g.W;
       hw += gridDim.x * blockDim.x) {
    const int h = hw / g.W, w = hw - (hw / g.W) * g.W;
    float acc = 0.f;
    for (int r = 0; r < g.R; ++r) {
      const int ph = h + g.ph - r * g.dh;
      if (ph < 0 || ph % g.sh != 0) continue;
      const int p = ph / g.sh;
      if (p >= g.P) continue;
      for (int s = 0; s < g.S; ++s) {
        const int qw = w + g.pw - s * g.dw;
        if (qw < 0 || qw % g.sw != 0) continue;
        const int q = qw / g.sw;
        if (q >= g.Q) continue;
        acc += __ldg(cb + static_cast<size_t>(r * g.S + s) * g.ldpq + p * g.Q + q);
      }
    }
    float o = alpha * acc;
    if (beta != 0.f) o = fmaf(beta, out[hw], o);
    out[hw] = o;
  }
}

// wt[k][kp] = W[k][c][r'][s'] for kp = (c,r,s) < CRS (r' = R-1-r, s' = S-1-s
// when the descriptor asks for CUDNN_CONVOLUTION), 0 for the padding kp in
// [CRS, Kp).  Kp is CRS rounded up to 4 floats so TMA can address rows.
__global__ void prepare_filter(const float* __restrict__ w, float* __restrict__ wt, int K, int C,
                               int R, int S, int Kp, int flip) {
  const int CRS = C * R * S;
  const size_t total = static_cast<size_t>(K) * Kp;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t k = i / Kp;
    const int kp = static_cast<int>(i - k * Kp);
    float v = 0.f;
    if (kp < CRS) {
      int src = kp;
      if (flip) {
        const int c = kp / (R * S), rs = kp - c * R * S;
        const int r = rs / S, s = rs - (rs / S) * S;
        src = (c * R + (R - 1 - r)) * S + (S - 1 - s);
      }
      v = w[k * CRS + src];
    }
    wt[i] = v;
  }
}

// dw = alpha * flip(g) + beta * dw
__global__ void flip_accumulate(const float* __restrict__ gsrc, float* dw, int KC, int R, int S,
                                float alpha, float beta) {
  const size_t total = static_cast<size_t>(KC) * R * S;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t kc = i / (R * S);
    const int rs = static_cast<int>(i - kc * R * S);
    const int r = rs / S, s = rs - (rs / S) * S;
    float o = alpha * gsrc[kc * R * S + static_cast<size_t>(R - 1 - r) * S + (S - 1 - s)];
    if (beta != 0.f) o = fmaf(beta, dw[i], o);
    dw[i] = o;
  }
}

int grid_1d(size_t total) {
  size_t b = (total + 255) / 256;
  size_t cap = 8ull * device_info().num_sms;
  return static_cast<int>(b < cap ? (b < 1 ? 1 : b) : cap);
}

int images_per_chunk(const ConvGeom& g) {
  const size_t per = static_cast<size_t>(g.CRS) * g.ldpq * sizeof(float);
  size_t nb = per ? kScratchBudget / per : g.N;
  if (nb < 1) nb = 1;
  if (nb > static_cast<size_t>(g.N)) nb = g.N;
  if (nb > 65535) nb = 65535;
  return static_cast<int>(nb);
}

// Inner GEMMs always run with host-side scalars.
kx_exec inner_exec(const kx_exec* ex, cudaStream_t st) {
  kx_exec e;
  std::memset(&e, 0, sizeof(e));
  if (ex != nullptr) e = *ex;
  e.stream = st;
  e.scalars_on_device = 0;
  e.yield_flag = nullptr;  // staging between GEMMs must not be interleaved with yields
  e.done_flag = nullptr;
  e.max_tiles = 0;
  return e;
}

__global__ void set_flag(volatile int* flag, int v) {
  *flag = v;
  __threadfence_system();
}

int finish_done(const Exec& e) {
  if (e.done_flag != nullptr) {
    note_launch();
    set_flag<<<1, 1, 0, e.stream>>>(e.done_flag, 1);
  }
  return launch_status();
}

int round4(int v) { return (v + 3) & ~3; }

// KX_CONV_IMPLICIT=0 lowers forward convolutions through im2col instead.
bool implicit_conv_enabled() {
  static const bool on = [] {
    const char* s = std::getenv("KX_CONV_IMPLICIT");
    return s == nullptr || s[0] != '0';
  }();
  return on;
}

}  // namespace
}  // namespace kx

using namespace kx;

extern "C" int kx_conv_out_dims(const kx_conv_desc* d, int* p, int* q) {
  ConvGeom g;
  if (!make_geom(d, g) || p == nullptr || q == nullptr) return KX_ERR_INVALID;
  *p = g.P;
  *q = g.Q;
  return KX_OK;
}

extern "C" int kx_conv_fwd(const kx_exec* ex, const kx_conv_desc* d, const float* alpha,
                           const float* x, const float* w, const float* beta, float* y) {
  ConvGeom g;
  if (!make_geom(d, g) || !x || !w || !y || !alpha || !beta) return KX_ERR_INVALID;
  Exec e = resolve_exec(ex);
  if (implicit_conv_enabled()) {
    // one persistent implicit-GEMM launch (preemptible like any kx GEMM)
    const ConvShape cs{g.N, g.C, g.H, g.W, g.K, g.R, g.S, g.ph, g.pw, g.sh,
                       g.sw, g.dh, g.dw, g.P, g.Q, g.xcorr == 0};
    const int rc = conv_fwd_implicit(e, cs, x, w, y, *alpha, *beta);
    if (rc != KX_ERR_UNSUPPORTED) return rc;
  }
  const int nb = images_per_chunk(g);
  const size_t col_elems = static_cast<size_t>(nb) * g.CRS * g.ldpq;
  const bool repack = !g.xcorr || (g.CRS & 3) != 0;
  const int Kp = repack ? round4(g.CRS) : g.CRS;
  const size_t wf_elems = repack ? static_cast<size_t>(g.K) * Kp : 0;
  float* col = static_cast<float*>(scratch_for(e.stream, (col_elems + wf_elems) * sizeof(float)));
  if (col == nullptr) return KX_ERR_NOMEM;
  const float* wt = w;
  if (repack) {
    float* wf = col + col_elems;
    note_launch();
    prepare_filter<<<grid_1d(wf_elems), 256, 0, e.stream>>>(w, wf, g.K, g.C, g.R, g.S, Kp,
                                                            g.xcorr ? 0 : 1);
    wt = wf;
  }
  kx_exec ie = inner_exec(ex, e.stream);
  const float a = *alpha, b = *beta;
  for (int n0 = 0; n0 < g.N; n0 += nb) {
    const int cnt = g.N - n0 < nb ? g.N - n0 : nb;
    dim3 grid((g.PQ + 255) / 256 < 64 ? (g.PQ + 255) / 256 : 64, g.CRS, cnt);
    note_launch();
    im2col_tap_major<<<grid, 256, 0, e.stream>>>(x, col, g, n0);
    // y_n (PQ x K, ld PQ) = colT_n^T * W^T
    int rc = kx_sgemm_strided_batched(&ie, KX_OP_N, KX_OP_N, g.PQ, g.K, g.CRS, &a, col, g.ldpq,
                                      static_cast<long long>(g.CRS) * g.ldpq, wt, Kp, 0, &b,
                                      y + static_cast<size_t>(n0) * g.K * g.PQ, g.PQ,
                                      static_cast<long long>(g.K) * g.PQ, cnt);
    if (rc != KX_OK) return rc;
  }
  return finish_done(e);
}

extern "C" int kx_conv_bwd_data(const kx_exec* ex, const kx_conv_desc* d, const float* alpha,
                                const float* w, const float* dy, const float* beta, float* dx) {
  ConvGeom g;
  if (!make_geom(d, g) || !w || !dy || !dx || !alpha || !beta) return KX_ERR_INVALID;
  Exec e = resolve_exec(ex);
  // Stride 1: dx is the forward cross-correlation of dy with the filter
  // transposed (K <-> C) and flipped (for cross-correlation; unflipped for
  // true convolution), padded by dil*(taps-1) - pad: one implicit-GEMM launch.
  const int pad_h = g.dh * (g.R - 1) - g.ph, pad_w = g.dw * (g.S - 1) - g.pw;
  if (implicit_conv_enabled() && g.sh == 1 && g.sw == 1 && pad_h >= 0 && pad_w >= 0) {
    ConvShape cs{g.N, g.K, g.P, g.Q, g.C, g.R, g.S, pad_h, pad_w, 1, 1, g.dh, g.dw, g.H, g.W,
                 g.xcorr != 0};
    cs.transposed = true;
    const int rc = conv_fwd_implicit(e, cs, dy, w, dx, *alpha, *beta);
    if (rc != KX_ERR_UNSUPPORTED) return rc;
  }
  const int nb = images_per_chunk(g);
  const size_t col_elems = static_cast<size_t>(nb) * g.CRS * g.ldpq;
  const bool repack = !g.xcorr || (g.CRS & 3) != 0;
  const int Kp = repack ? round4(g.CRS) : g.CRS;
  const size_t wf_elems = repack ? static_cast<size_t>(g.K) * Kp : 0;
  float* col = static_cast<float*>(scratch_for(e.stream, (col_elems + wf_elems) * sizeof(float)));
  if (col == nullptr) return KX_ERR_NOMEM;
  const float* wt = w;
  if (repack) {
    float* wf = col + col_elems;
    note_launch();
    prepare_filter<<<grid_1d(wf_elems), 256, 0, e.stream>>>(w, wf, g.K, g.C, g.R, g.S, Kp,
                                                            g.xcorr ? 0 : 1);
    wt = wf;
  }
  kx_exec ie = inner_exec(ex, e.stream);
  const float one = 1.f, zero = 0.f;
  for (int n0 = 0; n0 < g.N; n0 += nb) {
    const int cnt = g.N - n0 < nb ? g.N - n0 : nb;
    // colT_n (PQ x CRS col-major, ld ldpq) = dy_n (PQ x K) * W (K x CRS)
    int rc = kx_sgemm_strided_batched(&ie, KX_OP_N, KX_OP_T, g.PQ, g.CRS, g.K, &one,
                                      dy + static_cast<size_t>(n0) * g.K * g.PQ, g.PQ,
                                      static_cast<long long>(g.K) * g.PQ, wt, Kp, 0, &zero,
                                      col, g.ldpq, static_cast<long long>(g.CRS) * g.ldpq, cnt);
    if (rc != KX_OK) return rc;
    dim3 grid((g.H * g.W + 255) / 256 < 64 ? (g.H * g.W + 255) / 256 : 64, g.C, cnt);
    note_launch();
    col2im_gather<<<grid, 256, 0, e.stream>>>(col, dx, g, n0, *alpha, *beta);
  }
  return finish_done(e);
}

extern "C" int kx_conv_bwd_filter(const kx_exec* ex, const kx_conv_desc* d, const float* alpha,
                                  const float* x, const float* dy, const float* beta, float* dw) {
  ConvGeom g;
  if (!make_geom(d, g) || !x || !dy || !dw || !alpha || !beta) return KX_ERR_INVALID;
  Exec e = resolve_exec(ex);
  if (implicit_conv_enabled()) {
    // one implicit-GEMM launch over all images (split over the pixel sum)
    const ConvShape cs{g.N, g.C, g.H, g.W, g.K, g.R, g.S, g.ph, g.pw, g.sh,
                       g.sw, g.dh, g.dw, g.P, g.Q, g.xcorr == 0};
    const int rc = conv_bwd_filter_implicit(e, cs, x, dy, dw, *alpha, *beta);
    if (rc != KX_ERR_UNSUPPORTED) return rc;
  }
  const int nb = images_per_chunk(g);
  const size_t col_elems = static_cast<size_t>(nb) * g.CRS * g.ldpq;
  const size_t acc_elems = g.xcorr ? 0 : static_cast<size_t>(g.K) * g.CRS;
  float* col = static_cast<float*>(scratch_for(e.stream, (col_elems + acc_elems) * sizeof(float)));
  if (col == nullptr) return KX_ERR_NOMEM;
  // flipped filters accumulate the un-flipped gradient in scratch first
  float* dst = g.xcorr ? dw : col + col_elems;
  kx_exec ie = inner_exec(ex, e.stream);
  const float a_out = g.xcorr ? *alpha : 1.f;
  const float b_first = g.xcorr ? *beta : 0.f;
  bool first = true;
  for (int n0 = 0; n0 < g.N; n0 += nb) {
    const int cnt = g.N - n0 < nb ? g.N - n0 : nb;
    dim3 grid((g.PQ + 255) / 256 < 64 ? (g.PQ + 255) / 256 : 64, g.CRS, cnt);
    note_launch();
    im2col_tap_major<<<grid, 256, 0, e.stream>>>(x, col, g, n0);
    for (int i = 0; i < cnt; ++i) {
      // dW (CRS x K col-major, ld CRS) += colT_n (CRS x PQ) * dy_n^T (PQ x K)
      const float bb = first ? b_first : 1.f;
      int rc = kx_sgemm(&ie, KX_OP_T, KX_OP_N, g.CRS, g.K, g.PQ, &a_out,
                        col + static_cast<size_t>(i) * g.CRS * g.ldpq, g.ldpq,
                        dy + static_cast<size_t>(n0 + i) * g.K * g.PQ, g.PQ, &bb, dst, g.CRS);
      if (rc != KX_OK) return rc;
      first = false;
    }
  }
  if (!g.xcorr) {
    note_launch();
    flip_accumulate<<<grid_1d(acc_elems), 256, 0, e.stream>>>(dst, dw, g.K * g.C, g.R, g.S,
                                                              *alpha, *beta);
  }
  return finish_done(e);
}
