// kx_bn.cu — batch normalisation (cudnnBatchNormalization* replacements).
//
// HBM-bound kernels: per-channel statistics in one read of x (shifted sums,
// fp32 per thread, fp64 across threads/blocks), then one fused
// normalise/affine/alpha-beta pass (read x, read y when beta != 0, write y).
// Loads are 128-bit when the spatial extent allows it.  Spatial mode groups
// statistics per channel over N*H*W; per-activation mode per (c,h,w) over N.
// Reference call sites: src/cudnn_intercept.cpp:659-716 (forward training),
// declared inference/backward types at src/cudnn_intercept.cpp:112-143.
#include <cstring>

#include "kx_runtime.cuh"

namespace kx {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 4096;  // elements of one (n, c) row handled per work item

__device__ double block_sum(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < (blockDim.x >> 5)) t = sh[threadIdx.x];
  if (w == 0)
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;  // valid in thread 0
}

// Spatial statistics: block (c, s) accumulates sum(x-K) and sum((x-K)^2) over
// the work items s, s+S, ... of channel c, where K = x[0, c, 0] is a shift
// that keeps the second moment free of cancellation.
__global__ void __launch_bounds__(kThreads) bn_stats_spatial(const float* __restrict__ x, int N,
                                                              int C, int HW, int S, bool vec,
                                                              double* __restrict__ part) {
  __shared__ double sh[kThreads / 32];
  const int c = blockIdx.x, s = blockIdx.y;
  const float K = x[static_cast<size_t>(c) * HW];
  const int chunks = (HW + kChunk - 1) / kChunk;
  const long long items = static_cast<long long>(N) * chunks;
  float s1 = 0.f, s2 = 0.f;
  for (long long it = s; it < items; it += S) {
    const int n = static_cast<int>(it / chunks), ch = static_cast<int>(it % chunks);
    const float* row = x + (static_cast<size_t>(n) * C + c) * HW;
    const int lo = ch * kChunk, hi = min(HW, lo + kChunk);
    if (vec) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (int i = (lo >> 2) + threadIdx.x; i < (hi >> 2); i += kThreads) {
        float4 v = __ldg(r4 + i);
        float a = v.x - K, b = v.y - K, cc = v.z - K, d = v.w - K;
        s1 += (a + b) + (cc + d);
        s2 += (a * a + b * b) + (cc * cc + d * d);
      }
    } else {
      for (int i = lo + threadIdx.x; i < hi; i += kThreads) {
        float a = __ldg(row + i) - K;
        s1 += a;
        s2 += a * a;
      }
    }
  }
  double t1 = block_sum(static_cast<double>(s1), sh);
  double t2 = block_sum(static_cast<double>(s2), sh);
  if (threadIdx.x == 0) {
    part[(static_cast<size_t>(c) * S + s) * 2 + 0] = t1;
    part[(static_cast<size_t>(c) * S + s) * 2 + 1] = t2;
  }
}

// One thread per channel: combine partials, update running statistics, save
// mean / inverse std, and emit the affine coefficients y = a*x + b.
__global__ void bn_finalize_spatial(const float* __restrict__ x, int N, int C, int HW, int S,
                                    const double* __restrict__ part, const float* scale,
                                    const float* bias, double factor, float* running_mean,
                                    float* running_var, double eps, float* save_mean,
                                    float* save_inv_var, float2* coef) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double s1 = 0.0, s2 = 0.0;
  for (int s = 0; s < S; ++s) {
    s1 += part[(static_cast<size_t>(c) * S + s) * 2];
    s2 += part[(static_cast<size_t>(c) * S + s) * 2 + 1];
  }
  const double cnt = static_cast<double>(N) * HW;
  const double K = x[static_cast<size_t>(c) * HW];
  const double dm = s1 / cnt;
  double var = s2 / cnt - dm * dm;
  if (var < 0.0) var = 0.0;
  const double mean = K + dm;
  const double inv = 1.0 / sqrt(var + eps);
  if (running_mean != nullptr && running_var != nullptr) {
    const double unb = cnt > 1.0 ? var * cnt / (cnt - 1.0) : var;
    running_mean[c] = static_cast<float>((1.0 - factor) * running_mean[c] + factor * mean);
    running_var[c] = static_cast<float>((1.0 - factor) * running_var[c] + factor * unb);
  }
  if (save_mean != nullptr) save_mean[c] = static_cast<float>(mean);
  if (save_inv_var != nullptr) save_inv_var[c] = static_cast<float>(inv);
  const double a = static_cast<double>(scale[c]) * inv;
  coef[c] = make_float2(static_cast<float>(a), static_cast<float>(bias[c] - mean * a));
}

// y = alpha*(a_c*x + b_c) + beta*y over rows (n, c) of HW elements.
__global__ void __launch_bounds__(kThreads) bn_apply_spatial(const float* __restrict__ x, float* y,
                                                              int C, int HW, long long rows,
                                                              bool vec,
                                                              const float2* __restrict__ coef,
                                                              float alpha, float beta) {
  for (long long row = blockIdx.y; row < rows; row += gridDim.y) {
    const float2 ab = coef[row % C];
    const float a = alpha * ab.x, b = alpha * ab.y;
    const float* xr = x + row * HW;
    float* yr = y + row * HW;
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      float4* y4 = reinterpret_cast<float4*>(yr);
      for (int i = blockIdx.x * kThreads + threadIdx.x; i < (HW >> 2); i += gridDim.x * kThreads) {
        float4 v = __ldg(x4 + i);
        float4 o = make_float4(fmaf(a, v.x, b), fmaf(a, v.y, b), fmaf(a, v.z, b), fmaf(a, v.w, b));
        if (beta != 0.f) {
          float4 p = y4[i];
          o.x = fmaf(beta, p.x, o.x); o.y = fmaf(beta, p.y, o.y);
          o.z = fmaf(beta, p.z, o.z); o.w = fmaf(beta, p.w, o.w);
        }
        y4[i] = o;
      }
    } else {
      for (int i = blockIdx.x * kThreads + threadIdx.x; i < HW; i += gridDim.x * kThreads) {
        float o = fmaf(a, __ldg(xr + i), b);
        if (beta != 0.f) o = fmaf(beta, yr[i], o);
        yr[i] = o;
      }
    }
  }
}

// Per-activation mode: one thread per feature g (of G = C*H*W), samples at
// stride G.  Statistics + coefficients in one kernel.
__global__ void bn_stats_per_activation(const float* __restrict__ x, int N, int G,
                                        const float* scale, const float* bias, double factor,
                                        float* running_mean, float* running_var, double eps,
                                        float* save_mean, float* save_inv_var, float2* coef,
                                        const float* est_mean, const float* est_var) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  double mean, var;
  if (est_mean != nullptr) {
    mean = est_mean[g];
    var = est_var[g];
  } else {
    const float K = x[g];
    double s1 = 0.0, s2 = 0.0;
    for (int n = 0; n < N; ++n) {
      const double d = static_cast<double>(x[static_cast<size_t>(n) * G + g]) - K;
      s1 += d;
      s2 += d * d;
    }
    const double dm = s1 / N;
    var = s2 / N - dm * dm;
    if (var < 0.0) var = 0.0;
    mean = K + dm;
    if (running_mean != nullptr && running_var != nullptr) {
      const double unb = N > 1 ? var * N / (N - 1.0) : var;
      running_mean[g] = static_cast<float>((1.0 - factor) * running_mean[g] + factor * mean);
      running_var[g] = static_cast<float>((1.0 - factor) * running_var[g] + factor * unb);
    }
  }
  const double inv = 1.0 / sqrt(var + eps);
  if (save_mean != nullptr) save_mean[g] = static_cast<float>(mean);
  if (save_inv_var != nullptr) save_inv_var[g] = static_cast<float>(inv);
  const double a = static_cast<double>(scale[g]) * inv;
  coef[g] = make_float2(static_cast<float>(a), static_cast<float>(bias[g] - mean * a));
}

__global__ void bn_apply_per_activation(const float* __restrict__ x, float* y, int N, int G,
                                        const float2* __restrict__ coef, float alpha, float beta) {
  const size_t total = static_cast<size_t>(N) * G;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float2 ab = coef[i % G];
    float o = alpha * fmaf(ab.x, x[i], ab.y);
    if (beta != 0.f) o = fmaf(beta, y[i], o);
    y[i] = o;
  }
}

// ---- backward --------------------------------------------------------------

// Partials of sum(dy) and sum(dy * (x - mean)) per channel (spatial mode).
__global__ void __launch_bounds__(kThreads) bn_bwd_reduce_spatial(
    const float* __restrict__ x, const float* __restrict__ dy, int N, int C, int HW, int S,
    bool vec, const float* __restrict__ mean_c, double* __restrict__ part) {
  __shared__ double sh[kThreads / 32];
  const int c = blockIdx.x, s = blockIdx.y;
  const float mu = mean_c[c];
  const int chunks = (HW + kChunk - 1) / kChunk;
  const long long items = static_cast<long long>(N) * chunks;
  float sd = 0.f, sdx = 0.f;
  for (long long it = s; it < items; it += S) {
    const int n = static_cast<int>(it / chunks), ch = static_cast<int>(it % chunks);
    const size_t off = (static_cast<size_t>(n) * C + c) * HW;
    const int lo = ch * kChunk, hi = min(HW, lo + kChunk);
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(x + off);
      const float4* d4 = reinterpret_cast<const float4*>(dy + off);
      for (int i = (lo >> 2) + threadIdx.x; i < (hi >> 2); i += kThreads) {
        float4 a = __ldg(x4 + i), g = __ldg(d4 + i);
        sd += (g.x + g.y) + (g.z + g.w);
        sdx += (g.x * (a.x - mu) + g.y * (a.y - mu)) + (g.z * (a.z - mu) + g.w * (a.w - mu));
      }
    } else {
      for (int i = lo + threadIdx.x; i < hi; i += kThreads) {
        float g = __ldg(dy + off + i);
        sd += g;
        sdx += g * (__ldg(x + off + i) - mu);
      }
    }
  }
  double t1 = block_sum(static_cast<double>(sd), sh);
  double t2 = block_sum(static_cast<double>(sdx), sh);
  if (threadIdx.x == 0) {
    part[(static_cast<size_t>(c) * S + s) * 2 + 0] = t1;
    part[(static_cast<size_t>(c) * S + s) * 2 + 1] = t2;
  }
}

// dscale / dbias, and dx = k1*dy + k2*x + k3 coefficients per channel.
__global__ void bn_bwd_finalize(int G, double cnt, int S, const double* __restrict__ part,
                                const float* mean_c, const float* inv_c, const float* scale,
                                float* dscale, float* dbias, float alpha_p, float beta_p,
                                float4* coef) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  double sd = 0.0, sdx = 0.0;
  for (int s = 0; s < S; ++s) {
    sd += part[(static_cast<size_t>(g) * S + s) * 2];
    sdx += part[(static_cast<size_t>(g) * S + s) * 2 + 1];
  }
  const double inv = inv_c[g], mu = mean_c[g], sc = scale[g];
  const double sdxh = sdx * inv;  // sum(dy * xhat)
  double ds = alpha_p * sdxh, db = alpha_p * sd;
  if (beta_p != 0.f) {
    ds += static_cast<double>(beta_p) * dscale[g];
    db += static_cast<double>(beta_p) * dbias[g];
  }
  dscale[g] = static_cast<float>(ds);
  dbias[g] = static_cast<float>(db);
  const double k1 = sc * inv;
  const double k2 = -sc * inv * inv * sdxh / cnt;
  const double k3 = -sc * inv * sd / cnt - k2 * mu;
  coef[g] = make_float4(static_cast<float>(k1), static_cast<float>(k2), static_cast<float>(k3), 0.f);
}

__global__ void __launch_bounds__(kThreads) bn_bwd_apply_spatial(
    const float* __restrict__ x, const float* __restrict__ dy, float* dx, int C, int HW,
    long long rows, bool vec, const float4* __restrict__ coef, float alpha, float beta) {
  for (long long row = blockIdx.y; row < rows; row += gridDim.y) {
    const float4 k = coef[row % C];
    const float k1 = alpha * k.x, k2 = alpha * k.y, k3 = alpha * k.z;
    const size_t off = static_cast<size_t>(row) * HW;
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(x + off);
      const float4* d4 = reinterpret_cast<const float4*>(dy + off);
      float4* o4 = reinterpret_cast<float4*>(dx + off);
      for (int i = blockIdx.x * kThreads + threadIdx.x; i < (HW >> 2); i += gridDim.x * kThreads) {
        float4 a = __ldg(x4 + i), g = __ldg(d4 + i);
        float4 o = make_float4(fmaf(k1, g.x, fmaf(k2, a.x, k3)), fmaf(k1, g.y, fmaf(k2, a.y, k3)),
                               fmaf(k1, g.z, fmaf(k2, a.z, k3)), fmaf(k1, g.w, fmaf(k2, a.w, k3)));
        if (beta != 0.f) {
          float4 p = o4[i];
          o.x = fmaf(beta, p.x, o.x); o.y = fmaf(beta, p.y, o.y);
          o.z = fmaf(beta, p.z, o.z); o.w = fmaf(beta, p.w, o.w);
        }
        o4[i] = o;
      }
    } else {
      for (int i = blockIdx.x * kThreads + threadIdx.x; i < HW; i += gridDim.x * kThreads) {
        float o = fmaf(k1, dy[off + i], fmaf(k2, x[off + i], k3));
        if (beta != 0.f) o = fmaf(beta, dx[off + i], o);
        dx[off + i] = o;
      }
    }
  }
}

__global__ void bn_bwd_per_activation(const float* __restrict__ x, const float* __restrict__ dy,
                                      float* dx, int N, int G, const float* mean_g,
                                      const float* inv_g, const float* scale, float* dscale,
                                      float* dbias, float alpha_d, float beta_d, float alpha_p,
                                      float beta_p) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  const double mu = mean_g[g], inv = inv_g[g], sc = scale[g];
  double sd = 0.0, sdx = 0.0;
  for (int n = 0; n < N; ++n) {
    const size_t i = static_cast<size_t>(n) * G + g;
    sd += dy[i];
    sdx += static_cast<double>(dy[i]) * (x[i] - mu);
  }
  const double sdxh = sdx * inv;
  const double k1 = sc * inv, k2 = -sc * inv * inv * sdxh / N, k3 = -sc * inv * sd / N - k2 * mu;
  for (int n = 0; n < N; ++n) {
    const size_t i = static_cast<size_t>(n) * G + g;
    double o = alpha_d * (k1 * dy[i] + k2 * x[i] + k3);
    if (beta_d != 0.f) o += static_cast<double>(beta_d) * dx[i];
    dx[i] = static_cast<float>(o);
  }
  double ds = alpha_p * sdxh, db = alpha_p * sd;
  if (beta_p != 0.f) {
    ds += static_cast<double>(beta_p) * dscale[g];
    db += static_cast<double>(beta_p) * dbias[g];
  }
  dscale[g] = static_cast<float>(ds);
  dbias[g] = static_cast<float>(db);
}

int split_for(long long per_channel, int channels) {
  // enough blocks to cover ~4 waves of the device, never more than work items
  const int sms = device_info().num_sms;
  long long want = (4LL * sms + channels - 1) / channels;
  long long items = (per_channel + kChunk - 1) / kChunk;
  if (want > items) want = items;
  if (want < 1) want = 1;
  if (want > 1024) want = 1024;
  return static_cast<int>(want);
}

dim3 apply_grid(long long rows, int HW) {
  const int sms = device_info().num_sms;
  int gx = (((HW + 3) / 4) + kThreads - 1) / kThreads;
  if (gx < 1) gx = 1;
  long long gy = rows;
  long long cap = (8LL * sms + gx - 1) / gx;
  if (cap < 1) cap = 1;
  if (gy > cap) gy = cap;
  if (gy > 65535) gy = 65535;
  return dim3(gx, static_cast<unsigned>(gy));
}

// 128-bit loads and stores need every (n, c) row to start on a 16-byte
// boundary: HW a multiple of 4 floats and each tensor's base 16-byte aligned
// (cuDNN accepts any 4-byte aligned pointer, e.g. a view with a storage offset).
bool vec_ok(int HW, const void* a, const void* b = nullptr, const void* c = nullptr) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(c);
  return (HW & 3) == 0 && (bits & 15u) == 0;
}

// Sizes are ints in the ABI; c*h*w (one sample, the per-activation feature
// count) must also fit one, since the kernels index features with it.
bool bad_dims(int n, int c, int h, int w) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return true;
  return static_cast<long long>(c) * h * w > 0x7fffffffLL;
}

}  // namespace
}  // namespace kx

using namespace kx;

extern "C" int kx_bn_fwd_training(const kx_exec* ex, int mode, const float* alpha,
                                  const float* beta, int n, int c, int h, int w, const float* x,
                                  float* y, const float* scale, const float* bias,
                                  double exp_avg_factor, float* running_mean, float* running_var,
                                  double eps, float* save_mean, float* save_inv_var) {
  if (bad_dims(n, c, h, w) || !x || !y || !scale || !bias || !alpha || !beta) return KX_ERR_INVALID;
  if (mode != 0 && mode != 1 && mode != 2) return KX_ERR_UNSUPPORTED;
  Exec e = resolve_exec(ex);
  const int HW = h * w;
  if (mode == 0) {
    const int G = c * HW;
    float2* coef = static_cast<float2*>(scratch_for(e.stream, sizeof(float2) * G));
    if (!coef) return KX_ERR_NOMEM;
    note_launch();
    bn_stats_per_activation<<<(G + 255) / 256, 256, 0, e.stream>>>(
        x, n, G, scale, bias, exp_avg_factor, running_mean, running_var, eps, save_mean,
        save_inv_var, coef, nullptr, nullptr);
    const size_t total = static_cast<size_t>(n) * G;
    int blocks = static_cast<int>((total + 255) / 256 < 8u * device_info().num_sms ? (total + 255) / 256 : 8u * device_info().num_sms);
    note_launch();
    bn_apply_per_activation<<<blocks, 256, 0, e.stream>>>(x, y, n, G, coef, *alpha, *beta);
    set_last_kernel_name("kx_bn_apply_per_activation");
    return launch_status();
  }
  // spatial (mode 1) and persistent-spatial (mode 2, same numbers)
  const int S = split_for(static_cast<long long>(n) * HW, c);
  const size_t part_bytes = sizeof(double) * 2 * static_cast<size_t>(c) * S;
  char* base = static_cast<char*>(scratch_for(e.stream, part_bytes + sizeof(float2) * c + 256));
  if (!base) return KX_ERR_NOMEM;
  double* part = reinterpret_cast<double*>(base);
  float2* coef = reinterpret_cast<float2*>(base + ((part_bytes + 255) & ~static_cast<size_t>(255)));
  note_launch();
  bn_stats_spatial<<<dim3(c, S), kThreads, 0, e.stream>>>(x, n, c, HW, S, vec_ok(HW, x),
                                                           part);
  note_launch();
  bn_finalize_spatial<<<(c + 127) / 128, 128, 0, e.stream>>>(x, n, c, HW, S, part, scale, bias,
                                                             exp_avg_factor, running_mean,
                                                             running_var, eps, save_mean,
                                                             save_inv_var, coef);
  const long long rows = static_cast<long long>(n) * c;
  note_launch();
  bn_apply_spatial<<<apply_grid(rows, HW), kThreads, 0, e.stream>>>(
      x, y, c, HW, rows, vec_ok(HW, x, y), coef, *alpha, *beta);
  set_last_kernel_name("kx_bn_apply_spatial");
  return launch_status();
}

extern "C" int kx_bn_fwd_inference(const kx_exec* ex, int mode, const float* alpha,
                                   const float* beta, int n, int c, int h, int w, const float* x,
                                   float* y, const float* scale, const float* bias,
                                   const float* est_mean, const float* est_var, double eps) {
  if (bad_dims(n, c, h, w) || !x || !y || !scale || !bias || !est_mean || !est_var || !alpha ||
      !beta)
    return KX_ERR_INVALID;
  if (mode != 0 && mode != 1 && mode != 2) return KX_ERR_UNSUPPORTED;
  Exec e = resolve_exec(ex);
  const int HW = h * w;
  const int G = mode == 0 ? c * HW : c;
  float2* coef = static_cast<float2*>(scratch_for(e.stream, sizeof(float2) * G));
  if (!coef) return KX_ERR_NOMEM;
  note_launch();
  bn_stats_per_activation<<<(G + 255) / 256, 256, 0, e.stream>>>(
      x, n, G, scale, bias, 0.0, nullptr, nullptr, eps, nullptr, nullptr, coef, est_mean, est_var);
  if (mode == 0) {
    const size_t total = static_cast<size_t>(n) * G;
    int blocks = static_cast<int>((total + 255) / 256 < 8u * device_info().num_sms ? (total + 255) / 256 : 8u * device_info().num_sms);
    note_launch();
    bn_apply_per_activation<<<blocks, 256, 0, e.stream>>>(x, y, n, G, coef, *alpha, *beta);
  } else {
    const long long rows = static_cast<long long>(n) * c;
    note_launch();
    bn_apply_spatial<<<apply_grid(rows, HW), kThreads, 0, e.stream>>>(
        x, y, c, HW, rows, vec_ok(HW, x, y), coef, *alpha, *beta);
  }
  set_last_kernel_name("kx_bn_fwd_inference");
  return launch_status();
}

extern "C" int kx_bn_bwd(const kx_exec* ex, int mode, const float* alpha_data,
                         const float* beta_data, const float* alpha_param, const float* beta_param,
                         int n, int c, int h, int w, const float* x, const float* dy, float* dx,
                         const float* scale, float* dscale, float* dbias, double eps,
                         const float* save_mean, const float* save_inv_var) {
  if (bad_dims(n, c, h, w) || !x || !dy || !dx || !scale || !dscale || !dbias || !alpha_data ||
      !beta_data || !alpha_param || !beta_param)
    return KX_ERR_INVALID;
  if (mode != 0 && mode != 1 && mode != 2) return KX_ERR_UNSUPPORTED;
  Exec e = resolve_exec(ex);
  const int HW = h * w;
  const int G = mode == 0 ? c * HW : c;
  // saved statistics, or recomputed ones (cuDNN allows null savedMean/savedInvVariance)
  const int S = mode == 0 ? 1 : split_for(static_cast<long long>(n) * HW, c);
  const size_t stats_bytes = sizeof(float) * 2 * static_cast<size_t>(G);
  const size_t part_bytes = sizeof(double) * 2 * static_cast<size_t>(G) * S;
  const size_t coef_bytes = sizeof(float4) * static_cast<size_t>(G);
  auto r256 = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
  char* base = static_cast<char*>(scratch_for(e.stream, r256(stats_bytes) + r256(part_bytes) +
                                                            r256(coef_bytes) +
                                                            sizeof(float2) * G + 256));
  if (!base) return KX_ERR_NOMEM;
  float* mean_g = reinterpret_cast<float*>(base);
  float* inv_g = mean_g + G;
  double* part = reinterpret_cast<double*>(base + r256(stats_bytes));
  float4* coef = reinterpret_cast<float4*>(base + r256(stats_bytes) + r256(part_bytes));
  float2* fcoef = reinterpret_cast<float2*>(base + r256(stats_bytes) + r256(part_bytes) +
                                            r256(coef_bytes));
  const float* mu = save_mean;
  const float* iv = save_inv_var;
  if (mu == nullptr || iv == nullptr) {
    // recompute batch statistics into scratch (scale/bias only feed fcoef)
    if (mode == 0) {
      note_launch();
      bn_stats_per_activation<<<(G + 255) / 256, 256, 0, e.stream>>>(
          x, n, G, scale, scale, 0.0, nullptr, nullptr, eps, mean_g, inv_g, fcoef, nullptr,
          nullptr);
    } else {
      note_launch();
      bn_stats_spatial<<<dim3(c, S), kThreads, 0, e.stream>>>(x, n, c, HW, S, vec_ok(HW, x),
                                                           part);
      note_launch();
      bn_finalize_spatial<<<(c + 127) / 128, 128, 0, e.stream>>>(
          x, n, c, HW, S, part, scale, scale, 0.0, nullptr, nullptr, eps, mean_g, inv_g, fcoef);
    }
    mu = mean_g;
    iv = inv_g;
  }
  if (mode == 0) {
    note_launch();
    bn_bwd_per_activation<<<(G + 255) / 256, 256, 0, e.stream>>>(
        x, dy, dx, n, G, mu, iv, scale, dscale, dbias, *alpha_data, *beta_data, *alpha_param,
        *beta_param);
  } else {
    note_launch();
    bn_bwd_reduce_spatial<<<dim3(c, S), kThreads, 0, e.stream>>>(
        x, dy, n, c, HW, S, vec_ok(HW, x, dy), mu, part);
    note_launch();
    bn_bwd_finalize<<<(c + 127) / 128, 128, 0, e.stream>>>(
        c, static_cast<double>(n) * HW, S, part, mu, iv, scale, dscale, dbias, *alpha_param,
        *beta_param, coef);
    const long long rows = static_cast<long long>(n) * c;
    note_launch();
    bn_bwd_apply_spatial<<<apply_grid(rows, HW), kThreads, 0, e.stream>>>(
        x, dy, dx, c, HW, rows, vec_ok(HW, x, dy, dx), coef, *alpha_data, *beta_data);
  }
  set_last_kernel_name("kx_bn_bwd");
  return launch_status();
}

// ------------------------------------------------ allocation-free variant --
//
// kx_bn_fwd_training_noalloc: the same computation as kx_bn_fwd_training, for
// callers that cannot allocate device memory.  Its statistics scratch is the
// file-scope array below (kNoAllocScratchBytes = 4 MiB per device) instead of
// the stream's scratch arena; nothing in this path calls cudaMalloc,
// cudaFree or any allocating routine.  Every call shares the one array, so
// calls whose kernels overlap on the GPU (other streams, other host threads)
// race on it; callers serialise them.  No part of the array has to start at
// zero: every call writes all the scratch it reads (per-block partial sums,
// then per-channel coefficients) before reading it.

namespace kx {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
__device__ __align__(256) unsigned char g_bn_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of the array on the device that runs `stream`, looked up
// once per device with that device current.  The stream must belong to the
// current device (the launches below go to the current device's copy of the
// array); any other stream is rejected with KX_ERR_INVALID.
int noalloc_scratch(cudaStream_t stream, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KX_ERR_DEVICE;
  if (stream != nullptr) {
    int sdev = -1;
    if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) {
      cudaGetLastError();
      return KX_ERR_INVALID;
    }
    if (sdev != dev) return KX_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bn_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();
      return KX_ERR_DEVICE;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return KX_OK;
}

}  // namespace
}  // namespace kx

extern "C" int kx_bn_fwd_training_noalloc(const kx_exec* ex, int mode, const float* alpha,
                                          const float* beta, int n, int c, int h, int w,
                                          const float* x, float* y, const float* scale,
                                          const float* bias, double exp_avg_factor,
                                          float* running_mean, float* running_var, double eps,
                                          float* save_mean, float* save_inv_var) {
  if (bad_dims(n, c, h, w) || !x || !y || !scale || !bias || !alpha || !beta) return KX_ERR_INVALID;
  if (mode != 0 && mode != 1 && mode != 2) return KX_ERR_UNSUPPORTED;
  Exec e = resolve_exec(ex);
  // sizes in 64 bits (bad_dims has bounded c*h*w by INT_MAX, so HW fits an int)
  const long long hw64 = static_cast<long long>(h) * w;
  const int HW = static_cast<int>(hw64);
  // scratch this call needs; more than the array holds is rejected
  const int S = mode == 0 ? 0 : split_for(static_cast<long long>(n) * hw64, c);
  const size_t part_bytes = sizeof(double) * 2 * static_cast<size_t>(c) * S;
  const size_t coef_off = (part_bytes + 255) & ~static_cast<size_t>(255);
  const size_t need = mode == 0 ? sizeof(float2) * static_cast<size_t>(c) * hw64
                                : coef_off + sizeof(float2) * static_cast<size_t>(c);
  if (need > kNoAllocScratchBytes) return KX_ERR_INVALID;
  void* vbase = nullptr;
  const int st = noalloc_scratch(e.stream, &vbase);
  if (st != KX_OK) return st;
  char* base = static_cast<char*>(vbase);
  if (mode == 0) {
    const int G = c * HW;
    float2* coef = reinterpret_cast<float2*>(base);
    note_launch();
    bn_stats_per_activation<<<(G + 255) / 256, 256, 0, e.stream>>>(
        x, n, G, scale, bias, exp_avg_factor, running_mean, running_var, eps, save_mean,
        save_inv_var, coef, nullptr, nullptr);
    const size_t total = static_cast<size_t>(n) * G;
    const size_t cap = 8u * device_info().num_sms;
    const int blocks = static_cast<int>((total + 255) / 256 < cap ? (total + 255) / 256 : cap);
    note_launch();
    bn_apply_per_activation<<<blocks, 256, 0, e.stream>>>(x, y, n, G, coef, *alpha, *beta);
    set_last_kernel_name("kx_bn_apply_per_activation");
    return launch_status();
  }
  double* part = reinterpret_cast<double*>(base);
  float2* coef = reinterpret_cast<float2*>(base + coef_off);
  note_launch();
  bn_stats_spatial<<<dim3(c, S), kThreads, 0, e.stream>>>(x, n, c, HW, S, vec_ok(HW, x),
                                                           part);
  note_launch();
  bn_finalize_spatial<<<(c + 127) / 128, 128, 0, e.stream>>>(x, n, c, HW, S, part, scale, bias,
                                                             exp_avg_factor, running_mean,
                                                             running_var, eps, save_mean,
                                                             save_inv_var, coef);
  const long long rows = static_cast<long long>(n) * c;
  note_launch();
  bn_apply_spatial<<<apply_grid(rows, HW), kThreads, 0, e.stream>>>(
      x, y, c, HW, rows, vec_ok(HW, x, y), coef, *alpha, *beta);
  set_last_kernel_name("kx_bn_apply_spatial");
  return launch_status();
}
