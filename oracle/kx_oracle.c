/*
 * kx_oracle.c — CPU restatement of the dense operators the kernel_intercept
 * shim captures.  TEST INFRASTRUCTURE ONLY: the parity tests, smoke() and the
 * CPU-baseline leg of bench.py call it as the checker.  Nothing in the
 * product path (libkx.so, libgpu_scheduler.so, the Python package) links or
 * calls it.
 *
 * Where the arithmetic lives in the reference: the shim forwards every
 * captured op to the closed NVIDIA libraries (cuBLAS 12.x / cuBLASLt / cuDNN 9;
 * the reference pins none beyond the sonames libcublas.so.12/.11 at
 * src/cublas_intercept.cpp:218-223 and the nvcr.io/nvidia/pytorch:25.09 image
 * at Dockerfile:2-8).  This file restates the published semantics of those
 * calls, reached through the reference's call sites:
 *   - cublasSgemm_v2 / cublasSgemmStridedBatched as issued by
 *     execute_cublas_operation (src/cublas_intercept.cpp:455-491), with the
 *     parameters of CublasGemmParams (include/gpu_capture.h:140-169):
 *     column-major C = alpha*op(A)*op(B) + beta*C, C not read when beta == 0.
 *   - cublasGemmEx with bf16/fp16 A, B, C and fp32 compute
 *     (src/cublas_intercept.cpp:886-952).
 *   - cublasLtMatmul (src/cublas_intercept.cpp:1319-1443): D = epi(alpha*AB +
 *     beta*C + bias) with the bias broadcast along columns.
 *   - cudnnConvolutionForward/BackwardData/BackwardFilter
 *     (src/cudnn_intercept.cpp:433-627): NCHW/KCRS cross-correlation with
 *     padding, stride and dilation from the convolution descriptor.
 *   - cudnnBatchNormalizationForwardTraining/Inference/Backward
 *     (src/cudnn_intercept.cpp:659-716; parameters of CudnnBatchNormParams,
 *     include/gpu_capture.h:120-138): spatial and per-activation modes,
 *     running averages with factor f, unbiased running variance, saved
 *     inverse std.
 *
 * Accumulation is in double precision; results are rounded once to the output
 * type, so the oracle is at least as accurate as the library it restates.
 * Parallelised with OpenMP over output columns / channels.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define KXO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------ helpers --- */

static float bf16_to_f32(uint16_t v) {
    uint32_t u = ((uint32_t)v) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan */
        uint16_t r = (uint16_t)(u >> 16);
        if (u & 0x007fffffu) r |= 0x40; /* keep nan quiet */
        return r;
    }
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb; /* round to nearest even */
    return (uint16_t)(u >> 16);
}

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else { /* subnormal */
            float f = ldexpf((float)man, -24);
            memcpy(&u, &f, 4);
            u |= sign;
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t f32_to_f16(float f) {
    /* round-to-nearest-even via double arithmetic on the magnitude */
    uint32_t u;
    memcpy(&u, &f, 4);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    float a = fabsf(f);
    if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
    if (a >= 65520.0f) return (uint16_t)(sign | 0x7c00u);
    if (a < ldexpf(1.0f, -14)) { /* subnormal range: quantum 2^-24 */
        double q = nearbyint((double)a * 16777216.0);
        return (uint16_t)(sign | (uint16_t)q);
    }
    int e;
    double m = frexp((double)a, &e); /* a = m*2^e, m in [0.5,1) */
    double scaled = nearbyint(m * 2048.0); /* 11 significant bits */
    if (scaled >= 2048.0) { scaled /= 2.0; e += 1; }
    uint32_t exp = (uint32_t)(e - 1 + 15);
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t man = (uint32_t)scaled - 1024u;
    return (uint16_t)(sign | (exp << 10) | man);
}

/* type codes follow cudaDataType_t: 0 = f32, 2 = f16, 14 = bf16 */
static double load_elem(const void* p, int type, size_t idx) {
    switch (type) {
    case 0: return (double)((const float*)p)[idx];
    case 2: return (double)f16_to_f32(((const uint16_t*)p)[idx]);
    case 14: return (double)bf16_to_f32(((const uint16_t*)p)[idx]);
    default: return NAN;
    }
}

static void store_elem(void* p, int type, size_t idx, double v) {
    switch (type) {
    case 0: ((float*)p)[idx] = (float)v; break;
    case 2: ((uint16_t*)p)[idx] = f32_to_f16((float)v); break;
    case 14: ((uint16_t*)p)[idx] = f32_to_bf16((float)v); break;
    default: break;
    }
}

KXO_API float kxo_bf16_to_f32(uint16_t v) { return bf16_to_f32(v); }
KXO_API uint16_t kxo_f32_to_bf16(float f) { return f32_to_bf16(f); }
KXO_API float kxo_f16_to_f32(uint16_t v) { return f16_to_f32(v); }
KXO_API uint16_t kxo_f32_to_f16(float f) { return f32_to_f16(f); }

KXO_API int kxo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

KXO_API void kxo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

static double gelu_tanh(double x) {
    /* cublasLt CUBLASLT_EPILOGUE_GELU uses the tanh approximation */
    const double k0 = 0.7978845608028654; /* sqrt(2/pi) */
    return 0.5 * x * (1.0 + tanh(k0 * (x + 0.044715 * x * x * x)));
}

/* ---------------------------------------------------------------- GEMM --- */

/*
 * Generic column-major GEMM, one batch.  op(A)[i,p] = A[i + p*lda] (N) or
 * A[p + i*lda] (T/C, real data); op(B)[p,j] = B[p + j*ldb] (N) or
 * B[j + p*ldb] (T/C).  D[i + j*ldd] = epi(alpha*sum + beta*C[i + j*ldc] + bias[i]).
 * C is not read when beta == 0 (BLAS convention).
 */
static void gemm_one(int transa, int transb, int m, int n, int k, double alpha,
                     const void* A, int Atype, long long lda, const void* B, int Btype,
                     long long ldb, double beta, const void* C, int Ctype, long long ldc,
                     void* D, int Dtype, long long ldd, int epilogue, const void* bias,
                     int bias_type) {
    int relu = (epilogue == 2 || epilogue == 6);
    int gelu = (epilogue == 32 || epilogue == 36);
    int has_bias = (epilogue == 4 || epilogue == 6 || epilogue == 36) && bias;
#pragma omp parallel for schedule(dynamic, 1)
    for (int j = 0; j < n; ++j) {
        double* acc = (double*)calloc((size_t)(m > 0 ? m : 1), sizeof(double));
        for (int p = 0; p < k; ++p) {
            double b = (transb == 0) ? load_elem(B, Btype, (size_t)p + (size_t)j * ldb)
                                     : load_elem(B, Btype, (size_t)j + (size_t)p * ldb);
            if (b == 0.0) continue;
            if (transa == 0) {
                size_t base = (size_t)p * lda;
                for (int i = 0; i < m; ++i) acc[i] += load_elem(A, Atype, base + i) * b;
            } else {
                for (int i = 0; i < m; ++i)
                    acc[i] += load_elem(A, Atype, (size_t)p + (size_t)i * lda) * b;
            }
        }
        for (int i = 0; i < m; ++i) {
            double v = alpha * acc[i];
            if (beta != 0.0) v += beta * load_elem(C, Ctype, (size_t)i + (size_t)j * ldc);
            if (has_bias) v += load_elem(bias, bias_type, (size_t)i);
            if (relu && v < 0.0) v = 0.0;
            if (gelu) v = gelu_tanh(v);
            store_elem(D, Dtype, (size_t)i + (size_t)j * ldd, v);
        }
        free(acc);
    }
}

static size_t type_size(int t) { return t == 0 ? 4 : 2; }

/* cublasSgemm_v2 semantics (src/cublas_intercept.cpp:461-471). */
KXO_API void kxo_sgemm(int transa, int transb, int m, int n, int k, float alpha,
                       const float* A, int lda, const float* B, int ldb, float beta,
                       float* C, int ldc) {
    gemm_one(transa, transb, m, n, k, alpha, A, 0, lda, B, 0, ldb, beta, C, 0, ldc, C, 0,
             ldc, 1, NULL, 0);
}

/* cublasSgemmStridedBatched semantics (src/cublas_intercept.cpp:478-490). */
KXO_API void kxo_sgemm_strided_batched(int transa, int transb, int m, int n, int k,
                                       float alpha, const float* A, int lda,
                                       long long strideA, const float* B, int ldb,
                                       long long strideB, float beta, float* C, int ldc,
                                       long long strideC, int batch) {
    for (int b = 0; b < batch; ++b)
        gemm_one(transa, transb, m, n, k, alpha, A + (size_t)b * strideA, 0, lda,
                 B + (size_t)b * strideB, 0, ldb, beta, C + (size_t)b * strideC, 0, ldc,
                 C + (size_t)b * strideC, 0, ldc, 1, NULL, 0);
}

/* cublasGemmStridedBatchedEx / cublasLtMatmul with typed operands. */
KXO_API void kxo_gemm_ex(int transa, int transb, int m, int n, int k, float alpha,
                         const void* A, int Atype, int lda, long long strideA, const void* B,
                         int Btype, int ldb, long long strideB, float beta, const void* C,
                         int Ctype, int ldc, long long strideC, void* D, int Dtype, int ldd,
                         long long strideD, int batch, int epilogue, const void* bias,
                         int bias_type) {
    for (int b = 0; b < batch; ++b) {
        const char* a = (const char*)A + (size_t)b * strideA * type_size(Atype);
        const char* bb = (const char*)B + (size_t)b * strideB * type_size(Btype);
        const char* c = C ? (const char*)C + (size_t)b * strideC * type_size(Ctype) : NULL;
        char* d = (char*)D + (size_t)b * strideD * type_size(Dtype);
        gemm_one(transa, transb, m, n, k, alpha, a, Atype, lda, bb, Btype, ldb, c ? beta : 0.0,
                 c, Ctype, ldc, d, Dtype, ldd, epilogue, bias, bias_type);
    }
}

/* ------------------------------------------------------- convolution --- */

typedef struct kxo_conv {
    int n, c, h, w, k, r, s, pad_h, pad_w, stride_h, stride_w, dil_h, dil_w, xcorr;
} kxo_conv;

static void conv_out(const kxo_conv* d, int* p, int* q) {
    *p = (d->h + 2 * d->pad_h - ((d->r - 1) * d->dil_h + 1)) / d->stride_h + 1;
    *q = (d->w + 2 * d->pad_w - ((d->s - 1) * d->dil_w + 1)) / d->stride_w + 1;
}

/* filter tap used for output offset (rr, ss): flipped for CUDNN_CONVOLUTION */
static size_t wtap(const kxo_conv* d, int kk, int cc, int rr, int ss) {
    int fr = d->xcorr ? rr : d->r - 1 - rr;
    int fs = d->xcorr ? ss : d->s - 1 - ss;
    return (((size_t)kk * d->c + cc) * d->r + fr) * d->s + fs;
}

/* cudnnConvolutionForward: y = alpha*conv(x,w) + beta*y. */
KXO_API void kxo_conv_fwd(const kxo_conv* d, float alpha, const float* x, const float* w,
                          float beta, float* y) {
    int P, Q;
    conv_out(d, &P, &Q);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int nn = 0; nn < d->n; ++nn)
        for (int kk = 0; kk < d->k; ++kk) {
            for (int p = 0; p < P; ++p)
                for (int q = 0; q < Q; ++q) {
                    double acc = 0.0;
                    for (int cc = 0; cc < d->c; ++cc)
                        for (int rr = 0; rr < d->r; ++rr) {
                            int hh = p * d->stride_h - d->pad_h + rr * d->dil_h;
                            if (hh < 0 || hh >= d->h) continue;
                            for (int ss = 0; ss < d->s; ++ss) {
                                int ww = q * d->stride_w - d->pad_w + ss * d->dil_w;
                                if (ww < 0 || ww >= d->w) continue;
                                acc += (double)x[(((size_t)nn * d->c + cc) * d->h + hh) * d->w + ww] *
                                       (double)w[wtap(d, kk, cc, rr, ss)];
                            }
                        }
                    size_t yi = (((size_t)nn * d->k + kk) * P + p) * Q + q;
                    double v = alpha * acc;
                    if (beta != 0.0) v += beta * (double)y[yi];
                    y[yi] = (float)v;
                }
        }
}

/* cudnnConvolutionBackwardData: dx = alpha*conv^T(w,dy) + beta*dx. */
KXO_API void kxo_conv_bwd_data(const kxo_conv* d, float alpha, const float* w,
                               const float* dy, float beta, float* dx) {
    int P, Q;
    conv_out(d, &P, &Q);
    size_t nx = (size_t)d->n * d->c * d->h * d->w;
    double* acc = (double*)calloc(nx ? nx : 1, sizeof(double));
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int nn = 0; nn < d->n; ++nn)
        for (int cc = 0; cc < d->c; ++cc) {
            double* a = acc + ((size_t)nn * d->c + cc) * d->h * d->w;
            for (int kk = 0; kk < d->k; ++kk)
                for (int p = 0; p < P; ++p)
                    for (int q = 0; q < Q; ++q) {
                        double g = dy[(((size_t)nn * d->k + kk) * P + p) * Q + q];
                        if (g == 0.0) continue;
                        for (int rr = 0; rr < d->r; ++rr) {
                            int hh = p * d->stride_h - d->pad_h + rr * d->dil_h;
                            if (hh < 0 || hh >= d->h) continue;
                            for (int ss = 0; ss < d->s; ++ss) {
                                int ww = q * d->stride_w - d->pad_w + ss * d->dil_w;
                                if (ww < 0 || ww >= d->w) continue;
                                a[(size_t)hh * d->w + ww] += g * (double)w[wtap(d, kk, cc, rr, ss)];
                            }
                        }
                    }
        }
    for (size_t i = 0; i < nx; ++i) {
        double v = alpha * acc[i];
        if (beta != 0.0) v += beta * (double)dx[i];
        dx[i] = (float)v;
    }
    free(acc);
}

/* cudnnConvolutionBackwardFilter: dw = alpha*corr(x,dy) + beta*dw. */
KXO_API void kxo_conv_bwd_filter(const kxo_conv* d, float alpha, const float* x,
                                 const float* dy, float beta, float* dw) {
    int P, Q;
    conv_out(d, &P, &Q);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int kk = 0; kk < d->k; ++kk)
        for (int cc = 0; cc < d->c; ++cc) {
            for (int rr = 0; rr < d->r; ++rr)
                for (int ss = 0; ss < d->s; ++ss) {
                    double acc = 0.0;
                    for (int nn = 0; nn < d->n; ++nn)
                        for (int p = 0; p < P; ++p) {
                            int hh = p * d->stride_h - d->pad_h + rr * d->dil_h;
                            if (hh < 0 || hh >= d->h) continue;
                            for (int q = 0; q < Q; ++q) {
                                int ww = q * d->stride_w - d->pad_w + ss * d->dil_w;
                                if (ww < 0 || ww >= d->w) continue;
                                acc += (double)dy[(((size_t)nn * d->k + kk) * P + p) * Q + q] *
                                       (double)x[(((size_t)nn * d->c + cc) * d->h + hh) * d->w + ww];
                            }
                        }
                    size_t wi = wtap(d, kk, cc, rr, ss);
                    double v = alpha * acc;
                    if (beta != 0.0) v += beta * (double)dw[wi];
                    dw[wi] = (float)v;
                }
        }
}

/* -------------------------------------------------------- batch norm --- */

/*
 * Parameter vectors have one entry per channel (spatial, mode 1) or per
 * (c,h,w) activation (per-activation, mode 0).  Statistics are over N (and
 * H,W in spatial mode).  Running variance uses the unbiased estimator
 * (count/(count-1)), as cuDNN documents; save_inv_var = 1/sqrt(var + eps)
 * with the biased batch variance.
 */
/* mode 0 = CUDNN_BATCHNORM_PER_ACTIVATION (one group per c,h,w); 1 =
 * CUDNN_BATCHNORM_SPATIAL and 2 = CUDNN_BATCHNORM_SPATIAL_PERSISTENT (the
 * same numbers: one group per channel over n,h,w). */
static void bn_geometry(int mode, int n, int c, int h, int w, int* groups, size_t* count) {
    if (mode != 0) { *groups = c; *count = (size_t)n * h * w; }
    else { *groups = c * h * w; *count = (size_t)n; }
}

static size_t bn_index(int mode, int c, int h, int w, int g, size_t t) {
    /* t-th element of statistics group g, NCHW contiguous */
    if (mode != 0) {
        size_t hw = (size_t)h * w;
        size_t nn = t / hw, sp = t % hw;
        return (nn * c + g) * hw + sp;
    }
    size_t chw = (size_t)c * h * w;
    return t * chw + g;
}

KXO_API void kxo_bn_fwd_training(int mode, float alpha, float beta, int n, int c, int h, int w,
                                 const float* x, float* y, const float* scale,
                                 const float* bias, double factor, float* running_mean,
                                 float* running_var, double eps, float* save_mean,
                                 float* save_inv_var) {
    int G;
    size_t cnt;
    bn_geometry(mode, n, c, h, w, &G, &cnt);
#pragma omp parallel for schedule(dynamic, 1)
    for (int g = 0; g < G; ++g) {
        double s = 0.0, ss = 0.0;
        for (size_t t = 0; t < cnt; ++t) s += x[bn_index(mode, c, h, w, g, t)];
        double mean = s / (double)cnt;
        for (size_t t = 0; t < cnt; ++t) {
            double dlt = x[bn_index(mode, c, h, w, g, t)] - mean;
            ss += dlt * dlt;
        }
        double var = ss / (double)cnt;
        double inv = 1.0 / sqrt(var + eps);
        for (size_t t = 0; t < cnt; ++t) {
            size_t i = bn_index(mode, c, h, w, g, t);
            double v = alpha * ((x[i] - mean) * inv * scale[g] + bias[g]);
            if (beta != 0.0) v += beta * (double)y[i];
            y[i] = (float)v;
        }
        if (running_mean && running_var) {
            double unb = cnt > 1 ? var * (double)cnt / (double)(cnt - 1) : var;
            running_mean[g] = (float)((1.0 - factor) * running_mean[g] + factor * mean);
            running_var[g] = (float)((1.0 - factor) * running_var[g] + factor * unb);
        }
        if (save_mean) save_mean[g] = (float)mean;
        if (save_inv_var) save_inv_var[g] = (float)inv;
    }
}

KXO_API void kxo_bn_fwd_inference(int mode, float alpha, float beta, int n, int c, int h, int w,
                                  const float* x, float* y, const float* scale,
                                  const float* bias, const float* est_mean,
                                  const float* est_var, double eps) {
    int G;
    size_t cnt;
    bn_geometry(mode, n, c, h, w, &G, &cnt);
#pragma omp parallel for schedule(dynamic, 1)
    for (int g = 0; g < G; ++g) {
        double inv = 1.0 / sqrt((double)est_var[g] + eps);
        for (size_t t = 0; t < cnt; ++t) {
            size_t i = bn_index(mode, c, h, w, g, t);
            double v = alpha * ((x[i] - (double)est_mean[g]) * inv * scale[g] + bias[g]);
            if (beta != 0.0) v += beta * (double)y[i];
            y[i] = (float)v;
        }
    }
}

KXO_API void kxo_bn_bwd(int mode, float alpha_d, float beta_d, float alpha_p, float beta_p,
                        int n, int c, int h, int w, const float* x, const float* dy, float* dx,
                        const float* scale, float* dscale, float* dbias, double eps,
                        const float* save_mean, const float* save_inv_var) {
    int G;
    size_t cnt;
    bn_geometry(mode, n, c, h, w, &G, &cnt);
#pragma omp parallel for schedule(dynamic, 1)
    for (int g = 0; g < G; ++g) {
        double mean, inv;
        if (save_mean && save_inv_var) {
            mean = save_mean[g];
            inv = save_inv_var[g];
        } else {
            double s = 0.0, ss = 0.0;
            for (size_t t = 0; t < cnt; ++t) s += x[bn_index(mode, c, h, w, g, t)];
            mean = s / (double)cnt;
            for (size_t t = 0; t < cnt; ++t) {
                double dlt = x[bn_index(mode, c, h, w, g, t)] - mean;
                ss += dlt * dlt;
            }
            inv = 1.0 / sqrt(ss / (double)cnt + eps);
        }
        double sdy = 0.0, sdyx = 0.0;
        for (size_t t = 0; t < cnt; ++t) {
            size_t i = bn_index(mode, c, h, w, g, t);
            double xh = (x[i] - mean) * inv;
            sdy += dy[i];
            sdyx += dy[i] * xh;
        }
        for (size_t t = 0; t < cnt; ++t) {
            size_t i = bn_index(mode, c, h, w, g, t);
            double xh = (x[i] - mean) * inv;
            double v = (double)scale[g] * inv / (double)cnt *
                       ((double)cnt * dy[i] - sdy - xh * sdyx);
            double o = alpha_d * v;
            if (beta_d != 0.0) o += beta_d * (double)dx[i];
            dx[i] = (float)o;
        }
        double ds = alpha_p * sdyx, db = alpha_p * sdy;
        if (beta_p != 0.0) { ds += beta_p * (double)dscale[g]; db += beta_p * (double)dbias[g]; }
        dscale[g] = (float)ds;
        dbias[g] = (float)db;
    }
}
