// util.cu -- small device kernels the calibration drivers compose:
// column statistics, the smoothing vector, row/column gathers, deterministic
// reductions, argsort of a vector, dtype casts, refinement set-up.
// Reductions are two-pass through a caller-provided workspace so results are
// run-to-run deterministic (no float atomics).
#include <algorithm>

#include "common.cuh"

namespace hif4x {

constexpr int UT = 256;
constexpr int kRowChunks = 64;

// partial[ch][c] = sum_{r in chunk ch} |X[r][c]|
__global__ void col_abs_partial_kernel(const float *X, int64_t R, int64_t C, float *partial) {
  const int64_t c = (int64_t)blockIdx.x * UT + threadIdx.x;
  const int ch = blockIdx.y;
  if (c >= C) return;
  const int64_t rows_per = (R + kRowChunks - 1) / kRowChunks;
  const int64_t r0 = ch * rows_per, r1 = min(R, r0 + rows_per);
  float s = 0.0f;
  for (int64_t r = r0; r < r1; r++) s += fabsf(X[r * C + c]);
  partial[(int64_t)ch * C + c] = s;
}

__global__ void col_sum_chunks_kernel(const float *partial, int64_t C, float *out, int accumulate) {
  const int64_t c = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (c >= C) return;
  float s = 0.0f;
  for (int ch = 0; ch < kRowChunks; ch++) s += partial[(int64_t)ch * C + c];
  out[c] = accumulate ? out[c] + s : s;
}

// partial[ch][c] = sum_{r in chunk ch} X[r][c]^2 in float64 (each square is
// exact in float64; the sums of the few-bit HiF4 values that feed it are exact)
__global__ void col_sumsq_partial_kernel(const float *X, int64_t R, int64_t C, double *partial) {
  const int64_t c = (int64_t)blockIdx.x * UT + threadIdx.x;
  const int ch = blockIdx.y;
  if (c >= C) return;
  const int64_t rows_per = (R + kRowChunks - 1) / kRowChunks;
  const int64_t r0 = ch * rows_per, r1 = min(R, r0 + rows_per);
  double s = 0.0;
  for (int64_t r = r0; r < r1; r++) {
    const double x = (double)X[r * C + c];
    s = __dadd_rn(s, __dmul_rn(x, x));
  }
  partial[(int64_t)ch * C + c] = s;
}

__global__ void col_sumsq_final_kernel(const double *partial, int64_t C, float *out) {
  const int64_t c = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (c >= C) return;
  double s = 0.0;
  for (int ch = 0; ch < kRowChunks; ch++) s = __dadd_rn(s, partial[(int64_t)ch * C + c]);
  out[c] = __double2float_rn(s);
}

// m = max(abs_sum / n_tok, 1e-12); logm = log(m) - mean(log m)
// (example/solution/solution.py:855-857); one CTA.
__global__ void __launch_bounds__(1024) smooth_logm_kernel(const float *abs_sum, int64_t C, float inv_ntok,
                                                           float *logm) {
  __shared__ float red[32];
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float lm = logf(fmaxf(abs_sum[c] * inv_ntok, 1e-12f));
    logm[c] = lm;
    s += lm;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = red[0] / (float)C;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) logm[c] -= mean;
}

__global__ void exp_scale_kernel(const float *logm, int64_t C, float alpha, float *s) {
  const int64_t c = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (c < C) s[c] = expf(logm[c] * alpha);
}

__global__ void gather_rows_kernel(const float *src, const int64_t *idx, int64_t n, int64_t C, float *dst) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= n * C) return;
  const int64_t i = e / C, c = e % C;
  dst[e] = src[idx[i] * C + c];
}

__global__ void gather_cols_kernel(const float *src, const int64_t *idx, int64_t R, int64_t C, float *dst) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= R * C) return;
  const int64_t r = e / C, j = e % C;
  dst[e] = src[r * C + idx[j]];
}

__global__ void scatter_cols_kernel(const float *src, const int64_t *idx, int64_t R, int64_t C, float *dst) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= R * C) return;
  const int64_t r = e / C, j = e % C;
  dst[r * C + idx[j]] = src[e];
}

// out[i][j] = A[idx[i]][idx[j]]
__global__ void permute_sym_kernel(const float *A, const int64_t *idx, int64_t n, float *out) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= n * n) return;
  out[e] = A[idx[e / n] * n + idx[e % n]];
}

__global__ void scale_cols_kernel(const float *X, const float *s, int64_t R, int64_t C, int mode, float *out) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= R * C) return;
  const float v = X[e], f = s[e % C];
  out[e] = mode == HIF4X_SMOOTH_MUL ? __fmul_rn(v, f) : __fdiv_rn(v, f);
}

// partial sums in double for sum((A-B)^2) (B may be null -> sum(A^2)) or sum(|A|)
__global__ void reduce_partial_kernel(const float *A, const float *B, int64_t n, int op, double *partial) {
  __shared__ double red[UT / 32];
  double s = 0.0;
  for (int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x; e < n; e += (int64_t)gridDim.x * UT) {
    if (op == 0) {
      const double d = (double)A[e] - (B ? (double)B[e] : 0.0);
      s += d * d;
    } else {
      s += fabs((double)A[e]);
    }
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double v = 0.0;
    for (int w = 0; w < UT / 32; w++) v += red[w];
    partial[blockIdx.x] = v;
  }
}

__global__ void reduce_final_kernel(const double *partial, int n, double *out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double v = 0.0;
    for (int i = 0; i < n; i++) v += partial[i];
    *out = v;
  }
}

__global__ void diag_kernel(const float *A, int64_t n, float *out) {
  const int64_t i = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (i < n) out[i] = A[i * n + i];
}

// Bitonic argsort, descending by value, ascending index on ties; one CTA,
// n <= 16384 (padded to a power of two in shared memory).
__global__ void __launch_bounds__(1024) argsort_desc_kernel(const float *v, int n, int npow, int64_t *idx) {
  extern __shared__ unsigned char smraw[];
  float *key = reinterpret_cast<float *>(smraw);
  int *ix = reinterpret_cast<int *>(key + npow);
  for (int i = threadIdx.x; i < npow; i += blockDim.x) {
    key[i] = i < n ? v[i] : -INFINITY;
    ix[i] = i < n ? i : 0x7fffffff;
  }
  __syncthreads();
  // "before(a, b)": a sorts earlier than b
  for (int k = 2; k <= npow; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < npow; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const float ki = key[i], kl = key[l];
          const int ii = ix[i], il = ix[l];
          const bool l_before_i = (kl > ki) || (kl == ki && il < ii);
          const bool asc = (i & k) == 0;  // this half sorts in the "before" order
          if (asc ? l_before_i : !l_before_i) {
            key[i] = kl; key[l] = ki; ix[i] = il; ix[l] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) idx[i] = ix[i];
}

__global__ void f32_to_bf16_kernel(const float *in, __nv_bfloat16 *out, int64_t n) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e < n) out[e] = __float2bfloat16_rn(in[e]);
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16 *in, float *out, int64_t n) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e < n) out[e] = __bfloat162float(in[e]);
}

// v4 = round(values / unit * 4), d = 0.25 * unit  (solution.py:634-635, 680-681)
__global__ void refine_prep_kernel(const float *values, const float *unit, int64_t n, float *v4, float *d) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= n) return;
  const float u = unit[e];
  v4[e] = rintf(__fmul_rn(__fdiv_rn(values[e], u), 4.0f));
  d[e] = __fmul_rn(0.25f, u);
}

// out = a * b + c * alpha (elementwise; c may be null)
__global__ void axpby_kernel(const float *a, const float *b, const float *c, float alpha, int64_t n, float *out) {
  const int64_t e = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (e >= n) return;
  float v = b ? __fmul_rn(a[e], b[e]) : a[e];
  if (c) v = __fadd_rn(v, __fmul_rn(alpha, c[e]));
  out[e] = v;
}

// E2M1 value -> nibble (sign<<3 | index of |v| in {0, .5, 1, 1.5, 2, 3, 4, 6});
// -1 when v is not one of the 16 values (NaN and infinities included).
__device__ __forceinline__ int e2m1_nibble(float v) {
  const float a = fabsf(v);
  int idx;
  if (a == 0.0f) idx = 0;
  else if (a == 0.5f) idx = 1;
  else if (a == 1.0f) idx = 2;
  else if (a == 1.5f) idx = 3;
  else if (a == 2.0f) idx = 4;
  else if (a == 3.0f) idx = 5;
  else if (a == 4.0f) idx = 6;
  else if (a == 6.0f) idx = 7;
  else return -1;
  return idx | (signbit(v) ? 8 : 0);
}

// Pack an NVFP4 carrier (fp32 or bf16 E2M1 values, n even) two elements per
// byte, element 2i in the low nibble; counts the elements that are not E2M1
// values (their nibble is written as 0).
__global__ void e2m1_pack_kernel(const void *carrier, int dtype, int64_t npair, uint8_t *codes, int *bad) {
  const int64_t i = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (i >= npair) return;
  float v0, v1;
  if (dtype == HIF4X_DT_BF16) {
    const uint32_t w = ((const uint32_t *)carrier)[i];
    v0 = __uint_as_float(w << 16);
    v1 = __uint_as_float(w & 0xffff0000u);
  } else {
    const float2 w = ((const float2 *)carrier)[i];
    v0 = w.x;
    v1 = w.y;
  }
  int n0 = e2m1_nibble(v0), n1 = e2m1_nibble(v1);
  if (n0 < 0 || n1 < 0) {
    atomicAdd(bad, 1);
    n0 = n0 < 0 ? 0 : n0;
    n1 = n1 < 0 ? 0 : n1;
  }
  codes[i] = (uint8_t)(n0 | (n1 << 4));
}

// Inverse of e2m1_pack_kernel: codes -> bf16 or fp32 carrier (-0 kept).
__global__ void e2m1_unpack_kernel(const uint8_t *codes, int64_t npair, void *carrier, int dtype) {
  const int64_t i = (int64_t)blockIdx.x * UT + threadIdx.x;
  if (i >= npair) return;
  const uint32_t b = codes[i];
  const float v0 = e2m1_to_f32(b & 15u), v1 = e2m1_to_f32(b >> 4);
  if (dtype == HIF4X_DT_BF16) {
    ((uint32_t *)carrier)[i] = (__float_as_uint(v0) >> 16) | (__float_as_uint(v1) & 0xffff0000u);
  } else {
    ((float2 *)carrier)[i] = make_float2(v0, v1);
  }
}

}  // namespace hif4x

using namespace hif4x;
static inline unsigned nb_(int64_t n) { return (unsigned)((n + UT - 1) / UT); }

extern "C" int hif4x_col_abs_sum(const float *X, int64_t R, int64_t C, float *out, int accumulate, float *work,
                                 void *stream) {
  if (R < 0 || C <= 0 || !out || !work || (R > 0 && !X)) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  col_abs_partial_kernel<<<dim3(nb_(C), kRowChunks), UT, 0, s>>>(X, R, C, work);
  col_sum_chunks_kernel<<<nb_(C), UT, 0, s>>>(work, C, out, accumulate);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_col_sumsq(const float *X, int64_t R, int64_t C, float *out, double *work, void *stream) {
  if (R < 0 || C <= 0 || !out || !work || (R > 0 && !X)) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  col_sumsq_partial_kernel<<<dim3(nb_(C), kRowChunks), UT, 0, s>>>(X, R, C, work);
  col_sumsq_final_kernel<<<nb_(C), UT, 0, s>>>(work, C, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_smooth_logm(const float *abs_sum, int64_t C, int64_t n_tok, float *logm, void *stream) {
  if (C <= 0 || !abs_sum || !logm) return HIF4X_ERR_ARG;
  const float inv = 1.0f / (float)(n_tok > 0 ? n_tok : 1);
  smooth_logm_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(abs_sum, C, inv, logm);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_exp_scale(const float *logm, int64_t C, float alpha, float *s, void *stream) {
  if (C <= 0 || !logm || !s) return HIF4X_ERR_ARG;
  exp_scale_kernel<<<nb_(C), UT, 0, (cudaStream_t)stream>>>(logm, C, alpha, s);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_gather_rows(const float *src, const int64_t *idx, int64_t n, int64_t C, float *dst,
                                 void *stream) {
  if (n < 0 || C < 0) return HIF4X_ERR_ARG;
  if (n * C == 0) return HIF4X_OK;
  if (!src || !idx || !dst) return HIF4X_ERR_ARG;
  gather_rows_kernel<<<nb_(n * C), UT, 0, (cudaStream_t)stream>>>(src, idx, n, C, dst);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_gather_cols(const float *src, const int64_t *idx, int64_t R, int64_t C, float *dst,
                                 void *stream) {
  if (R < 0 || C < 0) return HIF4X_ERR_ARG;
  if (R * C == 0) return HIF4X_OK;
  if (!src || !idx || !dst) return HIF4X_ERR_ARG;
  gather_cols_kernel<<<nb_(R * C), UT, 0, (cudaStream_t)stream>>>(src, idx, R, C, dst);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_scatter_cols(const float *src, const int64_t *idx, int64_t R, int64_t C, float *dst,
                                  void *stream) {
  if (R < 0 || C < 0) return HIF4X_ERR_ARG;
  if (R * C == 0) return HIF4X_OK;
  if (!src || !idx || !dst) return HIF4X_ERR_ARG;
  scatter_cols_kernel<<<nb_(R * C), UT, 0, (cudaStream_t)stream>>>(src, idx, R, C, dst);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_permute_sym(const float *A, const int64_t *idx, int64_t n, float *out, void *stream) {
  if (n <= 0 || !A || !idx || !out) return HIF4X_ERR_ARG;
  permute_sym_kernel<<<nb_(n * n), UT, 0, (cudaStream_t)stream>>>(A, idx, n, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_scale_cols(const float *X, const float *s, int64_t R, int64_t C, int mode, float *out,
                                void *stream) {
  if (R < 0 || C <= 0 || (mode != HIF4X_SMOOTH_MUL && mode != HIF4X_SMOOTH_DIV)) return HIF4X_ERR_ARG;
  if (R == 0) return HIF4X_OK;
  if (!X || !s || !out) return HIF4X_ERR_ARG;
  scale_cols_kernel<<<nb_(R * C), UT, 0, (cudaStream_t)stream>>>(X, s, R, C, mode, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// op 0: sum((A - B)^2) (B may be NULL), op 1: sum(|A|); result in double.
// work: >= 1024 doubles.
extern "C" int hif4x_reduce(const float *A, const float *B, int64_t n, int op, double *out, double *work,
                            void *stream) {
  if (n < 0 || !out || !work || (op != 0 && op != 1) || (n > 0 && !A)) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  int blocks = (int)std::min<int64_t>(1024, std::max<int64_t>(1, (n + UT - 1) / UT));
  reduce_partial_kernel<<<blocks, UT, 0, s>>>(A, B, n, op, work);
  reduce_final_kernel<<<1, 32, 0, s>>>(work, blocks, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_diag(const float *A, int64_t n, float *out, void *stream) {
  if (n <= 0 || !A || !out) return HIF4X_ERR_ARG;
  diag_kernel<<<nb_(n), UT, 0, (cudaStream_t)stream>>>(A, n, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_argsort_desc(const float *v, int64_t n, int64_t *idx, void *stream) {
  if (n <= 0 || n > 16384 || !v || !idx) return HIF4X_ERR_ARG;
  int npow = 1;
  while (npow < n) npow <<= 1;
  const size_t smem = (size_t)npow * (sizeof(float) + sizeof(int));
  cudaFuncSetAttribute(argsort_desc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  argsort_desc_kernel<<<1, 1024, smem, (cudaStream_t)stream>>>(v, (int)n, npow, idx);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_cast(const void *in, int in_dtype, void *out, int out_dtype, int64_t n, void *stream) {
  if (n < 0) return HIF4X_ERR_ARG;
  if (n == 0) return HIF4X_OK;
  if (!in || !out) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  if (in_dtype == HIF4X_DT_F32 && out_dtype == HIF4X_DT_BF16)
    f32_to_bf16_kernel<<<nb_(n), UT, 0, s>>>((const float *)in, (__nv_bfloat16 *)out, n);
  else if (in_dtype == HIF4X_DT_BF16 && out_dtype == HIF4X_DT_F32)
    bf16_to_f32_kernel<<<nb_(n), UT, 0, s>>>((const __nv_bfloat16 *)in, (float *)out, n);
  else
    return HIF4X_ERR_UNSUPPORTED;
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_refine_prep(const float *values, const float *unit, int64_t n, float *v4, float *d,
                                 void *stream) {
  if (n < 0) return HIF4X_ERR_ARG;
  if (n == 0) return HIF4X_OK;
  if (!values || !unit || !v4 || !d) return HIF4X_ERR_ARG;
  refine_prep_kernel<<<nb_(n), UT, 0, (cudaStream_t)stream>>>(values, unit, n, v4, d);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_axpby(const float *a, const float *b, const float *c, float alpha, int64_t n, float *out,
                           void *stream) {
  if (n < 0) return HIF4X_ERR_ARG;
  if (n == 0) return HIF4X_OK;
  if (!a || !out) return HIF4X_ERR_ARG;
  axpby_kernel<<<nb_(n), UT, 0, (cudaStream_t)stream>>>(a, b, c, alpha, n, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_e2m1_pack(const void *carrier, int dtype, int64_t n, uint8_t *codes, int *bad_dev, void *stream) {
  if (n < 0 || (n & 1) || (dtype != HIF4X_DT_F32 && dtype != HIF4X_DT_BF16)) return HIF4X_ERR_ARG;
  if (n == 0) return HIF4X_OK;
  if (!carrier || !codes || !bad_dev) return HIF4X_ERR_ARG;
  e2m1_pack_kernel<<<nb_(n / 2), UT, 0, (cudaStream_t)stream>>>(carrier, dtype, n / 2, codes, bad_dev);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_e2m1_unpack(const uint8_t *codes, int64_t n, void *carrier, int dtype, void *stream) {
  if (n < 0 || (n & 1) || (dtype != HIF4X_DT_F32 && dtype != HIF4X_DT_BF16)) return HIF4X_ERR_ARG;
  if (n == 0) return HIF4X_OK;
  if (!carrier || !codes) return HIF4X_ERR_ARG;
  e2m1_unpack_kernel<<<nb_(n / 2), UT, 0, (cudaStream_t)stream>>>(codes, n / 2, carrier, dtype);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}
