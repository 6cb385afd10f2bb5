// vcomp.cu -- double-precision pieces of the attention V compensation
// (example/solution/solution.py:1288-1333, _v_compensate):
//
//   G[g]  = sum_{h in group g} Ph_h^T Ph_h                 (T x T, f64)
//   RHS[g] = sum_{h in group g} Ph_h^T (P_h V_g)            (T x dh, f64)
//   X[g]  = (G[g] + lam_g * 1 1^T)^-1 RHS[g]                (Cholesky, f64)
//
// with P_h / Ph_h the fp32 softmax probabilities of the original / quantized
// q and k.  The reference solves (G + lam) B = Cm with Cm = sum Ph^T P and
// then forms B V; X = (G + lam)^-1 (Cm V) is the same product with dh
// right-hand sides instead of T.  lam = 1e-4 * mean(diag G[g]) is added to
// every entry of G, as the reference's broadcast of a (kvh, 1, 1) tensor
// does (solution.py:1316-1317).
//
// gemm64_kernel: C = alpha op(A) op(B) + beta C with fp32 or f64 operands,
// f64 accumulation and output, batched by strides; 64 x 64 tiles, 16-deep
// K steps staged in shared memory, 256 threads with 4 x 4 outputs each.
// Products of two fp32 values are exact in f64, so G and RHS carry only the
// f64 summation error.
//
// chol64: blocked right-looking lower Cholesky with 64-wide panels.  One CTA
// per batch element factors the diagonal block in shared memory and inverts
// it; the panel below is A21 L11^-T and the trailing update A22 -= L21 L21^T
// (lower tiles only) are gemm64 launches.  The two triangular solves reuse
// the diagonal inverses: Y_j = L_jj^-1 R_j, then R below -= L21 Y_j; and
// backwards X_j = L_jj^-T Y_j, Y above -= L_j,:j^T X_j.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace hif4x {

constexpr int G64T = 64;     // output tile (square: the lower-only mode relies on it)
constexpr int G64K = 16;     // K step
constexpr int CB64 = 64;     // Cholesky panel

struct Gemm64Params {
  int ta, tb, lower;
  int64_t M, N, K;
  double alpha, beta;
  const void *A;
  int64_t lda, sA;
  const void *B;
  int64_t ldb, sB;
  double *C;
  int64_t ldc, sC;
};

template <typename TA, typename TB>
__global__ void __launch_bounds__(256) gemm64_kernel(const Gemm64Params g) {
  __shared__ double As[G64K][G64T + 1];
  __shared__ double Bs[G64K][G64T + 1];
  const int bx = blockIdx.x, by = blockIdx.y;
  if (g.lower && bx > by) return;  // tile strictly above the diagonal
  const int64_t m0 = (int64_t)by * G64T, n0 = (int64_t)bx * G64T;
  const int64_t bz = blockIdx.z;
  const TA *A = (const TA *)g.A + bz * g.sA;
  const TB *B = (const TB *)g.B + bz * g.sB;
  double *C = g.C + bz * g.sC;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  double acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
  for (int64_t k0 = 0; k0 < g.K; k0 += G64K) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int e = tid + 256 * q;
      int mm, kk;
      if (g.ta) {
        kk = e >> 6;
        mm = e & 63;
      } else {
        mm = e >> 4;
        kk = e & 15;
      }
      const int64_t gm = m0 + mm, gk = k0 + kk;
      double v = 0.0;
      if (gm < g.M && gk < g.K) v = (double)(g.ta ? A[gk * g.lda + gm] : A[gm * g.lda + gk]);
      As[kk][mm] = v;
      int nn;
      if (g.tb) {
        nn = e >> 4;
        kk = e & 15;
      } else {
        kk = e >> 6;
        nn = e & 63;
      }
      const int64_t gn = n0 + nn, gk2 = k0 + kk;
      double w = 0.0;
      if (gn < g.N && gk2 < g.K) w = (double)(g.tb ? B[gn * g.ldb + gk2] : B[gk2 * g.ldb + gn]);
      Bs[kk][nn] = w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < G64K; kk++) {
      double a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t gm = m0 + ty + 16 * i;
    if (gm >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int64_t gn = n0 + tx + 16 * j;
      if (gn >= g.N) continue;
      double r = g.alpha * acc[i][j];
      if (g.beta != 0.0) r += g.beta * C[gm * g.ldc + gn];
      C[gm * g.ldc + gn] = r;
    }
  }
}

// A[b][j][i] = A[b][i][j] for j > i (lower -> upper)
__global__ void mirror_lower64_kernel(double *A, int64_t n, int64_t nn) {
  const int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (e >= nn) return;
  const int64_t i = e / n, j = e % n;
  if (j > i) A[blockIdx.y * nn + e] = A[blockIdx.y * nn + j * n + i];
}

// A[b] += lam_rel * mean(diag A[b]) on every entry of the lower triangle
// (the factorisation reads only the lower triangle).
__global__ void __launch_bounds__(256) add_mean_diag64_kernel(double *A, int64_t n, double lam_rel) {
  __shared__ double red[256];
  double *Ab = A + (int64_t)blockIdx.x * n * n;
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 256) s += Ab[i * n + i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  const double lam = lam_rel * (red[0] / (double)n);
  for (int64_t e = threadIdx.x; e < n * n; e += 256) {
    const int64_t i = e / n, j = e % n;
    if (j <= i) Ab[e] += lam;
  }
}

// Factor the b x b diagonal block at (j, j) of every batch element's A
// (lower triangle read) into L (lower, zeros above left untouched) and its
// inverse into Dinv (64 x 64, identity-padded).  A non-positive (or NaN)
// pivot sets *info = 1 and continues with pivot 1 so the launch completes.
__global__ void __launch_bounds__(256) chol64_diag_kernel(const double *A, int64_t n, int64_t j, int b, double *L,
                                                          double *Dinv, int64_t nblk, int *info) {
  extern __shared__ double sm[];
  double *S = sm;                        // [64][65]
  double *I = sm + CB64 * (CB64 + 1);    // [64][65]
  const int64_t bz = blockIdx.x;
  const double *Ab = A + bz * n * n;
  double *Lb = L + bz * n * n;
  double *Db = Dinv + (bz * nblk + j / CB64) * CB64 * CB64;
  const int tid = threadIdx.x;
  for (int e = tid; e < CB64 * CB64; e += 256) {
    const int r = e / CB64, c = e % CB64;
    double v = (r == c) ? 1.0 : 0.0;
    if (r < b && c <= r) v = Ab[(j + r) * n + j + c];
    S[r * (CB64 + 1) + c] = v;
  }
  __syncthreads();
  for (int c = 0; c < b; c++) {
    if (tid == 0) {
      double p = S[c * (CB64 + 1) + c];
      if (!(p > 0.0)) {
        *info = 1;
        p = 1.0;
      }
      S[c * (CB64 + 1) + c] = sqrt(p);
    }
    __syncthreads();
    const double d = S[c * (CB64 + 1) + c];
    for (int r = c + 1 + tid; r < b; r += 256) S[r * (CB64 + 1) + c] /= d;
    __syncthreads();
    const int w = b - c - 1;
    for (int e = tid; e < w * w; e += 256) {
      const int r = c + 1 + e / w, s = c + 1 + e % w;
      if (s <= r) S[r * (CB64 + 1) + s] -= S[r * (CB64 + 1) + c] * S[s * (CB64 + 1) + c];
    }
    __syncthreads();
  }
  // inverse of the lower-triangular 64 x 64 block (identity-padded): thread
  // `col` solves L x = e_col by forward substitution
  if (tid < CB64) {
    const int col = tid;
    for (int r = 0; r < CB64; r++) {
      double v = 0.0;
      if (r >= col) {
        v = (r == col) ? 1.0 : 0.0;
        for (int k = col; k < r; k++) v -= S[r * (CB64 + 1) + k] * I[k * (CB64 + 1) + col];
        v /= S[r * (CB64 + 1) + r];
      }
      I[r * (CB64 + 1) + col] = v;
    }
  }
  __syncthreads();
  for (int e = tid; e < CB64 * CB64; e += 256) {
    const int r = e / CB64, c = e % CB64;
    Db[e] = I[r * (CB64 + 1) + c];
    if (r < b && c <= r) Lb[(j + r) * n + j + c] = S[r * (CB64 + 1) + c];
  }
}

// Row softmax in place: S[r, :] = softmax(S[r, :] / div), fp32 (torch's
// max-subtracted form).  One CTA per row.
__global__ void __launch_bounds__(256) softmax_rows_kernel(float *S, int64_t cols, float div) {
  __shared__ float red[256];
  float *row = S + (int64_t)blockIdx.x * cols;
  float mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += 256) mx = fmaxf(mx, __fdiv_rn(row[c], div));
  red[threadIdx.x] = mx;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] = fmaxf(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  mx = red[0];
  __syncthreads();
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += 256) {
    const float e = expf(__fsub_rn(__fdiv_rn(row[c], div), mx));
    row[c] = e;
    s += e;
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  const float tot = red[0];
  for (int64_t c = threadIdx.x; c < cols; c += 256) row[c] = __fdiv_rn(row[c], tot);
}

// out[b*obs + j*old + i] = in[b*ibs + i*ild + j] for i < R, j < Cc: a batched
// strided transpose through a 32 x 33 shared tile.
__global__ void transpose_batched_kernel(const float *in, int64_t R, int64_t Cc, int64_t ild, int64_t ibs,
                                         float *out, int64_t old, int64_t obs) {
  __shared__ float t[32][33];
  const int64_t i0 = (int64_t)blockIdx.y * 32, j0 = (int64_t)blockIdx.x * 32;
  const int64_t bz = blockIdx.z;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int k = ty; k < 32; k += 8) {
    const int64_t i = i0 + k, j = j0 + tx;
    if (i < R && j < Cc) t[k][tx] = in[bz * ibs + i * ild + j];
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int64_t j = j0 + k, i = i0 + tx;
    if (i < R && j < Cc) out[bz * obs + j * old + i] = t[tx][k];
  }
}

__global__ void f64_to_f32_kernel(const double *in, float *out, int64_t n) {
  const int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (e < n) out[e] = __double2float_rn(in[e]);
}

static inline unsigned nb64(int64_t n, int64_t b) { return (unsigned)((n + b - 1) / b); }

static int gemm64_launch(int ta, int tb, int a_dt, int b_dt, int64_t M, int64_t N, int64_t K, double alpha,
                         const void *A, int64_t lda, int64_t sA, const void *B, int64_t ldb, int64_t sB, double beta,
                         double *C, int64_t ldc, int64_t sC, int64_t batch, int lower, cudaStream_t s) {
  if (M < 0 || N < 0 || K < 0 || batch < 0) return HIF4X_ERR_ARG;
  if (M == 0 || N == 0 || batch == 0) return HIF4X_OK;
  if (!A || !B || !C) return HIF4X_ERR_ARG;
  if (lower && M != N) return HIF4X_ERR_ARG;
  const bool af = a_dt == HIF4X_DT_F32, bf = b_dt == HIF4X_DT_F32;
  if ((!af && a_dt != HIF4X_DT_F64) || (!bf && b_dt != HIF4X_DT_F64)) return HIF4X_ERR_UNSUPPORTED;
  const dim3 grid(nb64(N, G64T), nb64(M, G64T), (unsigned)batch);
  if (grid.y > 65535 || batch > 65535) return HIF4X_ERR_ARG;
  Gemm64Params g{ta, tb, lower, M, N, K, alpha, beta, A, lda, sA, B, ldb, sB, C, ldc, sC};
  if (af && bf)
    gemm64_kernel<float, float><<<grid, 256, 0, s>>>(g);
  else if (af)
    gemm64_kernel<float, double><<<grid, 256, 0, s>>>(g);
  else if (bf)
    gemm64_kernel<double, float><<<grid, 256, 0, s>>>(g);
  else
    gemm64_kernel<double, double><<<grid, 256, 0, s>>>(g);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

}  // namespace hif4x

using namespace hif4x;

extern "C" int hif4x_gemm_f64(int ta, int tb, int a_dtype, int b_dtype, int64_t M, int64_t N, int64_t K,
                              double alpha, const void *A, int64_t lda, int64_t sA, const void *B, int64_t ldb,
                              int64_t sB, double beta, double *C, int64_t ldc, int64_t sC, int64_t batch, int lower,
                              void *stream) {
  return gemm64_launch(ta, tb, a_dtype, b_dtype, M, N, K, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, batch,
                       lower, (cudaStream_t)stream);
}

extern "C" int hif4x_mirror_lower_f64(double *A, int64_t n, int64_t batch, void *stream) {
  if (n < 0 || batch < 0 || batch > 65535) return HIF4X_ERR_ARG;
  if (n == 0 || batch == 0) return HIF4X_OK;
  if (!A) return HIF4X_ERR_ARG;
  const int64_t nn = n * n;
  mirror_lower64_kernel<<<dim3(nb64(nn, 256), (unsigned)batch), 256, 0, (cudaStream_t)stream>>>(A, n, nn);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_chol_solve_f64(double *A, int64_t n, int64_t batch, double lam_rel, const double *Rhs,
                                    int64_t m, double *X, double *work, int *info_dev, void *stream) {
  if (n <= 0 || m <= 0 || batch <= 0 || batch > 65535) return HIF4X_ERR_ARG;
  if (!A || !Rhs || !X || !work || !info_dev) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nn = n * n, nm = n * m, nblk = (n + CB64 - 1) / CB64;
  double *L = work;                              // batch * n * n
  double *Dinv = L + batch * nn;                 // batch * nblk * 64 * 64
  double *R = Dinv + batch * nblk * CB64 * CB64; // batch * n * m
  double *Y = R + batch * nm;                    // batch * n * m
  if (cudaMemsetAsync(info_dev, 0, sizeof(int), s) != cudaSuccess ||
      cudaMemsetAsync(L, 0, sizeof(double) * batch * nn, s) != cudaSuccess ||
      cudaMemcpyAsync(R, Rhs, sizeof(double) * batch * nm, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  if (lam_rel != 0.0) add_mean_diag64_kernel<<<(unsigned)batch, 256, 0, s>>>(A, n, lam_rel);
  const int smem = (int)(2 * sizeof(double) * CB64 * (CB64 + 1));
  if (cudaFuncSetAttribute(chol64_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  const int64_t dstride = nblk * CB64 * CB64;
  for (int64_t j = 0; j < n; j += CB64) {
    const int b = (int)std::min<int64_t>(CB64, n - j);
    chol64_diag_kernel<<<(unsigned)batch, 256, smem, s>>>(A, n, j, b, L, Dinv, nblk, info_dev);
    HIF4X_CHECK_LAUNCH();
    const int64_t rest = n - j - b;
    if (rest <= 0) continue;
    const double *Djj = Dinv + (j / CB64) * CB64 * CB64;
    // L21 = A21 L11^-T
    int st = gemm64_launch(0, 1, HIF4X_DT_F64, HIF4X_DT_F64, rest, b, b, 1.0, A + (j + b) * n + j, n, nn, Djj, CB64,
                           dstride, 0.0, L + (j + b) * n + j, n, nn, batch, 0, s);
    if (st) return st;
    // A22 -= L21 L21^T (lower tiles)
    const double *L21 = L + (j + b) * n + j;
    st = gemm64_launch(0, 1, HIF4X_DT_F64, HIF4X_DT_F64, rest, rest, b, -1.0, L21, n, nn, L21, n, nn, 1.0,
                       A + (j + b) * n + (j + b), n, nn, batch, 1, s);
    if (st) return st;
  }
  // forward: L Y = R
  for (int64_t j = 0; j < n; j += CB64) {
    const int b = (int)std::min<int64_t>(CB64, n - j);
    const double *Djj = Dinv + (j / CB64) * CB64 * CB64;
    int st = gemm64_launch(0, 0, HIF4X_DT_F64, HIF4X_DT_F64, b, m, b, 1.0, Djj, CB64, dstride, R + j * m, m, nm, 0.0,
                           Y + j * m, m, nm, batch, 0, s);
    if (st) return st;
    const int64_t rest = n - j - b;
    if (rest <= 0) continue;
    st = gemm64_launch(0, 0, HIF4X_DT_F64, HIF4X_DT_F64, rest, m, b, -1.0, L + (j + b) * n + j, n, nn, Y + j * m, m,
                       nm, 1.0, R + (j + b) * m, m, nm, batch, 0, s);
    if (st) return st;
  }
  // backward: L^T X = Y
  for (int64_t j = ((n - 1) / CB64) * CB64; j >= 0; j -= CB64) {
    const int b = (int)std::min<int64_t>(CB64, n - j);
    const double *Djj = Dinv + (j / CB64) * CB64 * CB64;
    int st = gemm64_launch(1, 0, HIF4X_DT_F64, HIF4X_DT_F64, b, m, b, 1.0, Djj, CB64, dstride, Y + j * m, m, nm, 0.0,
                           X + j * m, m, nm, batch, 0, s);
    if (st) return st;
    if (j == 0) break;
    // Y[:j] -= L[j:j+b, :j]^T X_j
    st = gemm64_launch(1, 0, HIF4X_DT_F64, HIF4X_DT_F64, j, m, b, -1.0, L + j * n, n, nn, X + j * m, m, nm, 1.0, Y,
                       m, nm, batch, 0, s);
    if (st) return st;
  }
  int info = 0;
  if (cudaMemcpyAsync(&info, info_dev, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  return info ? HIF4X_NOT_PD : HIF4X_OK;
}

extern "C" int hif4x_softmax_rows(float *S, int64_t rows, int64_t cols, float div, void *stream) {
  if (rows < 0 || cols <= 0 || rows > 0x7fffffffLL) return HIF4X_ERR_ARG;
  if (rows == 0) return HIF4X_OK;
  if (!S) return HIF4X_ERR_ARG;
  softmax_rows_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(S, cols, div);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_transpose_batched(const float *in, int64_t R, int64_t Cc, int64_t batch, int64_t ild, int64_t ibs,
                                       float *out, int64_t old, int64_t obs, void *stream) {
  if (R < 0 || Cc < 0 || batch < 0 || batch > 65535) return HIF4X_ERR_ARG;
  if (R == 0 || Cc == 0 || batch == 0) return HIF4X_OK;
  if (!in || !out || nb64(R, 32) > 65535) return HIF4X_ERR_ARG;
  const dim3 grid(nb64(Cc, 32), nb64(R, 32), (unsigned)batch);
  transpose_batched_kernel<<<grid, dim3(32, 8), 0, (cudaStream_t)stream>>>(in, R, Cc, ild, ibs, out, old, obs);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_f64_to_f32(const double *in, int64_t n, float *out, void *stream) {
  if (n < 0) return HIF4X_ERR_ARG;
  if (n == 0) return HIF4X_OK;
  if (!in || !out) return HIF4X_ERR_ARG;
  f64_to_f32_kernel<<<nb64(n, 256), 256, 0, (cudaStream_t)stream>>>(in, out, n);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}
