// linalg.cu -- fp32 dense linear algebra for the calibration pipeline:
//   * strided-batched GEMM  C = alpha * op(A) op(B) + beta * C  (row-major)
//   * damped Cholesky -> upper factor of the inverse (GPTQ's Hinv)
//   * GPTQ column-sequential quantize-and-propagate inside a column block
//
// The GEMM is a register-tiled SIMT kernel (128x128x8 CTA tile, 8x8 per
// thread, double-buffered shared memory), fp32 in and out with fp32
// accumulation, so every product matches the reference's fp32 matmuls to
// rounding.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace hif4x {

// --------------------------------------------------------------------------
// GEMM
constexpr int GBM = 128, GBN = 128, GBK = 8, GTHREADS = 256;

struct GemmArgs {
  int ta, tb;
  int64_t M, N, K;
  float alpha, beta;
  const float *A;
  int64_t lda, sA;
  const float *B;
  int64_t ldb, sB;
  float *C;
  int64_t ldc, sC;
  int lower;   // 1: skip output tiles strictly above the diagonal
};

__global__ void __launch_bounds__(GTHREADS) gemm_kernel(const GemmArgs g) {
  __shared__ __align__(16) float As[2][GBK][GBM];
  __shared__ __align__(16) float Bs[2][GBK][GBN];
  const int64_t bz = blockIdx.z;
  const float *A = g.A + bz * g.sA;
  const float *B = g.B + bz * g.sB;
  float *C = g.C + bz * g.sC;
  const int64_t m0 = (int64_t)blockIdx.y * GBM, n0 = (int64_t)blockIdx.x * GBN;
  if (g.lower && n0 > m0 + GBM - 1) return;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;  // 16 x 16 threads, each 8x8 outputs

  // each thread loads 4 A elements and 4 B elements per K-tile
  auto loadA = [&](int64_t k0, float (&ra)[4]) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int e = tid + r * GTHREADS;  // 0..1023 over (BK x BM)
      int mm, kk;
      if (g.ta) { kk = e / GBM; mm = e % GBM; }   // A stored K x M: contiguous in m
      else { mm = e / GBK; kk = e % GBK; }        // A stored M x K: contiguous in k
      const int64_t gm = m0 + mm, gk = k0 + kk;
      float v = 0.0f;
      if (gm < g.M && gk < g.K) v = g.ta ? A[gk * g.lda + gm] : A[gm * g.lda + gk];
      ra[r] = v;
    }
  };
  auto storeA = [&](int buf, const float (&ra)[4]) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int e = tid + r * GTHREADS;
      int mm, kk;
      if (g.ta) { kk = e / GBM; mm = e % GBM; }
      else { mm = e / GBK; kk = e % GBK; }
      As[buf][kk][mm] = ra[r];
    }
  };
  auto loadB = [&](int64_t k0, float (&rb)[4]) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int e = tid + r * GTHREADS;
      int nn, kk;
      if (g.tb) { nn = e / GBK; kk = e % GBK; }   // B stored N x K: contiguous in k
      else { kk = e / GBN; nn = e % GBN; }        // B stored K x N: contiguous in n
      const int64_t gn = n0 + nn, gk = k0 + kk;
      float v = 0.0f;
      if (gn < g.N && gk < g.K) v = g.tb ? B[gn * g.ldb + gk] : B[gk * g.ldb + gn];
      rb[r] = v;
    }
  };
  auto storeB = [&](int buf, const float (&rb)[4]) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int e = tid + r * GTHREADS;
      int nn, kk;
      if (g.tb) { nn = e / GBK; kk = e % GBK; }
      else { kk = e / GBN; nn = e % GBN; }
      Bs[buf][kk][nn] = rb[r];
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

  float ra[4], rb[4];
  loadA(0, ra);
  loadB(0, rb);
  storeA(0, ra);
  storeB(0, rb);
  __syncthreads();
  const int64_t nk = (g.K + GBK - 1) / GBK;
  for (int64_t t = 0; t < nk; t++) {
    const int buf = (int)(t & 1);
    if (t + 1 < nk) {
      loadA((t + 1) * GBK, ra);
      loadB((t + 1) * GBK, rb);
    }
#pragma unroll
    for (int kk = 0; kk < GBK; kk++) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (t + 1 < nk) {
      storeA(buf ^ 1, ra);
      storeB(buf ^ 1, rb);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= g.N) continue;
      float *cp = C + gm * g.ldc + gn;
      const float v = g.alpha * acc[i][j];
      *cp = g.beta == 0.0f ? v : fmaf(g.beta, *cp, v);
    }
  }
}

// --------------------------------------------------------------------------
// Cholesky building blocks (lower, in place, row-major n x n, leading dim ld)
constexpr int CB = 64;  // panel width

// Factor the CB x CB (or smaller) diagonal block at (k, k) in place; one CTA.
// info = 1 on a non-positive or non-finite pivot.
__global__ void __launch_bounds__(256) potrf_diag_kernel(float *A, int64_t ld, int64_t k, int b, int *info) {
  __shared__ float S[CB][CB + 1];
  const int tid = threadIdx.x;
  for (int e = tid; e < b * b; e += blockDim.x) S[e / b][e % b] = A[(k + e / b) * ld + k + e % b];
  __syncthreads();
  for (int j = 0; j < b; j++) {
    if (tid == 0) {
      const float p = S[j][j];
      if (!(p > 0.0f) || !isfinite(p)) {
        atomicExch(info, 1);
        S[j][j] = 1.0f;
      } else {
        S[j][j] = sqrtf(p);
      }
    }
    __syncthreads();
    const float djj = S[j][j];
    for (int i = j + 1 + tid; i < b; i += blockDim.x) S[i][j] = S[i][j] / djj;
    __syncthreads();
    // rank-1 update of the trailing lower part
    for (int e = tid; e < b * b; e += blockDim.x) {
      const int r = e / b, c = e % b;
      if (c > j && r >= c) S[r][c] = fmaf(-S[r][j], S[c][j], S[r][c]);
    }
    __syncthreads();
  }
  for (int e = tid; e < b * b; e += blockDim.x) {
    const int r = e / b, c = e % b;
    A[(k + r) * ld + k + c] = (c <= r) ? S[r][c] : 0.0f;
  }
}

// Rows below the diagonal block: X <- X * L_kk^-T (forward substitution per row).
__global__ void __launch_bounds__(128) trsm_panel_kernel(float *A, int64_t ld, int64_t n, int64_t k, int b) {
  __shared__ float Lk[CB][CB + 1];
  for (int e = threadIdx.x; e < b * b; e += blockDim.x) Lk[e / b][e % b] = A[(k + e / b) * ld + k + e % b];
  __syncthreads();
  const int64_t r = k + b + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  float x[CB];
  float *row = A + r * ld + k;
#pragma unroll
  for (int j = 0; j < CB; j++) x[j] = j < b ? row[j] : 0.0f;
#pragma unroll
  for (int j = 0; j < CB; j++) {
    if (j < b) {
      float s = x[j];
#pragma unroll
      for (int i = 0; i < j; i++) s = fmaf(-x[i], Lk[j][i], s);
      x[j] = s / Lk[j][j];
    }
  }
#pragma unroll
  for (int j = 0; j < CB; j++)
    if (j < b) row[j] = x[j];
}

// Factor (optional) and invert one lower-triangular block of b <= 128 rows in
// shared memory, one CTA of 1024 threads.
//   do_factor: A's b x b block (leading dim ld) is SPD: Cholesky in place
//   (right-looking, one column per step), L written back with zeros above the
//   diagonal; info = 1 on a non-positive pivot.  Otherwise A already holds L.
//   Then X = L^-1 by forward substitution, 8 lanes per column (warp shuffles,
//   columns are independent so only warp-level syncs are needed), written to
//   Linv (leading dim ldi; may alias A).
constexpr int PB = 128;
__global__ void __launch_bounds__(1024) potrf_inv128_kernel(float *A, int64_t ld, int b, float *Linv, int64_t ldi,
                                                            int *info, int mode) {
  const int do_factor = mode & 1, do_invert = mode & 2;
  extern __shared__ float sm[];
  float *S = sm;                   // [PB][PB + 1]
  float *X = sm + PB * (PB + 1);   // [PB][PB + 1]
  const int tid = threadIdx.x;
  for (int e = tid; e < b * b; e += blockDim.x) {
    const int r = e / b, c = e % b;
    S[r * (PB + 1) + c] = (c <= r) ? A[r * ld + c] : 0.0f;
  }
  __syncthreads();
  if (do_factor) {
    for (int j = 0; j < b; j++) {
      if (tid == 0) {
        const float p = S[j * (PB + 1) + j];
        if (!(p > 0.0f) || !isfinite(p)) {
          atomicExch(info, 1);
          S[j * (PB + 1) + j] = 1.0f;
        } else {
          S[j * (PB + 1) + j] = sqrtf(p);
        }
      }
      __syncthreads();
      const float djj = S[j * (PB + 1) + j];
      for (int i = j + 1 + tid; i < b; i += blockDim.x) S[i * (PB + 1) + j] = S[i * (PB + 1) + j] / djj;
      __syncthreads();
      // rank-1 update of the trailing lower triangle: thread (ty, tx) of a
      // 32 x 32 grid walks rows j+1+ty and columns j+1+tx in steps of 32
      const int tx = tid & 31, ty = tid >> 5;
      for (int r = j + 1 + ty; r < b; r += 32) {
        const float srj = S[r * (PB + 1) + j];
        for (int c = j + 1 + tx; c <= r; c += 32)
          S[r * (PB + 1) + c] = fmaf(-srj, S[c * (PB + 1) + j], S[r * (PB + 1) + c]);
      }
      __syncthreads();
    }
    for (int e = tid; e < b * b; e += blockDim.x) {
      const int r = e / b, c = e % b;
      A[r * ld + c] = (c <= r) ? S[r * (PB + 1) + c] : 0.0f;
    }
  }
  if (!do_invert) return;
  // inverse: column c = tid / 8, sub-lane sl = tid % 8
  const int c = tid >> 3, sl = tid & 7;
  for (int i = 0; i < b; i++) {
    float part = 0.0f;
    if (c < b && i > c)
      for (int j = c + sl; j < i; j += 8) part = fmaf(S[i * (PB + 1) + j], X[j * (PB + 1) + c], part);
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    if (sl == 0 && c < b) X[i * (PB + 1) + c] = (i < c) ? 0.0f : ((i == c ? 1.0f : 0.0f) - part) / S[i * (PB + 1) + i];
    __syncwarp();
  }
  __syncthreads();
  for (int e = tid; e < b * b; e += blockDim.x) {
    const int r = e / b, cc = e % b;
    Linv[r * ldi + cc] = (cc <= r) ? X[r * (PB + 1) + cc] : 0.0f;
  }
}

// mode bits: 1 = factor A in place, 2 = write L^-1 to Linv
static int potrf_inv128(float *A, int64_t ld, int b, float *Linv, int64_t ldi, int *info, int mode,
                        cudaStream_t s) {
  const int smem = (int)(2 * PB * (PB + 1) * sizeof(float));
  if (cudaFuncSetAttribute(potrf_inv128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  potrf_inv128_kernel<<<1, 1024, smem, s>>>(A, ld, b, Linv, ldi, info, mode);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// out[i][j] = in[n-1-i][n-1-j] (batched, square)
__global__ void reverse_square_kernel(const float *in, float *out, int64_t n, int64_t nn_total) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nn_total) return;
  const int64_t b = e / (n * n), r = (e / n) % n, c = e % n;
  out[e] = in[b * n * n + (n - 1 - r) * n + (n - 1 - c)];
}

// Add the reference's damping d = max(mean(diag), 1e-30) * damp to the diagonal
// (example/solution/solution.py:290-295), one CTA per matrix.
__global__ void __launch_bounds__(1024) damp_diag_kernel(float *A, int64_t n, float damp) {
  float *M = A + (int64_t)blockIdx.x * n * n;
  __shared__ float red[32];
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += M[i * n + i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float d = fmaxf(red[0] / (float)n, 1e-30f) * damp;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) M[i * n + i] += d;
}

__global__ void zero_upper_kernel(float *A, int64_t n, int64_t total) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= total) return;
  const int64_t r = (e / n) % n, c = e % n;
  if (c > r) A[e] = 0.0f;
}

// --------------------------------------------------------------------------
// GPTQ: one CTA of 128 threads per 128 rows; thread t owns row r0 + t.
// For the column block [i1, i1+nb): quantize column i to the unit grid
//   m = clamp(round(|w| / u * 4), 0, 7) * 0.25;  q = (w >= 0 ? 1 : -1) * m * u
// record E[:, i] = (w - q) / U[i][i] and propagate w[:, j] -= E[:, i] * U[i][j]
// for j > i inside the block (example/solution/solution.py:316-326).
constexpr int GQ_THREADS = 128;
constexpr int GQ_BLK = 128;
constexpr int GQW_WARPS = 8;   // rows per CTA in the warp-per-row kernel

// Warp-per-row form: lane l owns block columns l, l+32, l+64, l+96 in
// registers; column i's owner quantizes it and broadcasts the scaled error,
// every lane updates its own later columns.  U's block sits in shared memory.
__global__ void __launch_bounds__(GQW_WARPS * 32) gptq_block_warp_kernel(float *W, const float *unit, const float *U,
                                                                         float *Q, float *E, int64_t R, int64_t C,
                                                                         int64_t i1, int nb, int64_t bstride_rows,
                                                                         int64_t bstride_u) {
  extern __shared__ float Hs[];   // [nb][nb]
  const int64_t bz = blockIdx.y;
  W += bz * bstride_rows * C;
  unit += bz * bstride_rows * C;
  Q += bz * bstride_rows * C;
  E += bz * bstride_rows * GQ_BLK;
  U += bz * bstride_u;
  for (int e = threadIdx.x; e < nb * nb; e += blockDim.x) Hs[e] = U[(i1 + e / nb) * C + i1 + e % nb];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * GQW_WARPS + (threadIdx.x >> 5);
  if (r >= R) return;
  float w[4], u[4], q[4], err[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int c = lane + 32 * k;
    w[k] = c < nb ? W[r * C + i1 + c] : 0.0f;
    u[k] = c < nb ? unit[r * C + i1 + c] : 1.0f;
    q[k] = 0.0f;
    err[k] = 0.0f;
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    for (int ii = 0; ii < 32; ii++) {
      const int i = 32 * k + ii;
      if (i >= nb) break;
      float ei = 0.0f;
      if (lane == ii) {
        const float wi = w[k], ui = u[k];
        float m = rintf(__fmul_rn(__fdiv_rn(fabsf(wi), ui), 4.0f));
        m = __fmul_rn(fminf(fmaxf(m, 0.0f), 7.0f), 0.25f);
        const float qi = __fmul_rn(__fmul_rn(wi >= 0.0f ? 1.0f : -1.0f, m), ui);
        q[k] = qi;
        ei = __fdiv_rn(__fsub_rn(wi, qi), fmaxf(Hs[i * nb + i], 1e-30f));
        err[k] = ei;
      }
      ei = __shfl_sync(0xffffffffu, ei, ii);
      const float *hrow = Hs + i * nb;
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const int c = lane + 32 * kk;
        if (kk >= k && c > i && c < nb) w[kk] = fmaf(-ei, hrow[c], w[kk]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int c = lane + 32 * k;
    if (c < nb) {
      Q[r * C + i1 + c] = q[k];
      E[r * GQ_BLK + c] = err[k];
    }
  }
}

__global__ void __launch_bounds__(GQ_THREADS) gptq_block_kernel(float *W, const float *unit, const float *U,
                                                                  float *Q, float *E, int64_t R, int64_t C,
                                                                  int64_t i1, int nb, int64_t bstride_rows,
                                                                  int64_t bstride_u) {
  extern __shared__ float sm[];
  float *Hs = sm;                        // [nb][nb] block of U
  float *Ws = sm + GQ_BLK * GQ_BLK;      // [nb][GQ_THREADS] row slices, column-major per thread
  const int64_t bz = blockIdx.y;
  W += bz * bstride_rows * C;
  unit += bz * bstride_rows * C;
  Q += bz * bstride_rows * C;
  E += bz * bstride_rows * GQ_BLK;
  U += bz * bstride_u;
  const int t = threadIdx.x;
  for (int e = t; e < nb * nb; e += GQ_THREADS) Hs[e] = U[(i1 + e / nb) * C + i1 + e % nb];
  const int64_t r = (int64_t)blockIdx.x * GQ_THREADS + t;
  const bool live = r < R;
  if (live)
    for (int j = 0; j < nb; j++) Ws[j * GQ_THREADS + t] = W[r * C + i1 + j];
  __syncthreads();
  if (!live) return;
  for (int i = 0; i < nb; i++) {
    const float w = Ws[i * GQ_THREADS + t];
    const float u = unit[r * C + i1 + i];
    float m = rintf(__fmul_rn(__fdiv_rn(fabsf(w), u), 4.0f));
    m = __fmul_rn(fminf(fmaxf(m, 0.0f), 7.0f), 0.25f);
    const float q = __fmul_rn(__fmul_rn(w >= 0.0f ? 1.0f : -1.0f, m), u);
    Q[r * C + i1 + i] = q;
    const float dii = fmaxf(Hs[i * nb + i], 1e-30f);
    const float err = __fdiv_rn(__fsub_rn(w, q), dii);
    E[r * GQ_BLK + i] = err;
    for (int j = i + 1; j < nb; j++) Ws[j * GQ_THREADS + t] = fmaf(-err, Hs[i * nb + j], Ws[j * GQ_THREADS + t]);
  }
  for (int j = 0; j < nb; j++) W[r * C + i1 + j] = Ws[j * GQ_THREADS + t];
}

// --------------------------------------------------------------------------
// Greedy top-1 lattice refinement, one CTA per row (example/solution/
// solution.py:428-663): per round, over the row's C columns,
//   g = d^2 * G[c][c] - 2 d |M|,  legal if v4 stays in [-7, 7] moving against
//   the sign of M;  pick the smallest g (first index on ties); if g < 0 flip
//   v4[idx] += dr (dr = +1 if M[idx] < 0 else -1) and M += dr * d[idx] * G[idx].
// A row without an improving legal flip never flips again (its state does not
// change), so it stops.  Each thread owns RC columns in registers.
constexpr int RC = 8;

__global__ void __launch_bounds__(1024) refine_rows_kernel(float *M, float *v4, const float *d, const float *G,
                                                           int64_t T, int64_t C, int rounds, int *flips) {
  __shared__ float rg[32];
  __shared__ int ri[32];
  __shared__ float s_coef;
  __shared__ int s_idx;
  const int64_t row = blockIdx.x;
  if (row >= T) return;
  const int t = threadIdx.x;
  const int nthr = blockDim.x;
  float m[RC], v[RC], dd[RC], d2c[RC];
#pragma unroll
  for (int k = 0; k < RC; k++) {
    const int64_t c = (int64_t)k * nthr + t;
    if (c < C) {
      m[k] = M[row * C + c];
      v[k] = v4[row * C + c];
      dd[k] = d[row * C + c];
      d2c[k] = __fmul_rn(__fmul_rn(dd[k], dd[k]), G[c * C + c]);
    } else {
      m[k] = 0.0f; v[k] = 0.0f; dd[k] = 0.0f; d2c[k] = 0.0f;
    }
  }
  int nflip = 0;
  for (int rd = 0; rd < rounds; rd++) {
    float best = INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int k = 0; k < RC; k++) {
      const int64_t c = (int64_t)k * nthr + t;
      if (c < C) {
        const bool up = m[k] < 0.0f;
        const bool ill = up ? (v[k] >= 7.0f) : (v[k] <= -7.0f);
        const float g = ill ? INFINITY : fmaf(fabsf(m[k]), -2.0f * dd[k], d2c[k]);
        if (g < best) { best = g; bi = (int)c; }
      }
    }
    // block argmin, smallest index on ties
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float og = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (og < best || (og == best && oi < bi)) { best = og; bi = oi; }
    }
    if ((t & 31) == 0) { rg[t >> 5] = best; ri[t >> 5] = bi; }
    __syncthreads();
    if (t < 32) {
      float b2 = t < (nthr >> 5) ? rg[t] : INFINITY;
      int i2 = t < (nthr >> 5) ? ri[t] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float og = __shfl_xor_sync(0xffffffffu, b2, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i2, o);
        if (og < b2 || (og == b2 && oi < i2)) { b2 = og; i2 = oi; }
      }
      if (t == 0) { s_idx = (b2 < 0.0f) ? i2 : -1; }
    }
    __syncthreads();
    const int idx = s_idx;
    if (idx < 0) break;  // frozen row
    // owner applies the flip and publishes the coefficient
    if (idx % nthr == t) {
      const int k = idx / nthr;
#pragma unroll
      for (int kk = 0; kk < RC; kk++)
        if (kk == k) {
          const float dr = m[kk] < 0.0f ? 1.0f : -1.0f;
          v[kk] += dr;
          s_coef = dr * dd[kk];
        }
    }
    __syncthreads();
    const float coef = s_coef;
    const float *gr = G + (int64_t)idx * C;
#pragma unroll
    for (int k = 0; k < RC; k++) {
      const int64_t c = (int64_t)k * nthr + t;
      if (c < C) m[k] = fmaf(coef, __ldg(gr + c), m[k]);
    }
    nflip++;
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < RC; k++) {
    const int64_t c = (int64_t)k * nthr + t;
    if (c < C) {
      M[row * C + c] = m[k];
      v4[row * C + c] = v[k];
    }
  }
  if (t == 0 && flips != nullptr) flips[row] = nflip;
}

}  // namespace hif4x

// ====================================================================== ABI
using namespace hif4x;

static inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

extern "C" int hif4x_gemm_tc(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
                             int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc,
                             void *stream);

extern "C" int hif4x_gemm_simt(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
                               int64_t lda, int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta,
                               float *C, int64_t ldc, int64_t strideC, int64_t batch, void *stream);
int hif4x_gemm_tc_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                     const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int lower, void *stream);
static int gemm_simt_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                        int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                        int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream);

// Products of at least this many multiply-adds go to the tensor cores.
static const int64_t kTcMinMacs = int64_t(1) << 26;

static int gemm_dispatch(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                         int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                         int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream);

static bool tc_disabled() {
  static const bool off = [] {
    const char *e = getenv("HIF4X_GEMM");
    return e != nullptr && e[0] == 's';  // HIF4X_GEMM=simt selects the SIMT kernel for every product
  }();
  return off;
}

extern "C" int hif4x_gemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                          int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                          int64_t ldc, int64_t strideC, int64_t batch, void *stream) {
  if (M < 0 || N < 0 || K < 0 || batch < 0) return HIF4X_ERR_ARG;
  if (M == 0 || N == 0 || batch == 0) return HIF4X_OK;
  if (!A || !B || !C || batch > 65535) return HIF4X_ERR_ARG;
  return gemm_dispatch(ta, tb, M, N, K, alpha, A, lda, strideA, B, ldb, strideB, beta, C, ldc, strideC, batch, 0,
                       stream);
}

static int gemm_dispatch(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                         int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                         int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream) {
  if (batch == 1 && K >= 64 && M * N * K >= kTcMinMacs && !tc_disabled()) {
    const int st = hif4x_gemm_tc_ex(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, lower, stream);
    if (st != HIF4X_ERR_UNSUPPORTED) return st;
  }
  return gemm_simt_ex(ta, tb, M, N, K, alpha, A, lda, strideA, B, ldb, strideB, beta, C, ldc, strideC, batch, lower,
                      stream);
}

extern "C" int hif4x_gemm_simt(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
                               int64_t lda, int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta,
                               float *C, int64_t ldc, int64_t strideC, int64_t batch, void *stream) {
  return gemm_simt_ex(ta, tb, M, N, K, alpha, A, lda, strideA, B, ldb, strideB, beta, C, ldc, strideC, batch, 0,
                      stream);
}

static int gemm_simt_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                        int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                        int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream) {
  if (M < 0 || N < 0 || K < 0 || batch < 0) return HIF4X_ERR_ARG;
  if (M == 0 || N == 0 || batch == 0) return HIF4X_OK;
  if (!A || !B || !C || batch > 65535) return HIF4X_ERR_ARG;
  GemmArgs g{ta, tb, M, N, K, alpha, beta, A, lda, strideA, B, ldb, strideB, C, ldc, strideC, lower};
  dim3 grid(nblk(N, GBN), nblk(M, GBM), (unsigned)batch);
  if (grid.y > 65535) return HIF4X_ERR_ARG;
  gemm_kernel<<<grid, GTHREADS, 0, (cudaStream_t)stream>>>(g);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// Lower Cholesky in place of the n x n block at A (row-major, leading dim
// ld), blocked right-looking with 64-wide panels.
static int potrf_lower_ld(float *A, int64_t n, int64_t ld, int *info_dev, cudaStream_t s) {
  for (int64_t k = 0; k < n; k += CB) {
    const int b = (int)std::min<int64_t>(CB, n - k);
    potrf_diag_kernel<<<1, 256, 0, s>>>(A, ld, k, b, info_dev);
    const int64_t rest = n - k - b;
    if (rest > 0) {
      trsm_panel_kernel<<<nblk(rest, 128), 128, 0, s>>>(A, ld, n, k, b);
      // trailing update A22 -= P P^T  (P = A[k+b:, k:k+b])
      const float *P = A + (k + b) * ld + k;
      int st = hif4x_gemm(0, 1, rest, rest, b, -1.0f, P, ld, 0, P, ld, 0, 1.0f, A + (k + b) * ld + (k + b), ld, 0, 1, s);
      if (st) return st;
    }
  }
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

static int potrf_lower(float *A, int64_t n, int *info_dev, cudaStream_t s) {
  return potrf_lower_ld(A, n, n, info_dev, s);
}

// dst (rows x cols, ldd) = src (lds); zero_upper clears dst[i][j] for j > i.
__global__ void copy2d_kernel(const float *src, int64_t lds, float *dst, int64_t ldd, int64_t rows, int64_t cols,
                              int zero_upper) {
  const int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (e >= rows * cols) return;
  const int64_t r = e / cols, c = e % cols;
  dst[r * ldd + c] = (zero_upper && c > r) ? 0.0f : src[r * lds + c];
}

static int trtri_lower(float *A, int64_t n, int64_t ld, float *work, cudaStream_t s);

// Recursive lower Cholesky in place of the n x n block at A (leading dim ld):
//   L11 = chol(A11);  L21 = A21 L11^-T;  L22 = chol(A22 - L21 L21^T).
// L21 is one GEMM against L11's inverse and the update one large-K GEMM over
// the lower-triangle tiles, so almost all flops run as big tensor-core GEMMs;
// leaves of <= 128 rows are factored in shared memory by one CTA.  The upper
// triangle is left stale (cleared by the caller).
// Split n1 = n/2 rounded down to a multiple of 128 (at least 128), so
// n1 <= n/2 and the workspace n1*n1 + max(n2*n1, n1*n1/4) is at most n*n/2
// floats (the recursive calls reuse it after this level is done with it).
static int potrf_rec(float *A, int64_t n, int64_t ld, int *info_dev, float *work, cudaStream_t s) {
  if (n <= PB) return potrf_inv128(A, ld, (int)n, nullptr, 0, info_dev, 1, s);
  const int64_t n1 = std::max<int64_t>(PB, (n / 2 / PB) * PB), n2 = n - n1;
  float *A11 = A, *A21 = A + n1 * ld, *A22 = A + n1 * ld + n1;
  int st = potrf_rec(A11, n1, ld, info_dev, work, s);
  if (st) return st;
  float *Linv = work;             // n1 x n1
  float *T = work + n1 * n1;      // n2 x n1, and trtri's n1*n1/4 scratch before that
  copy2d_kernel<<<nblk(n1 * n1, 256), 256, 0, s>>>(A11, ld, Linv, n1, n1, n1, 1);
  st = trtri_lower(Linv, n1, n1, T, s);
  if (st) return st;
  st = gemm_dispatch(0, 1, n2, n1, n1, 1.0f, A21, ld, 0, Linv, n1, 0, 0.0f, T, n1, 0, 1, 0, s);   // T = A21 L11^-T
  if (st) return st;
  copy2d_kernel<<<nblk(n2 * n1, 256), 256, 0, s>>>(T, n1, A21, ld, n2, n1, 0);
  st = gemm_dispatch(0, 1, n2, n2, n1, -1.0f, A21, ld, 0, A21, ld, 0, 1.0f, A22, ld, 0, 1, 1, s);
  if (st) return st;
  return potrf_rec(A22, n2, ld, info_dev, work, s);
}

// In-place inverse of a lower-triangular n x n block at A (leading dim ld):
// inv([[A11, 0], [A21, A22]]) = [[A11^-1, 0], [-A22^-1 A21 A11^-1, A22^-1]].
static int trtri_lower(float *A, int64_t n, int64_t ld, float *work, cudaStream_t s) {
  if (n <= PB) return potrf_inv128(A, ld, (int)n, A, ld, nullptr, 2, s);
  int64_t n1 = ((n / 2 + PB - 1) / PB) * PB;
  const int64_t n2 = n - n1;
  float *A11 = A, *A21 = A + n1 * ld, *A22 = A + n1 * ld + n1;
  int st = trtri_lower(A11, n1, ld, work, s);
  if (st) return st;
  st = trtri_lower(A22, n2, ld, work, s);
  if (st) return st;
  // T = A21 * A11^-1  (n2 x n1) into work; A21 = -A22^-1 * T
  st = hif4x_gemm(0, 0, n2, n1, n1, 1.0f, A21, ld, 0, A11, ld, 0, 0.0f, work, n1, 0, 1, s);
  if (st) return st;
  return hif4x_gemm(0, 0, n2, n1, n2, -1.0f, A22, ld, 0, work, n1, 0, 0.0f, A21, ld, 0, 1, s);
}

extern "C" int hif4x_chol_upper_inv(const float *H, int64_t n, int64_t batch, float damp, float *U, float *work,
                                    int *info_dev, void *stream) {
  if (n <= 0 || batch <= 0 || !H || !U || !work || !info_dev) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nn = n * n;
  if (cudaMemsetAsync(info_dev, 0, sizeof(int), s) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  // work: [nn] reversed matrix per batch element + [nn] scratch for trtri
  for (int64_t b = 0; b < batch; b++) {
    float *P = work;
    float *scratch = work + nn;
    reverse_square_kernel<<<nblk(nn, 256), 256, 0, s>>>(H + b * nn, P, n, nn);
    damp_diag_kernel<<<1, 1024, 0, s>>>(P, n, damp);
    int st;
    if (n <= PB) {
      st = potrf_inv128(P, n, (int)n, P, n, info_dev, 3, s);   // L^-1 in place
      if (st) return st;
    } else {
      st = potrf_rec(P, n, n, info_dev, scratch, s);
      if (st) return st;
      zero_upper_kernel<<<nblk(nn, 256), 256, 0, s>>>(P, n, nn);
      st = trtri_lower(P, n, n, scratch, s);
      if (st) return st;
    }
    reverse_square_kernel<<<nblk(nn, 256), 256, 0, s>>>(P, U + b * nn, n, nn);
  }
  HIF4X_CHECK_LAUNCH();
  int info = 0;
  if (cudaMemcpyAsync(&info, info_dev, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  return info ? HIF4X_NOT_PD : HIF4X_OK;
}

extern "C" int hif4x_gptq(const float *X, const float *unit, const float *U, int64_t R, int64_t C, int64_t batch,
                          int64_t u_batch_stride, float *Q, float *work, void *stream) {
  if (R < 0 || C <= 0 || batch <= 0) return HIF4X_ERR_ARG;
  if (R == 0) return HIF4X_OK;
  if (!X || !unit || !U || !Q || !work) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  // work: W (batch*R*C) followed by E (batch*R*128)
  float *W = work;
  float *E = work + batch * R * C;
  if (cudaMemcpyAsync(W, X, sizeof(float) * batch * R * C, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  const size_t smem = sizeof(float) * GQ_BLK * GQ_BLK;
  if (cudaFuncSetAttribute(gptq_block_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  for (int64_t i1 = 0; i1 < C; i1 += GQ_BLK) {
    const int nb = (int)std::min<int64_t>(GQ_BLK, C - i1);
    dim3 grid(nblk(R, GQW_WARPS), (unsigned)batch);
    gptq_block_warp_kernel<<<grid, GQW_WARPS * 32, smem, s>>>(W, unit, U, Q, E, R, C, i1, nb, R, u_batch_stride);
    HIF4X_CHECK_LAUNCH();
    const int64_t i2 = i1 + nb;
    if (i2 < C) {
      // W[:, i2:] -= E1 @ U[i1:i2, i2:]
      int st = hif4x_gemm(0, 0, R, C - i2, nb, -1.0f, E, GQ_BLK, R * GQ_BLK, U + i1 * C + i2, C, u_batch_stride,
                          1.0f, W + i2, C, R * C, batch, s);
      if (st) return st;
    }
  }
  return HIF4X_OK;
}

extern "C" int hif4x_refine_rows(float *M, float *v4, const float *d, const float *G, int64_t T, int64_t C,
                                 int rounds, int *flips, void *stream) {
  if (T < 0 || C <= 0 || rounds < 0) return HIF4X_ERR_ARG;
  if (T == 0 || rounds == 0) return HIF4X_OK;
  if (!M || !v4 || !d || !G) return HIF4X_ERR_ARG;
  int threads = (int)((C + RC - 1) / RC);
  threads = ((threads + 31) / 32) * 32;
  if (threads > 1024) return HIF4X_ERR_UNSUPPORTED;  // C > 8192
  if (T > 0x7fffffff) return HIF4X_ERR_ARG;
  refine_rows_kernel<<<(unsigned)T, threads, 0, (cudaStream_t)stream>>>(M, v4, d, G, T, C, rounds, flips);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// ====================================================================== no-allocation variant
// hif4x_chol_upper_inv_noalloc: the same damped Cholesky -> upper factor of
// the inverse, for callers that cannot allocate device memory at the call
// (a host whose device memory is planned up front by another runtime, or a
// latency-bound loop that must not call the allocator, which can synchronise
// the device).  Its scratch is a file-scope device array of fixed size, so
// it takes no work or info buffers: n is limited to kNoAllocMaxN.
//
// Host code cannot pass the array's name to a kernel (in host code that name
// is a host-side stand-in, not a device address), so the first call on each
// device resolves the device address with cudaGetSymbolAddress while that
// device is current and caches it; make that first call before any stream
// capture.  All calls share the one array: calls that overlap on the GPU
// (different streams or host threads at once) race on it.
#include <mutex>

namespace {
constexpr int64_t kNoAllocMaxN = 512;
constexpr int kNoAllocMaxDevices = 64;
// [0, n*n): index-reversed damped matrix, later L and L^-1; [n*n, 2*n*n): trtri work
static __device__ __align__(256) float g_chol_noalloc_scratch[2 * kNoAllocMaxN * kNoAllocMaxN];
// [0]: non-positive-pivot flag (cleared at the start of every call)
static __device__ __align__(256) int g_chol_noalloc_info[64];

struct NoAllocPtrs {
  float *scratch;
  int *info;
  bool ready;
};
NoAllocPtrs g_noalloc_ptrs[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

int noalloc_device_ptrs(float **scratch, int **info) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return HIF4X_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocPtrs &p = g_noalloc_ptrs[dev];
  if (!p.ready) {
    void *s = nullptr, *i = nullptr;
    if (cudaGetSymbolAddress(&s, g_chol_noalloc_scratch) != cudaSuccess) return HIF4X_ERR_LAUNCH;
    if (cudaGetSymbolAddress(&i, g_chol_noalloc_info) != cudaSuccess) return HIF4X_ERR_LAUNCH;
    p.scratch = static_cast<float *>(s);
    p.info = static_cast<int *>(i);
    p.ready = true;
  }
  *scratch = p.scratch;
  *info = p.info;
  return HIF4X_OK;
}
}  // namespace

extern "C" int hif4x_chol_upper_inv_noalloc(const float *H, int64_t n, int64_t batch, float damp, float *U,
                                            void *stream) {
  if (n <= 0 || batch <= 0 || !H || !U) return HIF4X_ERR_ARG;
  if (n > kNoAllocMaxN) return HIF4X_ERR_SCRATCH;
  float *scratch = nullptr;
  int *info_dev = nullptr;
  int st = noalloc_device_ptrs(&scratch, &info_dev);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nn = n * n;
  if (cudaMemsetAsync(info_dev, 0, sizeof(int), s) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  for (int64_t b = 0; b < batch; b++) {
    float *P = scratch;
    float *work = scratch + nn;
    reverse_square_kernel<<<nblk(nn, 256), 256, 0, s>>>(H + b * nn, P, n, nn);
    damp_diag_kernel<<<1, 1024, 0, s>>>(P, n, damp);
    st = potrf_lower(P, n, info_dev, s);
    if (st) return st;
    zero_upper_kernel<<<nblk(nn, 256), 256, 0, s>>>(P, n, nn);
    st = trtri_lower(P, n, n, work, s);
    if (st) return st;
    reverse_square_kernel<<<nblk(nn, 256), 256, 0, s>>>(P, U + b * nn, n, nn);
  }
  HIF4X_CHECK_LAUNCH();
  int info = 0;
  if (cudaMemcpyAsync(&info, info_dev, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  return info ? HIF4X_NOT_PD : HIF4X_OK;
}
