// linalg.cu -- fp32 dense linear algebra for the calibration pipeline:
//   * strided-batched GEMM  C = alpha * op(A) op(B) + beta * C  (row-major)
//   * damped Cholesky -> upper factor of the inverse (GPTQ's Hinv)
//   * GPTQ column-sequential quantize-and-propagate inside a column block
//
// Products of at least 2^26 multiply-adds go to the tensor-core GEMM
// (gemm_tc.cu, 3xTF32); smaller ones, and the products whose results are
// differenced (hif4x_gemm_simt), run the register-tiled SIMT kernels here
// (128x128x8 CTA tile with 8x8 per thread, or 32x32 tiles for small
// products), fp32 in and out with sequential fp32 FMA accumulation.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

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

// Small products: 32 x 32 output tiles so that a 128-sized product still
// spreads over 16 SMs, K in chunks of 64 (one global-memory round trip per
// chunk instead of one per 8), 2 x 2 outputs per thread.  Each output is the
// same sequential fp32 FMA chain over k as in gemm_kernel.
constexpr int SBM = 32, SBN = 32, SKC = 64, STHREADS = 256;

__global__ void __launch_bounds__(STHREADS, 2) gemm_small_kernel(const GemmArgs g) {
  __shared__ float As[SKC][SBM + 1];   // As[k][m]
  __shared__ float Bs[SKC][SBN + 1];   // Bs[k][n]
  const int64_t bz = blockIdx.z;
  const float *A = g.A + bz * g.sA;
  const float *B = g.B + bz * g.sB;
  float *C = g.C + bz * g.sC;
  const int64_t m0 = (int64_t)blockIdx.y * SBM, n0 = (int64_t)blockIdx.x * SBN;
  if (g.lower && n0 > m0 + SBM - 1) return;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  constexpr int PER = SBM * SKC / STHREADS;   // 8 elements of each operand per thread and chunk
  float ra[PER], rb[PER];
  auto load = [&](int64_t k0) {
#pragma unroll
    for (int r = 0; r < PER; r++) {
      const int e = tid + r * STHREADS;
      int mm, kk, nn, kb;
      if (g.ta) { kk = e / SBM; mm = e % SBM; } else { mm = e / SKC; kk = e % SKC; }
      if (g.tb) { nn = e / SKC; kb = e % SKC; } else { kb = e / SBN; nn = e % SBN; }
      const int64_t gm = m0 + mm, gka = k0 + kk, gn = n0 + nn, gkb = k0 + kb;
      ra[r] = (gm < g.M && gka < g.K) ? (g.ta ? A[gka * g.lda + gm] : A[gm * g.lda + gka]) : 0.0f;
      rb[r] = (gn < g.N && gkb < g.K) ? (g.tb ? B[gn * g.ldb + gkb] : B[gkb * g.ldb + gn]) : 0.0f;
    }
  };
  auto store = [&]() {
#pragma unroll
    for (int r = 0; r < PER; r++) {
      const int e = tid + r * STHREADS;
      int mm, kk, nn, kb;
      if (g.ta) { kk = e / SBM; mm = e % SBM; } else { mm = e / SKC; kk = e % SKC; }
      if (g.tb) { nn = e / SKC; kb = e % SKC; } else { kb = e / SBN; nn = e % SBN; }
      As[kk][mm] = ra[r];
      Bs[kb][nn] = rb[r];
    }
  };
  float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
  const int64_t nk = (g.K + SKC - 1) / SKC;
  load(0);
  store();
  __syncthreads();
  for (int64_t t = 0; t < nk; t++) {
    if (t + 1 < nk) load((t + 1) * SKC);
#pragma unroll 16
    for (int kk = 0; kk < SKC; kk++) {
      const float a0 = As[kk][ty], a1 = As[kk][ty + 16];
      const float b0 = Bs[kk][tx], b1 = Bs[kk][tx + 16];
      acc[0][0] = fmaf(a0, b0, acc[0][0]);
      acc[0][1] = fmaf(a0, b1, acc[0][1]);
      acc[1][0] = fmaf(a1, b0, acc[1][0]);
      acc[1][1] = fmaf(a1, b1, acc[1][1]);
    }
    __syncthreads();
    if (t + 1 < nk) {
      store();
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int64_t gm = m0 + ty + 16 * i;
    if (gm >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int64_t gn = n0 + tx + 16 * j;
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
// shared memory, one CTA of 256 threads, in 32-column panels.
//   mode 1 (factor): A's b x b block (leading dim ld) is SPD: Cholesky in
//   shared memory; info = 1 on a non-positive pivot (the pivot is then taken
//   as 1).  Without it A already holds L.
//   mode 2 (invert): X = L^-1 written to Linv (leading dim ldi; may alias A).
//   mode 4 (keep): L written back to A, zeros above the diagonal.
// The block is padded with the identity to bp = b rounded up to 32, which
// leaves the b x b results unchanged and makes every diagonal block a full
// 32 x 32 one, so the unrolled per-warp code below carries no bounds tests.
// Per panel p (columns c0 .. c0+32): all threads factor the diagonal block,
// one warp inverts it (lane c owns column c of the inverse); the rows below are
// L21 = A21 L11^-T, a product with that inverse; the trailing lower triangle
// gets the rank-32 update A22 -= L21 L21^T in 4 x 4 register tiles.  The
// inverse's off-diagonal blocks then follow block-row by block-row:
//   X_pq = -X_pp (sum_{k=q}^{p-1} L_pk X_kq).
constexpr int PB = 128;
constexpr int LP = 32;                  // panel width
constexpr int LTHREADS = 256;
constexpr int LDS = PB + 1;             // shared-memory row pitch (floats)
constexpr int LDT = PB - LP + 1;        // pitch of the T scratch (32 x 96)

// One warp: X[c0.., c0..] = inverse of the 32 x 32 lower block of S at
// (c0, c0), given rdiag = 1 / L[c0+lane][c0+lane] in each lane.  Lane c
// computes column c by right-looking substitution: step k fixes
// x_k = acc_k / L_kk and removes it from every later row, so each step is one
// multiply followed by independent FMAs (entries above the diagonal come out
// as zero).
__device__ __forceinline__ void leaf_diag_invert(const float *S, float *X, int c0, int lane, float rdiag) {
  float acc[LP], rd[LP];
#pragma unroll
  for (int i = 0; i < LP; i++) {
    acc[i] = (i == lane) ? 1.0f : 0.0f;
    rd[i] = __shfl_sync(0xffffffffu, rdiag, i);
  }
#pragma unroll
  for (int k = 0; k < LP; k++) {
    const float xk = acc[k] * rd[k];
    acc[k] = xk;
#pragma unroll
    for (int i = k + 1; i < LP; i++) acc[i] = fmaf(-S[(c0 + i) * LDS + c0 + k], xk, acc[i]);
  }
#pragma unroll
  for (int i = 0; i < LP; i++) X[(c0 + i) * LDS + c0 + lane] = acc[i];
}

// All threads: Cholesky of the 32 x 32 block of S at (c0, c0) in place
// (lower), then (warp 0) its inverse into X.  Right-looking on unscaled
// columns: step j subtracts S[i][j] S[k][j] / S[j][j] from the trailing
// triangle (one barrier per step, at most 4 elements per thread), and the
// columns are scaled by 1 / sqrt(pivot) at the end.  A non-positive or
// non-finite pivot sets info and is taken as 1.
__device__ __forceinline__ void leaf_diag_factor(float *S, float *X, int c0, int tid, int *info) {
  for (int j = 0; j < LP; j++) {
    const float piv = S[(c0 + j) * LDS + c0 + j];
    const bool bad = !(piv > 0.0f) || !isfinite(piv);
    const float rp = bad ? 1.0f : __fdividef(1.0f, piv);
    // element e = tid + 256 q of the rows below j: row j + 1 + e / 32, column e % 32
#pragma unroll
    for (int q = 0; q < LP * LP / LTHREADS; q++) {
      const int e = tid + LTHREADS * q, i = j + 1 + e / LP, k = e % LP;
      if (i < LP && k > j && k <= i)
        S[(c0 + i) * LDS + c0 + k] = fmaf(-S[(c0 + i) * LDS + c0 + j] * rp, S[(c0 + k) * LDS + c0 + j],
                                          S[(c0 + i) * LDS + c0 + k]);
    }
    __syncthreads();
    if (tid == 0 && bad) {
      if (info) atomicExch(info, 1);
      S[(c0 + j) * LDS + c0 + j] = 1.0f;
    }
  }
  __syncthreads();
  // scale: L[i][j] = S[i][j] / sqrt(S[j][j]) (i > j), L[j][j] = sqrt(S[j][j])
  float v[LP * LP / LTHREADS];
#pragma unroll
  for (int q = 0; q < LP * LP / LTHREADS; q++) {
    const int e = tid + LTHREADS * q, i = e / LP, j = e % LP;
    const float piv = S[(c0 + j) * LDS + c0 + j];
    v[q] = (j == i) ? sqrtf(piv) : (j < i ? S[(c0 + i) * LDS + c0 + j] * rsqrtf(piv) : 0.0f);
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < LP * LP / LTHREADS; q++) {
    const int e = tid + LTHREADS * q, i = e / LP, j = e % LP;
    S[(c0 + i) * LDS + c0 + j] = v[q];
  }
  __syncthreads();
  if (tid < 32) leaf_diag_invert(S, X, c0, tid, 1.0f / S[(c0 + tid) * LDS + c0 + tid]);
}

__global__ void __launch_bounds__(LTHREADS, 1) potrf_inv128_kernel(float *A, int64_t ld, int b, float *Linv,
                                                                   int64_t ldi, int *info, int mode) {
  const int do_factor = mode & 1, do_invert = mode & 2;
  extern __shared__ float sm[];
  float *S = sm;                   // [PB][LDS]  L (lower; zeros above)
  float *X = sm + PB * LDS;        // [PB][LDS]  L^-1
  float *T = X + PB * LDS;         // [LP][LDT]  block-row scratch of the inverse
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = LTHREADS / 32;
  constexpr int PER = PB * PB / LTHREADS;
  const int bp = (b + LP - 1) / LP * LP;
  {
    float v[PER];
#pragma unroll
    for (int q = 0; q < PER; q++) {
      const int e = tid + LTHREADS * q, r = e / PB, c = e % PB;
      v[q] = (r < b && c <= r) ? A[r * ld + c] : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < PER; q++) {
      const int e = tid + LTHREADS * q, r = e / PB, c = e % PB;
      S[r * LDS + c] = (r >= b && r == c) ? 1.0f : v[q];
      X[r * LDS + c] = 0.0f;
    }
  }
  __syncthreads();
  const int np = bp / LP;
  if (do_factor) {
    for (int p = 0; p < np; p++) {
      const int c0 = p * LP;
      leaf_diag_factor(S, X, c0, tid, info);
      __syncthreads();
      const int r0 = c0 + LP, nr = bp - r0;
      if (nr <= 0) break;
      // L21 = A21 * X11^T (nr <= 96 rows x 32 columns): thread (rg, cg), rg < 24,
      // cg < 8, owns rows r0 + rg + 24a and columns c0 + cg + 8c (a, c < 4);
      // X11 is zero above its diagonal, so k runs over the whole panel
      {
        const int rg = tid >> 3, cg = tid & 7;
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int c = 0; c < 4; c++) acc[a][c] = 0.0f;
        if (rg < 24) {
#pragma unroll 4
          for (int k = 0; k < LP; k++) {
            float av[4], xv[4];
#pragma unroll
            for (int a = 0; a < 4; a++) {
              const int i = r0 + rg + 24 * a;
              av[a] = i < bp ? S[i * LDS + c0 + k] : 0.0f;
              xv[a] = X[(c0 + cg + 8 * a) * LDS + c0 + k];
            }
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
              for (int c = 0; c < 4; c++) acc[a][c] = fmaf(av[a], xv[c], acc[a][c]);
          }
        }
        __syncthreads();
        if (rg < 24) {
#pragma unroll
          for (int a = 0; a < 4; a++) {
            const int i = r0 + rg + 24 * a;
            if (i < bp) {
#pragma unroll
              for (int c = 0; c < 4; c++) S[i * LDS + c0 + cg + 8 * c] = acc[a][c];
            }
          }
        }
      }
      __syncthreads();
      // A22 -= L21 L21^T on the lower triangle: warp tiles of 16 rows x 32
      // columns, lane = 4 x 4 register tile (rows 4*(lane/8), cols 4*(lane%8))
      const int wtr = nr / 16, wtc = nr / 32;
      for (int wt = warp; wt < wtr * wtc; wt += NW) {
        const int wr = wt / wtc, wc = wt % wtc;
        if (wc * 32 > wr * 16 + 15) continue;   // entirely above the diagonal
        const int i0 = r0 + wr * 16 + 4 * (lane >> 3), k0 = r0 + wc * 32 + 4 * (lane & 7);
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int c = 0; c < 4; c++) acc[a][c] = 0.0f;
#pragma unroll 4
        for (int j = 0; j < LP; j++) {
          float li[4], lk[4];
#pragma unroll
          for (int a = 0; a < 4; a++) {
            li[a] = S[(i0 + a) * LDS + c0 + j];
            lk[a] = S[(k0 + a) * LDS + c0 + j];
          }
#pragma unroll
          for (int a = 0; a < 4; a++)
#pragma unroll
            for (int c = 0; c < 4; c++) acc[a][c] = fmaf(li[a], lk[c], acc[a][c]);
        }
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const int i = i0 + a, k = k0 + c;
            if (k <= i) S[i * LDS + k] -= acc[a][c];
          }
      }
      __syncthreads();
    }
    if (mode & 4) {
#pragma unroll 8
      for (int q = 0; q < PER; q++) {
        const int e = tid + LTHREADS * q, r = e / PB, c = e % PB;
        if (r < b && c < b) A[r * ld + c] = (c <= r) ? S[r * LDS + c] : 0.0f;
      }
    }
  } else if (do_invert) {
    if (warp < np) {
      const int c0 = warp * LP;
      leaf_diag_invert(S, X, c0, lane, 1.0f / S[(c0 + lane) * LDS + c0 + lane]);
    }
    __syncthreads();
  }
  if (!do_invert) return;
  // off-diagonal blocks of the inverse, block-row p = 1 .. np-1; thread
  // (rg, cg), rg < 8, cg < 8p, owns rows rg + 8a and columns cg + 8p*c
  for (int p = 1; p < np; p++) {
    const int c0 = p * LP, cs = 8 * p;
    const int rg = tid / cs, cg = tid % cs;
    const bool act = rg < 8;
    float acc[4][4];
    // T[i][c] = sum_{k<c0} L[c0+i][k] X[k][c]   (X[k][c] = 0 for k < c)
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int c = 0; c < 4; c++) acc[a][c] = 0.0f;
    if (act) {
#pragma unroll 4
      for (int k = cg; k < c0; k++) {
        float lv[4], xv[4];
#pragma unroll
        for (int a = 0; a < 4; a++) {
          lv[a] = S[(c0 + rg + 8 * a) * LDS + k];
          xv[a] = X[k * LDS + cg + cs * a];
        }
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int c = 0; c < 4; c++) acc[a][c] = fmaf(lv[a], xv[c], acc[a][c]);
      }
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) T[(rg + 8 * a) * LDT + cg + cs * c] = acc[a][c];
    }
    __syncthreads();
    // X[c0+i][c] = -sum_m X[c0+i][c0+m] T[m][c]   (X_pp is lower)
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int c = 0; c < 4; c++) acc[a][c] = 0.0f;
    if (act) {
#pragma unroll 4
      for (int m = 0; m < LP; m++) {
        float xv[4], tv[4];
#pragma unroll
        for (int a = 0; a < 4; a++) {
          xv[a] = X[(c0 + rg + 8 * a) * LDS + c0 + m];
          tv[a] = T[m * LDT + cg + cs * a];
        }
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int c = 0; c < 4; c++) acc[a][c] = fmaf(xv[a], tv[c], acc[a][c]);
      }
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) X[(c0 + rg + 8 * a) * LDS + cg + cs * c] = -acc[a][c];
    }
    __syncthreads();
  }
#pragma unroll 8
  for (int q = 0; q < PER; q++) {
    const int e = tid + LTHREADS * q, r = e / PB, c = e % PB;
    if (r < b && c < b) Linv[r * ldi + c] = (c <= r) ? X[r * LDS + c] : 0.0f;
  }
}

// mode bits: 1 = factor A, 2 = write L^-1 to Linv, 4 = write L back to A
static int potrf_inv128(float *A, int64_t ld, int b, float *Linv, int64_t ldi, int *info, int mode,
                        cudaStream_t s) {
  const int smem = (int)((2 * PB * LDS + LP * LDT) * sizeof(float));
  // the shared-memory opt-in, once per device (a Cholesky calls this for every 128-row leaf)
  constexpr int kDevs = 64;
  static std::once_flag attr_once[kDevs];
  static bool attr_ok[kDevs];
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevs) return HIF4X_ERR_LAUNCH;
  std::call_once(attr_once[dev], [dev, smem] {
    attr_ok[dev] = cudaFuncSetAttribute(potrf_inv128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
                   cudaSuccess;
  });
  if (!attr_ok[dev]) return HIF4X_ERR_LAUNCH;
  potrf_inv128_kernel<<<1, LTHREADS, smem, s>>>(A, ld, b, Linv, ldi, info, mode);
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

// J X J in place for an n x n row-major X: element e <-> element n*n - 1 - e
__global__ void reverse_flat_kernel(float *X, int64_t nn) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nn / 2) return;
  const float a = X[e];
  X[e] = X[nn - 1 - e];
  X[nn - 1 - e] = a;
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
// GPTQ, one 128-column block at a time (kernels below, trailing update as a
// GEMM in hif4x_gptq).  For the column block [i1, i1+nb): quantize column i
// to the unit grid
//   m = clamp(round(|w| / u * 4), 0, 7) * 0.25;  q = (w >= 0 ? 1 : -1) * m * u
// record E[:, i] = (w - q) / U[i][i] and propagate w[:, j] -= E[:, i] * U[i][j]
// for j > i inside the block (example/solution/solution.py:316-326).  Every
// step rounds as the reference's elementwise torch/numpy ops do: the
// propagation is a rounded product then a rounded subtraction, never an FMA.
constexpr int GQ_BLK = 128;
constexpr int GQW_WARPS = 8;   // warps per CTA of the GPTQ block kernels

// U's nb x nb diagonal block at (i1, i1) into shared memory (row-major, nb
// per row).  A full 128-column block on 16-byte-aligned rows goes as 16
// independent float4 loads per thread (no index division): the small-input
// GPTQ launches run a few CTAs and were waiting on exactly this load.
__device__ __forceinline__ void gptq_load_u_block(float *Hs, const float *U, int64_t C, int64_t i1, int nb) {
  const float *base = U + i1 * C + i1;
  if (nb == GQ_BLK && (C & 3) == 0 && (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && blockDim.x == 256) {
    float4 v[16];
#pragma unroll
    for (int q = 0; q < 16; q++) {
      const int e = threadIdx.x + 256 * q;   // float4 index: row e / 32, column 4 (e % 32)
      v[q] = __ldg(reinterpret_cast<const float4 *>(base + (int64_t)(e >> 5) * C) + (e & 31));
    }
#pragma unroll
    for (int q = 0; q < 16; q++) reinterpret_cast<float4 *>(Hs)[threadIdx.x + 256 * q] = v[q];
    return;
  }
  for (int e = threadIdx.x; e < nb * nb; e += blockDim.x) Hs[e] = U[(i1 + e / nb) * C + i1 + e % nb];
}

// One-row-per-warp form for small inputs (proxies, hold-outs, short dynamic
// calls, a few thousand weight rows), where latency, not issue, sets the time.
// Lane l holds block columns l, l+32, l+64, l+96 of the warp's row.  For
// column i the owner's value is broadcast first and every lane rounds it (the
// warp issues the rounding once either way, without a divergent branch or a
// second shuffle); the unit, U[i][i] and U's row are loaded a column ahead.
// The operations and their order are those of the row-exchange kernel below,
// so the results are identical.
__global__ void __launch_bounds__(GQW_WARPS * 32) gptq_block_row_kernel(float *W, const float *unit, const float *U,
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
  gptq_load_u_block(Hs, U, C, i1, nb);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * GQW_WARPS + (threadIdx.x >> 5);
  if (r >= R) return;
  float w[4], qk[4], ek[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int c = lane + 32 * k;
    w[k] = c < nb ? W[r * C + i1 + c] : 0.0f;
    qk[k] = 0.0f;
    ek[k] = 0.0f;
  }
  const float *urow = unit + r * C + i1;
  float u_next = __ldg(urow);
  float h_next = Hs[0];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    for (int ii = 0; ii < 32; ii++) {
      const int i = 32 * k + ii;
      if (i >= nb) break;
      const float ui = u_next, hii = fmaxf(h_next, 1e-30f);
      if (i + 1 < nb) {
        u_next = __ldg(urow + i + 1);
        h_next = Hs[(i + 1) * nb + i + 1];
      }
      const float *hrow = Hs + i * nb;
      float hv[4];
#pragma unroll
      for (int kk = 0; kk < 4; kk++) hv[kk] = (kk >= k && lane + 32 * kk < nb) ? hrow[lane + 32 * kk] : 0.0f;
      const float wi = __shfl_sync(0xffffffffu, w[k], ii);
      float m = rintf(__fmul_rn(__fdiv_rn(fabsf(wi), ui), 4.0f));
      m = __fmul_rn(fminf(fmaxf(m, 0.0f), 7.0f), 0.25f);
      const float qi = __fmul_rn(__fmul_rn(wi >= 0.0f ? 1.0f : -1.0f, m), ui);
      const float ei = __fdiv_rn(__fsub_rn(wi, qi), hii);
      if (lane == ii) {
        qk[k] = qi;
        ek[k] = ei;
      }
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const int c = lane + 32 * kk;
        if (kk >= k && c > i && c < nb) w[kk] = __fsub_rn(w[kk], __fmul_rn(ei, hv[kk]));
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int c = lane + 32 * k;
    if (c < nb) {
      Q[r * C + i1 + c] = qk[k];
      E[r * GQ_BLK + c] = ek[k];
    }
  }
}

// Row-exchange form for large row counts: each warp owns RW rows (RW <= 16);
// lane l holds block columns l, l+32, l+64, l+96 of all of them.  For column
// i the owner lane publishes its RW values through shared memory, lanes
// 0..RW-1 quantize one row each (the warp issues the quantisation once, not
// once per row), publish the scaled errors back, and every lane updates its
// later columns.  Same operations in the same order as
// gptq_block_row_kernel, so the results are identical.
constexpr int GQX_MAXRW = 16;
template <int RW>
__global__ void __launch_bounds__(GQW_WARPS * 32) gptq_block_xch_kernel(float *W, const float *unit, const float *U,
                                                                        float *Q, float *E, int64_t R, int64_t C,
                                                                        int64_t i1, int nb, int64_t bstride_rows,
                                                                        int64_t bstride_u) {
  extern __shared__ float Hs[];   // [nb][nb], then per warp [RW] column values + [RW] errors
  const int64_t bz = blockIdx.y;
  W += bz * bstride_rows * C;
  unit += bz * bstride_rows * C;
  Q += bz * bstride_rows * C;
  E += bz * bstride_rows * GQ_BLK;
  U += bz * bstride_u;
  gptq_load_u_block(Hs, U, C, i1, nb);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *xw = Hs + GQ_BLK * GQ_BLK + warp * (2 * GQX_MAXRW);
  float *xe = xw + GQX_MAXRW;
  const int64_t r0 = ((int64_t)blockIdx.x * GQW_WARPS + warp) * RW;
  if (r0 >= R) return;
  float w[RW][4];
#pragma unroll
  for (int rr = 0; rr < RW; rr++) {
    const int64_t r = r0 + rr;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int c = lane + 32 * k;
      w[rr][k] = (r < R && c < nb) ? W[r * C + i1 + c] : 0.0f;
    }
  }
  const int64_t rq = r0 + lane;             // the row this lane quantizes (lanes < RW)
  const bool qlane = lane < RW;
  const bool qrow = qlane && rq < R;
  const float *urow = unit + (qrow ? rq : 0) * C + i1;
  float u_next = qrow ? __ldg(urow) : 1.0f;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    for (int ii = 0; ii < 32; ii++) {
      const int i = 32 * k + ii;
      if (i >= nb) break;
      if (lane == ii) {
#pragma unroll
        for (int rr = 0; rr < RW; rr += 4)
          *reinterpret_cast<float4 *>(xw + rr) = make_float4(w[rr][k], w[rr + 1][k], w[rr + 2][k], w[rr + 3][k]);
      }
      __syncwarp();
      if (qlane) {
        const float ui = u_next;
        if (qrow && i + 1 < nb) u_next = __ldg(urow + i + 1);
        float ei = 0.0f;
        if (qrow) {
          const float wi = xw[lane];
          const float hii = fmaxf(Hs[i * nb + i], 1e-30f);
          float m = rintf(__fmul_rn(__fdiv_rn(fabsf(wi), ui), 4.0f));
          m = __fmul_rn(fminf(fmaxf(m, 0.0f), 7.0f), 0.25f);
          const float qi = __fmul_rn(__fmul_rn(wi >= 0.0f ? 1.0f : -1.0f, m), ui);
          ei = __fdiv_rn(__fsub_rn(wi, qi), hii);
          Q[rq * C + i1 + i] = qi;
          E[rq * GQ_BLK + i] = ei;
        }
        xe[lane] = ei;
      }
      __syncwarp();
      float ev[RW];
#pragma unroll
      for (int rr = 0; rr < RW; rr += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xe + rr);
        ev[rr] = v.x; ev[rr + 1] = v.y; ev[rr + 2] = v.z; ev[rr + 3] = v.w;
      }
      const float *hrow = Hs + i * nb;
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const int c = lane + 32 * kk;
        if (kk >= k && c > i && c < nb) {
          const float h = hrow[c];
#pragma unroll
          for (int rr = 0; rr < RW; rr++) w[rr][kk] = __fsub_rn(w[rr][kk], __fmul_rn(ev[rr], h));
        }
      }
    }
  }
}

// --------------------------------------------------------------------------
// Greedy top-1 lattice refinement, one CTA per row (example/solution/
// solution.py:428-663): per round, over the row's C columns,
//   g = d^2 * G[c][c] - 2 d |M|,  legal if v4 stays in [-7, 7] moving against
//   the sign of M;  pick the smallest g (first index on ties); if g < 0 flip
//   v4[idx] += dr (dr = +1 if M[idx] < 0 else -1) and M += dr * d[idx] * G[idx].
// A row without an improving legal flip never flips again (its state does not
// change), so it stops.  Each thread owns RC columns in registers.
// Both g = d2col + |M|*(-2d) and M += coef*G[idx] are a rounded product then
// a rounded sum, as the reference's addcmul / numpy ops on the CPU (no FMA,
// solution.py:474-521, 541-546, 595), so near-ties resolve as they do there.
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
        const float g = ill ? INFINITY : __fadd_rn(__fmul_rn(fabsf(m[k]), -2.0f * dd[k]), d2c[k]);
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
      if (c < C) m[k] = __fadd_rn(m[k], __fmul_rn(coef, __ldg(gr + c)));
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
                     const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int lower, int kmode,
                     void *stream);
static int gemm_simt_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                        int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                        int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream);

// Products of at least this many multiply-adds go to the tensor cores;
// smaller ones (per batch element) take the SIMT kernels.  Measured alone on
// one B200: 256 x 3968 x 128 (a GPTQ trailing update of 256 rows) 16 us on
// the tensor cores against 32 us SIMT, 512 x 384 x 384 21 against 25 us;
// 256^3 12 us SIMT against 18 us (the tensor-core call's two operand splits
// and its launch dominate there).
static const int64_t kTcMinMacs = int64_t(1) << 26;
static const int64_t kSmallMaxMacs = int64_t(1) << 27;

static int gemm_dispatch(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                         int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                         int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream, int kmode = 0);

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
                         int64_t ldc, int64_t strideC, int64_t batch, int lower, void *stream, int kmode) {
  if (batch == 1 && K >= 64 && M * N * K >= kTcMinMacs && !tc_disabled()) {
    const int st = hif4x_gemm_tc_ex(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, lower, kmode, stream);
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
  if (M * N * K < kSmallMaxMacs) {
    dim3 grid(nblk(N, SBN), nblk(M, SBM), (unsigned)batch);
    if (grid.y > 65535) return HIF4X_ERR_ARG;
    gemm_small_kernel<<<grid, STHREADS, 0, (cudaStream_t)stream>>>(g);
    HIF4X_CHECK_LAUNCH();
    return HIF4X_OK;
  }
  dim3 grid(nblk(N, GBN), nblk(M, GBM), (unsigned)batch);
  if (grid.y > 65535) return HIF4X_ERR_ARG;
  gemm_kernel<<<grid, GTHREADS, 0, (cudaStream_t)stream>>>(g);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// Lower Cholesky in place of the n x n block at A (row-major, leading dim
// ld), blocked right-looking with 64-wide panels.  Used only by the
// allocation-free entry point: its products call the SIMT GEMM directly, never
// the tensor-core path (which allocates its split operands), whatever the
// dispatch thresholds are.
static int potrf_lower_ld(float *A, int64_t n, int64_t ld, int *info_dev, cudaStream_t s) {
  for (int64_t k = 0; k < n; k += CB) {
    const int b = (int)std::min<int64_t>(CB, n - k);
    potrf_diag_kernel<<<1, 256, 0, s>>>(A, ld, k, b, info_dev);
    const int64_t rest = n - k - b;
    if (rest > 0) {
      trsm_panel_kernel<<<nblk(rest, 128), 128, 0, s>>>(A, ld, n, k, b);
      // trailing update A22 -= P P^T  (P = A[k+b:, k:k+b])
      const float *P = A + (k + b) * ld + k;
      int st = gemm_simt_ex(0, 1, rest, rest, b, -1.0f, P, ld, 0, P, ld, 0, 1.0f, A + (k + b) * ld + (k + b), ld, 0,
                            1, 0, s);
      if (st) return st;
    }
  }
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

static int potrf_lower(float *A, int64_t n, int *info_dev, cudaStream_t s) {
  return potrf_lower_ld(A, n, n, info_dev, s);
}

static int trtri_lower(float *A, int64_t n, int64_t ld, float *work, cudaStream_t s);

// Recursive lower Cholesky that carries the inverse along, for the n x n
// block at A (leading dim ld) and the block at Inv (leading dim ldi):
//   L11 = chol(A11), L11^-1            recursively
//   L21 = A21 L11^-T                   one GEMM, into Inv21 (still free)
//   A22 -= L21 L21^T                   large-K GEMM over the lower tiles
//   L22 = chol(A22), L22^-1            recursively
//   Inv21 = -L22^-1 (L21 L11^-1)       two GEMMs (T = L21 L11^-1 in work)
// so L^-1 = [[L11^-1, 0], [Inv21, L22^-1]] is built without a separate
// triangular inverse, and all flops but the 128-row leaves (factor and
// inverse fused in shared memory by one CTA) run as GEMMs.  A keeps Schur
// complements, not the factor.  Inv must be zero above the diagonal on entry.
// Split n1 = n/2 rounded down to a multiple of 128 (at least 128).
//
// T = L21 L11^-1 depends only on L21 and L11^-1, not on A22's factorisation,
// so it runs on a second stream (`side`) from the moment L21 exists, beside
// the A22 update and recursion, whose leaves and small products leave most
// SMs idle; the caller's stream waits for it before the last product.  Each
// recursion depth has its own T buffer (work: n2 x n1 here, the deeper
// depths after it; about n*n/3 floats in all), because a T of this depth is
// still needed while the deeper calls compute theirs.
struct CholSide {
  cudaStream_t s = nullptr;
  cudaEvent_t l21 = nullptr;          // L21 written (recorded on the caller's stream)
  cudaEvent_t t[32] = {};             // T of depth d written (recorded on s)
};

static CholSide *chol_side(cudaStream_t main) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, CholSide *> sides;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  auto it = sides.find({dev, main});
  if (it != sides.end()) return it->second;
  CholSide *c = new CholSide();
  int prio = 0;
  bool ok = cudaStreamGetPriority(main, &prio) == cudaSuccess &&
            cudaStreamCreateWithPriority(&c->s, cudaStreamNonBlocking, prio) == cudaSuccess &&
            cudaEventCreateWithFlags(&c->l21, cudaEventDisableTiming) == cudaSuccess;
  for (int d = 0; ok && d < 32; d++) ok = cudaEventCreateWithFlags(&c->t[d], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return nullptr;   // the recursion then runs every product on the caller's stream
  }
  sides[{dev, main}] = c;
  return c;
}

static int potrf_inv_rec(float *A, int64_t n, int64_t ld, float *Inv, int64_t ldi, int *info_dev, float *work,
                         cudaStream_t s, CholSide *side, int depth) {
  if (n <= PB) return potrf_inv128(A, ld, (int)n, Inv, ldi, info_dev, 3, s);
  const int64_t n1 = std::max<int64_t>(PB, (n / 2 / PB) * PB), n2 = n - n1;
  float *A21 = A + n1 * ld, *A22 = A + n1 * ld + n1;
  float *I11 = Inv, *I21 = Inv + n1 * ldi, *I22 = Inv + n1 * ldi + n1;
  float *T = work, *deeper = work + n2 * n1;
  int st = potrf_inv_rec(A, n1, ld, I11, ldi, info_dev, deeper, s, side, depth + 1);
  if (st) return st;
  // L11^-1 and L22^-1 are lower triangular (zeros above the diagonal in
  // memory): kmode lets the tensor-core products skip their zero K-steps
  st = gemm_dispatch(0, 1, n2, n1, n1, 1.0f, A21, ld, 0, I11, ldi, 0, 0.0f, I21, ldi, 0, 1, 0, s, 1);
  if (st) return st;
  const bool overlap = side != nullptr && depth < 32;
  if (overlap) {
    if (cudaEventRecord(side->l21, s) != cudaSuccess || cudaStreamWaitEvent(side->s, side->l21, 0) != cudaSuccess)
      return HIF4X_ERR_LAUNCH;
    st = gemm_dispatch(0, 0, n2, n1, n1, 1.0f, I21, ldi, 0, I11, ldi, 0, 0.0f, T, n1, 0, 1, 0, side->s, 2);
    if (st) return st;
    if (cudaEventRecord(side->t[depth], side->s) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  }
  st = gemm_dispatch(0, 1, n2, n2, n1, -1.0f, I21, ldi, 0, I21, ldi, 0, 1.0f, A22, ld, 0, 1, 1, s);
  if (st) return st;
  st = potrf_inv_rec(A22, n2, ld, I22, ldi, info_dev, deeper, s, side, depth + 1);
  if (st) return st;
  if (overlap) {
    if (cudaStreamWaitEvent(s, side->t[depth], 0) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  } else {
    st = gemm_dispatch(0, 0, n2, n1, n1, 1.0f, I21, ldi, 0, I11, ldi, 0, 0.0f, T, n1, 0, 1, 0, s, 2);
    if (st) return st;
  }
  return gemm_dispatch(0, 0, n2, n1, n2, -1.0f, I22, ldi, 0, T, n1, 0, 0.0f, I21, ldi, 0, 1, 0, s, 3);
}

// In-place inverse of a lower-triangular n x n block at A (leading dim ld):
// inv([[A11, 0], [A21, A22]]) = [[A11^-1, 0], [-A22^-1 A21 A11^-1, A22^-1]].
// Allocation-free entry point only; SIMT products, as potrf_lower_ld.
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
  st = gemm_simt_ex(0, 0, n2, n1, n1, 1.0f, A21, ld, 0, A11, ld, 0, 0.0f, work, n1, 0, 1, 0, s);
  if (st) return st;
  return gemm_simt_ex(0, 0, n2, n1, n2, -1.0f, A22, ld, 0, work, n1, 0, 0.0f, A21, ld, 0, 1, 0, s);
}

extern "C" int hif4x_chol_upper_inv_async(const float *H, int64_t n, int64_t batch, float damp, float *U,
                                          float *work, int *info_dev, void *stream) {
  if (n <= 0 || batch <= 0 || !H || !U || !work || !info_dev) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nn = n * n;
  if (cudaMemsetAsync(info_dev, 0, sizeof(int), s) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  // work: [nn] reversed damped matrix (overwritten by Schur complements) +
  // the recursion's T buffers (<= nn/3 + n*128); L^-1 is built in U itself and
  // reversed in place.
  CholSide *side = n > PB ? chol_side(s) : nullptr;
  for (int64_t b = 0; b < batch; b++) {
    float *P = work;
    float *Inv = U + b * nn;
    reverse_square_kernel<<<nblk(nn, 256), 256, 0, s>>>(H + b * nn, P, n, nn);
    damp_diag_kernel<<<1, 1024, 0, s>>>(P, n, damp);
    if (cudaMemsetAsync(Inv, 0, (size_t)nn * sizeof(float), s) != cudaSuccess) return HIF4X_ERR_LAUNCH;
    const int st = potrf_inv_rec(P, n, n, Inv, n, info_dev, work + nn, s, side, 0);
    if (st) return st;
    reverse_flat_kernel<<<nblk((nn + 1) / 2, 256), 256, 0, s>>>(Inv, nn);
  }
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_chol_upper_inv(const float *H, int64_t n, int64_t batch, float damp, float *U, float *work,
                                    int *info_dev, void *stream) {
  const int st = hif4x_chol_upper_inv_async(H, n, batch, damp, U, work, info_dev, stream);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
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
  const size_t smem_x = smem + sizeof(float) * GQW_WARPS * 2 * GQX_MAXRW;
  // rows per warp: the most (16, 8, 4 with the row-exchange kernel) that still
  // leaves about eight warps per SM; 1 (gptq_block_row_kernel) for small inputs
  const int64_t rows_all = R * batch;
  const int rw = rows_all >= (int64_t)16 * 8 * 148 ? 16 : rows_all >= (int64_t)8 * 8 * 148 ? 8
               : rows_all >= (int64_t)4 * 8 * 148 ? 4 : 1;
  if (cudaFuncSetAttribute(gptq_block_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess ||
      cudaFuncSetAttribute(gptq_block_xch_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_x) !=
          cudaSuccess ||
      cudaFuncSetAttribute(gptq_block_xch_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_x) !=
          cudaSuccess ||
      cudaFuncSetAttribute(gptq_block_xch_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_x) !=
          cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  for (int64_t i1 = 0; i1 < C; i1 += GQ_BLK) {
    const int nb = (int)std::min<int64_t>(GQ_BLK, C - i1);
    const dim3 block(GQW_WARPS * 32);
    if (rw == 16)
      gptq_block_xch_kernel<16><<<dim3(nblk(R, GQW_WARPS * 16), (unsigned)batch), block, smem_x, s>>>(
          W, unit, U, Q, E, R, C, i1, nb, R, u_batch_stride);
    else if (rw == 8)
      gptq_block_xch_kernel<8><<<dim3(nblk(R, GQW_WARPS * 8), (unsigned)batch), block, smem_x, s>>>(
          W, unit, U, Q, E, R, C, i1, nb, R, u_batch_stride);
    else if (rw == 4)
      gptq_block_xch_kernel<4><<<dim3(nblk(R, GQW_WARPS * 4), (unsigned)batch), block, smem_x, s>>>(
          W, unit, U, Q, E, R, C, i1, nb, R, u_batch_stride);
    else
      gptq_block_row_kernel<<<dim3(nblk(R, GQW_WARPS), (unsigned)batch), block, smem, s>>>(
          W, unit, U, Q, E, R, C, i1, nb, R, u_batch_stride);
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

// --------------------------------------------------------------------------
// The upper factor of the rotated space from the unrotated one.
//
// The rotated Hessian is H1 = M^T H0 M, M the block-diagonal orthogonal
// rotation of _rot_blocks (64 x 64 blocks H64/8 with column signs;
// solution.py:222-245), and the damping is the same in both spaces (the mean
// diagonal is the trace over n, which M preserves).  So H1_d^-1 = M^T H0_d^-1 M
// = (U0 M)^T (U0 M), and U1 = chol_upper(H1_d^-1) is the R factor (positive
// diagonal) of a QR decomposition of Y = U0 M.  Y is U0 with each row's
// 64-blocks rotated: upper triangular except for dense 64 x 64 diagonal
// blocks D_b.  With D_b = Q_b R_b, Q = diag(Q_b) gives Q^T Y upper triangular,
// so U1 = [R_b on the diagonal, Q_b^T Y[b, c] above it]: 64 independent
// Householder QRs of 64 x 64 blocks and (n/64)^2/2 products of 64 x 64 blocks
// (about 64 n^2 multiply-adds) in place of a Gram of the rotated activations
// and a second Cholesky-inverse (about n^3).

// One CTA per 64 x 64 diagonal block of Y (leading dim n): Householder QR in
// shared memory (LAPACK's reflector convention), the explicit Q_b written to
// Qw[b] (row-major 64 x 64), R_b written over the block with zeros below the
// diagonal; rows of R_b with a negative diagonal are negated together with
// the matching columns of Q_b, so the factor's diagonal is positive.
__global__ void __launch_bounds__(256) block_qr64_kernel(float *Y, int64_t n, float *Qw) {
  // A: the block, then R above the diagonal and reflector k below it in
  // column k (its leading 1 implicit); Qs: the explicit Q_b
  __shared__ float A[64][65];
  __shared__ float Qs[64][65];
  __shared__ float tau[64], w[64], red[2];
  const int64_t b = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float *D = Y + (b * 64) * n + b * 64;
  for (int e = t; e < 4096; e += 256) A[e >> 6][e & 63] = D[(int64_t)(e >> 6) * n + (e & 63)];
  __syncthreads();
  for (int k = 0; k < 64; k++) {
    if (warp == 0) {
      // sigma = sum_{i > k} A[i][k]^2
      const int i0 = k + 1 + lane, i1 = k + 33 + lane;
      const float x0 = i0 < 64 ? A[i0][k] : 0.0f, x1 = i1 < 64 ? A[i1][k] : 0.0f;
      float sq = x0 * x0 + x1 * x1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      const float alpha = A[k][k];
      float tk = 0.0f, scale = 0.0f, beta = alpha;
      if (sq > 0.0f) {
        beta = -copysignf(sqrtf(alpha * alpha + sq), alpha);
        tk = (beta - alpha) / beta;
        scale = 1.0f / (alpha - beta);
      }
      __syncwarp();
      if (i0 < 64) A[i0][k] = x0 * scale;
      if (i1 < 64) A[i1][k] = x1 * scale;
      if (lane == 0) {
        tau[k] = tk;
        red[0] = beta;
      }
    }
    __syncthreads();
    // w_j = sum_{i >= k} v_i A[i][j] for j > k: four threads per column
    {
      const int j = t >> 2, part = t & 3;
      float acc = 0.0f;
      if (j > k)
        for (int i = k + part; i < 64; i += 4) acc = fmaf(i == k ? 1.0f : A[i][k], A[i][j], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (part == 0) w[j] = acc;
    }
    __syncthreads();
    const float tk = tau[k];
    for (int e = t; e < 4096; e += 256) {
      const int i = e >> 6, j = e & 63;
      if (i >= k && j > k) A[i][j] = fmaf(-tk * (i == k ? 1.0f : A[i][k]), w[j], A[i][j]);
    }
    if (t == 0) A[k][k] = red[0];
    __syncthreads();
  }
  // Q = H_0 H_1 ... H_63 I, accumulated backwards: Q <- H_k Q on rows k..63
  for (int e = t; e < 4096; e += 256) Qs[e >> 6][e & 63] = (e >> 6) == (e & 63) ? 1.0f : 0.0f;
  __syncthreads();
  for (int k = 63; k >= 0; k--) {
    {
      const int j = t >> 2, part = t & 3;
      float acc = 0.0f;
      for (int i = k + part; i < 64; i += 4) acc = fmaf(i == k ? 1.0f : A[i][k], Qs[i][j], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (part == 0) w[j] = acc;
    }
    __syncthreads();
    const float tk = tau[k];
    for (int e = t; e < 4096; e += 256) {
      const int i = e >> 6, j = e & 63;
      if (i >= k) Qs[i][j] = fmaf(-tk * (i == k ? 1.0f : A[i][k]), w[j], Qs[i][j]);
    }
    __syncthreads();
  }
  // positive diagonal: negate row k of R and column k of Q where R[k][k] < 0
  float *Q = Qw + b * 4096;
  for (int e = t; e < 4096; e += 256) {
    const int i = e >> 6, j = e & 63;
    const float rs = A[i][i] < 0.0f ? -1.0f : 1.0f;   // row i of R
    const float qs = A[j][j] < 0.0f ? -1.0f : 1.0f;   // column j of Q
    D[(int64_t)i * n + j] = j >= i ? rs * A[i][j] : 0.0f;
    Q[e] = qs * Qs[i][j];
  }
}

// Y[b, c] <- Q_b^T Y[b, c] for every 64 x 64 block above the diagonal
// (c > b), in place: one CTA per block, 4 x 4 outputs per thread.
__global__ void __launch_bounds__(256) block_qt_apply_kernel(float *Y, int64_t n, const float *Qw) {
  const int64_t c = blockIdx.x, b = blockIdx.y;
  if (c <= b) return;
  __shared__ float Qt[64][65];   // Qt[k][i] = Q_b[i][k]
  __shared__ float X[64][65];
  const int t = threadIdx.x;
  float *blk = Y + (b * 64) * n + c * 64;
  const float *Q = Qw + b * 4096;
  for (int e = t; e < 4096; e += 256) {
    const int i = e >> 6, j = e & 63;
    Qt[j][i] = Q[e];
    X[i][j] = blk[(int64_t)i * n + j];
  }
  __syncthreads();
  const int r0 = (t >> 4) * 4, c0 = (t & 15) * 4;
  float acc[4][4] = {};
  for (int i = 0; i < 64; i++) {
    float qv[4], xv[4];
#pragma unroll
    for (int a = 0; a < 4; a++) qv[a] = Qt[r0 + a][i];
#pragma unroll
    for (int d = 0; d < 4; d++) xv[d] = X[i][c0 + d];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int d = 0; d < 4; d++) acc[a][d] = fmaf(qv[a], xv[d], acc[a][d]);
  }
#pragma unroll
  for (int a = 0; a < 4; a++)
    *reinterpret_cast<float4 *>(blk + (int64_t)(r0 + a) * n + c0) = make_float4(acc[a][0], acc[a][1], acc[a][2],
                                                                                  acc[a][3]);
}

extern "C" int hif4x_rotate64(const float *x, const uint64_t *signs, int64_t rows, int64_t cols, float *out,
                              void *stream);

extern "C" int hif4x_chol_rotate64(const float *U0, int64_t n, const uint64_t *signs, float *U1, float *work,
                                   void *stream) {
  if (n <= 0 || n % 64 != 0 || !U0 || !signs || !U1 || !work || U0 == U1) return HIF4X_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(U1) & 15u) != 0) return HIF4X_ERR_ARG;
  const int64_t nb = n / 64;
  if (nb > 65535) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  int st = hif4x_rotate64(U0, signs, n, n, U1, stream);   // Y = U0 M, row by row
  if (st) return st;
  block_qr64_kernel<<<(unsigned)nb, 256, 0, s>>>(U1, n, work);
  block_qt_apply_kernel<<<dim3((unsigned)nb, (unsigned)nb), 256, 0, s>>>(U1, n, work);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// Copy the lower triangle of the n x n matrix G (leading dim ld) onto its
// upper triangle, one 32 x 32 tile pair per block through shared memory (both
// the tile read and the transposed write coalesced); blocks above the
// diagonal exit at once.
__global__ void mirror_lower_kernel(float *G, int64_t n, int64_t ld) {
  __shared__ float tile[32][33];
  const int64_t bi = blockIdx.y, bj = blockIdx.x;   // source tile (bi, bj), bi >= bj
  if (bj > bi) return;
  const int tx = threadIdx.x, ty = threadIdx.y;     // 32 x 8
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int64_t r = bi * 32 + ty + 8 * k, c = bj * 32 + tx;
    tile[ty + 8 * k][tx] = (r < n && c < n) ? G[r * ld + c] : 0.0f;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int64_t r = bj * 32 + ty + 8 * k, c = bi * 32 + tx;   // destination (r, c) = source (c, r)
    if (r < n && c < n && c > r) G[r * ld + c] = tile[tx][ty + 8 * k];
  }
}

// G = X^T X + beta G for X (T x C, leading dim ldx): only the output tiles on
// or below the diagonal are computed (about half the multiply-adds of the
// full product), then the lower triangle is mirrored, so G is exactly
// symmetric.  Large products on the tensor cores, small ones on the SIMT
// kernels, as hif4x_gemm.
extern "C" int hif4x_gram(const float *X, int64_t T, int64_t C, int64_t ldx, float beta, float *G, int64_t ldg,
                          void *stream) {
  if (T < 0 || C < 0 || ldx < C || ldg < C) return HIF4X_ERR_ARG;
  if (C == 0) return HIF4X_OK;
  if (!G || (T > 0 && !X)) return HIF4X_ERR_ARG;   // an empty X may have no storage
  cudaStream_t s = (cudaStream_t)stream;
  if (T == 0) {   // an empty sum: G stays (beta = 1) or becomes zero (beta = 0)
    if (beta == 1.0f) return HIF4X_OK;
    if (beta != 0.0f) return HIF4X_ERR_UNSUPPORTED;
    return cudaMemset2DAsync(G, (size_t)ldg * sizeof(float), 0, (size_t)C * sizeof(float), (size_t)C, s) ==
                   cudaSuccess ? HIF4X_OK : HIF4X_ERR_LAUNCH;
  }
  int st = gemm_dispatch(1, 0, C, C, T, 1.0f, X, ldx, 0, X, ldx, 0, beta, G, ldg, 0, 1, 1, s);
  if (st) return st;
  const int64_t nt = (C + 31) / 32;
  if (nt > 65535) return HIF4X_ERR_ARG;
  mirror_lower_kernel<<<dim3((unsigned)nt, (unsigned)nt), dim3(32, 8), 0, s>>>(G, C, ldg);
  HIF4X_CHECK_LAUNCH();
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
// device is current and caches it per device ordinal (the runtime's primary
// context of that device; a caller that makes another driver context current
// must not use this entry point).  Every call ends by copying the pivot flag
// to the host and synchronising its stream, so no call can be part of a
// stream capture.  All calls share the one array: calls that overlap on the
// GPU (different streams or host threads at once) race on it.  It computes the
// same factor as hif4x_chol_upper_inv in a different order (blocked Cholesky,
// then a triangular inverse), so the two agree to float rounding, not bit for
// bit.
#include <mutex>

namespace {
constexpr int64_t kNoAllocMaxN = 512;
constexpr int kNoAllocMaxDevices = 64;
// [0, n*n): index-reversed damped matrix, later L and L^-1; [n*n, 2*n*n): trtri work
// (its largest product needs n2*n1 <= n*n/4 floats)
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
