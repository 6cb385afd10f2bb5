// attention.cu -- fp32 GQA softmax attention and head-layout transposes for
// the attention calibration path (example/solution/solution.py:1120-1258).
//
// attention_kernel: out = softmax(Q_h K_g^T / sqrt(dh)) V_g per query head h,
// kv head g = h / (qh / kvh), non-causal, fp32 throughout, online softmax over
// 64-key tiles.  One CTA per (head, 64-query tile), 256 threads: thread
// (ty, tx) owns score rows 4ty..4ty+3 x cols 4tx..4tx+3 and output rows
// 4ty..4ty+3 x head-dim cols 8tx..8tx+7 (dh <= 128).
#include <algorithm>

#include "common.cuh"
#include "tc_gemm.cuh"

namespace hif4x {

constexpr int AT = 64;       // query / key tile
constexpr int ADH = 128;     // max head dim

__global__ void __launch_bounds__(256) attention_kernel(const float *Q, const float *K, const float *V, int64_t T,
                                                        int qh, int kvh, int dh, float scale, float *O) {
  extern __shared__ float sm[];
  float *Qs = sm;                    // [AT][ADH + 1]
  float *Ks = Qs + AT * (ADH + 1);   // [AT][ADH + 1]
  float *Vs = Ks + AT * (ADH + 1);   // [AT][ADH]
  float *Ps = Vs + AT * ADH;         // [AT][AT + 1]
  const int h = blockIdx.y;
  const int g = h / (qh / kvh);
  const int64_t q0 = (int64_t)blockIdx.x * AT;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t ldq = (int64_t)qh * dh, ldk = (int64_t)kvh * dh;
  for (int e = tid; e < AT * dh; e += 256) {
    const int r = e / dh, c = e % dh;
    Qs[r * (ADH + 1) + c] = (q0 + r < T) ? Q[(q0 + r) * ldq + (int64_t)h * dh + c] : 0.0f;
  }
  float m[4], l[4], o[4][8];
#pragma unroll
  for (int a = 0; a < 4; a++) {
    m[a] = -INFINITY;
    l[a] = 0.0f;
#pragma unroll
    for (int b = 0; b < 8; b++) o[a][b] = 0.0f;
  }
  for (int64_t k0 = 0; k0 < T; k0 += AT) {
    __syncthreads();
    for (int e = tid; e < AT * dh; e += 256) {
      const int r = e / dh, c = e % dh;
      const bool ok = k0 + r < T;
      Ks[r * (ADH + 1) + c] = ok ? K[(k0 + r) * ldk + (int64_t)g * dh + c] : 0.0f;
      Vs[r * ADH + c] = ok ? V[(k0 + r) * ldk + (int64_t)g * dh + c] : 0.0f;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int b = 0; b < 4; b++) s[a][b] = 0.0f;
    for (int c = 0; c < dh; c++) {
      float qa[4], kb[4];
#pragma unroll
      for (int a = 0; a < 4; a++) qa[a] = Qs[(ty * 4 + a) * (ADH + 1) + c];
#pragma unroll
      for (int b = 0; b < 4; b++) kb[b] = Ks[(tx * 4 + b) * (ADH + 1) + c];
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) s[a][b] = fmaf(qa[a], kb[b], s[a][b]);
    }
#pragma unroll
    for (int a = 0; a < 4; a++) {
      float mx = -INFINITY;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        s[a][b] = (k0 + tx * 4 + b < T) ? s[a][b] * scale : -INFINITY;
        mx = fmaxf(mx, s[a][b]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[a], mx);
      const float corr = (m[a] == -INFINITY) ? 0.0f : expf(m[a] - mnew);
      float rs = 0.0f;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const float p = (s[a][b] == -INFINITY) ? 0.0f : expf(s[a][b] - mnew);
        Ps[(ty * 4 + a) * (AT + 1) + tx * 4 + b] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[a] = l[a] * corr + rs;
      m[a] = mnew;
#pragma unroll
      for (int b = 0; b < 8; b++) o[a][b] *= corr;
    }
    __syncthreads();
    for (int j = 0; j < AT; j++) {
      float vv[8];
#pragma unroll
      for (int b = 0; b < 8; b++) {
        const int c = tx * 8 + b;
        vv[b] = c < dh ? Vs[j * ADH + c] : 0.0f;
      }
#pragma unroll
      for (int a = 0; a < 4; a++) {
        const float p = Ps[(ty * 4 + a) * (AT + 1) + j];
#pragma unroll
        for (int b = 0; b < 8; b++) o[a][b] = fmaf(p, vv[b], o[a][b]);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int64_t r = q0 + ty * 4 + a;
    if (r >= T) continue;
    const float inv = 1.0f / l[a];
#pragma unroll
    for (int b = 0; b < 8; b++) {
      const int c = tx * 8 + b;
      if (c < dh) O[r * ldq + (int64_t)h * dh + c] = o[a][b] * inv;
    }
  }
}

// Row softmax of S (qh * T rows of T scores, already scaled) into the TF32
// hi / lo split of P that the P V product reads: row r of head h goes to
// P[h][r] (hi) and P[h][T + r] (lo), row pitch kp.  One CTA per row, three
// passes over the row (max, sum of exponentials, normalise and split).
__global__ void __launch_bounds__(256) softmax_split_kernel(const float *__restrict__ S, int64_t T, int64_t kp,
                                                            float *__restrict__ P) {
  __shared__ float red[8];
  const int64_t hr = blockIdx.x, h = hr / T, r = hr % T;
  const float *srow = S + hr * T;
  float *phi = P + (h * 2 * T + r) * kp, *plo = P + (h * 2 * T + T + r) * kp;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m = -INFINITY;
  for (int64_t c = tid; c < T; c += 256) m = fmaxf(m, srow[c]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; w++) m = fmaxf(m, red[w]);
  __syncthreads();
  float l = 0.0f;
  for (int64_t c = tid; c < T; c += 256) l += expf(srow[c] - m);
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  l = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) l += red[w];
  const float inv = 1.0f / l;
  for (int64_t c = tid; c < T; c += 256) {
    const float p = expf(srow[c] - m) * inv;
    const float hi = __uint_as_float(__float_as_uint(p) & 0xffffe000u);
    phi[c] = hi;
    plo[c] = __fsub_rn(p, hi);
  }
}

// (T, H, D) <-> (H, T, D)
__global__ void heads_transpose_kernel(const float *in, int64_t T, int64_t H, int64_t D, int inverse, float *out) {
  const int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (e >= T * H * D) return;
  const int64_t d = e % D;
  if (!inverse) {  // out (H, T, D) from in (T, H, D); e indexes out
    const int64_t t = (e / D) % T, h = e / (D * T);
    out[e] = in[(t * H + h) * D + d];
  } else {         // out (T, H, D) from in (H, T, D); e indexes out
    const int64_t h = (e / D) % H, t = e / (D * H);
    out[e] = in[(h * T + t) * D + d];
  }
}

}  // namespace hif4x

using namespace hif4x;

// Long sequences on the tensor cores (3xTF32): S_h = scale Q_h K_g^T for all
// heads in one batched product, the row softmax written as the split P, and
// O_h = P_h V_g in a second batched product (g = h / (qh / kvh)).
static int attention_tc(const float *Q, const float *K, const float *V, int64_t T, int qh, int kvh, int dh,
                        float *O, cudaStream_t s) {
  const int64_t kpd = (dh + 3) / 4 * 4, kpt = (T + 3) / 4 * 4;
  // every sub-buffer a multiple of 4 floats: the tensor maps need 16-byte-aligned bases
  const int64_t nq = (int64_t)qh * 2 * T * kpd, nk = (int64_t)kvh * 2 * T * kpd, ns = ((int64_t)qh * T * T + 3) / 4 * 4;
  const int64_t np = (int64_t)qh * 2 * T * kpt, nv = (int64_t)kvh * 2 * dh * kpt;
  float *ws = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void **>(&ws), (size_t)(nq + nk + ns + np + nv) * sizeof(float), s) !=
      cudaSuccess) {
    cudaGetLastError();   // not sticky: clear it so later launch checks do not report it
    return HIF4X_ERR_NOMEM;
  }
  float *Qs = ws, *Ks = Qs + nq, *Sm = Ks + nk, *Ps = Sm + ns, *Vs = Ps + np;
  const int rep = qh / kvh;
  const float scale = 1.0f / sqrtf((float)dh);
  int st = tc::split_operand(Q, (int64_t)qh * dh, 1, T, dh, dh, qh, Qs, kpd, s);
  if (st == HIF4X_OK) st = tc::split_operand(K, (int64_t)kvh * dh, 1, T, dh, dh, kvh, Ks, kpd, s);
  if (st == HIF4X_OK) st = tc::gemm_split(Qs, qh, Ks, kvh, T, T, dh, kpd, scale, 0.0f, Sm, T, T * T, qh, rep, 0, 0, s);
  if (st == HIF4X_OK) {
    softmax_split_kernel<<<(unsigned)(qh * T), 256, 0, s>>>(Sm, T, kpt, Ps);
    if (cudaGetLastError() != cudaSuccess) st = HIF4X_ERR_LAUNCH;
  }
  if (st == HIF4X_OK) st = tc::split_operand(V, (int64_t)kvh * dh, 0, dh, T, dh, kvh, Vs, kpt, s);
  if (st == HIF4X_OK)
    st = tc::gemm_split(Ps, qh, Vs, kvh, T, dh, T, kpt, 1.0f, 0.0f, O, (int64_t)qh * dh, dh, qh, rep, 0, 0, s);
  cudaFreeAsync(ws, s);
  return st;
}

// Sequences from this length on take the tensor-core form.
static const int64_t kAttnTcMinT = 1024;

extern "C" int hif4x_attention(const float *Q, const float *K, const float *V, int64_t T, int qh, int kvh, int dh,
                               float *O, void *stream) {
  if (T < 0 || qh <= 0 || kvh <= 0 || qh % kvh != 0 || dh <= 0 || dh > ADH) return HIF4X_ERR_ARG;
  if (T == 0) return HIF4X_OK;
  if (!Q || !K || !V || !O) return HIF4X_ERR_ARG;
  if (T >= kAttnTcMinT && qh * T <= INT32_MAX) {
    const int st = attention_tc(Q, K, V, T, qh, kvh, dh, O, (cudaStream_t)stream);
    if (st != HIF4X_ERR_UNSUPPORTED) return st;
  }
  const size_t smem = sizeof(float) * (2 * AT * (ADH + 1) + AT * ADH + AT * (AT + 1));
  if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return HIF4X_ERR_LAUNCH;
  dim3 grid((unsigned)((T + AT - 1) / AT), (unsigned)qh);
  const float scale = 1.0f / sqrtf((float)dh);
  attention_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(Q, K, V, T, qh, kvh, dh, scale, O);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_heads_transpose(const float *in, int64_t T, int64_t H, int64_t D, int inverse, float *out,
                                     void *stream) {
  if (T < 0 || H <= 0 || D <= 0) return HIF4X_ERR_ARG;
  const int64_t n = T * H * D;
  if (n == 0) return HIF4X_OK;
  if (!in || !out) return HIF4X_ERR_ARG;
  heads_transpose_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(in, T, H, D, inverse, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}
