// codec.cu -- NVFP4 decode, 64-point block rotation and HiF4 encode/decode.
//
// One thread owns one 64-element HiF4 group end to end (decode -> smoothing
// -> rotation -> encode -> stores), so the tensor is read once and every
// reduction of the reference (amax, quad/sub-block/group error sums) is a
// thread-local sequential loop in exactly the reference's order.  The
// group's |x| is staged in shared memory, transposed (element k of thread t
// at k*blockDim + t), so the encode can loop over sub-blocks at run time
// without bank conflicts.
//
// Bit-exactness with the reference's torch CPU arithmetic:
//  * every rounding step is an explicit __f*_rn intrinsic (no contraction);
//  * floor(log2(t)) uses a table of torch's thresholds (log2_floor_table.h);
//  * |x| / unit with unit = sig * 2^E is computed by Markstein's correction
//    (q0 = |x|*y, r = fma(-q0, u, |x|), q = fma(r, y, q0), y = RN(1/u)),
//    which returns the correctly rounded quotient for sig in {1.25, 1.5,
//    1.75} (checked exhaustively over all fp32 significands on the CPU);
//  * round-half-even of q*4*2^-m in [0, 56] is fma(q, 2^(2-m), 1.5*2^23) -
//    1.5*2^23, exact in that range;
//  * the 64-point rotation is summed in the reference's sequential order,
//    or by a fast Walsh-Hadamard transform when every partial sum is
//    provably exact (then every summation order gives the same result).
#include "common.cuh"
#include "log2_floor_table.h"

namespace hif4x {

constexpr int kConvThreads = 128;
__device__ __constant__ float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

struct ConvParams {
  int64_t ngroups, nb;
  int src_kind, src_dtype, scale_dtype;
  float s_dec;
  const void *src;
  const void *src_scale;
  const float *smooth;
  int smooth_mode;
  const uint64_t *rot_signs;
  int encode_mode;
  float *out_x;
  float *sf, *lv2, *lv3, *sign, *mant;
  uint32_t *meta;
  uint8_t *codes;
  void *deq;
  int deq_dtype;
  float *unit;
};

// floor(torch.log2(t)) for finite t > 0.
__device__ __forceinline__ int floor_log2_torch(float t) {
  const uint32_t b = __float_as_uint(t);
  int e = (int)(b >> 23) - 127;
  if ((b >> 23) == 0) e = (31 - __clz((int)b)) - 149;
  e = min(e, HIF4X_LOG2_EMAX);
  return e + (b >= HIF4X_LOG2_UP[e - HIF4X_LOG2_EMIN] ? 1 : 0);
}

// ---------------------------------------------------------------- loading
__device__ __forceinline__ void load_group(const ConvParams &p, int64_t g, float (&x)[64]) {
  if (p.src_kind == HIF4X_SRC_NVFP4_PACKED) {
    const uint4 *c4 = reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.src) + g * 32);
    const uint4 v0 = __ldcs(c4), v1 = __ldcs(c4 + 1);
    const uint32_t sc = __ldcs(reinterpret_cast<const unsigned int *>(p.src_scale) + g);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // the 8 magnitudes of this 16-element block, bf16(E2M1[i] * s), as byte
      // tables: H = high bytes, Lo = low bytes of the bf16 patterns (i = 0..7)
      const float sk = __fmul_rn(e4m3_to_f32((sc >> (8 * k)) & 0xffu), p.s_dec);
      uint32_t W[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(__fmul_rn(kE2M1[2 * i], sk), __fmul_rn(kE2M1[2 * i + 1], sk));
        W[i] = *reinterpret_cast<const uint32_t *>(&b2);
      }
      const uint32_t Hlo = __byte_perm(W[0], W[1], 0x7531), Hhi = __byte_perm(W[2], W[3], 0x7531);
      const uint32_t Llo = __byte_perm(W[0], W[1], 0x6420), Lhi = __byte_perm(W[2], W[3], 0x6420);
#pragma unroll
      for (int h = 0; h < 2; h++) {           // two code words per 16-element block
        const uint32_t cw = w[2 * k + h];
#pragma unroll
        for (int q = 0; q < 2; q++) {         // 4 elements per lookup
          const uint32_t sel = (cw >> (16 * q)) & 0x7777u;
          const uint32_t hi4 = __byte_perm(Hlo, Hhi, sel), lo4 = __byte_perm(Llo, Lhi, sel);
          const uint32_t p01 = __byte_perm(lo4, hi4, 0x5140), p23 = __byte_perm(lo4, hi4, 0x7362);
          const uint32_t bf[4] = {p01 << 16, p01 & 0xffff0000u, p23 << 16, p23 & 0xffff0000u};
#pragma unroll
          for (int n = 0; n < 4; n++) {
            const int j = 4 * q + n;            // nibble j of cw carries its sign in bit 4j+3
            x[16 * k + 8 * h + j] = __uint_as_float(bf[n] | ((cw << (28 - 4 * j)) & 0x80000000u));
          }
        }
      }
    }
    return;
  }
  if (p.src_kind == HIF4X_SRC_NVFP4_PAIR) {
    float s[4];
    if (p.scale_dtype == HIF4X_DT_F32) {
      const float4 sv = __ldg(reinterpret_cast<const float4 *>(p.src_scale) + g);
      s[0] = sv.x; s[1] = sv.y; s[2] = sv.z; s[3] = sv.w;
    } else {
      const uint2 sv = __ldg(reinterpret_cast<const uint2 *>(p.src_scale) + g);
      s[0] = __uint_as_float(sv.x << 16); s[1] = __uint_as_float(sv.x & 0xffff0000u);
      s[2] = __uint_as_float(sv.y << 16); s[3] = __uint_as_float(sv.y & 0xffff0000u);
    }
    if (p.src_dtype == HIF4X_DT_F32) {
      const float4 *c4 = reinterpret_cast<const float4 *>(p.src) + g * 16;
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const float4 v = __ldcs(c4 + j);
        x[4 * j + 0] = bf16_round(__fmul_rn(v.x, s[j >> 2]));
        x[4 * j + 1] = bf16_round(__fmul_rn(v.y, s[j >> 2]));
        x[4 * j + 2] = bf16_round(__fmul_rn(v.z, s[j >> 2]));
        x[4 * j + 3] = bf16_round(__fmul_rn(v.w, s[j >> 2]));
      }
    } else {
      const uint4 *c4 = reinterpret_cast<const uint4 *>(p.src) + g * 8;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint4 v = __ldcs(c4 + j);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int n = 0; n < 4; n++) {
          x[8 * j + 2 * n] = bf16_round(__fmul_rn(__uint_as_float(w[n] << 16), s[j >> 1]));
          x[8 * j + 2 * n + 1] = bf16_round(__fmul_rn(__uint_as_float(w[n] & 0xffff0000u), s[j >> 1]));
        }
      }
    }
    return;
  }
  // plain values
  if (p.src_dtype == HIF4X_DT_F32) {
    const float4 *c4 = reinterpret_cast<const float4 *>(p.src) + g * 16;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float4 v = __ldg(c4 + j);
      x[4 * j] = v.x; x[4 * j + 1] = v.y; x[4 * j + 2] = v.z; x[4 * j + 3] = v.w;
    }
  } else {
    const uint4 *c4 = reinterpret_cast<const uint4 *>(p.src) + g * 8;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint4 v = __ldg(c4 + j);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int n = 0; n < 4; n++) {
        x[8 * j + 2 * n] = __uint_as_float(w[n] << 16);
        x[8 * j + 2 * n + 1] = __uint_as_float(w[n] & 0xffff0000u);
      }
    }
  }
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic, round-to-nearest per lane)
typedef unsigned long long u64;
__device__ __forceinline__ u64 pk2(float lo, float hi) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(u64 v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
  u64 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}


// ---------------------------------------------------------------- rotation
// out[e] = sum_{d=0..63} x[d] * (H64[d][e] / 8 * sign_e), summed d = 0..63
// from +0 as torch's CPU einsum does (solution.py:243-245).
// `stage` is the thread's transposed shared-memory column (stride `st`).
__device__ __forceinline__ void rot64_exact(float (&x)[64], uint64_t sgn, float *stage, int st, bool bf16_vals) {
  // Exactness test: all x are multiples of 2^L; if sum|x| < 2^(L+23) every
  // partial sum of any order is representable, so the FWHT equals the
  // sequential sum bit for bit.
  int L = 1 << 20;
  float S = 0.0f;
  if (bf16_vals) {
    // bf16-valued inputs (NVFP4 decode): a normal value's lowest set bit is at
    // least its exponent - 7, so L = exponent(min nonzero |x|) - 7 bounds it
    float mn = INFINITY;
#pragma unroll
    for (int k = 0; k < 64; k++) {
      const float a = fabsf(x[k]);
      mn = fminf(mn, a == 0.0f ? INFINITY : a);
      S = __fadd_rn(S, a);
    }
    if (mn != INFINITY) {
      const int ef = (int)(__float_as_uint(mn) >> 23);
      L = ef == 0 ? -(1 << 20) : ef - 134;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 64; k++) {
      const uint32_t b = __float_as_uint(x[k]);
      const int ef = (int)((b >> 23) & 255u);
      const uint32_t m = (b & 0x7fffffu) | 0x800000u;
      const int lsb = (b & 0x7fffffffu) == 0u ? (1 << 20) : (ef == 0 ? -(1 << 20) : ef - 150 + (__ffs((int)m) - 1));
      L = min(L, lsb);
      S = __fadd_rn(S, fabsf(x[k]));
    }
  }
  const bool fast = (L >= -120) && (L + 23 > 127 || S < exp2i(L + 23));
  if (fast) {
    // stage h = 1 pairs neighbours (scalar); stages h = 2..32 run on f32x2
    // pairs {x[2i], x[2i+1]} (the same IEEE operations lane by lane)
    u64 P[32];
#pragma unroll
    for (int i = 0; i < 32; i++) P[i] = pk2(__fadd_rn(x[2 * i], x[2 * i + 1]), __fsub_rn(x[2 * i], x[2 * i + 1]));
#pragma unroll
    for (int lg = 0; lg < 5; lg++) {
      const int h = 1 << lg;   // pair distance
#pragma unroll
      for (int i = 0; i < 32; i++) {
        if ((i & h) == 0) {
          const u64 a = P[i], b = P[i + h];
          P[i] = add2(a, b);
          P[i + h] = sub2(a, b);
        }
      }
    }
    // x[e] * (+-1/8): the exact power-of-two scaling packed, the sign of
    // column e flipped by xor from bit e of the column's sign word
    const u64 EIGHTH = pk2(0.125f, 0.125f);
    const uint32_t s_lo = (uint32_t)sgn, s_hi = (uint32_t)(sgn >> 32);
#pragma unroll
    for (int i = 0; i < 32; i++) {
      float lo, hi;
      upk2(mul2(P[i], EIGHTH), lo, hi);
      const int e = 2 * i;
      const uint32_t w = e < 32 ? s_lo : s_hi;
      const int b0 = e & 31;
      x[e] = __uint_as_float(__float_as_uint(lo) ^ ((w << (31 - b0)) & 0x80000000u));
      x[e + 1] = __uint_as_float(__float_as_uint(hi) ^ ((w << (30 - b0)) & 0x80000000u));
    }
    return;
  }
  // Sequential path (wide dynamic range): the reference's order exactly.
  // Walsh masks: bit d of W_b is bit b of d.
  const uint64_t W[6] = {0xAAAAAAAAAAAAAAAAull, 0xCCCCCCCCCCCCCCCCull, 0xF0F0F0F0F0F0F0F0ull,
                         0xFF00FF00FF00FF00ull, 0xFFFF0000FFFF0000ull, 0xFFFFFFFF00000000ull};
#pragma unroll 1
  for (int e = 0; e < 64; e++) {
    uint64_t par = 0;  // bit d = parity(d & e)
#pragma unroll
    for (int b = 0; b < 6; b++)
      if ((e >> b) & 1) par ^= W[b];
    const float de = ((sgn >> e) & 1ull) ? -1.0f : 1.0f;
    float acc = 0.0f;
#pragma unroll
    for (int d = 0; d < 64; d++) {
      const float rm = __fmul_rn(((par >> d) & 1ull) ? -0.125f : 0.125f, de);
      acc = __fadd_rn(acc, __fmul_rn(x[d], rm));
    }
    stage[e * st] = acc;
  }
#pragma unroll
  for (int e = 0; e < 64; e++) x[e] = stage[e * st];
}

// ---------------------------------------------------------------- encode
// Result of an encode: sf, lv bits (bit i = lv2 of sub-block i is 2, bit
// 8+j = lv3 of quad j is 2), and how to rebuild each element's unit.
struct Enc {
  float sf;
  uint32_t bits;
};

// Searched encode, fast path: every candidate scale is inside the E6M2
// range, so the 6 candidates x 3 lv units collapse onto 14 distinct units
// sig * 2^(e0+m) (sig in {1, 1.25, 1.5, 1.75}; m in 0..3 for sig 1, 1.25
// and 0..2 for 1.5, 1.75), each evaluated once per element.
// The per-element unit work runs on f32x2 pairs; each lane is an IEEE RN fp32
// operation, so values and order equal the scalar restatement.  Pairs
// (sig s, scale m):
//   A:(1,m)+(2,m) m=0,1,2 share the packed Markstein quotient {q(1.25), q(1.5)}
//   B:(0,0)+(0,1)  C:(0,2)+(0,3)  D:(3,0)+(3,1)  E:(3,2)+(1,3)
// The squared error is computed as fma(m4, -u/4, |x|)^2 (the negated
// difference, same square).
__device__ __forceinline__ Enc search_fast2(const float *stage, int st, int e0) {
  const float p2 = exp2i(e0);
  const float u[4] = {p2, __fmul_rn(p2, 1.25f), __fmul_rn(p2, 1.5f), __fmul_rn(p2, 1.75f)};
  const float y[4] = {exp2i(-e0), __fdiv_rn(1.0f, u[1]), __fdiv_rn(1.0f, u[2]), __fdiv_rn(1.0f, u[3])};
  auto qsc = [](int m) { return m == 0 ? 4.0f : m == 1 ? 2.0f : m == 2 ? 1.0f : 0.5f; };
  auto nuq = [&](int s, int m) { return -__fmul_rn(u[s], m == 0 ? 0.25f : m == 1 ? 0.5f : m == 2 ? 1.0f : 2.0f); };
  const u64 Y12 = pk2(y[1], y[2]), NU12 = pk2(-u[1], -u[2]);
  const u64 MAG2 = pk2(kMagic, kMagic), NMAG2 = pk2(-kMagic, -kMagic);
  // per pair: scale {qs_lo, qs_hi} and negated quarter unit {-uq_lo, -uq_hi}
  const u64 QS_A[3] = {pk2(qsc(0), qsc(0)), pk2(qsc(1), qsc(1)), pk2(qsc(2), qsc(2))};
  const u64 NU_A[3] = {pk2(nuq(1, 0), nuq(2, 0)), pk2(nuq(1, 1), nuq(2, 1)), pk2(nuq(1, 2), nuq(2, 2))};
  const u64 QS_B = pk2(qsc(0), qsc(1)), NU_B = pk2(nuq(0, 0), nuq(0, 1));
  const u64 QS_C = pk2(qsc(2), qsc(3)), NU_C = pk2(nuq(0, 2), nuq(0, 3));
  const u64 QS_D = pk2(qsc(0), qsc(1)), NU_D = pk2(nuq(3, 0), nuq(3, 1));
  const u64 QS_E = pk2(qsc(2), qsc(3)), NU_E = pk2(nuq(3, 2), nuq(1, 3));
  const float M7 = kMagic + 7.0f;
  float err[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  uint32_t bits[6] = {0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll 1
  for (int i = 0; i < 8; i++) {
    float Q[2][14];
#pragma unroll
    for (int qd = 0; qd < 2; qd++) {
      u64 acc[7];
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const float a = stage[(8 * i + 4 * qd + kk) * st];
        const u64 a2 = pk2(a, a);
        const float q0 = __fmul_rn(a, y[0]);
        const u64 q12a = mul2(a2, Y12);
        const u64 q12 = fma2(fma2(q12a, NU12, a2), Y12, q12a);
        const float q3a = __fmul_rn(a, y[3]);
        const float q3 = __fmaf_rn(__fmaf_rn(-q3a, u[3], a), y[3], q3a);
        float q1, q2;
        upk2(q12, q1, q2);
        const u64 QIN[7] = {q12, q12, q12, pk2(q0, q0), pk2(q0, q0), pk2(q3, q3), pk2(q3, q1)};
        const u64 QSV[7] = {QS_A[0], QS_A[1], QS_A[2], QS_B, QS_C, QS_D, QS_E};
        const u64 NUV[7] = {NU_A[0], NU_A[1], NU_A[2], NU_B, NU_C, NU_D, NU_E};
#pragma unroll
        for (int pi = 0; pi < 7; pi++) {
          float tl, th;
          upk2(fma2(QIN[pi], QSV[pi], MAG2), tl, th);
          // scales m = 3 never round above 7 (q < 14): C.hi = (0,3), E.hi = (1,3) skip the clamp
          const u64 t2 = pk2(fminf(tl, M7), (pi == 4 || pi == 6) ? th : fminf(th, M7));
          const u64 mm = add2(t2, NMAG2);
          const u64 d = fma2(mm, NUV[pi], a2);
          const u64 e = mul2(d, d);
          acc[pi] = kk ? add2(acc[pi], e) : e;
        }
      }
      // unit index = 4*s + m for s <= 1, 8 + m for s = 2, 11 + m for s = 3
      upk2(acc[0], Q[qd][4], Q[qd][8]);
      upk2(acc[1], Q[qd][5], Q[qd][9]);
      upk2(acc[2], Q[qd][6], Q[qd][10]);
      upk2(acc[3], Q[qd][0], Q[qd][1]);
      upk2(acc[4], Q[qd][2], Q[qd][3]);
      upk2(acc[5], Q[qd][11], Q[qd][12]);
      upk2(acc[6], Q[qd][13], Q[qd][7]);
    }
    const int BASE[6] = {0, 4, 8, 11, 1, 5};
#pragma unroll
    for (int c = 0; c < 6; c++) {
      const int b0 = BASE[c];
      const float a0 = Q[0][b0], a1 = Q[0][b0 + 1], a2 = Q[0][b0 + 2];
      const float c0 = Q[1][b0], c1 = Q[1][b0 + 1], c2 = Q[1][b0 + 2];
      // lv3 per quad: unit b0 on ties (<=); lv2: the first choice unless strictly better
      const float e2a = __fadd_rn(fminf(a0, a1), fminf(c0, c1));
      const float e2b = __fadd_rn(fminf(a1, a2), fminf(c1, c2));
      const bool take2 = e2b < e2a;
      const uint32_t l3 = take2 ? ((a1 > a2 ? 1u : 0u) | (c1 > c2 ? 2u : 0u))
                                : ((a0 > a1 ? 1u : 0u) | (c0 > c1 ? 2u : 0u));
      bits[c] |= ((take2 ? 1u : 0u) << i) | (l3 << (8 + 2 * i));
      err[c] = __fadd_rn(err[c], fminf(e2a, e2b));
    }
  }
  int cb = 0;
  float eb = err[0];
#pragma unroll
  for (int c = 1; c < 6; c++)
    if (err[c] < eb) { eb = err[c]; cb = c; }
  const int SIGI[6] = {0, 1, 2, 3, 0, 1};
  float ub = u[0];
  uint32_t bb = bits[0];
#pragma unroll
  for (int c = 1; c < 6; c++)
    if (cb == c) { ub = u[SIGI[c]]; bb = bits[c]; }
  Enc r;
  r.sf = __fmul_rn(ub, cb >= 4 ? 2.0f : 1.0f);
  r.bits = bb;
  return r;
}

// Literal restatement of _quant_chunk for groups whose candidate scales hit
// the E6M2 clamps (all-zero, tiny or huge groups).  IEEE divisions, rintf.
__device__ __forceinline__ float sq_err_ref(float a, float unit) {
  float q = __fmul_rn(__fdiv_rn(a, unit), 4.0f);
  q = clampf(__fmul_rn(rintf(q), 0.25f), 0.0f, 1.75f);
  const float d = __fsub_rn(__fmul_rn(q, unit), a);
  return __fmul_rn(d, d);
}

__device__ __noinline__ Enc search_generic(const float *stage, int st, int e0) {
  const int K[6] = {0, 0, 0, 0, 1, 1};
  const float SIG[6] = {1.0f, 1.25f, 1.5f, 1.75f, 1.0f, 1.25f};
  float eb = 0.0f, sfb = 0.0f;
  uint32_t bb = 0;
#pragma unroll 1
  for (int c = 0; c < 6; c++) {
    const float sf = clampf(__fmul_rn(exp2i(e0 + K[c]), SIG[c]), kSfMin, kSfMax);
    float err = 0.0f;
    uint32_t bits = 0;
#pragma unroll 1
    for (int i = 0; i < 8; i++) {
      float e3[2][2][2];  // [lv2][lv3][quad]
#pragma unroll
      for (int l2 = 0; l2 < 2; l2++)
#pragma unroll
        for (int l3 = 0; l3 < 2; l3++) {
          const float unit = __fmul_rn(__fmul_rn(sf, l2 ? 2.0f : 1.0f), l3 ? 2.0f : 1.0f);
#pragma unroll
          for (int qd = 0; qd < 2; qd++) {
            float s = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) s = __fadd_rn(s, sq_err_ref(stage[(8 * i + 4 * qd + kk) * st], unit));
            e3[l2][l3][qd] = s;
          }
        }
      float e2[2];
      uint32_t l3b[2];
#pragma unroll
      for (int l2 = 0; l2 < 2; l2++) {
        const bool t0 = e3[l2][0][0] <= e3[l2][1][0];
        const bool t1 = e3[l2][0][1] <= e3[l2][1][1];
        e2[l2] = __fadd_rn(t0 ? e3[l2][0][0] : e3[l2][1][0], t1 ? e3[l2][0][1] : e3[l2][1][1]);
        l3b[l2] = (t0 ? 0u : 1u) | (t1 ? 0u : 2u);
      }
      const bool take2 = e2[1] < e2[0];
      bits |= ((take2 ? 1u : 0u) << i) | ((take2 ? l3b[1] : l3b[0]) << (8 + 2 * i));
      err = __fadd_rn(err, take2 ? e2[1] : e2[0]);
    }
    if (c == 0 || err < eb) { eb = err; sfb = sf; bb = bits; }
  }
  Enc r;
  r.sf = sfb;
  r.bits = bb;
  return r;
}

// _quant_weight_fast (solution.py:787-823): greedy lv tree, anchor exponent,
// four significands; the 64 errors are summed left to right.
__device__ __noinline__ Enc encode_fast(const float *stage, int st, float amax) {
  float a4[16], a8[8];
#pragma unroll
  for (int j = 0; j < 16; j++) {
    float m = stage[(4 * j) * st];
#pragma unroll
    for (int k = 1; k < 4; k++) m = fmaxf(m, stage[(4 * j + k) * st]);
    a4[j] = m;
  }
#pragma unroll
  for (int i = 0; i < 8; i++) a8[i] = fmaxf(a4[2 * i], a4[2 * i + 1]);
  const float t = fmaxf(__fdiv_rn(amax, 7.0f), 1e-38f);
  const int e0 = floor_log2_torch(t);
  const float SIG[4] = {1.0f, 1.25f, 1.5f, 1.75f};
  float eb = 0.0f, sfb = 0.0f;
#pragma unroll 1
  for (int c = 0; c < 4; c++) {
    const float sf = clampf(__fmul_rn(exp2i(e0), SIG[c]), kSfMin, kSfMax);
    float err = 0.0f;
#pragma unroll 1
    for (int i = 0; i < 8; i++) {
      const float l2 = (__fdiv_rn(a8[i], sf) > 1.75f) ? 2.0f : 1.0f;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float l3 = (__fdiv_rn(a4[2 * i + k / 4], __fmul_rn(sf, l2)) > 1.75f) ? 2.0f : 1.0f;
        err = __fadd_rn(err, sq_err_ref(stage[(8 * i + k) * st], __fmul_rn(__fmul_rn(sf, l2), l3)));
      }
    }
    if (c == 0 || err < eb) { eb = err; sfb = sf; }
  }
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const bool l2 = __fdiv_rn(a8[i], sfb) > 1.75f;
    bits |= (l2 ? 1u : 0u) << i;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const bool l3 = __fdiv_rn(a4[2 * i + h], __fmul_rn(sfb, l2 ? 2.0f : 1.0f)) > 1.75f;
      bits |= (l3 ? 1u : 0u) << (8 + 2 * i + h);
    }
  }
  Enc r;
  r.sf = sfb;
  r.bits = bits;
  return r;
}

// _encode_e6m2 (dev/variants.py:240-246)
__device__ __forceinline__ float encode_e6m2(float x) {
  const float xc = fmaxf(x, 1e-30f);
  const int e = floor_log2_torch(xc);
  float m = rintf(__fmul_rn(xc, exp2i(2 - e)));
  m = clampf(m, 4.0f, 8.0f);
  return clampf(__fmul_rn(m, exp2i(e - 2)), kSfMin, kSfMax);
}

// ---------------------------------------------------------------- outputs
__device__ __forceinline__ uint32_t e6m2_code(float sf) {
  const uint32_t b = __float_as_uint(sf);
  const int E = (int)(b >> 23) - 127;
  return ((uint32_t)(E + 48) << 2) | ((b >> 21) & 3u);
}

template <bool PACKED_ONLY>
__global__ void __launch_bounds__(kConvThreads, 5) convert_kernel(const ConvParams p) {
  extern __shared__ float smem[];
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= p.ngroups) return;
  const int st = blockDim.x;
  float *stage = smem + threadIdx.x;
  const int64_t bcol = g % p.nb;  // 64-block index within the row

  float x[64];
  load_group(p, g, x);
  if (p.smooth_mode != HIF4X_SMOOTH_NONE) {
    const float4 *s4 = reinterpret_cast<const float4 *>(p.smooth) + bcol * 16;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const float4 s = __ldg(s4 + j);
      const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
      for (int n = 0; n < 4; n++)
        x[4 * j + n] = p.smooth_mode == HIF4X_SMOOTH_MUL ? __fmul_rn(x[4 * j + n], sv[n])
                                                          : __fdiv_rn(x[4 * j + n], sv[n]);
    }
  }
  if (p.rot_signs != nullptr)
    rot64_exact(x, __ldg(p.rot_signs + bcol), stage, st,
                p.src_kind != HIF4X_SRC_VALUES && p.smooth_mode == HIF4X_SMOOTH_NONE);
  if (p.out_x != nullptr) {
    float4 *o4 = reinterpret_cast<float4 *>(p.out_x) + g * 16;
#pragma unroll
    for (int j = 0; j < 16; j++) o4[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
  }
  if (p.encode_mode == HIF4X_ENC_NONE) return;

  // signs: neg (x < 0) and zero (x == 0) masks; stage |x|
  uint64_t neg = 0;
  float amax = 0.0f;
#pragma unroll
  for (int k = 0; k < 64; k++) {
    const float a = fabsf(x[k]);
    neg |= (x[k] < 0.0f ? 1ull : 0ull) << k;
    amax = fmaxf(amax, a);
    stage[k * st] = a;
  }

  Enc enc;
  if (p.encode_mode == HIF4X_ENC_SEARCH) {
    const float t = fmaxf(__fdiv_rn(amax, 7.0f), 1e-38f);
    const int e0 = floor_log2_torch(t);
    enc = (e0 >= -48 && e0 <= 14) ? search_fast2(stage, st, e0) : search_generic(stage, st, e0);
  } else if (p.encode_mode == HIF4X_ENC_FAST) {
    enc = encode_fast(stage, st, amax);
  } else {
    // Algorithm 1 (dev/variants.py:258-287): sf from the peak, lv bits by threshold.
    enc.sf = encode_e6m2(__fdiv_rn(amax, 7.0f));
    const float rec = __fdiv_rn(1.0f, enc.sf);
    uint32_t bits = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float v16[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float m = stage[(8 * i + 4 * h) * st];
#pragma unroll
        for (int k = 1; k < 4; k++) m = fmaxf(m, stage[(8 * i + 4 * h + k) * st]);
        v16[h] = m;
      }
      const float v8 = fmaxf(v16[0], v16[1]);
      const bool e8 = __fmul_rn(v8, rec) >= 4.0f;
      bits |= (e8 ? 1u : 0u) << i;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const bool e16 = __fmul_rn(__fmul_rn(v16[h], rec), e8 ? 0.5f : 1.0f) >= 2.0f;
        bits |= (e16 ? 1u : 0u) << (8 + 2 * i + h);
      }
    }
    enc.bits = bits;
  }

  // ---- element pass, packed HiF4 only (searched encode), on f32x2 pairs.
  // m4 = min(RNE(q), 7) with q = |x| / unit * 4 is RNE(min(q, 7.25)) (RNE is
  // monotone and 7.25 rounds to 7), so one clamp before the magic-number
  // rounding covers every q >= 0 (infinities too); t + 1.5*2^23 then holds m4
  // in its low three bits.
  if (PACKED_ONLY) {
    const float sf = enc.sf;
    const float ysf = __fdiv_rn(1.0f, sf);
    p.meta[g] = e6m2_code(sf) | ((enc.bits & 0xffu) << 8) | ((enc.bits >> 8) << 16);
    const u64 YSF2 = pk2(ysf, ysf), NSF2 = pk2(-sf, -sf), MAG2 = pk2(kMagic, kMagic);
    const uint32_t magic_bits = __float_as_uint(kMagic);
#pragma unroll 1
    for (int i = 0; i < 8; i++) {
      const uint32_t l2 = (enc.bits >> i) & 1u;
      uint32_t nib = 0;
#pragma unroll
      for (int qd = 0; qd < 2; qd++) {
        const uint32_t l3 = (enc.bits >> (8 + 2 * i + qd)) & 1u;
        const float mq = exp2i(2 - (int)(l2 + l3));            // 4, 2 or 1: unit = sf * 2^(l2+l3)
        const u64 M2 = pk2(mq, mq);
#pragma unroll
        for (int pr = 0; pr < 2; pr++) {
          const int el = 8 * i + 4 * qd + 2 * pr;
          const u64 a2 = pk2(stage[el * st], stage[(el + 1) * st]);
          const u64 q0 = mul2(a2, YSF2);
          const u64 q = mul2(fma2(fma2(q0, NSF2, a2), YSF2, q0), M2);   // Markstein quotient, rescaled
          float lo, hi;
          upk2(q, lo, hi);
          float rl, rh;
          upk2(add2(pk2(fminf(lo, 7.25f), fminf(hi, 7.25f)), MAG2), rl, rh);
          const uint32_t two = (__float_as_uint(rl) - magic_bits) | ((__float_as_uint(rh) - magic_bits) << 4);
          nib |= two << (4 * (4 * qd + 2 * pr));
        }
      }
      // sign bits of the sub-block to bit 3 of each nibble
      uint32_t sb = (uint32_t)(neg >> (8 * i)) & 0xffu;
      sb = (sb | (sb << 12)) & 0x000f000fu;
      sb = (sb | (sb << 6)) & 0x03030303u;
      sb = (sb | (sb << 3)) & 0x11111111u;
      reinterpret_cast<uint32_t *>(p.codes)[g * 8 + i] = nib | (sb << 3);
    }
    return;
  }

  // ---- element pass: mant, sign and every requested output
  const float sf = enc.sf;
  const bool alg1 = p.encode_mode == HIF4X_ENC_ALG1;
  const float rec = alg1 ? __fdiv_rn(1.0f, sf) : 0.0f;
  // Markstein reciprocal of the significand part: unit = sf * 2^(l2+l3)
  const float ysf = __fdiv_rn(1.0f, sf);
  uint32_t meta_word = e6m2_code(sf) | ((enc.bits & 0xffu) << 8) | ((enc.bits >> 8) << 16);
  if (p.sf != nullptr) p.sf[g] = sf;
  if (p.meta != nullptr) p.meta[g] = meta_word;
#pragma unroll 1
  for (int i = 0; i < 8; i++) {
    const uint32_t l2 = (enc.bits >> i) & 1u;
    if (p.lv2 != nullptr) p.lv2[g * 8 + i] = l2 ? 2.0f : 1.0f;
    float mant8[8], sign8[8], unit8[8], deq8[8];
    uint32_t nib = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int el = 8 * i + k;
      const uint32_t l3 = (enc.bits >> (8 + 2 * i + k / 4)) & 1u;
      const float a = stage[el * st];
      const bool isneg = (neg >> el) & 1ull;
      const float sg = a == 0.0f ? 0.0f : (isneg ? -1.0f : 1.0f);
      const float unit = __fmul_rn(__fmul_rn(sf, l2 ? 2.0f : 1.0f), l3 ? 2.0f : 1.0f);
      float m4;
      if (!alg1) {
        // round(|x| / unit * 4) clamped to 7; quotient by Markstein on sf
        // (the lv factors are powers of two: exact rescaling)
        const float q0 = __fmul_rn(a, ysf);
        const float r = __fmaf_rn(-q0, sf, a);
        float q = __fmaf_rn(r, ysf, q0);
        q = __fmul_rn(q, (l2 + l3) == 0 ? 4.0f : ((l2 + l3) == 1 ? 2.0f : 1.0f));
        m4 = q < 4194304.0f ? __fsub_rn(fminf(__fadd_rn(q, kMagic), kMagic + 7.0f), kMagic)
                                       : fminf(rintf(q), 7.0f);
      } else {
        const float xs = __fmul_rn(__fmul_rn(__fmul_rn(a, rec), l2 ? 0.5f : 1.0f), l3 ? 0.5f : 1.0f);
        m4 = clampf(floorf(__fadd_rn(__fmul_rn(xs, 4.0f), 0.5f)), 0.0f, 7.0f);
      }
      const float mant = __fmul_rn(m4, 0.25f);
      const float sgo = (alg1 && m4 == 0.0f) ? 0.0f : sg;
      mant8[k] = mant;
      sign8[k] = sgo;
      unit8[k] = unit;
      // value = sign * mant * lv3 * lv2 * sf (exact); keeps -0 for negative zeros
      deq8[k] = __fmul_rn(__fmul_rn(sgo, mant), __fmul_rn(__fmul_rn(l3 ? 2.0f : 1.0f, l2 ? 2.0f : 1.0f), sf));
      nib |= ((isneg && !(alg1 && m4 == 0.0f) ? 8u : 0u) | (uint32_t)m4) << (4 * k);
    }
    if (p.lv3 != nullptr) {
      p.lv3[g * 16 + 2 * i] = ((enc.bits >> (8 + 2 * i)) & 1u) ? 2.0f : 1.0f;
      p.lv3[g * 16 + 2 * i + 1] = ((enc.bits >> (9 + 2 * i)) & 1u) ? 2.0f : 1.0f;
    }
    const int64_t e0i = g * 64 + 8 * i;
    if (p.mant != nullptr) {
      reinterpret_cast<float4 *>(p.mant + e0i)[0] = make_float4(mant8[0], mant8[1], mant8[2], mant8[3]);
      reinterpret_cast<float4 *>(p.mant + e0i)[1] = make_float4(mant8[4], mant8[5], mant8[6], mant8[7]);
    }
    if (p.sign != nullptr) {
      reinterpret_cast<float4 *>(p.sign + e0i)[0] = make_float4(sign8[0], sign8[1], sign8[2], sign8[3]);
      reinterpret_cast<float4 *>(p.sign + e0i)[1] = make_float4(sign8[4], sign8[5], sign8[6], sign8[7]);
    }
    if (p.unit != nullptr) {
      reinterpret_cast<float4 *>(p.unit + e0i)[0] = make_float4(unit8[0], unit8[1], unit8[2], unit8[3]);
      reinterpret_cast<float4 *>(p.unit + e0i)[1] = make_float4(unit8[4], unit8[5], unit8[6], unit8[7]);
    }
    if (p.codes != nullptr) reinterpret_cast<uint32_t *>(p.codes)[g * 8 + i] = nib;
    if (p.deq != nullptr) {
      if (p.deq_dtype == HIF4X_DT_F32) {
        float4 *d4 = reinterpret_cast<float4 *>(static_cast<float *>(p.deq) + e0i);
        d4[0] = make_float4(deq8[0], deq8[1], deq8[2], deq8[3]);
        d4[1] = make_float4(deq8[4], deq8[5], deq8[6], deq8[7]);
      } else {
        uint32_t w[4];
#pragma unroll
        for (int n = 0; n < 4; n++)
          w[n] = (__float_as_uint(deq8[2 * n]) >> 16) | (__float_as_uint(deq8[2 * n + 1]) & 0xffff0000u);
        reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.deq) + e0i)[0] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// ---------------------------------------------------------------- decoders
// HiF4 packed -> values.  Each thread decodes eight 8-element sub-blocks
// lane + 32 j (j = 0..7) of its warp's run of 256, so all eight code loads
// (4 bytes each) are in flight together and every load and store
// instruction of the warp is contiguous.  One 4-byte load per thread left the
// kernel latency-bound at 3.8 TB/s; a whole group per thread (strided 16-byte
// stores) was slower still.
constexpr int kDecSubs = 8;
__global__ void __launch_bounds__(256) decode_packed_kernel(const uint32_t *__restrict__ meta,
                                                            const uint32_t *__restrict__ codes, int64_t nsub,
                                                            void *out, int out_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * (32 * kDecSubs) + lane;
  uint32_t w[kDecSubs], m[kDecSubs];
#pragma unroll
  for (int j = 0; j < kDecSubs; j++) {
    const int64_t t = base + 32 * j;
    w[j] = t < nsub ? __ldcs(codes + t) : 0u;
    m[j] = t < nsub ? __ldg(meta + (t >> 3)) : 0u;
  }
#pragma unroll
  for (int j = 0; j < kDecSubs; j++) {
    const int64_t t = base + 32 * j;
    if (t >= nsub) return;
    const int i = (int)(t & 7);
    const int E = (int)((m[j] & 0xffu) >> 2) - 48;
    const float sf = __fmul_rn(exp2i(E), 1.0f + 0.25f * (float)(m[j] & 3u));
    const int l2 = (int)((m[j] >> (8 + i)) & 1u);
    // sf * lv2 * lv3 / 4 for the two quads of the sub-block (exact powers of two of sf)
    const float sq0 = __fmul_rn(sf, exp2i(l2 + (int)((m[j] >> (16 + 2 * i)) & 1u) - 2));
    const float sq1 = __fmul_rn(sf, exp2i(l2 + (int)((m[j] >> (17 + 2 * i)) & 1u) - 2));
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const uint32_t nib = (w[j] >> (4 * k)) & 15u;
      const float mag = __fmul_rn((float)(nib & 7u), k < 4 ? sq0 : sq1);
      v[k] = __uint_as_float(__float_as_uint(mag) | ((nib & 8u) << 28));   // -0 for a negative-zero code
    }
    if (out_dtype == HIF4X_DT_F32) {
      float4 *o = reinterpret_cast<float4 *>(out) + t * 2;
      __stcs(o, make_float4(v[0], v[1], v[2], v[3]));
      __stcs(o + 1, make_float4(v[4], v[5], v[6], v[7]));
    } else {
      // every HiF4 value is exact in bf16: its pattern is the float's upper half
      uint32_t q[4];
#pragma unroll
      for (int n = 0; n < 4; n++) q[n] = __byte_perm(__float_as_uint(v[2 * n]), __float_as_uint(v[2 * n + 1]), 0x7632);
      __stcs(reinterpret_cast<uint4 *>(out) + t, make_uint4(q[0], q[1], q[2], q[3]));
    }
  }
}

// Packed HiF4 rows: row r of the output is its C/2 code bytes followed by
// its C/64 meta words (9C/16 bytes per row), one thread per 4-byte word.
__global__ void hif4_rows_kernel(const uint32_t *__restrict__ meta, const uint32_t *__restrict__ codes,
                                 int64_t rows, int64_t cw, int64_t mw, uint32_t *__restrict__ out) {
  const int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t pw = cw + mw;
  if (w >= rows * pw) return;
  const int64_t r = w / pw, j = w - r * pw;
  out[w] = j < cw ? __ldcs(codes + r * cw + j) : __ldcs(meta + r * mw + (j - cw));
}

// dict5 -> values, one thread per element: ((((sign*mant)*lv3)*lv2)*sf)
__global__ void decode_dict5_kernel(const float *sf, const float *lv2, const float *lv3, const float *sign,
                                    const float *mant, int64_t n, void *out, int out_dtype) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int64_t g = e >> 6;
  const int k = (int)(e & 63);
  float v = __fmul_rn(sign[e], mant[e]);
  v = __fmul_rn(v, lv3[g * 16 + k / 4]);
  v = __fmul_rn(v, lv2[g * 8 + k / 8]);
  v = __fmul_rn(v, sf[g]);
  if (out_dtype == HIF4X_DT_F32) static_cast<float *>(out)[e] = v;
  else static_cast<__nv_bfloat16 *>(out)[e] = __float2bfloat16_rn(v);
}

__global__ void values_to_params_kernel(const float *q, const float *sf, const float *lv2, const float *lv3,
                                        int64_t n, float *sign, float *mant) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int64_t g = e >> 6;
  const int k = (int)(e & 63);
  const float unit = __fmul_rn(__fmul_rn(sf[g], lv2[g * 8 + k / 8]), lv3[g * 16 + k / 4]);
  const float v = q[e];
  float m = rintf(__fmul_rn(__fdiv_rn(fabsf(v), unit), 4.0f));
  mant[e] = __fmul_rn(clampf(m, 0.0f, 7.0f), 0.25f);
  sign[e] = torch_sign(v);
}

__global__ void unit_flat_kernel(const float *sf, const float *lv2, const float *lv3, int64_t n, float *unit) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int64_t g = e >> 6;
  const int k = (int)(e & 63);
  unit[e] = __fmul_rn(__fmul_rn(sf[g], lv2[g * 8 + k / 8]), lv3[g * 16 + k / 4]);
}

__global__ void pack_dict5_kernel(const float *sf, const float *lv2, const float *lv3, const float *sign,
                                  const float *mant, int64_t ngroups, uint32_t *meta, uint8_t *codes) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ngroups) return;
  uint32_t w = e6m2_code(sf[g]);
  for (int i = 0; i < 8; i++) w |= (lv2[g * 8 + i] == 2.0f ? 1u : 0u) << (8 + i);
  for (int j = 0; j < 16; j++) w |= (lv3[g * 16 + j] == 2.0f ? 1u : 0u) << (16 + j);
  meta[g] = w;
  for (int i = 0; i < 8; i++) {
    uint32_t nib = 0;
    for (int k = 0; k < 8; k++) {
      const int64_t e = g * 64 + 8 * i + k;
      nib |= ((sign[e] < 0.0f ? 8u : 0u) | (uint32_t)(mant[e] * 4.0f)) << (4 * k);
    }
    reinterpret_cast<uint32_t *>(codes)[g * 8 + i] = nib;
  }
}

__global__ void unpack_dict5_kernel(const uint32_t *meta, const uint8_t *codes, int64_t ngroups, float *sf,
                                    float *lv2, float *lv3, float *sign, float *mant) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ngroups) return;
  const uint32_t m = meta[g];
  const int E = (int)((m & 0xffu) >> 2) - 48;
  sf[g] = __fmul_rn(exp2i(E), 1.0f + 0.25f * (float)(m & 3u));
  for (int i = 0; i < 8; i++) lv2[g * 8 + i] = ((m >> (8 + i)) & 1u) ? 2.0f : 1.0f;
  for (int j = 0; j < 16; j++) lv3[g * 16 + j] = ((m >> (16 + j)) & 1u) ? 2.0f : 1.0f;
  for (int i = 0; i < 8; i++) {
    const uint32_t w = reinterpret_cast<const uint32_t *>(codes)[g * 8 + i];
    for (int k = 0; k < 8; k++) {
      const uint32_t nib = (w >> (4 * k)) & 15u;
      const int64_t e = g * 64 + 8 * i + k;
      mant[e] = 0.25f * (float)(nib & 7u);
      sign[e] = (nib & 8u) ? -1.0f : ((nib & 7u) ? 1.0f : 0.0f);
    }
  }
}

// NVFP4 -> values, one thread per 16-element scale block.
__global__ void nvfp4_decode_kernel(int src_kind, const void *src, int src_dtype, const void *scale,
                                    int scale_dtype, float s_dec, int64_t nblk, void *out, int out_dtype) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblk) return;
  float v[16];
  if (src_kind == HIF4X_SRC_NVFP4_PACKED) {
    const float s = __fmul_rn(e4m3_to_f32(static_cast<const uint8_t *>(scale)[b]), s_dec);
    const uint2 w = __ldcs(reinterpret_cast<const uint2 *>(src) + b);
    const uint32_t ww[2] = {w.x, w.y};
#pragma unroll
    for (int n = 0; n < 16; n++) v[n] = bf16_round(__fmul_rn(e2m1_to_f32((ww[n >> 3] >> (4 * (n & 7))) & 15u), s));
  } else {
    const float s = scale_dtype == HIF4X_DT_F32 ? static_cast<const float *>(scale)[b]
                                                : bf16_bits_to_f32(static_cast<const uint16_t *>(scale)[b]);
#pragma unroll
    for (int n = 0; n < 16; n++) {
      const float c = src_dtype == HIF4X_DT_F32 ? static_cast<const float *>(src)[b * 16 + n]
                                                : bf16_bits_to_f32(static_cast<const uint16_t *>(src)[b * 16 + n]);
      v[n] = bf16_round(__fmul_rn(c, s));
    }
  }
#pragma unroll
  for (int n = 0; n < 16; n++) {
    if (out_dtype == HIF4X_DT_F32) static_cast<float *>(out)[b * 16 + n] = v[n];
    else static_cast<__nv_bfloat16 *>(out)[b * 16 + n] = __float2bfloat16_rn(v[n]);
  }
}

// Packed NVFP4 -> bf16 / fp32, the layout of decode_packed_kernel: each
// thread decodes eight 8-element sub-blocks (lane + 32 j of its warp's run of
// 256), one 4-byte code word each, so a warp's loads and its 16-byte stores are
// contiguous.  Per sub-block the 8 magnitudes bf16(E2M1[i] * s) of its scale
// are built once as byte tables and picked per nibble by byte permutes (as
// load_group does); the nibble's bit 3 becomes the bf16 sign bit, so a
// negative-zero code decodes to -0 as the reference's -0.0 carrier does.
__global__ void __launch_bounds__(256) nvfp4_decode_packed_kernel(const uint32_t *__restrict__ codes,
                                                                  const uint8_t *__restrict__ e4m3, float s_dec,
                                                                  int64_t nsub, void *out, int out_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * (32 * kDecSubs) + lane;
  uint32_t w[kDecSubs], sc[kDecSubs];
#pragma unroll
  for (int j = 0; j < kDecSubs; j++) {
    const int64_t t = base + 32 * j;
    w[j] = t < nsub ? __ldcs(codes + t) : 0u;
    sc[j] = t < nsub ? (uint32_t)__ldg(e4m3 + (t >> 1)) : 0u;
  }
#pragma unroll
  for (int j = 0; j < kDecSubs; j++) {
    const int64_t t = base + 32 * j;
    if (t >= nsub) return;
    const float sk = __fmul_rn(e4m3_to_f32(sc[j]), s_dec);
    uint32_t W[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(__fmul_rn(kE2M1[2 * i], sk), __fmul_rn(kE2M1[2 * i + 1], sk));
      W[i] = *reinterpret_cast<const uint32_t *>(&b2);
    }
    const uint32_t Hlo = __byte_perm(W[0], W[1], 0x7531), Hhi = __byte_perm(W[2], W[3], 0x7531);
    const uint32_t Llo = __byte_perm(W[0], W[1], 0x6420), Lhi = __byte_perm(W[2], W[3], 0x6420);
    uint32_t o[4];   // bf16 pairs of elements (0,1), (2,3), (4,5), (6,7)
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint32_t c16 = (w[j] >> (16 * q)) & 0xffffu;
      const uint32_t sel = c16 & 0x7777u;
      const uint32_t hi4 = __byte_perm(Hlo, Hhi, sel), lo4 = __byte_perm(Llo, Lhi, sel);
      // nibble sign bits 3, 7, 11, 15 of c16 -> bits 15 and 31 of the pairs
      o[2 * q] = __byte_perm(lo4, hi4, 0x5140) | ((c16 & 0x8u) << 12) | ((c16 & 0x80u) << 24);
      o[2 * q + 1] = __byte_perm(lo4, hi4, 0x7362) | ((c16 & 0x800u) << 4) | ((c16 & 0x8000u) << 16);
    }
    if (out_dtype == HIF4X_DT_F32) {
      float4 *d = reinterpret_cast<float4 *>(out) + t * 2;
      __stcs(d, make_float4(__uint_as_float(o[0] << 16), __uint_as_float(o[0] & 0xffff0000u),
                            __uint_as_float(o[1] << 16), __uint_as_float(o[1] & 0xffff0000u)));
      __stcs(d + 1, make_float4(__uint_as_float(o[2] << 16), __uint_as_float(o[2] & 0xffff0000u),
                                __uint_as_float(o[3] << 16), __uint_as_float(o[3] & 0xffff0000u)));
    } else {
      __stcs(reinterpret_cast<uint4 *>(out) + t, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// standalone rotation: one thread per group
__global__ void __launch_bounds__(kConvThreads) rotate64_kernel(const float *x, const uint64_t *signs, int64_t ngroups,
                                                                 int64_t nb, float *out) {
  extern __shared__ float smem[];
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ngroups) return;
  float v[64];
  const float4 *x4 = reinterpret_cast<const float4 *>(x) + g * 16;
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const float4 a = __ldg(x4 + j);
    v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = a.z; v[4 * j + 3] = a.w;
  }
  rot64_exact(v, __ldg(signs + g % nb), smem + threadIdx.x, blockDim.x, false);
  float4 *o4 = reinterpret_cast<float4 *>(out) + g * 16;
#pragma unroll
  for (int j = 0; j < 16; j++) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

}  // namespace hif4x

// ====================================================================== ABI
using namespace hif4x;

static inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static inline unsigned nblocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

extern "C" int hif4x_version(void) { return 100; }

extern "C" int hif4x_convert(const hif4x_convert_desc *d, void *stream) {
  if (d == nullptr || d->rows < 0 || d->cols <= 0 || d->cols % 64 != 0) return HIF4X_ERR_ARG;
  if (d->rows == 0) return HIF4X_OK;  // empty tensors may carry null pointers
  if (d->src == nullptr) return HIF4X_ERR_ARG;
  if (d->src_kind != HIF4X_SRC_VALUES && d->src_scale == nullptr) return HIF4X_ERR_ARG;
  if (d->smooth_mode != HIF4X_SMOOTH_NONE && d->smooth == nullptr) return HIF4X_ERR_ARG;
  if (d->encode_mode < HIF4X_ENC_NONE || d->encode_mode > HIF4X_ENC_ALG1) return HIF4X_ERR_ARG;
  const void *ptrs[] = {d->src, d->src_scale, d->smooth, d->out_x, d->sign, d->mant, d->deq, d->unit, d->codes};
  for (const void *q : ptrs)
    if (q != nullptr && !al16(q)) return HIF4X_ERR_ARG;
  if (d->src_kind == HIF4X_SRC_NVFP4_PACKED && (reinterpret_cast<uintptr_t>(d->src_scale) & 3u)) return HIF4X_ERR_ARG;
  if (d->src_kind == HIF4X_SRC_NVFP4_PAIR && d->scale_dtype == HIF4X_DT_BF16 &&
      (reinterpret_cast<uintptr_t>(d->src_scale) & 7u))
    return HIF4X_ERR_ARG;
  ConvParams p;
  p.nb = d->cols / 64;
  p.ngroups = d->rows * p.nb;
  p.src_kind = d->src_kind; p.src_dtype = d->src_dtype; p.scale_dtype = d->scale_dtype;
  p.s_dec = d->s_dec; p.src = d->src; p.src_scale = d->src_scale;
  p.smooth = d->smooth; p.smooth_mode = d->smooth_mode; p.rot_signs = d->rot_signs;
  p.encode_mode = d->encode_mode; p.out_x = d->out_x;
  p.sf = d->sf; p.lv2 = d->lv2; p.lv3 = d->lv3; p.sign = d->sign; p.mant = d->mant;
  p.meta = d->meta; p.codes = d->codes; p.deq = d->deq; p.deq_dtype = d->deq_dtype; p.unit = d->unit;
  const size_t smem = 64 * kConvThreads * sizeof(float);
  const bool packed_only = d->encode_mode == HIF4X_ENC_SEARCH && d->meta && d->codes && !d->out_x && !d->sf &&
                           !d->lv2 && !d->lv3 && !d->sign && !d->mant && !d->deq && !d->unit;
  if (packed_only)
    convert_kernel<true><<<nblocks(p.ngroups, kConvThreads), kConvThreads, smem, (cudaStream_t)stream>>>(p);
  else
    convert_kernel<false><<<nblocks(p.ngroups, kConvThreads), kConvThreads, smem, (cudaStream_t)stream>>>(p);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_nvfp4_decode(const void *carrier, int carrier_dtype, const void *scale, int scale_dtype,
                                  int64_t rows, int64_t cols, void *out, int out_dtype, void *stream) {
  if (!carrier || !scale || !out || rows < 0 || cols % 16 != 0) return HIF4X_ERR_ARG;
  const int64_t nblk = rows * (cols / 16);
  if (nblk == 0) return HIF4X_OK;
  nvfp4_decode_kernel<<<nblocks(nblk, 256), 256, 0, (cudaStream_t)stream>>>(
      HIF4X_SRC_NVFP4_PAIR, carrier, carrier_dtype, scale, scale_dtype, 0.0f, nblk, out, out_dtype);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_nvfp4_decode_packed(const uint8_t *codes, const uint8_t *e4m3, float s_dec, int64_t rows,
                                         int64_t cols, void *out, int out_dtype, void *stream) {
  if (!codes || !e4m3 || !out || rows < 0 || cols % 16 != 0 || (reinterpret_cast<uintptr_t>(codes) & 7u))
    return HIF4X_ERR_ARG;
  const int64_t nsub = rows * (cols / 8);
  if (nsub == 0) return HIF4X_OK;
  if (!al16(out)) {   // the vector stores need a 16-byte aligned output; the one-block-per-thread kernel does not
    nvfp4_decode_kernel<<<nblocks(nsub / 2, 256), 256, 0, (cudaStream_t)stream>>>(
        HIF4X_SRC_NVFP4_PACKED, codes, 0, e4m3, 0, s_dec, nsub / 2, out, out_dtype);
  } else {
    nvfp4_decode_packed_kernel<<<nblocks(nsub, 256 * kDecSubs), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint32_t *>(codes), e4m3, s_dec, nsub, out, out_dtype);
  }
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_rotate64(const float *x, const uint64_t *signs, int64_t rows, int64_t cols, float *out,
                              void *stream) {
  if (!x || !signs || !out || rows < 0 || cols % 64 != 0 || !al16(x) || !al16(out)) return HIF4X_ERR_ARG;
  const int64_t ng = rows * (cols / 64);
  if (ng == 0) return HIF4X_OK;
  rotate64_kernel<<<nblocks(ng, kConvThreads), kConvThreads, 64 * kConvThreads * sizeof(float),
                    (cudaStream_t)stream>>>(x, signs, ng, cols / 64, out);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

static int encode_values(const float *x, int mode, int64_t rows, int64_t cols, float *sf, float *lv2, float *lv3,
                         float *sign, float *mant, void *stream) {
  hif4x_convert_desc d = {};
  d.rows = rows; d.cols = cols; d.src_kind = HIF4X_SRC_VALUES; d.src_dtype = HIF4X_DT_F32; d.src = x;
  d.encode_mode = mode; d.sf = sf; d.lv2 = lv2; d.lv3 = lv3; d.sign = sign; d.mant = mant;
  return hif4x_convert(&d, stream);
}

extern "C" int hif4x_encode_search(const float *x, int64_t rows, int64_t cols, float *sf, float *lv2, float *lv3,
                                   float *sign, float *mant, void *stream) {
  return encode_values(x, HIF4X_ENC_SEARCH, rows, cols, sf, lv2, lv3, sign, mant, stream);
}

extern "C" int hif4x_encode_alg1(const float *x, int64_t rows, int64_t cols, float *sf, float *lv2, float *lv3,
                                 float *sign, float *mant, void *stream) {
  return encode_values(x, HIF4X_ENC_ALG1, rows, cols, sf, lv2, lv3, sign, mant, stream);
}

extern "C" int hif4x_decode_dict5(const float *sf, const float *lv2, const float *lv3, const float *sign,
                                  const float *mant, int64_t rows, int64_t cols, void *out, int out_dtype,
                                  void *stream) {
  if (!sf || !lv2 || !lv3 || !sign || !mant || !out || rows < 0 || cols % 64 != 0) return HIF4X_ERR_ARG;
  const int64_t n = rows * cols;
  if (n == 0) return HIF4X_OK;
  decode_dict5_kernel<<<nblocks(n, 256), 256, 0, (cudaStream_t)stream>>>(sf, lv2, lv3, sign, mant, n, out, out_dtype);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_decode_packed(const uint32_t *meta, const uint8_t *codes, int64_t rows, int64_t cols, void *out,
                                   int out_dtype, void *stream) {
  if (!meta || !codes || !out || rows < 0 || cols % 64 != 0 || !al16(codes) || !al16(out)) return HIF4X_ERR_ARG;
  const int64_t nsub = rows * (cols / 8);
  if (nsub == 0) return HIF4X_OK;
  decode_packed_kernel<<<nblocks(nsub, 256 * kDecSubs), 256, 0, (cudaStream_t)stream>>>(
      meta, reinterpret_cast<const uint32_t *>(codes), nsub, out, out_dtype);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_values_to_params(const float *q, const float *sf, const float *lv2, const float *lv3,
                                      int64_t rows, int64_t cols, float *sign, float *mant, void *stream) {
  if (!q || !sf || !lv2 || !lv3 || !sign || !mant || rows < 0 || cols % 64 != 0) return HIF4X_ERR_ARG;
  const int64_t n = rows * cols;
  if (n == 0) return HIF4X_OK;
  values_to_params_kernel<<<nblocks(n, 256), 256, 0, (cudaStream_t)stream>>>(q, sf, lv2, lv3, n, sign, mant);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_unit_flat(const float *sf, const float *lv2, const float *lv3, int64_t rows, int64_t cols,
                               float *unit, void *stream) {
  if (!sf || !lv2 || !lv3 || !unit || rows < 0 || cols % 64 != 0) return HIF4X_ERR_ARG;
  const int64_t n = rows * cols;
  if (n == 0) return HIF4X_OK;
  unit_flat_kernel<<<nblocks(n, 256), 256, 0, (cudaStream_t)stream>>>(sf, lv2, lv3, n, unit);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_pack_dict5(const float *sf, const float *lv2, const float *lv3, const float *sign,
                                const float *mant, int64_t rows, int64_t cols, uint32_t *meta, uint8_t *codes,
                                void *stream) {
  if (!sf || !lv2 || !lv3 || !sign || !mant || !meta || !codes || rows < 0 || cols % 64 != 0) return HIF4X_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(codes) & 3u) return HIF4X_ERR_ARG;
  const int64_t ng = rows * (cols / 64);
  if (ng == 0) return HIF4X_OK;
  pack_dict5_kernel<<<nblocks(ng, 128), 128, 0, (cudaStream_t)stream>>>(sf, lv2, lv3, sign, mant, ng, meta, codes);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_unpack_dict5(const uint32_t *meta, const uint8_t *codes, int64_t rows, int64_t cols, float *sf,
                                  float *lv2, float *lv3, float *sign, float *mant, void *stream) {
  if (!sf || !lv2 || !lv3 || !sign || !mant || !meta || !codes || rows < 0 || cols % 64 != 0) return HIF4X_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(codes) & 3u) return HIF4X_ERR_ARG;
  const int64_t ng = rows * (cols / 64);
  if (ng == 0) return HIF4X_OK;
  unpack_dict5_kernel<<<nblocks(ng, 128), 128, 0, (cudaStream_t)stream>>>(meta, codes, ng, sf, lv2, lv3, sign, mant);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

extern "C" int hif4x_hif4_rows(const uint32_t *meta, const uint8_t *codes, int64_t rows, int64_t cols, uint8_t *out,
                               void *stream) {
  if (!meta || !codes || !out || rows < 0 || cols % 64 != 0 || (reinterpret_cast<uintptr_t>(codes) & 3u) ||
      (reinterpret_cast<uintptr_t>(out) & 3u))
    return HIF4X_ERR_ARG;
  const int64_t cw = cols / 8, mw = cols / 64, n = rows * (cw + mw);
  if (n == 0) return HIF4X_OK;
  hif4_rows_kernel<<<nblocks(n, 256), 256, 0, (cudaStream_t)stream>>>(
      meta, reinterpret_cast<const uint32_t *>(codes), rows, cw, mw, reinterpret_cast<uint32_t *>(out));
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}
