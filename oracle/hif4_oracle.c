/*
 * hif4_oracle.c -- CPU restatement of the reference's NVFP4 -> HiF4 codec.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the CUDA
 * codec: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs may load it, and only as the checker or as the timed CPU
 * baseline.  The product path never calls it.
 *
 * Every routine restates one reference function, step for step, in plain
 * scalar fp32 C so that each rounding happens where torch's CPU kernels round:
 *   - no FMA contraction (built with -ffp-contract=off), IEEE division;
 *   - torch.round == rintf (round half to even, default rounding mode);
 *   - size-4 and size-8 inner sums run left to right (measured on torch 2.11
 *     CPU; pinned by tests/golden);
 *   - floor(log2(t)) uses glibc log2f, which agrees with torch's vectorised
 *     log2 at every binade boundary (pinned by a CPU test).
 *
 * Parity pins: tests/golden/*.npz hold outputs of the reference itself
 * (example/solution/solution.py, dev/variants.py) on seeded inputs; the
 * generating script is tests/golden/gen_golden.py.
 *
 * Reference functions restated (paths relative to the reference project):
 *   orc_nvfp4_decode        example/solution/solution.py:49-57 (= dev/hif4.py:17-20)
 *   orc_rot64               example/solution/solution.py:222-245 (_rot_blocks)
 *   orc_encode_search       example/solution/solution.py:60-124 (_quant_chunk),
 *                           :744-770 (_quantize_weighted with ones weight)
 *   orc_encode_fast         example/solution/solution.py:787-823 (_quant_weight_fast)
 *   orc_encode_alg1         dev/variants.py:249-287 (quant_alg1, _encode_e6m2)
 *   orc_hif4_decode         dev/hif4.py:37-38 (hif4_dequantize), solution.py:1090-1092
 *   orc_values_to_params    example/solution/solution.py:734-741
 *   orc_rot_signs           example/solution/solution.py:240-242 (seeded sign draw)
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define SF_MIN_F (3.5527136788005009e-15f) /* 2^-48 */
#define SF_MAX_F (49152.0f)

static inline float clampf_(float x, float lo, float hi) {
  /* torch.clamp(x, lo, hi) == min(max(x, lo), hi) for finite x */
  x = x < lo ? lo : x;
  return x > hi ? hi : x;
}

static inline float torch_sign(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

static inline float bf16_round(float x) {
  /* round-to-nearest-even fp32 -> bf16 -> fp32 (finite inputs) */
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  u &= 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

static inline float e4m3_to_f32(uint8_t b) {
  int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) v = ldexpf((float)m, -9); /* m/8 * 2^-6 */
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

static const float E2M1_VAL[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* ------------------------------------------------------------------------ */
/* A1: NVFP4 decode.  (carrier * scale) in the promoted dtype, then bf16.     */
/* carrier_dt / scale_dt: 0 = fp32, 1 = bf16.  Output fp32 holding the bf16. */
void orc_nvfp4_decode(const void *carrier, int carrier_dt, const void *scale, int scale_dt,
                      int64_t R, int64_t C, float *out) {
  const int64_t nbs = C / 16;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < R; r++) {
    for (int64_t c = 0; c < C; c++) {
      float a = carrier_dt ? bf16_to_f32(((const uint16_t *)carrier)[r * C + c])
                           : ((const float *)carrier)[r * C + c];
      float s = scale_dt ? bf16_to_f32(((const uint16_t *)scale)[r * nbs + c / 16])
                         : ((const float *)scale)[r * nbs + c / 16];
      float p = a * s; /* exact product of two bf16 fits fp32; else one fp32 rounding */
      /* bf16 x bf16 promotes to bf16 in torch: one rounding of the exact
       * product to bf16, which is what bf16_round(p) does here too. */
      out[r * C + c] = bf16_round(p);
    }
  }
}

/* Packed NVFP4: codes (R, C/2) nibbles (low nibble = even element; bit 3 =
 * sign, bits 0-2 = E2M1 index), e4m3 block scales (R, C/16), fp32 tensor
 * scale s_dec.  The block scale is fp32(e4m3) * s_dec rounded once to fp32,
 * which is the fp32 scale tensor the reference receives. */
void orc_nvfp4_decode_packed(const uint8_t *codes, const uint8_t *e4m3, float s_dec, int64_t R,
                             int64_t C, float *out) {
  const int64_t nbs = C / 16;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < R; r++) {
    for (int64_t c = 0; c < C; c++) {
      uint8_t byte = codes[r * (C / 2) + c / 2];
      uint8_t nib = (c & 1) ? (byte >> 4) : (byte & 15);
      float a = E2M1_VAL[nib & 7];
      if (nib & 8) a = -a;
      float s = e4m3_to_f32(e4m3[r * nbs + c / 16]) * s_dec;
      out[r * C + c] = bf16_round(a * s);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Sign vectors of _rot_blocks: torch.Generator().manual_seed(seed+b),         */
/* torch.rand(64) < 0.5 -> +1 else -1.  torch's CPU generator is MT19937 and   */
/* rand(float) keeps the low 24 bits of each 32-bit draw, so rand < 0.5 iff    */
/* bit 23 of the draw is clear.  Bit e of out[b] set  <=>  sign -1.            */
typedef struct {
  uint32_t mt[624];
  int idx;
} mt19937_t;

static void mt_seed(mt19937_t *g, uint32_t s) {
  g->mt[0] = s;
  for (int i = 1; i < 624; i++) g->mt[i] = 1812433253u * (g->mt[i - 1] ^ (g->mt[i - 1] >> 30)) + (uint32_t)i;
  g->idx = 624;
}

static uint32_t mt_next(mt19937_t *g) {
  if (g->idx >= 624) {
    for (int i = 0; i < 624; i++) {
      uint32_t y = (g->mt[i] & 0x80000000u) | (g->mt[(i + 1) % 624] & 0x7fffffffu);
      uint32_t v = g->mt[(i + 397) % 624] ^ (y >> 1);
      if (y & 1u) v ^= 0x9908b0dfu;
      g->mt[i] = v;
    }
    g->idx = 0;
  }
  uint32_t y = g->mt[g->idx++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

void orc_rot_signs(int64_t n_vec, int64_t len, uint32_t seed0, uint64_t *out) {
  for (int64_t b = 0; b < n_vec; b++) {
    mt19937_t g;
    mt_seed(&g, (uint32_t)(seed0 + b));
    uint64_t m = 0;
    for (int64_t e = 0; e < len; e++) {
      uint32_t v = mt_next(&g);
      if (v & (1u << 23)) m |= (1ull << e);
    }
    out[b] = m;
  }
}

/* ------------------------------------------------------------------------ */
/* A2: block rotation.  out[r, 64b+e] = sum_d x[r, 64b+d] * Rm[b,d,e] with     */
/* Rm = H64/8 * sign_b[e]; the sum runs d = 0..63 in order from +0, which is   */
/* the order torch's CPU einsum/bmm uses here (pinned by tests/golden).        */
void orc_rot64(const float *x, const uint64_t *signs, int64_t R, int64_t C, float *out) {
  const int64_t nb = C / 64;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < R; r++) {
    for (int64_t b = 0; b < nb; b++) {
      const float *xb = x + r * C + b * 64;
      for (int e = 0; e < 64; e++) {
        float de = ((signs[b] >> e) & 1ull) ? -1.0f : 1.0f;
        float acc = 0.0f;
        for (int d = 0; d < 64; d++) {
          float h = (__builtin_popcount((unsigned)(d & e)) & 1) ? -0.125f : 0.125f;
          float rm = h * de;
          acc = acc + xb[d] * rm;
        }
        out[r * C + b * 64 + e] = acc;
      }
    }
  }
}

/* ------------------------------------------------------------------------ */
static inline float mant_of(float ab, float unit) {
  /* torch.clamp(torch.round(ab / unit * 4.0) / 4.0, 0.0, 1.75) */
  float q = ab / unit;
  q = q * 4.0f;
  q = rintf(q);
  q = q / 4.0f;
  return clampf_(q, 0.0f, 1.75f);
}

static inline float sq_err(float ab, float unit) {
  float m = mant_of(ab, unit);
  float d = m * unit - ab;
  return d * d; /* times the ones weight: exact no-op */
}

static inline float floor_log2(float t) { return floorf(log2f(t)); }

static const int CAND_K[6] = {0, 0, 0, 0, 1, 1};
static const float CAND_SIG[6] = {1.0f, 1.25f, 1.5f, 1.75f, 1.0f, 1.25f};

/* A3: searched hierarchical encode of one 64-group (solution.py:60-124). */
static void encode_search_group(const float *x, float *sf_o, float *lv2_o, float *lv3_o,
                                float *sign_o, float *mant_o) {
  float ab[64], amax = 0.0f;
  for (int i = 0; i < 64; i++) {
    ab[i] = fabsf(x[i]);
    amax = ab[i] > amax ? ab[i] : amax;
  }
  float t = amax / 7.0f;
  t = t < 1e-38f ? 1e-38f : t;
  float e0 = floor_log2(t);

  float err_best = 0.0f, sf_best = 0.0f, l2_best[8], l3_best[16];
  for (int c = 0; c < 6; c++) {
    float sf = clampf_(exp2f(e0 + (float)CAND_K[c]) * CAND_SIG[c], SF_MIN_F, SF_MAX_F);
    float be2[8], bl2[8], bl3[16];
    for (int l2i = 0; l2i < 2; l2i++) {
      float lv2c = l2i ? 2.0f : 1.0f;
      float e3a[16], e3b[16];
      for (int l3i = 0; l3i < 2; l3i++) {
        float unit = (sf * lv2c) * (l3i ? 2.0f : 1.0f);
        float *dst = l3i ? e3b : e3a;
        for (int j = 0; j < 16; j++) {
          float s = sq_err(ab[4 * j + 0], unit);
          s = s + sq_err(ab[4 * j + 1], unit);
          s = s + sq_err(ab[4 * j + 2], unit);
          s = s + sq_err(ab[4 * j + 3], unit);
          dst[j] = s;
        }
      }
      float e3[16], l3[16], e2[8];
      for (int j = 0; j < 16; j++) {
        int take1 = e3a[j] <= e3b[j];
        e3[j] = take1 ? e3a[j] : e3b[j];
        l3[j] = take1 ? 1.0f : 2.0f;
      }
      for (int i = 0; i < 8; i++) e2[i] = e3[2 * i] + e3[2 * i + 1];
      if (l2i == 0) {
        for (int i = 0; i < 8; i++) { be2[i] = e2[i]; bl2[i] = 1.0f; }
        for (int j = 0; j < 16; j++) bl3[j] = l3[j];
      } else {
        for (int i = 0; i < 8; i++) {
          if (e2[i] < be2[i]) {
            be2[i] = e2[i];
            bl2[i] = 2.0f;
            bl3[2 * i] = l3[2 * i];
            bl3[2 * i + 1] = l3[2 * i + 1];
          }
        }
      }
    }
    float err = be2[0];
    for (int i = 1; i < 8; i++) err = err + be2[i];
    if (c == 0 || err < err_best) {
      err_best = err;
      sf_best = sf;
      memcpy(l2_best, bl2, sizeof bl2);
      memcpy(l3_best, bl3, sizeof bl3);
    }
  }
  *sf_o = sf_best;
  for (int i = 0; i < 8; i++) lv2_o[i] = l2_best[i];
  for (int j = 0; j < 16; j++) lv3_o[j] = l3_best[j];
  for (int i = 0; i < 64; i++) {
    float unit = (sf_best * l2_best[i / 8]) * l3_best[i / 4];
    mant_o[i] = mant_of(ab[i], unit);
    sign_o[i] = torch_sign(x[i]);
  }
}

/* dict5 outputs: sf (R, nb), lv2 (R, nb, 8), lv3 (R, nb, 16), sign/mant (R, C) */
void orc_encode_search(const float *x, int64_t R, int64_t C, float *sf, float *lv2, float *lv3,
                       float *sign, float *mant) {
  const int64_t nb = C / 64;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < R * nb; g++) {
    encode_search_group(x + g * 64, sf + g, lv2 + g * 8, lv3 + g * 16, sign + g * 64, mant + g * 64);
  }
}

/* A6 helper: _quant_weight_fast (solution.py:787-823).  Greedy lv tree, four
 * significands at the anchor exponent.  The 64-term error sum is taken left
 * to right here; torch reduces it with a vectorised cascade whose order is
 * CPU-dependent, so this routine is pinned by tolerance, not bit for bit. */
static void encode_fast_group(const float *x, float *sf_o, float *lv2_o, float *lv3_o, float *sign_o,
                              float *mant_o) {
  float ab[64], amax = 0.0f, a8[8], a4[16];
  for (int i = 0; i < 64; i++) {
    ab[i] = fabsf(x[i]);
    amax = ab[i] > amax ? ab[i] : amax;
  }
  for (int j = 0; j < 16; j++) {
    float m = ab[4 * j];
    for (int k = 1; k < 4; k++) m = ab[4 * j + k] > m ? ab[4 * j + k] : m;
    a4[j] = m;
  }
  for (int i = 0; i < 8; i++) a8[i] = a4[2 * i] > a4[2 * i + 1] ? a4[2 * i] : a4[2 * i + 1];
  float t = amax / 7.0f;
  t = t < 1e-38f ? 1e-38f : t;
  float e0 = floor_log2(t);
  float best = 0.0f, sfb = 0.0f;
  for (int c = 0; c < 4; c++) {
    float sf = clampf_(exp2f(e0) * CAND_SIG[c], SF_MIN_F, SF_MAX_F);
    float err = 0.0f;
    for (int i = 0; i < 64; i++) {
      float l2 = (a8[i / 8] / sf > 1.75f) ? 2.0f : 1.0f;
      float l3 = (a4[i / 4] / (sf * l2) > 1.75f) ? 2.0f : 1.0f;
      float unit = (sf * l2) * l3;
      err = err + sq_err(ab[i], unit);
    }
    if (c == 0 || err < best) {
      best = err;
      sfb = sf;
    }
  }
  *sf_o = sfb;
  for (int i = 0; i < 8; i++) lv2_o[i] = (a8[i] / sfb > 1.75f) ? 2.0f : 1.0f;
  for (int j = 0; j < 16; j++) lv3_o[j] = (a4[j] / (sfb * lv2_o[j / 2]) > 1.75f) ? 2.0f : 1.0f;
  for (int i = 0; i < 64; i++) {
    float unit = (sfb * lv2_o[i / 8]) * lv3_o[i / 4];
    mant_o[i] = mant_of(ab[i], unit);
    sign_o[i] = torch_sign(x[i]);
  }
}

void orc_encode_fast(const float *x, int64_t R, int64_t C, float *sf, float *lv2, float *lv3,
                     float *sign, float *mant) {
  const int64_t nb = C / 64;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < R * nb; g++)
    encode_fast_group(x + g * 64, sf + g, lv2 + g * 8, lv3 + g * 16, sign + g * 64, mant + g * 64);
}

/* ------------------------------------------------------------------------ */
/* A4: paper Algorithm 1 exactly as dev/variants.py:249-287 computes it.     */
static float encode_e6m2(float x) {
  float xc = x < 1e-30f ? 1e-30f : x;
  float e = floor_log2(xc);
  float m = rintf(xc * exp2f(2.0f - e));
  m = clampf_(m, 4.0f, 8.0f);
  float out = m * exp2f(e - 2.0f);
  return clampf_(out, SF_MIN_F, SF_MAX_F);
}

static void encode_alg1_group(const float *x, float *sf_o, float *lv2_o, float *lv3_o, float *sign_o,
                              float *mant_o) {
  float v16[16], v8[8], vmax;
  for (int j = 0; j < 16; j++) {
    float m = fabsf(x[4 * j]);
    for (int k = 1; k < 4; k++) {
      float a = fabsf(x[4 * j + k]);
      m = a > m ? a : m;
    }
    v16[j] = m;
  }
  for (int i = 0; i < 8; i++) v8[i] = v16[2 * i] > v16[2 * i + 1] ? v16[2 * i] : v16[2 * i + 1];
  vmax = v8[0];
  for (int i = 1; i < 8; i++) vmax = v8[i] > vmax ? v8[i] : vmax;
  float sf = encode_e6m2(vmax / 7.0f);
  float rec = 1.0f / sf;
  float e18[8], e116[16];
  for (int i = 0; i < 8; i++) e18[i] = (v8[i] * rec >= 4.0f) ? 1.0f : 0.0f;
  for (int j = 0; j < 16; j++) e116[j] = ((v16[j] * rec) * exp2f(-e18[j / 2]) >= 2.0f) ? 1.0f : 0.0f;
  *sf_o = sf;
  for (int i = 0; i < 8; i++) lv2_o[i] = exp2f(e18[i]);
  for (int j = 0; j < 16; j++) lv3_o[j] = exp2f(e116[j]);
  for (int i = 0; i < 64; i++) {
    float xs = ((x[i] * rec) * exp2f(-e18[i / 8])) * exp2f(-e116[i / 4]);
    float sg = torch_sign(xs);
    float qi = floorf(fabsf(xs) * 4.0f + 0.5f);
    qi = clampf_(qi, 0.0f, 7.0f);
    float mant = qi / 4.0f;
    mant_o[i] = mant;
    sign_o[i] = (mant == 0.0f) ? 0.0f : sg;
  }
}

void orc_encode_alg1(const float *x, int64_t R, int64_t C, float *sf, float *lv2, float *lv3,
                     float *sign, float *mant) {
  const int64_t nb = C / 64;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < R * nb; g++)
    encode_alg1_group(x + g * 64, sf + g, lv2 + g * 8, lv3 + g * 16, sign + g * 64, mant + g * 64);
}

/* ------------------------------------------------------------------------ */
/* A5: decode dict5 -> values: sign * mant * lv3 * lv2 * sf, left to right.  */
void orc_hif4_decode(const float *sf, const float *lv2, const float *lv3, const float *sign,
                     const float *mant, int64_t R, int64_t C, float *out) {
  const int64_t nb = C / 64;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < R * nb; g++) {
    for (int i = 0; i < 64; i++) {
      float v = sign[g * 64 + i] * mant[g * 64 + i];
      v = v * lv3[g * 16 + i / 4];
      v = v * lv2[g * 8 + i / 8];
      out[g * 64 + i] = v * sf[g];
    }
  }
}

/* _params_unit_flat: unit = sf * lv2 * lv3 (solution.py:726-731). */
void orc_unit_flat(const float *sf, const float *lv2, const float *lv3, int64_t R, int64_t C,
                   float *unit) {
  const int64_t nb = C / 64;
  for (int64_t g = 0; g < R * nb; g++)
    for (int i = 0; i < 64; i++) unit[g * 64 + i] = (sf[g] * lv2[g * 8 + i / 8]) * lv3[g * 16 + i / 4];
}

/* _values_to_params: re-encode grid values on fixed sf/lv2/lv3. */
void orc_values_to_params(const float *q, const float *sf, const float *lv2, const float *lv3,
                          int64_t R, int64_t C, float *sign, float *mant) {
  const int64_t nb = C / 64;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < R * nb; g++) {
    for (int i = 0; i < 64; i++) {
      float unit = (sf[g] * lv2[g * 8 + i / 8]) * lv3[g * 16 + i / 4];
      float v = q[g * 64 + i];
      float m = rintf(fabsf(v) / unit * 4.0f);
      m = clampf_(m, 0.0f, 7.0f) * 0.25f;
      mant[g * 64 + i] = m;
      sign[g * 64 + i] = torch_sign(v);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Packed HiF4 (4.5 bit/elem): per 64-group a 32-bit word (bits 0-7 E6M2 code
 * = (E+48)<<2 | M, bits 8-15 E1_8, bits 16-31 E1_16) and 32 bytes of S1P2
 * nibbles (low nibble = even element; bit 3 = sign, bits 0-2 = mant*4).   */
static inline uint32_t e6m2_code(float sf) {
  int e;
  float m = frexpf(sf, &e); /* sf = m * 2^e, m in [0.5, 1) */
  int E = e - 1;
  int M = (int)rintf((m * 2.0f - 1.0f) * 4.0f);
  return (uint32_t)(((E + 48) << 2) | M);
}

void orc_pack_hif4(const float *sf, const float *lv2, const float *lv3, const float *sign,
                   const float *mant, int64_t R, int64_t C, uint32_t *meta, uint8_t *codes) {
  const int64_t nb = C / 64;
  for (int64_t g = 0; g < R * nb; g++) {
    uint32_t w = e6m2_code(sf[g]);
    for (int i = 0; i < 8; i++) w |= (lv2[g * 8 + i] == 2.0f ? 1u : 0u) << (8 + i);
    for (int j = 0; j < 16; j++) w |= (lv3[g * 16 + j] == 2.0f ? 1u : 0u) << (16 + j);
    meta[g] = w;
    for (int i = 0; i < 64; i += 2) {
      uint8_t n0 = (uint8_t)((sign[g * 64 + i] < 0.0f ? 8 : 0) | (int)(mant[g * 64 + i] * 4.0f));
      uint8_t n1 = (uint8_t)((sign[g * 64 + i + 1] < 0.0f ? 8 : 0) | (int)(mant[g * 64 + i + 1] * 4.0f));
      codes[g * 32 + i / 2] = (uint8_t)(n0 | (n1 << 4));
    }
  }
}
