/*
 * hif4x.h -- C ABI of the B200 NVFP4 -> HiF4 conversion engine.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns an
 * int status (HIF4X_OK = 0; > 0 recoverable, the caller takes the
 * reference's fallback branch; < 0 a caller or launch error).  Pointers are
 * borrowed: the library never frees caller memory.  Tensors are dense
 * row-major; a matrix (R, C) has C % 64 == 0 unless noted.
 *
 * Each declaration names the reference function it replaces (paths relative
 * to the reference project, openaddr/hif4-contest).
 *
 * Formats
 *   NVFP4 packed : codes uint8 (R, C/2), nibble = sign<<3 | E2M1 index,
 *                  element 2i in the low nibble of byte i; e4m3 uint8
 *                  (R, C/16) one E4M3 scale per 16 elements; fp32 s_dec.
 *   NVFP4 pair   : the reference's [carrier, scale] pair: carrier (R, C)
 *                  bf16 or fp32 holding E2M1 values, scale (R, C/16) fp32
 *                  or bf16 (example/solution/solution.py:49-57).
 *   dict5        : the reference's HiF4 parameters as five fp32 arrays:
 *                  sf (R, C/64), lv2 (R, C/64, 8), lv3 (R, C/64, 16),
 *                  sign (R, C), mant (R, C)  (example/self_check.py:75-95).
 *   HiF4 packed  : meta uint32 (R, C/64): bits 0-7 E6M2 code
 *                  ((E+48)<<2 | M), bits 8-15 E1_8, bits 16-31 E1_16;
 *                  codes uint8 (R, C/2): nibble = sign<<3 | mant*4
 *                  (hif4_paper.txt section II-A layout, 4.5 bit/elem).
 */
#ifndef HIF4X_H_
#define HIF4X_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define HIF4X_OK 0
#define HIF4X_NOT_PD 1            /* Cholesky met a non-positive pivot        */
#define HIF4X_TIMEOUT 2           /* a bounded device wait gave up            */
#define HIF4X_ERR_ARG (-1)        /* bad pointer / size / alignment           */
#define HIF4X_ERR_LAUNCH (-2)     /* CUDA launch or runtime error             */
#define HIF4X_ERR_UNSUPPORTED (-3)
#define HIF4X_ERR_SCRATCH (-4)    /* size above a static scratch maximum      */
#define HIF4X_ERR_NOMEM (-5)      /* a stream-ordered workspace (the tensor-core
                                     GEMM's split operands, the attention's
                                     buffers) could not be allocated          */

/* ---- enums ------------------------------------------------------------- */
#define HIF4X_DT_F32 0
#define HIF4X_DT_BF16 1
#define HIF4X_DT_F64 2             /* vcomp entry points only                */

#define HIF4X_SRC_NVFP4_PACKED 0  /* src = codes, src_scale = e4m3, s_dec     */
#define HIF4X_SRC_NVFP4_PAIR 1    /* src = carrier, src_scale = scale         */
#define HIF4X_SRC_VALUES 2        /* src = values (src_dtype), no decode      */

#define HIF4X_SMOOTH_NONE 0
#define HIF4X_SMOOTH_MUL 1        /* x * s[c]  (activations)                  */
#define HIF4X_SMOOTH_DIV 2        /* x / s[c]  (weights)                      */

#define HIF4X_ENC_NONE 0          /* decode / transform only                  */
#define HIF4X_ENC_SEARCH 1        /* 6-candidate searched encode              */
#define HIF4X_ENC_FAST 2          /* 4-candidate greedy-lv encode             */
#define HIF4X_ENC_ALG1 3          /* paper Algorithm 1 (standard quantizer)   */

/* One fused pass: source decode -> optional per-channel smoothing ->
 * optional 64-point block rotation -> optional HiF4 encode, writing any
 * subset of the outputs (NULL = not written).  One thread per 64-group; the
 * input is read once. */
typedef struct hif4x_convert_desc {
  int64_t rows, cols;
  int src_kind;              /* HIF4X_SRC_*                                   */
  int src_dtype;             /* carrier / values dtype (HIF4X_DT_*)           */
  int scale_dtype;           /* pair scale dtype (HIF4X_DT_*)                 */
  float s_dec;               /* packed NVFP4 tensor scale                     */
  const void *src;           /* codes | carrier | values                      */
  const void *src_scale;     /* e4m3 | scale | NULL                           */
  const float *smooth;       /* (cols,) per-channel factor or NULL            */
  int smooth_mode;           /* HIF4X_SMOOTH_*                                */
  const uint64_t *rot_signs; /* (cols/64,) sign masks, NULL = no rotation     */
  int encode_mode;           /* HIF4X_ENC_*                                   */
  float *out_x;              /* (R, C) transformed fp32 values                */
  float *sf, *lv2, *lv3, *sign, *mant; /* dict5                               */
  uint32_t *meta;            /* packed HiF4 metadata                          */
  uint8_t *codes;            /* packed HiF4 nibbles                           */
  void *deq;                 /* (R, C) HiF4-decoded values                    */
  int deq_dtype;             /* HIF4X_DT_*                                    */
  float *unit;               /* (R, C) sf*lv2*lv3                             */
} hif4x_convert_desc;

/* Library version (major*10000 + minor*100 + patch). */
int hif4x_version(void);

/* Fused convert.  Replaces, in one launch, the chain
 *   dequantize_nvfp4 (example/solution/solution.py:49-57)
 *   -> a * s / w / s smoothing (solution.py:871-873, 1049)
 *   -> _rot_blocks (solution.py:222-245)
 *   -> _quantize_weighted / _quant_chunk (solution.py:744-770, 60-124)
 *      | _quant_weight_fast (solution.py:787-823)
 *      | quant_alg1 (dev/variants.py:249-287). */
int hif4x_convert(const hif4x_convert_desc *desc, void *stream);

/* dequantize_nvfp4, pair form (example/solution/solution.py:49-57,
 * dev/hif4.py:17-20).  out (R, C) of out_dtype; C % 16 == 0. */
int hif4x_nvfp4_decode(const void *carrier, int carrier_dtype, const void *scale, int scale_dtype,
                       int64_t rows, int64_t cols, void *out, int out_dtype, void *stream);

/* dequantize_nvfp4 of the packed form (same result as the pair form whose
 * scale is fp32(e4m3) * s_dec). */
int hif4x_nvfp4_decode_packed(const uint8_t *codes, const uint8_t *e4m3, float s_dec, int64_t rows,
                              int64_t cols, void *out, int out_dtype, void *stream);

/* _rot_blocks (example/solution/solution.py:222-245): bit-exact with the
 * reference's fp32 einsum.  signs: device table of cols/64 masks from
 * hif4x_rot_signs (seed0 777). */
int hif4x_rotate64(const float *x, const uint64_t *signs, int64_t rows, int64_t cols, float *out,
                   void *stream);

/* Host: the reference's rotation sign masks.  Vector b (ceil(len/64) words)
 * has bit e set when torch.Generator().manual_seed(seed0 + b) draws
 * rand(len)[e] >= 0.5, i.e. sign -1 (solution.py:240-242 with seed0 777,
 * len 64; _make_R, solution.py:1114-1115, with seed0 0xA5A5 + dh, len dh). */
int hif4x_rot_signs(int64_t n_vec, int64_t len, uint32_t seed0, uint64_t *out_host);

/* _quantize_weighted(x, ones) (example/solution/solution.py:744-770) on fp32
 * values; writes dict5 (all five non-NULL). */
int hif4x_encode_search(const float *x, int64_t rows, int64_t cols, float *sf, float *lv2,
                        float *lv3, float *sign, float *mant, void *stream);

/* quant_alg1 (dev/variants.py:249-287), dict5 out. */
int hif4x_encode_alg1(const float *x, int64_t rows, int64_t cols, float *sf, float *lv2, float *lv3,
                      float *sign, float *mant, void *stream);

/* hif4_dequantize / _deq_params (dev/hif4.py:37-38, solution.py:1090-1092):
 * dict5 -> values (out_dtype). */
int hif4x_decode_dict5(const float *sf, const float *lv2, const float *lv3, const float *sign,
                       const float *mant, int64_t rows, int64_t cols, void *out, int out_dtype,
                       void *stream);

/* HiF4 packed -> values (out_dtype); the packed twin of hif4_dequantize. */
int hif4x_decode_packed(const uint32_t *meta, const uint8_t *codes, int64_t rows, int64_t cols,
                        void *out, int out_dtype, void *stream);

/* _values_to_params (example/solution/solution.py:734-741): re-encode values
 * q onto fixed sf/lv2/lv3; writes sign and mant (dict5 form). */
int hif4x_values_to_params(const float *q, const float *sf, const float *lv2, const float *lv3,
                           int64_t rows, int64_t cols, float *sign, float *mant, void *stream);

/* _params_unit_flat (example/solution/solution.py:726-731): unit (R, C). */
int hif4x_unit_flat(const float *sf, const float *lv2, const float *lv3, int64_t rows, int64_t cols,
                    float *unit, void *stream);

/* Packed HiF4 rows (no counterpart in the reference, which only
 * materialises dict5): row r of `out` is the row's C/2 code bytes followed by
 * its C/64 meta words, 9C/16 bytes per row, so a row range of a converted
 * tensor leaves the device in one contiguous copy.  codes, out 4-byte aligned. */
int hif4x_hif4_rows(const uint32_t *meta, const uint8_t *codes, int64_t rows, int64_t cols, uint8_t *out,
                    void *stream);
/* dict5 <-> HiF4 packed.  Unpack writes sign = 0 where mant == 0 and the
 * packed sign bit is clear, -1 where it is set (the packed form keeps the
 * value, not the sign of a zero element). */
int hif4x_pack_dict5(const float *sf, const float *lv2, const float *lv3, const float *sign,
                     const float *mant, int64_t rows, int64_t cols, uint32_t *meta, uint8_t *codes,
                     void *stream);
int hif4x_unpack_dict5(const uint32_t *meta, const uint8_t *codes, int64_t rows, int64_t cols,
                       float *sf, float *lv2, float *lv3, float *sign, float *mant, void *stream);


/* ---- calibration pipeline: linear algebra (csrc/linalg.cu) ------------- */

/* Strided-batched fp32 GEMM, row-major:  C = alpha * op(A) op(B) + beta * C,
 * op(A) = A (M x K, lda) or A^T (A stored K x M) when ta; same for B.
 * Replaces every fp32 `@` / torch.matmul / einsum of the calibration path
 * (e.g. example/solution/solution.py:860, 868, 894, 906, 928-931, 941, 1011-1012). */
int hif4x_gemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
               int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C, int64_t ldc,
               int64_t strideC, int64_t batch, void *stream);

/* The same GEMM on the CUDA cores only: round-to-nearest fp32 FMAs, for
 * products whose result is differenced against another product (the guard
 * MSEs and the refinement residual image, solution.py:637, 868, 906, 930-931,
 * 970-971), where the tensor cores' truncating accumulation would be
 * amplified by cancellation. */
int hif4x_gemm_simt(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                    int64_t strideA, const float *B, int64_t ldb, int64_t strideB, float beta, float *C,
                    int64_t ldc, int64_t strideC, int64_t batch, void *stream);

/* G = X^T X + beta G (beta 0 or 1), G (C x C, leading dim ldg) exactly
 * symmetric: the Hessians and Grams of the calibration (example/solution/
 * solution.py:891-894 sum_i tf_i^T tf_i, 941 and 1011 q^T q, 682-692 Gxx)
 * with only the tiles on or below the diagonal multiplied, then mirrored.
 * X: T x C, leading dim ldx. */
int hif4x_gram(const float *X, int64_t T, int64_t C, int64_t ldx, float beta, float *G, int64_t ldg, void *stream);

/* Tensor-core form of hif4x_gemm (batch 1): tcgen05.mma kind::tf32 with
 * operands split hi + lo (3 products, fp32-faithful), TMA-fed, accumulators
 * in tensor memory.  Needs 16-byte aligned A/B and lda, ldb % 4 == 0, else
 * returns HIF4X_ERR_UNSUPPORTED.  hif4x_gemm uses it for large products. */
int hif4x_gemm_tc(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                  const float *B, int64_t ldb, float beta, float *C, int64_t ldc, void *stream);

/* Synchronises the stream; returns (and clears) the sticky device status:
 * HIF4X_TIMEOUT if a bounded device-side wait expired since the last call.
 * One status word per device (not per stream): a read clears it for every
 * stream of that device. */
int hif4x_device_status(void *stream);

/* Failure-path check of the bounded device-side wait (no counterpart in the
 * reference, which has no device code): one thread waits `spins` polls
 * (1 .. 2^22) on an mbarrier that nothing arrives on, with no copy or MMA in
 * flight, and gives up; *done_dev becomes 2 and the device status then reads
 * HIF4X_TIMEOUT.  Synchronises the stream. */
int hif4x_wait_selftest(long long spins, int *done_dev, void *stream);

/* _upper_cholesky_inv (example/solution/solution.py:287-300): U upper with
 * U^T U = (H + damp * max(mean(diag H), 1e-30) I)^-1, for `batch` n x n
 * matrices.  Computed as U = J L^-1 J with J H J = L L^T: one recursive
 * Cholesky of the index-reversed matrix that builds L^-1 as it goes.
 * Synchronises the stream; returns HIF4X_NOT_PD (U undefined) where the
 * reference's torch Cholesky would raise.  work: 2*n*n floats (about
 * 1.34*n*n used); info_dev: one device int.  Part of the products run on a
 * second stream the library keeps per caller stream, joined before return. */
int hif4x_chol_upper_inv(const float *H, int64_t n, int64_t batch, float damp, float *U, float *work,
                         int *info_dev, void *stream);

/* hif4x_chol_upper_inv without the synchronisation: launches the work on
 * `stream` and returns; *info_dev becomes nonzero (once the stream reaches
 * it) where hif4x_chol_upper_inv would return HIF4X_NOT_PD.  Lets a caller
 * run independent factorisations on several streams. */
int hif4x_chol_upper_inv_async(const float *H, int64_t n, int64_t batch, float damp, float *U, float *work,
                               int *info_dev, void *stream);

/* The rotated space's factor from the unrotated one, for the transform
 * choice (example/solution/solution.py:875-911 factors the Hessian of the
 * rotated activations anew): with M the block rotation of _rot_blocks
 * (solution.py:222-245), H1 = M^T H0 M and the damping is the same in both
 * spaces, so U1 = chol_upper(H1_d^-1) is the positive-diagonal R factor of
 * U0 M -- upper triangular but for its 64 x 64 diagonal blocks.  Computed as
 * a Householder QR of each diagonal block and the blocks above it multiplied
 * by Q_b^T (about 64 n^2 multiply-adds instead of the Gram and Cholesky's n^3).
 * U0: n x n upper factor of H0_d^-1 (hif4x_chol_upper_inv); signs: the n/64
 * masks of hif4x_rot_signs (seed0 777); U1: n x n, 16-byte aligned, not U0;
 * work: 64*n floats.  n % 64 == 0.  Equal to hif4x_chol_upper_inv of the
 * rotated activations' Gram up to float rounding. */
int hif4x_chol_rotate64(const float *U0, int64_t n, const uint64_t *signs, float *U1, float *work, void *stream);

/* Allocation-free twin of hif4x_chol_upper_inv (no counterpart in the
 * reference).  For callers that cannot allocate device memory at the call --
 * a host whose device memory another runtime plans up front, or a
 * latency-bound loop that must not call the allocator (which can synchronise
 * the device) -- it takes no work or info buffers: its scratch is a static
 * device array of 2*512*512 floats (2 MiB, held by every GPU that loads the
 * library until exit), so n <= 512; larger n returns HIF4X_ERR_SCRATCH.
 * The first call on a device, with that device current, looks up the array's
 * device address (cudaGetSymbolAddress) and caches it per device ordinal, for
 * the runtime's primary context of that device.  Every call copies its pivot
 * flag to the host and synchronises `stream`, so it can never run inside a
 * stream capture.  All calls share the one array and each call clears the
 * pivot flag it needs; calls that overlap on the GPU race.  Its products run
 * on the SIMT GEMM only (the tensor-core path allocates).  The same factor as
 * hif4x_chol_upper_inv up to float rounding (blocked Cholesky then triangular
 * inverse, not the recursion), with the same status codes. */
int hif4x_chol_upper_inv_noalloc(const float *H, int64_t n, int64_t batch, float damp, float *U, void *stream);

/* _gptq_quantize_values / _gptq_quantize_batched (example/solution/
 * solution.py:303-425): column-sequential GPTQ over the last axis in blocks of
 * 128 with lazy trailing updates.  X, unit, Q: batch x R x C; U: C x C with
 * batch stride u_batch_stride (0 = shared).  work: batch*R*(C+128) floats. */
int hif4x_gptq(const float *X, const float *unit, const float *U, int64_t R, int64_t C, int64_t batch,
               int64_t u_batch_stride, float *Q, float *work, void *stream);

/* _rounds_active / _rounds_np (example/solution/solution.py:474-618): greedy
 * top-1 flips per row for `rounds` rounds against the Gram G (C x C); M, v4
 * (T x C) updated in place, d = 0.25*unit.  C <= 8192.  flips (T ints, may be
 * NULL) receives the flip count per row. */
int hif4x_refine_rows(float *M, float *v4, const float *d, const float *G, int64_t T, int64_t C, int rounds,
                      int *flips, void *stream);

/* ---- calibration pipeline: helpers (csrc/util.cu) ---------------------- */

/* Column sums of squares, float64 accumulation rounded once to fp32: the
 * diagonal of q^T q that orders the act-order permutation (example/solution/
 * solution.py:946, argsort(Ha.diagonal())).  For the few-bit HiF4 values it
 * is the exact diagonal, as the reference's fp32 GEMM computes it, where a
 * tensor-core product's truncating accumulation is not.  work: 64*C doubles. */
int hif4x_col_sumsq(const float *X, int64_t R, int64_t C, float *out, double *work, void *stream);

/* out[c] (+)= sum_r |X[r][c]| (solution.py:850).  work: 64*C floats. */
int hif4x_col_abs_sum(const float *X, int64_t R, int64_t C, float *out, int accumulate, float *work,
                      void *stream);
/* logm = log(max(abs_sum/n_tok, 1e-12)) centred (solution.py:855-857). */
int hif4x_smooth_logm(const float *abs_sum, int64_t C, int64_t n_tok, float *logm, void *stream);
/* s = exp(alpha * logm) (solution.py:864, 871). */
int hif4x_exp_scale(const float *logm, int64_t C, float alpha, float *s, void *stream);
/* dst = src[idx] (rows), dst = src[:, idx], dst[:, idx] = src, out = A[idx][:, idx]
 * (solution.py:858-859, 946, 958-967, 1060-1064). */
int hif4x_gather_rows(const float *src, const int64_t *idx, int64_t n, int64_t C, float *dst, void *stream);
int hif4x_gather_cols(const float *src, const int64_t *idx, int64_t R, int64_t C, float *dst, void *stream);
int hif4x_scatter_cols(const float *src, const int64_t *idx, int64_t R, int64_t C, float *dst, void *stream);
int hif4x_permute_sym(const float *A, const int64_t *idx, int64_t n, float *out, void *stream);
/* out = X * s[c] or X / s[c] (solution.py:865-873, 1049). */
int hif4x_scale_cols(const float *X, const float *s, int64_t R, int64_t C, int mode, float *out, void *stream);
/* op 0: sum((A - B)^2), op 1: sum(|A|), double result (the guards' MSEs,
 * solution.py:868, 906, 930-931; the weight hash, solution.py:995).
 * work: 1024 doubles. */
int hif4x_reduce(const float *A, const float *B, int64_t n, int op, double *out, double *work, void *stream);
/* out[i] = A[i][i] */
int hif4x_diag(const float *A, int64_t n, float *out, void *stream);
/* torch.argsort(v, descending=True) (solution.py:945); ties by index; n <= 16384. */
int hif4x_argsort_desc(const float *v, int64_t n, int64_t *idx, void *stream);
/* fp32 <-> bf16 (solution.py:1011-1012, 1077). */
int hif4x_cast(const void *in, int in_dtype, void *out, int out_dtype, int64_t n, void *stream);
/* v4 = round(values/unit*4), d = unit/4 (solution.py:634-635). */
int hif4x_refine_prep(const float *values, const float *unit, int64_t n, float *v4, float *d, void *stream);
/* out = a*b + alpha*c elementwise (b, c may be NULL). */
int hif4x_axpby(const float *a, const float *b, const float *c, float alpha, int64_t n, float *out, void *stream);

/* Compact activation state (no counterpart in the reference, which carries
 * u_act / gw / gwf as C x C tensors, solution.py:1016-1025): an NVFP4
 * carrier of E2M1 values (fp32 or bf16, n even) packed two per byte, element
 * 2i in the low nibble, nibble = sign<<3 | E2M1 index (-0 kept); *bad_dev
 * (device int, not cleared here) counts elements that are not E2M1 values. */
int hif4x_e2m1_pack(const void *carrier, int dtype, int64_t n, uint8_t *codes, int *bad_dev, void *stream);
/* Inverse of hif4x_e2m1_pack into a bf16 or fp32 carrier. */
int hif4x_e2m1_unpack(const uint8_t *codes, int64_t n, void *carrier, int dtype, void *stream);

/* ---- attention path (csrc/attention.cu) -------------------------------- */

/* _attention_out / attn_ref (example/solution/solution.py:1247-1258,
 * dev/hif4.py:59-71): fp32 GQA softmax(Q K^T / sqrt(dh)) V, non-causal.
 * Q, O: (T, qh*dh); K, V: (T, kvh*dh); dh <= 128. */
int hif4x_attention(const float *Q, const float *K, const float *V, int64_t T, int qh, int kvh, int dh, float *O,
                    void *stream);

/* (T, H, D) -> (H, T, D) (inverse = 0) or back (inverse = 1); the head
 * permutes of solution.py:1217-1225, 1353-1361. */
int hif4x_heads_transpose(const float *in, int64_t T, int64_t H, int64_t D, int inverse, float *out, void *stream);

/* ---- attention V compensation (csrc/vcomp.cu) --------------------------- */

/* f64 GEMM for _v_compensate's Grams and products (example/solution/
 * solution.py:1306-1319, torch .double() matmuls): C = alpha op(A) op(B) +
 * beta C with A, B fp32 or f64 (a_dtype / b_dtype: HIF4X_DT_F32 or
 * HIF4X_DT_F64), f64 accumulation and C; batched by element strides sA, sB,
 * sC.  lower = 1 (M == N) computes only the 64 x 64 tiles on or below the
 * diagonal. */
int hif4x_gemm_f64(int ta, int tb, int a_dtype, int b_dtype, int64_t M, int64_t N, int64_t K, double alpha,
                   const void *A, int64_t lda, int64_t sA, const void *B, int64_t ldb, int64_t sB, double beta,
                   double *C, int64_t ldc, int64_t sC, int64_t batch, int lower, void *stream);
/* Copy the lower triangle of each n x n f64 matrix onto its upper one. */
int hif4x_mirror_lower_f64(double *A, int64_t n, int64_t batch, void *stream);
/* torch.linalg.solve(G + lam, Cm) V of solution.py:1316-1319, as
 * X = (A + lam 1 1^T)^-1 Rhs with lam = lam_rel * mean(diag A) added to every
 * entry (the reference's broadcast), by a blocked f64 Cholesky and two
 * triangular solves.  A (batch, n, n) f64, lower triangle read, overwritten;
 * Rhs, X (batch, n, m) f64.  work: batch * (n*n + ceil(n/64)*4096 + 2*n*m)
 * doubles; info_dev: one int.  Synchronises the stream; HIF4X_NOT_PD where a
 * pivot is not positive (the reference's solve raising takes its fallback). */
int hif4x_chol_solve_f64(double *A, int64_t n, int64_t batch, double lam_rel, const double *Rhs, int64_t m,
                         double *X, double *work, int *info_dev, void *stream);
/* torch.softmax(S / div, dim=-1) in place, fp32, rows x cols (solution.py:
 * 1308-1311). */
int hif4x_softmax_rows(float *S, int64_t rows, int64_t cols, float div, void *stream);
/* out[b*obs + j*old + i] = in[b*ibs + i*ild + j], i < R, j < Cc: the
 * (T, kvh, dh) <-> (kvh, dh, T) permutes of solution.py:1324-1330. */
int hif4x_transpose_batched(const float *in, int64_t R, int64_t Cc, int64_t batch, int64_t ild, int64_t ibs,
                            float *out, int64_t old, int64_t obs, void *stream);
/* fp32 round-to-nearest of f64 (G.float(), solution.py:1327). */
int hif4x_f64_to_f32(const double *in, int64_t n, float *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* HIF4X_H_ */
