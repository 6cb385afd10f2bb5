// gemm_tc.cu -- fp32-faithful GEMM on the sm_100a tensor cores (tcgen05).
//
//   C = alpha * op(A) op(B) + beta * C,  fp32 in / fp32 out, row-major.
//
// Each fp32 operand x is split in shared memory into x_hi = x with the low 13
// mantissa bits cleared (an exact TF32 value) and x_lo = x - x_hi (exact in
// fp32); the tile product is accumulated as hi*hi + hi*lo + lo*hi by
// tcgen05.mma kind::tf32 into fp32 accumulators in tensor memory, which keeps
// ~21 significant bits per product (the dropped lo*lo term is < 2^-20 of it).
//
// CTA tile 128 x 128, K step 32, 3-stage pipeline, 192 threads:
//   warp 0   TMA producer (one lane) + tensor-memory allocation (whole warp)
//   warp 1   MMA issuer (one lane): 4 K-substeps x 3 products per stage
//   warps 2-5 split fp32 tiles into hi/lo, then the epilogue (tcgen05.ld of
//            their TMEM lane quarter -> alpha/beta -> global)
// Operands are TMA-loaded with 128-byte swizzle either K-major (K contiguous:
// one 128 x 32 box) or MN-major (M/N contiguous: four 32 x 32 boxes), matching
// the UMMA shared-memory descriptors below.  Every mbarrier wait is bounded:
// on expiry the kernel records HIF4X_TIMEOUT in a device status word and
// finishes without further waits; hif4x_device_status() reports it.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace hif4x {
namespace tc {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int TILE_BYTES = BM * BK * 4;           // 16 KiB (A and B tiles are the same size)
constexpr int STAGE_BYTES = 4 * TILE_BYTES;        // A hi, A lo, B hi, B lo
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /* align */ + 256 /* barriers */;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 128;
constexpr long long SPIN_LIMIT = 1ll << 22;

__device__ int g_status;   // sticky device status: 0 or HIF4X_TIMEOUT

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait: false (and the device status set) if the phase never completes
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  for (long long i = 0; i < SPIN_LIMIT; i++)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(&g_status, HIF4X_TIMEOUT);
  return false;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap *map, void *dst, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// UMMA shared-memory descriptor (sm100 version bits).  layout 2 = 128-byte
// swizzle of 16-byte chunks (K-major tiles); layout 1 = 128-byte swizzle of
// 32-byte chunks, the only MN-major layout for 32-bit (tf32) operands.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1 << 46;   // version (sm100)
  d |= (uint64_t)layout << 61;
  return d;
}

// Instruction descriptor: D fp32, A/B tf32, M = 128, N = 128, majors.
__host__ __device__ constexpr uint32_t instr_desc(int a_mn_major, int b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

struct TcArgs {
  int64_t M, N, K;
  float alpha, beta;
  float *C;
  int64_t ldc;
  int a_mn, b_mn;   // operand majors: 1 = M/N contiguous in global (and smem)
  int lower;        // 1: only tiles touching the lower triangle (n0 <= m0 + BM - 1)
};

// operand tile loads for one stage (K-major: one 128x32 box; MN-major: four 32x32 boxes)
__device__ __forceinline__ void load_operand(const CUtensorMap *map, int mn_major, uint8_t *dst, uint64_t *bar,
                                             int mn0, int k0) {
  if (!mn_major) {
    tma_load_2d(map, dst, bar, k0, mn0);
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) tma_load_2d(map, dst + i * 4096, bar, mn0 + 32 * i, k0);
  }
}

// descriptor of K-substep j (8 K-elements) of an operand tile.
// K-major: rows of 128 B (32 K values), 8-row groups 1 KiB apart; a substep
// moves 32 B along the row.  MN-major: per 32-element MN atom (one 4 KiB TMA
// box, LBO apart) K-rows of 128 B, 4-row swizzle groups 512 B apart (SBO); a
// substep moves 8 K-rows = 1 KiB.
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int mn_major, int j) {
  if (!mn_major) return smem_desc(base + 32u * j, 16u, 1024u, 2u);
  return smem_desc(base + 1024u * j, 4096u, 512u, 1u);
}

__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA,
                                                             const __grid_constant__ CUtensorMap mapB,
                                                             const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *conv = full + STAGES;
  uint64_t *empty = conv + STAGES;
  uint64_t *accum = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nk = (int)((args.K + BK - 1) / BK);
  if (args.lower && n0 > m0 + BM - 1) return;   // tile strictly above the diagonal: nothing to do

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int issued_last[STAGES] = {-1, -1, -1};
      for (int kt = 0; kt < nk && ok; kt++) {
        const int s = kt % STAGES;
        if (kt >= STAGES) ok = mbar_wait(&empty[s], ((kt / STAGES) - 1) & 1);
        if (!ok) break;
        uint8_t *st = smem + s * STAGE_BYTES;
        mbar_expect_tx(&full[s], 2 * TILE_BYTES);
        load_operand(&mapA, args.a_mn, st, &full[s], m0, kt * BK);
        load_operand(&mapB, args.b_mn, st + 2 * TILE_BYTES, &full[s], n0, kt * BK);
        issued_last[s] = kt;
      }
      // drain: every issued copy has landed before the CTA may exit
      for (int s = 0; s < STAGES; s++)
        if (issued_last[s] >= 0) mbar_wait(&full[s], (issued_last[s] / STAGES) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc(args.a_mn, args.b_mn);
      for (int kt = 0; kt < nk && ok; kt++) {
        const int s = kt % STAGES;
        ok = mbar_wait(&conv[s], (kt / STAGES) & 1);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
        const uint32_t a_hi = base, a_lo = base + TILE_BYTES;
        const uint32_t b_hi = base + 2 * TILE_BYTES, b_lo = base + 3 * TILE_BYTES;
#pragma unroll
        for (int j = 0; j < BK / 8; j++) {
          const uint64_t dah = operand_desc(a_hi, args.a_mn, j), dal = operand_desc(a_lo, args.a_mn, j);
          const uint64_t dbh = operand_desc(b_hi, args.b_mn, j), dbl = operand_desc(b_lo, args.b_mn, j);
          mma_tf32(tmem, dah, dbh, idesc, (kt > 0 || j > 0) ? 1u : 0u);
          mma_tf32(tmem, dah, dbl, idesc, 1u);
          mma_tf32(tmem, dal, dbh, idesc, 1u);
        }
        mma_commit(&empty[s]);   // stage s free once these MMAs have read it
      }
      mma_commit(accum);         // accumulators complete
    }
  } else {
    // ---------------- split fp32 -> tf32 hi + lo (threads 64..191)
    const int t = threadIdx.x - 64;
    for (int kt = 0; kt < nk && ok; kt++) {
      const int s = kt % STAGES;
      ok = mbar_wait(&full[s], (kt / STAGES) & 1);
      if (!ok) break;
      uint8_t *st = smem + s * STAGE_BYTES;
#pragma unroll
      for (int op = 0; op < 2; op++) {
        float4 *hi = reinterpret_cast<float4 *>(st + op * 2 * TILE_BYTES);
        float4 *lo = reinterpret_cast<float4 *>(st + op * 2 * TILE_BYTES + TILE_BYTES);
#pragma unroll
        for (int i = 0; i < TILE_BYTES / 16 / 128; i++) {
          const int e = t + 128 * i;
          float4 v = hi[e];
          float4 h, l;
          h.x = __uint_as_float(__float_as_uint(v.x) & 0xffffe000u); l.x = __fsub_rn(v.x, h.x);
          h.y = __uint_as_float(__float_as_uint(v.y) & 0xffffe000u); l.y = __fsub_rn(v.y, h.y);
          h.z = __uint_as_float(__float_as_uint(v.z) & 0xffffe000u); l.z = __fsub_rn(v.z, h.z);
          h.w = __uint_as_float(__float_as_uint(v.w) & 0xffffe000u); l.w = __fsub_rn(v.w, h.w);
          hi[e] = h;
          lo[e] = l;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&conv[s]);
    }
    // ---------------- epilogue: TMEM lane quarter (warp % 4) -> rows
    ok = __all_sync(0xffffffffu, ok);
    if (ok) ok = mbar_wait(accum, 0);
    ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld below is warp-collective
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;");
      const int quarter = warp & 3;
      const int64_t row = (int64_t)m0 + quarter * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
              "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
              "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < args.M) {
          float *crow = args.C + row * args.ldc;
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int64_t col = (int64_t)n0 + c * 32 + j;
            if (col < args.N) {
              const float v = args.alpha * __uint_as_float(r[j]);
              crow[col] = args.beta == 0.0f ? v : fmaf(args.beta, crow[col], v);
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D fp32 tensor map: inner dim (contiguous) x outer dim, row stride ld floats.
static bool make_map(CUtensorMap *map, const float *base, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                     int box_outer, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace hif4x

using namespace hif4x;

// Tensor-core path of hif4x_gemm (batch 1).  Returns HIF4X_ERR_UNSUPPORTED
// when the operands do not meet the TMA rules (16-byte aligned bases,
// leading dimensions a multiple of 4 floats), so the caller can take the
// SIMT kernel instead.
int hif4x_gemm_tc_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                     const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int lower, void *stream);

extern "C" int hif4x_gemm_tc(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
                             int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc,
                             void *stream) {
  return hif4x_gemm_tc_ex(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, 0, stream);
}

// Same, optionally restricted to output tiles that touch the lower triangle.
int hif4x_gemm_tc_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                     const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int lower, void *stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) return HIF4X_ERR_ARG;
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(A) || !al16(B) || (lda & 3) || (ldb & 3)) return HIF4X_ERR_UNSUPPORTED;
  if ((M + tc::BM - 1) / tc::BM > 65535) return HIF4X_ERR_UNSUPPORTED;
  CUtensorMap ma, mb;
  // A: ta = 0 -> stored M x K (K contiguous, K-major); ta = 1 -> stored K x M (MN-major)
  const CUtensorMapSwizzle KSW = CU_TENSOR_MAP_SWIZZLE_128B, MNSW = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const bool okA = ta ? tc::make_map(&ma, A, M, K, lda, 32, 32, MNSW) : tc::make_map(&ma, A, K, M, lda, 32, 128, KSW);
  // B: tb = 1 -> stored N x K (K-major); tb = 0 -> stored K x N (MN-major)
  const bool okB = tb ? tc::make_map(&mb, B, K, N, ldb, 32, 128, KSW) : tc::make_map(&mb, B, N, K, ldb, 32, 32, MNSW);
  if (!okA || !okB) return HIF4X_ERR_UNSUPPORTED;
  tc::TcArgs args{M, N, K, alpha, beta, C, ldc, ta ? 1 : 0, tb ? 0 : 1, lower ? 1 : 0};
  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(tc::gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_BYTES);
  });
  dim3 grid((unsigned)((N + tc::BN - 1) / tc::BN), (unsigned)((M + tc::BM - 1) / tc::BM));
  tc::gemm_tc_kernel<<<grid, tc::THREADS, tc::SMEM_BYTES, (cudaStream_t)stream>>>(ma, mb, args);
  HIF4X_CHECK_LAUNCH();
  return HIF4X_OK;
}

// Synchronises the stream and reports (then clears) the sticky device status
// set by bounded waits that expired: HIF4X_OK or HIF4X_TIMEOUT.
extern "C" int hif4x_device_status(void *stream) {
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  int st = 0;
  if (cudaMemcpyFromSymbol(&st, tc::g_status, sizeof(int)) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  if (st != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(tc::g_status, &zero, sizeof(int));
  }
  return st;
}
