// gemm_tc.cu -- fp32-faithful GEMM on the sm_100a tensor cores (tcgen05).
//
//   C = alpha * op(A) op(B) + beta * C,  fp32 in / fp32 out, row-major.
//
// Each fp32 operand x is split once, in a pass over global memory, into
// x_hi = x with the low 13 mantissa bits cleared (an exact TF32 value) and
// x_lo = x - x_hi (exact in fp32), written K-contiguous whatever the
// operand's storage order; the product is accumulated as hi*hi + hi*lo +
// lo*hi by tcgen05.mma kind::tf32 into fp32 accumulators in tensor memory,
// which keeps ~21 significant bits per product (the dropped lo*lo term is
// < 2^-20 of it).  Splitting outside the GEMM keeps shared memory for the
// TMA writes and the tensor core's operand reads alone: an in-kernel split
// made the conversion's loads/stores and the MMA operand reads compete for
// the shared-memory banks and capped the tensor pipe near 40 %.
//
// Persistent kernel, one CTA per SM (all but kTcFreeSms of them), 128 x 128
// or 128 x 256 output tiles (Tile<BN_>, chosen per call) visited in bands of
// GROUP tile-rows (column by column within a band) so that the CTAs running
// at one time share A and B panels in L2.  192 threads:
//   warp 0   TMA producer (one lane) + tensor-memory allocation (whole warp)
//   warp 1   MMA issuer (one lane): 4 K-substeps x 3 products per stage
//   warps 2-5 epilogue: tcgen05.ld of their TMEM lane quarter -> alpha/beta
//            -> global, on one of two accumulator buffers while the MMA
//            warp fills the other
// The epilogue writes C through the TMA when beta is 0 or 1 and C allows a
// tensor map: each warp stages 32 x 32 boxes of its rows in shared memory
// (128-byte swizzle, so the row-per-lane writes are conflict-free) and one
// lane issues a bulk tensor store (beta 0) or a bulk tensor add-reduction
// into C (beta 1: C + v rounded to nearest, the value fmaf(1, C, v) gives).
// Lane-per-row stores straight from registers touch 32 rows per instruction
// and made products with short K (the rank-128 updates of GPTQ) bound by
// the epilogue; other betas and batched products keep that path.
// Every mbarrier wait is bounded: on expiry the kernel records
// HIF4X_TIMEOUT in a device status word and finishes without further
// waits; hif4x_device_status() reports it.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tc_gemm.cuh"

namespace hif4x {
namespace tc {

constexpr int BM = 128, BK = 32;
constexpr int TILE_A_BYTES = BM * BK * 4;          // 16 KiB per A half (hi or lo) and stage
// epilogue staging: per epilogue warp two 32 x 32 fp32 boxes (4 KiB each)
constexpr int EPI_BOX_BYTES = 32 * 32 * 4;
constexpr int EPI_BYTES = 4 * 2 * EPI_BOX_BYTES;
constexpr int THREADS = 192;
constexpr int GROUP = 8;                          // tile-rows per rasterisation band

// Output tiles are BM x BN_ with BN_ 128 or 256 (one tcgen05.mma of N = BN_).
// A 128 x 128 MMA reads 8 KiB of operands from shared memory per 128x128x8
// step while the TMA writes as much again, which holds the tensor pipe near
// 70 %; N = 256 reads 12 KiB per twice the work.  The wider tile has two
// stages of 96 KiB (A hi, A lo, B hi, B lo), the narrow one three of 64 KiB,
// so both take the same shared memory; TMEM holds two accumulator buffers of
// BN_ fp32 columns (512 of 512 columns for BN_ = 256).
template <int BN_>
struct Tile {
  static constexpr int BN = BN_;
  static constexpr int STAGES = BN_ == 256 ? 2 : 3;
  static constexpr int TILE_B = BN_ * BK * 4;
  static constexpr int STAGE_BYTES = 2 * TILE_A_BYTES + 2 * TILE_B;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /* align */ + 256 /* barriers */;
  static constexpr uint32_t TMEM_COLS = 2 * BN_;
};
static_assert(Tile<128>::SMEM_BYTES <= 232448 && Tile<256>::SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert(Tile<256>::TMEM_COLS <= 512, "tensor memory columns");
constexpr long long SPIN_LIMIT = 1ll << 22;
// SMs a persistent GEMM leaves free: 16 of 148 took down_proj's calibration
// (tensor-core Grams and Cholesky products beside one-CTA leaves and GPTQ
// blocks on side streams) from 106.3 to 104 ms; 8, 24 and 36 did less well
constexpr int kTcFreeSms = 16;

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
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t parity, long long limit) {
  for (long long i = 0; i < limit; i++)
    if (mbar_try_wait(bar, parity)) return true;
  atomicExch(&g_status, HIF4X_TIMEOUT);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  return mbar_wait_limit(bar, parity, SPIN_LIMIT);
}

// The failure path of the bounded wait, run on its own: one thread waits on an
// mbarrier that nothing arrives on (no copy or MMA is ever in flight here), so
// the wait runs out after `limit` polls and records HIF4X_TIMEOUT.
__global__ void wait_selftest_kernel(long long limit, int *done) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const bool ok = mbar_wait_limit(&bar, 0, limit);
  *done = ok ? 1 : 2;
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

// Instruction descriptor: D fp32, A/B tf32, M = 128, N = BN_, majors.
template <int BN_>
__host__ __device__ constexpr uint32_t instr_desc(int a_mn_major, int b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(BN_ >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
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

// K-major operand descriptor of K-substep j (8 K-elements) of a 128 x 32
// tile: rows of 128 B (32 K values), 8-row swizzle groups 1 KiB apart; a
// substep moves 32 B along the row.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int j) {
  return smem_desc(base + 32u * j, 16u, 1024u, 2u);
}

struct TcArgs {
  int64_t M, N, K;
  float alpha, beta;
  float *C;
  int64_t ldc;
  int a_lo, b_lo;   // row of the lo half in each split operand (hi rows come first)
  int tm, tn;       // tile rows / columns of one product
  int lower;        // 1: only tiles reaching the diagonal or below it (square C)
  int vec;          // 1: C rows take 16-byte stores
  int64_t ntiles;   // batch * tiles_per
  int64_t tiles_per;
  int a_bstride, b_bstride;   // split-operand rows between products (2M, 2N)
  int b_div;                  // product b reads B's product b / b_div
  int64_t c_bstride;          // C elements between products
  int tma_c;                  // 1: epilogue through the C tensor map (batch 1, beta 0 or 1)
  int kmode;                  // triangular operand: K-steps a tile may skip (tile_krange)
  const unsigned *lo_nz;      // bit 0 / 1: A's / B's lo half has a nonzero (null: assume both)
};

// K-steps [kb, ke) that can be nonzero for output tile (ti, tj) when one
// operand is triangular (its other entries are zeros in memory, so skipping
// them only saves work):
//   kmode 1: B(n, k) = 0 for k > n  ->  k < (tj + 1) * BN_
//   kmode 2: B(n, k) = 0 for k < n  ->  k >= tj * BN_
//   kmode 3: A(m, k) = 0 for k > m  ->  k < (ti + 1) * BM
// At least one step is always kept, so every accumulator is written.
template <int BN_>
__device__ __forceinline__ void tile_krange(const TcArgs &a, int ti, int tj, int nk, int &kb, int &ke) {
  kb = 0;
  ke = nk;
  if (a.kmode == 1) ke = min(nk, (tj + 1) * (BN_ / BK));
  else if (a.kmode == 2) kb = min(nk - 1, tj * (BN_ / BK));
  else if (a.kmode == 3) ke = min(nk, (ti + 1) * (BM / BK));
}

// Tile t of the visiting order -> (tile row, tile column).  Bands of GROUP
// tile-rows; inside a band, column by column.  With `lower` (M == N) only the
// tiles that reach the diagonal or lie below it exist: with R = BN_ / BM
// (1 or 2) row ti has columns 0 .. ti / R, and column p starts at row R p.
// In band b (rows [r0, r0 + g), r0 = bG) the columns p <= r0 / R have all g
// rows, the later ones r0 + g - R p rows.  A tile that crosses the diagonal is
// computed whole (its entries above the diagonal are written too).
template <int BN_>
__device__ __forceinline__ void tile_coords(const TcArgs &a, int64_t t, int &ti, int &tj) {
  if (!a.lower) {
    const int64_t per_band = (int64_t)GROUP * a.tn;
    const int band = (int)(t / per_band);
    const int64_t r = t - band * per_band;
    const int g = min(GROUP, a.tm - band * GROUP);
    tj = (int)(r / g);
    ti = band * GROUP + (int)(r % g);
    return;
  }
  constexpr int R = BN_ / BM;
  int band = 0;
  int64_t start = 0;
  for (;;) {
    const int r0 = band * GROUP, g = min(GROUP, a.tm - r0);
    const int p0 = r0 / R + 1, pmax = (r0 + g - 1) / R;   // full columns 0 .. p0-1
    int64_t size = (int64_t)p0 * g;
    for (int p = p0; p <= pmax; p++) size += r0 + g - R * p;
    if (t < start + size) break;
    start += size;
    band++;
  }
  const int r0 = band * GROUP, g = min(GROUP, a.tm - r0);
  const int p0 = r0 / R + 1;
  int64_t u = t - start;
  if (u < (int64_t)p0 * g) {
    tj = (int)(u / g);
    ti = r0 + (int)(u % g);
    return;
  }
  u -= (int64_t)p0 * g;
  int p = p0;
  while (u >= r0 + g - R * p) {
    u -= r0 + g - R * p;
    p++;
  }
  tj = p;
  ti = R * p + (int)u;
}

// Number of tiles of one product in the order above.
template <int BN_>
static int64_t tiles_of(int tm, int tn, int lower) {
  if (!lower) return (int64_t)tm * tn;
  constexpr int R = BN_ / BM;
  int64_t n = 0;
  for (int ti = 0; ti < tm; ti++) n += ti / R + 1;
  return n;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory source of all but the newest bulk group has been read
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int BN_>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA,
                                                             const __grid_constant__ CUtensorMap mapB,
                                                             const __grid_constant__ CUtensorMap mapC,
                                                             const TcArgs args) {
  using Cfg = Tile<BN_>;
  constexpr int BN = BN_, STAGES = Cfg::STAGES, STAGE_BYTES = Cfg::STAGE_BYTES, TILE_B = Cfg::TILE_B;
  constexpr uint32_t TMEM_COLS = Cfg::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *epi = smem + STAGES * STAGE_BYTES;   // EPI_BYTES of staging, 1 KiB aligned
  uint64_t *full = reinterpret_cast<uint64_t *>(epi + EPI_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;   // [2] accumulator buffer complete
  uint64_t *tempty = tfull + 2;       // [2] accumulator buffer drained by the epilogue
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)((args.K + BK - 1) / BK);
  // An operand whose every value is exact in TF32 (HiF4 values, bf16 inputs)
  // has an all-zero lo half: its lo tiles are neither loaded nor multiplied,
  // which leaves the sum unchanged (those products are exact zeros).  The
  // split pass recorded which halves are nonzero; producer and MMA warp read
  // the same word, so they agree on the stage layout.
  const unsigned lz = args.lo_nz != nullptr ? *args.lo_nz : 3u;
  const bool a_lo_on = (lz & 1u) != 0u, b_lo_on = (lz & 2u) != 0u;
  const uint32_t stage_tx =
      (uint32_t)TILE_A_BYTES * (a_lo_on ? 2u : 1u) + (uint32_t)TILE_B * (b_lo_on ? 2u : 1u);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
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
    // ---------------- TMA producer: hi and lo tiles of A and B per stage
    if (lane == 0) {
      int64_t g = 0;   // stage fills issued so far (a failed wait leaves g unissued)
      for (int64_t t = blockIdx.x; t < args.ntiles && ok; t += gridDim.x) {
        const int64_t b = t / args.tiles_per;
        int ti, tj;
        tile_coords<BN>(args, t - b * args.tiles_per, ti, tj);
        const int m0 = (int)b * args.a_bstride + ti * BM, n0 = (int)(b / args.b_div) * args.b_bstride + tj * BN;
        int kb, ke;
        tile_krange<BN>(args, ti, tj, nk, kb, ke);
        for (int kt = kb; kt < ke; kt++, g++) {
          const int s = (int)(g % STAGES);
          if (g >= STAGES) ok = mbar_wait(&empty[s], (uint32_t)(((g / STAGES) - 1) & 1));
          if (!ok) break;
          uint8_t *st = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], stage_tx);
          // stage layout: A hi, A lo (TILE_A_BYTES each), B hi, B lo (TILE_B each)
          tma_load_2d(&mapA, st, &full[s], kt * BK, m0);
          if (a_lo_on) tma_load_2d(&mapA, st + TILE_A_BYTES, &full[s], kt * BK, args.a_lo + m0);
          tma_load_2d(&mapB, st + 2 * TILE_A_BYTES, &full[s], kt * BK, n0);
          if (b_lo_on) tma_load_2d(&mapB, st + 2 * TILE_A_BYTES + TILE_B, &full[s], kt * BK, args.b_lo + n0);
        }
      }
      // drain: every issued copy has landed before the CTA may exit (the
      // last fill of stage s is the largest g' < g with g' % STAGES == s)
#pragma unroll
      for (int s = 0; s < STAGES; s++)
        if (g > s) mbar_wait(&full[s], (uint32_t)(((s + STAGES * ((g - 1 - s) / STAGES)) / STAGES) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc<BN>(0, 0);
      int64_t g = 0;
      int lt = 0;
      for (int64_t t = blockIdx.x; t < args.ntiles && ok; t += gridDim.x, lt++) {
        const int buf = lt & 1, use = lt >> 1;
        if (use > 0) ok = mbar_wait(&tempty[buf], (uint32_t)((use - 1) & 1));
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        int kb = 0, ke = nk;
        if (args.kmode != 0) {
          const int64_t b = t / args.tiles_per;
          int ti, tj;
          tile_coords<BN>(args, t - b * args.tiles_per, ti, tj);
          tile_krange<BN>(args, ti, tj, nk, kb, ke);
        }
        for (int kt = kb; kt < ke; kt++, g++) {
          const int s = (int)(g % STAGES);
          ok = mbar_wait(&full[s], (uint32_t)((g / STAGES) & 1));
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;");
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t a_hi = base, a_lo = base + TILE_A_BYTES;
          const uint32_t b_hi = base + 2 * TILE_A_BYTES, b_lo = base + 2 * TILE_A_BYTES + TILE_B;
#pragma unroll
          for (int j = 0; j < BK / 8; j++) {
            const uint64_t dah = kmajor_desc(a_hi, j), dal = kmajor_desc(a_lo, j);
            const uint64_t dbh = kmajor_desc(b_hi, j), dbl = kmajor_desc(b_lo, j);
            mma_tf32(d, dah, dbh, idesc, (kt > kb || j > 0) ? 1u : 0u);
            if (b_lo_on) mma_tf32(d, dah, dbl, idesc, 1u);
            if (a_lo_on) mma_tf32(d, dal, dbh, idesc, 1u);
          }
          mma_commit(&empty[s]);   // stage s free once these MMAs have read it
        }
        if (!ok) break;
        mma_commit(&tfull[buf]);   // accumulator buffer complete
      }
      // every issued MMA has finished before tensor memory is released
      mma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else {
    // ---------------- epilogue (threads 64..191): TMEM lane quarter (warp % 4) -> rows
    const int quarter = warp & 3;
    uint8_t *stg = epi + quarter * 2 * EPI_BOX_BYTES;   // this warp's two staging boxes
    int boxes = 0;                                      // boxes this warp has handed to the TMA
    int lt = 0;
    for (int64_t t = blockIdx.x; t < args.ntiles; t += gridDim.x, lt++) {
      const int buf = lt & 1, use = lt >> 1;
      ok = mbar_wait(&tfull[buf], (uint32_t)(use & 1));
      ok = __all_sync(0xffffffffu, ok);   // tcgen05.ld below is warp-collective
      if (!ok) break;
      asm volatile("tcgen05.fence::after_thread_sync;");
      const int64_t b = t / args.tiles_per;
      int ti, tj;
      tile_coords<BN>(args, t - b * args.tiles_per, ti, tj);
      const int64_t row = (int64_t)ti * BM + quarter * 32 + lane;
      // 128 accumulator columns at a time (BN / 128 halves); the buffer goes
      // back to the MMA warp once the last of them is in registers
#pragma unroll 1
      for (int h = 0; h < BN / 128; h++) {
      const int64_t n0 = (int64_t)tj * BN + h * 128;
      uint32_t r[128];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN + h * 128 + c * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(r[c * 32 + 0]), "=r"(r[c * 32 + 1]), "=r"(r[c * 32 + 2]), "=r"(r[c * 32 + 3]),
              "=r"(r[c * 32 + 4]), "=r"(r[c * 32 + 5]), "=r"(r[c * 32 + 6]), "=r"(r[c * 32 + 7]),
              "=r"(r[c * 32 + 8]), "=r"(r[c * 32 + 9]), "=r"(r[c * 32 + 10]), "=r"(r[c * 32 + 11]),
              "=r"(r[c * 32 + 12]), "=r"(r[c * 32 + 13]), "=r"(r[c * 32 + 14]), "=r"(r[c * 32 + 15]),
              "=r"(r[c * 32 + 16]), "=r"(r[c * 32 + 17]), "=r"(r[c * 32 + 18]), "=r"(r[c * 32 + 19]),
              "=r"(r[c * 32 + 20]), "=r"(r[c * 32 + 21]), "=r"(r[c * 32 + 22]), "=r"(r[c * 32 + 23]),
              "=r"(r[c * 32 + 24]), "=r"(r[c * 32 + 25]), "=r"(r[c * 32 + 26]), "=r"(r[c * 32 + 27]),
              "=r"(r[c * 32 + 28]), "=r"(r[c * 32 + 29]), "=r"(r[c * 32 + 30]), "=r"(r[c * 32 + 31])
            : "r"(taddr));
      }
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (h == BN / 128 - 1) {
        // the buffer's values are in registers: hand it back to the MMA warp
        asm volatile("tcgen05.fence::before_thread_sync;");
        mbar_arrive(&tempty[buf]);
      }
      if (args.tma_c) {
        // rows >= M and columns >= N of a box lie outside the tensor map: the copy skips them
        const float alpha = args.alpha;
        const int y = ti * BM + quarter * 32;
#pragma unroll
        for (int c = 0; c < 4; c++, boxes++) {
          uint8_t *box = stg + (boxes & 1) * EPI_BOX_BYTES;
          if (boxes >= 2) {   // the box's previous copy has finished reading it
            if (lane == 0) bulk_wait_read_1();
            __syncwarp();
          }
          // row `lane` of the box is 128 bytes; its 16-byte chunk q sits at chunk q ^ (lane & 7)
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const float4 v = make_float4(alpha * __uint_as_float(r[c * 32 + 4 * q + 0]),
                                         alpha * __uint_as_float(r[c * 32 + 4 * q + 1]),
                                         alpha * __uint_as_float(r[c * 32 + 4 * q + 2]),
                                         alpha * __uint_as_float(r[c * 32 + 4 * q + 3]));
            *reinterpret_cast<float4 *>(box + lane * 128 + ((q ^ (lane & 7)) << 4)) = v;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            if (args.beta == 0.0f) tma_store_2d(&mapC, box, (int)n0 + c * 32, y);
            else tma_reduce_add_2d(&mapC, box, (int)n0 + c * 32, y);
            bulk_commit();
          }
        }
      } else if (row < args.M) {
        float *crow = args.C + b * args.c_bstride + row * args.ldc;
        const float alpha = args.alpha, beta = args.beta;
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int64_t col0 = n0 + c * 32;
          if (args.vec && col0 + 32 <= args.N) {
            float4 *dst = reinterpret_cast<float4 *>(crow + col0);
#pragma unroll
            for (int q = 0; q < 8; q++) {
              float4 v = make_float4(alpha * __uint_as_float(r[c * 32 + 4 * q + 0]),
                                     alpha * __uint_as_float(r[c * 32 + 4 * q + 1]),
                                     alpha * __uint_as_float(r[c * 32 + 4 * q + 2]),
                                     alpha * __uint_as_float(r[c * 32 + 4 * q + 3]));
              if (beta != 0.0f) {
                const float4 o = dst[q];
                v.x = fmaf(beta, o.x, v.x);
                v.y = fmaf(beta, o.y, v.y);
                v.z = fmaf(beta, o.z, v.z);
                v.w = fmaf(beta, o.w, v.w);
              }
              dst[q] = v;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; j++) {
              const int64_t col = col0 + j;
              if (col < args.N) {
                const float v = alpha * __uint_as_float(r[c * 32 + j]);
                crow[col] = beta == 0.0f ? v : fmaf(beta, crow[col], v);
              }
            }
          }
        }
      }
      }   // halves
    }
    // every C box written before the CTA ends
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// Split an operand into TF32 hi / lo halves, K-contiguous:
//   dst[r * kp + k] = hi(x(r, k)),  dst[(R + r) * kp + k] = lo(x(r, k))
// where x(r, k) = src[r * ld + k] (k_contig) or src[k * ld + r].  32 x 32
// tiles; the transposing form goes through shared memory so that both the
// loads and the stores are coalesced.  blockIdx.z indexes a batch of
// operands src_bstride apart, written 2 R kp apart.
__global__ void split_tf32_kernel(const float *__restrict__ src, int64_t ld, int k_contig, int64_t R, int64_t K,
                                  int64_t src_bstride, float *__restrict__ dst, int64_t kp, unsigned *lo_nz,
                                  unsigned lo_bit) {
  __shared__ float tile[32][33];
  src += (int64_t)blockIdx.z * src_bstride;
  dst += (int64_t)blockIdx.z * 2 * R * kp;
  const int64_t k0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;   // 32 x 8
  if (!k_contig) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t k = k0 + ty + 8 * i, r = r0 + tx;
      tile[ty + 8 * i][tx] = (k < K && r < R) ? src[k * ld + r] : 0.0f;
    }
    __syncthreads();
  }
  bool lo_any = false;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t r = r0 + ty + 8 * i, k = k0 + tx;
    if (r < R && k < K) {
      const float x = k_contig ? src[r * ld + k] : tile[tx][ty + 8 * i];
      const float hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
      const float lo = __fsub_rn(x, hi);
      dst[r * kp + k] = hi;
      dst[(R + r) * kp + k] = lo;
      lo_any |= lo != 0.0f;
    }
  }
  // record (once per block) that this operand's lo half is not all zero
  if (lo_nz != nullptr && __syncthreads_or(lo_any) && tx == 0 && ty == 0) atomicOr(lo_nz, lo_bit);
}

__device__ __forceinline__ void split_store4(float *dst, int64_t R, int64_t r, int64_t kp, int64_t k, int64_t K,
                                             float4 x, bool &lo_any) {
  float4 hi, lo;
  hi.x = __uint_as_float(__float_as_uint(x.x) & 0xffffe000u);
  hi.y = __uint_as_float(__float_as_uint(x.y) & 0xffffe000u);
  hi.z = __uint_as_float(__float_as_uint(x.z) & 0xffffe000u);
  hi.w = __uint_as_float(__float_as_uint(x.w) & 0xffffe000u);
  lo.x = __fsub_rn(x.x, hi.x);
  lo.y = __fsub_rn(x.y, hi.y);
  lo.z = __fsub_rn(x.z, hi.z);
  lo.w = __fsub_rn(x.w, hi.w);
  if (k + 3 < K) {
    *reinterpret_cast<float4 *>(dst + r * kp + k) = hi;
    *reinterpret_cast<float4 *>(dst + (R + r) * kp + k) = lo;
    lo_any |= (lo.x != 0.0f) | (lo.y != 0.0f) | (lo.z != 0.0f) | (lo.w != 0.0f);
  } else {
    const float h4[4] = {hi.x, hi.y, hi.z, hi.w}, l4[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
    for (int j = 0; j < 4; j++)
      if (k + j < K) {
        dst[r * kp + k + j] = h4[j];
        dst[(R + r) * kp + k + j] = l4[j];
        lo_any |= l4[j] != 0.0f;
      }
  }
}

// The same split with 16-byte accesses, for sources whose rows start on 16
// bytes (ld a multiple of 4, aligned base) and destinations with kp a
// multiple of 4.  K-contiguous sources: one float4 of a row per thread, 32
// rows x 128 K per block.  Transposed sources: 64 (K) x 64 (R) tiles through
// shared memory, float4 loads along R and float4 stores along K.  Elements
// past R or K are neither read nor written.
template <bool KC>
__global__ void __launch_bounds__(256) split_tf32_vec_kernel(const float *__restrict__ src, int64_t ld, int64_t R,
                                                             int64_t K, int64_t src_bstride, float *__restrict__ dst,
                                                             int64_t kp, unsigned *lo_nz, unsigned lo_bit) {
  __shared__ float tile[KC ? 1 : 64][KC ? 1 : 65];
  src += (int64_t)blockIdx.z * src_bstride;
  dst += (int64_t)blockIdx.z * 2 * R * kp;
  const int tid = threadIdx.x;
  bool lo_any = false;
  if (KC) {
    const int64_t k = (int64_t)blockIdx.x * 128 + (tid & 31) * 4;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const int64_t r = (int64_t)blockIdx.y * 32 + p * 8 + (tid >> 5);
      if (r >= R || k >= K) continue;
      const float *sp = src + r * ld + k;
      float4 x;
      if (k + 3 < K) {
        x = *reinterpret_cast<const float4 *>(sp);
      } else {
        x.x = sp[0];
        x.y = k + 1 < K ? sp[1] : 0.0f;
        x.z = k + 2 < K ? sp[2] : 0.0f;
        x.w = 0.0f;
      }
      split_store4(dst, R, r, kp, k, K, x, lo_any);
    }
  } else {
    const int64_t k0 = (int64_t)blockIdx.x * 64, r0 = (int64_t)blockIdx.y * 64;
    {
      const int rl = (tid & 15) * 4, kl = tid >> 4;   // 16 float4 along R, 16 K rows per pass
      const int64_t r = r0 + rl;
#pragma unroll
      for (int p = 0; p < 4; p++) {
        const int kk = kl + 16 * p;
        const int64_t k = k0 + kk;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k < K && r < R) {
          const float *sp = src + k * ld + r;
          if (r + 3 < R) {
            x = *reinterpret_cast<const float4 *>(sp);
          } else {
            x.x = sp[0];
            x.y = r + 1 < R ? sp[1] : 0.0f;
            x.z = r + 2 < R ? sp[2] : 0.0f;
          }
        }
        tile[kk][rl + 0] = x.x;
        tile[kk][rl + 1] = x.y;
        tile[kk][rl + 2] = x.z;
        tile[kk][rl + 3] = x.w;
      }
    }
    __syncthreads();
    const int kl = (tid & 15) * 4, rl = tid >> 4;   // 16 float4 along K, 16 rows per pass
    const int64_t k = k0 + kl;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const int rr = rl + 16 * p;
      const int64_t r = r0 + rr;
      if (r >= R || k >= K) continue;
      const float4 x = make_float4(tile[kl][rr], tile[kl + 1][rr], tile[kl + 2][rr], tile[kl + 3][rr]);
      split_store4(dst, R, r, kp, k, K, x, lo_any);
    }
  }
  if (lo_nz != nullptr && __syncthreads_or(lo_any) && tid == 0) atomicOr(lo_nz, lo_bit);
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

// 2-D fp32 tensor map over a split operand: `inner` (K) x `outer` (2R) floats,
// row stride ld floats, 32 x box_rows boxes, 128-byte swizzle; K beyond
// `inner` reads as zero.
static bool make_map(CUtensorMap *map, const float *base, int64_t inner, int64_t outer, int64_t ld,
                     int box_rows = BM) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D fp32 tensor map over C (N columns x M rows, row stride ldc floats),
// 32 x 32 boxes, 128-byte swizzle: the epilogue's bulk stores and reductions.
static bool make_map_c(CUtensorMap *map, float *C, int64_t N, int64_t M, int64_t ldc) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)ldc * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kMaxDevices = 64;

// Per device: SM count, and the stream-ordered pool the split operands come
// from set to keep its memory between calls (the split buffers are
// allocated and freed around every product).
static int device_sms(int dev) {
  static int sms[kMaxDevices];
  static std::once_flag once[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return 0;
  std::call_once(once[dev], [dev] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 0;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    sms[dev] = n;
  });
  return sms[dev];
}

int split_operand(const float *src, int64_t ld, int k_contig, int64_t R, int64_t K, int64_t src_bstride,
                  int batch, float *dst, int64_t kp, cudaStream_t s, unsigned *lo_nz, unsigned lo_bit) {
  if (batch < 1 || batch > 65535) return HIF4X_ERR_UNSUPPORTED;
  const bool vec = (ld & 3) == 0 && (src_bstride & 3) == 0 && (kp & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  if (vec && k_contig && (R + 31) / 32 <= 65535) {
    dim3 grid((unsigned)((K + 127) / 128), (unsigned)((R + 31) / 32), (unsigned)batch);
    split_tf32_vec_kernel<true><<<grid, 256, 0, s>>>(src, ld, R, K, src_bstride, dst, kp, lo_nz, lo_bit);
    return HIF4X_OK;
  }
  if (vec && !k_contig && (R + 63) / 64 <= 65535) {
    dim3 grid((unsigned)((K + 63) / 64), (unsigned)((R + 63) / 64), (unsigned)batch);
    split_tf32_vec_kernel<false><<<grid, 256, 0, s>>>(src, ld, R, K, src_bstride, dst, kp, lo_nz, lo_bit);
    return HIF4X_OK;
  }
  const int64_t gy = (R + 31) / 32;
  if (gy > 65535) return HIF4X_ERR_UNSUPPORTED;
  dim3 grid((unsigned)((K + 31) / 32), (unsigned)gy, (unsigned)batch);
  split_tf32_kernel<<<grid, dim3(32, 8), 0, s>>>(src, ld, k_contig, R, K, src_bstride, dst, kp, lo_nz, lo_bit);
  return HIF4X_OK;
}

int gemm_split(const float *As, int a_products, const float *Bs, int b_products, int64_t M, int64_t N, int64_t K,
               int64_t kp, float alpha, float beta, float *C, int64_t ldc, int64_t c_bstride, int batch, int b_div,
               int lower, int kmode, cudaStream_t s, const unsigned *lo_nz) {
  if (M <= 0 || N <= 0 || K <= 0 || batch < 1 || b_div < 1 || (batch - 1) / b_div >= b_products ||
      batch > a_products)
    return HIF4X_ERR_ARG;
  if (2 * M * a_products > INT32_MAX || 2 * N * b_products > INT32_MAX) return HIF4X_ERR_UNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HIF4X_ERR_LAUNCH;
  const int sms = device_sms(dev);
  if (sms <= 0) return HIF4X_ERR_LAUNCH;
  const int lower_ok = (lower && M == N) ? 1 : 0;
  const int tm = (int)((M + BM - 1) / BM);
  // 128 x 256 tiles for long products that still fill two waves of CTAs with
  // them; the 128 x 128 tiles otherwise (short K is bound by C's traffic, and
  // small products need the CTA count)
  const int64_t cap = sms > 2 * kTcFreeSms ? sms - kTcFreeSms : sms;
  const bool wide = K >= 512 && tiles_of<256>(tm, (int)((N + 255) / 256), lower_ok) * batch >= 2 * cap;
  const int bn = wide ? 256 : 128;
  CUtensorMap ma, mb;
  if (!make_map(&ma, As, K, 2 * M * a_products, kp) || !make_map(&mb, Bs, K, 2 * N * b_products, kp, bn))
    return HIF4X_ERR_UNSUPPORTED;
  TcArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.alpha = alpha;
  args.beta = beta;
  args.C = C;
  args.ldc = ldc;
  args.a_lo = (int)M;
  args.b_lo = (int)N;
  args.tm = tm;
  args.tn = (int)((N + bn - 1) / bn);
  args.lower = lower_ok;
  args.vec = ((ldc & 3) == 0 && (c_bstride & 3) == 0 && (reinterpret_cast<uintptr_t>(C) & 15u) == 0) ? 1 : 0;
  args.tiles_per = wide ? tiles_of<256>(args.tm, args.tn, args.lower) : tiles_of<128>(args.tm, args.tn, args.lower);
  args.ntiles = args.tiles_per * batch;
  args.a_bstride = (int)(2 * M);
  args.b_bstride = (int)(2 * N);
  args.b_div = b_div;
  args.c_bstride = c_bstride;
  args.kmode = (kmode >= 0 && kmode <= 3) ? kmode : 0;
  args.lo_nz = lo_nz;
  CUtensorMap mc{};
  // N a multiple of 4: a bulk store past the tensor map's last column was seen
  // to write up to the next 16-byte boundary, so C's row ends must fall on one
  args.tma_c = (batch == 1 && args.vec && (N & 3) == 0 && (beta == 0.0f || beta == 1.0f) && M <= INT32_MAX &&
                N <= INT32_MAX && make_map_c(&mc, C, N, M, ldc))
                   ? 1
                   : 0;
  // the shared-memory opt-in is a property of the kernel in each device's context: once per device
  static std::once_flag attr_once[kMaxDevices];
  static bool attr_ok[kMaxDevices];
  if (dev >= kMaxDevices) return HIF4X_ERR_UNSUPPORTED;
  std::call_once(attr_once[dev], [dev] {
    attr_ok[dev] = cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Tile<128>::SMEM_BYTES) == cudaSuccess &&
                   cudaFuncSetAttribute(gemm_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Tile<256>::SMEM_BYTES) == cudaSuccess;
  });
  if (!attr_ok[dev]) return HIF4X_ERR_LAUNCH;
  // leave kTcFreeSms SMs to the latency-bound kernels of other streams (the
  // Cholesky leaves and GPTQ column blocks of the same or another
  // calibration): a persistent grid on every SM holds them off until it ends
  const int64_t grid = std::min<int64_t>(args.ntiles, cap);
  if (wide)
    gemm_tc_kernel<256><<<(unsigned)grid, THREADS, Tile<256>::SMEM_BYTES, s>>>(ma, mb, mc, args);
  else
    gemm_tc_kernel<128><<<(unsigned)grid, THREADS, Tile<128>::SMEM_BYTES, s>>>(ma, mb, mc, args);
  return cudaGetLastError() == cudaSuccess ? HIF4X_OK : HIF4X_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace hif4x

using namespace hif4x;

int hif4x_gemm_tc_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                     const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int lower, int kmode,
                     void *stream);

extern "C" int hif4x_gemm_tc(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
                             int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc,
                             void *stream) {
  return hif4x_gemm_tc_ex(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, 0, 0, stream);
}

// Same, optionally restricted to output tiles on or below the diagonal
// (lower != 0 and M == N; a diagonal tile is written whole) and to the
// K-steps a triangular operand leaves nonzero (kmode, see tile_krange).  The split
// operands live in a stream-ordered allocation of 2 * kp * (M + N) floats
// (2 * kp * M when A and B are the same operand, as in X^T X or L L^T).
// Returns HIF4X_ERR_UNSUPPORTED when a tensor map cannot be built, so the
// caller can take the SIMT kernel instead.
int hif4x_gemm_tc_ex(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                     const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int lower, int kmode,
                     void *stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) return HIF4X_ERR_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t kp = (K + 3) / 4 * 4;   // 16-byte row pitch for the tensor maps
  // operand (r, k) is K-contiguous in memory for A when ta == 0 and for B when tb == 1
  const int a_kc = ta ? 0 : 1, b_kc = tb ? 1 : 0;
  const bool same = A == B && lda == ldb && a_kc == b_kc && M == N;
  const int64_t a_floats = 2 * kp * M, b_floats = same ? 0 : 2 * kp * N;
  float *ws = nullptr;
  // split operands, then one word: which operands have a nonzero lo half
  if (cudaMallocAsync(reinterpret_cast<void **>(&ws), (size_t)(a_floats + b_floats + 4) * sizeof(float), s) !=
      cudaSuccess) {
    cudaGetLastError();   // not sticky: clear it so later launch checks do not report it
    return HIF4X_ERR_NOMEM;
  }
  float *As = ws, *Bs = same ? ws : ws + a_floats;
  unsigned *lo_nz = reinterpret_cast<unsigned *>(ws + a_floats + b_floats);
  if (cudaMemsetAsync(lo_nz, 0, sizeof(unsigned), s) != cudaSuccess) {
    cudaFreeAsync(ws, s);
    return HIF4X_ERR_LAUNCH;
  }
  int st = tc::split_operand(A, lda, a_kc, M, K, 0, 1, As, kp, s, lo_nz, same ? 3u : 1u);
  if (st == HIF4X_OK && !same) st = tc::split_operand(B, ldb, b_kc, N, K, 0, 1, Bs, kp, s, lo_nz, 2u);
  if (st == HIF4X_OK)
    st = tc::gemm_split(As, 1, Bs, 1, M, N, K, kp, alpha, beta, C, ldc, 0, 1, 1, lower, kmode, s, lo_nz);
  cudaFreeAsync(ws, s);
  return st;
}

// Runs wait_selftest_kernel with a spin limit of `spins` polls (1 .. 2^22)
// and returns once it has finished; *done_dev is set to 2 when the wait ran
// out (it always does: nothing arrives), and the device status then reads
// HIF4X_TIMEOUT.
extern "C" int hif4x_wait_selftest(long long spins, int *done_dev, void *stream) {
  if (spins < 1 || spins > tc::SPIN_LIMIT || !done_dev) return HIF4X_ERR_ARG;
  tc::wait_selftest_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(spins, done_dev);
  HIF4X_CHECK_LAUNCH();
  return cudaStreamSynchronize((cudaStream_t)stream) == cudaSuccess ? HIF4X_OK : HIF4X_ERR_LAUNCH;
}

// Synchronises the stream and reports (then clears) the sticky device status
// set by bounded waits that expired: HIF4X_OK or HIF4X_TIMEOUT.  The word is
// one per device, not per stream: a read from any stream clears it for all.
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
