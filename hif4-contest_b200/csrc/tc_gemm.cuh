// tc_gemm.cuh -- the tensor-core GEMM on operands already split into TF32
// hi / lo halves (csrc/gemm_tc.cu), for kernels that chain products.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace hif4x {
namespace tc {

// Split `batch` operands (R x K each, src_bstride floats apart) into
// dst[b][2R][kp]: rows [0, R) the TF32 hi parts, [R, 2R) the lo parts,
// K-contiguous; x(r, k) = src[r * ld + k] (k_contig) or src[k * ld + r].
// With lo_nz, ORs lo_bit into *lo_nz when any lo part is nonzero (an
// operand exact in TF32 -- HiF4 values, bf16 values -- leaves it clear).
int split_operand(const float *src, int64_t ld, int k_contig, int64_t R, int64_t K, int64_t src_bstride,
                  int batch, float *dst, int64_t kp, cudaStream_t s, unsigned *lo_nz = nullptr,
                  unsigned lo_bit = 0);

// C_b = alpha * A_b B_{b / b_div}^T + beta * C_b for b < batch, with A_b the
// split operand b of As (M rows, a_products of them) and B_g the split
// operand g of Bs (N rows); C_b at C + b * c_bstride, leading dimension ldc.
// lower: only output tiles on or below the diagonal; kmode: skip the K-steps
// a triangular operand leaves zero (1: B(n,k)=0 for k>n, 2: B(n,k)=0 for
// k<n, 3: A(m,k)=0 for k>m; 0: none).  lo_nz (device word written by the
// splits, or null): bit 0 clear = A's lo half is all zero, bit 1 = B's; those
// tiles are then neither loaded nor multiplied.
int gemm_split(const float *As, int a_products, const float *Bs, int b_products, int64_t M, int64_t N, int64_t K,
               int64_t kp, float alpha, float beta, float *C, int64_t ldc, int64_t c_bstride, int batch, int b_div,
               int lower, int kmode, cudaStream_t s, const unsigned *lo_nz = nullptr);

}  // namespace tc
}  // namespace hif4x
