// host.cu -- host-side entry points (no device work).
#include <random>

#include "common.cuh"

// The reference draws its rotation signs with torch's CPU generator, which is
// the standard 32-bit MT19937 seeded with seed0 + b; torch.rand(float) keeps
// the low 24 bits of each draw, so rand < 0.5 exactly when bit 23 of the draw
// is clear (example/solution/solution.py:240-242, 1114-1115).
// Vector b takes ceil(len/64) words; bit e%64 of word e/64 is sign e.
extern "C" int hif4x_rot_signs(int64_t n_vec, int64_t len, uint32_t seed0, uint64_t *out_host) {
  if (n_vec < 0 || len < 0 || len > 4096 || (n_vec > 0 && out_host == nullptr)) return HIF4X_ERR_ARG;
  const int64_t words = (len + 63) / 64;
  for (int64_t b = 0; b < n_vec; b++) {
    std::mt19937 gen(static_cast<uint32_t>(seed0 + static_cast<uint32_t>(b)));
    for (int64_t w = 0; w < words; w++) out_host[b * words + w] = 0;
    for (int64_t e = 0; e < len; e++)
      if (gen() & (1u << 23)) out_host[b * words + e / 64] |= (1ull << (e % 64));
  }
  return HIF4X_OK;
}
