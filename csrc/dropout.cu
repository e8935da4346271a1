// Inverted dropout with a counter-based mask: element i of a call with seed s
// is kept iff hash(s, i) >= p * 2^32 (hash = the splitmix64 finaliser of
// s xor i * 0x9E3779B97F4A7C15, high 32 bits), and kept values are scaled by
// 1 / (1 - p).  The mask is a pure function of (seed, index), so the backward
// regenerates it instead of storing it, and activation recomputation
// reproduces the forward exactly.  x and y may alias (in place).
//
// Reference: Dropout (include/nn/training_enhancements.hpp:215-242, an
// inverted Bernoulli mask drawn from a host RNG and stored).
#include "common.cuh"
#include "host_util.h"
#include "lk_api.h"

namespace lk {
namespace {

__device__ __forceinline__ uint32_t drop_hash(uint64_t seed, uint64_t i) {
  uint64_t z = seed ^ (i * 0x9E3779B97F4A7C15ull);
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (uint32_t)(z >> 32);
}

__global__ void dropout_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int64_t n8, uint64_t seed,
                               uint32_t thresh, float scale) {
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n8; v += (int64_t)gridDim.x * blockDim.x) {
    const uint4 a = reinterpret_cast<const uint4*>(x)[v];
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      const uint64_t i = (uint64_t)v * 8 + 2 * e;
      const float k0 = drop_hash(seed, i) >= thresh ? scale : 0.f;
      const float k1 = drop_hash(seed, i + 1) >= thresh ? scale : 0.f;
      o[e] = pack_bf16x2(f.x * k0, f.y * k1);
    }
    reinterpret_cast<uint4*>(y)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace lk

using namespace lk;

extern "C" int lk_dropout(const void* x, void* y, int64_t n, float p, uint64_t seed, cudaStream_t s) {
  LK_REQUIRE(n % 8 == 0, "dropout: element count must be a multiple of 8");
  LK_REQUIRE(p >= 0.f && p < 1.f, "dropout: p must be in [0, 1)");
  if (n == 0) return 0;
  const uint32_t thresh = (uint32_t)std::min(4294967295.0, (double)p * 4294967296.0);
  const int grid = (int)std::min<int64_t>((n / 8 + 255) / 256, 8 * num_sms());
  dropout_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, n / 8, seed, thresh,
                                      1.f / (1.f - p));
  return check_launch("dropout");
}
