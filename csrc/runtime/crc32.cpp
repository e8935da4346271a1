#include "crc32.h"

#include <cstring>
#include <vector>

#include "thread_pool.h"

namespace lkrt {

namespace {

constexpr uint32_t kPoly = 0xEDB88320u;  // x^32 + x^26 + ... + 1, bit-reversed

struct Tables {
  uint32_t t[8][256];
  uint32_t x2k[64];  // x^(2^k) mod P, reflected
  Tables() {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int b = 0; b < 8; ++b) c = (c & 1) ? (c >> 1) ^ kPoly : c >> 1;
      t[0][i] = c;
    }
    for (int k = 1; k < 8; ++k)
      for (int i = 0; i < 256; ++i) t[k][i] = (t[k - 1][i] >> 8) ^ t[0][t[k - 1][i] & 0xff];
    x2k[0] = 0x40000000u;  // x^1 (bit 31 is x^0 in the reflected form)
    for (int k = 1; k < 64; ++k) x2k[k] = mulmod(x2k[k - 1], x2k[k - 1]);
  }
  // a(x) * b(x) mod P in the reflected representation: walk a's coefficients
  // from x^0 upward, adding the running b(x) * x^i for every set one
  static uint32_t mulmod(uint32_t a, uint32_t b) {
    uint32_t prod = 0;
    for (uint32_t m = 0x80000000u; m != 0; m >>= 1) {
      if (a & m) prod ^= b;
      b = (b & 1) ? (b >> 1) ^ kPoly : b >> 1;  // b *= x
    }
    return prod;
  }
};

const Tables& tables() {
  static const Tables tb;
  return tb;
}

}  // namespace

uint32_t crc32_update(uint32_t crc, const void* data, size_t n) {
  const Tables& tb = tables();
  const uint8_t* p = (const uint8_t*)data;
  uint32_t c = ~crc;
  while (n >= 8) {
    uint64_t w;
    std::memcpy(&w, p, 8);  // little-endian host
    const uint32_t lo = (uint32_t)w ^ c, hi = (uint32_t)(w >> 32);
    c = tb.t[7][lo & 0xff] ^ tb.t[6][(lo >> 8) & 0xff] ^ tb.t[5][(lo >> 16) & 0xff] ^ tb.t[4][lo >> 24] ^
        tb.t[3][hi & 0xff] ^ tb.t[2][(hi >> 8) & 0xff] ^ tb.t[1][(hi >> 16) & 0xff] ^ tb.t[0][hi >> 24];
    p += 8;
    n -= 8;
  }
  while (n--) c = tb.t[0][(c ^ *p++) & 0xff] ^ (c >> 8);
  return ~c;
}

uint32_t crc32_combine(uint32_t crc_a, uint32_t crc_b, uint64_t len_b) {
  const Tables& tb = tables();
  // x^(8 len_b) mod P by binary powering over the precomputed x^(2^k)
  uint32_t xp = 0x80000000u;  // x^0
  const uint64_t e = len_b;
  for (int k = 0; k < 61; ++k)
    if ((e >> k) & 1) xp = Tables::mulmod(tb.x2k[k + 3], xp);
  return Tables::mulmod(xp, crc_a) ^ crc_b;
}

uint32_t crc32_parallel(const void* data, size_t n, WorkStealingPool& pool, size_t chunk) {
  if (chunk == 0) chunk = 8u << 20;
  const size_t nchunks = (n + chunk - 1) / chunk;
  if (nchunks <= 1) return crc32_update(0, data, n);
  std::vector<uint32_t> part(nchunks);
  const uint8_t* p = (const uint8_t*)data;
  pool.parallel_for((int64_t)nchunks, 1, [&](int64_t c0, int64_t c1) {
    for (int64_t c = c0; c < c1; ++c) {
      const size_t off = (size_t)c * chunk;
      part[c] = crc32_update(0, p + off, std::min(chunk, n - off));
    }
  });
  uint32_t crc = part[0];
  for (size_t c = 1; c < nchunks; ++c) {
    const size_t len = std::min(chunk, n - c * chunk);
    crc = crc32_combine(crc, part[c], len);
  }
  return crc;
}

}  // namespace lkrt
