// CRC-32 (IEEE 802.3, reflected polynomial 0xEDB88320, init and final xor
// 0xFFFFFFFF: the checksum zlib and the safetensors index use) computed in
// parallel: the buffer is cut into chunks whose CRCs the pool computes with a
// slicing-by-8 table walk, then the chunk CRCs are joined with
//   crc(A || B) = (x^(8|B|) * crc(A) mod P) xor crc(B),
// the multiplication done in GF(2)[x] modulo the CRC polynomial.
//
// Reference: ChecksumValidator (include/crypto/crypto_engine.hpp:134-161),
// a bytewise single-threaded CRC32.
#pragma once

#include <cstddef>
#include <cstdint>

namespace lkrt {

class WorkStealingPool;

uint32_t crc32_update(uint32_t crc, const void* data, size_t n);
uint32_t crc32_combine(uint32_t crc_a, uint32_t crc_b, uint64_t len_b);
uint32_t crc32_parallel(const void* data, size_t n, WorkStealingPool& pool, size_t chunk = 8u << 20);

}  // namespace lkrt
