// SHA-256 (FIPS 180-4) for the det checkpoint commitments, which hash
// canonical little-endian bytes with domain tags
// (reference src/shared/numerics/transformer_kernels.rs:1395-1482).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <string>

namespace rdet {

// Compresses nblocks whole 64-byte blocks at p into st (csrc/sha256.cpp: the
// x86 SHA extensions when the CPU has them, else scalar).
void sha256_compress(uint32_t st[8], const uint8_t* p, size_t nblocks);
// 1 when sha256_compress runs on the SHA extensions, 0 for the scalar loop.
int sha256_impl();

struct Sha256 {
  uint32_t st[8];
  uint8_t blk[64];
  uint64_t nbytes = 0;
  int fill = 0;

  Sha256() {
    const uint32_t iv[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                            0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    memcpy(st, iv, sizeof(st));
  }
  void put(const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    nbytes += n;
    if (fill) {  // top up the partial block first
      size_t c = 64 - fill < n ? 64 - fill : n;
      memcpy(blk + fill, b, c);
      fill += (int)c;
      b += c;
      n -= c;
      if (fill < 64) return;
      sha256_compress(st, blk, 1);
      fill = 0;
    }
    if (n >= 64) {  // whole blocks straight from the caller's bytes
      sha256_compress(st, b, n / 64);
      b += n & ~(size_t)63;
      n &= 63;
    }
    memcpy(blk, b, n);
    fill = (int)n;
  }
  void put_u64(uint64_t x) {
    uint8_t b[8];
    for (int i = 0; i < 8; ++i) b[i] = (uint8_t)(x >> (8 * i));
    put(b, 8);
  }
  std::string hex() {
    uint64_t bits = nbytes * 8;
    uint8_t pad[72] = {0x80};
    const size_t npad = fill < 56 ? 56 - fill : 120 - fill;
    put(pad, npad);
    uint8_t lb[8];
    for (int i = 0; i < 8; ++i) lb[i] = (uint8_t)(bits >> (56 - 8 * i));
    put(lb, 8);
    static const char* hx = "0123456789abcdef";
    std::string s;
    for (int i = 0; i < 8; ++i)
      for (int j = 28; j >= 0; j -= 4) s += hx[(st[i] >> j) & 15];
    return s;
  }
};

}  // namespace rdet
