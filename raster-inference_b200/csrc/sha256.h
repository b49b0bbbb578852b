// SHA-256 (FIPS 180-4) for the det checkpoint commitments, which hash
// canonical little-endian bytes with domain tags
// (reference src/shared/numerics/transformer_kernels.rs:1395-1482).
#pragma once
#include <cstdint>
#include <cstring>
#include <string>

namespace rdet {

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
  static uint32_t ror(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void compress() {
    static const uint32_t k[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
        0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
        0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
        0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
        0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
        0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) w[i] = (uint32_t)blk[4 * i] << 24 | (uint32_t)blk[4 * i + 1] << 16 | (uint32_t)blk[4 * i + 2] << 8 | blk[4 * i + 3];
    for (int i = 16; i < 64; ++i)
      w[i] = w[i - 16] + (ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3)) + w[i - 7] +
             (ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10));
    uint32_t v[8];
    memcpy(v, st, sizeof(v));
    for (int i = 0; i < 64; ++i) {
      uint32_t t1 = v[7] + (ror(v[4], 6) ^ ror(v[4], 11) ^ ror(v[4], 25)) + ((v[4] & v[5]) ^ (~v[4] & v[6])) + k[i] + w[i];
      uint32_t t2 = (ror(v[0], 2) ^ ror(v[0], 13) ^ ror(v[0], 22)) + ((v[0] & v[1]) ^ (v[0] & v[2]) ^ (v[1] & v[2]));
      memmove(v + 1, v, 7 * sizeof(uint32_t));
      v[4] += t1;
      v[0] = t1 + t2;
    }
    for (int i = 0; i < 8; ++i) st[i] += v[i];
  }
  void put(const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    nbytes += n;
    while (n) {
      size_t c = 64 - fill < n ? 64 - fill : n;
      memcpy(blk + fill, b, c);
      fill += (int)c;
      b += c;
      n -= c;
      if (fill == 64) { compress(); fill = 0; }
    }
  }
  void put_u64(uint64_t x) {
    uint8_t b[8];
    for (int i = 0; i < 8; ++i) b[i] = (uint8_t)(x >> (8 * i));
    put(b, 8);
  }
  std::string hex() {
    uint64_t bits = nbytes * 8;
    uint8_t one = 0x80, zero = 0;
    put(&one, 1);
    while (fill != 56) put(&zero, 1);
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
