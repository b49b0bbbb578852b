// SHA-256 block compression for the det checkpoint commitments.
//
// Two implementations of the FIPS 180-4 compression function over whole
// 64-byte blocks: the x86 SHA extensions (SHA256RNDS2 / SHA256MSG1 /
// SHA256MSG2, following the round and message-schedule structure Intel
// published with the extensions in 2013) when the host CPU has them, else a
// portable scalar loop.  The choice is made once from CPUID; both produce the
// same state for every input (tests/test_sha256.py compares each against
// Python's hashlib on the same bytes).
#include "sha256.h"

#include <cstdlib>

#if defined(__x86_64__)
#include <cpuid.h>
#include <immintrin.h>
#endif

namespace rdet {

alignas(64) static const uint32_t kK[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

static inline uint32_t ror(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void compress_scalar(uint32_t st[8], const uint8_t* p, size_t nblocks) {
  for (; nblocks; --nblocks, p += 64) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i)
      w[i] = w[i - 16] + (ror(w[i - 15], 7) ^ ror(w[i - 15], 18) ^ (w[i - 15] >> 3)) + w[i - 7] +
             (ror(w[i - 2], 17) ^ ror(w[i - 2], 19) ^ (w[i - 2] >> 10));
    uint32_t a = st[0], b = st[1], c = st[2], d = st[3], e = st[4], f = st[5], g = st[6], h = st[7];
    for (int i = 0; i < 64; ++i) {
      uint32_t t1 = h + (ror(e, 6) ^ ror(e, 11) ^ ror(e, 25)) + ((e & f) ^ (~e & g)) + kK[i] + w[i];
      uint32_t t2 = (ror(a, 2) ^ ror(a, 13) ^ ror(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      h = g; g = f; f = e; e = d + t1;
      d = c; c = b; b = a; a = t1 + t2;
    }
    st[0] += a; st[1] += b; st[2] += c; st[3] += d;
    st[4] += e; st[5] += f; st[6] += g; st[7] += h;
  }
}

#if defined(__x86_64__)
// The extension keeps the eight working words as two vectors, (A,B,E,F) and
// (C,D,G,H), highest word first; SHA256RNDS2 runs two rounds from the low two
// words of its third operand (message word + round constant) and returns the
// new (A,B,E,F), the old one becoming (C,D,G,H).  Message words are big-endian
// in the block; W[t..t+3] for t >= 16 come from MSG1 (W[t-16] + s0(W[t-15]))
// plus W[t-7..t-4], finished by MSG2 (+ s1(W[t-2])).
__attribute__((target("sha,sse4.1,ssse3"))) static void compress_shani(uint32_t st[8], const uint8_t* p,
                                                                       size_t nblocks) {
  const __m128i bswap = _mm_set_epi64x(0x0c0d0e0f08090a0bLL, 0x0405060700010203LL);
  __m128i t = _mm_loadu_si128(reinterpret_cast<const __m128i*>(st));      // A B C D (word 0 first)
  __m128i s1 = _mm_loadu_si128(reinterpret_cast<const __m128i*>(st + 4));  // E F G H
  t = _mm_shuffle_epi32(t, 0xB1);                                          // B A D C
  s1 = _mm_shuffle_epi32(s1, 0x1B);                                        // H G F E
  __m128i s0 = _mm_alignr_epi8(t, s1, 8);                                  // F E B A  = (A,B,E,F)
  s1 = _mm_blend_epi16(s1, t, 0xF0);                                       // H G D C  = (C,D,G,H)
  for (; nblocks; --nblocks, p += 64) {
    const __m128i abef = s0, cdgh = s1;
    __m128i m[4];
    for (int i = 0; i < 4; ++i)
      m[i] = _mm_shuffle_epi8(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * i)), bswap);
#pragma GCC unroll 16
    for (int g = 0; g < 16; ++g) {
      __m128i k = _mm_add_epi32(m[g & 3], _mm_load_si128(reinterpret_cast<const __m128i*>(kK + 4 * g)));
      s1 = _mm_sha256rnds2_epu32(s1, s0, k);
      k = _mm_shuffle_epi32(k, 0x0E);
      s0 = _mm_sha256rnds2_epu32(s0, s1, k);
      if (g < 12) {  // W for group g+4 replaces group g's words
        __m128i x = _mm_sha256msg1_epu32(m[g & 3], m[(g + 1) & 3]);
        x = _mm_add_epi32(x, _mm_alignr_epi8(m[(g + 3) & 3], m[(g + 2) & 3], 4));
        m[g & 3] = _mm_sha256msg2_epu32(x, m[(g + 3) & 3]);
      }
    }
    s0 = _mm_add_epi32(s0, abef);
    s1 = _mm_add_epi32(s1, cdgh);
  }
  t = _mm_shuffle_epi32(s0, 0x1B);   // A B E F (word 0 first)
  s1 = _mm_shuffle_epi32(s1, 0xB1);  // G H C D
  s0 = _mm_blend_epi16(t, s1, 0xF0);  // A B C D
  s1 = _mm_alignr_epi8(s1, t, 8);     // E F G H
  _mm_storeu_si128(reinterpret_cast<__m128i*>(st), s0);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(st + 4), s1);
}

static bool cpu_has_sha() {
  unsigned a, b, c, d;
  if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
  const bool sha = (b >> 29) & 1;
  if (!__get_cpuid(1, &a, &b, &c, &d)) return false;
  const bool sse41 = (c >> 19) & 1, ssse3 = (c >> 9) & 1;
  return sha && sse41 && ssse3;
}
#endif

// 0: scalar, 1: SHA extensions.  RDET_SHA256_SCALAR=1 pins the scalar loop.
static int pick_impl() {
  const char* e = getenv("RDET_SHA256_SCALAR");
  if (e && e[0] == '1') return 0;
#if defined(__x86_64__)
  return cpu_has_sha() ? 1 : 0;
#else
  return 0;
#endif
}

int sha256_impl() {
  static const int impl = pick_impl();
  return impl;
}

void sha256_compress(uint32_t st[8], const uint8_t* p, size_t nblocks) {
#if defined(__x86_64__)
  if (sha256_impl() == 1) return compress_shani(st, p, nblocks);
#endif
  compress_scalar(st, p, nblocks);
}

}  // namespace rdet
