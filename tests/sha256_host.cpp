// Test driver for the commitment hash (csrc/sha256.cpp): the streaming
// hasher with caller-chosen split points, and each block-compression
// implementation called directly.  Compiled with g++ by tests/test_sha256.py.
#include "../raster-inference_b200/csrc/sha256.cpp"

#include <cstring>

using namespace rdet;

extern "C" int rdet_test_sha_impl() { return sha256_impl(); }

extern "C" int rdet_test_sha_has_ext() {
#if defined(__x86_64__)
  return cpu_has_sha() ? 1 : 0;
#else
  return 0;
#endif
}

// SHA-256 of p[0, n) fed in pieces whose lengths come from a seeded LCG
// (0..max_piece bytes, zero-length pieces included); writes 64 hex digits.
extern "C" void rdet_test_sha_stream(const uint8_t* p, size_t n, uint64_t seed, size_t max_piece, char* out) {
  Sha256 h;
  uint64_t x = seed * 6364136223846793005ull + 1442695040888963407ull;
  size_t off = 0;
  while (off < n) {
    x = x * 6364136223846793005ull + 1442695040888963407ull;
    size_t len = max_piece ? (size_t)(x >> 33) % (max_piece + 1) : n;
    if (len > n - off) len = n - off;
    h.put(p + off, len);
    off += len;
  }
  std::string s = h.hex();
  memcpy(out, s.c_str(), 65);
}

// One implementation's compression of whole blocks: impl 0 scalar, 1 SHA
// extensions (returns -1 when the CPU lacks them).
extern "C" int rdet_test_compress(int impl, uint32_t* st, const uint8_t* p, size_t nblocks) {
  if (impl == 0) { compress_scalar(st, p, nblocks); return 0; }
#if defined(__x86_64__)
  if (!cpu_has_sha()) return -1;
  compress_shani(st, p, nblocks);
  return 0;
#else
  return -1;
#endif
}
