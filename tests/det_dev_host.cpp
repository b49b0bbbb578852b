// Host build of the device det arithmetic (raster-inference_b200/csrc/
// det_dev.cuh) checked against the CPU oracle (oracle/det_num.hpp), which
// restates the reference's det_num ops.rs.  Test infrastructure: compiled by
// tests/test_det_dev_host.py with g++ and called through ctypes; the kernels
// include the same header, so a mismatch here is a kernel parity bug found
// without a GPU.
#define RDET_HD inline
#include "../raster-inference_b200/csrc/det_dev.cuh"
#include "../oracle/det_num.hpp"

#include <algorithm>
#include <cstring>

namespace {

struct Rng {
  uint64_t s;
  uint64_t next() {
    s += 0x9E3779B97F4A7C15ull;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  // magnitude drawn uniformly over bit lengths 0..bits, random sign if signed
  int64_t wide(int bits, bool sign) {
    int b = (int)(next() % (uint64_t)(bits + 1));
    uint64_t v = b == 0 ? 0 : (next() >> (64 - b));
    if (b == 64) v &= 0x7fffffffffffffffull;
    int64_t r = (int64_t)v;
    return (sign && (next() & 1)) ? -r : r;
  }
  int32_t act(int bits = 31) { return (int32_t)wide(bits, true); }
};

const int32_t kActEdges[] = {0, 1, -1, 2, -2, 0x8000, -0x8000, 0x10000, -0x10000, 3 << 16, -(3 << 16),
                             (3 << 16) - 1, -(3 << 16) + 1, INT32_MAX, INT32_MIN, INT32_MAX - 1, INT32_MIN + 1};

}  // namespace

extern "C" int64_t rdet_host_check(const char* fn, uint64_t seed, int64_t n) {
  Rng g{seed};
  int64_t bad = 0;
  auto edge = [&](int64_t i) -> bool { return i < (int64_t)(sizeof(kActEdges) / sizeof(kActEdges[0])); };
  if (!strcmp(fn, "inv_sqrt_acc")) {
    // every power of two and its neighbours, then random magnitudes
    for (int b = 0; b < 63; ++b)
      for (int64_t d = -2; d <= 2; ++d) {
        int64_t x = ((int64_t)1 << b) + d;
        if (x < 0) continue;
        bad += rdet::inv_sqrt_acc(x) != dor::inv_sqrt_acc(x);
      }
    for (int64_t i = 0; i < n; ++i) {
      int64_t x = g.wide(63, false);
      bad += rdet::inv_sqrt_acc(x) != dor::inv_sqrt_acc(x);
    }
  } else if (!strcmp(fn, "rms_norm_scale")) {
    int32_t v[64];
    for (int64_t i = 0; i < n; ++i) {
      int len = 1 + (int)(g.next() % 64);
      int bits = 1 + (int)(g.next() % 31);
      for (int k = 0; k < len; ++k) v[k] = g.act(bits);
      int64_t eps = g.wide(20, false);
      int64_t s = 0;
      for (int k = 0; k < len; ++k) s = rdet::acc_add_sat(s, (int64_t)v[k] * v[k]);
      int32_t dev = rdet::inv_sqrt_acc(rdet::acc_add_sat(rdet::div_acc_by_u32(s, (uint32_t)len), eps));
      bad += dev != dor::rms_norm_scale(v, (size_t)len, eps);
    }
  } else if (!strcmp(fn, "requantize")) {
    for (int64_t i = 0; i < n; ++i) {
      int64_t a = g.wide(64, true);
      bad += rdet::requantize(a) != dor::requantize(a);
    }
  } else if (!strcmp(fn, "requantize_edges")) {
    // every value within 2^17 of the saturation and sign boundaries, and of
    // the ties around them
    const int64_t centers[] = {0, (int64_t)1 << 47, -((int64_t)1 << 47), ((int64_t)INT32_MAX << 16),
                               ((int64_t)INT32_MIN << 16), INT64_MAX - (1 << 17), INT64_MIN + (1 << 17),
                               (int64_t)1 << 32, -((int64_t)1 << 32)};
    for (int64_t c : centers)
      for (int64_t o = -(1 << 17); o <= (1 << 17); ++o) {
        const int64_t a = c + o;
        bad += rdet::requantize(a) != dor::requantize(a);
      }
    (void)n;
  } else if (!strcmp(fn, "rshift_rte")) {
    for (int64_t i = 0; i < n; ++i) {
      int64_t a = g.wide(64, true);
      uint32_t s = 1 + (uint32_t)(g.next() % 63);
      bad += rdet::rshift_rte(a, s) != dor::rshift_rte(a, s);
    }
  } else if (!strcmp(fn, "div_act")) {
    for (int64_t i = 0; i < n; ++i) {
      int32_t a = edge(i) ? kActEdges[i] : g.act();
      int32_t b = g.act();
      if (b == 0) b = 1;
      bad += rdet::div_act(a, b) != dor::div_act(a, b);
    }
  } else if (!strcmp(fn, "div_acc_by_u32")) {
    for (int64_t i = 0; i < n; ++i) {
      int64_t a = g.wide(64, true);
      uint32_t d = 1 + (uint32_t)(g.next() % 0xfffffffeull);
      bad += rdet::div_acc_by_u32(a, d) != dor::div_acc_by_u32(a, d);
    }
  } else if (!strcmp(fn, "div_edges")) {
    // the run-time-divisor division at its edges: every divisor class (small,
    // the model dims, around 2^31 and 2^32), dividends at the i64 limits,
    // exact multiples, ties and their neighbours, and divisors of 1..12 bits
    // with full-range dividends (the largest first estimates)
    const uint32_t ds[] = {1, 2, 3, 5, 6, 7, 24, 120, 255, 256, 257, 512, 2560, 5040, 10240, 65535, 65536,
                           0x7fffffffu, 0x80000000u, 0x80000001u, 0xfffffffeu, 0xffffffffu};
    const int64_t as[] = {INT64_MIN, INT64_MIN + 1, INT64_MAX, INT64_MAX - 1, -1, 0, 1,
                          (int64_t)1 << 62, -((int64_t)1 << 62), (int64_t)1 << 53, ((int64_t)1 << 53) + 1};
    for (uint32_t d : ds) {
      for (int64_t a : as) bad += rdet::div_acc_by_u32(a, d) != dor::div_acc_by_u32(a, d);
      for (int k = 0; k < 64; ++k) {
        const int64_t base = (int64_t)(g.next() >> 2) / (int64_t)d * (int64_t)d;  // a multiple of d
        for (int64_t off = -2; off <= 2; ++off)
          for (int64_t sgn = -1; sgn <= 1; sgn += 2) {
            const int64_t m = sgn * base;
            int64_t a = m + off;
            bad += rdet::div_acc_by_u32(a, d) != dor::div_acc_by_u32(a, d);
            a = m + (int64_t)(d / 2) + off;  // around the tie
            bad += rdet::div_acc_by_u32(a, d) != dor::div_acc_by_u32(a, d);
          }
      }
    }
    for (int64_t i = 0; i < n; ++i) {
      const int bits = 1 + (int)(g.next() % 12);
      uint32_t d = (uint32_t)(g.next() & ((1u << bits) - 1));
      if (d == 0) d = 1;
      const int64_t a = g.wide(64, true);
      bad += rdet::div_acc_by_u32(a, d) != dor::div_acc_by_u32(a, d);
      const int32_t x = g.act();
      int32_t y = (int32_t)(g.next() & ((1u << bits) - 1)) * ((g.next() & 1) ? 1 : -1);
      if (y == 0) y = -1;
      bad += rdet::div_act(x, y) != dor::div_act(x, y);
    }
    const int32_t acts[] = {INT32_MIN, INT32_MIN + 1, INT32_MAX, -1, 0, 1, 32768, -32768};
    for (int32_t x : acts)
      for (int32_t y : acts)
        if (y) bad += rdet::div_act(x, y) != dor::div_act(x, y);
  } else if (!strcmp(fn, "exp_term_all")) {
    // every logit - max difference the series sees (beyond -16 the term is
    // 0), with the max at 0, at the i32 extremes and at random values
    const int32_t maxes[] = {0, INT32_MAX, INT32_MIN + (16 << 16) + 8, 123456789};
    for (int32_t m : maxes)
      for (int64_t dd = -(16 << 16) - 64; dd <= 0; ++dd) {
        if ((int64_t)m + dd < INT32_MIN) continue;
        const int32_t l = (int32_t)((int64_t)m + dd);
        bad += rdet::exp_term(l, m) != dor::attention_softmax_exp_term(l, m);
      }
    for (int64_t i = 0; i < n; ++i) {
      const int32_t m = g.act();
      const int32_t l = (int32_t)std::max<int64_t>(INT32_MIN, (int64_t)m - (int64_t)(g.next() % (17u << 16)));
      bad += rdet::exp_term(l, m) != dor::attention_softmax_exp_term(l, m);
    }
  } else if (!strcmp(fn, "acc_mul")) {
    for (int64_t i = 0; i < n; ++i) {
      int64_t a = g.wide(64, true), b = g.wide(64, true);
      bad += rdet::acc_mul(a, b) != dor::acc_mul(a, b);
    }
  } else if (!strcmp(fn, "exp_term")) {
    for (int64_t i = 0; i < n; ++i) {
      int32_t m = g.act(), l = g.act();
      if (l > m) { int32_t t = l; l = m; m = t; }
      bad += rdet::exp_term(l, m) != dor::attention_softmax_exp_term(l, m);
    }
  } else if (!strcmp(fn, "softmax_weight")) {
    for (int64_t i = 0; i < n; ++i) {
      int64_t sum = (int64_t)1 << 32;
      sum += g.wide(62, false);
      if (sum < 0) sum = INT64_MAX;
      int64_t e = (int64_t)(g.next() % ((uint64_t)1 << 32)) + 1;
      if (g.next() % 8 == 0) e = (int64_t)1 << 32;
      bad += rdet::softmax_weight(e, sum) != dor::requantize(dor::div_acc(e, sum));
    }
    // sums of a few exp terms (the windows' range) with e at and around the
    // ties of both roundings, and sums at the 2^61 switch
    for (int64_t i = 0; i < n; ++i) {
      const int64_t sum = ((int64_t)1 << 32) + (int64_t)(g.next() % ((uint64_t)1 << (33 + i % 17)));
      const int64_t q = (int64_t)(g.next() % (((uint64_t)1 << 32) + 1));  // a target quotient
      const int64_t e0 = (int64_t)(((unsigned __int128)q * (uint64_t)sum) >> 32);
      for (int64_t off = -1; off <= 1; ++off) {
        const int64_t e = std::min<int64_t>(std::max<int64_t>(e0 + off, 1), std::min<int64_t>(sum, (int64_t)1 << 32));
        bad += rdet::softmax_weight(e, sum) != dor::requantize(dor::div_acc(e, sum));
      }
    }
    const int64_t sums[] = {((int64_t)1 << 61) - 1, (int64_t)1 << 61, ((int64_t)1 << 61) + 1, INT64_MAX};
    for (int64_t sum : sums)
      for (int64_t e : {(int64_t)1, (int64_t)2, ((int64_t)1 << 32) - 1, (int64_t)1 << 32})
        bad += rdet::softmax_weight(e, sum) != dor::requantize(dor::div_acc(e, sum));
  } else if (!strcmp(fn, "tanh_act")) {
    for (int64_t i = 0; i < n; ++i) {
      int32_t x = edge(i) ? kActEdges[i] : g.act(20);
      bad += rdet::tanh_act(x) != dor::tanh_act(x);
    }
  } else if (!strcmp(fn, "softcap_act")) {
    for (int64_t i = 0; i < n; ++i) {
      int32_t x = edge(i) ? kActEdges[i] : g.act(24);
      int32_t cap = 1 + (int32_t)(g.next() % (64u << 16));
      bad += rdet::softcap_act(x, cap) != dor::softcap_act(x, cap);
    }
  } else if (!strcmp(fn, "gelu_act")) {
    for (int64_t i = 0; i < n; ++i) {
      int32_t x = edge(i) ? kActEdges[i] : g.act(22);
      bad += rdet::gelu_act(x) != dor::gelu_act(x);
    }
  } else if (!strcmp(fn, "sin_cos_acc")) {
    for (int64_t i = 0; i < n; ++i) {
      int64_t a = g.wide(64, true);
      int32_t c0, s0, c1, s1;
      rdet::sin_cos_acc(a, &c0, &s0);
      dor::sin_cos_acc(a, &c1, &s1);
      bad += (c0 != c1) || (s0 != s1);
    }
  } else if (!strcmp(fn, "pos_angle")) {
    for (int64_t i = 0; i < n; ++i) {
      uint32_t p = (uint32_t)(g.next() % (1u << 20));
      int64_t f = g.wide(64, true);
      bad += rdet::pos_angle(p, f) != dor::mul_usize_by_acc(p, f);
    }
  } else {
    return -1;
  }
  return bad;
}
