// Device-side det_num v1 arithmetic for the B200 kernels.
//
// Semantics follow casettek/raster-inference src/shared/numerics/det_num/
// ops.rs (the function each helper restates is named beside it).  Act and
// Wgt are i32 Q16.16 bit patterns, Acc is i64 Q32.32; MAC reductions wrap
// (two's complement), every narrowing is round-half-to-even.
//
// GPU formulations (all exact):
//  * a right shift with round-half-even is done as an arithmetic (floor)
//    shift plus a look at the dropped bits; for ties-to-even this equals the
//    reference's truncating-division form, because rounding half to even is
//    symmetric in sign.
//  * 64x64 -> 128-bit products use __int128 only where the reference uses
//    i128 (acc_mul, div_acc);
//  * the softmax division div_acc(e, sum) (e <= 2^32 <= sum) is computed from
//    a double estimate corrected with an exact 128-bit remainder.
#pragma once
#include <cmath>
#include <cstdint>

#ifndef RDET_HD
#define RDET_HD __host__ __device__ __forceinline__
#endif

namespace rdet {

constexpr int32_t kOneAct = 1 << 16;
constexpr int64_t kOneAcc = (int64_t)1 << 32;

// ops.rs:770 + :445 — floor shift by 16 then ties-to-even on the low half,
// on the two 32-bit words of a: q = low word of a >> 16; the quotient fits
// in i32 iff bits 47..63 of a all equal q's sign bit; the dropped half r
// rounds up iff r + 0x7fff + (q & 1) carries into bit 16.
RDET_HD int32_t requantize(int64_t a) {
  const uint32_t lo = (uint32_t)a;
  const int32_t hi = (int32_t)(a >> 32);
  const int32_t q = (int32_t)(((uint32_t)hi << 16) | (lo >> 16));
  const uint32_t inc = ((lo & 0xffffu) + 0x7fffu + ((uint32_t)q & 1u)) >> 16;
  if ((hi >> 15) != (q >> 31)) return hi < 0 ? INT32_MIN : INT32_MAX;
  if (q == INT32_MAX && inc) return INT32_MAX;
  return q + (int32_t)inc;
}

// ops.rs:770 for an arbitrary shift in [1, 63]
RDET_HD int64_t rshift_rte(int64_t a, uint32_t s) {
  if (s == 0) return a;
  int64_t q = a >> s;
  uint64_t mask = ((uint64_t)1 << s) - 1, half = (uint64_t)1 << (s - 1);
  uint64_t r = (uint64_t)a & mask;
  if (r > half || (r == half && (q & 1))) q += 1;
  return q;
}

RDET_HD int32_t add_sat(int32_t a, int32_t b) {  // ops.rs:33
  int64_t s = (int64_t)a + b;
  return s > INT32_MAX ? INT32_MAX : (s < INT32_MIN ? INT32_MIN : (int32_t)s);
}
RDET_HD int32_t sub_sat(int32_t a, int32_t b) {  // ops.rs:428
  int64_t s = (int64_t)a - b;
  return s > INT32_MAX ? INT32_MAX : (s < INT32_MIN ? INT32_MIN : (int32_t)s);
}
RDET_HD int32_t neg_sat(int32_t a) { return a == INT32_MIN ? INT32_MAX : -a; }
RDET_HD int64_t neg_sat64(int64_t a) { return a == INT64_MIN ? INT64_MAX : -a; }
RDET_HD int64_t acc_add_sat(int64_t a, int64_t b) {  // ops.rs:433
  uint64_t s = (uint64_t)a + (uint64_t)b;
  // overflow iff a and b share a sign that s does not
  if (((a ^ (int64_t)s) & (b ^ (int64_t)s)) < 0) return a < 0 ? INT64_MIN : INT64_MAX;
  return (int64_t)s;
}
// a * b widened to i64 (one widening multiply on the device)
RDET_HD int64_t mul_wide(int32_t a, int32_t b) {
#ifdef __CUDA_ARCH__
  int64_t d;
  asm("mul.wide.s32 %0, %1, %2;" : "=l"(d) : "r"(a), "r"(b));
  return d;
#else
  return (int64_t)a * (int64_t)b;
#endif
}
RDET_HD int32_t mul_sat(int32_t a, int32_t b) { return requantize(mul_wide(a, b)); }  // ops.rs:38

// c + a * b for i32 a, b and an i64 accumulator, wrapping (the MAC step of
// every det dot product).  On the device one widening multiply-add: written
// as (int64_t)a * b + c the compiler emits a slower sequence.
RDET_HD int64_t mac_wide(int64_t c, int32_t a, int32_t b) {
#ifdef __CUDA_ARCH__
  int64_t d;
  asm("mad.wide.s32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(c));
  return d;
#else
  return (int64_t)((uint64_t)c + (uint64_t)((int64_t)a * (int64_t)b));
#endif
}

// ops.rs:688 specialised to an i64 dividend and a positive i64 divisor.
RDET_HD int64_t rte_div_i64(int64_t n, int64_t d) {
  int64_t q = n / d, r = n % d;
  if (r == 0) return q;
  int64_t ar = r < 0 ? -r : r;
  int64_t step = n < 0 ? -1 : 1;
  uint64_t twice = (uint64_t)ar * 2;
  if (twice < (uint64_t)d) return q;
  if (twice > (uint64_t)d) return q + step;
  return (q & 1) ? q + step : q;
}

// floor(a / d) and its remainder for a <= 2^63 and 0 < d < 2^32, for a
// divisor known only at run time (a 64-bit integer division is a long
// software sequence on the GPU).  The double quotient is off by at most
// 2^11 / d + 1 (a rounds to 53 bits, the quotient once more); the exact
// remainder of that estimate lies within 2^11 + 2d, so a second estimate from
// it (when still large) leaves the quotient within one, and whole-d steps on
// the exact remainder finish it.
RDET_HD uint64_t udiv_u64_u32(uint64_t a, uint32_t d, uint64_t* rem) {
  const double dd = (double)d;
  uint64_t q = (uint64_t)((double)a / dd);
  int64_t r = (int64_t)(a - q * (uint64_t)d);
  if (r < -4 * (int64_t)d || r >= 5 * (int64_t)d) {
    q += (uint64_t)(int64_t)((double)r / dd);
    r = (int64_t)(a - q * (uint64_t)d);
  }
  while (r < 0) { --q; r += d; }
  while (r >= (int64_t)d) { ++q; r -= d; }
  *rem = (uint64_t)r;
  return q;
}

// ops.rs:688 on magnitudes: |n| / |d| rounded half to even, then the sign
// (`neg`) applied.  The reference truncates toward zero and rounds the
// remainder's magnitude, ties to the even truncated quotient: the same value.
RDET_HD int64_t rte_div_mag(uint64_t a, uint32_t d, bool neg) {
  uint64_t r;
  uint64_t q = udiv_u64_u32(a, d, &r);
  const uint64_t twice = 2 * r;  // r < 2^32
  if (twice > d || (twice == d && (q & 1))) q += 1;
  return neg ? (int64_t)(0 - q) : (int64_t)q;
}

// ops.rs:50 div_act: ties-even (n << 16) / d, clamped to i32 (d != 0).
RDET_HD int32_t div_act(int32_t n, int32_t d) {
  const int64_t dividend = (int64_t)n * 65536;  // |dividend| <= 2^47
  const uint64_t a = dividend < 0 ? (uint64_t)(-dividend) : (uint64_t)dividend;
  const uint32_t m = d < 0 ? 0u - (uint32_t)d : (uint32_t)d;
  const int64_t q = rte_div_mag(a, m, (dividend < 0) != (d < 0));
  return q > INT32_MAX ? INT32_MAX : (q < INT32_MIN ? INT32_MIN : (int32_t)q);
}

// ops.rs:78 div_acc_by_u32 (d > 0).  Constant divisors (the series of
// exp_term and sin_cos_acc) call rte_div_i64, which the compiler turns into
// a multiply by a reciprocal.
RDET_HD int64_t div_acc_by_u32(int64_t v, uint32_t d) {
  const uint64_t a = v < 0 ? 0 - (uint64_t)v : (uint64_t)v;
  return rte_div_mag(a, d, v < 0);
}

// ops.rs:682 acc_mul: (l*r) / 2^32, ties to even, clamped to i64.
RDET_HD int64_t acc_mul(int64_t l, int64_t r) {
  __int128 p = (__int128)l * (__int128)r;
  __int128 q = p >> 32;
  uint64_t low = (uint64_t)p & 0xffffffffull;
  if (low > 0x80000000ull || (low == 0x80000000ull && ((uint64_t)q & 1))) q += 1;
  if (q > (__int128)INT64_MAX) return INT64_MAX;
  if (q < (__int128)INT64_MIN) return INT64_MIN;
  return (int64_t)q;
}

// ops.rs:719 inv_sqrt_acc: largest r with r^2*x <= 2^64, then nearest of r,
// r+1 (ties to even).  c^2*x is a 128-bit product; <= 2^64 iff hi==0 or
// (hi==1 and lo==0).
RDET_HD bool isq_le(uint32_t c, uint64_t x) {
  uint64_t cc = (uint64_t)c * c;
  unsigned __int128 p = (unsigned __int128)cc * x;
  uint64_t hi = (uint64_t)(p >> 64), lo = (uint64_t)p;
  return hi == 0 || (hi == 1 && lo == 0);
}
RDET_HD unsigned __int128 isq_prod(uint32_t c, uint64_t x) {
  return (unsigned __int128)((uint64_t)c * c) * x;
}
// The reference bisects on r; isq_le(r, x) is monotone in r, so the same r is
// found by starting from the double estimate 2^32/sqrt(x) (relative error
// below 2^-50, i.e. off by at most one for r < 2^31) and stepping with the
// exact predicate until it flips (the steps make any estimate exact; the
// device takes the estimate from the double reciprocal square root).
RDET_HD int32_t inv_sqrt_acc(int64_t xs) {
  if (xs <= 0) return INT32_MAX;  // x == 0 (negative inputs cannot occur)
  uint64_t x = (uint64_t)xs;
  const uint32_t maxb = 0x7fffffffu;
  if (isq_le(maxb, x)) return INT32_MAX;
#ifdef __CUDA_ARCH__
  const double est = 4294967296.0 * rsqrt((double)x);
#else
  const double est = 4294967296.0 / sqrt((double)x);
#endif
  uint32_t lo = est >= (double)(maxb - 1) ? maxb - 1 : (uint32_t)est;
  while (lo > 0 && !isq_le(lo, x)) --lo;
  while (lo + 1 < maxb && isq_le(lo + 1, x)) ++lo;
  uint32_t up = lo + 1 > maxb ? maxb : lo + 1;
  const unsigned __int128 target = (unsigned __int128)1 << 64;
  unsigned __int128 le = target - isq_prod(lo, x);
  unsigned __int128 upp = isq_prod(up, x);
  unsigned __int128 ue = upp > target ? upp - target : 0;
  uint32_t out;
  if (up == lo || le < ue) out = lo;
  else if (ue < le) out = up;
  else out = (lo & 1) ? up : lo;
  return (int32_t)out;
}

// ops.rs:505 softmax_exp_term for delta = act_to_acc(sub_sat(logit, max)) <= 0.
RDET_HD int64_t softmax_exp_term(int64_t delta) {
  const int64_t LN2 = 2977044472LL;
  if (delta <= -((int64_t)16 << 32)) return 0;
  int64_t pos = -delta;
  int64_t shift = pos / LN2;
  int64_t r = pos - shift * LN2;
  int64_t r2 = acc_mul(r, r), r3 = acc_mul(r2, r), r4 = acc_mul(r3, r), r5 = acc_mul(r4, r);
  int64_t inner = acc_add_sat(rte_div_i64(r4, 24), neg_sat64(rte_div_i64(r5, 120)));
  inner = acc_add_sat(neg_sat64(rte_div_i64(r3, 6)), inner);
  inner = acc_add_sat(rte_div_i64(r2, 2), inner);
  int64_t approx = acc_add_sat(acc_add_sat(kOneAcc, neg_sat64(r)), inner);
  if (approx <= 0) return 0;
  if (shift >= 64) return 0;
  return rshift_rte(approx, (uint32_t)shift);
}
// acc_mul (ops.rs:682) of two values in [0, 2^32): the product fits 64 bits.
RDET_HD uint32_t acc_mul_u32(uint32_t a, uint32_t b) {
  const uint64_t p = (uint64_t)a * b;
  uint32_t q = (uint32_t)(p >> 32);  // <= 2^32 - 2, so the rounding step cannot wrap
  const uint32_t low = (uint32_t)p;
  if (low > 0x80000000u || (low == 0x80000000u && (q & 1))) q += 1;
  return q;
}
// rte_div_i64 of a value in [0, 2^32) by a small constant
RDET_HD uint32_t rte_div_u32(uint32_t v, uint32_t d) {
  const uint32_t q = v / d, r = v - q * d;
  return (2 * r > d || (2 * r == d && (q & 1))) ? q + 1 : q;
}

// ops.rs:261 + :505 for logit <= max_logit (the row maximum): the same
// value as softmax_exp_term in 32-bit pieces.  With delta = -pos in
// (-16, 0], the reduced argument r = pos mod ln2 lies in [0, 2^32), so every
// power r^k is an acc_mul of values below 2^32 and every series term a
// division of such a value by a constant; no term reaches 2^33, so the
// reference's saturating adds add exactly.
RDET_HD int64_t exp_term(int32_t logit, int32_t max_logit) {
  const int32_t d = sub_sat(logit, max_logit);
  if (d > 0) return softmax_exp_term((int64_t)d * 65536);  // a logit above the max: the general form
  if (d <= -(16 << 16)) return 0;                            // delta <= -16
  const uint64_t LN2 = 2977044472ull;
  const uint64_t pos = (uint64_t)(-(int64_t)d) << 16;       // [0, 2^36)
  const uint32_t shift = (uint32_t)(pos / LN2);              // <= 23
  const uint32_t r = (uint32_t)(pos - shift * LN2);
  const uint32_t r2 = acc_mul_u32(r, r), r3 = acc_mul_u32(r2, r), r4 = acc_mul_u32(r3, r),
                 r5 = acc_mul_u32(r4, r);
  const int64_t approx = kOneAcc - (int64_t)r + rte_div_u32(r2, 2) - (int64_t)rte_div_u32(r3, 6) +
                         rte_div_u32(r4, 24) - (int64_t)rte_div_u32(r5, 120);
  if (approx <= 0) return 0;
  return rshift_rte(approx, shift);
}

// ops.rs:64 + :266: requantize(div_acc(e, sum)) for 0 <= e <= sum, sum > 0.
// The quotient q = round_te(e * 2^32 / sum) lies in [0, 2^32]; a double
// estimate is corrected to the exact floor with a 128-bit remainder.
RDET_HD int32_t softmax_weight(int64_t e, int64_t sum) {
  if (e <= 0) return 0;
  unsigned __int128 n = (unsigned __int128)(uint64_t)e << 32;
  uint64_t d = (uint64_t)sum;
  uint64_t q = (uint64_t)((double)e * 4294967296.0 / (double)sum);
  __int128 rem = (__int128)n - (__int128)((unsigned __int128)q * d);
  while (rem < 0) { q -= 1; rem += d; }
  while (rem >= (__int128)d) { q += 1; rem -= d; }
  unsigned __int128 twice = (unsigned __int128)rem * 2;
  if (twice > d || (twice == d && (q & 1))) q += 1;
  return requantize((int64_t)q);
}

// ops.rs:354 tanh_act
RDET_HD int32_t tanh_act(int32_t x) {
  if (x >= (3 << 16)) return kOneAct;
  if (x <= -(3 << 16)) return -kOneAct;
  int32_t sq = mul_sat(x, x);
  int32_t num = mul_sat(x, add_sat(27 << 16, sq));
  int32_t den = add_sat(27 << 16, mul_sat(9 << 16, sq));
  return div_act(num, den);
}
// ops.rs:377 softcap_act (cap > 0)
RDET_HD int32_t softcap_act(int32_t x, int32_t cap) { return mul_sat(cap, tanh_act(div_act(x, cap))); }
// ops.rs:388 gelu_pytorch_tanh_act
RDET_HD int32_t gelu_act(int32_t x) {
  int32_t cu = mul_sat(mul_sat(x, x), x);
  int32_t inner = add_sat(x, mul_sat(2930, cu));
  int32_t t = tanh_act(mul_sat(52290, inner));
  return mul_sat(mul_sat(1 << 15, x), add_sat(kOneAct, t));
}

// ops.rs:619-680 sin_cos_acc -> (cos, sin) for a Q32.32 angle.
RDET_HD void sin_cos_acc(int64_t angle, int32_t* c_out, int32_t* s_out) {
  const int64_t HALF_PI = 6746518852LL, PI = 13493037705LL, THREE_HALF_PI = 20239556557LL,
                TWO_PI = 26986075409LL;
  int64_t red = angle % TWO_PI;
  if (red < 0) red += TWO_PI;
  int64_t a;
  bool sneg, cneg;
  if (red <= HALF_PI) { a = red; sneg = false; cneg = false; }
  else if (red <= PI) { a = PI - red; sneg = false; cneg = true; }
  else if (red <= THREE_HALF_PI) { a = red - PI; sneg = true; cneg = true; }
  else { a = TWO_PI - red; sneg = true; cneg = false; }
  int64_t a2 = acc_mul(a, a);
  int64_t a3 = acc_mul(a2, a), a5 = acc_mul(a3, a2), a7 = acc_mul(a5, a2);
  int64_t sp = acc_add_sat(acc_add_sat(a, neg_sat64(rte_div_i64(a3, 6))),
                           acc_add_sat(rte_div_i64(a5, 120), neg_sat64(rte_div_i64(a7, 5040))));
  int64_t a4 = acc_mul(a2, a2), a6 = acc_mul(a4, a2);
  int64_t cp = acc_add_sat(acc_add_sat(kOneAcc, neg_sat64(rte_div_i64(a2, 2))),
                           acc_add_sat(rte_div_i64(a4, 24), neg_sat64(rte_div_i64(a6, 720))));
  int32_t s = requantize(sp), c = requantize(cp);
  *s_out = sneg ? neg_sat(s) : s;
  *c_out = cneg ? neg_sat(c) : c;
}

// ops.rs:613 mul_usize_by_acc (position * inv_frequency, clamped)
RDET_HD int64_t pos_angle(uint32_t pos, int64_t inv_f) {
  __int128 p = (__int128)pos * inv_f;
  if (p > (__int128)INT64_MAX) return INT64_MAX;
  if (p < (__int128)INT64_MIN) return INT64_MIN;
  return (int64_t)p;
}

}  // namespace rdet
