// CPU ORACLE — TEST INFRASTRUCTURE ONLY.
//
// Plain restatement of the reference det_num v1 arithmetic
// (casettek/raster-inference, src/shared/numerics/det_num/ops.rs and
// convert.rs).  Used by tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline / reference arm as the checker.  The product path
// (raster-inference_b200/) never includes, links or calls this file.
//
// Every function names the reference function it restates.  Arithmetic is
// written with 128-bit intermediates exactly where the reference uses i128,
// so that rounding and saturation follow it bit for bit.
#pragma once
#include <cstdint>
#include <cstring>
#include <cassert>

namespace dor {

typedef __int128 i128;
typedef unsigned __int128 u128;

static const int ACT_FRAC = 16;   // types.rs:24
static const int ACC_FRAC = 32;   // types.rs:25
static const int REQ_SHIFT = 16;  // types.rs:26
static const int32_t ONE_ACT = 1 << 16;
static const int64_t ONE_ACC = (int64_t)1 << 32;

inline int32_t clamp_i128_i32(i128 v) {  // ops.rs:485
  if (v < (i128)INT32_MIN) return INT32_MIN;
  if (v > (i128)INT32_MAX) return INT32_MAX;
  return (int32_t)v;
}
inline int64_t clamp_i128_i64(i128 v) {  // ops.rs:489
  if (v < (i128)INT64_MIN) return INT64_MIN;
  if (v > (i128)INT64_MAX) return INT64_MAX;
  return (int64_t)v;
}
inline i128 iabs128(i128 v) { return v < 0 ? -v : v; }

// ops.rs:688 round_ties_even_division (truncating / and %, then ties-to-even)
inline i128 round_ties_even_division(i128 dividend, i128 divisor) {
  i128 q = dividend / divisor;
  i128 r = dividend % divisor;
  if (r == 0) return q;
  i128 twice = iabs128(r) * 2;
  i128 ad = iabs128(divisor);
  i128 step = ((dividend < 0) != (divisor < 0)) ? -1 : 1;
  if (twice < ad) return q;
  if (twice > ad) return q + step;
  return (q & 1) == 0 ? q : q + step;
}

// ops.rs:770 rshift_round_ties_even_bits
inline int64_t rshift_rte(int64_t x, uint32_t shift) {
  if (shift == 0) return x;
  assert(shift < 64);
  i128 divisor = (i128)1 << shift;
  i128 xx = x;
  i128 q = xx / divisor, r = xx % divisor;
  if (r == 0) return (int64_t)q;
  i128 twice = iabs128(r) * 2;
  i128 step = xx < 0 ? -1 : 1;
  i128 out;
  if (twice < divisor) out = q;
  else if (twice > divisor) out = q + step;
  else out = (q & 1) == 0 ? q : q + step;
  return (int64_t)out;
}

// ops.rs:480 narrow_act_sat + ops.rs:445 requantize
inline int32_t requantize(int64_t acc) {
  int64_t r = rshift_rte(acc, REQ_SHIFT);
  if (r < INT32_MIN) return INT32_MIN;
  if (r > INT32_MAX) return INT32_MAX;
  return (int32_t)r;
}

inline int64_t mac_bits(int64_t acc, int32_t a, int32_t b) {  // ops.rs:14
  return (int64_t)((uint64_t)acc + (uint64_t)((int64_t)a * (int64_t)b));
}
inline int64_t acc_combine(int64_t a, int64_t b) {  // ops.rs:28
  return (int64_t)((uint64_t)a + (uint64_t)b);
}
inline int32_t add_sat(int32_t a, int32_t b) {  // ops.rs:33
  int32_t r;
  if (__builtin_add_overflow(a, b, &r)) return a < 0 ? INT32_MIN : INT32_MAX;
  return r;
}
inline int32_t sub_sat(int32_t a, int32_t b) {  // ops.rs:428
  int32_t r;
  if (__builtin_sub_overflow(a, b, &r)) return a < 0 ? INT32_MIN : INT32_MAX;
  return r;
}
inline int32_t neg_sat32(int32_t a) { return a == INT32_MIN ? INT32_MAX : -a; }
inline int64_t neg_sat64(int64_t a) { return a == INT64_MIN ? INT64_MAX : -a; }
inline int64_t acc_add_sat(int64_t a, int64_t b) {  // ops.rs:433
  int64_t r;
  if (__builtin_add_overflow(a, b, &r)) return a < 0 ? INT64_MIN : INT64_MAX;
  return r;
}
inline int32_t mul_sat(int32_t a, int32_t b) {  // ops.rs:38
  return requantize((int64_t)a * (int64_t)b);
}
inline int32_t scale_act(int32_t v, int32_t s) { return mul_sat(v, s); }  // ops.rs:45

inline int32_t div_act(int32_t n, int32_t d) {  // ops.rs:50
  assert(d != 0);
  i128 dividend = (i128)n * ((i128)1 << ACT_FRAC);
  return clamp_i128_i32(round_ties_even_division(dividend, (i128)d));
}
inline int64_t div_acc(int64_t n, int64_t d) {  // ops.rs:64
  assert(d != 0);
  i128 dividend = (i128)n * ((i128)1 << ACC_FRAC);
  return clamp_i128_i64(round_ties_even_division(dividend, (i128)d));
}
inline int64_t div_acc_by_u32(int64_t v, uint32_t d) {  // ops.rs:78
  assert(d != 0);
  return clamp_i128_i64(round_ties_even_division((i128)v, (i128)d));
}
inline int64_t acc_mul(int64_t l, int64_t r) {  // ops.rs:682
  i128 p = (i128)l * (i128)r;
  return clamp_i128_i64(round_ties_even_division(p, (i128)1 << ACC_FRAC));
}
inline int64_t act_to_acc(int32_t v) { return (int64_t)v * ((int64_t)1 << REQ_SHIFT); }  // ops.rs:493

// ops.rs:463 argmax_first: larger wins, ties keep the lowest index.
inline size_t argmax_first(const int32_t* xs, size_t n) {
  size_t best = 0;
  int32_t bv = xs[0];
  for (size_t i = 1; i < n; ++i)
    if (xs[i] > bv) { best = i; bv = xs[i]; }
  return best;
}

// ops.rs:765 / ops.rs:719 inv_sqrt_acc: bisection on r with r^2 * x <= 2^64.
inline u128 inv_sqrt_product(uint32_t c, u128 d) {
  u128 cc = (u128)c * (u128)c;
  // saturating multiplies (never saturate for the value ranges reached)
  if (d != 0 && cc > (~(u128)0) / d) return ~(u128)0;
  return cc * d;
}
inline int32_t inv_sqrt_acc(int64_t x) {
  assert(x >= 0);
  if (x == 0) return INT32_MAX;
  const u128 target = (u128)1 << 64;
  const u128 d = (u128)(uint64_t)x;
  const uint32_t maxb = (uint32_t)INT32_MAX;
  if (inv_sqrt_product(maxb, d) <= target) return INT32_MAX;
  uint32_t lo = 0, hi = maxb;
  while (lo < hi) {
    uint32_t mid = lo + ((hi - lo + 1) / 2);
    if (inv_sqrt_product(mid, d) <= target) lo = mid;
    else hi = mid - 1;
  }
  uint32_t lower = lo;
  uint32_t upper = lower == UINT32_MAX ? lower : lower + 1;
  if (upper > maxb) upper = maxb;
  u128 lp = inv_sqrt_product(lower, d), up = inv_sqrt_product(upper, d);
  u128 le = target - lp;
  u128 ue = up > target ? up - target : 0;
  uint32_t out;
  if (upper == lower || le < ue) out = lower;
  else if (ue < le) out = upper;
  else out = (lower & 1) == 0 ? lower : upper;
  return (int32_t)out;
}

// ops.rs:406 rms_norm_scale
inline int32_t rms_norm_scale(const int32_t* x, size_t n, int64_t eps) {
  assert(n > 0 && eps >= 0);
  int64_t s = 0;
  for (size_t i = 0; i < n; ++i) s = acc_add_sat(s, (int64_t)x[i] * (int64_t)x[i]);
  int64_t mean = div_acc_by_u32(s, (uint32_t)n);
  return inv_sqrt_acc(acc_add_sat(mean, eps));
}
// ops.rs:95 rms_norm_in_place
inline void rms_norm_in_place(int32_t* x, const int32_t* w, size_t n, int64_t eps) {
  int32_t scale = rms_norm_scale(x, n, eps);
  for (size_t i = 0; i < n; ++i) x[i] = mul_sat(mul_sat(x[i], scale), w[i]);
}
// ops.rs:121 value_rms_norm_in_place
inline void value_rms_norm_in_place(int32_t* x, size_t n, int64_t eps) {
  int32_t scale = rms_norm_scale(x, n, eps);
  for (size_t i = 0; i < n; ++i) x[i] = mul_sat(x[i], scale);
}

// ops.rs:505 softmax_exp_term
inline int64_t softmax_exp_term(int64_t delta) {
  const int64_t LN2 = 2977044472LL;
  const int64_t MIN_DELTA = -((int64_t)16 << ACC_FRAC);
  assert(delta <= 0);
  if (delta <= MIN_DELTA) return 0;
  int64_t pos = neg_sat64(delta);
  int64_t shift = pos / LN2;
  int64_t r = pos % LN2;
  int64_t r2 = acc_mul(r, r), r3 = acc_mul(r2, r), r4 = acc_mul(r3, r), r5 = acc_mul(r4, r);
  int64_t approx = acc_add_sat(
      acc_add_sat(ONE_ACC, neg_sat64(r)),
      acc_add_sat(div_acc_by_u32(r2, 2),
                  acc_add_sat(neg_sat64(div_acc_by_u32(r3, 6)),
                              acc_add_sat(div_acc_by_u32(r4, 24), neg_sat64(div_acc_by_u32(r5, 120))))));
  if (approx <= 0) return 0;
  if (shift >= 0 && shift < 64) return rshift_rte(approx, (uint32_t)shift);
  return 0;
}
// ops.rs:261
inline int64_t attention_softmax_exp_term(int32_t logit, int32_t max_logit) {
  return softmax_exp_term(act_to_acc(sub_sat(logit, max_logit)));
}
// ops.rs:230 attention_softmax_into (weights[n]; exp scratch caller-provided)
inline void attention_softmax(const int32_t* logits, size_t n, int64_t* expv, int32_t* w) {
  assert(n > 0);
  size_t mi = argmax_first(logits, n);
  int32_t ml = logits[mi];
  int64_t sum = 0;
  for (size_t i = 0; i < n; ++i) { expv[i] = attention_softmax_exp_term(logits[i], ml); }
  for (size_t i = 0; i < n; ++i) sum = acc_add_sat(sum, expv[i]);
  int32_t sw = 0;
  for (size_t i = 0; i < n; ++i) { w[i] = requantize(div_acc(expv[i], sum)); }
  for (size_t i = 0; i < n; ++i) sw = add_sat(sw, w[i]);
  w[mi] = add_sat(w[mi], sub_sat(ONE_ACT, sw));
}

// ops.rs:354 tanh_act
inline int32_t tanh_act(int32_t x) {
  const int32_t LIN = 27 << 16, QUAD = 9 << 16, SAT = 3 << 16;
  if (x >= SAT) return ONE_ACT;
  if (x <= -SAT) return neg_sat32(ONE_ACT);
  int32_t sq = mul_sat(x, x);
  int32_t num_scale = add_sat(LIN, sq);
  int32_t den_scale = add_sat(LIN, mul_sat(QUAD, sq));
  return div_act(mul_sat(x, num_scale), den_scale);
}
// ops.rs:377 softcap_act
inline int32_t softcap_act(int32_t x, int32_t cap) {
  assert(cap > 0);
  return mul_sat(cap, tanh_act(div_act(x, cap)));
}
// ops.rs:388 gelu_pytorch_tanh_act
inline int32_t gelu_act(int32_t x) {
  const int32_t HALF = 1 << 15, INNER = 52290, CUBIC = 2930;
  int32_t sq = mul_sat(x, x);
  int32_t cu = mul_sat(sq, x);
  int32_t inner = add_sat(x, mul_sat(CUBIC, cu));
  int32_t t = tanh_act(mul_sat(INNER, inner));
  return mul_sat(mul_sat(HALF, x), add_sat(ONE_ACT, t));
}

// ops.rs:605 pow_acc_u32
inline int64_t pow_acc_u32(int64_t b, uint32_t e) {
  int64_t r = ONE_ACC;
  for (uint32_t i = 0; i < e; ++i) r = acc_mul(r, b);
  return r;
}
// ops.rs:561 nth_root_acc
inline int64_t nth_root_acc(int64_t v, uint32_t deg) {
  assert(deg > 0 && v > 0);
  if (deg == 1 || v == ONE_ACC) return v;
  int64_t lo = 0, hi = v > ONE_ACC ? v : ONE_ACC;
  while (lo < hi) {
    int64_t mid = lo + ((hi - lo + 1) / 2);
    if (pow_acc_u32(mid, deg) <= v) lo = mid;
    else hi = mid - 1;
  }
  int64_t lower = lo;
  int64_t upper = lower == INT64_MAX ? lower : lower + 1;
  int64_t lv = pow_acc_u32(lower, deg), uv = pow_acc_u32(upper, deg);
  i128 le = iabs128((i128)v - (i128)lv), ue = iabs128((i128)uv - (i128)v);
  if (ue < le) return upper;
  if (le < ue) return lower;
  return (lower & 1) == 0 ? lower : upper;
}
// ops.rs:555 rope_frequency_step
inline int64_t rope_frequency_step(int64_t base, size_t freq_base_dim) {
  return div_acc(ONE_ACC, nth_root_acc(base, (uint32_t)(freq_base_dim / 2)));
}
// ops.rs:647 / :665 polynomials
inline int64_t sin_poly(int64_t x) {
  int64_t x2 = acc_mul(x, x), x3 = acc_mul(x2, x), x5 = acc_mul(x3, x2), x7 = acc_mul(x5, x2);
  return acc_add_sat(acc_add_sat(x, neg_sat64(div_acc_by_u32(x3, 6))),
                     acc_add_sat(div_acc_by_u32(x5, 120), neg_sat64(div_acc_by_u32(x7, 5040))));
}
inline int64_t cos_poly(int64_t x) {
  int64_t x2 = acc_mul(x, x), x4 = acc_mul(x2, x2), x6 = acc_mul(x4, x2);
  return acc_add_sat(acc_add_sat(ONE_ACC, neg_sat64(div_acc_by_u32(x2, 2))),
                     acc_add_sat(div_acc_by_u32(x4, 24), neg_sat64(div_acc_by_u32(x6, 720))));
}
// ops.rs:619 sin_cos_acc -> (cos, sin)
inline void sin_cos_acc(int64_t angle, int32_t* cos_out, int32_t* sin_out) {
  const int64_t HALF_PI = 6746518852LL, PI = 13493037705LL, THREE_HALF_PI = 20239556557LL,
                TWO_PI = 26986075409LL;
  int64_t red = angle % TWO_PI;
  if (red < 0) red += TWO_PI;  // rem_euclid
  int64_t qa;
  int ss, cs;
  if (red <= HALF_PI) { qa = red; ss = 1; cs = 1; }
  else if (red <= PI) { qa = PI - red; ss = 1; cs = -1; }
  else if (red <= THREE_HALF_PI) { qa = red - PI; ss = -1; cs = -1; }
  else { qa = TWO_PI - red; ss = -1; cs = 1; }
  int32_t s = requantize(sin_poly(qa)), c = requantize(cos_poly(qa));
  if (ss < 0) s = neg_sat32(s);
  if (cs < 0) c = neg_sat32(c);
  *cos_out = c;
  *sin_out = s;
}
// ops.rs:613
inline int64_t mul_usize_by_acc(size_t m, int64_t v) { return clamp_i128_i64((i128)m * (i128)v); }

// ops.rs:151 rope_rotate_pairs_in_place.  `step` = rope_frequency_step(base,
// freq_base_dim), computed once per (base, dim) by the caller: the reference
// recomputes the identical value on every call.
inline void rope_rotate_with_step(int32_t* v, size_t rotary_dim, int64_t step, size_t position) {
  if (rotary_dim == 0 || position == 0) return;
  size_t half = rotary_dim / 2;
  int64_t inv_f = ONE_ACC;
  for (size_t i = 0; i < half; ++i) {
    int32_t c, s;
    sin_cos_acc(mul_usize_by_acc(position, inv_f), &c, &s);
    int32_t l = v[i], r = v[i + half];
    v[i] = sub_sat(mul_sat(l, c), mul_sat(r, s));
    v[i + half] = add_sat(mul_sat(r, c), mul_sat(l, s));
    inv_f = acc_mul(inv_f, step);
  }
}

// convert.rs:108 f32_to_fixed_bits and helpers.
inline u128 rte_div_pow2(u128 v, uint32_t shift) {
  if (shift == 0) return v;
  if (shift >= 128) return 0;
  u128 q = v >> shift, rem = v & (((u128)1 << shift) - 1), half = (u128)1 << (shift - 1);
  if (rem > half || (rem == half && (q & 1) == 1)) return q + 1;
  return q;
}
inline u128 sat_shl(u128 v, uint32_t shift, u128 maxm) {
  if (v == 0) return 0;
  if (shift >= 128) return maxm;
  if (v > (maxm >> shift)) return maxm;
  return v << shift;
}
inline i128 f32_to_fixed_bits(float x, int frac, u128 maxpos, u128 maxneg) {
  uint32_t bits;
  memcpy(&bits, &x, 4);
  bool neg = (bits >> 31) != 0;
  int32_t eb = (int32_t)((bits >> 23) & 0xff);
  uint32_t fb = bits & 0x7fffff;
  if (eb == 0 && fb == 0) return 0;
  u128 sig;
  int32_t e;
  if (eb == 0) { sig = fb; e = -149; }
  else { sig = (u128)((1u << 23) | fb); e = eb - 127 - 23; }
  int32_t se = e + frac;
  u128 maxm = neg ? maxneg : maxpos;
  u128 mag;
  if (se >= 0) mag = sat_shl(sig, (uint32_t)se, maxm);
  else { mag = rte_div_pow2(sig, (uint32_t)(-se)); if (mag > maxm) mag = maxm; }
  if (neg) return mag >= maxneg ? -(i128)maxneg : -(i128)mag;
  return (i128)mag;
}
// convert.rs:82
inline int32_t f32_to_act(float x) {
  i128 b = f32_to_fixed_bits(x, ACT_FRAC, (u128)INT32_MAX, (u128)1 << 31);
  if (b < 0) return b <= (i128)INT32_MIN ? INT32_MIN : (int32_t)b;
  return b > (i128)INT32_MAX ? INT32_MAX : (int32_t)b;
}
// convert.rs:95
inline int64_t f32_to_acc(float x) {
  i128 b = f32_to_fixed_bits(x, ACC_FRAC, (u128)INT64_MAX, (u128)1 << 63);
  if (b < 0) return b <= (i128)INT64_MIN ? INT64_MIN : (int64_t)b;
  return b > (i128)INT64_MAX ? INT64_MAX : (int64_t)b;
}

}  // namespace dor
