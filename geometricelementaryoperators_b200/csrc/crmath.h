// crmath.h -- correctly rounded exp and tanh for binary64 (round to nearest,
// ties to even), the same code for the host and the device.
//
// The reference evaluates its graph nonlinearities with the C library's exp and
// tanh (full_cycle_v8.c: tanh node, sigmoid via exp); a GPU port that calls
// CUDA's own functions differs from that by an ulp here and there, and Adam
// amplifies those differences. These functions return the correctly rounded
// result, which is the best any implementation can do: where the C library is
// correctly rounded the two agree bit for bit, and where they differ the result
// here is the closer one.
//
// Method (Ziv's strategy):
//  1. fast path: Tang's table-driven exp, x = (64 m + j) ln2/64 + r, |r| <~ ln2/128,
//     exp(x) = 2^m 2^(j/64) exp(r) with 2^(j/64) and exp(r) - 1 (Taylor series to
//     r^11) in double-double arithmetic (relative error below 2^-100); tanh(x) =
//     expm1(2|x|) / (expm1(2|x|) + 2) in the same arithmetic (below 2^-93 once
//     the cancellation in expm1 is counted). The rounding test accepts the
//     double-double result when both ends of an interval of relative width
//     2^-80 (exp) or 2^-75 (tanh) around it round to the same double; the
//     bounds hold with a factor of 2^15 or more to spare.
//  2. otherwise (about one argument in 2^20 or fewer) an exact path in 256-bit
//     fixed point (232 fraction bits): the same reduction and Taylor series, the
//     table in fixed point and, for tanh, a long division; its error is below
//     2^-220, far inside the margin any binary64 exp or tanh argument needs.
// Constants come from crmath_tables.h (generated from their definitions by
// gen_crmath_tables.py).
#pragma once

#include <math.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define GEO_CR_FN __host__ __device__ __forceinline__
#define GEO_CR_NOINLINE static __host__ __device__ __noinline__
#else
#define GEO_CR_FN inline
#define GEO_CR_NOINLINE inline
#endif

namespace geo {
namespace cr {

struct Tables {
    double exp_t[64][2];
    uint64_t exp_tfix[64][4];
    double l1, l2, l3;
    uint64_t ln2_64fix[4];
    double inv_ln2_64;
    double c_hi[4], c_lo[4];  // 1/n!, n = 2..5
    double c_tail[6];         // 1/n!, n = 6..11
};

#include "crmath_tables.h"

static const Tables kTablesHost = GEO_CR_TABLES_INIT;
#if defined(__CUDACC__)
static __device__ const Tables kTablesDev = GEO_CR_TABLES_INIT;
#endif

GEO_CR_FN const Tables &tables() {
#if defined(__CUDA_ARCH__)
    return kTablesDev;
#else
    return kTablesHost;
#endif
}

GEO_CR_FN uint64_t bits_of(double v) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(v);
#else
    uint64_t b;
    __builtin_memcpy(&b, &v, 8);
    return b;
#endif
}
GEO_CR_FN double from_bits(uint64_t b) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)b);
#else
    double v;
    __builtin_memcpy(&v, &b, 8);
    return v;
#endif
}
// 2^e for -1022 <= e <= 1023.
GEO_CR_FN double pow2(int e) { return from_bits((uint64_t)(e + 1023) << 52); }

// ---- double-double arithmetic (error-free transformations; explicit fma)
struct DD {
    double hi, lo;
};
GEO_CR_FN DD two_sum(double a, double b) {
    const double s = a + b;
    const double bb = s - a;
    return {s, (a - (s - bb)) + (b - bb)};
}
GEO_CR_FN DD fast_two_sum(double a, double b) {  // |a| >= |b| or a == 0
    const double s = a + b;
    return {s, b - (s - a)};
}
GEO_CR_FN DD two_prod(double a, double b) {
    const double p = a * b;
    return {p, fma(a, b, -p)};
}
GEO_CR_FN DD dd_add(DD a, DD b) {
    DD s = two_sum(a.hi, b.hi);
    const DD t = two_sum(a.lo, b.lo);
    s.lo += t.hi;
    s = fast_two_sum(s.hi, s.lo);
    s.lo += t.lo;
    return fast_two_sum(s.hi, s.lo);
}
GEO_CR_FN DD dd_mul(DD a, DD b) {
    DD p = two_prod(a.hi, b.hi);
    p.lo = fma(a.hi, b.lo, fma(a.lo, b.hi, p.lo));
    return fast_two_sum(p.hi, p.lo);
}
GEO_CR_FN DD dd_mul_d(DD a, double b) {
    DD p = two_prod(a.hi, b);
    p.lo = fma(a.lo, b, p.lo);
    return fast_two_sum(p.hi, p.lo);
}
GEO_CR_FN DD dd_div(DD a, DD b) {
    const double q1 = a.hi / b.hi;
    DD r = dd_add(a, dd_mul_d(b, -q1));
    const double q2 = r.hi / b.hi;
    r = dd_add(r, dd_mul_d(b, -q2));
    const double q3 = r.hi / b.hi;
    DD q = fast_two_sum(q1, q2);
    return dd_add(q, DD{q3, 0.0});
}

// Round hi + lo + d (|d| <= eps) to double when every such value rounds alike.
GEO_CR_FN bool ziv_round(DD v, double eps, double *out) {
    const double up = v.hi + (v.lo + eps);
    const double dn = v.hi + (v.lo - eps);
    if (up != dn) return false;
    *out = up;
    return true;
}

// ---- 256-bit fixed point (four 64-bit words, low first; 232 fraction bits)
constexpr int kFrac = 232;
struct U256 {
    uint64_t w[4];
};
GEO_CR_FN uint64_t mulhi(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
    return __umul64hi(a, b);
#else
    return (uint64_t)(((unsigned __int128)a * b) >> 64);
#endif
}
GEO_CR_FN U256 u_zero() { return U256{{0, 0, 0, 0}}; }
GEO_CR_FN bool u_is_zero(const U256 &a) { return (a.w[0] | a.w[1] | a.w[2] | a.w[3]) == 0; }
GEO_CR_FN U256 u_add(const U256 &a, const U256 &b) {
    U256 r;
    uint64_t c = 0;
    for (int i = 0; i < 4; ++i) {
        const uint64_t s = a.w[i] + b.w[i];
        const uint64_t c1 = s < a.w[i];
        r.w[i] = s + c;
        c = c1 | (r.w[i] < s);
    }
    return r;
}
GEO_CR_FN U256 u_sub(const U256 &a, const U256 &b) {
    U256 r;
    uint64_t br = 0;
    for (int i = 0; i < 4; ++i) {
        const uint64_t d = a.w[i] - b.w[i];
        const uint64_t b1 = a.w[i] < b.w[i];
        r.w[i] = d - br;
        br = b1 | (d < br);
    }
    return r;
}
GEO_CR_FN bool u_neg_sign(const U256 &a) { return (a.w[3] >> 63) != 0; }
GEO_CR_FN U256 u_neg(const U256 &a) { return u_sub(u_zero(), a); }
GEO_CR_FN bool u_ge(const U256 &a, const U256 &b) {
    for (int i = 3; i >= 0; --i)
        if (a.w[i] != b.w[i]) return a.w[i] > b.w[i];
    return true;
}
GEO_CR_FN U256 u_shl1(const U256 &a) {
    return U256{{a.w[0] << 1, (a.w[1] << 1) | (a.w[0] >> 63), (a.w[2] << 1) | (a.w[1] >> 63),
                 (a.w[3] << 1) | (a.w[2] >> 63)}};
}
GEO_CR_FN bool u_bit(const U256 &a, int i) { return i >= 0 && i < 256 && ((a.w[i >> 6] >> (i & 63)) & 1u) != 0; }
// Any bit below position i set.
GEO_CR_FN bool u_any_below(const U256 &a, int i) {
    if (i <= 0) return false;
    if (i >= 256) return !u_is_zero(a);
    for (int k = 0; k < (i >> 6); ++k)
        if (a.w[k]) return true;
    const int r = i & 63;
    return r != 0 && (a.w[i >> 6] & ((1ull << r) - 1)) != 0;
}
// floor(a / 2^s) for 0 <= s.
GEO_CR_FN U256 u_shr(const U256 &a, int s) {
    U256 r = u_zero();
    if (s >= 256) return r;
    const int q = s >> 6, b = s & 63;
    for (int i = 0; i + q < 4; ++i) {
        uint64_t v = a.w[i + q] >> b;
        if (b && i + q + 1 < 4) v |= a.w[i + q + 1] << (64 - b);
        r.w[i] = v;
    }
    return r;
}
GEO_CR_FN U256 u_mul_small(const U256 &a, uint64_t k) {  // a * k mod 2^256
    U256 r;
    uint64_t carry = 0;
    for (int i = 0; i < 4; ++i) {
        const uint64_t lo = a.w[i] * k, hi = mulhi(a.w[i], k);
        r.w[i] = lo + carry;
        carry = hi + (r.w[i] < lo);
    }
    return r;
}
GEO_CR_FN U256 u_div_small(const U256 &a, uint32_t n) {  // floor(a / n)
    U256 r = u_zero();
    uint64_t rem = 0;
    for (int i = 7; i >= 0; --i) {
        const uint64_t cur = (rem << 32) | ((a.w[i >> 1] >> (32 * (i & 1))) & 0xffffffffull);
        const uint64_t q = cur / n;
        rem = cur - q * n;
        r.w[i >> 1] |= q << (32 * (i & 1));
    }
    return r;
}
// floor(a * b / 2^232) (both non-negative, product below 2^488).
GEO_CR_FN U256 u_mul_fix(const U256 &a, const U256 &b) {
    uint64_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < 4; ++i) {
        uint64_t carry = 0;
        for (int j = 0; j < 4; ++j) {
            const uint64_t lo = a.w[i] * b.w[j], hi = mulhi(a.w[i], b.w[j]);
            const uint64_t t = r[i + j] + lo;
            const uint64_t c1 = t < lo;
            const uint64_t t2 = t + carry;
            const uint64_t c2 = t2 < t;
            r[i + j] = t2;
            carry = hi + c1 + c2;
        }
        r[i + 4] = carry;
    }
    U256 out;
    for (int k = 0; k < 4; ++k) out.w[k] = (r[3 + k] >> 40) | (k + 4 < 8 ? r[4 + k] << 24 : 0);
    return out;
}
GEO_CR_FN int u_msb(const U256 &a) {
    for (int i = 3; i >= 0; --i)
        if (a.w[i]) {
#if defined(__CUDA_ARCH__)
            return 64 * i + 63 - __clzll((long long)a.w[i]);
#else
            return 64 * i + 63 - __builtin_clzll(a.w[i]);
#endif
        }
    return -1;
}

// Round v = M * 2^(e2 - 232) (M > 0) to the nearest double, ties to even;
// `sticky` says that the exact value lies strictly above M's.
GEO_CR_FN double u_round(const U256 &M, int e2, bool sticky) {
    const int b = u_msb(M);
    if (b < 0) return 0.0;
    const int e = b - kFrac + e2;  // unbiased exponent of v
    if (e > 1023) return INFINITY;
    // s: position of the last kept bit (the ulp) in M
    const int s = e >= -1022 ? b - 52 : b - 52 + (-1022 - e);
    uint64_t mant;
    bool rnd, st;
    if (s > 256) {  // below half the least subnormal
        mant = 0;
        rnd = false;
        st = true;
    } else if (s <= 0) {  // M has no bits below the ulp
        mant = u_shr(M, 0).w[0] << (-s);
        rnd = false;
        st = sticky;
    } else {
        const U256 q = u_shr(M, s);
        mant = q.w[0];
        rnd = u_bit(M, s - 1);
        st = sticky || u_any_below(M, s - 1);
    }
    if (rnd && (st || (mant & 1u))) ++mant;
    if (e >= -1022) {
        int ee = e;
        if (mant >> 53) {
            mant >>= 1;
            ++ee;
        }
        if (ee > 1023) return INFINITY;
        return from_bits(((uint64_t)(ee + 1023) << 52) | (mant & ((1ull << 52) - 1)));
    }
    return from_bits(mant);  // subnormal (2^52 here is the least normal)
}

// x as fixed point (two's complement), |x| in [2^-54, 2^20).
GEO_CR_FN U256 u_from_double(double x) {
    const uint64_t bx = bits_of(x);
    const int ex = (int)((bx >> 52) & 0x7ff) - 1075;  // x = mant * 2^ex
    const uint64_t mant = (bx & ((1ull << 52) - 1)) | (1ull << 52);
    const int sh = ex + kFrac;  // >= 232 - 54 - 52 > 0
    U256 r = u_zero();
    const int q = sh >> 6, b = sh & 63;
    r.w[q] = mant << b;
    if (b && q + 1 < 4) r.w[q + 1] = mant >> (64 - b);
    return (bx >> 63) ? u_neg(r) : r;
}

// exp(y) = M * 2^(m - 232) with M the fixed-point product 2^(j/64) exp(r); the
// error of M is below 2^-224 relative. |y| < 746.
GEO_CR_NOINLINE void exp_fixed(double y, int k, U256 *M, int *m) {
    const Tables &T = tables();
    const U256 Y = u_from_double(y);
    U256 C;
    for (int i = 0; i < 4; ++i) C.w[i] = T.ln2_64fix[i];
    U256 KC = u_mul_small(C, (uint64_t)(k < 0 ? -k : k));
    if (k < 0) KC = u_neg(KC);
    U256 R = u_sub(Y, KC);
    const bool neg = u_neg_sign(R);
    if (neg) R = u_neg(R);
    U256 sum = u_zero();
    sum.w[3] = 1ull << (kFrac - 192);  // 1.0
    U256 term = sum;
    for (uint32_t n = 1; n < 64; ++n) {
        term = u_div_small(u_mul_fix(term, R), n);
        if (u_is_zero(term)) break;
        sum = (neg && (n & 1u)) ? u_sub(sum, term) : u_add(sum, term);
    }
    U256 Tj;
    const int j = k & 63;
    for (int i = 0; i < 4; ++i) Tj.w[i] = T.exp_tfix[j][i];
    *M = u_mul_fix(Tj, sum);
    *m = k >> 6;  // floor(k / 64)
}

GEO_CR_FN int exp_reduce_k(double x) {
    const double t = x * tables().inv_ln2_64;
    return (int)rint(t);
}

// exp(r) - 1 as double-double, |r| < 0.0062 given as r_hi + r_lo.
GEO_CR_FN DD expm1_poly(DD r) {
    const Tables &T = tables();
    const double y = r.hi;
    double tail = T.c_tail[5];
    for (int i = 4; i >= 0; --i) tail = fma(y, tail, T.c_tail[i]);  // sum_{n>=6} r^(n-6)/n!
    DD s = dd_mul_d(r, tail);                                          // r * tail
    for (int i = 3; i >= 0; --i) s = dd_mul(r, dd_add(DD{T.c_hi[i], T.c_lo[i]}, s));
    // s = sum_{n>=2} r^(n-1)/n! = r/2 + r^2/6 + ...; exp(r) - 1 = r + r s
    return dd_add(r, dd_mul(r, s));
}

// Argument reduction: r = x - k ln2/64 as double-double.
GEO_CR_FN DD exp_reduce(double x, int k) {
    const Tables &T = tables();
    const double kd = (double)k;
    const double r1 = fma(-kd, T.l1, x);  // exact
    const DD p2 = two_prod(kd, T.l2);
    DD s = two_sum(r1, -p2.hi);
    s.lo = (s.lo - p2.lo) - kd * T.l3;
    return fast_two_sum(s.hi, s.lo);
}

GEO_CR_NOINLINE double exp_accurate(double x) {
    U256 M;
    int m;
    exp_fixed(x, exp_reduce_k(x), &M, &m);
    return u_round(M, m, false);
}

// Correctly rounded exp(x).
GEO_CR_FN double exp(double x) {
    const double ax = fabs(x);
    if (!(ax <= 708.0)) {
        if (x != x) return x + x;
        if (x > 710.0) return INFINITY;
        if (x < -746.0) return 0.0;
        return exp_accurate(x);
    }
    if (ax < 0x1p-54) return 1.0;
    const int k = exp_reduce_k(x);
    const DD r = exp_reduce(x, k);
    const DD p = expm1_poly(r);
    const Tables &T = tables();
    const DD t{T.exp_t[k & 63][0], T.exp_t[k & 63][1]};
    const DD v = dd_add(t, dd_mul(t, p));
    double out;
    if (ziv_round(v, 0x1p-80 * v.hi, &out)) return out * pow2(k >> 6);
    return exp_accurate(x);
}

GEO_CR_NOINLINE double tanh_accurate(double x) {
    const double ax = fabs(x);
    const double y = 2.0 * ax;
    U256 M;
    int m;
    exp_fixed(y, exp_reduce_k(y), &M, &m);  // exp(2|x|) = M * 2^(m - 232), m in [-1, 56]
    U256 one = u_zero();
    const int pos = kFrac - m;  // 2^-m in M's scale
    one.w[pos >> 6] = 1ull << (pos & 63);
    const U256 num = u_sub(M, one), den = u_add(M, one);
    // Q = floor(num * 2^233 / den): one more bit than the fraction, then the sticky remainder.
    U256 rem = num, q = u_zero();
    for (int i = 0; i < kFrac + 1; ++i) {
        rem = u_shl1(rem);
        q = u_shl1(q);
        if (u_ge(rem, den)) {
            rem = u_sub(rem, den);
            q.w[0] |= 1u;
        }
    }
    const double t = u_round(q, -1, !u_is_zero(rem));
    return x < 0 ? -t : t;
}

// Correctly rounded tanh(x).
GEO_CR_FN double tanh(double x) {
    const double ax = fabs(x);
    if (!(ax < 19.1)) {
        if (x != x) return x + x;
        return x < 0 ? -1.0 : 1.0;
    }
    if (ax < 0x1p-27) return x;
    const double y = 2.0 * ax;
    const int k = exp_reduce_k(y);
    const DD r = exp_reduce(y, k);
    const DD p = expm1_poly(r);
    DD em1;
    if (k == 0) {
        em1 = p;
    } else {
        const Tables &T = tables();
        const DD t{T.exp_t[k & 63][0], T.exp_t[k & 63][1]};
        const DD v = dd_add(t, dd_mul(t, p));
        const double sc = pow2(k >> 6);
        em1 = dd_add(DD{v.hi * sc, v.lo * sc}, DD{-1.0, 0.0});
    }
    const DD q = dd_div(em1, dd_add(em1, DD{2.0, 0.0}));
    double out;
    if (ziv_round(q, 0x1p-75 * q.hi, &out)) return x < 0 ? -out : out;
    return tanh_accurate(x);
}

}  // namespace cr
}  // namespace geo
