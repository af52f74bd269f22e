// Modular arithmetic for 60-bit RNS primes (q < 2^62), usable on host and device.
//
// Restated from the published methods, not from any library source:
//  * Shoup multiplication by a fixed operand w with w' = floor(w 2^64 / q)
//    (Harvey, "Faster arithmetic for number-theoretic transforms", 2014, Alg. 2);
//    the reference uses it for NTT twiddles (IV1/experiments/matrix_gpu/matrix.cu:44-46).
//  * Barrett (1986) reduction of a 128-bit value with r = floor((2^128-1)/q), the
//    quotient assembled exactly from 64-bit partial products; the reference uses the
//    same reduction for dyadic products (matrix.cu:37-43).  Because every carry of the
//    middle column is kept, the estimate is off by at most one for ANY 128-bit input,
//    so it also reduces lazily accumulated sums of products.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define BFV_HD __host__ __device__ __forceinline__
#else
#define BFV_HD inline
#endif

namespace bfvgpu {

BFV_HD uint64_t mulhi64(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
  return __umul64hi(a, b);
#else
  return (uint64_t)(((unsigned __int128)a * b) >> 64);
#endif
}

// Per-prime constants, 128 bytes, one per prime of a context.
struct Modulus {
  uint64_t q;
  uint64_t r0, r1;                      // floor((2^128-1)/q) = r1*2^64 + r0
  uint64_t invn, invn_q;                // n^-1 mod q, Shoup pair
  uint64_t inv_special, inv_special_q;  // q_special^-1 mod q (data primes), Shoup pair
  uint64_t half_special_mod;            // floor(q_special/2) mod q
  uint64_t delta, delta_q;              // floor(Q/t) mod q (data primes), Shoup pair
  // FP64-pipe constants (f64mod.cuh), set for primes below 2^50 when the context computes on
  // that pipe (f64 != 0); doubles are centred residues with their quotients fl(v / q)
  uint64_t f64;
  double f64_qinv;                      // fl(1/q)
  double f64_invn, f64_invn_q;          // n^-1
  double f64_inv_special, f64_inv_special_q;  // q_special^-1 (data primes)
};
static_assert(sizeof(Modulus) == 128, "Modulus is one 128-byte line");

BFV_HD uint64_t add_mod(uint64_t a, uint64_t b, uint64_t q) {
  const uint64_t x = a + b;
  return x >= q ? x - q : x;
}
BFV_HD uint64_t sub_mod(uint64_t a, uint64_t b, uint64_t q) {
  const uint64_t x = a + q - b;
  return x >= q ? x - q : x;
}
BFV_HD uint64_t neg_mod(uint64_t a, uint64_t q) { return a ? q - a : 0; }

// a*w mod q in [0, 2q) for any a < 2^64 (lazy Shoup).
BFV_HD uint64_t shoup_lazy(uint64_t a, uint64_t w, uint64_t wq, uint64_t q) {
  return a * w - mulhi64(a, wq) * q;
}
BFV_HD uint64_t shoup(uint64_t a, uint64_t w, uint64_t wq, uint64_t q) {
  const uint64_t r = shoup_lazy(a, w, wq, q);
  return r >= q ? r - q : r;
}

// (hi*2^64 + lo) mod q for any 128-bit value x.  Barrett: with r = floor((2^128-1)/q)
// = r1*2^64 + r0, the product x*r splits into the columns 2^128 (hi*r1), 2^64
// (hi*r0 + lo*r1, plus the high word of lo*r0) and 2^0.  The quotient estimate
// floor(x*r / 2^128) is hi*r1 plus the high words of the 2^64-column terms plus the
// carries out of summing their low words; it falls short of floor(x/q) by at most one,
// which the final conditional subtraction corrects.
BFV_HD uint64_t reduce128(uint64_t lo, uint64_t hi, const Modulus& m) {
  const uint64_t lo_r1 = lo * m.r1, hi_r0 = hi * m.r0;
  uint64_t column = mulhi64(lo, m.r0) + lo_r1;
  uint64_t carries = column < lo_r1;
  column += hi_r0;
  carries += column < hi_r0;
  const uint64_t qhat = hi * m.r1 + mulhi64(lo, m.r1) + mulhi64(hi, m.r0) + carries;
  const uint64_t rem = lo - qhat * m.q;
  return rem >= m.q ? rem - m.q : rem;
}

// a*b mod q, a*b < 2^128.
BFV_HD uint64_t mul_mod(uint64_t a, uint64_t b, const Modulus& m) {
  return reduce128(a * b, mulhi64(a, b), m);
}

// Shoup companion floor(v 2^64 / q) of v < q, by exact division: v 2^64 - r (r = v 2^64 mod q)
// is a multiple of q, so the quotient is -r . q^-1 mod 2^64 (q odd).
BFV_HD uint64_t shoup_companion(uint64_t v, const Modulus& m) {
  const uint64_t r = reduce128(0, v, m);
  uint64_t inv = m.q;  // q^-1 mod 2^64 by Newton's iteration (3 -> 96 correct bits)
#pragma unroll
  for (int it = 0; it < 5; ++it) inv *= 2 - m.q * inv;
  return (uint64_t(0) - r) * inv;
}

// v mod q for v < 2^64 with the 64-bit Barrett ratio floor(2^64/q) = r1.
BFV_HD uint64_t reduce64(uint64_t v, const Modulus& m) {
  const uint64_t r = v - mulhi64(v, m.r1) * m.q;
  return r >= m.q ? r - m.q : r;
}

// 128-bit accumulator for lazy sums of products of canonical residues.
struct Acc128 {
  uint64_t lo = 0, hi = 0;
  BFV_HD void mac(uint64_t a, uint64_t b) {
    const uint64_t pl = a * b, ph = mulhi64(a, b);
    lo += pl;
    hi += ph + (lo < pl);
  }
  BFV_HD uint64_t reduce(const Modulus& m) const { return reduce128(lo, hi, m); }
  BFV_HD void fold(const Modulus& m) {
    lo = reduce128(lo, hi, m);
    hi = 0;
  }
};

// Scaled plaintext coefficient for BFV: m*floor(Q/t) + floor(((Q mod t)*m + half)/t)
// mod q, with t a power of two (log2 t = tlog) or t < 2^32.
BFV_HD uint64_t scale_plain_coeff(uint64_t mval, uint64_t q_mod_t, uint64_t half, uint64_t t,
                                  int tlog, const Modulus& m) {
  uint64_t fix;
  if (tlog > 0) {
    const uint64_t lo = mval * q_mod_t, hi = mulhi64(mval, q_mod_t);
    const uint64_t added = lo + half;
    const uint64_t h2 = hi + (added < lo);
    fix = (tlog >= 64) ? h2 : ((h2 << (64 - tlog)) | (added >> tlog));
  } else {
    fix = (mval * q_mod_t + half) / t;  // t < 2^32 and mval, q_mod_t < t
  }
  const uint64_t base = shoup(mval >= m.q ? mval % m.q : mval, m.delta, m.delta_q, m.q);
  return add_mod(base, fix >= m.q ? fix % m.q : fix, m.q);
}

}  // namespace bfvgpu
