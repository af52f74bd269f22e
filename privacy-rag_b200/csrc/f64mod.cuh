// Exact modular arithmetic on the FP64 pipe, for primes q < 2^50.
//
// A 64-bit integer residue product costs several 32-bit multiply-adds on the SM's integer
// pipe, while B200 runs 64-bit floating-point add / multiply / FMA on a pipe of its own at 64
// lanes per SM per clock.  For primes below 2^50 a residue product can be formed EXACTLY in
// doubles, with residues held as integer-valued doubles (signed, centred representatives):
//
//  * TwoProduct (Dekker 1971; in its FMA form, Ogita, Rump and Oishi, "Accurate sum and dot
//    product", 2005): h = fl(y w) and l = fma(y, w, -h) satisfy y w = h + l exactly;
//  * the quotient estimate k = rint(y w / q) from the precomputed wq = fl(w / q) (the
//    floating-point form of Shoup's precomputed quotient), rounded to an integer by adding and
//    subtracting 1.5 * 2^52: for |x| < 2^51 the sum lies in (2^52, 2^53), where consecutive
//    doubles are 1 apart, so one round-to-nearest addition rounds x to an integer;
//  * r = fma(-k, q, h) + l: h - k q is an integer of magnitude below 2^53 and the FMA rounds
//    it once, so it is exact, and so is the final sum.
//
// This is the floating-point modular multiplication of the GPU literature (e.g. Emmart, Zheng
// and Weems, "Faster modular exponentiation using double precision floating point arithmetic
// on the GPU", ARITH 2018), restated for NTT butterflies.  Bounds used by the callers
// (q < 2^50, twiddles centred, |w| <= q/2, |wq| <= 1/2):
//   mulmod(y, w):   |y| < 2^52  ->  |k - y w / q| <= 1/2 + 1/8  ->  |r| <= 0.75 q
//   reduce(v):      |v| < 2^52  ->  |k - v / q| <= 1/2 + 1/(2q)  ->  |r| <= (q + 1) / 2
// and every sum formed stays below 2^53 in magnitude, so it is exact.
//
// The explicit round-to-nearest intrinsics keep the compiler from contracting or reordering
// any of these steps; the host build (tests/emu) uses std::fma and is compiled without
// floating-point contraction, so both run the identical IEEE operations.
#pragma once
#include <cstdint>
#include <cstring>
#if !defined(__CUDA_ARCH__)
#include <cmath>
#endif

#include "arith.cuh"

namespace bfvgpu {

constexpr double kF64Round = 6755399441055744.0;  // 1.5 * 2^52
constexpr double kF64Two52 = 4503599627370496.0;  // 2^52
constexpr uint64_t kF64Two52Bits = 0x4330000000000000ull;
constexpr uint64_t kF64MaxPrime = uint64_t(1) << 50;

BFV_HD double f64_mul(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __dmul_rn(a, b);
#else
  return a * b;
#endif
}
BFV_HD double f64_add(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __dadd_rn(a, b);
#else
  return a + b;
#endif
}
BFV_HD double f64_sub(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __dsub_rn(a, b);
#else
  return a - b;
#endif
}
BFV_HD double f64_fma(double a, double b, double c) {
#if defined(__CUDA_ARCH__)
  return __fma_rn(a, b, c);
#else
  return std::fma(a, b, c);
#endif
}
BFV_HD uint64_t f64_bits(double d) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(d);
#else
  uint64_t u;
  std::memcpy(&u, &d, 8);
  return u;
#endif
}
BFV_HD double f64_from_bits(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)u);
#else
  double d;
  std::memcpy(&d, &u, 8);
  return d;
#endif
}

// x < 2^52 as a double (exact): the bit pattern of 2^52 + x, minus 2^52.
BFV_HD double u64_to_f64(uint64_t x) { return f64_sub(f64_from_bits(x | kF64Two52Bits), kF64Two52); }
// An integer-valued double in [0, 2^52) back to its integer.
BFV_HD uint64_t f64_to_u64(double v) { return f64_bits(f64_add(v, kF64Two52)) - kF64Two52Bits; }

// y w mod q as a centred representative, |r| <= 0.75 q (|y| < 2^52, |w| <= q/2, wq = fl(w/q)).
BFV_HD double mulmod_f64(double y, double w, double wq, double q) {
  const double h = f64_mul(y, w);
  const double l = f64_fma(y, w, -h);
  const double k = f64_sub(f64_fma(y, wq, kF64Round), kF64Round);
  return f64_add(f64_fma(-k, q, h), l);
}

// y w mod q for an operand without a precomputed quotient (Barrett's form: the quotient from
// fl(1/q)), for |y| <= (q + 1)/2 and 0 <= w < q: |y w| < q^2 / 2, so |l| <= |y w| 2^-53 and
// |h fl(1/q) - y w / q| <= q 2^-53 <= 1/8; with the rounding, |k - y w / q| <= 5/8 and
// |r| <= 0.75 q.
BFV_HD double mulmod_f64_barrett(double y, double w, double q, double qinv) {
  const double h = f64_mul(y, w);
  const double l = f64_fma(y, w, -h);
  const double k = f64_sub(f64_fma(h, qinv, kF64Round), kF64Round);
  return f64_add(f64_fma(-k, q, h), l);
}

// v mod q as a centred representative, |r| <= (q + 1) / 2 (|v| < 2^52, qinv = fl(1/q)).
BFV_HD double reduce_f64(double v, double q, double qinv) {
  const double k = f64_sub(f64_fma(v, qinv, kF64Round), kF64Round);
  return f64_fma(-k, q, v);
}

// v mod q in [0, q) as an integer (|v| < 2^52).
BFV_HD uint64_t canon_f64(double v, double q, double qinv) {
  double r = reduce_f64(v, q, qinv);
  if (r < 0.0) r = f64_add(r, q);
  return f64_to_u64(r);
}

// Centred double of a canonical residue w < q (|w_c| <= (q-1)/2).
BFV_HD double centred_f64(uint64_t w, uint64_t q) {
  return w > q / 2 ? -(double)(q - w) : (double)w;
}

// Host setup: the FP64 constants of a prime's record (its integer fields already set) -- the
// centred operands with their quotients fl(v_c / q), by IEEE double division (correctly
// rounded).  Primes of 2^50 and above keep f64 = 0 and compute on the integer pipe.
inline void f64_fill_modulus(Modulus& m) {
  if (m.q >= kF64MaxPrime) return;
  const double qd = (double)m.q;
  m.f64 = 1;
  m.f64_qinv = 1.0 / qd;
  m.f64_invn = centred_f64(m.invn, m.q);
  m.f64_invn_q = m.f64_invn / qd;
  m.f64_inv_special = centred_f64(m.inv_special, m.q);
  m.f64_inv_special_q = m.f64_inv_special / qd;
}

}  // namespace bfvgpu
