// Per-thread-block bodies of the BFV kernels, written against an executor (ntt_core.cuh)
// so the same code runs as a CUDA thread block (BlockExec) and, for the CPU pre-checks
// in tests/emu, as a host loop over the block's work units (HostExec).  The __global__
// wrappers in kernels.cu only pick the block index and shared memory.
//
// Reference behaviour restated here (IV1 = implementation_v1/):
//   op_lift_ntt ...... `lift` + forward stages (IV1/experiments/matrix_gpu/matrix.cu:48-51, :96)
//   op_mac_intt ...... `product` + inverse stages (matrix.cu:59-63, :96) with the sub_plain
//                      mask (IV1/native/src/bfv_matrix.inc:215-219) and Enc(0) add (:220-227)
//   op_ks_main ....... apply_galois (IV1/experiments/keyswitch_full_gpu/seal_adapter.cpp:50),
//                      `decompose`, forward stages, `product`, inverse stages (switch.cu:92-102)
//   op_ks_moddown .... `moddown` (switch.cu:103-111)
//   op_enc0_x ........ PublicZero::evaluate up to noise_add (IV1/native/gpu/enc0/enc0.cu:74-80, :129-134)
//   op_client_phase .. NTT, `client_dyadic`, INTT (IV1/native/gpu/client_phase/ntt.cu:96-98, :186-194)
//   op_token_* ....... `lift`, `accumulate`, inverse stages, `add_shift`
//                      (IV1/experiments/resident_token_gpu/resident.cu:71-107)
//   crt_target ....... rns_coefficient (IV1/native/src/bfv.cpp:138-147) in fixed-width limbs
#pragma once
#include "layout.cuh"
#include "ntt_core.cuh"

namespace bfvgpu {

// Largest radix (log2) of the register butterfly units: radix-8 passes keep a unit in
// ~16 registers, which lets 2-3 blocks share an SM (measured fastest on B200).
constexpr int kMaxRadix = 3;

// Read-only global load on the non-coherent path, for an operand that no kernel of the launch
// writes: a transform's storer uses it for its epilogue operand so that the compiler may issue
// the load ahead of the pass's stores to the output (which it cannot prove do not alias).
BFV_HD uint64_t ldro(const uint64_t* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(reinterpret_cast<const unsigned long long*>(p));
#else
  return *p;
#endif
}
BFV_HD ulonglong2 ldro_pair(const ulonglong2* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}
BFV_HD double2 ldro2(const double2* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2,
// issued by one thread of the block; the block's demand loads of that range then hit L2
// instead of waiting a DRAM round trip each.  No effect on the host.
BFV_HD void block_prefetch_l2(const void* p, uint32_t bytes) {
#if defined(__CUDA_ARCH__)
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
#else
  (void)p;
  (void)bytes;
#endif
}


// Divide-and-round by the special prime q_s (last prime) of one coefficient:
// (x_p - ((x_s + floor(q_s/2)) mod q_s mod q_p - floor(q_s/2) mod q_p)) * q_s^-1 mod q_p.
BFV_HD uint64_t moddown_elem(uint64_t xv, uint64_t xs, const Modulus& mp, const Modulus& ms) {
  const uint64_t last = add_mod(xs, ms.q >> 1, ms.q);
  const uint64_t lastp = reduce64(last, mp);
  const uint64_t corr = sub_mod(lastp, mp.half_special_mod, mp.q);
  return shoup(sub_mod(xv, corr, mp.q), mp.inv_special, mp.inv_special_q, mp.q);
}

struct ProtectArgs {
  const uint64_t* mask;    // [groups][n] ring-59 words, or null
  const uint64_t* enc0_x;  // [groups][2][k][n] pre-moddown Enc(0) polys, or null
  uint64_t q_mod_t, upper_half, t;
  int tlog;
};

// ---- batched transform: block = one poly -----------------------------------------------
// Primes whose record has f64 set transform on the FP64 pipe (one limb per block only).
template <int LOGN, class Ex>
BFV_HD void op_ntt(const Ex& ex, uint64_t* s, uint64_t blk, bool inverse, uint64_t* data, uint32_t prime_count,
                   uint32_t prime_offset, const Modulus* mods, const ulonglong2* fwd, const ulonglong2* inv,
                   const double2* fwd64, const double2* inv64) {
  const uint32_t p = prime_offset + (uint32_t)(blk % prime_count);
  const Modulus m = mods[p];
  uint64_t* a = data + (blk << LOGN);
  if constexpr (!Ex::kSplit) {
    if (m.f64) {
      const F64Prime fp = f64_prime(m);
      auto ldf = [a](int i) { return u64_to_f64(a[i]); };
      auto stf = [a, fp](int i, double v) { a[i] = canon_f64(v, fp.q, fp.qinv); };
      if (inverse)
        ntt_inverse_f64<LOGN, kMaxRadix>(ex, s, inv64 + ((size_t)p << LOGN), m, ldf, stf);
      else
        ntt_forward_f64<LOGN, kMaxRadix>(ex, s, fwd64 + ((size_t)p << LOGN), m, ldf, stf);
      return;
    }
  }
  auto ld = [a](int i) { return a[i]; };
  auto st = [a](int i, uint64_t v) { a[i] = v; };
  if (inverse)
    ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
  else
    ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
}

// ---- weight lift + NTT: block = (weight block b, data prime p) --------------------------
template <int LOGN, class Ex>
BFV_HD void op_lift_ntt(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* ring, uint64_t* out, uint32_t dk,
                        const Modulus* mods, const ulonglong2* fwd) {
  const uint64_t b = blk / dk;
  const uint32_t p = (uint32_t)(blk % dk);
  const Modulus m = mods[p];
  const uint64_t* r = ring + (b << LOGN);
  uint64_t* o = out + ((b * dk + p) << LOGN);
  const uint64_t adjust = m.q - (uint64_t(1) << 59);
  auto ld = [r, adjust](int i) {
    const uint64_t v = r[i];
    return v + (adjust & (uint64_t(0) - (v >> 58)));
  };
  auto st = [o](int i, uint64_t v) { o[i] = v; };
  ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
}

// ---- product over input blocks + INTT (+ mask, + Enc(0)): block = (group g, c, p) -------
template <int LOGN, class Ex>
BFV_HD void op_mac_intt(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* in, const uint64_t* w, uint64_t* out,
                        uint32_t inputs, uint32_t k, uint32_t dk, const Modulus* mods, const ulonglong2* inv,
                        const ProtectArgs& prot) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t g = blk / (2 * dk);
  const uint32_t cp = (uint32_t)(blk % (2 * dk)), c = cp / dk, p = cp % dk;
  const Modulus m = mods[p];
  const uint64_t* in_cp = in + (uint64_t)cp * N;
  const uint64_t in_stride = 2 * (uint64_t)dk * N;
  const uint64_t* w_gp = w + ((g * inputs) * dk + p) * N;
  const uint64_t w_stride = (uint64_t)dk * N;
  auto ld = [=](int i) {
    Acc128 acc;
    for (uint32_t b = 0; b < inputs; ++b) {
      acc.mac(in_cp[b * in_stride + i], w_gp[b * w_stride + i]);
      if ((b & 127u) == 127u) acc.fold(m);
    }
    return acc.reduce(m);
  };
  uint64_t* o = out + ((g * 2 + c) * dk + p) * N;
  const uint64_t* x = prot.enc0_x ? prot.enc0_x + g * 2 * k * N : nullptr;
  const uint64_t* mask = (prot.mask && c == 0) ? prot.mask + g * N : nullptr;
  const Modulus* ms = mods + (k - 1);
  const ProtectArgs pa = prot;
  auto st = [=](int i, uint64_t v) {
    if (x) {
      const uint64_t xv = ldro(x + ((uint64_t)c * k + p) * N + i);
      const uint64_t xs = ldro(x + ((uint64_t)c * k + k - 1) * N + i);
      v = add_mod(v, moddown_elem(xv, xs, m, *ms), m.q);
    }
    if (mask) v = sub_mod(v, scale_plain_coeff(ldro(mask + i), pa.q_mod_t, pa.upper_half, pa.t, pa.tlog, m), m.q);
    o[i] = v;
  };
  ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
}

// ---- Galois automorphism + keyswitch main part: block = (ciphertext, key-level prime p) --
// For each digit j (data prime j of c1) the coefficient-domain digit is built in
// natural order from the UNPERMUTED c1, pre-negated where the automorphism will negate
// it, so that the mod-q_p automorphism applied afterwards as an NTT-slot permutation
// yields exactly the reference's digit: sigma(c1)_j with its "q_j - x" negation, then
// reduced into q_p.  acc [ct][2][k][n] receives INTT(sum_j digit_j . key_j).
template <int LOGN, class Ex>
BFV_HD void op_ks_main(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* cts, const uint64_t* key,
                       uint64_t* acc, uint32_t elt, uint32_t k, uint32_t dk, const Modulus* mods, const uint64_t* qjp,
                       const ulonglong2* fwd, const ulonglong2* inv, const double2* fwd64, const double2* inv64) {
  constexpr int N = 1 << LOGN;
  const uint64_t ct = blk / k;
  const uint32_t p = (uint32_t)(blk % k);
  const Modulus m = mods[p];
  const uint64_t* c1 = cts + (ct * 2 * dk + dk) * (uint64_t)N;
  uint64_t* acc0 = acc + ((ct * 2 + 0) * k + p) * (uint64_t)N;
  uint64_t* acc1 = acc + ((ct * 2 + 1) * k + p) * (uint64_t)N;
  const uint32_t mask2n = 2u * N - 1u;
  if constexpr (!Ex::kSplit) {
    if (m.f64) {
      // FP64 form: the digit transforms and both inverse transforms on the FP64 pipe; the key
      // products in Barrett's form (the raw key words carry no quotients) on the gathered
      // slot reduced to |v| <= (q+1)/2, accumulated as doubles in acc (at most 0.75 q per
      // product, folded every four digits), made canonical by the inverse transforms' storer
      const F64Prime fp = f64_prime(m);
      double* d = reinterpret_cast<double*>(s);
      for (uint32_t j = 0; j < dk; ++j) {
        const uint64_t* src = c1 + (uint64_t)j * N;
        const uint64_t adj = qjp[j * k + p];
        const bool reduce = mods[j].q > m.q;
        auto ld = [=](int i) {
          const uint64_t x = src[i];
          uint64_t y = reduce ? reduce64(x, m) : x;
          const bool neg = (((uint32_t)i * elt) & mask2n) >= (uint32_t)N;
          if (neg && x) y = sub_mod(y, adj, m.q);
          return u64_to_f64(y);
        };
        auto st = [d](int i, double v) { d[spad(i)] = v; };
        ntt_forward_f64<LOGN, kMaxRadix, false>(ex, s, fwd64 + ((size_t)p << LOGN), m, ld, st);
        const uint64_t* k0 = key + ((uint64_t)(j * 2 + 0) * k + p) * N;
        const uint64_t* k1 = key + ((uint64_t)(j * 2 + 1) * k + p) * N;
        const bool fold = (j & 3) == 3 && j + 1 < dk;
        ex.run(N, [&](int i) {
          const double v = reduce_f64(d[spad(galois_slot(i, elt, LOGN))], fp.q, fp.qinv);
          double a = mulmod_f64_barrett(v, u64_to_f64(k0[i]), fp.q, fp.qinv);
          double b = mulmod_f64_barrett(v, u64_to_f64(k1[i]), fp.q, fp.qinv);
          if (j) {
            a = f64_add(a, f64_from_bits(acc0[i]));
            b = f64_add(b, f64_from_bits(acc1[i]));
          }
          if (fold) {
            a = reduce_f64(a, fp.q, fp.qinv);
            b = reduce_f64(b, fp.q, fp.qinv);
          }
          acc0[i] = f64_bits(a);
          acc1[i] = f64_bits(b);
        });
        ex.sync();
      }
      for (int c = 0; c < 2; ++c) {
        uint64_t* a = c ? acc1 : acc0;
        auto ld = [a](int i) { return f64_from_bits(a[i]); };
        auto st = [a, fp](int i, double v) { a[i] = canon_f64(v, fp.q, fp.qinv); };
        ntt_inverse_f64<LOGN, kMaxRadix>(ex, s, inv64 + ((size_t)p << LOGN), m, ld, st);
      }
      return;
    }
  }
  for (uint32_t j = 0; j < dk; ++j) {
    const uint64_t* src = c1 + (uint64_t)j * N;
    const uint64_t adj = qjp[j * k + p];
    const bool reduce = mods[j].q > m.q;
    auto ld = [=](int i) {
      const uint64_t x = src[i];
      uint64_t y = reduce ? reduce64(x, m) : x;
      const bool neg = (((uint32_t)i * elt) & mask2n) >= (uint32_t)N;
      if (neg && x) y = sub_mod(y, adj, m.q);
      return y;
    };
    auto st = [s](int i, uint64_t v) { s[spad(i)] = v; };
    ntt_forward<LOGN, kMaxRadix, false>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
    const uint64_t* k0 = key + ((uint64_t)(j * 2 + 0) * k + p) * N;
    const uint64_t* k1 = key + ((uint64_t)(j * 2 + 1) * k + p) * N;
    ex.run(N, [&](int i) {
      const uint64_t v = s[spad(galois_slot(i, elt, LOGN))];
      const uint64_t a = mul_mod(v, k0[i], m), b = mul_mod(v, k1[i], m);
      if (j == 0) {
        acc0[i] = a;
        acc1[i] = b;
      } else {
        acc0[i] = add_mod(acc0[i], a, m.q);
        acc1[i] = add_mod(acc1[i], b, m.q);
      }
    });
    ex.sync();
  }
  for (int c = 0; c < 2; ++c) {
    uint64_t* a = c ? acc1 : acc0;
    auto ld = [a](int i) { return a[i]; };
    auto st = [a](int i, uint64_t v) { a[i] = v; };
    ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
  }
}

// out_c[p] = moddown(acc_c)[p] (+ sigma(c0)[p] for c = 0).  Block (ct, data prime p);
// the c0 limb is staged unpadded in shared memory so the automorphism is a gather there.
template <int LOGN, class Ex>
BFV_HD void op_ks_moddown(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* acc, const uint64_t* cts,
                          uint64_t* out, uint32_t ginv, uint32_t k, uint32_t dk, const Modulus* mods) {
  constexpr int N = 1 << LOGN;
  const uint64_t ct = blk / dk;
  const uint32_t p = (uint32_t)(blk % dk);
  const Modulus m = mods[p], ms = mods[k - 1];
  const uint64_t* c0 = cts + (ct * 2 * dk + p) * (uint64_t)N;
  ex.run(N, [&](int i) { s[i] = c0[i]; });
  ex.sync();
  const uint32_t mask2n = 2u * N - 1u;
  ex.run(N, [&](int i) {
    const uint32_t src = ((uint32_t)i * ginv) & mask2n;
    const uint64_t w = src < (uint32_t)N ? s[src] : neg_mod(s[src - N], m.q);
    for (int c = 0; c < 2; ++c) {
      const uint64_t* a = acc + ((ct * 2 + c) * k) * (uint64_t)N;
      uint64_t v = moddown_elem(a[(uint64_t)p * N + i], a[(uint64_t)(k - 1) * N + i], m, ms);
      if (c == 0) v = add_mod(v, w, m.q);
      out[((ct * 2 + c) * dk + p) * (uint64_t)N + i] = v;
    }
  });
  ex.sync();
}

// ---- hoisted rotations: many Galois elements over one ciphertext batch -------------------
// With slot(i) the NTT-slot permutation of X -> X^g, the reference's keyswitch product
// acc_c[i] = sum_j NTT(digit_j)[i] key_j[c][i] is acc_c[i] = A_c[slot(i)] where
//   A_c[s] = sum_j NTT(b_j)[s] Kt_j[c][s],   Kt_j[c][s] = key_j[c][slot^-1(s)]
// and b_j is the pre-negated digit of op_ks_main.  Without zero coefficients in c1,
// NTT(b_j) = Y_j - (q_j mod q_p) W with Y_j = NTT(c1_j mod q_p) (independent of g) and
// W = NTT(neg_g) (neg_g[s] = 1 where X -> X^g negates coefficient s), so
//   A_c[s] = sum_j Y_j[s] Kt_j[c][s] - Ct_c[s],   Ct_c[s] = W[s] sum_j (q_j mod q_p) Kt_j[c][s].
// INTT(A_c permuted by slot) = sigma_g(INTT(A_c)), and divide-and-round by the odd special
// prime commutes with sigma_g, so the output is sigma_g(moddown(INTT(A_c)) + [c=0] c0):
// the automorphism becomes one coefficient permutation at the very end.

// Y [ct][dk][k][n]: hoisted digit transforms; zflag[ct] set if c1 has a zero coefficient.
template <int LOGN, class Ex>
BFV_HD void op_ks_hoist(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* cts, uint64_t* Y, uint32_t* zflag,
                        uint32_t k, uint32_t dk, const Modulus* mods, const ulonglong2* fwd) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t ct = blk / ((uint64_t)dk * k);
  const uint32_t j = (uint32_t)((blk / k) % dk), p = (uint32_t)(blk % k);
  const Modulus m = mods[p];
  const uint64_t* src = cts + (ct * 2 * dk + dk + j) * N;
  uint64_t* y = Y + ((ct * dk + j) * k + p) * N;
  const bool reduce = mods[j].q > m.q;
  uint32_t zero = 0;
  auto ld = [&](int i) {
    const uint64_t x = src[i];
    zero |= (x == 0);
    return reduce ? reduce64(x, m) : x;
  };
  auto st = [y](int i, uint64_t v) { y[i] = v; };
  ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
  if (zero && p == 0) {
#if defined(__CUDA_ARCH__)
    atomicOr(zflag + ct, 1u);
#else
    zflag[ct] = 1;
#endif
  }
}

// Key preparation for a batch of keys, in two kernels, into the prepared layout of
// layout.cuh: Kt as {key word, Shoup companion} pairs (so the rotation's key product is one
// lazy Shoup multiplication per digit) -- for a prime whose record has f64 set, as the bit
// patterns of {centred key word, fl(word / q)}, the operand pair of mulmod_f64 -- then Ct.
// (1) block (r, p): W = NTT_p(neg_g) written to Ct[c = 0][p] of key r.
template <int LOGN, class Ex>
BFV_HD void op_ks_negntt(const Ex& ex, uint64_t* s, uint64_t blk, uint64_t* prepared, uint64_t prepared_words,
                         const uint32_t* elts, uint32_t k, uint32_t dk, const Modulus* mods, const ulonglong2* fwd) {
  constexpr int N = 1 << LOGN;
  const uint64_t r = blk / k;
  const uint32_t p = (uint32_t)(blk % k);
  const Modulus m = mods[p];
  const uint32_t elt = elts[r], mask2n = 2u * N - 1u;
  uint64_t* w = prepared + r * prepared_words + ks_ct_offset(k, dk, N) + (uint64_t)p * N;
  auto ld = [=](int i) { return (uint64_t)((((uint32_t)i * elt) & mask2n) >= (uint32_t)N ? 1 : 0); };
  auto st = [w](int i, uint64_t v) { w[i] = v; };
  ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
}

// (2) one (key r, prime p, slot s) per work item: Kt_j[c][p][s] = key_j[c][p][slot^-1(s)],
// Ct[c][p][s] = W[s] * sum_j (q_j mod q_p) Kt_j[c][p][s].
BFV_HD void ks_keyperm_item(uint64_t item, const uint64_t* keys, uint64_t* prepared, uint64_t prepared_words,
                            const uint32_t* ginvs, int logn, uint32_t k, uint32_t dk, const Modulus* mods,
                            const uint64_t* qjp) {
  const uint64_t N = uint64_t(1) << logn;
  const uint64_t r = item / (k * N);
  const uint32_t p = (uint32_t)((item >> logn) % k);
  const int sl = (int)(item & (N - 1));
  const Modulus& m = mods[p];
  const uint64_t* key = keys + r * (uint64_t)dk * 2 * k * N;
  ulonglong2* Kt = reinterpret_cast<ulonglong2*>(prepared + r * prepared_words);
  uint64_t* Ct = prepared + r * prepared_words + ks_ct_offset(k, dk, N);
  const int from = galois_slot(sl, ginvs[r], logn);
  const uint64_t w = Ct[(uint64_t)p * N + sl];  // NTT(neg_g), overwritten below
  for (uint32_t c = 0; c < 2; ++c) {
    uint64_t sum = 0;
    for (uint32_t j = 0; j < dk; ++j) {
      const uint64_t v = key[((uint64_t)(j * 2 + c) * k + p) * N + from];
      ulonglong2 kv;
      if (m.f64) {
        const double vc = centred_f64(v, m.q);
#if defined(__CUDA_ARCH__)
        const double vq = __ddiv_rn(vc, u64_to_f64(m.q));
#else
        const double vq = vc / (double)m.q;
#endif
        kv.x = f64_bits(vc);
        kv.y = f64_bits(vq);
      } else {
        kv.x = v;
        kv.y = shoup_companion(v, m);
      }
      Kt[((uint64_t)(j * 2 + c) * k + p) * N + sl] = kv;
      sum = add_mod(sum, mul_mod(v, qjp[j * k + p], m), m.q);
    }
    Ct[((uint64_t)c * k + p) * N + sl] = mul_mod(sum, w, m);
  }
}

// The FP64 form of op_ks_rotate_into for one prime below 2^50 (Kd: its {centred key word,
// quotient} pairs).  Hoisted: sum_j Y_j . Kt_j - Ct as a representative (at most 0.75 q per
// product; folded every four digits so it stays below 4q) staged into shared memory, then the
// FP64 inverse transform.  Zero-word ciphertexts: per digit the FP64 forward transform of the
// pre-negated digit, its product with Kt_j accumulated canonically in x, then the inverse.
template <int LOGN, class Ex, class StF>
BFV_HD void op_ks_rotate_into_f64(const Ex& ex, uint64_t* s, uint64_t ct, uint32_t c, uint32_t p, const uint64_t* cts,
                                  const uint64_t* Y, const uint32_t* zflag, const double2* Kd, uint64_t kstride,
                                  const uint64_t* Ct, uint64_t* x, uint32_t elt, uint32_t k, uint32_t dk,
                                  const Modulus* mods, const uint64_t* qjp, const double2* fwd64,
                                  const double2* inv64, const StF& stf) {
  constexpr int N = 1 << LOGN;
  const Modulus m = mods[p];
  const F64Prime fp = f64_prime(m);
  const double2* tinv = inv64 + ((size_t)p << LOGN);
  double* d = reinterpret_cast<double*>(s);
  if (!zflag[ct]) {
    const uint64_t* y = Y + (ct * dk * k + p) * (uint64_t)N;  // digit j at + j*k*N
    const uint64_t ystride = (uint64_t)k * N;
    // Stage the transform's input with every operand load issued well before the products
    // that consume it: the loads (digits, key pairs, correction) are the latency this step
    // waits on, and occupancy is capped by registers.  dk = 4: four coefficients (i + r n/4)
    // per call in two interleaved streams, the next coefficient's loads in flight during each
    // product.  Otherwise two coefficients (i, i + n/2) per call.
    if (dk == 4) {
      struct Ops {
        uint64_t ct, y[4];
        double2 k[4];
      };
      auto load = [&](int i, Ops& o) {
        o.ct = ldro(Ct + i);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o.y[j] = ldro(y + j * ystride + i);
          o.k[j] = ldro2(Kd + j * kstride + i);
        }
      };
      auto finish = [&](int i, const Ops& o) {
        double sum = -u64_to_f64(o.ct);
#pragma unroll
        for (int j = 0; j < 4; ++j) sum = f64_add(sum, mulmod_f64(u64_to_f64(o.y[j]), o.k[j].x, o.k[j].y, fp.q));
        d[spad(i)] = sum;
      };
      ex.run(N / 4, [&](int u) {
        Ops a, b;
        load(u, a);
        load(u + N / 4, b);
        finish(u, a);
        load(u + N / 2, a);
        finish(u + N / 4, b);
        load(u + 3 * N / 4, b);
        finish(u + N / 2, a);
        finish(u + 3 * N / 4, b);
      });
    } else {
      ex.run(N / 2, [&](int i0) {
        const int i1 = i0 + N / 2;
        double s0 = -u64_to_f64(ldro(Ct + i0)), s1 = -u64_to_f64(ldro(Ct + i1));
        for (uint32_t j = 0; j < dk; ++j) {
          const double2 a = ldro2(Kd + j * kstride + i0), b = ldro2(Kd + j * kstride + i1);
          s0 = f64_add(s0, mulmod_f64(u64_to_f64(ldro(y + j * ystride + i0)), a.x, a.y, fp.q));
          s1 = f64_add(s1, mulmod_f64(u64_to_f64(ldro(y + j * ystride + i1)), b.x, b.y, fp.q));
          if ((j & 3) == 3 && j + 1 < dk) {
            s0 = reduce_f64(s0, fp.q, fp.qinv);
            s1 = reduce_f64(s1, fp.q, fp.qinv);
          }
        }
        d[spad(i0)] = s0;
        d[spad(i1)] = s1;
      });
    }
    ex.sync();
    auto from_smem = [d](int i) { return d[spad(i)]; };
    ntt_inverse_f64<LOGN, kMaxRadix, false>(ex, s, tinv, m, from_smem, stf);
    return;
  }
  uint64_t* xo = x + ((ct * 2 + c) * k + p) * (uint64_t)N;
  const uint64_t* c1 = cts + (ct * 2 * dk + dk) * (uint64_t)N;
  const uint32_t mask2n = 2u * N - 1u;
  for (uint32_t j = 0; j < dk; ++j) {
    const uint64_t* src = c1 + (uint64_t)j * N;
    const uint64_t adj = qjp[j * k + p];
    const bool reduce = mods[j].q > m.q;
    auto ldj = [=](int i) {
      const uint64_t xv = src[i];
      uint64_t yv = reduce ? reduce64(xv, m) : xv;
      if (xv && (((uint32_t)i * elt) & mask2n) >= (uint32_t)N) yv = sub_mod(yv, adj, m.q);
      return u64_to_f64(yv);
    };
    auto stj = [d](int i, double v) { d[spad(i)] = v; };
    ntt_forward_f64<LOGN, kMaxRadix, false>(ex, s, fwd64 + ((size_t)p << LOGN), m, ldj, stj);
    const double2* kj = Kd + j * kstride;
    ex.run(N, [&](int i) {
      const double2 kv = kj[i];
      const uint64_t v = canon_f64(mulmod_f64(d[spad(i)], kv.x, kv.y, fp.q), fp.q, fp.qinv);
      xo[i] = j ? add_mod(xo[i], v, m.q) : v;
    });
    ex.sync();
  }
  auto ldx = [xo](int i) { return u64_to_f64(xo[i]); };
  ntt_inverse_f64<LOGN, kMaxRadix>(ex, s, tinv, m, ldx, stf);
}

// One rotation for (ct, c, p): st(i, v) receives INTT(A_c)[i] (canonical); for a prime whose
// record has f64 set the transforms and products run on the FP64 pipe and stf(i, v) receives
// it instead, as a representative |v| <= 0.75 q.  Ciphertexts flagged in zflag take the
// exact path: A_c accumulated from fresh pre-negated digit transforms in the global scratch
// x [ct][2][k][n], then transformed.
template <int LOGN, class Ex, class St, class StF>
BFV_HD void op_ks_rotate_into(const Ex& ex, uint64_t* s, uint64_t ct, uint32_t c, uint32_t p, const uint64_t* cts,
                              const uint64_t* Y, const uint32_t* zflag, const uint64_t* prepared, uint64_t* x,
                              uint32_t elt, uint32_t k, uint32_t dk, const Modulus* mods, const uint64_t* qjp,
                              const ulonglong2* fwd, const ulonglong2* inv, const double2* fwd64,
                              const double2* inv64, const St& st, const StF& stf) {
  constexpr int N = 1 << LOGN;
  const Modulus m = mods[p];
  const ulonglong2* Kt = reinterpret_cast<const ulonglong2*>(prepared) + ((uint64_t)c * k + p) * N;  // digit j: + j*2*k*N
  const uint64_t kstride = 2ull * k * N;
  const uint64_t* Ct = prepared + ks_ct_offset(k, dk, N) + ((uint64_t)c * k + p) * N;
  const bool hoisted = !zflag[ct];
  // the block's hoisted digits stream from DRAM once per element: start them all into L2
  if (hoisted)
    for (uint32_t j = 0; j < dk; ++j) block_prefetch_l2(Y + ((ct * dk + j) * k + p) * (uint64_t)N, N * 8);
  if constexpr (!Ex::kSplit) {
    if (m.f64) {
      op_ks_rotate_into_f64<LOGN>(ex, s, ct, c, p, cts, Y, zflag, reinterpret_cast<const double2*>(Kt), kstride, Ct,
                                  x, elt, k, dk, mods, qjp, fwd64, inv64, stf);
      return;
    }
  }
  if (hoisted) {
    const uint64_t* y = Y + (ct * dk * k + p) * (uint64_t)N;  // digit j at + j*k*N
    const uint64_t ystride = (uint64_t)k * N;
    if (dk == 4) {
      // as in the FP64 form: four coefficients per call in two interleaved streams, each
      // coefficient's operand loads in flight during the previous one's products; the sum
      // is a lazy residue in [0, 2q), the inverse transform's input range
      struct Ops {
        uint64_t ct, y[4];
        ulonglong2 k[4];
      };
      auto load = [&](int i, Ops& o) {
        o.ct = ldro(Ct + i);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o.y[j] = ldro(y + j * ystride + i);
          o.k[j] = ldro_pair(Kt + j * kstride + i);
        }
      };
      const uint64_t q = m.q, two_q = 2 * m.q;
      auto finish = [&](int i, const Ops& o) {
        uint64_t sum = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sum += shoup_lazy(o.y[j], o.k[j].x, o.k[j].y, q);
          if (sum >= two_q) sum -= two_q;
        }
        uint64_t v = sum + q - o.ct;
        if (v >= two_q) v -= two_q;
        s[spad(i)] = v;
      };
      ex.run(N / 4, [&](int u) {
        Ops a, b;
        load(u, a);
        load(u + N / 4, b);
        finish(u, a);
        load(u + N / 2, a);
        finish(u + N / 4, b);
        load(u + 3 * N / 4, b);
        finish(u + N / 2, a);
        finish(u + 3 * N / 4, b);
      });
      ex.sync();
      auto from_smem = [s](int i) { return s[spad(i)]; };
      ntt_inverse<LOGN, kMaxRadix, false>(ex, s, inv + ((size_t)p << LOGN), m, from_smem, st);
      return;
    }
    // sum_j Y_j . Kt_j - Ct as a lazy residue in [0, 2q), the inverse transform's input range:
    // each Shoup product lies in [0, 2q) and the running sum is folded back below 2q
    auto ld = [=](int i) {
      const uint64_t two_q = 2 * m.q;
      uint64_t sum = 0;
      for (uint32_t j = 0; j < dk; ++j) {
        const ulonglong2 kv = Kt[j * kstride + i];
        sum += shoup_lazy(y[j * ystride + i], kv.x, kv.y, m.q);
        if (sum >= two_q) sum -= two_q;
      }
      uint64_t v = sum + m.q - Ct[i];  // in (0, 3q)
      if (v >= two_q) v -= two_q;
      return v;
    };
    ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
    return;
  }
  uint64_t* xo = x + ((ct * 2 + c) * k + p) * (uint64_t)N;
  const uint64_t* c1 = cts + (ct * 2 * dk + dk) * (uint64_t)N;
  const uint32_t mask2n = 2u * N - 1u;
  for (uint32_t j = 0; j < dk; ++j) {
    const uint64_t* src = c1 + (uint64_t)j * N;
    const uint64_t adj = qjp[j * k + p];
    const bool reduce = mods[j].q > m.q;
    auto ldj = [=](int i) {
      const uint64_t xv = src[i];
      uint64_t y = reduce ? reduce64(xv, m) : xv;
      if (xv && (((uint32_t)i * elt) & mask2n) >= (uint32_t)N) y = sub_mod(y, adj, m.q);
      return y;
    };
    auto stj = [s](int i, uint64_t v) { s[spad(i)] = v; };
    ntt_forward<LOGN, kMaxRadix, false>(ex, s, fwd + ((size_t)p << LOGN), m, ldj, stj);
    const ulonglong2* kj = Kt + j * kstride;
    ex.run(N, [&](int i) {
      const ulonglong2 kv = kj[i];
      const uint64_t v = shoup(s[spad(i)], kv.x, kv.y, m.q);
      xo[i] = j ? add_mod(xo[i], v, m.q) : v;
    });
    ex.sync();
  }
  auto ldx = [xo](int i) { return xo[i]; };
  ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ldx, st);
}

// Block (ct, c, p): x [ct][2][k][n] = INTT(A_c); op_ks_finish completes the keyswitch.
template <int LOGN, class Ex>
BFV_HD void op_ks_rotate(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* cts, const uint64_t* Y,
                         const uint32_t* zflag, const uint64_t* prepared, uint64_t* x, uint32_t elt, uint32_t k,
                         uint32_t dk, const Modulus* mods, const uint64_t* qjp, const ulonglong2* fwd,
                         const ulonglong2* inv, const double2* fwd64, const double2* inv64) {
  const uint64_t ct = blk / (2 * k);
  const uint32_t cp = (uint32_t)(blk % (2 * k)), c = cp / k, p = cp % k;
  uint64_t* xo = x + ((ct * 2 + c) * k + p) * ((uint64_t)1 << LOGN);
  auto st = [xo](int i, uint64_t v) { xo[i] = v; };
  const F64Prime fp = f64_prime(mods[p]);
  auto stf = [xo, fp](int i, double v) { xo[i] = canon_f64(v, fp.q, fp.qinv); };
  op_ks_rotate_into<LOGN>(ex, s, ct, c, p, cts, Y, zflag, prepared, x, elt, k, dk, mods, qjp, fwd, inv, fwd64, inv64,
                          st, stf);
}

// out [ct][2][dk][n] = sigma_g(moddown(x_c) + [c=0] c0).  Block (ct, data prime p); the
// pre-permutation limb is staged unpadded in shared memory and gathered per output.
template <int LOGN, class Ex>
BFV_HD void op_ks_finish(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* x, const uint64_t* cts,
                         uint64_t* out, uint32_t ginv, uint32_t k, uint32_t dk, const Modulus* mods) {
  constexpr int N = 1 << LOGN;
  const uint64_t ct = blk / dk;
  const uint32_t p = (uint32_t)(blk % dk);
  const Modulus m = mods[p], ms = mods[k - 1];
  const uint32_t mask2n = 2u * N - 1u;
  for (uint32_t c = 0; c < 2; ++c) {
    const uint64_t* xc = x + (ct * 2 + c) * k * (uint64_t)N;
    const uint64_t* c0 = cts + (ct * 2 * dk + p) * (uint64_t)N;
    ex.run(N, [&](int i) {
      uint64_t v = moddown_elem(xc[(uint64_t)p * N + i], xc[(uint64_t)(k - 1) * N + i], m, ms);
      if (c == 0) v = add_mod(v, c0[i], m.q);
      s[i] = v;
    });
    ex.sync();
    uint64_t* o = out + ((ct * 2 + c) * dk + p) * (uint64_t)N;
    ex.run(N, [&](int i) {
      const uint32_t src = ((uint32_t)i * ginv) & mask2n;
      o[i] = src < (uint32_t)N ? s[src] : neg_mod(s[src - N], m.q);
    });
    ex.sync();
  }
}

// Hoisted rotations of a list of elements, software-pipelined across elements.  Launch r
// holds two kinds of blocks, independent of each other:
//  * blk < s_blocks = count * 2 (element r; absent in the last launch): block (ct, c) of the
//    special prime -- the key product and inverse NTT of op_ks_rotate_into -- stored
//    compactly into xs_w [count][2][n];
//  * the rest (element r - 1; absent in the first launch): block (ct, c, data prime p), the
//    same key product and inverse NTT, whose last pass leaves in the block's own shared
//    memory the finished word moddown(x_p, x_s) (+ c0 for c = 0), with x_s read from xs_r
//    (written by the previous launch); the block then stores its limb of out_d through the
//    Galois permutation (out[i] = +-limb[i * g^-1 mod 2n]).
// The outputs equal op_ks_rotate + op_ks_finish for each element; the data-prime limbs never
// leave shared memory between the product and the finished ciphertext.  x is the zero-word
// path's scratch [count][2][k][n] (special and data blocks use disjoint parts of it).
// Block order of one pipelined launch (order bit 0: the launch holds special-prime blocks):
// the special-prime blocks (ciphertext, component) first -- they are the longest, so they
// start in the first wave -- then the data-prime blocks (ciphertext, component, prime).
// (Ordering the blocks by ciphertext, alternate launches in reverse so that a launch starts
// on the digits the previous one read last, measured slower: 0.367 against 0.350 ms.)
BFV_HD void pipe_block(uint64_t blk, uint64_t count, uint32_t order, uint32_t dk, bool* special, uint64_t* ct,
                       uint32_t* c, uint32_t* p) {
  const uint64_t s_blocks = (order & 1) ? 2 * count : 0;
  *special = blk < s_blocks;
  if (*special) {
    *ct = blk >> 1;
    *c = (uint32_t)(blk & 1);
    *p = 0;
    return;
  }
  const uint64_t d = blk - s_blocks;
  *ct = d / (2ull * dk);
  *c = (uint32_t)((d / dk) & 1);
  *p = (uint32_t)(d % dk);
}

template <int LOGN, class Ex>
BFV_HD void op_ks_rotate_pipe(const Ex& ex, uint64_t* s, uint64_t blk, uint64_t count, uint32_t order, const uint64_t* cts,
                              const uint64_t* Y, const uint32_t* zflag, uint64_t* x, const uint64_t* prep_s,
                              uint32_t elt_s, uint64_t* xs_w, const uint64_t* prep_d, uint32_t elt_d, uint32_t ginv_d,
                              const uint64_t* xs_r, uint64_t* out_d, uint32_t k, uint32_t dk, const Modulus* mods,
                              const uint64_t* qjp, const ulonglong2* fwd, const ulonglong2* inv, const double2* fwd64,
                              const double2* inv64) {
  constexpr int N = 1 << LOGN;
  bool special_block;
  uint64_t ct;
  uint32_t c, p;
  pipe_block(blk, count, order, dk, &special_block, &ct, &c, &p);
  if (special_block) {
    uint64_t* xo = xs_w + (ct * 2 + c) * (uint64_t)N;
    auto st = [xo](int i, uint64_t v) { xo[i] = v; };
    const F64Prime fs = f64_prime(mods[k - 1]);
    auto stf = [xo, fs](int i, double v) { xo[i] = canon_f64(v, fs.q, fs.qinv); };
    op_ks_rotate_into<LOGN>(ex, s, ct, c, k - 1, cts, Y, zflag, prep_s, x, elt_s, k, dk, mods, qjp, fwd, inv, fwd64,
                            inv64, st, stf);
    return;
  }
  const Modulus m = mods[p], ms = mods[k - 1];
  const uint64_t* xs = xs_r + (ct * 2 + c) * (uint64_t)N;
  const uint64_t* c0 = cts + (ct * 2 * dk + p) * (uint64_t)N;
  block_prefetch_l2(xs, N * 8);  // the finish's operands, read in the transform's last pass
  if (c == 0) block_prefetch_l2(c0, N * 8);
  auto st = [=](int i, uint64_t v) {
    uint64_t w = moddown_elem(v, ldro(xs + i), m, ms);
    if (c == 0) w = add_mod(w, ldro(c0 + i), m.q);
    s[spad(i)] = w;  // the last pass writes only the words it read: in place
  };
  // FP64 form of the same finish: (v - corr) . q_s^-1 (+ c0), corr from the special-prime limb
  // on the integer pipe (|v - corr| < 1.75 q, the sum with c0 below 1.75 q), made canonical
  const F64Prime fp = f64_prime(m);
  const uint64_t qs = ms.q, qp = m.q, r1 = m.r1;  // reduce64 needs q and the 64-bit ratio only
  const double half_s = u64_to_f64(m.half_special_mod), isp = m.f64_inv_special, isp_q = m.f64_inv_special_q;
  auto stf = [=](int i, double v) {
    const uint64_t last = add_mod(ldro(xs + i), qs >> 1, qs);
    uint64_t lastp = last - mulhi64(last, r1) * qp;
    if (lastp >= qp) lastp -= qp;
    const double corr = f64_sub(u64_to_f64(lastp), half_s);
    double w = mulmod_f64(f64_sub(v, corr), isp, isp_q, fp.q);
    if (c == 0) w = f64_add(w, u64_to_f64(ldro(c0 + i)));
    s[spad(i)] = canon_f64(w, fp.q, fp.qinv);  // in place, as above
  };
  op_ks_rotate_into<LOGN>(ex, s, ct, c, p, cts, Y, zflag, prep_d, x, elt_d, k, dk, mods, qjp, fwd, inv, fwd64, inv64,
                          st, stf);
  uint64_t* o = out_d + ((ct * 2 + c) * dk + p) * (uint64_t)N;
  const uint32_t mask2n = 2u * N - 1u;
  const uint64_t q = m.q;
  ex.run(N, [&](int i) {
    const uint32_t src = ((uint32_t)i * ginv_d) & mask2n;
    o[i] = src < (uint32_t)N ? s[spad((int)src)] : neg_mod(s[spad((int)src - N)], q);
  });
  ex.sync();
}

// ---- Enc(0) pre-moddown polys: block = (group, key-level prime p) ------------------------
template <int LOGN, class Ex>
BFV_HD void op_enc0_x(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* samples, const uint64_t* pk,
                      uint64_t* u_ntt, uint64_t* x, uint32_t k, const Modulus* mods, const ulonglong2* fwd,
                      const ulonglong2* inv) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t g = blk / k;
  const uint32_t p = (uint32_t)(blk % k);
  const Modulus m = mods[p];
  const uint64_t* u = samples + (g * 3 * k + p) * N;
  uint64_t* U = u_ntt + (g * k + p) * N;
  {
    auto ld = [u](int i) { return u[i]; };
    auto st = [U](int i, uint64_t v) { U[i] = v; };
    ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
  }
  for (uint32_t c = 0; c < 2; ++c) {
    const uint64_t* pkc = pk + ((uint64_t)c * k + p) * N;
    const uint64_t* e = samples + ((g * 3 + 1 + c) * k + p) * N;
    uint64_t* xo = x + ((g * 2 + c) * k + p) * N;
    auto ld = [=](int i) { return mul_mod(U[i], pkc[i], m); };
    auto st = [=](int i, uint64_t v) { xo[i] = add_mod(v, ldro(e + i), m.q); };
    ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
  }
}

// ---- multi-tile product and folded Enc(0) (the layer pipeline) -----------------------------
// For T tiles that share one weight matrix, the product of group g is a per-coefficient
// contraction acc[t][c] = sum_b in[t][b][c] . W[g][b] over residues < 2^60.  Each product
// is taken over 30-bit halves (a = a1 2^30 + a0, w = w1 2^30 + w0): four 32x32->64-bit
// multiply-adds into three 64-bit sums, folded exactly into a 128-bit sum every 8 terms.
// The inputs are stored with their halves pre-split (split30) by the transform that
// produces them.
constexpr uint64_t kMask30 = (uint64_t(1) << 30) - 1;
BFV_HD uint64_t split30(uint64_t v) { return ((v >> 30) << 32) | (v & kMask30); }
BFV_HD uint64_t join30(uint64_t s) { return ((s >> 32) << 30) | (s & 0xffffffffull); }

struct Mac30 {
  uint64_t s0 = 0, s1 = 0, s2 = 0;
  // a in split form, w0/w1 < 2^30.  At most 8 calls between folds: s1 gains < 2^61 per call.
  BFV_HD void mac(uint64_t a, uint32_t w0, uint32_t w1) {
    const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
#ifdef __CUDA_ARCH__
    // one fused 32x32+64 multiply-add each
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(s0) : "r"(a0), "r"(w0));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(s1) : "r"(a0), "r"(w1));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(s1) : "r"(a1), "r"(w0));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(s2) : "r"(a1), "r"(w1));
#else
    s0 += (uint64_t)a0 * w0;
    s1 += (uint64_t)a0 * w1;
    s1 += (uint64_t)a1 * w0;
    s2 += (uint64_t)a1 * w1;
#endif
  }
  // A += s0 + s1 2^30 + s2 2^60, then clear.
  BFV_HD void fold(Acc128& A) {
    uint64_t lo = s0 + (s1 << 30);
    uint64_t hi = (s1 >> 34) + (lo < s0);
    const uint64_t t = s2 << 60;
    lo += t;
    hi += (s2 >> 4) + (lo < t);
    A.lo += lo;
    A.hi += hi + (A.lo < lo);
    s0 = s1 = s2 = 0;
  }
};

// Block of the product kernel: 16 warps x 32 coefficient lanes of one data prime p; warp w
// takes tiles [h*TH, h*TH+TH) (h = w % H) of group g0 + w / H, so GB = 16 / H groups share
// the block's staged inputs.  Input blocks are staged 8 at a time (one Mac30 fold each):
// shared memory holds in [T][8][2][32] (split form) then W [GB][8][32], double-buffered.
template <int T, int TH>
struct MacShape {
  static constexpr int kWarps = 16, kThreads = 32 * kWarps, kBc = 8;
  static constexpr int H = T / TH, GB = kWarps / H;
  static constexpr int kInWords = T * kBc * 2 * 32, kWWords = GB * kBc * 32;
  static constexpr int kBufWords = kInWords + kWWords;
  static constexpr int kSegs = kBufWords / 2;  // 16-byte staging segments per chunk
  static_assert(T % TH == 0 && kWarps % H == 0, "tile split");
};

// Staging segment seg (two coefficients) of the chunk starting at input block b0: its
// shared-memory word offset and its global source, or null where the segment is zero
// (input block past `inputs`, or group past `groups`).
template <int T, int TH>
BFV_HD const uint64_t* mac_stage_src(int seg, uint32_t b0, const uint64_t* in, const uint64_t* w, uint32_t inputs,
                                     uint32_t groups, uint32_t g0, uint32_t p, uint32_t z0, uint32_t dk, int logn,
                                     int* dst) {
  using S = MacShape<T, TH>;
  const uint64_t N = uint64_t(1) << logn;
  if (seg < S::kInWords / 2) {
    const int row = seg >> 4, sg = seg & 15;
    const int c = row & 1, bb = (row >> 1) % S::kBc, t = (row >> 1) / S::kBc;
    *dst = row * 32 + 2 * sg;
    const uint32_t b = b0 + bb;
    if (b >= inputs) return nullptr;
    return in + (((uint64_t)t * inputs + b) * 2 + c) * dk * N + (uint64_t)p * N + z0 + 2 * sg;
  }
  const int sw = seg - S::kInWords / 2;
  const int row = sw >> 4, sg = sw & 15;
  const int bb = row % S::kBc, gl = row / S::kBc;
  *dst = S::kInWords + row * 32 + 2 * sg;
  const uint32_t b = b0 + bb, g = g0 + gl;
  if (b >= inputs || g >= groups) return nullptr;
  return w + (((uint64_t)g * inputs + b) * dk + p) * N + z0 + 2 * sg;
}

// One staged chunk for thread (warp, lane); chunk index k (every 32 chunks the 128-bit sums
// are reduced so that any number of input blocks stays exact).
template <int T, int TH>
BFV_HD void mac_chunk(const uint64_t* buf, int warp, int lane, Mac30 (&acc)[TH][2], Acc128 (&A)[TH][2],
                      const Modulus& m, uint32_t k) {
  using S = MacShape<T, TH>;
  const int h = warp % S::H, gl = warp / S::H;
  const uint64_t* sw = buf + S::kInWords + gl * S::kBc * 32 + lane;
  const uint64_t* si = buf + h * TH * S::kBc * 2 * 32 + lane;
#pragma unroll
  for (int bb = 0; bb < S::kBc; ++bb) {
    const uint64_t wv = sw[bb * 32];
    const uint32_t w0 = (uint32_t)(wv & kMask30), w1 = (uint32_t)(wv >> 30);
#pragma unroll
    for (int tt = 0; tt < TH; ++tt)
#pragma unroll
      for (int c = 0; c < 2; ++c) acc[tt][c].mac(si[((tt * S::kBc + bb) * 2 + c) * 32], w0, w1);
  }
#pragma unroll
  for (int tt = 0; tt < TH; ++tt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      acc[tt][c].fold(A[tt][c]);
      if ((k & 31u) == 31u) A[tt][c].fold(m);
    }
}

// Result of thread (warp, lane): acc_out [T][G][2][dk][n] (skipped for groups past G).
template <int T, int TH>
BFV_HD void mac_store(uint64_t* out, int warp, int lane, const Acc128 (&A)[TH][2], const Modulus& m,
                      uint32_t groups, uint32_t g0, uint32_t p, uint32_t z0, uint32_t dk, int logn) {
  using S = MacShape<T, TH>;
  const int h = warp % S::H, gl = warp / S::H;
  const uint32_t g = g0 + gl;
  if (g >= groups) return;
  const uint64_t N = uint64_t(1) << logn;
#pragma unroll
  for (int tt = 0; tt < TH; ++tt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint64_t t = (uint64_t)h * TH + tt;
      out[((t * groups + g) * 2 + c) * dk * N + (uint64_t)p * N + z0 + lane] = A[tt][c].reduce(m);
    }
}

// Forward transform of client ciphertext limbs into the product's operand form (split30).
template <int LOGN, class Ex>
BFV_HD void op_ntt_split(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* data, uint64_t* out, uint32_t dk,
                         const Modulus* mods, const ulonglong2* fwd) {
  const uint32_t p = (uint32_t)(blk % dk);
  const Modulus m = mods[p];
  const uint64_t* a = data + (blk << LOGN);
  uint64_t* o = out + (blk << LOGN);
  auto ld = [a](int i) { return a[i]; };
  auto st = [o](int i, uint64_t v) { o[i] = split30(v); };
  ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
}

// Public key prepared for the layer pipeline: pk_prep[c][p][z] = {v, floor(v 2^64 / q_p)} with
// v = pk_c,p . q_s^-1 mod q_p for the data primes (the moddown scale folded in) and
// v = pk_c,s for the special prime.  One work item per (c, p, z).
BFV_HD void pk_prep_item(uint64_t item, const uint64_t* pk, ulonglong2* prep, uint32_t k, int logn,
                         const Modulus* mods) {
  const uint64_t N = uint64_t(1) << logn;
  const uint32_t p = (uint32_t)((item >> logn) % k);
  const Modulus& m = mods[p];
  const uint64_t x = pk[item];
  const uint64_t v = p + 1 == k ? x : shoup(x, m.inv_special, m.inv_special_q, m.q);
  ulonglong2 w;
  w.x = v;
  w.y = shoup_companion(v, m);
  prep[item] = w;
  (void)N;
}

// Enc(0) preparation for item e (a tile-group pair): block (e, key-level prime p) stores
// U[e][p] = NTT(u).
template <int LOGN, class Ex>
BFV_HD void op_enc0_prep(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* samples, uint64_t* U, uint32_t k,
                         const Modulus* mods, const ulonglong2* fwd) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t e = blk / k;
  const uint32_t p = (uint32_t)(blk % k);
  const Modulus m = mods[p];
  const uint64_t* u = samples + (e * 3 * k + p) * N;
  uint64_t* Up = U + (e * k + p) * N;
  auto ld = [u](int i) { return u[i]; };
  auto st = [Up](int i, uint64_t v) { Up[i] = v; };
  ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
}

// Special-prime coefficients of item e's Enc(0), block (e, c): xs[e][c] = INTT(U_s . pk_c,s)
// + e_c,s, which the divide-and-round by q_s needs (after op_enc0_prep; a block of its own
// so that no block runs more than one transform).
template <int LOGN, class Ex>
BFV_HD void op_enc0_xs(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* samples, const ulonglong2* pk,
                       const uint64_t* U, uint64_t* xs, uint32_t k, const Modulus* mods, const ulonglong2* inv) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t e = blk >> 1;
  const uint32_t c = (uint32_t)(blk & 1), p = k - 1;
  const Modulus m = mods[p];
  const uint64_t* Up = U + (e * k + p) * N;
  const ulonglong2* pkc = pk + ((uint64_t)c * k + p) * N;
  const uint64_t* ec = samples + ((e * 3 + 1 + c) * k + p) * N;
  uint64_t* xo = xs + (e * 2 + c) * N;
  auto ld = [=](int i) {
    const ulonglong2 w = pkc[i];
    return shoup(Up[i], w.x, w.y, m.q);
  };
  auto st = [=](int i, uint64_t v) { xo[i] = add_mod(v, ldro(ec + i), m.q); };
  ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
}

// Additive output term of item e, component c, data prime p, coefficient z (elementwise,
// after op_enc0_prep / op_enc0_xs, beside the product):
//   E = (e_c,p - corr(x_s,c)) . q_s^-1  (if Enc(0))  -  [c = 0] Delta . mask  (if masked)
// i.e. everything op_intt_protect adds after its transform except the part that must go
// through it.  Layout E [items][2][dk][n]; row r = (e * 2 + c) * dk + p.
BFV_HD uint64_t enc0_fin_elem(uint64_t e, uint32_t c, uint32_t p, uint64_t z, const uint64_t* samples,
                              const uint64_t* xs, const uint64_t* mask, uint32_t k, int logn, const Modulus* mods,
                              uint64_t q_mod_t, uint64_t upper_half, uint64_t t, int tlog) {
  const uint64_t N = uint64_t(1) << logn;
  const Modulus& m = mods[p];
  uint64_t v = 0;
  if (samples)
    v = moddown_elem(samples[((e * 3 + 1 + c) * k + p) * N + z], xs[(e * 2 + c) * N + z], m, mods[k - 1]);
  if (mask && c == 0) v = sub_mod(v, scale_plain_coeff(mask[e * N + z], q_mod_t, upper_half, t, tlog, m), m.q);
  return v;
}
BFV_HD void enc0_fin_item(uint64_t item, const uint64_t* samples, const uint64_t* xs, const uint64_t* mask,
                          uint64_t* E, uint32_t k, uint32_t dk, int logn, const Modulus* mods, uint64_t q_mod_t,
                          uint64_t upper_half, uint64_t t, int tlog) {
  const uint64_t z = item & ((uint64_t(1) << logn) - 1), r = item >> logn;
  E[item] = enc0_fin_elem(r / (2 * dk), (uint32_t)((r / dk) & 1), (uint32_t)(r % dk), z, samples, xs, mask, k, logn,
                          mods, q_mod_t, upper_half, t, tlog);
}

// INTT of the accumulated product with the Enc(0) and mask epilogue, block (e, c, p):
//   out = INTT(acc + U_p . pk_c,p . q_s^-1) + E[e][c][p]
// which equals INTT(acc) + moddown(INTT(U . pk_c) + e_c) - Delta mask exactly, because
// moddown_p(x) = (x_p - corr(x_s)) q_s^-1 is linear in x_p.  U (with pk) and E may be null.
template <int LOGN, class Ex>
BFV_HD void op_intt_protect(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* acc, uint64_t* out,
                            const uint64_t* U, const ulonglong2* pk, const uint64_t* E, uint32_t k, uint32_t dk,
                            const Modulus* mods, const ulonglong2* inv) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t e = blk / (2 * dk);
  const uint32_t cp = (uint32_t)(blk % (2 * dk)), c = cp / dk, p = cp % dk;
  const Modulus m = mods[p];
  const uint64_t* a = acc + (e * 2 * dk + cp) * N;
  uint64_t* o = out + (e * 2 * dk + cp) * N;
  const uint64_t* Up = U ? U + (e * k + p) * N : nullptr;
  const ulonglong2* pkc = U ? pk + ((uint64_t)c * k + p) * N : nullptr;
  const uint64_t* Ep = E ? E + (e * 2 * dk + cp) * N : nullptr;
  auto ld = [=](int i) {
    uint64_t v = a[i];
    if (Up) {
      const ulonglong2 w = pkc[i];  // pk . q_s^-1 with its Shoup companion
      v = add_mod(v, shoup(Up[i], w.x, w.y, m.q), m.q);
    }
    return v;
  };
  auto st = [=](int i, uint64_t v) { o[i] = Ep ? add_mod(v, ldro(Ep + i), m.q) : v; };
  ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
}

// ---- client phase: block = (batch b, data prime p) -----------------------------------------
template <int LOGN, class Ex>
BFV_HD void op_client_phase(const Ex& ex, uint64_t* s, uint64_t blk, uint64_t* data, const uint64_t* sk, uint32_t dk,
                            const Modulus* mods, const ulonglong2* fwd, const ulonglong2* inv) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint64_t b = blk / dk;
  const uint32_t p = (uint32_t)(blk % dk);
  const Modulus m = mods[p];
  uint64_t* a = data + (b * dk + p) * N;
  const uint64_t* key = sk + (uint64_t)p * N;
  {
    auto ld = [a](int i) { return a[i]; };
    auto st = [s](int i, uint64_t v) { s[spad(i)] = v; };
    ntt_forward<LOGN, kMaxRadix, false>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
  }
  {
    auto ld = [=](int i) { return mul_mod(s[spad(i)], key[i], m); };
    auto st = [a](int i, uint64_t v) { a[i] = v; };
    ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
  }
}

// ---- resident token product (n = 16384: 19 blocks of 8192 weights) -------------------------
constexpr int kTokenBlocks = 19, kTokenWidth = 8192;

template <int LOGN, class Ex>
BFV_HD void op_token_lift_ntt(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* ring, uint64_t* w, uint32_t dk,
                              const Modulus* mods, const ulonglong2* fwd) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint32_t b = (uint32_t)(blk / dk), p = (uint32_t)(blk % dk);
  const Modulus m = mods[p];
  const uint64_t* r = ring + (uint64_t)b * kTokenWidth;
  uint64_t* o = w + ((uint64_t)b * dk + p) * N;
  const uint64_t adjust = m.q - (uint64_t(1) << 59);
  auto ld = [=](int i) {
    if (i >= kTokenWidth) return uint64_t(0);
    const uint64_t v = r[kTokenWidth - 1 - i];
    return v + (adjust & (uint64_t(0) - (v >> 58)));
  };
  auto st = [o](int i, uint64_t v) { o[i] = v; };
  ntt_forward<LOGN, kMaxRadix>(ex, s, fwd + ((size_t)p << LOGN), m, ld, st);
}

template <int LOGN, class Ex>
BFV_HD void op_token_mac_intt(const Ex& ex, uint64_t* s, uint64_t blk, const uint64_t* in, const uint64_t* w,
                              const uint64_t* scaled, uint64_t* out, uint32_t slots, uint32_t dk, const Modulus* mods,
                              const ulonglong2* inv) {
  constexpr uint64_t N = uint64_t(1) << LOGN;
  const uint32_t sl = (uint32_t)(blk / (2 * dk)), cp = (uint32_t)(blk % (2 * dk)), c = cp / dk, p = cp % dk;
  const Modulus m = mods[p];
  const uint64_t words = (uint64_t)slots * 2 * dk * N;
  const uint64_t* inb = in + ((uint64_t)sl * 2 * dk + cp) * N;
  const uint64_t* wp = w + (uint64_t)p * N;
  auto ld = [=](int i) {
    Acc128 acc;
    for (int b = 0; b < kTokenBlocks; ++b) acc.mac(inb[b * words + i], wp[(uint64_t)b * dk * N + i]);
    return acc.reduce(m);
  };
  uint64_t* o = out + ((uint64_t)sl * 2 * dk + cp) * N;
  const uint64_t add = scaled[(uint64_t)sl * dk + p];
  auto st = [=](int j, uint64_t v) {
    if (c == 0 && j == kTokenWidth - 1) v = add_mod(v, add, m.q);
    const uint32_t dest = ((uint32_t)j + 2u * (uint32_t)N - (kTokenWidth - 1)) & (2u * (uint32_t)N - 1u);
    o[dest & (N - 1)] = dest >= N ? neg_mod(v, m.q) : v;
  };
  ntt_inverse<LOGN, kMaxRadix>(ex, s, inv + ((size_t)p << LOGN), m, ld, st);
}

// ---- CRT of one target's dk residues to dk little-endian 64-bit limbs in [0, Q) ------------
// sum_j (a_j (Q/q_j)^-1 mod q_j) (Q/q_j) < dk*Q, then Q is subtracted while the sum >= Q.
BFV_HD void crt_target(const uint64_t* res, uint32_t dk, const Modulus* mods, const uint64_t* crt_part,
                       const uint64_t* crt_inv, const uint64_t* crt_q, uint64_t* limbs) {
  uint64_t acc[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  for (uint32_t j = 0; j < dk; ++j) {
    const uint64_t y = shoup(res[j], crt_inv[2 * j], crt_inv[2 * j + 1], mods[j].q);
    uint64_t carry = 0;
    for (uint32_t l = 0; l < dk; ++l) {
      const uint64_t plo = y * crt_part[j * dk + l], phi = mulhi64(y, crt_part[j * dk + l]);
      const uint64_t s1 = acc[l] + plo;
      const uint64_t c1 = s1 < plo;
      const uint64_t s2 = s1 + carry;
      const uint64_t c2 = s2 < s1;
      acc[l] = s2;
      carry = phi + c1 + c2;
    }
    for (uint32_t l = dk; l < 9 && carry; ++l) {
      const uint64_t s1 = acc[l] + carry;
      carry = s1 < carry;
      acc[l] = s1;
    }
  }
  for (uint32_t iter = 0; iter <= dk; ++iter) {
    bool ge = acc[dk] != 0;
    if (!ge) {
      ge = true;
      for (int l = (int)dk - 1; l >= 0; --l) {
        if (acc[l] != crt_q[l]) {
          ge = acc[l] > crt_q[l];
          break;
        }
      }
    }
    if (!ge) break;
    uint64_t borrow = 0;
    for (uint32_t l = 0; l <= dk; ++l) {
      const uint64_t ql = l < dk ? crt_q[l] : 0;
      const uint64_t d1 = acc[l] - ql;
      const uint64_t b1 = acc[l] < ql;
      const uint64_t d2 = d1 - borrow;
      const uint64_t b2 = d1 < borrow;
      acc[l] = d2;
      borrow = b1 | b2;
    }
  }
  for (uint32_t l = 0; l < dk; ++l) limbs[l] = acc[l];
}

}  // namespace bfvgpu
