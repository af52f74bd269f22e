/*
 * bfv_oracle.h -- CPU restatement of privacy-rag's BFV ciphertext-arithmetic hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * privacy-rag_b200/ and the timed CPU baseline of bench.py.  Nothing in the product
 * path may link or call it.
 *
 * Every function restates the behaviour of a reference file (paths relative to the
 * privacy-rag checkout, "IV1" = implementation_v1/).  The reference arithmetic sits
 * on Microsoft SEAL 4.1.2 and GMP, neither of which is available; each algorithm
 * is restated here from its mathematics and the published methods it uses
 * (Barrett 1986; Harvey, "Faster arithmetic for number-theoretic transforms", 2014).
 *
 * Parity status: plaintext-level results (decrypt(target) = sum x*w mod t), parameter
 * values (IV1/artifacts/bfv_context.json), packing decisions and all
 * coefficient-domain integer steps are pinned.  NTT-domain values and key material
 * are pinned only against this restatement (SEAL is absent).
 *
 * Layouts follow the reference: a polynomial set is [..][prime][N] of uint64 words,
 * a ciphertext is [2][k][N], a keyswitch key is [digit][2][k+1][N] (NTT form).
 */
#ifndef BFV_ORACLE_H
#define BFV_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define OR_MAX_PRIMES 16

/* Parameter context: n, the prime chain (data primes first, special prime last),
 * per-prime NTT tables in the reference's table layout, and BFV scaling constants. */
typedef struct or_ctx {
  size_t n, logn;
  size_t k;            /* total primes held (data + special)                       */
  size_t data_k;       /* data-level primes; k - data_k special primes (0 or 1)     */
  uint64_t t;          /* plaintext modulus                                          */
  uint64_t q[OR_MAX_PRIMES];
  uint64_t r0[OR_MAX_PRIMES], r1[OR_MAX_PRIMES]; /* floor((2^128-1)/q) split        */
  uint64_t *fwd;       /* [k][n][2] {w, floor(w 2^64/q)}: fwd[brv(i)] = psi^i        */
  uint64_t *inv;       /* [k][n][2]: inv[brv(i-1)+1] = psi^-i, inv[0] = 1            */
  uint64_t invn[OR_MAX_PRIMES][2];
  uint64_t psi[OR_MAX_PRIMES];
  /* inverse of the special prime modulo each data prime (Shoup pair) */
  uint64_t inv_special[OR_MAX_PRIMES][2];
  /* BFV constants at the data level: delta_p = floor(Q/t) mod q_p, Q mod t, (t+1)/2 */
  uint64_t delta[OR_MAX_PRIMES];
  uint64_t q_mod_t, upper_half;
} or_ctx;

/* ---- primes, roots, tables ---------------------------------------------------- */
int or_is_prime(uint64_t n);
size_t or_get_primes(uint64_t factor, int bits, size_t count, uint64_t *out);
int or_coeff_modulus(size_t n, const int *bits, size_t count, uint64_t *out);
uint64_t or_minimal_root(uint64_t q, uint64_t order);
uint64_t or_shoup_quotient(uint64_t w, uint64_t q);
or_ctx *or_ctx_new(size_t n, size_t k, const uint64_t *q, size_t data_k, uint64_t t);
void or_ctx_free(or_ctx *c);
const uint64_t *or_ctx_fwd(const or_ctx *c);
const uint64_t *or_ctx_inv(const or_ctx *c);

/* ---- scalar arithmetic --------------------------------------------------------- */
uint64_t or_mul_barrett(uint64_t a, uint64_t b, uint64_t q, uint64_t r0, uint64_t r1);
uint64_t or_mul_shoup(uint64_t a, uint64_t w, uint64_t wq, uint64_t q);
uint64_t or_mulmod(uint64_t a, uint64_t b, uint64_t q);

/* ---- NTT ----------------------------------------------------------------------- */
void or_ntt_forward(const or_ctx *c, size_t prime, uint64_t *a);
void or_ntt_inverse(const or_ctx *c, size_t prime, uint64_t *a);
void or_ntt_forward_canonical(const or_ctx *c, size_t prime, uint64_t *a);
void or_ntt_inverse_canonical(const or_ctx *c, size_t prime, uint64_t *a);
/* data [polys][n], prime of poly i = prime_offset + i % prime_count */
void or_ntt_batch(const or_ctx *c, uint64_t *data, size_t polys, size_t prime_count,
                  size_t prime_offset, int inverse, int threads);
/* O(n^2) evaluation definition of the forward transform, for small-n tests */
void or_ntt_naive(const or_ctx *c, size_t prime, const uint64_t *a, uint64_t *out);

/* ---- matrix protocol (coefficient packing) ------------------------------------- */
typedef struct or_packing { uint64_t reduction, columns, returns, inputs; } or_packing;
int or_matrix_packing(size_t b, size_t k, size_t o, or_packing *out);
int or_matrix_packing_qk_reverse64(size_t b, or_packing *out);
size_t or_packed_rows_per_ciphertext(size_t d);
void or_lift(const or_ctx *c, const uint64_t *ring, size_t blocks, uint64_t *out);
/* inputs: [I][2][k][n] coefficient form -> NTT form, in place (k = data_k) */
void or_matrix_open(const or_ctx *c, uint64_t *cts, size_t inputs, int threads);
/* ring [I][n] ring-59 words; cts_ntt from or_matrix_open; out [2][k][n].
 * targets==NULL: full output; else c0 zero except at the targets. */
void or_matrix_evaluate(const or_ctx *c, const uint64_t *cts_ntt, size_t inputs,
                        const uint64_t *ring, const uint64_t *targets, size_t count,
                        uint64_t *out, int threads);

/* ---- masking and re-randomisation ---------------------------------------------- */
void or_scale_plain(const or_ctx *c, uint64_t m, uint64_t *out /* [data_k] */);
void or_sub_plain(const or_ctx *c, uint64_t *c0, const uint64_t *mask);
void or_add_plain(const or_ctx *c, uint64_t *c0, const uint64_t *plain, size_t count);
/* samples [3][k][n] (u, e0, e1 at key level); pk [2][k][n] NTT form; out [2][data_k][n] */
void or_enc0(const or_ctx *c, const uint64_t *samples, const uint64_t *pk, uint64_t *out);
/* x [k][n] coefficient form at key level -> out [data_k][n] = round(x / q_special) */
void or_moddown(const or_ctx *c, const uint64_t *x, uint64_t *out);
void or_add_inplace(const or_ctx *c, uint64_t *a, const uint64_t *b, size_t polys);

/* ---- Galois / keyswitch / packing ---------------------------------------------- */
void or_galois(const or_ctx *c, const uint64_t *in, uint64_t *out, size_t polys,
               size_t prime_count, uint32_t elt);
/* key [data_k][2][k][n] NTT form; ct [2][data_k][n] coefficient form; out same */
void or_keyswitch_galois(const or_ctx *c, const uint64_t *ct, const uint64_t *key,
                         uint32_t elt, uint64_t *out);
void or_keyswitch_many(const or_ctx *c, const uint64_t *cts, size_t count,
                       const uint64_t *keys, const uint32_t *elts, size_t rotations,
                       uint64_t *out, int threads);
void or_monomial_shift(const or_ctx *c, uint64_t *ct, size_t exponent);
/* acyclic pack of two cts: switch(L + X^s R, key1, elt 1) + switch(sigma? ...) */
void or_packing_pair(const or_ctx *c, const uint64_t *left, const uint64_t *right,
                     const uint64_t *key_one, const uint64_t *key_level, unsigned level,
                     uint64_t *out);

/* ---- client phase ---------------------------------------------------------------- */
/* c1 [data_k][n] coefficient form, sk_ntt [data_k][n] -> out = INTT(NTT(c1) . sk) */
void or_client_phase(const or_ctx *c, const uint64_t *c1, const uint64_t *sk_ntt, uint64_t *out);

/* ---- resident token product ------------------------------------------------------ */
/* inputs_ntt [19][slots][2][k][n]; ring [19][8192]; scaled [slots][k] -> out
 * [slots][2][k][n] = add_shift(INTT(sum_b in_b . NTT(lift(reverse(ring_b))))) */
void or_token_evaluate(const or_ctx *c, const uint64_t *inputs_ntt, size_t slots,
                       const uint64_t *ring, const uint64_t *scaled, uint64_t *out);
void or_token_local_scaled(const or_ctx *c, const uint64_t *shares, size_t slots,
                           const uint64_t *ring, uint64_t *scaled);

/* ---- deterministic generator (seeded synthetic inputs) -------------------------- */
uint64_t or_splitmix64(uint64_t *state);
void or_fill_uniform(uint64_t seed, const uint64_t *q, size_t prime_count, size_t n,
                     size_t polys, uint64_t *out);

#ifdef __cplusplus
}
#endif
#endif
