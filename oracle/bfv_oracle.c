/*
 * bfv_oracle.c -- CPU restatement of privacy-rag's BFV hot path (TEST INFRASTRUCTURE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
 * library, and only as the checker or the timed CPU baseline; the CUDA product path
 * never calls it.  See bfv_oracle.h for the parity status.
 *
 * Reference files restated (IV1 = implementation_v1/):
 *   parameters ........ IV1/native/src/bfv.cpp:91-105, IV1/artifacts/bfv_context.json
 *   tables ............ IV1/experiments/matrix_gpu/adapter.cpp:22-31 (table extraction),
 *                       IV1/native/gpu/client_phase/seal_tables.cpp:22-33
 *   NTT stages ........ IV1/experiments/matrix_gpu/matrix.cu:52-58, :79
 *   Barrett / Shoup ... IV1/experiments/matrix_gpu/matrix.cu:37-46
 *   lift .............. IV1/experiments/matrix_gpu/matrix.cu:48-51
 *   packing ........... IV1/native/include/prag/bfv_layout.hpp:9-27,
 *                       IV1/native/src/bfv_matrix.inc:25-29, :156-163
 *   matrix evaluate ... IV1/experiments/matrix_gpu/matrix.cu:59-63, :95-106
 *   mask scaling ...... IV1/experiments/resident_token_gpu/seal_adapter.cpp:47-50,
 *                       IV1/native/src/bfv_matrix.inc:215-219
 *   Enc(0) ............ IV1/native/gpu/enc0/enc0.cu:74-89, :125-140,
 *                       IV1/native/gpu/enc0/seal_adapter.cpp:56-61
 *   keyswitch ......... IV1/experiments/keyswitch_full_gpu/switch.cu:76-111, :142-154
 *   packing pair ...... IV1/experiments/keyswitch_full_gpu/switch.cu:78-90, :155-185,
 *                       IV1/native/src/bfv_acyclic_pack.hpp:9-52
 *   client phase ...... IV1/native/gpu/client_phase/ntt.cu:96-98, :181-199
 *   resident token .... IV1/experiments/resident_token_gpu/resident.cu:71-122, :200-221
 */
#include "bfv_oracle.h"

#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

/* ------------------------------------------------------------------------------ */
/* scalar arithmetic                                                               */
/* ------------------------------------------------------------------------------ */
uint64_t or_mulmod(uint64_t a, uint64_t b, uint64_t q) { return (uint64_t)(((u128)a * b) % q); }

static uint64_t addmod(uint64_t a, uint64_t b, uint64_t q) {
  uint64_t x = a + b;
  return x >= q ? x - q : x;
}
static uint64_t submod(uint64_t a, uint64_t b, uint64_t q) {
  uint64_t x = a + q - b;
  return x >= q ? x - q : x;
}
static uint64_t negmod(uint64_t a, uint64_t q) { return a ? q - a : 0; }

static uint64_t powmod(uint64_t a, uint64_t e, uint64_t q) {
  uint64_t r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = or_mulmod(r, a, q);
    a = or_mulmod(a, a, q);
    e >>= 1;
  }
  return r;
}

static uint64_t invmod(uint64_t a, uint64_t q) { /* q prime */
  return powmod(a, q - 2, q);
}

/* Barrett (1986) reduction of the 128-bit product x = a*b with the precomputed ratio
 * r = floor((2^128-1)/q) held as two 64-bit limbs (r1:r0).  The quotient estimate
 * floor(x*r / 2^128) is formed in 128-bit host arithmetic as hi*r1 plus the high half of
 * the 2^64 column (lo*r1 + hi*r0 + high(lo*r0)); it is the estimate the reference's limb
 * sequence produces (matrix.cu:37-43) and undershoots floor(x/q) by at most one, so one
 * conditional subtraction makes the result canonical for a, b < q < 2^63. */
uint64_t or_mul_barrett(uint64_t a, uint64_t b, uint64_t q, uint64_t r0, uint64_t r1) {
  const u128 x = (u128)a * b;
  const uint64_t lo = (uint64_t)x, hi = (uint64_t)(x >> 64);
  const u128 column = (((u128)lo * r0) >> 64) + (u128)lo * r1 + (u128)hi * r0;
  const uint64_t qhat = hi * r1 + (uint64_t)(column >> 64);
  const uint64_t rem = lo - qhat * q;
  return rem >= q ? rem - q : rem;
}

/* Shoup multiplication by a constant w with wq = floor(w*2^64/q): the remainder
 * a*w - floor(a*wq/2^64)*q lies in [0,2q) for any a < 2^64 (Harvey 2014, Alg. 2). */
static inline uint64_t shoup_lazy(uint64_t a, uint64_t w, uint64_t wq, uint64_t q) {
  const uint64_t h = (uint64_t)(((u128)a * wq) >> 64);
  return a * w - h * q;
}
uint64_t or_mul_shoup(uint64_t a, uint64_t w, uint64_t wq, uint64_t q) {
  uint64_t r = shoup_lazy(a, w, wq, q);
  return r >= q ? r - q : r;
}
uint64_t or_shoup_quotient(uint64_t w, uint64_t q) { return (uint64_t)(((u128)w << 64) / q); }

/* ------------------------------------------------------------------------------ */
/* primes, roots, tables                                                           */
/* ------------------------------------------------------------------------------ */
int or_is_prime(uint64_t n) {
  /* deterministic Miller-Rabin for 64-bit inputs (first 12 prime bases) */
  static const uint64_t bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  if (n < 2) return 0;
  for (size_t i = 0; i < 12; ++i) {
    if (n == bases[i]) return 1;
    if (n % bases[i] == 0) return 0;
  }
  uint64_t d = n - 1;
  int s = 0;
  while (!(d & 1)) { d >>= 1; ++s; }
  for (size_t i = 0; i < 12; ++i) {
    uint64_t x = powmod(bases[i], d, n);
    if (x == 1 || x == n - 1) continue;
    int composite = 1;
    for (int r = 1; r < s; ++r) {
      x = or_mulmod(x, x, n);
      if (x == n - 1) { composite = 0; break; }
    }
    if (composite) return 0;
  }
  return 1;
}

/* Primes p = 1 mod factor of exactly `bits` bits, searched downward from the largest
 * candidate below 2^bits.  This is the search behind the locked ART-002 chain
 * (bfv.cpp:91-105 creates it with CoeffModulus::Create(16384, {60 x 7})). */
size_t or_get_primes(uint64_t factor, int bits, size_t count, uint64_t *out) {
  uint64_t value = ((((uint64_t)1 << bits) - 1) / factor) * factor + 1;
  const uint64_t lower = (uint64_t)1 << (bits - 1);
  size_t found = 0;
  while (found < count && value > lower) {
    if (or_is_prime(value)) out[found++] = value;
    value -= factor;
  }
  return found;
}

/* A chain of primes with the given bit sizes, all = 1 mod 2n.  Primes of equal size
 * are handed out smallest-first in the order the sizes appear, which reproduces the
 * ascending ART-002 list of IV1/artifacts/bfv_context.json. */
int or_coeff_modulus(size_t n, const int *bits, size_t count, uint64_t *out) {
  if (count > OR_MAX_PRIMES) return -1;
  for (size_t i = 0; i < count; ++i) {
    int seen = 0;
    for (size_t j = 0; j < i; ++j) seen |= bits[j] == bits[i];
    if (seen) continue;
    size_t same = 0;
    for (size_t j = 0; j < count; ++j) same += bits[j] == bits[i];
    uint64_t found[OR_MAX_PRIMES];
    if (or_get_primes(2 * (uint64_t)n, bits[i], same, found) != same) return -2;
    size_t take = same;
    for (size_t j = 0; j < count; ++j)
      if (bits[j] == bits[i]) out[j] = found[--take];
  }
  return 0;
}

/* The smallest primitive `order`-th root of unity modulo q (order a power of two):
 * the least x in [1,q) with x^(order/2) = -1.  All primitive roots are the odd
 * powers of any one of them. */
uint64_t or_minimal_root(uint64_t q, uint64_t order) {
  if ((q - 1) % order) return 0;
  uint64_t root = 0;
  for (uint64_t x = 2; x < q; ++x) {
    uint64_t c = powmod(x, (q - 1) / order, q);
    if (powmod(c, order / 2, q) == q - 1) { root = c; break; }
  }
  if (!root) return 0;
  const uint64_t step = or_mulmod(root, root, q);
  uint64_t best = root, cur = root;
  for (uint64_t i = 1; i < order / 2; ++i) {
    cur = or_mulmod(cur, step, q);
    if (cur < best) best = cur;
  }
  return best;
}

static size_t bit_reverse(size_t x, size_t bits) {
  size_t r = 0;
  for (size_t i = 0; i < bits; ++i) r |= ((x >> i) & 1) << (bits - 1 - i);
  return r;
}

or_ctx *or_ctx_new(size_t n, size_t k, const uint64_t *q, size_t data_k, uint64_t t) {
  if (k == 0 || k > OR_MAX_PRIMES || data_k == 0 || data_k > k || k - data_k > 1) return NULL;
  if (n < 4 || (n & (n - 1))) return NULL;
  or_ctx *c = (or_ctx *)calloc(1, sizeof(or_ctx));
  if (!c) return NULL;
  c->n = n;
  while (((size_t)1 << c->logn) < n) ++c->logn;
  c->k = k;
  c->data_k = data_k;
  c->t = t;
  c->fwd = (uint64_t *)calloc(k * n * 2, sizeof(uint64_t));
  c->inv = (uint64_t *)calloc(k * n * 2, sizeof(uint64_t));
  if (!c->fwd || !c->inv) { or_ctx_free(c); return NULL; }
  for (size_t p = 0; p < k; ++p) {
    const uint64_t qi = q[p];
    if (!or_is_prime(qi) || (qi - 1) % (2 * n) || qi >= ((uint64_t)1 << 62)) { or_ctx_free(c); return NULL; }
    c->q[p] = qi;
    const u128 ratio = (~(u128)0) / qi;
    c->r0[p] = (uint64_t)ratio;
    c->r1[p] = (uint64_t)(ratio >> 64);
    const uint64_t psi = or_minimal_root(qi, 2 * n);
    c->psi[p] = psi;
    const uint64_t psi_inv = invmod(psi, qi);
    uint64_t *f = c->fwd + p * n * 2, *r = c->inv + p * n * 2;
    uint64_t power = 1;
    for (size_t i = 0; i < n; ++i) {
      const size_t at = bit_reverse(i, c->logn);
      f[2 * at] = power;
      f[2 * at + 1] = or_shoup_quotient(power, qi);
      power = or_mulmod(power, psi, qi);
    }
    r[0] = 1;
    r[1] = or_shoup_quotient(1, qi);
    power = psi_inv;
    for (size_t i = 1; i < n; ++i) {
      const size_t at = bit_reverse(i - 1, c->logn) + 1;
      r[2 * at] = power;
      r[2 * at + 1] = or_shoup_quotient(power, qi);
      power = or_mulmod(power, psi_inv, qi);
    }
    const uint64_t ninv = invmod(n % qi, qi);
    c->invn[p][0] = ninv;
    c->invn[p][1] = or_shoup_quotient(ninv, qi);
  }
  if (k > data_k) {
    const uint64_t special = q[k - 1];
    for (size_t p = 0; p < data_k; ++p) {
      const uint64_t v = invmod(special % q[p], q[p]);
      c->inv_special[p][0] = v;
      c->inv_special[p][1] = or_shoup_quotient(v, q[p]);
    }
  }
  /* BFV scaling constants at the data level: r = Q mod t, delta_p = floor(Q/t) mod q_p
   * = (Q - r)/t mod q_p = -r * t^-1 mod q_p (Q = 0 mod q_p). */
  if (t >= 2) {
    uint64_t r = 1 % t;
    for (size_t p = 0; p < data_k; ++p) r = or_mulmod(r, q[p] % t, t);
    c->q_mod_t = r;
    c->upper_half = (t + 1) >> 1;
    for (size_t p = 0; p < data_k; ++p) {
      const uint64_t tinv = invmod(t % q[p], q[p]);
      c->delta[p] = or_mulmod(negmod(r % q[p], q[p]), tinv, q[p]);
    }
  }
  return c;
}

void or_ctx_free(or_ctx *c) {
  if (!c) return;
  free(c->fwd);
  free(c->inv);
  free(c);
}
const uint64_t *or_ctx_fwd(const or_ctx *c) { return c->fwd; }
const uint64_t *or_ctx_inv(const or_ctx *c) { return c->inv; }

/* ------------------------------------------------------------------------------ */
/* NTT                                                                             */
/* ------------------------------------------------------------------------------ */
/* Forward negacyclic transform, natural order in, bit-reversed order out: the
 * Cooley-Tukey level l (gap n>>(l+1)) uses table entry 2^l + group, as the reference
 * stage kernel does (matrix.cu:52-58, :79).  Lazy Harvey butterflies keep values in
 * [0,4q); the result is reduced to [0,q) at the end. */
void or_ntt_forward(const or_ctx *c, size_t prime, uint64_t *a) {
  const size_t n = c->n;
  const uint64_t q = c->q[prime], two_q = 2 * q;
  const uint64_t *tab = c->fwd + prime * n * 2;
  for (size_t m = 1, gap = n >> 1; m < n; m <<= 1, gap >>= 1) {
    for (size_t g = 0; g < m; ++g) {
      const uint64_t w = tab[2 * (m + g)], wq = tab[2 * (m + g) + 1];
      uint64_t *x = a + 2 * g * gap, *y = x + gap;
      for (size_t j = 0; j < gap; ++j) {
        uint64_t u = x[j];
        if (u >= two_q) u -= two_q;
        const uint64_t v = shoup_lazy(y[j], w, wq, q);
        x[j] = u + v;
        y[j] = u + two_q - v;
      }
    }
  }
  for (size_t i = 0; i < n; ++i) {
    uint64_t v = a[i];
    if (v >= two_q) v -= two_q;
    if (v >= q) v -= q;
    a[i] = v;
  }
}

/* Inverse transform, bit-reversed in, natural out, Gentleman-Sande level l (gap 2^l)
 * with table entry n-(n>>l)+1+group, scaled by n^-1 at the end. */
void or_ntt_inverse(const or_ctx *c, size_t prime, uint64_t *a) {
  const size_t n = c->n;
  const uint64_t q = c->q[prime], two_q = 2 * q;
  const uint64_t *tab = c->inv + prime * n * 2;
  size_t idx = 1;
  for (size_t gap = 1, m = n >> 1; m >= 1; gap <<= 1, m >>= 1) {
    for (size_t g = 0; g < m; ++g, ++idx) {
      const uint64_t w = tab[2 * idx], wq = tab[2 * idx + 1];
      uint64_t *x = a + 2 * g * gap, *y = x + gap;
      for (size_t j = 0; j < gap; ++j) {
        const uint64_t u = x[j], v = y[j];
        uint64_t s = u + v;
        if (s >= two_q) s -= two_q;
        x[j] = s;
        y[j] = shoup_lazy(u + two_q - v, w, wq, q);
      }
    }
  }
  for (size_t i = 0; i < n; ++i) a[i] = or_mul_shoup(a[i], c->invn[prime][0], c->invn[prime][1], q);
}

/* The same transforms with canonical reduction after every butterfly, in the
 * reference GPU stage-kernel form; the lazy and canonical results must agree. */
void or_ntt_forward_canonical(const or_ctx *c, size_t prime, uint64_t *a) {
  const size_t n = c->n;
  const uint64_t q = c->q[prime];
  const uint64_t *tab = c->fwd + prime * n * 2;
  for (size_t l = 0; l < c->logn; ++l) {
    const size_t gap = n >> (l + 1), start = (size_t)1 << l;
    for (size_t i = 0; i < n / 2; ++i) {
      const size_t group = i / gap, offset = i % gap, x = group * 2 * gap + offset, y = x + gap;
      const uint64_t t = or_mul_shoup(a[y], tab[2 * (start + group)], tab[2 * (start + group) + 1], q);
      const uint64_t u = a[x];
      a[x] = addmod(u, t, q);
      a[y] = submod(u, t, q);
    }
  }
}
void or_ntt_inverse_canonical(const or_ctx *c, size_t prime, uint64_t *a) {
  const size_t n = c->n;
  const uint64_t q = c->q[prime];
  const uint64_t *tab = c->inv + prime * n * 2;
  for (size_t l = 0; l < c->logn; ++l) {
    const size_t gap = (size_t)1 << l, start = n - (n >> l) + 1;
    for (size_t i = 0; i < n / 2; ++i) {
      const size_t group = i / gap, offset = i % gap, x = group * 2 * gap + offset, y = x + gap;
      const uint64_t u = a[x], v = a[y];
      uint64_t s = addmod(u, v, q);
      uint64_t d = or_mul_shoup(submod(u, v, q), tab[2 * (start + group)], tab[2 * (start + group) + 1], q);
      if (l + 1 == c->logn) {
        s = or_mul_shoup(s, c->invn[prime][0], c->invn[prime][1], q);
        d = or_mul_shoup(d, c->invn[prime][0], c->invn[prime][1], q);
      }
      a[x] = s;
      a[y] = d;
    }
  }
}

void or_ntt_batch(const or_ctx *c, uint64_t *data, size_t polys, size_t prime_count,
                  size_t prime_offset, int inverse, int threads) {
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
  for (size_t i = 0; i < polys; ++i) {
    const size_t p = prime_offset + i % prime_count;
    if (inverse)
      or_ntt_inverse(c, p, data + i * c->n);
    else
      or_ntt_forward(c, p, data + i * c->n);
  }
}

/* Definition of the forward transform as evaluation: output k holds
 * a(psi^(2*brv(k)+1)). */
void or_ntt_naive(const or_ctx *c, size_t prime, const uint64_t *a, uint64_t *out) {
  const size_t n = c->n;
  const uint64_t q = c->q[prime];
  for (size_t k = 0; k < n; ++k) {
    const uint64_t x = powmod(c->psi[prime], 2 * bit_reverse(k, c->logn) + 1, q);
    uint64_t acc = 0, xp = 1;
    for (size_t j = 0; j < n; ++j) {
      acc = addmod(acc, or_mulmod(a[j] % q, xp, q), q);
      xp = or_mulmod(xp, x, q);
    }
    out[k] = acc;
  }
}

/* ------------------------------------------------------------------------------ */
/* matrix protocol                                                                 */
/* ------------------------------------------------------------------------------ */
/* Cost-selected packing (bfv_layout.hpp:14-27): over power-of-two reductions d,
 * minimise inputs*1572960 + returns*786528 bytes; ties keep the smallest d. */
int or_matrix_packing(size_t b, size_t k, size_t o, or_packing *out) {
  if (!b || b > 16 || !k || k > 8192 || !o || o > 155648) return -1;
  uint64_t cost = ~(uint64_t)0;
  or_packing best = {0, 0, 0, 0};
  const size_t gc = 512 / b;
  for (size_t d = 16; d <= 8192 / b; d *= 2) {
    const size_t cap = gc < 8192 / (b * d) ? gc : 8192 / (b * d);
    const size_t full = o / gc, tail = o % gc;
    const size_t returns = full * ((gc + cap - 1) / cap) + (tail ? (tail + cap - 1) / cap : 0);
    const size_t inputs = (k + d - 1) / d;
    const uint64_t bytes = (uint64_t)inputs * 1572960u + (uint64_t)returns * 786528u;
    if (bytes < cost) {
      cost = bytes;
      best.reduction = d;
      best.columns = cap;
      best.returns = returns;
      best.inputs = inputs;
    }
  }
  *out = best;
  return 0;
}

int or_matrix_packing_qk_reverse64(size_t b, or_packing *out) {
  if (!b || b > 64) return -1;
  out->reduction = 128;
  out->columns = 1;
  out->returns = 1;
  out->inputs = 1;
  return 0;
}

/* bfv.cpp:112-116 */
size_t or_packed_rows_per_ciphertext(size_t d) {
  if (d == 0 || d > 8192) return 0;
  const size_t a = 16384 / (2 * d - 1), b = 8192 / d;
  return a < b ? a : b;
}

/* Centred lift of ring-59 words into each data prime: v >= 2^58 is negative and maps
 * to v + q - 2^59 (matrix.cu:48-51).  out [blocks][data_k][n]. */
void or_lift(const or_ctx *c, const uint64_t *ring, size_t blocks, uint64_t *out) {
  const size_t n = c->n, k = c->data_k;
  for (size_t b = 0; b < blocks; ++b)
    for (size_t p = 0; p < k; ++p)
      for (size_t z = 0; z < n; ++z) {
        const uint64_t v = ring[b * n + z];
        out[(b * k + p) * n + z] = v + ((c->q[p] - ((uint64_t)1 << 59)) & ((uint64_t)0 - (v >> 58)));
      }
}

/* Matrix::Matrix: forward NTT of both components of every input ciphertext
 * (matrix.cu:56-62 / matrix.cu:85). */
void or_matrix_open(const or_ctx *c, uint64_t *cts, size_t inputs, int threads) {
  or_ntt_batch(c, cts, inputs * 2 * c->data_k, c->data_k, 0, 0, threads);
}

/* Matrix::evaluate_impl (matrix.cu:95-106): lift and NTT every weight block, multiply-
 * accumulate against the NTT'd inputs over blocks, inverse NTT both components; with
 * targets, c0 is zero except at the strictly increasing target coefficients. */
void or_matrix_evaluate(const or_ctx *c, const uint64_t *cts_ntt, size_t inputs,
                        const uint64_t *ring, const uint64_t *targets, size_t count,
                        uint64_t *out, int threads) {
  const size_t n = c->n, k = c->data_k, limbs = n * k;
  uint64_t *weight = (uint64_t *)malloc(inputs * limbs * sizeof(uint64_t));
  or_lift(c, ring, inputs, weight);
  or_ntt_batch(c, weight, inputs * k, k, 0, 0, threads);
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
  for (size_t cp = 0; cp < 2 * k; ++cp) {
    const size_t p = cp % k;
    const uint64_t q = c->q[p], r0 = c->r0[p], r1 = c->r1[p];
    uint64_t *dst = out + cp * n;
    for (size_t z = 0; z < n; ++z) {
      uint64_t sum = 0;
      for (size_t b = 0; b < inputs; ++b)
        sum = addmod(sum, or_mul_barrett(cts_ntt[(b * 2 * k) * n + cp * n + z], weight[(b * k + p) * n + z], q, r0, r1), q);
      dst[z] = sum;
    }
    or_ntt_inverse(c, p, dst);
  }
  free(weight);
  if (targets) {
    uint64_t *keep = (uint64_t *)malloc(count * k * sizeof(uint64_t));
    for (size_t p = 0; p < k; ++p)
      for (size_t i = 0; i < count; ++i) keep[p * count + i] = out[p * n + targets[i]];
    memset(out, 0, limbs * sizeof(uint64_t));
    for (size_t p = 0; p < k; ++p)
      for (size_t i = 0; i < count; ++i) out[p * n + targets[i]] = keep[p * count + i];
    free(keep);
  }
}

/* ------------------------------------------------------------------------------ */
/* masking / Enc(0)                                                                */
/* ------------------------------------------------------------------------------ */
/* Delta-scaling of one plaintext coefficient m < t into each data prime:
 * m*floor(Q/t) + floor(((Q mod t)*m + floor((t+1)/2)) / t)  mod q_p
 * (resident/seal_adapter.cpp:47-50, the scaling-variant rule behind sub_plain). */
void or_scale_plain(const or_ctx *c, uint64_t m, uint64_t *out) {
  const u128 numerator = (u128)c->q_mod_t * m + c->upper_half;
  const u128 fix128 = numerator / c->t;
  for (size_t p = 0; p < c->data_k; ++p) {
    const uint64_t q = c->q[p];
    const uint64_t fix = (uint64_t)(fix128 % q);
    out[p] = addmod(or_mulmod(m % q, c->delta[p], q), fix, q);
  }
}

/* Evaluator::sub_plain_inplace on c0 (bfv_matrix.inc:215-219). c0 [data_k][n]. */
void or_sub_plain(const or_ctx *c, uint64_t *c0, const uint64_t *mask) {
  uint64_t s[OR_MAX_PRIMES];
  for (size_t z = 0; z < c->n; ++z) {
    or_scale_plain(c, mask[z], s);
    for (size_t p = 0; p < c->data_k; ++p) c0[p * c->n + z] = submod(c0[p * c->n + z], s[p], c->q[p]);
  }
}
void or_add_plain(const or_ctx *c, uint64_t *c0, const uint64_t *plain, size_t count) {
  uint64_t s[OR_MAX_PRIMES];
  for (size_t z = 0; z < count && z < c->n; ++z) {
    or_scale_plain(c, plain[z], s);
    for (size_t p = 0; p < c->data_k; ++p) c0[p * c->n + z] = addmod(c0[p * c->n + z], s[p], c->q[p]);
  }
}

/* Divide-and-round by the special prime (enc0.cu:81-89, switch.cu:103-111):
 * out_p = (x_p - ((x_s + floor(q_s/2)) mod q_s mod q_p - floor(q_s/2) mod q_p)) * q_s^-1.
 * The reference reduces mod q_p with one conditional subtraction, valid for ART-002
 * where every prime is within a factor two of q_s; here the reduction is exact. */
void or_moddown(const or_ctx *c, const uint64_t *x, uint64_t *out) {
  const size_t n = c->n, s = c->k - 1;
  const uint64_t special = c->q[s], half = special >> 1;
  for (size_t p = 0; p < c->data_k; ++p) {
    const uint64_t q = c->q[p], halfmod = half % q;
    for (size_t z = 0; z < n; ++z) {
      const uint64_t last = addmod(x[s * n + z], half, special);
      const uint64_t correction = submod(last % q, halfmod, q);
      out[p * n + z] = or_mul_shoup(submod(x[p * n + z], correction, q), c->inv_special[p][0], c->inv_special[p][1], q);
    }
  }
}

void or_add_inplace(const or_ctx *c, uint64_t *a, const uint64_t *b, size_t polys) {
  for (size_t i = 0; i < polys; ++i) {
    const uint64_t q = c->q[i % c->data_k];
    for (size_t z = 0; z < c->n; ++z) a[i * c->n + z] = addmod(a[i * c->n + z], b[i * c->n + z], q);
  }
}

/* PublicZero::evaluate (enc0.cu:125-140) and reference() (enc0/seal_adapter.cpp:56-61):
 * Enc(0)_c = moddown(INTT(NTT(u) . pk_c) + e_c) at the key level. */
void or_enc0(const or_ctx *c, const uint64_t *samples, const uint64_t *pk, uint64_t *out) {
  const size_t n = c->n, k = c->k, dk = c->data_k;
  uint64_t *u = (uint64_t *)malloc(k * n * sizeof(uint64_t));
  uint64_t *prod = (uint64_t *)malloc(k * n * sizeof(uint64_t));
  memcpy(u, samples, k * n * sizeof(uint64_t));
  for (size_t p = 0; p < k; ++p) or_ntt_forward(c, p, u + p * n);
  for (size_t comp = 0; comp < 2; ++comp) {
    for (size_t p = 0; p < k; ++p) {
      const uint64_t q = c->q[p];
      for (size_t z = 0; z < n; ++z)
        prod[p * n + z] = or_mul_barrett(u[p * n + z], pk[(comp * k + p) * n + z], q, c->r0[p], c->r1[p]);
      or_ntt_inverse(c, p, prod + p * n);
      const uint64_t *e = samples + (comp + 1) * k * n + p * n;
      for (size_t z = 0; z < n; ++z) prod[p * n + z] = addmod(prod[p * n + z], e[z], q);
    }
    or_moddown(c, prod, out + comp * dk * n);
  }
  free(u);
  free(prod);
}

/* ------------------------------------------------------------------------------ */
/* Galois automorphism, keyswitch, acyclic packing                                 */
/* ------------------------------------------------------------------------------ */
/* X -> X^elt on coefficient-form polynomials: coefficient j moves to j*elt mod 2n,
 * negated when that index is >= n (the permutation of switch.cu:78-87). */
void or_galois(const or_ctx *c, const uint64_t *in, uint64_t *out, size_t polys,
               size_t prime_count, uint32_t elt) {
  const size_t n = c->n, mask2 = 2 * n - 1;
  for (size_t i = 0; i < polys; ++i) {
    const uint64_t q = c->q[i % prime_count];
    for (size_t j = 0; j < n; ++j) {
      const size_t dest = (j * (size_t)elt) & mask2;
      const uint64_t v = in[i * n + j];
      out[i * n + (dest & (n - 1))] = dest >= n ? negmod(v, q) : v;
    }
  }
}

/* Key switch of the ciphertext (c0, c1) (coefficient form) with an alpha = 1 RNS
 * decomposition and one special prime (switch.cu:92-111, :142-154): digit j is the
 * residue of c1 at data prime j, reduced into every prime; products with the key
 * are accumulated in the NTT domain, brought back, and divided by the special prime.
 * out_0 = c0 + ks_0, out_1 = ks_1. */
static void keyswitch_core(const or_ctx *c, const uint64_t *ct, const uint64_t *key, uint64_t *out) {
  const size_t n = c->n, k = c->k, dk = c->data_k;
  uint64_t *digit = (uint64_t *)malloc(n * sizeof(uint64_t));
  uint64_t *acc = (uint64_t *)calloc(2 * k * n, sizeof(uint64_t));
  for (size_t p = 0; p < k; ++p) {
    const uint64_t q = c->q[p];
    for (size_t j = 0; j < dk; ++j) {
      const uint64_t *src = ct + (dk + j) * n; /* c1, prime j */
      for (size_t z = 0; z < n; ++z) digit[z] = src[z] % q;
      or_ntt_forward(c, p, digit);
      for (size_t comp = 0; comp < 2; ++comp) {
        const uint64_t *kk = key + ((j * 2 + comp) * k + p) * n;
        uint64_t *a = acc + (comp * k + p) * n;
        for (size_t z = 0; z < n; ++z) a[z] = addmod(a[z], or_mul_barrett(digit[z], kk[z], q, c->r0[p], c->r1[p]), q);
      }
    }
  }
  for (size_t comp = 0; comp < 2; ++comp) {
    for (size_t p = 0; p < k; ++p) or_ntt_inverse(c, p, acc + (comp * k + p) * n);
    or_moddown(c, acc + comp * k * n, out + comp * dk * n);
  }
  or_add_inplace(c, out, ct, dk);
  free(digit);
  free(acc);
}

/* Switch::apply (keyswitch seal_adapter.cpp:44-52): Galois automorphism of both
 * components, then key switch of the permuted c1 back to the key's target secret. */
void or_keyswitch_galois(const or_ctx *c, const uint64_t *ct, const uint64_t *key,
                         uint32_t elt, uint64_t *out) {
  const size_t words = 2 * c->data_k * c->n;
  uint64_t *perm = (uint64_t *)malloc(words * sizeof(uint64_t));
  or_galois(c, ct, perm, 2 * c->data_k, c->data_k, elt);
  keyswitch_core(c, perm, key, out);
  free(perm);
}

/* Every (rotation r, ciphertext i) pair: out [r][i][2][dk][n]. */
void or_keyswitch_many(const or_ctx *c, const uint64_t *cts, size_t count,
                       const uint64_t *keys, const uint32_t *elts, size_t rotations,
                       uint64_t *out, int threads) {
  const size_t words = 2 * c->data_k * c->n, key_words = c->data_k * 2 * c->k * c->n;
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic)
  for (size_t u = 0; u < rotations * count; ++u) {
    const size_t r = u / count, i = u % count;
    or_keyswitch_galois(c, cts + i * words, keys + r * key_words, elts[r], out + u * words);
  }
}

/* Multiplication by X^exponent in Z_q[X]/(X^n+1) (bfv_acyclic_pack.hpp:9-21). */
void or_monomial_shift(const or_ctx *c, uint64_t *ct, size_t exponent) {
  const size_t n = c->n;
  uint64_t *tmp = (uint64_t *)malloc(n * sizeof(uint64_t));
  exponent %= 2 * n;
  for (size_t i = 0; i < 2 * c->data_k; ++i) {
    const uint64_t q = c->q[i % c->data_k];
    uint64_t *a = ct + i * n;
    for (size_t j = 0; j < n; ++j) {
      const size_t dest = (j + exponent) % (2 * n);
      tmp[dest % n] = dest >= n ? negmod(a[j], q) : a[j];
    }
    memcpy(a, tmp, n * sizeof(uint64_t));
  }
  free(tmp);
}

/* pack_pair (bfv_acyclic_pack.hpp:37-46; GPU form switch.cu:155-185):
 * R' = X^(n>>(level+1)) R;  out = switch_1(L + R') + switch_g(sigma_g(L - R')),
 * g = 2^(level+1) + 1. */
void or_packing_pair(const or_ctx *c, const uint64_t *left, const uint64_t *right,
                     const uint64_t *key_one, const uint64_t *key_level, unsigned level,
                     uint64_t *out) {
  const size_t dk = c->data_k, n = c->n, words = 2 * dk * n;
  uint64_t *r = (uint64_t *)malloc(words * sizeof(uint64_t));
  uint64_t *sum = (uint64_t *)malloc(words * sizeof(uint64_t));
  uint64_t *diff = (uint64_t *)malloc(words * sizeof(uint64_t));
  uint64_t *tmp = (uint64_t *)malloc(words * sizeof(uint64_t));
  memcpy(r, right, words * sizeof(uint64_t));
  or_monomial_shift(c, r, n >> (level + 1));
  for (size_t i = 0; i < words; ++i) {
    const uint64_t q = c->q[(i / n) % dk];
    sum[i] = addmod(left[i], r[i], q);
    diff[i] = submod(left[i], r[i], q);
  }
  or_keyswitch_galois(c, sum, key_one, 1, out);
  or_keyswitch_galois(c, diff, key_level, (1u << (level + 1)) + 1, tmp);
  or_add_inplace(c, out, tmp, 2 * dk);
  free(r);
  free(sum);
  free(diff);
  free(tmp);
}

/* ------------------------------------------------------------------------------ */
/* client phase                                                                    */
/* ------------------------------------------------------------------------------ */
/* NttBatch::client_phase (ntt.cu:181-199): c1 . s for each data prime. */
void or_client_phase(const or_ctx *c, const uint64_t *c1, const uint64_t *sk_ntt, uint64_t *out) {
  const size_t n = c->n;
  memcpy(out, c1, c->data_k * n * sizeof(uint64_t));
  for (size_t p = 0; p < c->data_k; ++p) {
    uint64_t *a = out + p * n;
    or_ntt_forward(c, p, a);
    for (size_t z = 0; z < n; ++z) a[z] = or_mulmod(a[z], sk_ntt[p * n + z], c->q[p]);
    or_ntt_inverse(c, p, a);
  }
}

/* ------------------------------------------------------------------------------ */
/* resident token product                                                          */
/* ------------------------------------------------------------------------------ */
#define TOKEN_BLOCKS 19
#define TOKEN_WIDTH 8192

/* TokenWeights::evaluate_device (resident.cu:200-221): the weight column of block b
 * enters reversed in the low 8192 coefficients (lift kernel :71-78), is NTT'd, the
 * 19 block products are accumulated, inverse NTT'd, then add_shift (:102-107) adds
 * the scaled local share at coefficient 8191 of c0 and multiplies by X^(2n-8191). */
void or_token_evaluate(const or_ctx *c, const uint64_t *inputs_ntt, size_t slots,
                       const uint64_t *ring, const uint64_t *scaled, uint64_t *out) {
  const size_t n = c->n, k = c->data_k, limbs = n * k, words = slots * 2 * limbs;
  uint64_t *w = (uint64_t *)calloc(TOKEN_BLOCKS * limbs, sizeof(uint64_t));
  uint64_t *acc = (uint64_t *)calloc(words, sizeof(uint64_t));
  for (size_t b = 0; b < TOKEN_BLOCKS; ++b)
    for (size_t p = 0; p < k; ++p) {
      uint64_t *dst = w + (b * k + p) * n;
      for (size_t z = 0; z < TOKEN_WIDTH && z < n; ++z) {
        const uint64_t v = ring[b * TOKEN_WIDTH + (TOKEN_WIDTH - 1 - z)];
        dst[z] = v + ((c->q[p] - ((uint64_t)1 << 59)) & ((uint64_t)0 - (v >> 58)));
      }
      or_ntt_forward(c, p, dst);
    }
  for (size_t i = 0; i < words; ++i) {
    const size_t coefficient = i % limbs, p = coefficient / n;
    uint64_t sum = 0;
    for (size_t b = 0; b < TOKEN_BLOCKS; ++b)
      sum = addmod(sum, or_mul_barrett(inputs_ntt[b * words + i], w[b * limbs + coefficient], c->q[p], c->r0[p], c->r1[p]), c->q[p]);
    acc[i] = sum;
  }
  for (size_t i = 0; i < words / n; ++i) or_ntt_inverse(c, i % k, acc + i * n);
  for (size_t i = 0; i < words; ++i) {
    const size_t j = i % n, p = (i / n) % k, comp = (i / limbs) % 2, slot = i / (2 * limbs);
    const uint64_t q = c->q[p];
    uint64_t v = acc[i];
    if (comp == 0 && j == TOKEN_WIDTH - 1) v = addmod(v, scaled[slot * k + p], q);
    const size_t dest = (j + 2 * n - (TOKEN_WIDTH - 1)) % (2 * n);
    out[i - j + dest % n] = dest >= n ? negmod(v, q) : v;
  }
  free(w);
  free(acc);
}

/* local_partials/local_scale (resident.cu:109-122): m = (sum_j share_j * w_j mod 2^64)
 * mod 2^59, then Delta-scaled into each prime. */
void or_token_local_scaled(const or_ctx *c, const uint64_t *shares, size_t slots,
                           const uint64_t *ring, uint64_t *scaled) {
  const size_t words = TOKEN_BLOCKS * TOKEN_WIDTH;
  for (size_t s = 0; s < slots; ++s) {
    uint64_t sum = 0;
    for (size_t j = 0; j < words; ++j) sum += shares[s * words + j] * ring[j];
    or_scale_plain(c, sum & (((uint64_t)1 << 59) - 1), scaled + s * c->data_k);
  }
}

/* ------------------------------------------------------------------------------ */
/* deterministic generator                                                         */
/* ------------------------------------------------------------------------------ */
uint64_t or_splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9e3779b97f4a7c15ULL);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

/* Residues uniform in [0,q_p) for [polys][n] with prime p = poly % prime_count. */
void or_fill_uniform(uint64_t seed, const uint64_t *q, size_t prime_count, size_t n,
                     size_t polys, uint64_t *out) {
  uint64_t s = seed;
  for (size_t i = 0; i < polys; ++i)
    for (size_t z = 0; z < n; ++z) out[i * n + z] = or_splitmix64(&s) % q[i % prime_count];
}
