// Shared-memory-resident negacyclic NTT / inverse NTT of one RNS limb per thread block.
//
// Transform definition (the reference's stage kernels, IV1/experiments/matrix_gpu/
// matrix.cu:52-58 and :79, and every other `stage` copy):
//   forward  natural -> bit-reversed, Cooley-Tukey level l has gap n>>(l+1) and uses
//            twiddle table entry 2^l + group;
//   inverse  bit-reversed -> natural, Gentleman-Sande level l has gap 2^l and uses
//            entry n-(n>>l)+1+group; the result is scaled by n^-1.
// Tables hold {w, floor(w 2^64/q)} pairs (ulonglong2) in that layout.
//
// B200 schedule: instead of one global-memory launch per level (14 launches for
// n = 16384 in the reference), one thread block keeps the whole limb in shared memory
// (padded one word per 16 to spread 64-bit accesses over the 32 banks) and runs the
// log2(n) levels as 3 or 4 passes of radix-16 / radix-8 butterfly units held in
// registers.  The first pass reads through a loader functor (global memory, with any
// fused prologue: lift, Galois pre-negation, digit reduction, multiply-accumulate) and
// the last pass writes through a storer functor (fused epilogue).  Values stay lazy
// (forward in [0,4q), inverse in [0,2q)) between levels and are made canonical once.
//
// Every pass is written as a per-unit function driven by an executor, so the exact
// index arithmetic also runs on the host (tests/emu) against the CPU oracle.
#pragma once
#include "arith.cuh"

#if !defined(__CUDACC__)
struct ulonglong2 {
  unsigned long long x, y;
};
#endif

namespace bfvgpu {

// Padded shared-memory word index: one spare word after every 16.
BFV_HD int spad(int i) { return i + (i >> 4); }

// Padded index of base + off for the words of one butterfly unit.  A unit's words are
// base + k*stride with (base mod 16) + (k*stride mod 16) < 16 (base mod 16 < stride when
// stride < 16, and k*stride is a multiple of 16 otherwise), so the pad of base + off is
// pad(base) + pad(off): one compile-time offset per word.  The host build checks the
// identity on every access.
BFV_HD int spad_unit(int base, int sbase, int off) {
#if !defined(__CUDA_ARCH__)
  if (spad(base + off) != sbase + off + (off >> 4)) __builtin_trap();
#else
  (void)base;
#endif
  return sbase + off + (off >> 4);
}
template <int LOGN>
struct SmemWords {
  static constexpr int value = (1 << LOGN) + ((1 << LOGN) >> 4);
};

// Pass schedule: ceil(LOGN / MAXR) passes, the larger radices first (forward) and
// reversed for the inverse.  MAXR = 4 gives radix-16/8 passes, MAXR = 3 radix-8/4.
template <int LOGN, int MAXR = 4>
struct Schedule {
  static constexpr int passes = LOGN <= MAXR ? 1 : (LOGN + MAXR - 1) / MAXR;
  static constexpr int base = LOGN / passes;
  static constexpr int extra = LOGN % passes;  // passes with radix base + 1
  // radix (log2) of forward pass p
  static constexpr int fwd_r(int p) { return p < extra ? base + 1 : base; }
  static constexpr int fwd_level(int p) {
    int l = 0;
    for (int i = 0; i < p; ++i) l += fwd_r(i);
    return l;
  }
  static constexpr int inv_r(int p) { return fwd_r(passes - 1 - p); }
  static constexpr int inv_level(int p) {
    int l = 0;
    for (int i = 0; i < p; ++i) l += inv_r(i);
    return l;
  }
};

BFV_HD uint64_t reduce_4q(uint64_t v, uint64_t q) {
  const uint64_t two_q = 2 * q;
  if (v >= two_q) v -= two_q;
  if (v >= q) v -= q;
  return v;
}

// U radix-2^R Cooley-Tukey units of the forward pass starting at level L: units u0 + j*us
// (j < U), interleaved so that one thread has U independent butterfly chains in flight.
template <int LOGN, int R, bool FIRST, bool LAST, int U, class Ld, class St>
BFV_HD void fwd_unit(uint64_t* s, int u0, int us, int L, const ulonglong2* tw, uint64_t q, const Ld& ld,
                     const St& st) {
  constexpr int K = 1 << R;
  const int shift = LOGN - L - R;  // smallest gap of the pass is 2^shift
  int base[U], sbase[U], gl[U];
  uint64_t x[U][K];
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const int u = u0 + j * us;
    const int o = u & ((1 << shift) - 1);
    gl[j] = u >> shift;
    base[j] = (gl[j] << (LOGN - L)) + o;
    sbase[j] = spad(base[j]);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (FIRST)
        x[j][k] = ld(base[j] + (k << shift));
      else
        x[j][k] = s[spad_unit(base[j], sbase[j], k << shift)];
    }
  }
  const uint64_t two_q = 2 * q;
#pragma unroll
  for (int t = 0; t < R; ++t) {
    const int hs = R - t - 1;  // half = 2^hs pairs per twiddle group
#pragma unroll
    for (int pr = 0; pr < K / 2; ++pr) {
      const int jj = pr >> hs, kk = pr & ((1 << hs) - 1);
      const int k = (jj << (hs + 1)) + kk;
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const ulonglong2 w = tw[(1 << (L + t)) + (gl[j] << t) + jj];
        uint64_t a = x[j][k];
        if (a >= two_q) a -= two_q;
        const uint64_t b = shoup_lazy(x[j][k + (1 << hs)], w.x, w.y, q);
        x[j][k] = a + b;
        x[j][k + (1 << hs)] = a + two_q - b;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < U; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (LAST)
        st(base[j] + (k << shift), reduce_4q(x[j][k], q));
      else
        s[spad_unit(base[j], sbase[j], k << shift)] = x[j][k];
    }
}

// U radix-2^R Gentleman-Sande units of the inverse pass starting at level L.
template <int LOGN, int R, bool FIRST, bool LAST, int U, class Ld, class St>
BFV_HD void inv_unit(uint64_t* s, int u0, int us, int L, const ulonglong2* tw, uint64_t q, uint64_t invn,
                     uint64_t invn_q, const Ld& ld, const St& st) {
  constexpr int K = 1 << R;
  constexpr int N = 1 << LOGN;
  int base[U], sbase[U], gg[U];
  uint64_t x[U][K];
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const int u = u0 + j * us;
    const int o = u & ((1 << L) - 1);
    gg[j] = u >> L;
    base[j] = (gg[j] << (L + R)) + o;
    sbase[j] = spad(base[j]);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (FIRST)
        x[j][k] = ld(base[j] + (k << L));
      else
        x[j][k] = s[spad_unit(base[j], sbase[j], k << L)];
    }
  }
  const uint64_t two_q = 2 * q;
#pragma unroll
  for (int t = 0; t < R; ++t) {
    const int l = L + t;
#pragma unroll
    for (int pr = 0; pr < K / 2; ++pr) {
      const int jj = pr >> t, kk = pr & ((1 << t) - 1);
      const int k = (jj << (t + 1)) + kk;
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const ulonglong2 w = tw[N - (N >> l) + 1 + (gg[j] << (R - t - 1)) + jj];
        const uint64_t a = x[j][k], b = x[j][k + (1 << t)];
        uint64_t sum = a + b;
        if (sum >= two_q) sum -= two_q;
        x[j][k] = sum;
        x[j][k + (1 << t)] = shoup_lazy(a + two_q - b, w.x, w.y, q);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < U; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (LAST)
        st(base[j] + (k << L), shoup(x[j][k], invn, invn_q, q));
      else
        s[spad_unit(base[j], sbase[j], k << L)] = x[j][k];
    }
}

// Executors: device (threads of one block + __syncthreads) and host (all units in turn).
#if defined(__CUDACC__)
struct BlockExec {
  template <class F>
  __device__ __forceinline__ void run(int units, F&& f) const {
    for (int u = threadIdx.x; u < units; u += blockDim.x) f(u);
  }
  // f(u0, us) covers units u0 and u0 + us; every unit once when units % (2 blockDim) == 0,
  // else each unit alone through f1(u).
  template <class F2, class F1>
  __device__ __forceinline__ void run2(int units, F2&& f2, F1&& f1) const {
    const int t = blockDim.x;
    if (units % (2 * t) == 0) {
      for (int u = threadIdx.x; u < units; u += 2 * t) f2(u, t);
    } else {
      for (int u = threadIdx.x; u < units; u += t) f1(u);
    }
  }
  __device__ __forceinline__ void sync() const { __syncthreads(); }
};
#endif
struct HostExec {
  template <class F>
  void run(int units, F&& f) const {
    for (int u = 0; u < units; ++u) f(u);
  }
  // the pairs of a block of units/2 threads: (u, u + units/2)
  template <class F2, class F1>
  void run2(int units, F2&& f2, F1&& f1) const {
    if (units % 2 == 0) {
      const int t = units / 2;
      for (int u = 0; u < t; ++u) f2(u, t);
    } else {
      for (int u = 0; u < units; ++u) f1(u);
    }
  }
  void sync() const {}
};

// Units per thread per pass: two interleaved units at n = 16384 (one 512-thread block per SM,
// registers to spare); one below, where three blocks share an SM under an 80-register cap.
template <int LOGN>
struct DualUnits {
  static constexpr bool value = LOGN >= 14;
};

template <int LOGN, int MAXR, int P, class Ex, class Ld, class St>
BFV_HD void fwd_passes(const Ex& ex, uint64_t* s, const ulonglong2* tw, uint64_t q, const Ld& ld,
                       const St& st) {
  using S = Schedule<LOGN, MAXR>;
  if constexpr (P < S::passes) {
    constexpr int R = S::fwd_r(P);
    constexpr int L = S::fwd_level(P);
    constexpr bool first = P == 0, last = P == S::passes - 1;
    if constexpr (DualUnits<LOGN>::value)
      ex.run2(
          1 << (LOGN - R), [&](int u0, int us) { fwd_unit<LOGN, R, first, last, 2>(s, u0, us, L, tw, q, ld, st); },
          [&](int u) { fwd_unit<LOGN, R, first, last, 1>(s, u, 0, L, tw, q, ld, st); });
    else
      ex.run(1 << (LOGN - R), [&](int u) { fwd_unit<LOGN, R, first, last, 1>(s, u, 0, L, tw, q, ld, st); });
    ex.sync();
    fwd_passes<LOGN, MAXR, P + 1>(ex, s, tw, q, ld, st);
  }
}

template <int LOGN, int MAXR, int P, class Ex, class Ld, class St>
BFV_HD void inv_passes(const Ex& ex, uint64_t* s, const ulonglong2* tw, uint64_t q, uint64_t invn,
                       uint64_t invn_q, const Ld& ld, const St& st) {
  using S = Schedule<LOGN, MAXR>;
  if constexpr (P < S::passes) {
    constexpr int R = S::inv_r(P);
    constexpr int L = S::inv_level(P);
    constexpr bool first = P == 0, last = P == S::passes - 1;
    if constexpr (DualUnits<LOGN>::value)
      ex.run2(
          1 << (LOGN - R),
          [&](int u0, int us) { inv_unit<LOGN, R, first, last, 2>(s, u0, us, L, tw, q, invn, invn_q, ld, st); },
          [&](int u) { inv_unit<LOGN, R, first, last, 1>(s, u, 0, L, tw, q, invn, invn_q, ld, st); });
    else
      ex.run(1 << (LOGN - R),
             [&](int u) { inv_unit<LOGN, R, first, last, 1>(s, u, 0, L, tw, q, invn, invn_q, ld, st); });
    ex.sync();
    inv_passes<LOGN, MAXR, P + 1>(ex, s, tw, q, invn, invn_q, ld, st);
  }
}

// Forward NTT of one limb: ld(i) gives input coefficient i (< 4q), st(i, v) receives
// canonical NTT slot i.  Ends with a block-wide barrier.  The block needs at most
// n >> MAXR threads' worth of units per pass (any block size up to that works).
// The first forward pass reads each unit's words n/2^R apart, so consecutive threads
// read consecutive words.  Its last pass writes 2^R contiguous words per thread; with
// STAGE_OUT the results go to shared memory first and st(i, v) is called in index order
// (consecutive threads, consecutive i), which coalesces global stores.  Storers that
// write shared memory themselves pass STAGE_OUT = false.
template <int LOGN, int MAXR = 4, bool STAGE_OUT = true, class Ex, class Ld, class St>
BFV_HD void ntt_forward(const Ex& ex, uint64_t* s, const ulonglong2* tw, const Modulus& m, const Ld& ld,
                        const St& st) {
  if constexpr (STAGE_OUT) {
    auto to_smem = [s](int i, uint64_t v) { s[spad(i)] = v; };
    fwd_passes<LOGN, MAXR, 0>(ex, s, tw, m.q, ld, to_smem);
    ex.run(1 << LOGN, [&](int i) { st(i, s[spad(i)]); });
    ex.sync();
  } else {
    fwd_passes<LOGN, MAXR, 0>(ex, s, tw, m.q, ld, st);
  }
}

// Inverse NTT of one limb: ld(i) gives NTT slot i (< 2q), st(i, v) receives canonical
// coefficient i.  Ends with a block-wide barrier.  Its first pass reads 2^R contiguous
// words per thread; with STAGE_IN, ld(i) is called in index order into shared memory
// first (coalesced global loads, and each word of a fused prologue computed once).
// Loaders that read shared memory themselves pass STAGE_IN = false.
template <int LOGN, int MAXR = 4, bool STAGE_IN = true, class Ex, class Ld, class St>
BFV_HD void ntt_inverse(const Ex& ex, uint64_t* s, const ulonglong2* tw, const Modulus& m, const Ld& ld,
                        const St& st) {
  if constexpr (STAGE_IN) {
    ex.run(1 << LOGN, [&](int i) { s[spad(i)] = ld(i); });
    ex.sync();
    auto from_smem = [s](int i) { return s[spad(i)]; };
    inv_passes<LOGN, MAXR, 0>(ex, s, tw, m.q, m.invn, m.invn_q, from_smem, st);
  } else {
    inv_passes<LOGN, MAXR, 0>(ex, s, tw, m.q, m.invn, m.invn_q, ld, st);
  }
}

// Bit reversal of an index of LOGN bits.
BFV_HD int bit_reverse(int x, int logn) {
#if defined(__CUDA_ARCH__)
  return (int)(__brev((unsigned)x) >> (32 - logn));
#else
  unsigned r = 0;
  for (int i = 0; i < logn; ++i) r |= ((unsigned)(x >> i) & 1u) << (logn - 1 - i);
  return (int)r;
#endif
}

// NTT-slot permutation of the Galois automorphism X -> X^g: with slot i holding the
// evaluation at psi^(2 brv(i)+1), NTT(sigma_g a)[i] = NTT(a)[galois_slot(i)].
BFV_HD int galois_slot(int i, uint32_t g, int logn) {
  const uint32_t two_n_mask = (2u << logn) - 1u;
  const uint32_t e = ((2u * (uint32_t)bit_reverse(i, logn) + 1u) * g) & two_n_mask;
  return bit_reverse((int)(e >> 1), logn);
}

}  // namespace bfvgpu
