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
#include "f64mod.cuh"

#if defined(__CUDACC__)
#include <cooperative_groups.h>
#endif
#if !defined(__CUDACC__)
struct ulonglong2 {
  unsigned long long x, y;
};
struct double2 {
  double x, y;
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
// SPLIT: the unit belongs to half `rank` of a transform of size 2^(LOGN+1) split between the
// two blocks of a cluster (level 0 done by fwd_cross): its level L + t is the full
// transform's level L + t + 1 and its groups start at rank * 2^(L+t).
template <int LOGN, int R, bool FIRST, bool LAST, int U, bool SPLIT, class Ld, class St>
BFV_HD void fwd_unit(uint64_t* s, int u0, int us, int L, const ulonglong2* tw, uint64_t q, const Ld& ld,
                     const St& st, int rank) {
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
        const int ti = SPLIT ? (1 << (L + t + 1)) + (rank << (L + t)) + (gl[j] << t) + jj
                             : (1 << (L + t)) + (gl[j] << t) + jj;
        const ulonglong2 w = tw[ti];
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
// SPLIT: the unit belongs to half `rank` of a transform of size 2^(LOGN+1) split between two
// blocks (the last level done by inv_cross): levels keep their gaps, the full transform's
// table offsets apply and its groups at level l start at rank * 2^(LOGN-1-l).
template <int LOGN, int R, bool FIRST, bool LAST, int U, bool SPLIT, class Ld, class St>
BFV_HD void inv_unit(uint64_t* s, int u0, int us, int L, const ulonglong2* tw, uint64_t q, uint64_t invn,
                     uint64_t invn_q, const Ld& ld, const St& st, int rank) {
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
        const int ti = SPLIT ? 2 * N - ((2 * N) >> l) + 1 + (rank << (LOGN - 1 - l)) + (gg[j] << (R - t - 1)) + jj
                             : N - (N >> l) + 1 + (gg[j] << (R - t - 1)) + jj;
        const ulonglong2 w = tw[ti];
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
  static constexpr bool kSplit = false;
};

// A limb split between the two blocks of a cluster (launched with cluster dimension 2, the
// block pair of a limb consecutive): each block holds half the limb in its shared memory
// and reaches the other half through distributed shared memory.
struct ClusterPairExec : BlockExec {
  static constexpr bool kSplit = true;
  __device__ __forceinline__ int rank() const { return (int)cooperative_groups::this_cluster().block_rank(); }
  // block r's buffer, s being this block's own
  __device__ __forceinline__ uint64_t* buffer(uint64_t* s, int r) const {
    return r == rank() ? s : cooperative_groups::this_cluster().map_shared_rank(s, (unsigned)r);
  }
  __device__ __forceinline__ void cluster_sync() const { cooperative_groups::this_cluster().sync(); }
  template <class F>
  __device__ __forceinline__ void for_ranks(uint64_t* s, F&& f) const {
    f(rank(), s);
  }
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
  static constexpr bool kSplit = false;
};

// The host form of ClusterPairExec: s holds both halves' buffers, `words` apart; every phase
// between cluster barriers runs for block 0, then block 1 (the phases of the two blocks read
// and write disjoint words, so running them in turn is exact).
struct HostPairExec : HostExec {
  int words = 0;
  static constexpr bool kSplit = true;
  uint64_t* buffer(uint64_t* s, int r) const { return s + (size_t)r * words; }
  void cluster_sync() const {}
  template <class F>
  void for_ranks(uint64_t* s, F&& f) const {
    f(0, s);
    f(1, s + words);
  }
};

// Units per thread per pass: two interleaved units at n = 16384 (one 512-thread block per SM,
// registers to spare); one below, where three blocks share an SM under an 80-register cap.
template <int LOGN>
struct DualUnits {
  static constexpr bool value = LOGN >= 14;
};

// SPLIT: the passes of one half of a split transform (after fwd_cross): the first pass reads
// shared memory, the twiddles are the full transform's.
template <int LOGN, int MAXR, int P, bool SPLIT = false, class Ex, class Ld, class St>
BFV_HD void fwd_passes(const Ex& ex, uint64_t* s, const ulonglong2* tw, uint64_t q, const Ld& ld,
                       const St& st, int rank = 0) {
  using S = Schedule<LOGN, MAXR>;
  if constexpr (P < S::passes) {
    constexpr int R = S::fwd_r(P);
    constexpr int L = S::fwd_level(P);
    constexpr bool first = P == 0 && !SPLIT, last = P == S::passes - 1;
    if constexpr (DualUnits<LOGN>::value)
      ex.run2(
          1 << (LOGN - R),
          [&](int u0, int us) { fwd_unit<LOGN, R, first, last, 2, SPLIT>(s, u0, us, L, tw, q, ld, st, rank); },
          [&](int u) { fwd_unit<LOGN, R, first, last, 1, SPLIT>(s, u, 0, L, tw, q, ld, st, rank); });
    else
      ex.run(1 << (LOGN - R),
             [&](int u) { fwd_unit<LOGN, R, first, last, 1, SPLIT>(s, u, 0, L, tw, q, ld, st, rank); });
    ex.sync();
    fwd_passes<LOGN, MAXR, P + 1, SPLIT>(ex, s, tw, q, ld, st, rank);
  }
}

// SPLIT: the passes of one half of a split transform (before inv_cross): the last pass keeps
// its results in shared memory, unscaled, the twiddles are the full transform's.
template <int LOGN, int MAXR, int P, bool SPLIT = false, class Ex, class Ld, class St>
BFV_HD void inv_passes(const Ex& ex, uint64_t* s, const ulonglong2* tw, uint64_t q, uint64_t invn,
                       uint64_t invn_q, const Ld& ld, const St& st, int rank = 0) {
  using S = Schedule<LOGN, MAXR>;
  if constexpr (P < S::passes) {
    constexpr int R = S::inv_r(P);
    constexpr int L = S::inv_level(P);
    constexpr bool first = P == 0, last = P == S::passes - 1 && !SPLIT;
    if constexpr (DualUnits<LOGN>::value)
      ex.run2(
          1 << (LOGN - R),
          [&](int u0, int us) {
            inv_unit<LOGN, R, first, last, 2, SPLIT>(s, u0, us, L, tw, q, invn, invn_q, ld, st, rank);
          },
          [&](int u) { inv_unit<LOGN, R, first, last, 1, SPLIT>(s, u, 0, L, tw, q, invn, invn_q, ld, st, rank); });
    else
      ex.run(1 << (LOGN - R),
             [&](int u) { inv_unit<LOGN, R, first, last, 1, SPLIT>(s, u, 0, L, tw, q, invn, invn_q, ld, st, rank); });
    ex.sync();
    inv_passes<LOGN, MAXR, P + 1, SPLIT>(ex, s, tw, q, invn, invn_q, ld, st, rank);
  }
}

// ---- a limb split between two blocks ------------------------------------------------------
// Half r (of H = n/2 words) lives in block r's shared memory.  The one level whose pairs
// straddle the halves (forward level 0, inverse level log n - 1, gap H) runs as a "cross"
// step: block r takes the pairs j in [r H/2, (r+1) H/2) and writes both outputs, one into its
// own half and one into the other block's.  The two blocks' read and write sets are disjoint,
// so a cluster barrier before and after the step is all the ordering it needs.
template <int LOGH, class Ex>
BFV_HD void fwd_cross(const Ex& ex, uint64_t* s0, uint64_t* s1, int rank, const ulonglong2* tw, uint64_t q) {
  constexpr int H = 1 << LOGH;
  const ulonglong2 w = tw[1];
  const uint64_t two_q = 2 * q;
  ex.run(H / 2, [&](int jj) {
    const int sj = spad(rank * (H / 2) + jj);
    uint64_t a = s0[sj];
    if (a >= two_q) a -= two_q;
    const uint64_t t = shoup_lazy(s1[sj], w.x, w.y, q);
    s0[sj] = a + t;
    s1[sj] = a + two_q - t;
  });
}
template <int LOGH, class Ex>
BFV_HD void inv_cross(const Ex& ex, uint64_t* s0, uint64_t* s1, int rank, const ulonglong2* tw, uint64_t q) {
  constexpr int H = 1 << LOGH;
  const ulonglong2 w = tw[2 * H - 1];  // the last level's single entry, n - (n >> (log n - 1)) + 1
  const uint64_t two_q = 2 * q;
  ex.run(H / 2, [&](int jj) {
    const int sj = spad(rank * (H / 2) + jj);
    const uint64_t a = s0[sj], b = s1[sj];
    uint64_t sum = a + b;
    if (sum >= two_q) sum -= two_q;
    s0[sj] = sum;
    s1[sj] = shoup_lazy(a + two_q - b, w.x, w.y, q);
  });
}

// Forward NTT of a limb split between two blocks: stage each half through ld, the cross
// level, then the remaining log n - 1 levels on each half (the schedule of an n/2 transform
// with the full transform's twiddles), stored in index order through st (global indices).
template <int LOGN, int MAXR, class Ex, class Ld, class St>
BFV_HD void ntt_forward_split(const Ex& ex, uint64_t* s, const ulonglong2* tw, const Modulus& m, const Ld& ld,
                              const St& st) {
  constexpr int LOGH = LOGN - 1, H = 1 << LOGH;
  ex.for_ranks(s, [&](int r, uint64_t* own) {
    ex.run(H, [&](int j) { own[spad(j)] = ld(r * H + j); });
  });
  ex.cluster_sync();
  ex.for_ranks(s, [&](int r, uint64_t*) { fwd_cross<LOGH>(ex, ex.buffer(s, 0), ex.buffer(s, 1), r, tw, m.q); });
  ex.cluster_sync();
  ex.for_ranks(s, [&](int r, uint64_t* own) {
    auto unused = [](int) { return uint64_t(0); };
    auto to_smem = [own](int j, uint64_t v) { own[spad(j)] = v; };
    fwd_passes<LOGH, MAXR, 0, true>(ex, own, tw, m.q, unused, to_smem, r);
    ex.run(H, [&](int j) { st(r * H + j, own[spad(j)]); });
    ex.sync();
  });
}

// Inverse NTT of a limb split between two blocks: each half staged through ld and taken
// through the first log n - 1 levels, the cross level, then scaled by n^-1 and stored in
// index order through st (global indices).
template <int LOGN, int MAXR, class Ex, class Ld, class St>
BFV_HD void ntt_inverse_split(const Ex& ex, uint64_t* s, const ulonglong2* tw, const Modulus& m, const Ld& ld,
                              const St& st) {
  constexpr int LOGH = LOGN - 1, H = 1 << LOGH;
  ex.for_ranks(s, [&](int r, uint64_t* own) {
    ex.run(H, [&](int j) { own[spad(j)] = ld(r * H + j); });
    ex.sync();
    auto from_smem = [own](int j) { return own[spad(j)]; };
    auto unused = [](int, uint64_t) {};
    inv_passes<LOGH, MAXR, 0, true>(ex, own, tw, m.q, m.invn, m.invn_q, from_smem, unused, r);
  });
  ex.cluster_sync();
  ex.for_ranks(s, [&](int r, uint64_t*) { inv_cross<LOGH>(ex, ex.buffer(s, 0), ex.buffer(s, 1), r, tw, m.q); });
  ex.cluster_sync();
  ex.for_ranks(s, [&](int r, uint64_t* own) {
    ex.run(H, [&](int j) { st(r * H + j, shoup(own[spad(j)], m.invn, m.invn_q, m.q)); });
    ex.sync();
  });
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
  if constexpr (Ex::kSplit) {
    static_assert(STAGE_OUT, "a split transform stores its output from shared memory");
    ntt_forward_split<LOGN, MAXR>(ex, s, tw, m, ld, st);
  } else if constexpr (STAGE_OUT) {
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
  if constexpr (Ex::kSplit) {
    static_assert(STAGE_IN, "a split transform stages its input into shared memory");
    ntt_inverse_split<LOGN, MAXR>(ex, s, tw, m, ld, st);
  } else if constexpr (STAGE_IN) {
    ex.run(1 << LOGN, [&](int i) { s[spad(i)] = ld(i); });
    ex.sync();
    auto from_smem = [s](int i) { return s[spad(i)]; };
    inv_passes<LOGN, MAXR, 0>(ex, s, tw, m.q, m.invn, m.invn_q, from_smem, st);
  } else {
    inv_passes<LOGN, MAXR, 0>(ex, s, tw, m.q, m.invn, m.invn_q, ld, st);
  }
}

// ---- the same transforms on the FP64 pipe (primes below 2^50, f64mod.cuh) -----------------
// Shared memory holds integer-valued doubles (centred representatives) in place of words;
// twiddle tables hold {w_c, fl(w_c / q)} with w_c the centred twiddle (f64_twiddles), at the
// integer tables' indices.  Bounds (q < 2^50): a product is at most 0.75 q whatever its input
// (below 2^52).  Forward: each pass first reduces its level-0 upper inputs to |v| <= (q+1)/2
// (the lower inputs only enter products), so after a radix-2^R pass |v| <= (0.5 + 0.75 R) q + 1,
// below 4q for R <= 4.  Inverse: each pass reduces all its inputs to |v| <= (q+1)/2; a level at
// most doubles the sums, so after a radix-8 pass |v| <= 4q + 4 < 2^52 and every product input
// stays in range.  All sums stay below 2^53, so every operation is exact and the canonical
// results equal the integer transforms' word for word.
struct F64Prime {
  double q, qinv;
};
BFV_HD F64Prime f64_prime(const Modulus& m) { return F64Prime{u64_to_f64(m.q), m.f64_qinv}; }

// Twiddle load on the read-only path (no kernel writes the tables), which lets the compiler
// issue it ahead of the shared-memory stores of the previous unit.
BFV_HD double2 ldg_tw(const double2* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}

// Host setup: the FP64 twiddle table {w_c, fl(w_c / q)} of an integer table {w, w'} (n entries).
inline void f64_twiddles(const ulonglong2* tw, uint64_t q, size_t n, double2* out) {
  const double qd = (double)q;
  for (size_t i = 0; i < n; ++i) {
    out[i].x = centred_f64(tw[i].x, q);
    out[i].y = out[i].x / qd;
  }
}

// U interleaved units per thread (u0 + j us), so that one thread has U independent chains of
// butterflies -- and of twiddle loads -- in flight.
template <int LOGN, int R, bool FIRST, bool LAST, int U, class Ld, class St>
BFV_HD void fwd_unit_f64(double* s, int u0, int us, int L, const double2* tw, F64Prime fp, const Ld& ld,
                         const St& st) {
  constexpr int K = 1 << R;
  const int shift = LOGN - L - R;
  int base[U], sbase[U], gl[U];
  double x[U][K];
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
#pragma unroll
  for (int t = 0; t < R; ++t) {
    const int hs = R - t - 1;
#pragma unroll
    for (int pr = 0; pr < K / 2; ++pr) {
      const int jj = pr >> hs, kk = pr & ((1 << hs) - 1);
      const int k = (jj << (hs + 1)) + kk;
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const double2 w = ldg_tw(tw + (1 << (L + t)) + (gl[j] << t) + jj);
        double a = x[j][k];
        if (t == 0) a = reduce_f64(a, fp.q, fp.qinv);
        const double b = mulmod_f64(x[j][k + (1 << hs)], w.x, w.y, fp.q);
        x[j][k] = f64_add(a, b);
        x[j][k + (1 << hs)] = f64_sub(a, b);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < U; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (LAST)
        st(base[j] + (k << shift), x[j][k]);
      else
        s[spad_unit(base[j], sbase[j], k << shift)] = x[j][k];
    }
}

template <int LOGN, int R, bool FIRST, bool LAST, int U, class Ld, class St>
BFV_HD void inv_unit_f64(double* s, int u0, int us, int L, const double2* tw, F64Prime fp, double invn,
                         double invn_q, const Ld& ld, const St& st) {
  static_assert(R <= 3, "inverse FP64 passes are at most radix 8 (sums grow 2x per level)");
  constexpr int K = 1 << R;
  constexpr int N = 1 << LOGN;
  int base[U], sbase[U], gg[U];
  double x[U][K];
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const int u = u0 + j * us;
    const int o = u & ((1 << L) - 1);
    gg[j] = u >> L;
    base[j] = (gg[j] << (L + R)) + o;
    sbase[j] = spad(base[j]);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const double v = FIRST ? ld(base[j] + (k << L)) : s[spad_unit(base[j], sbase[j], k << L)];
      x[j][k] = reduce_f64(v, fp.q, fp.qinv);
    }
  }
#pragma unroll
  for (int t = 0; t < R; ++t) {
    const int l = L + t;
#pragma unroll
    for (int pr = 0; pr < K / 2; ++pr) {
      const int jj = pr >> t, kk = pr & ((1 << t) - 1);
      const int k = (jj << (t + 1)) + kk;
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const double2 w = ldg_tw(tw + N - (N >> l) + 1 + (gg[j] << (R - t - 1)) + jj);
        const double a = x[j][k], b = x[j][k + (1 << t)];
        x[j][k] = f64_add(a, b);
        x[j][k + (1 << t)] = mulmod_f64(f64_sub(a, b), w.x, w.y, fp.q);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < U; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (LAST)
        st(base[j] + (k << L), mulmod_f64(x[j][k], invn, invn_q, fp.q));
      else
        s[spad_unit(base[j], sbase[j], k << L)] = x[j][k];
    }
}

// Units per thread per pass of the FP64 transforms: two interleaved units (the FP64 unit
// holds its 8 values in 16 registers, so two fit under the 80-register cap of three blocks
// per SM), which doubles the loads and butterfly chains each thread has in flight; the last
// pass, whose storer carries the callers' epilogues, keeps one unit.
template <int LOGN>
struct DualUnitsF64 {
  static constexpr bool value = LOGN >= 12;
};

template <int LOGN, int MAXR, int P, class Ex, class Ld, class St>
BFV_HD void fwd_passes_f64(const Ex& ex, double* s, const double2* tw, F64Prime fp, const Ld& ld, const St& st) {
  using S = Schedule<LOGN, MAXR>;
  if constexpr (P < S::passes) {
    constexpr int R = S::fwd_r(P);
    constexpr int L = S::fwd_level(P);
    constexpr bool first = P == 0, last = P == S::passes - 1;
    if constexpr (DualUnitsF64<LOGN>::value && !last)
      ex.run2(
          1 << (LOGN - R),
          [&](int u0, int us) { fwd_unit_f64<LOGN, R, first, last, 2>(s, u0, us, L, tw, fp, ld, st); },
          [&](int u) { fwd_unit_f64<LOGN, R, first, last, 1>(s, u, 0, L, tw, fp, ld, st); });
    else
      ex.run(1 << (LOGN - R), [&](int u) { fwd_unit_f64<LOGN, R, first, last, 1>(s, u, 0, L, tw, fp, ld, st); });
    ex.sync();
    fwd_passes_f64<LOGN, MAXR, P + 1>(ex, s, tw, fp, ld, st);
  }
}
template <int LOGN, int MAXR, int P, class Ex, class Ld, class St>
BFV_HD void inv_passes_f64(const Ex& ex, double* s, const double2* tw, F64Prime fp, double invn, double invn_q,
                           const Ld& ld, const St& st) {
  using S = Schedule<LOGN, MAXR>;
  if constexpr (P < S::passes) {
    constexpr int R = S::inv_r(P);
    constexpr int L = S::inv_level(P);
    constexpr bool first = P == 0, last = P == S::passes - 1;
    if constexpr (DualUnitsF64<LOGN>::value && !last)
      ex.run2(
          1 << (LOGN - R),
          [&](int u0, int us) {
            inv_unit_f64<LOGN, R, first, last, 2>(s, u0, us, L, tw, fp, invn, invn_q, ld, st);
          },
          [&](int u) { inv_unit_f64<LOGN, R, first, last, 1>(s, u, 0, L, tw, fp, invn, invn_q, ld, st); });
    else
      ex.run(1 << (LOGN - R),
             [&](int u) { inv_unit_f64<LOGN, R, first, last, 1>(s, u, 0, L, tw, fp, invn, invn_q, ld, st); });
    ex.sync();
    inv_passes_f64<LOGN, MAXR, P + 1>(ex, s, tw, fp, invn, invn_q, ld, st);
  }
}

// Forward NTT of one limb on the FP64 pipe: ld(i) gives input coefficient i as a double with
// |v| < 2^52 (any representative), st(i, v) receives NTT slot i as a representative with
// |v| < 4q (canon_f64 makes it canonical).  STAGE_OUT as for ntt_forward.  Ends with a
// block-wide barrier.  s: the block's shared words, reused as doubles.
template <int LOGN, int MAXR = 3, bool STAGE_OUT = true, class Ex, class Ld, class St>
BFV_HD void ntt_forward_f64(const Ex& ex, uint64_t* s, const double2* tw, const Modulus& m, const Ld& ld,
                            const St& st) {
  static_assert(!Ex::kSplit, "FP64 transforms run one limb per block");
  double* d = reinterpret_cast<double*>(s);
  const F64Prime fp = f64_prime(m);
  if constexpr (STAGE_OUT) {
    auto to_smem = [d](int i, double v) { d[spad(i)] = v; };
    fwd_passes_f64<LOGN, MAXR, 0>(ex, d, tw, fp, ld, to_smem);
    ex.run(1 << LOGN, [&](int i) { st(i, d[spad(i)]); });
    ex.sync();
  } else {
    fwd_passes_f64<LOGN, MAXR, 0>(ex, d, tw, fp, ld, st);
  }
}

// Inverse NTT of one limb on the FP64 pipe: ld(i) gives NTT slot i as a double with
// |v| < 2^52, st(i, v) receives coefficient i times n^-1 as a representative with
// |v| <= 0.75 q.  STAGE_IN as for ntt_inverse.  Ends with a block-wide barrier.
template <int LOGN, int MAXR = 3, bool STAGE_IN = true, class Ex, class Ld, class St>
BFV_HD void ntt_inverse_f64(const Ex& ex, uint64_t* s, const double2* tw, const Modulus& m, const Ld& ld,
                            const St& st) {
  static_assert(!Ex::kSplit, "FP64 transforms run one limb per block");
  double* d = reinterpret_cast<double*>(s);
  const F64Prime fp = f64_prime(m);
  if constexpr (STAGE_IN) {
    ex.run(1 << LOGN, [&](int i) { d[spad(i)] = ld(i); });
    ex.sync();
    auto from_smem = [d](int i) { return d[spad(i)]; };
    inv_passes_f64<LOGN, MAXR, 0>(ex, d, tw, fp, m.f64_invn, m.f64_invn_q, from_smem, st);
  } else {
    inv_passes_f64<LOGN, MAXR, 0>(ex, d, tw, fp, m.f64_invn, m.f64_invn_q, ld, st);
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
