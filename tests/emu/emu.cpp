// Host emulation of the CUDA kernel bodies (TEST INFRASTRUCTURE).
//
// Compiles privacy-rag_b200/csrc/block_ops.cuh with the host compiler and runs every
// thread block's work units in turn (HostExec), so the exact index arithmetic, pass
// schedule, prologues and epilogues of the kernels are checked against the CPU oracle
// without a GPU, and before any of them is launched on one.  Constants (the 16-word
// per-prime records and the twiddle tables) come from the product library's host-only
// context, so they are the same values the kernels receive.
#include <cstdint>
#include <algorithm>
#include <cstring>
#include <vector>

#include "block_ops.cuh"
#include "f64mod.cuh"
#include "mac_tc.cuh"

using namespace bfvgpu;

namespace {
struct Tabs {
  std::vector<Modulus> mods;
  const ulonglong2* fwd;
  const ulonglong2* inv;
  std::vector<double2> fwd64_v, inv64_v;  // FP64 twiddles of the primes with f64 set
  const double2* fwd64 = nullptr;
  const double2* inv64 = nullptr;
};
Tabs tabs(uint32_t k, const uint64_t* mods16, const uint64_t* fwd, const uint64_t* inv, int logn) {
  Tabs t;
  t.mods.resize(k);
  std::memcpy(t.mods.data(), mods16, k * sizeof(Modulus));
  t.fwd = reinterpret_cast<const ulonglong2*>(fwd);
  t.inv = reinterpret_cast<const ulonglong2*>(inv);
  const size_t n = size_t(1) << logn;
  t.fwd64_v.assign(k * n, double2{0.0, 0.0});
  t.inv64_v.assign(k * n, double2{0.0, 0.0});
  for (uint32_t p = 0; p < k; ++p) {
    if (!t.mods[p].f64) continue;
    f64_twiddles(t.fwd + p * n, t.mods[p].q, n, t.fwd64_v.data() + p * n);
    f64_twiddles(t.inv + p * n, t.mods[p].q, n, t.inv64_v.data() + p * n);
  }
  t.fwd64 = t.fwd64_v.data();
  t.inv64 = t.inv64_v.data();
  return t;
}
uint32_t inv_mod_2n(uint32_t g, uint32_t two_n) {
  uint64_t r = 1, b = g % two_n, e = two_n / 2 - 1;
  while (e) {
    if (e & 1) r = (r * b) % two_n;
    b = (b * b) % two_n;
    e >>= 1;
  }
  return (uint32_t)r;
}
}  // namespace

#define EMU_DISPATCH(LOGN_VAR, ...)                        \
  switch (LOGN_VAR) {                                      \
    case 5: { constexpr int L_ = 5; __VA_ARGS__; } break;   \
    case 6: { constexpr int L_ = 6; __VA_ARGS__; } break;   \
    case 12: { constexpr int L_ = 12; __VA_ARGS__; } break; \
    case 13: { constexpr int L_ = 13; __VA_ARGS__; } break; \
    case 14: { constexpr int L_ = 14; __VA_ARGS__; } break; \
    default: return -1;                                    \
  }

// One launch of the product kernel for T tiles: every block's staging (zero fill where the
// source is null), chunk loop and store, run thread by thread.
template <int T, int TH>
static void emu_mac_launch(const uint64_t* in, const uint64_t* w, uint64_t* out, uint32_t inputs, uint32_t groups,
                           uint32_t dk, int logn, const Modulus* mods) {
  using S = MacShape<T, TH>;
  const uint32_t gblocks = (groups + S::GB - 1) / S::GB, zchunks = (1u << logn) >> 5;
  const uint32_t chunks = (inputs + S::kBc - 1) / S::kBc;
  struct Thread {
    Mac30 acc[TH][2];
    Acc128 A[TH][2];
  };
  std::vector<uint64_t> buf(S::kBufWords);
  std::vector<Thread> th(S::kThreads);
  for (uint64_t blk = 0; blk < (uint64_t)dk * zchunks * gblocks; ++blk) {
    const uint32_t gq = blk % gblocks, r = blk / gblocks;
    const uint32_t p = r / zchunks, z0 = (r % zchunks) * 32, g0 = gq * S::GB;
    std::fill(th.begin(), th.end(), Thread{});
    for (uint32_t k = 0; k < chunks; ++k) {
      for (int seg = 0; seg < S::kSegs; ++seg) {
        int dst = -1;
        const uint64_t* src = mac_stage_src<T, TH>(seg, k * S::kBc, in, w, inputs, groups, g0, p, z0, dk, logn, &dst);
        if (dst < 0 || dst + 2 > S::kBufWords || (dst & 1)) throw 1;
        buf[dst] = src ? src[0] : 0;
        buf[dst + 1] = src ? src[1] : 0;
      }
      for (int i = 0; i < S::kThreads; ++i) mac_chunk<T, TH>(buf.data(), i >> 5, i & 31, th[i].acc, th[i].A, mods[p], k);
    }
    for (int i = 0; i < S::kThreads; ++i)
      mac_store<T, TH>(out, i >> 5, i & 31, th[i].A, mods[p], groups, g0, p, z0, dk, logn);
  }
}

// One launch of the tensor-core product (8 tiles), unit by unit as the persistent kernel
// walks them: per slot pair the A boxes and per round the B box are built as the TMA writes
// them (dense box images, zero fill past the extents), the int8 MMA is evaluated from those
// images at the canonical MN-major layout without swizzle (operand byte (mn, k) at
// (mn/16)*K*16 + k*16 + mn%16), then every warp's TMEM drain (lane = TMEM lane of its
// quarter, 32-column loads), the byte-limb recombination of its slot and the shuffle
// reduce-scatter are replayed lane by lane, followed by the mod-q reduction, the output
// buffer and its flush.
template <int KPAD>
static void emu_mac_tc_launch(const uint64_t* in, const uint64_t* w, uint64_t* out, uint32_t inputs,
                              uint32_t groups, uint32_t dk, int logn, const Modulus* mods) {
  using S = tc::Smem<KPAD>;
  const uint32_t N = 1u << logn, zblocks = N / tc::kSlots;
  const uint32_t gchunks = (groups + tc::kGroups - 1) / tc::kGroups;
  const uint32_t units = dk * zblocks * gchunks;
  const uint64_t out_words = 8ull * groups * 2 * dk << logn;
  std::vector<uint8_t> A(2 * S::kABox), B(S::kBBox);
  std::vector<uint64_t> ob(tc::kSlots * 16 * tc::kGroups);
  std::vector<uint32_t> D(128 * 512);
  auto put = [](std::vector<uint8_t>& img, uint32_t box_base, uint32_t lin, uint64_t v) {
    const uint32_t off = box_base + lin;
    if (off + 8 > img.size() || (off & 7)) throw 2;
    std::memcpy(&img[off], &v, 8);
  };
  for (uint32_t u = 0; u < units; ++u) {
    uint32_t gc, p, z0;
    tc::unit_coords(u, gchunks, zblocks, &gc, &p, &z0);
    for (uint32_t zp = 0; zp < tc::kSlots / tc::kPair; ++zp) {
      const uint32_t z = z0 + zp * tc::kPair;
      if (z & 1) throw 5;  // TMA x coordinate: 16-byte multiple
      // A boxes: (z..z+1, c, t4 + 4 mb, b < KPAD, p)
      for (uint32_t mb = 0; mb < 2; ++mb)
        for (uint32_t b = 0; b < KPAD; ++b)
          for (uint32_t t4 = 0; t4 < 4; ++t4)
            for (uint32_t c = 0; c < 2; ++c)
              for (uint32_t zs = 0; zs < 2; ++zs) {
                const uint32_t t = 4 * mb + t4;
                const uint64_t v = b < inputs ? in[((((uint64_t)t * inputs + b) * 2 + c) * dk + p) * N + z + zs] : 0;
                put(A, mb * S::kABox, tc::a_img<KPAD>(b, t4, c, zs), v);
              }
      for (uint32_t gr = 0; gr < tc::kRoundsPerPair; ++gr) {
        for (uint32_t b = 0; b < KPAD; ++b)
          for (uint32_t gl = 0; gl < tc::kGroupsRound; ++gl)
            for (uint32_t zs = 0; zs < 2; ++zs) {
              const uint32_t g = gc * tc::kGroups + gr * tc::kGroupsRound + gl;
              const uint64_t v = (b < inputs && g < groups) ? w[(((uint64_t)g * inputs + b) * dk + p) * N + z + zs] : 0;
              put(B, 0, tc::b_img<KPAD>(b, gl, zs), v);
            }
        // MMA: D[m][mb*256 + n] = sum_k A_mb[m][k] . B[k][n]
        for (uint32_t mb = 0; mb < 2; ++mb)
          for (uint32_t m = 0; m < 128; ++m)
            for (uint32_t n = 0; n < 256; ++n) {
              uint32_t acc = 0;
              for (uint32_t k = 0; k < KPAD; ++k)
                acc += (uint32_t)A[mb * S::kABox + (m >> 4) * KPAD * 16 + k * 16 + (m & 15)] *
                       (uint32_t)B[(n >> 4) * KPAD * 16 + k * 16 + (n & 15)];
              D[m * 512 + 256 * mb + n] = acc;
            }
        for (uint32_t warp = 0; warp < 16; ++warp) {
          const uint32_t quarter = warp & 3, mb = warp >> 3, gh = (warp >> 2) & 1;
          uint64_t vlo[32][8], vhi[32][8];
          for (uint32_t lane = 0; lane < 32; ++lane) {
            const uint32_t m = quarter * 32 + lane, zs = (m >> 3) & 1, i = m & 7;
            for (uint32_t h = 0; h < 4; ++h) {
              uint32_t cols[32];
              for (uint32_t c = 0; c < 32; ++c) cols[c] = D[m * 512 + 256 * mb + 128 * gh + 32 * h + c];
              tc::lane_values2(cols, zs, i, vlo[lane] + 2 * h, vhi[lane] + 2 * h);
            }
          }
          for (int lev = 4; lev >= 1; lev >>= 1) {
            uint64_t nlo[32][8], nhi[32][8], slo[32][8], shi[32][8];
            for (uint32_t lane = 0; lane < 32; ++lane) {
              const bool sel = (lane & 7) & lev;
              for (int q = 0; q < lev; ++q) {
                nlo[lane][q] = sel ? vlo[lane][q + lev] : vlo[lane][q];
                nhi[lane][q] = sel ? vhi[lane][q + lev] : vhi[lane][q];
                slo[lane][q] = sel ? vlo[lane][q] : vlo[lane][q + lev];
                shi[lane][q] = sel ? vhi[lane][q] : vhi[lane][q + lev];
              }
            }
            for (uint32_t lane = 0; lane < 32; ++lane)
              for (int q = 0; q < lev; ++q) {
                vlo[lane][q] = nlo[lane][q];
                vhi[lane][q] = nhi[lane][q];
                tc::add128(vlo[lane][q], vhi[lane][q], slo[lane ^ lev][q], shi[lane ^ lev][q]);
              }
          }
          for (uint32_t lane = 0; lane < 32; ++lane) {
            const uint32_t m = quarter * 32 + lane, tc4 = m >> 4, zs = (m >> 3) & 1, i = m & 7;
            ob[tc::out_buf_word(zp * tc::kPair + zs, mb * 8 + tc4, gr * tc::kGroupsRound + gh * 8 + i)] =
                reduce128(vlo[lane][0], vhi[lane][0], mods[p]);
          }
        }
      }
    }
    for (uint32_t tid = 0; tid < 512; ++tid) {
      const uint32_t rtc = tid >> 5, rgl = tid & 31, g = gc * tc::kGroups + rgl;
      if (g >= groups) continue;
      const uint64_t row = tc::out_row(rtc, g, groups, p, z0, dk, N);
      if ((row & 1) || row + tc::kSlots > out_words) throw 4;  // 16-byte stores
      for (uint32_t zz = 0; zz < tc::kSlots; ++zz) out[row + zz] = ob[tc::out_buf_word(zz, rtc, rgl)];
    }
  }
}

extern "C" {

int emu_ntt(int logn, uint32_t k, const uint64_t* mods16, const uint64_t* fwd, const uint64_t* inv, uint64_t* data,
            uint64_t polys, uint32_t prime_count, uint32_t prime_offset, int inverse) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < polys; ++b)
      op_ntt<L_>(HostExec{}, s.data(), b, inverse != 0, data, prime_count, prime_offset, T.mods.data(), T.fwd, T.inv,
                 T.fwd64, T.inv64);
  });
  return 0;
}

// The same batched transform with every limb split between a pair of blocks (the form the
// n = 16384 kernels launch as 2-block clusters): both halves' buffers side by side.
int emu_ntt_pair(int logn, uint32_t k, const uint64_t* mods16, const uint64_t* fwd, const uint64_t* inv, uint64_t* data,
                 uint64_t polys, uint32_t prime_count, uint32_t prime_offset, int inverse) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  EMU_DISPATCH(logn, {
    if constexpr (L_ >= 6) {
      HostPairExec ex;
      ex.words = SmemWords<L_ - 1>::value;
      std::vector<uint64_t> s(2 * (size_t)ex.words);
      for (uint64_t b = 0; b < polys; ++b)
        op_ntt<L_>(ex, s.data(), b, inverse != 0, data, prime_count, prime_offset, T.mods.data(), T.fwd, T.inv,
                   T.fwd64, T.inv64);
    }
  });
  return 0;
}

// cts [count][2][dk][n], key [dk][2][k][n] -> out [count][2][dk][n]
int emu_keyswitch(int logn, uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd, const uint64_t* inv,
                  const uint64_t* cts, uint64_t count, const uint64_t* key, uint32_t elt, uint64_t* out) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  const uint64_t n = 1ull << logn;
  std::vector<uint64_t> qjp((size_t)dk * k);
  for (uint32_t j = 0; j < dk; ++j)
    for (uint32_t p = 0; p < k; ++p) qjp[j * k + p] = T.mods[j].q % T.mods[p].q;
  std::vector<uint64_t> acc(count * 2 * k * n);
  const uint32_t ginv = inv_mod_2n(elt, 2 * (uint32_t)n);
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < count * k; ++b)
      op_ks_main<L_>(HostExec{}, s.data(), b, cts, key, acc.data(), elt, k, dk, T.mods.data(), qjp.data(), T.fwd,
                     T.inv, T.fwd64, T.inv64);
    std::vector<uint64_t> s2(n);
    for (uint64_t b = 0; b < count * dk; ++b)
      op_ks_moddown<L_>(HostExec{}, s2.data(), b, acc.data(), cts, out, ginv, k, dk, T.mods.data());
  });
  return 0;
}

// Hoisted path: hoist, key preparation, rotate + finish for one element.
int emu_keyswitch_hoisted(int logn, uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd,
                          const uint64_t* inv, const uint64_t* cts, uint64_t count, const uint64_t* key, uint32_t elt,
                          uint64_t* out, uint32_t* zflag_out) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  const uint64_t n = 1ull << logn;
  std::vector<uint64_t> qjp((size_t)dk * k);
  for (uint32_t j = 0; j < dk; ++j)
    for (uint32_t p = 0; p < k; ++p) qjp[j * k + p] = T.mods[j].q % T.mods[p].q;
  std::vector<uint64_t> Y(count * dk * k * n), prepared(ks_prepared_words(k, dk, n)), x(count * 2 * k * n);
  std::vector<uint32_t> zflag(count, 0);
  const uint32_t ginv = inv_mod_2n(elt, 2 * (uint32_t)n);
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < count * dk * k; ++b)
      op_ks_hoist<L_>(HostExec{}, s.data(), b, cts, Y.data(), zflag.data(), k, dk, T.mods.data(), T.fwd);
    const uint64_t pw = prepared.size();
    for (uint64_t b = 0; b < k; ++b)
      op_ks_negntt<L_>(HostExec{}, s.data(), b, prepared.data(), pw, &elt, k, dk, T.mods.data(), T.fwd);
    for (uint64_t item = 0; item < k * n; ++item)
      ks_keyperm_item(item, key, prepared.data(), pw, &ginv, L_, k, dk, T.mods.data(), qjp.data());
    for (uint64_t b = 0; b < count * 2 * k; ++b)
      op_ks_rotate<L_>(HostExec{}, s.data(), b, cts, Y.data(), zflag.data(), prepared.data(), x.data(), elt, k, dk,
                       T.mods.data(), qjp.data(), T.fwd, T.inv, T.fwd64, T.inv64);
    std::vector<uint64_t> s2(n);
    for (uint64_t b = 0; b < count * dk; ++b)
      op_ks_finish<L_>(HostExec{}, s2.data(), b, x.data(), cts, out, ginv, k, dk, T.mods.data());
  });
  for (uint64_t i = 0; i < count; ++i) zflag_out[i] = zflag[i];
  return 0;
}

// Hoisted rotations of E elements, pipelined as launch_ks_rotate_pipe issues them: keys
// [E][dk][2][k][n], elts [E] -> outs [E][count][2][dk][n].  Launch r runs the special-prime
// blocks of element r and the data-prime blocks of element r - 1 over the same buffers the
// device uses (xs parity buffers, one zero-word scratch).
int emu_keyswitch_pipe(int logn, uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd,
                       const uint64_t* inv, const uint64_t* cts, uint64_t count, const uint64_t* keys,
                       const uint32_t* elts, uint64_t elements, uint64_t* outs) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  const uint64_t n = 1ull << logn;
  std::vector<uint64_t> qjp((size_t)dk * k);
  for (uint32_t j = 0; j < dk; ++j)
    for (uint32_t p = 0; p < k; ++p) qjp[j * k + p] = T.mods[j].q % T.mods[p].q;
  const uint64_t pw = ks_prepared_words(k, dk, n), kw = (uint64_t)dk * 2 * k * n, ctw = 2ull * dk * n;
  std::vector<uint64_t> Y(count * dk * k * n), prepared(elements * pw), x(count * 2 * k * n), xs(2 * count * 2 * n);
  std::vector<uint32_t> zflag(count, 0);
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < count * dk * k; ++b)
      op_ks_hoist<L_>(HostExec{}, s.data(), b, cts, Y.data(), zflag.data(), k, dk, T.mods.data(), T.fwd);
    for (uint64_t e = 0; e < elements; ++e) {
      uint64_t* pr = prepared.data() + e * pw;
      const uint32_t ginv = inv_mod_2n(elts[e], 2 * (uint32_t)n);
      for (uint64_t b = 0; b < k; ++b)
        op_ks_negntt<L_>(HostExec{}, s.data(), b, pr, pw, &elts[e], k, dk, T.mods.data(), T.fwd);
      for (uint64_t item = 0; item < k * n; ++item)
        ks_keyperm_item(item, keys + e * kw, pr, pw, &ginv, L_, k, dk, T.mods.data(), qjp.data());
    }
    for (uint64_t r = 0; r <= elements; ++r) {
      const bool special = r < elements, data = r >= 1;
      const uint64_t blocks = (special ? count * 2 : 0) + (data ? count * 2 * dk : 0);
      const uint32_t order = special ? 1u : 0u;
      const uint32_t elt_d = data ? elts[r - 1] : 1;
      for (uint64_t b = 0; b < blocks; ++b)
        op_ks_rotate_pipe<L_>(HostExec{}, s.data(), b, count, order, cts, Y.data(), zflag.data(), x.data(),
                              special ? prepared.data() + r * pw : nullptr, special ? elts[r] : 1,
                              xs.data() + (r & 1) * count * 2 * n, data ? prepared.data() + (r - 1) * pw : nullptr,
                              elt_d, inv_mod_2n(elt_d, 2 * (uint32_t)n), xs.data() + ((r + 1) & 1) * count * 2 * n,
                              data ? outs + (r - 1) * count * ctw : nullptr, k, dk, T.mods.data(), qjp.data(), T.fwd,
                              T.inv, T.fwd64, T.inv64);
    }
  });
  return 0;
}

// Full protected matrix evaluation for `groups` groups:
// cts [inputs][2][dk][n] coefficient form; ring [groups][inputs][n]; mask [groups][n]
// or null; samples [groups][3][k][n] or null (pk [2][k][n]); out [groups][2][dk][n].
int emu_matrix(int logn, uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd, const uint64_t* inv,
               const uint64_t* cts, uint64_t inputs, const uint64_t* ring, uint64_t groups, const uint64_t* mask,
               const uint64_t* samples, const uint64_t* pk, uint64_t q_mod_t, uint64_t upper_half, uint64_t t,
               int tlog, uint64_t* out) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  const uint64_t n = 1ull << logn;
  std::vector<uint64_t> in(cts, cts + inputs * 2 * dk * n);
  std::vector<uint64_t> w(groups * inputs * dk * n);
  std::vector<uint64_t> u_ntt(groups * k * n), x(groups * 2 * k * n);
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < inputs * 2 * dk; ++b)
      op_ntt<L_>(HostExec{}, s.data(), b, false, in.data(), dk, 0, T.mods.data(), T.fwd, T.inv, T.fwd64, T.inv64);
    for (uint64_t b = 0; b < groups * inputs * dk; ++b)
      op_lift_ntt<L_>(HostExec{}, s.data(), b, ring, w.data(), dk, T.mods.data(), T.fwd);
    ProtectArgs prot{mask, nullptr, q_mod_t, upper_half, t, tlog};
    if (samples) {
      for (uint64_t b = 0; b < groups * k; ++b)
        op_enc0_x<L_>(HostExec{}, s.data(), b, samples, pk, u_ntt.data(), x.data(), k, T.mods.data(), T.fwd, T.inv);
      prot.enc0_x = x.data();
    }
    for (uint64_t b = 0; b < groups * 2 * dk; ++b)
      op_mac_intt<L_>(HostExec{}, s.data(), b, in.data(), w.data(), out, (uint32_t)inputs, k, dk, T.mods.data(),
                      T.inv, prot);
  });
  return 0;
}

// Layer pipeline over T tiles: cts [T][I][2][dk][n] coefficient form, ring [G][I][n],
// masks [T][G][n] or null, samples [T][G][3][k][n] or null (pk [2][k][n]);
// out [T][G][2][dk][n].  Tiles are taken in launches of 8/4/2/1 as the launcher does, and
// out doubles as the product accumulator as on the device.
int emu_matrix_tiles(int logn, uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd,
                     const uint64_t* inv, const uint64_t* cts, uint64_t tiles, uint64_t inputs, const uint64_t* ring,
                     uint64_t groups, const uint64_t* masks, const uint64_t* samples, const uint64_t* pk,
                     uint64_t q_mod_t, uint64_t upper_half, uint64_t t, int tlog, uint64_t* out, int path) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  const uint64_t n = 1ull << logn;
  const uint64_t items = tiles * groups;
  std::vector<uint64_t> in(cts, cts + tiles * inputs * 2 * dk * n);
  std::vector<uint64_t> w(groups * inputs * dk * n);
  std::vector<uint64_t> U(items * k * n), xs(items * 2 * n), E(items * 2 * dk * n);
  std::vector<ulonglong2> pkp(pk ? 2 * k * n : 0);
  for (uint64_t e = 0; e < pkp.size(); ++e) pk_prep_item(e, pk, pkp.data(), k, logn, T.mods.data());
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < tiles * inputs * 2 * dk; ++b)
      op_ntt_split<L_>(HostExec{}, s.data(), b, in.data(), in.data(), dk, T.mods.data(), T.fwd);
    for (uint64_t b = 0; b < groups * inputs * dk; ++b)
      op_lift_ntt<L_>(HostExec{}, s.data(), b, ring, w.data(), dk, T.mods.data(), T.fwd);
    const uint64_t in_tile = inputs * 2 * dk * n, acc_tile = groups * 2 * dk * n;
    for (uint64_t t0 = 0; t0 < tiles;) {
      const uint64_t left = tiles - t0;
      const int TT = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
      const uint64_t* ip = in.data() + t0 * in_tile;
      uint64_t* ap = out + t0 * acc_tile;
      if (path == 0 && TT == tc::kTiles && inputs <= (uint64_t)tc::kMaxK && n >= (uint64_t)tc::kSlots) {
        if (inputs <= 32)
          emu_mac_tc_launch<32>(ip, w.data(), ap, (uint32_t)inputs, (uint32_t)groups, dk, L_, T.mods.data());
        else
          emu_mac_tc_launch<64>(ip, w.data(), ap, (uint32_t)inputs, (uint32_t)groups, dk, L_, T.mods.data());
        t0 += TT;
        continue;
      }
      switch (TT) {
        case 8: emu_mac_launch<8, 4>(ip, w.data(), ap, (uint32_t)inputs, (uint32_t)groups, dk, L_, T.mods.data()); break;
        case 4: emu_mac_launch<4, 4>(ip, w.data(), ap, (uint32_t)inputs, (uint32_t)groups, dk, L_, T.mods.data()); break;
        case 2: emu_mac_launch<2, 2>(ip, w.data(), ap, (uint32_t)inputs, (uint32_t)groups, dk, L_, T.mods.data()); break;
        default: emu_mac_launch<1, 1>(ip, w.data(), ap, (uint32_t)inputs, (uint32_t)groups, dk, L_, T.mods.data()); break;
      }
      t0 += TT;
    }
    if (samples) {
      for (uint64_t b = 0; b < items * k; ++b)
        op_enc0_prep<L_>(HostExec{}, s.data(), b, samples, U.data(), k, T.mods.data(), T.fwd);
      for (uint64_t b = 0; b < items * 2; ++b)
        op_enc0_xs<L_>(HostExec{}, s.data(), b, samples, pkp.data(), U.data(), xs.data(), k, T.mods.data(), T.inv);
    }
    const bool fin = samples || masks;
    if (fin)
      for (uint64_t e = 0; e < items * 2 * dk * n; ++e)
        enc0_fin_item(e, samples, xs.data(), masks, E.data(), k, dk, L_, T.mods.data(), q_mod_t, upper_half, t, tlog);
    for (uint64_t b = 0; b < items * 2 * dk; ++b)
      op_intt_protect<L_>(HostExec{}, s.data(), b, out, out, samples ? U.data() : nullptr, pkp.data(),
                          fin ? E.data() : nullptr, k, dk, T.mods.data(), T.inv);
  });
  return 0;
}

// data [batches][dk][n] in place, sk [dk][n] NTT form.
int emu_client_phase(int logn, uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd,
                     const uint64_t* inv, uint64_t* data, const uint64_t* sk, uint64_t batches) {
  Tabs T = tabs(k, mods16, fwd, inv, logn);
  EMU_DISPATCH(logn, {
    std::vector<uint64_t> s(SmemWords<L_>::value);
    for (uint64_t b = 0; b < batches * dk; ++b)
      op_client_phase<L_>(HostExec{}, s.data(), b, data, sk, dk, T.mods.data(), T.fwd, T.inv);
  });
  return 0;
}

// res [count][dk] residues -> limbs [count][dk]; CRT constants from the caller.
int emu_crt(uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* res, uint64_t count,
            const uint64_t* part, const uint64_t* cinv, const uint64_t* qlimbs, uint64_t* limbs) {
  std::vector<Modulus> mods(k);
  std::memcpy(mods.data(), mods16, k * sizeof(Modulus));
  for (uint64_t i = 0; i < count; ++i) crt_target(res + i * dk, dk, mods.data(), part, cinv, qlimbs, limbs + i * dk);
  return 0;
}

// Token product: cts_ntt [19][slots][2][dk][n] NTT form, ring [19][8192], scaled [slots][dk].
int emu_token(uint32_t k, uint32_t dk, const uint64_t* mods16, const uint64_t* fwd, const uint64_t* inv,
              const uint64_t* cts_ntt, uint64_t slots, const uint64_t* ring, const uint64_t* scaled, uint64_t* out) {
  Tabs T = tabs(k, mods16, fwd, inv, 14);
  constexpr int L_ = 14;
  const uint64_t n = 1ull << L_;
  std::vector<uint64_t> w(19 * dk * n), s(SmemWords<L_>::value);
  for (uint64_t b = 0; b < 19 * dk; ++b)
    op_token_lift_ntt<L_>(HostExec{}, s.data(), b, ring, w.data(), dk, T.mods.data(), T.fwd);
  for (uint64_t b = 0; b < slots * 2 * dk; ++b)
    op_token_mac_intt<L_>(HostExec{}, s.data(), b, cts_ntt, w.data(), scaled, out, (uint32_t)slots, dk,
                          T.mods.data(), T.inv);
  return 0;
}

}  // extern "C"

// FP64-pipe modular arithmetic (f64mod.cuh) on arrays: r[i] = mulmod_f64(y[i], w[i]) (signed
// representatives) and c[i] = canon_f64 of it; red[i] = reduce_f64(y[i]).
extern "C" int emu_f64_mulmod(const int64_t* y, const int64_t* w, uint64_t count, uint64_t q, int64_t* r,
                              uint64_t* c, int64_t* red) {
  const double qd = (double)q, qinv = 1.0 / qd;
  for (uint64_t i = 0; i < count; ++i) {
    const double wd = (double)w[i], wq = wd / qd;
    const double v = mulmod_f64((double)y[i], wd, wq, qd);
    r[i] = (int64_t)v;
    c[i] = canon_f64(v, qd, qinv);
    red[i] = (int64_t)reduce_f64((double)y[i], qd, qinv);
  }
  return 0;
}
// Barrett-form products: r[i] = mulmod_f64_barrett(y[i], w[i]) for |y| <= (q+1)/2, 0 <= w < q.
extern "C" int emu_f64_mulmod_barrett(const int64_t* y, const uint64_t* w, uint64_t count, uint64_t q, int64_t* r) {
  const double qd = (double)q, qinv = 1.0 / qd;
  for (uint64_t i = 0; i < count; ++i) r[i] = (int64_t)mulmod_f64_barrett((double)y[i], (double)w[i], qd, qinv);
  return 0;
}
// u64_to_f64 / f64_to_u64 round trip of values below 2^52.
extern "C" int emu_f64_convert(const uint64_t* x, uint64_t count, uint64_t* out) {
  for (uint64_t i = 0; i < count; ++i) out[i] = f64_to_u64(u64_to_f64(x[i]));
  return 0;
}
