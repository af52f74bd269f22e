// The ct-pt contraction of the layer pipeline on the 5th-generation tensor cores
// (tcgen05.mma kind::i8), for launches of 8 token tiles.  Host-compilable pieces: the
// shared-memory images the tensor memory accelerator (TMA) writes, the MMA descriptors and
// the exact recombination of the byte-limb products.
//
// Per NTT slot (data prime p, coefficient z) the contraction
//   X[tc][g] = sum_b in[t][b][c] . W[g][b]          (tc = 2t + c, residues < 2^60)
// is an int8 MMA over the bytes of the words, D = sum_b A[.][b] . B[b][.], recombined as
//   X[tc][g] = sum_{i,j} D[(tc, i)][(g, j)] . 2^(limb_shift(i) + 8j)
// (an exact integer < I . 2^120 < 2^126 for I <= 64) and reduced mod q once.
//
// Operands come straight from the natural HBM layouts (inputs [t][b][c][p][z], weights
// [g][b][p][z]) by TMA tiled copies without swizzle, which write each box densely in box
// order.  A TMA box's innermost extent is at least 16 bytes, i.e. two consecutive
// coefficients, so every copy carries a slot pair; the boxes are ordered so that the dense
// image is the canonical MN-major layout without swizzle (16-byte MN chunks, each holding
// its K rows 16 bytes apart):
//   A box (per M-block mb = tiles 4mb..4mb+3): [t4][c][b][zs][8 bytes]
//       -> M index m = ((t4*2 + c)*2 + zs)*8 + i, chunk m/16 at (m/16)*K*16 + b*16
//   B box (16 groups):                         [g][b][zs][8 bytes]
//       -> N index n = (g*2 + zs)*8 + j (N = 256)
// The MMA therefore also forms the cross-slot products (zs of A != zs of B); they land in
// TMEM columns the epilogue never reads.  That doubles the tensor work, which is cheap
// next to the recombination, and it leaves all staging to TMA with no register traffic.
// (With the 128-byte swizzle a 16-byte-wide box is not written densely: each 16-byte row
// takes a 128-byte pitch, so that mode is not used here.)
#pragma once
#include "arith.cuh"

namespace bfvgpu {
namespace tc {

constexpr int kTiles = 8;       // two M-blocks of 4 tiles
constexpr int kGroupsRound = 16;  // groups per MMA round (N = 256)
constexpr int kGroups = 32;     // groups per work unit (two rounds per slot pair)
constexpr int kSlots = 16;      // slots per work unit (one 128-byte run per output row)
constexpr int kPair = 2;        // slots per TMA box
constexpr int kThreads = 512;
constexpr int kMaxK = 64;       // input blocks per call handled here (K padded to 32 or 64)
constexpr int kRoundsPerPair = kGroups / kGroupsRound;
constexpr int kRoundsPerUnit = (kSlots / kPair) * kRoundsPerPair;

// Byte offsets inside the block's shared memory (from a 1024-byte aligned base).
template <int KPAD>
struct Smem {
  static constexpr uint32_t kABox = KPAD * 128;                 // one M-block box (8 chunks)
  static constexpr uint32_t kA = 0;                             // [2 buffers][2 M-blocks] boxes
  static constexpr uint32_t kABuf = 2 * kABox;
  static constexpr uint32_t kBBox = KPAD * 256;                 // one 16-group box (16 chunks)
  static constexpr uint32_t kB = kA + 2 * kABuf;                // [2 buffers] boxes
  static constexpr uint32_t kOut = kB + 2 * kBBox;              // [16 z][16 tc][32 g] u64
  static constexpr uint32_t kOutBytes = kSlots * 16 * kGroups * 8;
  static constexpr uint32_t kBar = kOut + kOutBytes;            // 8 mbarriers, TMEM base, abort flag
  static constexpr uint32_t kBytes = kBar + 80;
  // Requested dynamic size: slack for the 1024-byte alignment, and above half an SM's shared
  // memory so that one block holds an SM (and all 512 TMEM columns) alone.
  static constexpr uint32_t kLaunchBytes = (kBytes + 1024) > 120 * 1024 ? (kBytes + 1024) : 120 * 1024;
};

// Byte offsets in the dense box images.
template <int KPAD>
BFV_HD uint32_t a_img(uint32_t b, uint32_t t4, uint32_t c, uint32_t zs) { return ((t4 * 2 + c) * KPAD + b) * 16 + zs * 8; }
template <int KPAD>
BFV_HD uint32_t b_img(uint32_t b, uint32_t g, uint32_t zs) { return (g * KPAD + b) * 16 + zs * 8; }

// tcgen05 shared-memory matrix descriptor: start, leading/stride byte offsets (16-byte
// units), version 1, base offset 0, layout type 0 = no swizzle.  For an MN-major operand
// without swizzle the stride byte offset steps between 16-byte MN chunks and the leading
// byte offset between groups of 8 K rows.
BFV_HD uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3fff) | ((uint64_t)((lbo_bytes >> 4) & 0x3fff) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3fff) << 32) | (uint64_t(1) << 46);
}
// A of M-block mb, K-step kk (32 rows = 512 bytes into every chunk).
template <int KPAD>
BFV_HD uint64_t a_desc(uint32_t base, uint32_t buf, uint32_t mb, uint32_t kk) {
  return smem_desc(base + Smem<KPAD>::kA + buf * Smem<KPAD>::kABuf + mb * Smem<KPAD>::kABox + kk * 512, 128, KPAD * 16);
}
template <int KPAD>
BFV_HD uint64_t b_desc(uint32_t base, uint32_t buf, uint32_t kk) {
  return smem_desc(base + Smem<KPAD>::kB + buf * Smem<KPAD>::kBBox + kk * 512, 128, KPAD * 16);
}
// Instruction descriptor, kind::i8: D s32 (2 << 4), A and B unsigned 8-bit (0), both
// MN-major (bits 15, 16), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 15) | (1u << 16) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

// Work unit u -> (group chunk gc, data prime p, first slot z0); group chunks fastest.
BFV_HD void unit_coords(uint32_t u, uint32_t gchunks, uint32_t zblocks, uint32_t* gc, uint32_t* p, uint32_t* z0) {
  *gc = u % gchunks;
  const uint32_t r0 = u / gchunks;
  *p = r0 / zblocks;
  *z0 = (r0 % zblocks) * kSlots;
}
// Output buffer word (slot zi of the unit, tc, group gl of the unit's chunk) and the global
// element offset of output row (tc, g) of the unit (16 consecutive coefficients from z0).
BFV_HD uint32_t out_buf_word(uint32_t zi, uint32_t tcx, uint32_t gl) { return (zi * 16 + tcx) * kGroups + gl; }
BFV_HD uint64_t out_row(uint32_t tcx, uint32_t g, uint32_t groups, uint32_t p, uint32_t z0, uint32_t dk, uint32_t N) {
  return ((((uint64_t)(tcx >> 1) * groups + g) * 2 + (tcx & 1)) * dk + p) * N + z0;
}

// Weight of byte i of an input word in the split form a1 . 2^32 + a0 (a0, a1 < 2^30) that
// the client-limb transform stores: bytes 0-3 are a0's (2^(8i)), bytes 4-7 a1's, which
// stand for a1 . 2^30 (2^(8i-2)).  The MMA reads the split words as they are.
BFV_HD uint32_t limb_shift(uint32_t i) { return i < 4 ? 8 * i : 8 * i - 2; }

// Byte-limb recombination of one TMEM lane (input byte i of slot zs) from one 32-column
// load (2 groups x 2 slots x 8 bytes): for both groups k, V[k] = sum_j D[(2k + zs)*8 + j] .
// 2^(limb_shift(i) + 8j) as 128 bits.  Every V is a partial sum of the exact product sum,
// so it stays below 2^126.
BFV_HD void lane_values2(const uint32_t* D, uint32_t zs, uint32_t i, uint64_t* vlo, uint64_t* vhi) {
  const uint32_t sh = limb_shift(i);
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint32_t d[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = zs ? D[(2 * k + 1) * 8 + j] : D[2 * k * 8 + j];
    const uint64_t p0 = d[0] + ((uint64_t)d[1] << 8), p1 = d[2] + ((uint64_t)d[3] << 8);
    const uint64_t p2 = d[4] + ((uint64_t)d[5] << 8), p3 = d[6] + ((uint64_t)d[7] << 8);
    const uint64_t lo = p0 + (p1 << 16) + (p2 << 32);  // < 2^64
    const uint64_t t = p3 << 48;
    const uint64_t l2 = lo + t;
    const uint64_t h2 = (p3 >> 16) + (l2 < t);
    vlo[k] = l2 << sh;
    vhi[k] = sh ? ((h2 << sh) | (l2 >> (64 - sh))) : h2;
  }
}

BFV_HD void add128(uint64_t& lo, uint64_t& hi, uint64_t blo, uint64_t bhi) {
  lo += blo;
  hi += bhi + (lo < blo);
}

}  // namespace tc
}  // namespace bfvgpu
