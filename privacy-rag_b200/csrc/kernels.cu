// BFV ciphertext-arithmetic kernels for sm_100a.
//
// Every transform-bearing kernel runs one RNS limb per thread block with the limb
// resident in shared memory (ntt_core.cuh); the reference's separate elementwise
// kernels (lift, product, decompose, moddown, gather, add_shift) become prologues
// and epilogues of those transforms, so each limb crosses HBM once per kernel.
//
// Reference kernels restated (IV1 = implementation_v1/):
//   k_ntt ............. `stage` (matrix.cu:52-58; switch.cu:47-58; ntt.cu:83-94; enc0.cu:45-56)
//   k_lift_ntt ........ `lift` + forward stages (matrix.cu:48-51, :96)
//   k_mac_intt ........ `product` + inverse stages (matrix.cu:59-63, :96), with the
//                       sub_plain mask (bfv_matrix.inc:215-219) and the Enc(0) add
//                       (bfv_matrix.inc:220-227) fused into the epilogue
//   k_gather_targets .. `gather_c0` (matrix.cu:66-69) + rns_coefficient (bfv.cpp:138-147)
//   k_ks_main ......... CPU apply_galois (keyswitch seal_adapter.cpp:50) + `decompose`,
//                       forward stages, `product`, inverse stages (switch.cu:92-102, :146-149)
//   k_ks_moddown ...... `moddown` (switch.cu:103-111) with the permuted c0 add
//   k_enc0_x/k_moddown  PublicZero::evaluate (enc0.cu:74-89, :125-140)
//   k_client_phase .... client_phase (ntt.cu:96-98, :181-199)
//   k_token_* ......... TokenWeights::evaluate_device (resident.cu:71-107, :200-221)
//   k_packing_prepare . packing_prepare (switch.cu:78-87)
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include "kernels.cuh"
#include "block_ops.cuh"
#include "mac_tc.cuh"

namespace bfvgpu {

// NVTX range around each launch group (named "bfvgpu:<group>"), so a profiler timeline
// shows which fused kernels a library call issued.  Header-only NVTX v3: without an
// attached tool a push/pop is a check of one function pointer.
struct LaunchRange {
  explicit LaunchRange(const char* name) { nvtxRangePushA(name); }
  ~LaunchRange() { nvtxRangePop(); }
  LaunchRange(const LaunchRange&) = delete;
  LaunchRange& operator=(const LaunchRange&) = delete;
};

// Block shape per degree, from a sweep of radix x blocks/SM x block size on B200:
// n <= 8192: 256 threads, 3 blocks per SM (<= 80 registers); n = 16384: 512 threads,
// one block per SM (136 KiB of shared memory).  Small test degrees use n/16 threads.
template <int LOGN>
constexpr int threads_for() {
  return LOGN >= 14 ? 512 : (((1 << LOGN) / 16) < 256 ? ((1 << LOGN) / 16) : 256);
}
template <int LOGN>
constexpr int blocks_per_sm() {
  return LOGN >= 14 ? 1 : 3;
}
template <int LOGN>
constexpr size_t smem_bytes() {
  return (size_t)SmemWords<LOGN>::value * sizeof(uint64_t);
}

// ---------------------------------------------------------------------------------
// transform-bearing kernels: one block per limb, bodies in block_ops.cuh
// ---------------------------------------------------------------------------------
template <int LOGN, bool INV>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ntt(uint64_t* data, uint32_t prime_count, uint32_t prime_offset, const Modulus* mods, const ulonglong2* fwd,
          const ulonglong2* inv, const double2* fwd64, const double2* inv64) {
  extern __shared__ uint64_t smem[];
  op_ntt<LOGN>(BlockExec{}, smem, blockIdx.x, INV, data, prime_count, prime_offset, mods, fwd, inv, fwd64, inv64);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_lift_ntt(const uint64_t* ring, uint64_t* out, uint32_t dk, const Modulus* mods, const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_lift_ntt<LOGN>(BlockExec{}, smem, blockIdx.x, ring, out, dk, mods, fwd);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_mac_intt(const uint64_t* in, const uint64_t* w, uint64_t* out, uint32_t inputs, uint32_t k, uint32_t dk,
               const Modulus* mods, const ulonglong2* inv, ProtectArgs prot) {
  extern __shared__ uint64_t smem[];
  op_mac_intt<LOGN>(BlockExec{}, smem, blockIdx.x, in, w, out, inputs, k, dk, mods, inv, prot);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_main(const uint64_t* cts, const uint64_t* key, uint64_t* acc, uint32_t elt, uint32_t k, uint32_t dk,
              const Modulus* mods, const uint64_t* qjp, const ulonglong2* fwd, const ulonglong2* inv,
              const double2* fwd64, const double2* inv64) {
  extern __shared__ uint64_t smem[];
  op_ks_main<LOGN>(BlockExec{}, smem, blockIdx.x, cts, key, acc, elt, k, dk, mods, qjp, fwd, inv, fwd64, inv64);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_moddown(const uint64_t* acc, const uint64_t* cts, uint64_t* out, uint32_t ginv, uint32_t k, uint32_t dk,
                 const Modulus* mods) {
  extern __shared__ uint64_t smem[];
  op_ks_moddown<LOGN>(BlockExec{}, smem, blockIdx.x, acc, cts, out, ginv, k, dk, mods);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_enc0_x(const uint64_t* samples, const uint64_t* pk, uint64_t* u_ntt, uint64_t* x, uint32_t k,
             const Modulus* mods, const ulonglong2* fwd, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_enc0_x<LOGN>(BlockExec{}, smem, blockIdx.x, samples, pk, u_ntt, x, k, mods, fwd, inv);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_client_phase(uint64_t* data, const uint64_t* sk, uint32_t dk, const Modulus* mods, const ulonglong2* fwd,
                   const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_client_phase<LOGN>(BlockExec{}, smem, blockIdx.x, data, sk, dk, mods, fwd, inv);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_token_lift_ntt(const uint64_t* ring, uint64_t* w, uint32_t dk, const Modulus* mods, const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_token_lift_ntt<LOGN>(BlockExec{}, smem, blockIdx.x, ring, w, dk, mods, fwd);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_token_mac_intt(const uint64_t* in, const uint64_t* w, const uint64_t* scaled, uint64_t* out, uint32_t slots,
                     uint32_t dk, const Modulus* mods, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_token_mac_intt<LOGN>(BlockExec{}, smem, blockIdx.x, in, w, scaled, out, slots, dk, mods, inv);
}

// The same two steps for many coordinates in one launch each: coordinate j's weights at
// ring + j * 19 * 8192, its transforms at w + j * 19 * dk * n, its scaled local shares at
// scaled + j * slots * dk and its products at out + j * slots * 2 * dk * n.
template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_token_lift_ntt_many(const uint64_t* ring, uint64_t* w, uint32_t dk, const Modulus* mods, const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  const uint64_t per = (uint64_t)kTokenBlocks * dk, j = blockIdx.x / per;
  op_token_lift_ntt<LOGN>(BlockExec{}, smem, blockIdx.x % per, ring + j * kTokenBlocks * kTokenWidth,
                          w + ((j * per) << LOGN), dk, mods, fwd);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_token_mac_intt_many(const uint64_t* in, const uint64_t* w, const uint64_t* scaled, uint64_t* out, uint32_t slots,
                          uint32_t dk, const Modulus* mods, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  const uint64_t per = (uint64_t)slots * 2 * dk, j = blockIdx.x / per;
  op_token_mac_intt<LOGN>(BlockExec{}, smem, blockIdx.x % per, in, w + ((j * kTokenBlocks * dk) << LOGN),
                          scaled + j * slots * dk, out + ((j * per) << LOGN), slots, dk, mods, inv);
}

// scaled [count][dk] = the Delta-scaled plaintext coefficient of local [count] per data prime.
__global__ void k_scale_local(const uint64_t* local, uint64_t count, uint64_t* scaled, uint32_t dk,
                              const Modulus* mods, uint64_t q_mod_t, uint64_t upper_half, uint64_t t, int tlog) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < count * dk;
       e += (uint64_t)gridDim.x * blockDim.x)
    scaled[e] = scale_plain_coeff(local[e / dk], q_mod_t, upper_half, t, tlog, mods[e % dk]);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_hoist(const uint64_t* cts, uint64_t* Y, uint32_t* zflag, uint32_t k, uint32_t dk, const Modulus* mods,
               const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_ks_hoist<LOGN>(BlockExec{}, smem, blockIdx.x, cts, Y, zflag, k, dk, mods, fwd);
}

// ---- layer pipeline: multi-tile product, Enc(0) preparation, INTT with epilogue -------
__device__ __forceinline__ void cp_async16(uint64_t* dst, const uint64_t* src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  const int bytes = src ? 16 : 0;  // 0: zero-fill, nothing is read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src ? src : dst), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Persistent product kernel: one 16-warp block per SM walks work units u = blockIdx.x +
// i * gridDim.x, unit = (data prime, 32 coefficients, GB groups) with the group block
// fastest, so the blocks running at one time share a coefficient chunk (its inputs stay in
// L2) while every weight word is streamed from HBM once.  Staging runs kMacStages - 1
// chunks ahead through cp.async, across unit boundaries.  Bodies in block_ops.cuh.
constexpr int kMacStages = 4;

template <int T, int TH>
__global__ void __launch_bounds__(512, 1)
    k_mac_split(const uint64_t* in, const uint64_t* w, uint64_t* out, uint32_t inputs, uint32_t groups,
                uint32_t gblocks, uint32_t units, uint32_t dk, int logn, const Modulus* mods) {
  using S = MacShape<T, TH>;
  extern __shared__ uint64_t smem[];
  const uint32_t zchunks = (1u << logn) >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t chunks = (inputs + S::kBc - 1) / S::kBc;
  const uint32_t my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const uint64_t steps = (uint64_t)my_units * chunks;
  // step s -> unit blockIdx.x + (s / chunks) * gridDim.x, chunk s % chunks
  auto issue = [&](uint64_t s) {
    if (s < steps) {
      const uint32_t u = blockIdx.x + (uint32_t)(s / chunks) * gridDim.x, k = (uint32_t)(s % chunks);
      const uint32_t gq = u % gblocks, r = u / gblocks;
      const uint32_t p = r / zchunks, z0 = (r % zchunks) * 32;
      uint64_t* buf = smem + (s % kMacStages) * S::kBufWords;
      for (int seg = threadIdx.x; seg < S::kSegs; seg += S::kThreads) {
        int dst;
        const uint64_t* src =
            mac_stage_src<T, TH>(seg, k * S::kBc, in, w, inputs, groups, gq * S::GB, p, z0, dk, logn, &dst);
        cp_async16(buf + dst, src);
      }
    }
    cp_async_commit();  // one group per step, empty past the end, so the wait count holds
  };
  Mac30 acc[TH][2];
  Acc128 A[TH][2];
  for (int s = 0; s < kMacStages - 1; ++s) issue(s);
  for (uint64_t s = 0; s < steps; ++s) {
    cp_async_wait<kMacStages - 2>();
    __syncthreads();  // step s is in shared memory; every warp is done with step s - 1
    issue(s + kMacStages - 1);
    const uint32_t u = blockIdx.x + (uint32_t)(s / chunks) * gridDim.x, k = (uint32_t)(s % chunks);
    const uint32_t r = u / gblocks, p = r / zchunks;
    const Modulus& m = mods[p];
    mac_chunk<T, TH>(smem + (s % kMacStages) * S::kBufWords, warp, lane, acc, A, m, k);
    if (k + 1 == chunks) {
      mac_store<T, TH>(out, warp, lane, A, m, groups, (u % gblocks) * S::GB, p, (r % zchunks) * 32, dk, logn);
#pragma unroll
      for (int tt = 0; tt < TH; ++tt)
#pragma unroll
        for (int c = 0; c < 2; ++c) A[tt][c] = Acc128{};
    }
  }
  cp_async_wait<0>();
}

// ---- the same contraction on tcgen05 (8 tiles, at most 64 input blocks) ------------------
// Persistent: one 16-warp block per SM walks units (data prime, 16 slots, 32 groups), group
// chunk fastest.  Thread 0 is the producer and MMA issuer: per slot pair it loads the two
// A boxes (inputs, 4 tiles each) by TMA into one of two A buffers, per round (16 groups)
// the two B boxes (weights) into one of two B buffers, issues 2 M-blocks x K/32 MMAs into
// TMEM columns [256 mb, 256 mb + 256) and commits to an mbarrier.  All 16 warps then drain
// TMEM (warp w: lanes 32 (w%4).., M-block and 8 groups from w/4), recombine the byte-limb
// sums of their slot, reduce mod q into the unit's output buffer, which is written out as
// 128-byte rows when the unit ends.  Every mbarrier wait is bounded: on expiry the block
// records kErrMmaTimeout in *err, frees TMEM and returns.  Layouts and descriptors:
// mac_tc.cuh.
constexpr uint32_t kErrMmaTimeout = 1;
constexpr uint32_t kMbarPolls = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  uint32_t done = 0;
  for (uint32_t it = 0; it < kMbarPolls && !done; ++it)
    asm volatile(
        "{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}"
        : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %0;" ::"r"(bytes), "r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Barrier `id` over `count` threads that also ORs `pred` across them.
__device__ __forceinline__ bool bar_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(count) : "memory");
  return r != 0;
}

// Warp roles: warps 0-7 drain TMEM buffer 0 (M-block 0, tiles 0-3), warps 8-15 buffer 1
// (M-block 1, tiles 4-7), lane 0 of warp 16 loads operands and issues the MMAs.  Round R =
// ((unit * 8 + slot pair) * 2 + group round) * 2 + M-block; round R uses TMEM buffer R % 2, so
// the MMA of one M-block runs while the other consumer group recombines.
constexpr int kMacTcThreads = 17 * 32;

template <int KPAD>
__global__ void __launch_bounds__(kMacTcThreads, 1)
    k_mac_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, uint64_t* out,
             uint32_t groups, uint32_t gchunks, uint32_t units, uint32_t dk, int logn, const Modulus* mods,
             uint32_t* err) {
  using S = tc::Smem<KPAD>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t N = 1u << logn, zblocks = N / tc::kSlots;
  // barriers: fullA[2], fullB[2], mma_done[2], tmem_free[2]; then the TMEM base and an abort flag
  const uint32_t barA = base + S::kBar, barB = barA + 16, barM = barA + 32, barF = barA + 48;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kBar + 64);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(sm + S::kBar + 68);
  const uint64_t pA = reinterpret_cast<uint64_t>(&tmA), pB = reinterpret_cast<uint64_t>(&tmB);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(base + S::kBar + 64));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (uint32_t b = 0; b < 6; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(barA + 8 * b) : "memory");
    for (uint32_t b = 0; b < 2; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 256;" ::"r"(barF + 8 * b) : "memory");
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const uint32_t my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  constexpr uint32_t kRoundsPerUnit = tc::kRoundsPerUnit * 2;  // x 2 M-blocks
  const uint32_t rounds = my_units * kRoundsPerUnit;
  // round R -> unit coordinates, slot pair zp, group round gr (M-block = R % 2)
  auto coords = [&](uint32_t R, uint32_t* gc, uint32_t* p, uint32_t* z0, uint32_t* zp, uint32_t* gr) {
    const uint32_t u = blockIdx.x + (R / kRoundsPerUnit) * gridDim.x;
    tc::unit_coords(u, gchunks, zblocks, gc, p, z0);
    const uint32_t rr = (R % kRoundsPerUnit) >> 1;
    *zp = rr / tc::kRoundsPerPair;
    *gr = rr % tc::kRoundsPerPair;
  };

  if (warp == 16) {
    // ---- producer: TMA loads and MMA issue ----
    if (lane == 0 && rounds) {
      auto load_a = [&](uint32_t P) {  // slot pair P (block-local index) -> A buffer P % 2
        uint32_t gc, p, z0, zp, gr;
        coords(P * 4, &gc, &p, &z0, &zp, &gr);
        const uint32_t bar = barA + 8 * (P & 1), z = z0 + zp * tc::kPair;
        mbar_expect(bar, 2 * S::kABox);
#pragma unroll
        for (uint32_t mb = 0; mb < 2; ++mb)
          asm volatile(
              "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
              ::"r"(base + S::kA + (P & 1) * S::kABuf + mb * S::kABox), "l"(pA), "r"((int)z), "r"(0), "r"(0),
              "r"((int)(4 * mb)), "r"((int)p), "r"(bar) : "memory");
      };
      auto load_b = [&](uint32_t Q) {  // (pair, group round) Q -> B buffer Q % 2
        uint32_t gc, p, z0, zp, gr;
        coords(Q * 2, &gc, &p, &z0, &zp, &gr);
        const uint32_t bar = barB + 8 * (Q & 1), z = z0 + zp * tc::kPair;
        mbar_expect(bar, S::kBBox);
        asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
            ::"r"(base + S::kB + (Q & 1) * S::kBBox), "l"(pB), "r"((int)z), "r"(0),
            "r"((int)(gc * tc::kGroups + gr * tc::kGroupsRound)), "r"((int)p), "r"(bar) : "memory");
      };
      const uint32_t pairs = rounds / 4, qs = rounds / 2;
      // the last A / B copy issued and the last round committed: each barrier has at most
      // one operation outstanding (a copy is issued only after the previous one into the
      // other buffer was seen complete, and MMAs complete in commit order), so on abort one
      // wait per barrier drains everything this thread started
      uint32_t a_last = 0, b_last = 0, m_next = 0;
      load_a(0);
      load_b(0);
      bool ok = true;
      for (uint32_t R = 0; R < rounds && ok; ++R) {
        const uint32_t mb = R & 1, Q = R >> 1, P = R >> 2;
        if (mb == 0) {
          if ((R & 3) == 0) ok = ok && mbar_wait(barA + 8 * (P & 1), (P >> 1) & 1);
          ok = ok && mbar_wait(barB + 8 * (Q & 1), (Q >> 1) & 1);
          // the buffers for the next pair / group round were last read by round R - 1
          if (ok && R >= 1) ok = mbar_wait(barM + 8 * ((R - 1) & 1), ((R - 1) >> 1) & 1);
          if (ok && (R & 3) == 0 && P + 1 < pairs) {
            load_a(P + 1);
            a_last = P + 1;
          }
          if (ok && Q + 1 < qs) {
            load_b(Q + 1);
            b_last = Q + 1;
          }
        }
        // the consumer of this TMEM buffer has finished round R - 2
        if (ok && R >= 2) ok = mbar_wait(barF + 8 * mb, ((R >> 1) - 1) & 1);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (uint32_t kk = 0; kk < KPAD / 32; ++kk) {
          const uint64_t ad = tc::a_desc<KPAD>(base, P & 1, mb, kk), bd = tc::b_desc<KPAD>(base, Q & 1, kk);
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem + 256 * mb),
              "l"(ad), "l"(bd), "r"(tc::kIdesc), "r"(kk) : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(barM + 8 * mb)
                     : "memory");
        m_next = R + 1;
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrMmaTimeout);
        // before the block frees its tensor memory and exits: the copies still writing its
        // shared memory and the MMAs still reading it (each wait bounded; a copy or MMA
        // already complete passes at once)
        mbar_wait(barA + 8 * (a_last & 1), (a_last >> 1) & 1);
        mbar_wait(barB + 8 * (b_last & 1), (b_last >> 1) & 1);
        if (m_next) mbar_wait(barM + 8 * ((m_next - 1) & 1), ((m_next - 1) >> 1) & 1);
      }
    }
  } else {
    // ---- consumers: group g drains TMEM buffer g (M-block g) every other round ----
    const uint32_t g = warp >> 3, wq = warp & 7;
    const uint32_t quarter = wq & 3, gh = wq >> 2;
    const uint32_t m = quarter * 32 + lane, tc4 = m >> 4, zs = (m >> 3) & 1, i = m & 7;
    const uint32_t tcx = g * 8 + tc4;
    uint64_t* ob = reinterpret_cast<uint64_t*>(sm + S::kOut);
    for (uint32_t R = g; R < rounds; R += 2) {
      const bool done = mbar_wait(barM + 8 * g, (R >> 1) & 1) && !*abort_flag;
      if (bar_or(1 + g, 256, !done)) {
        if (threadIdx.x == 0) atomicOr(err, kErrMmaTimeout);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t gc, p, z0, zp, gr;
      coords(R, &gc, &p, &z0, &zp, &gr);
      const Modulus& mod = mods[p];
      uint64_t vlo[8], vhi[8];
#pragma unroll
      for (uint32_t h = 0; h < 4; ++h) {
        uint32_t D[32];
        const uint32_t taddr = tmem + ((quarter * 32) << 16) + 256 * g + 128 * gh + 32 * h;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(D[0]), "=r"(D[1]), "=r"(D[2]), "=r"(D[3]), "=r"(D[4]), "=r"(D[5]), "=r"(D[6]), "=r"(D[7]),
              "=r"(D[8]), "=r"(D[9]), "=r"(D[10]), "=r"(D[11]), "=r"(D[12]), "=r"(D[13]), "=r"(D[14]),
              "=r"(D[15]), "=r"(D[16]), "=r"(D[17]), "=r"(D[18]), "=r"(D[19]), "=r"(D[20]), "=r"(D[21]),
              "=r"(D[22]), "=r"(D[23]), "=r"(D[24]), "=r"(D[25]), "=r"(D[26]), "=r"(D[27]), "=r"(D[28]),
              "=r"(D[29]), "=r"(D[30]), "=r"(D[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        tc::lane_values2(D, zs, i, vlo + 2 * h, vhi + 2 * h);
      }
      // TMEM buffer g is free once every thread of the group has its values in registers
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(barF + 8 * g);
      // reduce-scatter over the 8 lanes of one (tc, zs): lane i ends with group k = i
#pragma unroll
      for (int lev = 4; lev >= 1; lev >>= 1) {
        const bool sel = i & lev;
#pragma unroll
        for (int q = 0; q < lev; ++q) {
          const uint64_t kl = sel ? vlo[q + lev] : vlo[q], kh = sel ? vhi[q + lev] : vhi[q];
          const uint64_t sl = sel ? vlo[q] : vlo[q + lev], sh = sel ? vhi[q] : vhi[q + lev];
          vlo[q] = kl;
          vhi[q] = kh;
          tc::add128(vlo[q], vhi[q], __shfl_xor_sync(0xffffffffu, sl, lev), __shfl_xor_sync(0xffffffffu, sh, lev));
        }
      }
      ob[tc::out_buf_word(zp * tc::kPair + zs, tcx, gr * tc::kGroupsRound + gh * 8 + i)] = reduce128(vlo[0], vhi[0], mod);
      if ((R % kRoundsPerUnit) + 2 >= kRoundsPerUnit) {  // this group's last round of the unit
        asm volatile("bar.sync %0, 256;" ::"r"(1 + g) : "memory");
        // flush the group's rows: tc in [8 g, 8 g + 8) x 32 groups, one row per thread
        const uint32_t t8 = (warp & 7) * 32 + lane, rtc = g * 8 + (t8 >> 5), rgl = t8 & 31;
        const uint32_t gg = gc * tc::kGroups + rgl;
        if (gg < groups) {
          uint64_t* dst = out + tc::out_row(rtc, gg, groups, p, z0, dk, N);
#pragma unroll
          for (int zz = 0; zz < tc::kSlots; zz += 2) {
            ulonglong2 v;
            v.x = ob[tc::out_buf_word(zz, rtc, rgl)];
            v.y = ob[tc::out_buf_word(zz + 1, rtc, rgl)];
            *reinterpret_cast<ulonglong2*>(dst + zz) = v;
          }
        }
        asm volatile("bar.sync %0, 256;" ::"r"(1 + g) : "memory");
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

template <int T, int TH>
constexpr size_t mac_smem_bytes() {
  return kMacStages * (size_t)MacShape<T, TH>::kBufWords * sizeof(uint64_t);
}

// The same persistent product with its operands staged by the tensor memory accelerator:
// per step one tiled copy brings the chunk's inputs (box 32 coefficients x 1 prime x 2
// components x 8 blocks x T tiles of [T][I][2][dk][n]) and one its weights (32 x 1 x 8
// blocks x GB groups of [G][I][dk][n]) into the stage buffer, in exactly the layout
// mac_chunk reads, with zeros past the input blocks and groups.  One thread issues both
// copies for step s + kMacStages - 1 after the block barrier of step s; every thread waits
// on the stage's mbarrier (bounded: on expiry the block records kErrMacTimeout, waits for its
// copies still in flight and returns).  Instead of 2,304 16-byte asynchronous copies per
// step spread over the block's threads, two instructions move the 36-48 KiB.
constexpr uint32_t kErrMacTimeout = 2;

template <int T, int TH>
__global__ void __launch_bounds__(MacShape<T, TH>::kThreads, 1)
    k_mac_stream(const __grid_constant__ CUtensorMap tmIn, const __grid_constant__ CUtensorMap tmW, uint64_t* out,
                 uint32_t inputs, uint32_t groups, uint32_t gblocks, uint32_t units, uint32_t dk, int logn,
                 const Modulus* mods, uint32_t* err) {
  using S = MacShape<T, TH>;
  constexpr uint32_t kStageBytes = S::kBufWords * 8;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 127) & ~127u;
  const uint64_t* buf0 = reinterpret_cast<const uint64_t*>(smem_raw + (base - raw));
  const uint32_t bar0 = base + kMacStages * kStageBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t zchunks = (1u << logn) >> 5;
  const uint32_t chunks = (inputs + S::kBc - 1) / S::kBc;
  const uint32_t my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const uint64_t steps = (uint64_t)my_units * chunks;
  const uint64_t pIn = reinterpret_cast<uint64_t>(&tmIn), pW = reinterpret_cast<uint64_t>(&tmW);
  if (threadIdx.x == 0) {
    for (int b = 0; b < kMacStages; ++b) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * b) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Step s = (unit blockIdx.x + i * gridDim.x, chunk k) with s = i * chunks + k, walked by
  // cursors (no division per step): one for the consumers, one for the issuing thread.
  const int zshift = logn - 5;
  struct Cursor {
    uint32_t k, u, gq, p, z0;
  };
  auto place = [&](Cursor& c, uint32_t u) {
    c.u = u;
    c.gq = u % gblocks;
    const uint32_t r = u / gblocks;
    c.p = r >> zshift;
    c.z0 = (r & (zchunks - 1)) << 5;
  };
  auto advance = [&](Cursor& c) {
    if (++c.k == chunks) {
      c.k = 0;
      place(c, c.u + gridDim.x);
    }
  };
  Cursor ic{0, 0, 0, 0, 0}, cc{0, 0, 0, 0, 0};
  place(ic, blockIdx.x);
  place(cc, blockIdx.x);
  auto issue = [&](uint64_t s) {  // thread 0: step s, at the issue cursor, which then advances
    if (s >= steps) return;
    const int p = (int)ic.p, z0 = (int)ic.z0, b0 = (int)(ic.k * S::kBc);
    const uint32_t st = (uint32_t)(s % kMacStages), bar = bar0 + 8 * st, dst = base + st * kStageBytes;
    mbar_expect(bar, kStageBytes);
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        ::"r"(dst), "l"(pIn), "r"(z0), "r"(p), "r"(0), "r"(b0), "r"(0), "r"(bar) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
        ::"r"(dst + (uint32_t)S::kInWords * 8), "l"(pW), "r"(z0), "r"(p), "r"(b0), "r"((int)(ic.gq * S::GB)), "r"(bar)
        : "memory");
    advance(ic);
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < kMacStages - 1; ++s) issue(s);
  Mac30 acc[TH][2];
  Acc128 A[TH][2];
  uint64_t s = 0;
  bool failed = false;
  for (; s < steps; ++s) {
    const bool ok = mbar_wait(bar0 + 8 * (uint32_t)(s % kMacStages), (uint32_t)((s / kMacStages) & 1));
    if (__syncthreads_or(!ok)) {  // step s is in shared memory; every warp is done with step s - 1
      failed = true;
      break;
    }
    if (threadIdx.x == 0) issue(s + kMacStages - 1);
    const Modulus& m = mods[cc.p];
    mac_chunk<T, TH>(buf0 + (s % kMacStages) * S::kBufWords, warp, lane, acc, A, m, cc.k);
    if (cc.k + 1 == chunks) {
      mac_store<T, TH>(out, warp, lane, A, m, groups, cc.gq * S::GB, cc.p, cc.z0, dk, logn);
#pragma unroll
      for (int tt = 0; tt < TH; ++tt)
#pragma unroll
        for (int c = 0; c < 2; ++c) A[tt][c] = Acc128{};
    }
    advance(cc);
  }
  if (failed && threadIdx.x == 0) {
    atomicOr(err, kErrMacTimeout);
    for (uint64_t d = s; d < s + kMacStages - 1 && d < steps; ++d)  // copies still in flight
      mbar_wait(bar0 + 8 * (uint32_t)(d % kMacStages), (uint32_t)((d / kMacStages) & 1));
  }
}

template <int T, int TH>
constexpr size_t mac_stream_smem_bytes() {
  return 128 + kMacStages * ((size_t)MacShape<T, TH>::kBufWords * sizeof(uint64_t) + 8);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ntt_split(const uint64_t* data, uint64_t* out, uint32_t dk, const Modulus* mods, const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_ntt_split<LOGN>(BlockExec{}, smem, blockIdx.x, data, out, dk, mods, fwd);
}

__global__ void k_pk_prep(const uint64_t* pk, ulonglong2* prep, uint64_t items, uint32_t k, int logn,
                          const Modulus* mods) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < items; e += (uint64_t)gridDim.x * blockDim.x)
    pk_prep_item(e, pk, prep, k, logn, mods);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_enc0_prep(const uint64_t* samples, uint64_t* U, uint32_t k, const Modulus* mods, const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_enc0_prep<LOGN>(BlockExec{}, smem, blockIdx.x, samples, U, k, mods, fwd);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_enc0_xs(const uint64_t* samples, const ulonglong2* pk, const uint64_t* U, uint64_t* xs, uint32_t k,
              const Modulus* mods, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_enc0_xs<LOGN>(BlockExec{}, smem, blockIdx.x, samples, pk, U, xs, k, mods, inv);
}

// Rows (e, c, p) of E along y (grid-stride), kFinPer x 256 coefficients of a row per block
// along x; the row's coordinates are decoded once per block.
constexpr int kFinPer = 4;
__global__ void __launch_bounds__(256) k_enc0_fin(const uint64_t* samples, const uint64_t* xs, const uint64_t* mask,
                                                  uint64_t* E, uint64_t rows, uint32_t k, uint32_t dk, int logn,
                                                  const Modulus* mods, uint64_t q_mod_t, uint64_t upper_half,
                                                  uint64_t t, int tlog) {
  const uint32_t N = 1u << logn;
  for (uint64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const uint64_t e = r / (2 * dk);
    const uint32_t cp = (uint32_t)(r % (2 * dk)), c = cp / dk, p = cp % dk;
    const uint32_t z0 = blockIdx.x * (256 * kFinPer) + threadIdx.x;
    uint64_t v[kFinPer];
#pragma unroll
    for (int j = 0; j < kFinPer; ++j) {
      const uint32_t z = z0 + j * 256;
      if (z < N) v[j] = enc0_fin_elem(e, c, p, z, samples, xs, mask, k, logn, mods, q_mod_t, upper_half, t, tlog);
    }
#pragma unroll
    for (int j = 0; j < kFinPer; ++j) {
      const uint32_t z = z0 + j * 256;
      if (z < N) E[r * N + z] = v[j];
    }
  }
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_intt_protect(const uint64_t* acc, uint64_t* out, const uint64_t* U, const ulonglong2* pk, const uint64_t* E,
                   uint32_t k, uint32_t dk, const Modulus* mods, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_intt_protect<LOGN>(BlockExec{}, smem, blockIdx.x, acc, out, U, pk, E, k, dk, mods, inv);
}

// ---- n = 16384 transforms with each limb split between the two blocks of a cluster -----------
// For the ops whose only shared-memory work is one forward or inverse transform: a block holds
// half a limb (68 KiB instead of 136), so three blocks share an SM instead of one, and the level
// whose pairs straddle the halves runs through distributed shared memory (ntt_core.cuh).
// Launched by launch_pair: cluster dimension 2, limb i = blocks 2i and 2i + 1.
constexpr int kPairLogN = 14;
#define BFV_PAIR_BOUNDS __launch_bounds__(threads_for<kPairLogN - 1>(), blocks_per_sm<kPairLogN - 1>())

template <bool INV>
__global__ void BFV_PAIR_BOUNDS k_ntt_pair(uint64_t* data, uint32_t prime_count, uint32_t prime_offset,
                                           const Modulus* mods, const ulonglong2* fwd, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_ntt<kPairLogN>(ClusterPairExec{}, smem, blockIdx.x >> 1, INV, data, prime_count, prime_offset, mods, fwd, inv,
                    nullptr, nullptr);
}
__global__ void BFV_PAIR_BOUNDS k_lift_ntt_pair(const uint64_t* ring, uint64_t* out, uint32_t dk, const Modulus* mods,
                                                const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_lift_ntt<kPairLogN>(ClusterPairExec{}, smem, blockIdx.x >> 1, ring, out, dk, mods, fwd);
}
__global__ void BFV_PAIR_BOUNDS k_ntt_split_pair(const uint64_t* data, uint64_t* out, uint32_t dk, const Modulus* mods,
                                                 const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_ntt_split<kPairLogN>(ClusterPairExec{}, smem, blockIdx.x >> 1, data, out, dk, mods, fwd);
}
__global__ void BFV_PAIR_BOUNDS k_enc0_prep_pair(const uint64_t* samples, uint64_t* U, uint32_t k, const Modulus* mods,
                                                 const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_enc0_prep<kPairLogN>(ClusterPairExec{}, smem, blockIdx.x >> 1, samples, U, k, mods, fwd);
}
__global__ void BFV_PAIR_BOUNDS k_enc0_xs_pair(const uint64_t* samples, const ulonglong2* pk, const uint64_t* U,
                                               uint64_t* xs, uint32_t k, const Modulus* mods, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_enc0_xs<kPairLogN>(ClusterPairExec{}, smem, blockIdx.x >> 1, samples, pk, U, xs, k, mods, inv);
}
__global__ void BFV_PAIR_BOUNDS k_intt_protect_pair(const uint64_t* acc, uint64_t* out, const uint64_t* U,
                                                    const ulonglong2* pk, const uint64_t* E, uint32_t k, uint32_t dk,
                                                    const Modulus* mods, const ulonglong2* inv) {
  extern __shared__ uint64_t smem[];
  op_intt_protect<kPairLogN>(ClusterPairExec{}, smem, blockIdx.x >> 1, acc, out, U, pk, E, k, dk, mods, inv);
}

// Galois elements of up to kKeyBatch keys and their inverses mod 2n, passed by value.
constexpr int kKeyBatch = 256;
struct EltBatch {
  uint32_t elt[kKeyBatch];
  uint32_t ginv[kKeyBatch];
};

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_negntt(uint64_t* prepared, uint64_t prepared_words, EltBatch eb, uint32_t k, uint32_t dk,
                const Modulus* mods, const ulonglong2* fwd) {
  extern __shared__ uint64_t smem[];
  op_ks_negntt<LOGN>(BlockExec{}, smem, blockIdx.x, prepared, prepared_words, eb.elt, k, dk, mods, fwd);
}

__global__ void k_ks_keyperm(const uint64_t* keys, uint64_t* prepared, uint64_t prepared_words, EltBatch eb,
                             uint64_t items, int logn, uint32_t k, uint32_t dk, const Modulus* mods,
                             const uint64_t* qjp) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < items; e += (uint64_t)gridDim.x * blockDim.x)
    ks_keyperm_item(e, keys, prepared, prepared_words, eb.ginv, logn, k, dk, mods, qjp);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_rotate(const uint64_t* cts, const uint64_t* Y, const uint32_t* zflag, const uint64_t* prepared, uint64_t* x,
                uint32_t elt, uint32_t k, uint32_t dk, const Modulus* mods, const uint64_t* qjp,
                const ulonglong2* fwd, const ulonglong2* inv, const double2* fwd64, const double2* inv64) {
  extern __shared__ uint64_t smem[];
  op_ks_rotate<LOGN>(BlockExec{}, smem, blockIdx.x, cts, Y, zflag, prepared, x, elt, k, dk, mods, qjp, fwd, inv, fwd64,
                     inv64);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_finish(const uint64_t* x, const uint64_t* cts, uint64_t* out, uint32_t ginv, uint32_t k, uint32_t dk,
                const Modulus* mods) {
  extern __shared__ uint64_t smem[];
  op_ks_finish<LOGN>(BlockExec{}, smem, blockIdx.x, x, cts, out, ginv, k, dk, mods);
}

// One launch of the pipelined rotations: the special-prime blocks of one element beside the
// data-prime blocks (which finish the keyswitch in shared memory) of the previous one.
template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_rotate_pipe(const uint64_t* cts, uint64_t count, uint32_t order, const uint64_t* Y, const uint32_t* zflag,
                     uint64_t* x, const uint64_t* prep_s, uint32_t elt_s, uint64_t* xs_w, const uint64_t* prep_d, uint32_t elt_d,
                     uint32_t ginv_d, const uint64_t* xs_r, uint64_t* out_d, uint32_t k, uint32_t dk,
                     const Modulus* mods, const uint64_t* qjp, const ulonglong2* fwd, const ulonglong2* inv,
                     const double2* fwd64, const double2* inv64) {
  extern __shared__ uint64_t smem[];
  op_ks_rotate_pipe<LOGN>(BlockExec{}, smem, blockIdx.x, count, order, cts, Y, zflag, x, prep_s, elt_s, xs_w, prep_d,
                          elt_d, ginv_d, xs_r, out_d, k, dk, mods, qjp, fwd, inv, fwd64, inv64);
}

// Hoisted rotations of many (element, ciphertext) pairs in one launch pair.  paired != 0:
// ciphertext i with element i (blocks (i, c, p); x [count][2][k][n], out [count][2][dk][n]);
// else every element e with every ciphertext (x [m][count][2][k][n], out [m][count][2][dk][n]).
// Element e uses prepared key e (prepared + e * prepared_words).
template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_rotate_multi(const uint64_t* cts, uint64_t count, const uint64_t* Y, const uint32_t* zflag,
                      const uint64_t* prepared, uint64_t prepared_words, EltBatch eb, int paired, uint64_t* x,
                      uint32_t k, uint32_t dk, const Modulus* mods, const uint64_t* qjp, const ulonglong2* fwd,
                      const ulonglong2* inv, const double2* fwd64, const double2* inv64) {
  extern __shared__ uint64_t smem[];
  const uint64_t per = paired ? 2ull * k : count * 2 * k;
  const uint64_t e = blockIdx.x / per, blk = paired ? blockIdx.x : blockIdx.x % per;
  uint64_t* xe = paired ? x : x + ((e * count * 2 * k) << LOGN);
  op_ks_rotate<LOGN>(BlockExec{}, smem, blk, cts, Y, zflag, prepared + e * prepared_words, xe, eb.elt[e], k, dk, mods,
                     qjp, fwd, inv, fwd64, inv64);
}

template <int LOGN>
__global__ void __launch_bounds__(threads_for<LOGN>(), blocks_per_sm<LOGN>())
    k_ks_finish_multi(const uint64_t* x, const uint64_t* cts, uint64_t count, uint64_t* out, EltBatch eb, int paired,
                      uint32_t k, uint32_t dk, const Modulus* mods) {
  extern __shared__ uint64_t smem[];
  const uint64_t per = paired ? (uint64_t)dk : count * dk;
  const uint64_t e = blockIdx.x / per, blk = paired ? blockIdx.x : blockIdx.x % per;
  const uint64_t* xe = paired ? x : x + ((e * count * 2 * k) << LOGN);
  uint64_t* oe = paired ? out : out + ((e * count * 2 * dk) << LOGN);
  op_ks_finish<LOGN>(BlockExec{}, smem, blk, xe, cts, oe, eb.ginv[e], k, dk, mods);
}

// out [G][2][dk][n] -> acc [2][dk][n] = sum over the G ciphertexts (mod q_p), elementwise.
__global__ void k_sum_cts(const uint64_t* in, uint64_t groups, uint64_t* acc, uint32_t dk, int logn,
                          const Modulus* mods) {
  const uint64_t words = (2ull * dk) << logn;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < words; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t q = mods[(i >> logn) % dk].q;
    uint64_t v = 0;
    for (uint64_t g = 0; g < groups; ++g) v = add_mod(v, in[g * words + i], q);
    acc[i] = v;
  }
}

// c0 target gather (+ CRT): thread = (group, target)
__global__ void k_gather_targets(const uint64_t* out, const uint64_t* targets, const uint32_t* counts,
                                 uint32_t max_count, uint32_t dk, int logn, const Modulus* mods,
                                 const uint64_t* crt_part, const uint64_t* crt_inv, const uint64_t* crt_q,
                                 uint64_t* selected, uint64_t* crt) {
  const uint64_t g = blockIdx.y;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= counts[g]) return;
  const uint64_t N = uint64_t(1) << logn;
  const uint64_t idx = targets[g * max_count + i];
  uint64_t res[8];
  for (uint32_t p = 0; p < dk; ++p) {
    res[p] = out[((g * 2) * dk + p) * N + idx];
    selected[(g * dk + p) * max_count + i] = res[p];
  }
  if (crt) crt_target(res, dk, mods, crt_part, crt_inv, crt_q, crt + (g * max_count + i) * dk);
}

__global__ void k_moddown(const uint64_t* x, uint64_t* out, uint64_t groups, uint32_t k, uint32_t dk, int logn,
                          const Modulus* mods) {
  const uint64_t N = uint64_t(1) << logn;
  const uint64_t total = groups * 2 * dk * N;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = e & (N - 1);
    const uint64_t row = e >> logn;  // (g*2 + c)*dk + p
    const uint32_t p = (uint32_t)(row % dk);
    const uint64_t gc = row / dk;
    const uint64_t* xr = x + gc * k * N;
    out[e] = moddown_elem(xr[(uint64_t)p * N + i], xr[(uint64_t)(k - 1) * N + i], mods[p], mods[k - 1]);
  }
}

// out [cts][2][dk][n]: c0 of ciphertext j += Delta-scaled plain [j][n] (coefficient form).
__global__ void k_add_plain_many(uint64_t* out, const uint64_t* plain, uint64_t cts, uint32_t dk, int logn,
                                 const Modulus* mods, uint64_t q_mod_t, uint64_t upper_half, uint64_t t, int tlog) {
  const uint64_t N = uint64_t(1) << logn, total = cts * dk * N;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = e & (N - 1), row = e >> logn, j = row / dk;
    const uint32_t p = (uint32_t)(row % dk);
    const Modulus& m = mods[p];
    uint64_t* a = out + ((j * 2 * dk + p) << logn) + i;
    *a = add_mod(*a, scale_plain_coeff(plain[(j << logn) + i], q_mod_t, upper_half, t, tlog, m), m.q);
  }
}

// ---------------------------------------------------------------------------------
// small elementwise kernels
// ---------------------------------------------------------------------------------
__global__ void k_packing_prepare(const uint64_t* left, const uint64_t* right, uint64_t* sum, uint64_t* diff,
                                  uint32_t dk, int logn, uint32_t shift, const Modulus* mods) {
  const uint64_t N = uint64_t(1) << logn;
  const uint64_t total = 2 * (uint64_t)dk * N;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t j = e & (N - 1), base = e - j;
    const uint64_t q = mods[(e >> logn) % dk].q;
    const uint64_t src = (j + N - shift) & (N - 1);
    uint64_t v = right[base + src];
    if (j < shift) v = neg_mod(v, q);
    sum[e] = add_mod(left[e], v, q);
    diff[e] = sub_mod(left[e], v, q);
  }
}

// One level of the packing tree for many pairs: pair (m, s) merges left = in[2m][s] with
// right = in[2m+1][s] (ciphertexts [2][dk][n], `slots` per row) into sum / diff [m][s].
__global__ void k_packing_prepare_many(const uint64_t* in, uint64_t pairs, uint64_t slots, uint64_t* sum,
                                       uint64_t* diff, uint32_t dk, int logn, uint32_t shift, const Modulus* mods) {
  const uint64_t N = uint64_t(1) << logn, ctw = 2ull * dk * N;
  const uint64_t total = pairs * slots * ctw;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t ps = e / ctw, w = e - ps * ctw, m = ps / slots, sl = ps - m * slots;
    const uint64_t j = w & (N - 1), base = w - j;
    const uint64_t* left = in + ((2 * m) * slots + sl) * ctw;
    const uint64_t* right = in + ((2 * m + 1) * slots + sl) * ctw;
    const uint64_t q = mods[(w >> logn) % dk].q;
    const uint64_t src = (j + N - shift) & (N - 1);
    uint64_t v = right[base + src];
    if (j < shift) v = neg_mod(v, q);
    sum[e] = add_mod(left[w], v, q);
    diff[e] = sub_mod(left[w], v, q);
  }
}

// c0 [dk][n] += Delta-scaled plaintext coefficient (add_plain with the scaling variant),
// for coefficients i < count (bfv_matrix.inc:40-46: encrypt_zero then add_plain_inplace).
// Output protection of coefficient-form ciphertexts [items][2][dk][n]: out = ct + Enc(0) -
// [c = 0] Delta mask, with Enc(0) = moddown(x) from its pre-moddown polys x [items][2][k][n]
// (nullable) and mask [items][n] ring-59 words (nullable).  The tile return of
// bfv_token_batch.inc:271-272 (sub_plain_inplace(mask), encrypt_zero, add_inplace) in one pass.
__global__ void k_protect_ct(const uint64_t* ct, const uint64_t* x, const uint64_t* mask, uint64_t* out, uint64_t items,
                             uint32_t k, uint32_t dk, int logn, const Modulus* mods, uint64_t q_mod_t,
                             uint64_t upper_half, uint64_t t, int tlog) {
  const uint64_t N = uint64_t(1) << logn;
  const uint64_t total = items * 2 * dk * N;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = e & (N - 1);
    const uint64_t row = e >> logn;  // (item*2 + c)*dk + p
    const uint32_t p = (uint32_t)(row % dk);
    const uint64_t gc = row / dk;
    const Modulus& m = mods[p];
    uint64_t v = ct[e];
    if (x) {
      const uint64_t* xr = x + gc * k * N;
      v = add_mod(v, moddown_elem(xr[(uint64_t)p * N + i], xr[(uint64_t)(k - 1) * N + i], m, mods[k - 1]), m.q);
    }
    if (mask && (gc & 1) == 0)
      v = sub_mod(v, scale_plain_coeff(mask[(gc >> 1) * N + i], q_mod_t, upper_half, t, tlog, m), m.q);
    out[e] = v;
  }
}
// The packed-tile targets of bfv_acyclic_pack.hpp:53-56 for `slots` tiles: targets
// [slots][512] = 32 * (9-bit reversal of the coordinate), counts [slots] = 512.
__global__ void k_packed_targets(uint64_t* targets, uint32_t* counts, uint64_t slots) {
  const uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (e < slots * 512) targets[e] = (uint64_t)(__brev((uint32_t)(e & 511)) >> 23) * 32;
  if (e < slots) counts[e] = 512;
}
__global__ void k_add_plain(uint64_t* c0, const uint64_t* plain, uint64_t count, uint32_t dk, int logn,
                            const Modulus* mods, uint64_t q_mod_t, uint64_t upper_half, uint64_t t, int tlog) {
  const uint64_t total = (uint64_t)dk * count;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t p = (uint32_t)(e / count);
    const uint64_t i = e % count;
    const Modulus& m = mods[p];
    uint64_t* a = c0 + ((uint64_t)p << logn) + i;
    *a = add_mod(*a, scale_plain_coeff(plain[i], q_mod_t, upper_half, t, tlog, m), m.q);
  }
}

__global__ void k_add(uint64_t* a, const uint64_t* b, uint64_t polys, uint32_t dk, int logn, const Modulus* mods) {
  const uint64_t total = polys << logn;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x)
    a[e] = add_mod(a[e], b[e], mods[(e >> logn) % dk].q);
}

__global__ void k_check_canonical(const uint64_t* data, uint64_t polys, uint32_t count, uint32_t offset, int logn,
                                  const Modulus* mods, uint32_t* bad) {
  const uint64_t total = polys << logn;
  uint32_t found = 0;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x)
    found |= data[e] >= mods[offset + (e >> logn) % count].q;
  if (__any_sync(0xffffffffu, found) && (threadIdx.x & 31) == 0) atomicOr(bad, 1u);
}

// ---------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------
bool logn_supported(int logn) { return logn == 5 || logn == 6 || (logn >= 12 && logn <= 14); }

#define BFV_DISPATCH(LOGN_VAR, ...)                      \
  switch (LOGN_VAR) {                                     \
    case 5: { constexpr int L_ = 5; __VA_ARGS__; } break;   \
    case 6: { constexpr int L_ = 6; __VA_ARGS__; } break;   \
    case 12: { constexpr int L_ = 12; __VA_ARGS__; } break; \
    case 13: { constexpr int L_ = 13; __VA_ARGS__; } break; \
    case 14: { constexpr int L_ = 14; __VA_ARGS__; } break; \
    default: return cudaErrorInvalidValue;                \
  }

template <class K>
static cudaError_t allow_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int L>
static cudaError_t configure_for() {
  const size_t s = smem_bytes<L>();
  cudaError_t e = cudaSuccess;
  auto chk = [&](cudaError_t r) { if (e == cudaSuccess) e = r; };
  chk(allow_smem(k_ntt<L, false>, s));
  chk(allow_smem(k_ntt<L, true>, s));
  chk(allow_smem(k_lift_ntt<L>, s));
  chk(allow_smem(k_mac_intt<L>, s));
  chk(allow_smem(k_ks_main<L>, s));
  chk(allow_smem(k_ks_moddown<L>, (size_t(1) << L) * 8));
  chk(allow_smem(k_enc0_x<L>, s));
  chk(allow_smem(k_ks_hoist<L>, s));
  chk(allow_smem(k_ks_negntt<L>, s));
  chk(allow_smem(k_ks_rotate<L>, s));
  chk(allow_smem(k_ks_finish<L>, (size_t(1) << L) * 8));
  chk(allow_smem(k_ks_rotate_multi<L>, s));
  chk(allow_smem(k_ks_rotate_pipe<L>, s));
  chk(allow_smem(k_ks_finish_multi<L>, (size_t(1) << L) * 8));
  chk(allow_smem(k_client_phase<L>, s));
  chk(allow_smem(k_enc0_prep<L>, s));
  chk(allow_smem(k_enc0_xs<L>, s));
  chk(allow_smem(k_ntt_split<L>, s));
  chk(allow_smem(k_mac_split<8, 4>, mac_smem_bytes<8, 4>()));
  chk(allow_smem(k_mac_split<4, 4>, mac_smem_bytes<4, 4>()));
  chk(allow_smem(k_mac_split<2, 2>, mac_smem_bytes<2, 2>()));
  chk(allow_smem(k_mac_split<1, 1>, mac_smem_bytes<1, 1>()));
  chk(allow_smem(k_mac_stream<8, 4>, mac_stream_smem_bytes<8, 4>()));
  chk(allow_smem(k_mac_stream<4, 4>, mac_stream_smem_bytes<4, 4>()));
  chk(allow_smem(k_mac_stream<2, 2>, mac_stream_smem_bytes<2, 2>()));
  chk(allow_smem(k_mac_stream<1, 1>, mac_stream_smem_bytes<1, 1>()));
  chk(allow_smem(k_mac_tc<32>, tc::Smem<32>::kLaunchBytes));
  chk(allow_smem(k_mac_tc<64>, tc::Smem<64>::kLaunchBytes));
  chk(allow_smem(k_intt_protect<L>, s));
  if constexpr (L == 14) {
    const size_t half = smem_bytes<L - 1>();
    chk(allow_smem(k_ntt_pair<false>, half));
    chk(allow_smem(k_ntt_pair<true>, half));
    chk(allow_smem(k_lift_ntt_pair, half));
    chk(allow_smem(k_ntt_split_pair, half));
    chk(allow_smem(k_enc0_prep_pair, half));
    chk(allow_smem(k_enc0_xs_pair, half));
    chk(allow_smem(k_intt_protect_pair, half));
    chk(allow_smem(k_token_lift_ntt<L>, s));
    chk(allow_smem(k_token_mac_intt<L>, s));
    chk(allow_smem(k_token_lift_ntt_many<L>, s));
    chk(allow_smem(k_token_mac_intt_many<L>, s));
  }
  return e;
}

cudaError_t configure_kernels(int logn) {
  BFV_DISPATCH(logn, return configure_for<L_>());
  return cudaSuccess;
}

static unsigned elementwise_blocks(uint64_t total) {
  uint64_t b = (total + 255) / 256;
  const uint64_t cap = 148ull * 16;
  return (unsigned)(b < cap ? (b ? b : 1) : cap);
}

// Launch of a pair kernel over `limbs` limbs: 2 x limbs blocks in clusters of 2.
template <class... KArgs, class... Args>
static cudaError_t launch_pair(void (*kernel)(KArgs...), uint64_t limbs, cudaStream_t st, Args... args) {
  if (2 * limbs > 0x7fffffffull) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * limbs));
  cfg.blockDim = dim3(threads_for<kPairLogN - 1>());
  cfg.dynamicSmemBytes = smem_bytes<kPairLogN - 1>();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
static bool use_pair(const DevParams& P) { return P.logn == kPairLogN && P.split_limbs; }

cudaError_t launch_ntt(const DevParams& P, uint64_t* data, uint64_t polys, uint32_t prime_count,
                       uint32_t prime_offset, bool inverse, cudaStream_t st) {
  const LaunchRange range("bfvgpu:ntt");
  if (!polys) return cudaSuccess;
  if (use_pair(P))
    return inverse ? launch_pair(k_ntt_pair<true>, polys, st, data, prime_count, prime_offset, P.mod, P.fwd, P.inv)
                   : launch_pair(k_ntt_pair<false>, polys, st, data, prime_count, prime_offset, P.mod, P.fwd, P.inv);
  BFV_DISPATCH(P.logn, {
    if (inverse)
      k_ntt<L_, true><<<(unsigned)polys, threads_for<L_>(), smem_bytes<L_>(), st>>>(data, prime_count, prime_offset,
                                                                                 P.mod, P.fwd, P.inv, P.fwd64, P.inv64);
    else
      k_ntt<L_, false><<<(unsigned)polys, threads_for<L_>(), smem_bytes<L_>(), st>>>(data, prime_count, prime_offset,
                                                                                  P.mod, P.fwd, P.inv, P.fwd64, P.inv64);
  });
  return cudaGetLastError();
}

cudaError_t launch_lift_ntt(const DevParams& P, const uint64_t* ring, uint64_t* out, uint64_t blocks,
                            cudaStream_t st) {
  const LaunchRange range("bfvgpu:lift_ntt");
  if (!blocks) return cudaSuccess;
  if (use_pair(P)) return launch_pair(k_lift_ntt_pair, blocks * P.dk, st, ring, out, P.dk, P.mod, P.fwd);
  BFV_DISPATCH(P.logn, {
    k_lift_ntt<L_><<<(unsigned)(blocks * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(ring, out, P.dk, P.mod,
                                                                                            P.fwd);
  });
  return cudaGetLastError();
}

cudaError_t launch_mac_intt(const DevParams& P, const uint64_t* in, const uint64_t* w, uint64_t* out,
                            uint64_t inputs, uint64_t groups, const Protect& prot, cudaStream_t st) {
  const LaunchRange range("bfvgpu:mac_intt");
  if (!groups) return cudaSuccess;
  ProtectArgs a{prot.mask, prot.enc0_x, P.q_mod_t, P.upper_half, P.t, P.tlog};
  BFV_DISPATCH(P.logn, {
    k_mac_intt<L_><<<(unsigned)(groups * 2 * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(
        in, w, out, (uint32_t)inputs, P.k, P.dk, P.mod, P.inv, a);
  });
  return cudaGetLastError();
}

cudaError_t launch_gather_targets(const DevParams& P, const uint64_t* out, const uint64_t* targets,
                                  const uint32_t* counts, uint32_t max_count, uint64_t groups, uint64_t* selected,
                                  uint64_t* crt, cudaStream_t st) {
  const LaunchRange range("bfvgpu:gather_targets");
  if (!groups || !max_count) return cudaSuccess;
  if (P.dk > 8) return cudaErrorInvalidValue;
  dim3 grid((max_count + 127) / 128, (unsigned)groups);
  k_gather_targets<<<grid, 128, 0, st>>>(out, targets, counts, max_count, P.dk, P.logn, P.mod, P.crt_part,
                                         P.crt_inv, P.crt_q, selected, crt);
  return cudaGetLastError();
}

static uint32_t inverse_mod_2n(uint32_t g, uint32_t two_n) {
  // g odd; the units mod 2^m have exponent dividing 2^(m-1) = n, so g^(n-1) = g^-1.
  uint64_t r = 1, b = g % two_n, e = two_n / 2 - 1;
  while (e) {
    if (e & 1) r = (r * b) % two_n;
    b = (b * b) % two_n;
    e >>= 1;
  }
  return (uint32_t)r;
}

cudaError_t launch_keyswitch(const DevParams& P, const uint64_t* cts, const uint64_t* key, uint32_t elt,
                             uint64_t count, uint64_t* acc, uint64_t* out, cudaStream_t st) {
  const LaunchRange range("bfvgpu:keyswitch");
  if (!count) return cudaSuccess;
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  const uint32_t ginv = inverse_mod_2n(elt, 2 * P.n);
  BFV_DISPATCH(P.logn, {
    k_ks_main<L_><<<(unsigned)(count * P.k), threads_for<L_>(), smem_bytes<L_>(), st>>>(cts, key, acc, elt, P.k,
                                                                                        P.dk, P.mod, P.qjp, P.fwd,
                                                                                        P.inv, P.fwd64, P.inv64);
    k_ks_moddown<L_><<<(unsigned)(count * P.dk), threads_for<L_>(), (size_t(1) << L_) * 8, st>>>(acc, cts, out, ginv,
                                                                                                 P.k, P.dk, P.mod);
  });
  return cudaGetLastError();
}

cudaError_t launch_ks_hoist(const DevParams& P, const uint64_t* cts, uint64_t count, uint64_t* Y, uint32_t* zflag,
                            cudaStream_t st) {
  const LaunchRange range("bfvgpu:ks_hoist");
  if (!count) return cudaSuccess;
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(zflag, 0, count * sizeof(uint32_t), st);
  if (e != cudaSuccess) return e;
  BFV_DISPATCH(P.logn, {
    k_ks_hoist<L_><<<(unsigned)(count * P.dk * P.k), threads_for<L_>(), smem_bytes<L_>(), st>>>(cts, Y, zflag, P.k,
                                                                                               P.dk, P.mod, P.fwd);
  });
  return cudaGetLastError();
}

cudaError_t launch_ks_keyprep(const DevParams& P, const uint64_t* keys, const uint32_t* elts, uint64_t count,
                              uint64_t* prepared, cudaStream_t st) {
  const LaunchRange range("bfvgpu:ks_keyprep");
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  const uint64_t pw = ks_prepared_words(P.k, P.dk, P.n);
  const uint64_t kw = 2ull * P.dk * P.k * P.n;
  for (uint64_t first = 0; first < count; first += kKeyBatch) {
    const uint64_t m = count - first < (uint64_t)kKeyBatch ? count - first : (uint64_t)kKeyBatch;
    EltBatch eb{};
    for (uint64_t r = 0; r < m; ++r) {
      eb.elt[r] = elts[first + r];
      eb.ginv[r] = inverse_mod_2n(elts[first + r], 2 * P.n);
    }
    uint64_t* pr = prepared + first * pw;
    BFV_DISPATCH(P.logn, {
      k_ks_negntt<L_><<<(unsigned)(m * P.k), threads_for<L_>(), smem_bytes<L_>(), st>>>(pr, pw, eb, P.k, P.dk, P.mod,
                                                                                        P.fwd);
    });
    const uint64_t items = m * P.k * P.n;
    k_ks_keyperm<<<elementwise_blocks(items), 256, 0, st>>>(keys + first * kw, pr, pw, eb, items, P.logn, P.k, P.dk,
                                                           P.mod, P.qjp);
  }
  return cudaGetLastError();
}

cudaError_t launch_ks_rotate(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                             const uint32_t* zflag, const uint64_t* prepared, uint32_t elt, uint64_t* x, uint64_t* out,
                             cudaStream_t st) {
  const LaunchRange range("bfvgpu:ks_rotate");
  if (!count) return cudaSuccess;
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  const uint32_t ginv = inverse_mod_2n(elt, 2 * P.n);
  BFV_DISPATCH(P.logn, {
    k_ks_rotate<L_><<<(unsigned)(count * 2 * P.k), threads_for<L_>(), smem_bytes<L_>(), st>>>(
        cts, Y, zflag, prepared, x, elt, P.k, P.dk, P.mod, P.qjp, P.fwd, P.inv, P.fwd64, P.inv64);
    k_ks_finish<L_><<<(unsigned)(count * P.dk), threads_for<L_>(), (size_t(1) << L_) * 8, st>>>(x, cts, out, ginv,
                                                                                               P.k, P.dk, P.mod);
  });
  return cudaGetLastError();
}

cudaError_t launch_ks_rotate_pipe_step(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                                       const uint32_t* zflag, const uint64_t* prepared, const uint32_t* elts,
                                       uint64_t elements, uint64_t r, uint64_t* x, uint64_t* xs, uint64_t* out_d,
                                       cudaStream_t st) {
  if (!count || r > elements) return cudaSuccess;
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  const uint64_t pw = ks_prepared_words(P.k, P.dk, P.n), xsw = count * 2ull * P.n;
  const bool special = r < elements, data = r >= 1;
  const uint64_t blocks = (special ? count * 2 : 0) + (data ? count * 2 * P.dk : 0);
  const uint32_t order = special ? 1u : 0u;
  if (!blocks) return cudaSuccess;
  const uint64_t* prep_s = special ? prepared + r * pw : nullptr;
  const uint32_t elt_s = special ? elts[r] : 1;
  uint64_t* xs_w = xs + (r & 1) * xsw;
  const uint64_t* prep_d = data ? prepared + (r - 1) * pw : nullptr;
  const uint32_t elt_d = data ? elts[r - 1] : 1, ginv_d = inverse_mod_2n(elt_d, 2u * P.n);
  const uint64_t* xs_r = xs + ((r + 1) & 1) * xsw;  // written by launch r - 1
  BFV_DISPATCH(P.logn, {
    k_ks_rotate_pipe<L_><<<(unsigned)blocks, threads_for<L_>(), smem_bytes<L_>(), st>>>(
        cts, count, order, Y, zflag, x, prep_s, elt_s, xs_w, prep_d, elt_d, ginv_d, xs_r, data ? out_d : nullptr, P.k,
        P.dk, P.mod, P.qjp, P.fwd, P.inv, P.fwd64, P.inv64);
  });
  return cudaGetLastError();
}

cudaError_t launch_ks_rotate_pipe(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                                  const uint32_t* zflag, const uint64_t* prepared, const uint32_t* elts,
                                  uint64_t elements, uint64_t* x, uint64_t* xs, uint64_t* const* outs, cudaStream_t st) {
  const LaunchRange range("bfvgpu:ks_rotate_pipe");
  if (!count || !elements) return cudaSuccess;
  for (uint64_t r = 0; r <= elements; ++r) {
    const cudaError_t e =
        launch_ks_rotate_pipe_step(P, cts, count, Y, zflag, prepared, elts, elements, r, x, xs, r ? outs[r - 1] : nullptr, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_ks_rotate_multi(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                                   const uint32_t* zflag, const uint64_t* prepared, const uint32_t* elts,
                                   uint64_t elements, int paired, uint64_t* x, uint64_t* out, cudaStream_t st) {
  const LaunchRange range("bfvgpu:ks_rotate_multi");
  if (!count || !elements) return cudaSuccess;
  if (P.k != P.dk + 1 || (paired && elements != count)) return cudaErrorInvalidValue;
  const uint64_t pw = ks_prepared_words(P.k, P.dk, P.n);
  const uint64_t ctw = 2ull * P.dk * P.n, yw = (uint64_t)P.dk * P.k * P.n, xw = 2ull * P.k * P.n;
  for (uint64_t first = 0; first < elements; first += kKeyBatch) {
    const uint64_t m = elements - first < (uint64_t)kKeyBatch ? elements - first : (uint64_t)kKeyBatch;
    EltBatch eb{};
    for (uint64_t r = 0; r < m; ++r) {
      eb.elt[r] = elts[first + r];
      eb.ginv[r] = inverse_mod_2n(elts[first + r], 2 * P.n);
    }
    // paired: this chunk's ciphertexts are first..first+m; else all ciphertexts, elements first..
    const uint64_t c0 = paired ? first : 0, cn = paired ? m : count;
    const uint64_t* cp = cts + c0 * ctw;
    const uint64_t* yp = Y + c0 * yw;
    const uint32_t* zp = zflag + c0;
    uint64_t* xp = paired ? x + c0 * xw : x;
    uint64_t* op = paired ? out + c0 * ctw : out + first * count * ctw;
    const uint64_t rot_blocks = m * (paired ? 1 : cn) * 2 * P.k, fin_blocks = m * (paired ? 1 : cn) * P.dk;
    if (rot_blocks > 0x7fffffffull) return cudaErrorInvalidValue;
    BFV_DISPATCH(P.logn, {
      k_ks_rotate_multi<L_><<<(unsigned)rot_blocks, threads_for<L_>(), smem_bytes<L_>(), st>>>(
          cp, cn, yp, zp, prepared + first * pw, pw, eb, paired, xp, P.k, P.dk, P.mod, P.qjp, P.fwd, P.inv,
          P.fwd64, P.inv64);
      k_ks_finish_multi<L_><<<(unsigned)fin_blocks, threads_for<L_>(), (size_t(1) << L_) * 8, st>>>(
          xp, cp, cn, op, eb, paired, P.k, P.dk, P.mod);
    });
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_sum_cts(const DevParams& P, const uint64_t* in, uint64_t groups, uint64_t* acc, cudaStream_t st) {
  const LaunchRange range("bfvgpu:sum_cts");
  const uint64_t words = (2ull * P.dk) << P.logn;
  k_sum_cts<<<elementwise_blocks(words), 256, 0, st>>>(in, groups, acc, P.dk, P.logn, P.mod);
  return cudaGetLastError();
}

cudaError_t launch_enc0_x(const DevParams& P, const uint64_t* samples, const uint64_t* pk, uint64_t* u_ntt,
                          uint64_t* x, uint64_t groups, cudaStream_t st) {
  const LaunchRange range("bfvgpu:enc0_x");
  if (!groups) return cudaSuccess;
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  BFV_DISPATCH(P.logn, {
    k_enc0_x<L_><<<(unsigned)(groups * P.k), threads_for<L_>(), smem_bytes<L_>(), st>>>(samples, pk, u_ntt, x, P.k,
                                                                                       P.mod, P.fwd, P.inv);
  });
  return cudaGetLastError();
}

cudaError_t launch_moddown(const DevParams& P, const uint64_t* x, uint64_t* out, uint64_t groups, cudaStream_t st) {
  const LaunchRange range("bfvgpu:moddown");
  if (!groups) return cudaSuccess;
  if (P.k != P.dk + 1) return cudaErrorInvalidValue;
  const uint64_t total = groups * 2 * P.dk * P.n;
  k_moddown<<<elementwise_blocks(total), 256, 0, st>>>(x, out, groups, P.k, P.dk, P.logn, P.mod);
  return cudaGetLastError();
}

cudaError_t launch_client_phase(const DevParams& P, uint64_t* data, const uint64_t* sk, uint64_t batches,
                                cudaStream_t st) {
  const LaunchRange range("bfvgpu:client_phase");
  if (!batches) return cudaSuccess;
  BFV_DISPATCH(P.logn, {
    k_client_phase<L_><<<(unsigned)(batches * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(data, sk, P.dk,
                                                                                               P.mod, P.fwd, P.inv);
  });
  return cudaGetLastError();
}

cudaError_t launch_check_canonical(const DevParams& P, const uint64_t* data, uint64_t polys, uint32_t prime_count,
                                   uint32_t prime_offset, uint32_t* bad, cudaStream_t st) {
  const LaunchRange range("bfvgpu:check_canonical");
  if (!polys) return cudaSuccess;
  k_check_canonical<<<elementwise_blocks(polys << P.logn), 256, 0, st>>>(data, polys, prime_count, prime_offset,
                                                                         P.logn, P.mod, bad);
  return cudaGetLastError();
}

cudaError_t launch_token_evaluate(const DevParams& P, const uint64_t* inputs, uint64_t slots, const uint64_t* ring,
                                  const uint64_t* scaled, uint64_t* wscratch, uint64_t* acc, uint64_t* out,
                                  cudaStream_t st) {
  const LaunchRange range("bfvgpu:token_evaluate");
  (void)acc;
  if (P.logn != 14) return cudaErrorInvalidValue;
  constexpr int L_ = 14;
  k_token_lift_ntt<L_><<<kTokenBlocks * P.dk, threads_for<L_>(), smem_bytes<L_>(), st>>>(ring, wscratch, P.dk, P.mod,
                                                                                        P.fwd);
  k_token_mac_intt<L_><<<(unsigned)(slots * 2 * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(
      inputs, wscratch, scaled, out, (uint32_t)slots, P.dk, P.mod, P.inv);
  return cudaGetLastError();
}

cudaError_t launch_token_evaluate_many(const DevParams& P, const uint64_t* inputs, uint64_t slots, const uint64_t* ring,
                                       uint64_t coords, const uint64_t* local, uint64_t* scaled, uint64_t* wscratch,
                                       uint64_t* out, cudaStream_t st) {
  const LaunchRange range("bfvgpu:token_evaluate_many");
  if (!coords || !slots) return cudaSuccess;
  if (P.logn != 14 || coords * kTokenBlocks * P.dk > 0x7fffffffull || coords * slots * 2 * P.dk > 0x7fffffffull)
    return cudaErrorInvalidValue;
  constexpr int L_ = 14;
  k_scale_local<<<elementwise_blocks(coords * slots * P.dk), 256, 0, st>>>(local, coords * slots, scaled, P.dk, P.mod,
                                                                         P.q_mod_t, P.upper_half, P.t, P.tlog);
  k_token_lift_ntt_many<L_><<<(unsigned)(coords * kTokenBlocks * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(
      ring, wscratch, P.dk, P.mod, P.fwd);
  k_token_mac_intt_many<L_><<<(unsigned)(coords * slots * 2 * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(
      inputs, wscratch, scaled, out, (uint32_t)slots, P.dk, P.mod, P.inv);
  return cudaGetLastError();
}

cudaError_t launch_packing_prepare_many(const DevParams& P, const uint64_t* in, uint64_t pairs, uint64_t slots,
                                        uint64_t* sum, uint64_t* diff, unsigned level, cudaStream_t st) {
  const LaunchRange range("bfvgpu:packing_prepare_many");
  if (!pairs || !slots) return cudaSuccess;
  const uint64_t total = pairs * slots * 2 * (uint64_t)P.dk * P.n;
  k_packing_prepare_many<<<elementwise_blocks(total), 256, 0, st>>>(in, pairs, slots, sum, diff, P.dk, P.logn,
                                                                   P.n >> (level + 1), P.mod);
  return cudaGetLastError();
}

cudaError_t launch_packing_prepare(const DevParams& P, const uint64_t* left, const uint64_t* right, uint64_t* sum,
                                   uint64_t* diff, unsigned level, cudaStream_t st) {
  const LaunchRange range("bfvgpu:packing_prepare");
  const uint64_t total = 2 * (uint64_t)P.dk * P.n;
  k_packing_prepare<<<elementwise_blocks(total), 256, 0, st>>>(left, right, sum, diff, P.dk, P.logn,
                                                              P.n >> (level + 1), P.mod);
  return cudaGetLastError();
}

cudaError_t launch_add_plain(const DevParams& P, uint64_t* c0, const uint64_t* plain, uint64_t count,
                             cudaStream_t st) {
  const LaunchRange range("bfvgpu:add_plain");
  if (!count) return cudaSuccess;
  k_add_plain<<<elementwise_blocks(count * P.dk), 256, 0, st>>>(c0, plain, count, P.dk, P.logn, P.mod, P.q_mod_t,
                                                               P.upper_half, P.t, P.tlog);
  return cudaGetLastError();
}

cudaError_t launch_encrypt_many(const DevParams& P, const uint64_t* samples, const uint64_t* pk, const uint64_t* plain,
                                uint64_t cts, uint64_t* u_ntt, uint64_t* x, uint64_t* out, cudaStream_t st) {
  const LaunchRange range("bfvgpu:encrypt_many");
  if (!cts) return cudaSuccess;
  cudaError_t e = launch_enc0_x(P, samples, pk, u_ntt, x, cts, st);
  if (e == cudaSuccess) e = launch_moddown(P, x, out, cts, st);
  if (e != cudaSuccess) return e;
  k_add_plain_many<<<elementwise_blocks(cts * P.dk * P.n), 256, 0, st>>>(out, plain, cts, P.dk, P.logn, P.mod,
                                                                         P.q_mod_t, P.upper_half, P.t, P.tlog);
  return cudaGetLastError();
}

cudaError_t launch_protect_ct(const DevParams& P, const uint64_t* cts, uint64_t items, const uint64_t* masks,
                              const uint64_t* samples, const uint64_t* pk, uint64_t* u_ntt, uint64_t* x, uint64_t* out,
                              cudaStream_t st) {
  const LaunchRange range("bfvgpu:protect_ct");
  if (!items) return cudaSuccess;
  if (samples) {
    const cudaError_t e = launch_enc0_x(P, samples, pk, u_ntt, x, items, st);
    if (e != cudaSuccess) return e;
  }
  k_protect_ct<<<elementwise_blocks(items * 2 * P.dk * P.n), 256, 0, st>>>(
      cts, samples ? x : nullptr, masks, out, items, P.k, P.dk, P.logn, P.mod, P.q_mod_t, P.upper_half, P.t, P.tlog);
  return cudaGetLastError();
}

cudaError_t launch_packed_targets(uint64_t* targets, uint32_t* counts, uint64_t slots, cudaStream_t st) {
  const LaunchRange range("bfvgpu:packed_targets");
  if (!slots) return cudaSuccess;
  k_packed_targets<<<(unsigned)((slots * 512 + 255) / 256), 256, 0, st>>>(targets, counts, slots);
  return cudaGetLastError();
}

cudaError_t launch_add(const DevParams& P, uint64_t* a, const uint64_t* b, uint64_t polys, cudaStream_t st) {
  const LaunchRange range("bfvgpu:add");
  if (!polys) return cudaSuccess;
  k_add<<<elementwise_blocks(polys << P.logn), 256, 0, st>>>(a, b, polys, P.dk, P.logn, P.mod);
  return cudaGetLastError();
}

template <int T, int TH>
static cudaError_t mac_split_launch(const DevParams& P, const uint64_t* in, uint64_t inputs, const uint64_t* w,
                                    uint64_t groups, uint64_t* out, cudaStream_t st) {
  using S = MacShape<T, TH>;
  const size_t smem = mac_smem_bytes<T, TH>();
  const uint64_t gblocks = (groups + S::GB - 1) / S::GB;
  const uint64_t units = (uint64_t)P.dk * (P.n >> 5) * gblocks;
  if (units > 0xffffffffull) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const uint64_t avail = sms > P.reserved_sms ? (uint64_t)(sms - P.reserved_sms) : 1;
  const unsigned grid = (unsigned)(units < avail ? units : avail);
  k_mac_split<T, TH><<<grid, S::kThreads, smem, st>>>(in, w, out, (uint32_t)inputs, (uint32_t)groups,
                                                      (uint32_t)gblocks, (uint32_t)units, P.dk, P.logn, P.mod);
  return cudaGetLastError();
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tensor maps of one launch: inputs [8 tiles][I][2][dk][n] viewed as (z, b, c, t, p) with box
// (2, KPAD, 2, 4, 1); weights [G][I][dk][n] viewed as (z, b, g, p) with box (2, KPAD, 16, 1);
// both u64, no swizzle (dense box images), zero fill past the extents.
template <int KPAD>
static cudaError_t encode_mac_maps(const DevParams& P, const uint64_t* in, uint64_t inputs, const uint64_t* w,
                                   uint64_t groups, CUtensorMap* a, CUtensorMap* b) {
  auto enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t n = P.n, dk = P.dk, I = inputs, G = groups;
  const cuuint64_t dimA[5] = {n, I, 2, (cuuint64_t)tc::kTiles, dk};
  const cuuint64_t strA[4] = {2 * dk * n * 8, dk * n * 8, I * 2 * dk * n * 8, n * 8};
  const cuuint32_t boxA[5] = {2, (cuuint32_t)KPAD, 2, 4, 1};
  const cuuint64_t dimB[4] = {n, I, G, dk};
  const cuuint64_t strB[3] = {dk * n * 8, I * dk * n * 8, n * 8};
  const cuuint32_t boxB[4] = {2, (cuuint32_t)KPAD, (cuuint32_t)tc::kGroupsRound, 1};
  const cuuint32_t ones[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(a, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5, const_cast<uint64_t*>(in), dimA, strA, boxA, ones,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  r = enc(b, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<uint64_t*>(w), dimB, strB, boxB, ones,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Tensor maps of a streamed product launch: inputs [T][I][2][dk][n] as (z, p, c, b, t) with
// box (32, 1, 2, 8, T); weights [G][I][dk][n] as (z, p, b, g) with box (32, 1, 8, GB).
template <int T, int TH>
static cudaError_t encode_stream_maps(const DevParams& P, const uint64_t* in, uint64_t inputs, const uint64_t* w,
                                      uint64_t groups, CUtensorMap* mi, CUtensorMap* mw) {
  using S = MacShape<T, TH>;
  auto enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t n = P.n, dk = P.dk, I = inputs, G = groups;
  const cuuint64_t dimI[5] = {n, dk, 2, I, (cuuint64_t)T};
  const cuuint64_t strI[4] = {n * 8, dk * n * 8, 2 * dk * n * 8, I * 2 * dk * n * 8};
  const cuuint32_t boxI[5] = {32, 1, 2, (cuuint32_t)S::kBc, (cuuint32_t)T};
  const cuuint64_t dimW[4] = {n, dk, I, G};
  const cuuint64_t strW[3] = {n * 8, dk * n * 8, I * dk * n * 8};
  const cuuint32_t boxW[4] = {32, 1, (cuuint32_t)S::kBc, (cuuint32_t)S::GB};
  const cuuint32_t ones[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(mi, CU_TENSOR_MAP_DATA_TYPE_UINT64, 5, const_cast<uint64_t*>(in), dimI, strI, boxI, ones,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  r = enc(mw, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<uint64_t*>(w), dimW, strW, boxW, ones,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int T, int TH>
static cudaError_t mac_stream_launch(const DevParams& P, const uint64_t* in, uint64_t inputs, const uint64_t* w,
                                     uint64_t groups, uint64_t* out, cudaStream_t st) {
  using S = MacShape<T, TH>;
  const uint64_t gblocks = (groups + S::GB - 1) / S::GB;
  const uint64_t units = (uint64_t)P.dk * (P.n >> 5) * gblocks;
  if (units > 0xffffffffull) return cudaErrorInvalidValue;
  CUtensorMap mi, mw;
  cudaError_t e = encode_stream_maps<T, TH>(P, in, inputs, w, groups, &mi, &mw);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const uint64_t avail = sms > P.reserved_sms ? (uint64_t)(sms - P.reserved_sms) : 1;
  const unsigned grid = (unsigned)(units < avail ? units : avail);
  k_mac_stream<T, TH><<<grid, S::kThreads, mac_stream_smem_bytes<T, TH>(), st>>>(
      mi, mw, out, (uint32_t)inputs, (uint32_t)groups, (uint32_t)gblocks, (uint32_t)units, P.dk, P.logn, P.mod,
      P.err);
  return cudaGetLastError();
}

template <int KPAD>
static cudaError_t mac_tc_launch(const DevParams& P, const uint64_t* in, uint64_t inputs, const uint64_t* w,
                                 uint64_t groups, uint64_t* out, cudaStream_t st) {
  const uint64_t gchunks = (groups + tc::kGroups - 1) / tc::kGroups;
  const uint64_t units = (uint64_t)P.dk * (P.n / tc::kSlots) * gchunks;
  if (units > 0xffffffffull / tc::kRoundsPerUnit) return cudaErrorInvalidValue;
  CUtensorMap a, b;
  cudaError_t e = encode_mac_maps<KPAD>(P, in, inputs, w, groups, &a, &b);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const uint64_t avail = sms > P.reserved_sms ? (uint64_t)(sms - P.reserved_sms) : 1;
  const unsigned grid = (unsigned)(units < avail ? units : avail);
  k_mac_tc<KPAD><<<grid, kMacTcThreads, tc::Smem<KPAD>::kLaunchBytes, st>>>(
      a, b, out, (uint32_t)groups, (uint32_t)gchunks, (uint32_t)units, P.dk, P.logn, P.mod, P.err);
  return cudaGetLastError();
}

bool mac_tc_applies(const DevParams& P, uint64_t tiles_in_launch, uint64_t inputs) {
  return P.product_path == 0 && tiles_in_launch == tc::kTiles && inputs >= 1 && inputs <= tc::kMaxK &&
         P.n >= (uint32_t)tc::kSlots && P.err != nullptr;
}

cudaError_t launch_mac_tiles(const DevParams& P, const uint64_t* in, uint64_t tiles, uint64_t inputs,
                             const uint64_t* w, uint64_t groups, uint64_t* acc, cudaStream_t st) {
  const LaunchRange range("bfvgpu:mac_tiles");
  if (!tiles || !groups) return cudaSuccess;
  if (P.n < 32 || inputs > 0xffffffffull || groups > 0xffffffffull) return cudaErrorInvalidValue;
  const uint64_t in_tile = inputs * 2 * P.dk * (uint64_t)P.n, acc_tile = groups * 2 * P.dk * (uint64_t)P.n;
  uint64_t t0 = 0;
  while (t0 < tiles) {
    const uint64_t left = tiles - t0;
    const int T = left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
    const uint64_t* ip = in + t0 * in_tile;
    uint64_t* ap = acc + t0 * acc_tile;
    cudaError_t e;
    if (mac_tc_applies(P, T, inputs)) {
      e = inputs <= 32 ? mac_tc_launch<32>(P, ip, inputs, w, groups, ap, st)
                       : mac_tc_launch<64>(P, ip, inputs, w, groups, ap, st);
      if (e != cudaSuccess) return e;
      t0 += T;
      continue;
    }
    if (P.product_path == 2 || !P.err || inputs > 0x7fffffffull) {  // cp.async-staged form
      switch (T) {
        case 8: e = mac_split_launch<8, 4>(P, ip, inputs, w, groups, ap, st); break;
        case 4: e = mac_split_launch<4, 4>(P, ip, inputs, w, groups, ap, st); break;
        case 2: e = mac_split_launch<2, 2>(P, ip, inputs, w, groups, ap, st); break;
        default: e = mac_split_launch<1, 1>(P, ip, inputs, w, groups, ap, st); break;
      }
    } else {
      switch (T) {
        case 8: e = mac_stream_launch<8, 4>(P, ip, inputs, w, groups, ap, st); break;
        case 4: e = mac_stream_launch<4, 4>(P, ip, inputs, w, groups, ap, st); break;
        case 2: e = mac_stream_launch<2, 2>(P, ip, inputs, w, groups, ap, st); break;
        default: e = mac_stream_launch<1, 1>(P, ip, inputs, w, groups, ap, st); break;
      }
    }
    if (e != cudaSuccess) return e;
    t0 += T;
  }
  return cudaSuccess;
}

uint64_t mac_tiles_launches(uint64_t tiles) {
  uint64_t c = 0;
  while (tiles) {
    tiles -= tiles >= 8 ? 8 : tiles >= 4 ? 4 : tiles >= 2 ? 2 : 1;
    ++c;
  }
  return c;
}

cudaError_t launch_ntt_split(const DevParams& P, const uint64_t* data, uint64_t* out, uint64_t polys,
                             cudaStream_t st) {
  const LaunchRange range("bfvgpu:ntt_split");
  if (!polys) return cudaSuccess;
  if (polys > 0x7fffffffull) return cudaErrorInvalidValue;
  if (use_pair(P)) return launch_pair(k_ntt_split_pair, polys, st, data, out, P.dk, P.mod, P.fwd);
  BFV_DISPATCH(P.logn, {
    k_ntt_split<L_><<<(unsigned)polys, threads_for<L_>(), smem_bytes<L_>(), st>>>(data, out, P.dk, P.mod, P.fwd);
  });
  return cudaGetLastError();
}

cudaError_t launch_pk_prep(const DevParams& P, const uint64_t* pk, ulonglong2* prep, cudaStream_t st) {
  const LaunchRange range("bfvgpu:pk_prep");
  const uint64_t items = 2ull * P.k * P.n;
  k_pk_prep<<<elementwise_blocks(items), 256, 0, st>>>(pk, prep, items, P.k, P.logn, P.mod);
  return cudaGetLastError();
}

cudaError_t launch_enc0_prep(const DevParams& P, const uint64_t* samples, const ulonglong2* pk, uint64_t items,
                             uint64_t* U, uint64_t* xs, cudaStream_t st) {
  const LaunchRange range("bfvgpu:enc0_prep");
  if (!items) return cudaSuccess;
  if (items * P.k > 0x7fffffffull) return cudaErrorInvalidValue;
  if (use_pair(P)) {
    const cudaError_t e = launch_pair(k_enc0_prep_pair, items * P.k, st, samples, U, P.k, P.mod, P.fwd);
    if (e != cudaSuccess) return e;
    return launch_pair(k_enc0_xs_pair, items * 2, st, samples, pk, U, xs, P.k, P.mod, P.inv);
  }
  BFV_DISPATCH(P.logn, {
    k_enc0_prep<L_><<<(unsigned)(items * P.k), threads_for<L_>(), smem_bytes<L_>(), st>>>(samples, U, P.k, P.mod,
                                                                                         P.fwd);
  });
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  BFV_DISPATCH(P.logn, {
    k_enc0_xs<L_><<<(unsigned)(items * 2), threads_for<L_>(), smem_bytes<L_>(), st>>>(samples, pk, U, xs, P.k,
                                                                                    P.mod, P.inv);
  });
  return cudaGetLastError();
}

cudaError_t launch_enc0_fin(const DevParams& P, const uint64_t* samples, const uint64_t* xs, const uint64_t* mask,
                            uint64_t items, uint64_t* E, cudaStream_t st) {
  const LaunchRange range("bfvgpu:enc0_fin");
  if (!items || (!samples && !mask)) return cudaSuccess;
  const uint64_t rows = items * 2 * P.dk;
  // about 16 blocks per SM in all; each walks rows (grid-stride along y)
  const unsigned gx = (P.n + 256 * kFinPer - 1) / (256 * kFinPer);
  const uint64_t want = (148ull * 16 + gx - 1) / gx;
  const dim3 grid(gx, (unsigned)(rows < want ? rows : want));
  k_enc0_fin<<<grid, 256, 0, st>>>(samples, xs, mask, E, rows, P.k, P.dk, P.logn, P.mod, P.q_mod_t, P.upper_half,
                                   P.t, P.tlog);
  return cudaGetLastError();
}

cudaError_t launch_intt_protect(const DevParams& P, const uint64_t* acc, uint64_t items, const uint64_t* U,
                                const ulonglong2* pk, const uint64_t* E, uint64_t* out, cudaStream_t st) {
  const LaunchRange range("bfvgpu:intt_protect");
  if (!items) return cudaSuccess;
  if (items * 2 * P.dk > 0x7fffffffull) return cudaErrorInvalidValue;
  if (use_pair(P))
    return launch_pair(k_intt_protect_pair, items * 2 * P.dk, st, acc, out, U, pk, E, P.k, P.dk, P.mod, P.inv);
  BFV_DISPATCH(P.logn, {
    k_intt_protect<L_><<<(unsigned)(items * 2 * P.dk), threads_for<L_>(), smem_bytes<L_>(), st>>>(
        acc, out, U, pk, E, P.k, P.dk, P.mod, P.inv);
  });
  return cudaGetLastError();
}

}  // namespace bfvgpu
