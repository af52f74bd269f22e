// Integer-pipe peak of the 64-bit modular operations the BFV kernels are built from.
//
// Every transform-bearing kernel of this library is bound by the SM's integer issue rate,
// not by HBM: a 60-bit residue product is assembled from 32-bit multiply-adds.  The roofline
// that bounds those kernels is therefore the rate at which THIS GPU runs these operations
// when nothing else limits it.  Each kernel below runs one operation from registers only
// (no memory traffic inside the loop), kChains independent dependency chains per thread and
// a full SM of threads, so issue -- not latency -- bounds it:
//   kind 0  NTT butterfly: Harvey's lazy Cooley-Tukey butterfly with a Shoup twiddle
//           (the unit of every forward and inverse pass, ntt_core.cuh)
//   kind 1  multiply-accumulate: 64 x 64 -> 128-bit product added to a 128-bit sum
//           (Acc128::mac, the key inner product and ct-pt products)
//   kind 2  modular product: 128-bit product + Barrett reduction (mul_mod)
//   kind 3  Shoup product by a fixed operand with its precomputed companion, made canonical
//           (twiddle-free products of the kernels: key products, n^-1 scaling,
//           divide-and-round by the special prime)
//   kind 4  NTT butterfly on the FP64 pipe (f64mod.cuh, primes < 2^50): two Cooley-Tukey
//           butterflies per step with one centred reduction, the mix of a radix-8 pass
//           (a product, an add and a subtract per butterfly, one reduction per two)
//   kind 5  product by a fixed operand on the FP64 pipe (mulmod_f64)
// The bench times each with CUDA events and reports, per hot kernel, the time these peaks
// would need for the kernel's algorithmic operation counts divided by its measured time.
// Operands feed back into the chain every step, so no product is loop-invariant; every
// chain's final value goes to `sink` so none is dead.  No counterpart in the reference.
#include <cuda_runtime.h>

#include <cstdint>
#include <exception>
#include <new>
#include <string>

#include "bfvgpu.h"
#include "ctx_internal.h"
#include "f64mod.cuh"
#include "kernels.cuh"
#include "ntt_core.cuh"

namespace bfvgpu {
namespace {

constexpr int kPeakThreads = 256;
constexpr int kChains = 8;

// Deterministic per-chain start values below q (any values work; these are reproducible so
// the host can check the sink).
BFV_HD uint64_t start_value(uint64_t thread, int chain, int which, uint64_t q) {
  uint64_t z = thread * 0x9E3779B97F4A7C15ull + (uint64_t)(chain * 2 + which) * 0xD1B54A32D192ED03ull + 1;
  z ^= z >> 31;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 29;
  return z % q;
}

template <int KIND>
__global__ void __launch_bounds__(kPeakThreads) k_int_peak(const Modulus* mods, const ulonglong2* tw, uint32_t iters,
                                                           uint64_t* sink) {
  const Modulus m = mods[0];
  const uint64_t q = m.q, two_q = 2 * q;
  const ulonglong2 w[4] = {tw[1], tw[2], tw[3], tw[4]};
  const uint64_t thread = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t a[kChains], b[kChains];
#pragma unroll
  for (int j = 0; j < kChains; ++j) {
    a[j] = start_value(thread, j, 0, q);
    b[j] = start_value(thread, j, 1, q);
  }
  if constexpr (KIND == 0) {
#pragma unroll 2
    for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < kChains; ++j) {
        uint64_t x = a[j];
        if (x >= two_q) x -= two_q;
        const uint64_t t = shoup_lazy(b[j], w[j & 3].x, w[j & 3].y, q);
        a[j] = x + t;
        b[j] = x + two_q - t;
      }
    }
  } else if constexpr (KIND == 1) {
    Acc128 acc[kChains];
#pragma unroll 2
    for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < kChains; ++j) {
        acc[j].mac(a[j], b[j]);
        a[j] = acc[j].lo;
      }
    }
#pragma unroll
    for (int j = 0; j < kChains; ++j) b[j] = acc[j].hi;
  } else if constexpr (KIND == 2) {
#pragma unroll 2
    for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < kChains; ++j) a[j] = mul_mod(a[j], b[j], m);
    }
  } else if constexpr (KIND == 3) {
#pragma unroll 2
    for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
      for (int j = 0; j < kChains; ++j) a[j] = shoup(a[j], w[j & 3].x, w[j & 3].y, q);
    }
  } else {
    const double qd = (double)q, qinv = __ddiv_rn(1.0, qd);
    double wc[4], wq[4], fa[kChains], fb[kChains];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      wc[k] = centred_f64(w[k].x, q);
      wq[k] = __ddiv_rn(wc[k], qd);
    }
#pragma unroll
    for (int j = 0; j < kChains; ++j) {
      fa[j] = u64_to_f64(a[j]);
      fb[j] = u64_to_f64(b[j]);
    }
    if constexpr (KIND == 4) {
      // |a| <= q/2 after the reduction, then |a|, |b| <= 1.25 q and 2 q: inside mulmod's range
#pragma unroll 2
      for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < kChains; ++j) {
          const double x = reduce_f64(fa[j], qd, qinv);
          const double t = mulmod_f64(fb[j], wc[j & 3], wq[j & 3], qd);
          const double x1 = f64_add(x, t), y1 = f64_sub(x, t);
          const double t2 = mulmod_f64(y1, wc[j & 3], wq[j & 3], qd);
          fa[j] = f64_add(x1, t2);
          fb[j] = f64_sub(x1, t2);
        }
      }
    } else {
#pragma unroll 2
      for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < kChains; ++j) fa[j] = mulmod_f64(fa[j], wc[j & 3], wq[j & 3], qd);
      }
    }
#pragma unroll
    for (int j = 0; j < kChains; ++j) {
      a[j] = canon_f64(fa[j], qd, qinv);
      b[j] = canon_f64(fb[j], qd, qinv);
    }
  }
  uint64_t h = 0;
#pragma unroll
  for (int j = 0; j < kChains; ++j) h ^= a[j] * 0x9E3779B97F4A7C15ull + b[j];
  sink[thread] = h;
}

int32_t fail(int32_t code, const std::string& what) {
  internal_set_error(what);
  return code;
}

int32_t int_peak(bfvgpu_ctx* ctx, int32_t kind, uint32_t blocks, uint32_t iters, uint64_t* sink, uint64_t* ops,
                 void* stream) {
  int device = -1;
  cudaStream_t ctx_stream = nullptr;
  const DevParams* P = internal_params(ctx, &device, &ctx_stream);
  if (!P || !sink || !ops || blocks == 0) return fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
  if (kind < 0 || kind > 5) return fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_PEAK_KIND");
  if (device < 0) return fail(BFVGPU_E_DEVICE, "E_BFVGPU_HOST_ONLY_CONTEXT");
  if (P->n < 8) return fail(BFVGPU_E_CONTEXT, "E_BFVGPU_PEAK_DEGREE");
  if (kind >= 4 && internal_first_prime(ctx) >= kF64MaxPrime) return fail(BFVGPU_E_CONTEXT, "E_BFVGPU_PEAK_PRIME");
  *ops = (uint64_t)blocks * kPeakThreads * kChains * iters * (kind == 4 ? 2 : 1);
  int previous = -1;
  if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
  if (previous != device && cudaSetDevice(device) != cudaSuccess)
    return fail(BFVGPU_E_CUDA, "E_BFVGPU_CUDA: cudaSetDevice");
  const cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx_stream;
  if (kind == 0)
    k_int_peak<0><<<blocks, kPeakThreads, 0, st>>>(P->mod, P->fwd, iters, sink);
  else if (kind == 1)
    k_int_peak<1><<<blocks, kPeakThreads, 0, st>>>(P->mod, P->fwd, iters, sink);
  else if (kind == 2)
    k_int_peak<2><<<blocks, kPeakThreads, 0, st>>>(P->mod, P->fwd, iters, sink);
  else if (kind == 3)
    k_int_peak<3><<<blocks, kPeakThreads, 0, st>>>(P->mod, P->fwd, iters, sink);
  else if (kind == 4)
    k_int_peak<4><<<blocks, kPeakThreads, 0, st>>>(P->mod, P->fwd, iters, sink);
  else
    k_int_peak<5><<<blocks, kPeakThreads, 0, st>>>(P->mod, P->fwd, iters, sink);
  const cudaError_t e = cudaGetLastError();
  if (previous >= 0 && previous != device) cudaSetDevice(previous);
  if (e != cudaSuccess) return fail(BFVGPU_E_CUDA, std::string("E_BFVGPU_CUDA: int peak: ") + cudaGetErrorString(e));
  internal_count_launch(1);
  return BFVGPU_OK;
}

}  // namespace
}  // namespace bfvgpu

extern "C" int32_t bfvgpu_int_peak_device(bfvgpu_ctx* ctx, int32_t kind, uint32_t blocks, uint32_t iters,
                                          uint64_t* sink, uint64_t* ops, void* stream) {
  try {
    return bfvgpu::int_peak(ctx, kind, blocks, iters, sink, ops, stream);
  } catch (const std::bad_alloc&) {
    return BFVGPU_E_ALLOC;
  } catch (const std::exception&) {
    return BFVGPU_E_ARGUMENT;
  }
}
