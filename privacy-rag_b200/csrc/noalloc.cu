// Keyswitch entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the point where they need a keyswitch: a
// protocol worker that fixes (and audits) its device footprint when the session starts
// and must not grow it afterwards, or code running where cudaMalloc's implicit device
// synchronisation would stall other streams.  bfvgpu_keyswitch_device needs the caller
// to allocate a scratch buffer of 2*k*n words per ciphertext; this variant uses a
// fixed scratch array that lives in the library's device image instead.
//
// The array is a file-scope __device__ object of kNoAllocScratchBytes (8 MiB).  Every
// GPU on which the library's module is loaded holds it until the process exits.  Its
// device address is looked up once per device, with that device current, on the first
// call made for a context on that device; that first call should therefore happen
// before any CUDA stream capture.  All calls share the one array: calls that overlap on
// the GPU (different streams, or threads calling concurrently) race on it.  Nothing in
// it needs to start at zero -- every word the kernels read in a call is first written in
// the same call -- and it keeps the last call's contents afterwards.
//
// The cached address belongs to the CUDA primary context that was current when it was
// looked up.  A process that resets the device (cudaDeviceReset) or otherwise destroys
// that primary context must not call this entry point again on that device: the cache
// is not invalidated, and the kernels would run with a stale address.
#include <cuda_runtime.h>

#include <cstdint>
#include <exception>
#include <mutex>
#include <new>
#include <string>

#include "bfvgpu.h"
#include "ctx_internal.h"
#include "kernels.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr size_t kNoAllocScratchWords = kNoAllocScratchBytes / sizeof(uint64_t);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint64_t g_noalloc_scratch[kNoAllocScratchWords];

std::mutex g_setup_mutex;
uint64_t* g_scratch_address[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
cudaError_t scratch_address(int device, uint64_t** out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_address[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_address[device] = static_cast<uint64_t*>(p);
  }
  *out = g_scratch_address[device];
  return cudaSuccess;
}

int32_t fail(int32_t code, const std::string& what) {
  bfvgpu::internal_set_error(what);
  return code;
}

}  // namespace

namespace {

int32_t keyswitch_noalloc(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count, const uint64_t* key,
                          uint32_t galois_elt, uint64_t* out, void* stream) {
  int device = -1;
  cudaStream_t ctx_stream = nullptr;
  const bfvgpu::DevParams* P = bfvgpu::internal_params(ctx, &device, &ctx_stream);
  if (!P || !cts || !key || !out) return fail(BFVGPU_E_ARGUMENT, "E_BFVGPU_ARGUMENT");
  if (device < 0) return fail(BFVGPU_E_DEVICE, "E_BFVGPU_HOST_ONLY_CONTEXT");
  if (device >= kMaxDevices) return fail(BFVGPU_E_DEVICE, "E_BFVGPU_NOALLOC_DEVICE_ORDINAL");
  if (P->k != P->dk + 1) return fail(BFVGPU_E_CONTEXT, "E_BFVGPU_NO_SPECIAL_PRIME");
  if (!(galois_elt & 1) || galois_elt >= 2 * P->n) return fail(BFVGPU_E_ELEMENT, "E_BFVGPU_GALOIS_ELEMENT");
  if (count == 0) return BFVGPU_OK;  // an empty batch is a no-op, as in bfvgpu_keyswitch_device
  const uint64_t max_count = kNoAllocScratchWords / (2ull * P->k * P->n);
  if (count > max_count)
    return fail(BFVGPU_E_SHAPE, "E_BFVGPU_NOALLOC_SCRATCH_LIMIT: " + std::to_string(count) +
                                    " ciphertexts need " + std::to_string(count * 2ull * P->k * P->n * 8) +
                                    " scratch bytes; the fixed array holds " + std::to_string(kNoAllocScratchBytes) +
                                    " (at most " + std::to_string(max_count) + " ciphertexts per call)");
  int previous = -1;
  if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
  if (previous != device && cudaSetDevice(device) != cudaSuccess)
    return fail(BFVGPU_E_CUDA, "E_BFVGPU_CUDA: cudaSetDevice");
  uint64_t* scratch = nullptr;
  cudaError_t e = scratch_address(device, &scratch);
  if (e == cudaSuccess)
    e = bfvgpu::launch_keyswitch(*P, cts, key, galois_elt, count, scratch, out,
                                 stream ? static_cast<cudaStream_t>(stream) : ctx_stream);
  if (previous >= 0 && previous != device) cudaSetDevice(previous);
  if (e != cudaSuccess) return fail(BFVGPU_E_CUDA, std::string("E_BFVGPU_CUDA: noalloc keyswitch: ") + cudaGetErrorString(e));
  bfvgpu::internal_count_launch(2);
  return BFVGPU_OK;
}

}  // namespace

// No C++ exception crosses the ABI: host allocation failures while building an error
// message map to BFVGPU_E_ALLOC, like every other entry point of the library.
extern "C" int32_t bfvgpu_keyswitch_device_noalloc(bfvgpu_ctx* ctx, const uint64_t* cts, uint64_t count,
                                                   const uint64_t* key, uint32_t galois_elt, uint64_t* out,
                                                   void* stream) {
  try {
    return keyswitch_noalloc(ctx, cts, count, key, galois_elt, out, stream);
  } catch (const std::bad_alloc&) {
    return BFVGPU_E_ALLOC;
  } catch (const std::exception&) {
    return BFVGPU_E_ARGUMENT;
  }
}
