// Library-internal hooks shared between translation units of libbfvgpu.so
// (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "bfvgpu.h"
#include "kernels.cuh"

namespace bfvgpu {
// Device parameters, device ordinal and stream of a context (device < 0: host-only).
const DevParams* internal_params(const bfvgpu_ctx* ctx, int* device, cudaStream_t* stream);
// Thread-local message returned by bfvgpu_last_error().
void internal_set_error(const std::string& what);
// Adds to the process-wide launch counter of bfvgpu_launch_count().
void internal_count_launch(uint64_t n);
// The context's first prime (0 for a null context).
uint64_t internal_first_prime(const bfvgpu_ctx* ctx);
}  // namespace bfvgpu
