// Device-buffer layouts shared by the kernel bodies (block_ops.cuh), their launchers and the
// C ABI (kernels.cu, bfvgpu.cu) and the host emulation of the kernel bodies.
#pragma once
#include "arith.cuh"

namespace bfvgpu {

// Prepared keyswitch key of one Galois element (op_ks_negntt + ks_keyperm_item): Kt
// [dk][2][k][n] as {key word, its Shoup companion floor(word 2^64 / q_p)} pairs, then Ct
// [2][k][n] -- ks_prepared_words words in all, Ct at word ks_ct_offset.
BFV_HD uint64_t ks_ct_offset(uint32_t k, uint32_t dk, uint64_t n) { return 4ull * dk * k * n; }
BFV_HD uint64_t ks_prepared_words(uint32_t k, uint32_t dk, uint64_t n) { return (4ull * dk + 2) * k * n; }

}  // namespace bfvgpu
