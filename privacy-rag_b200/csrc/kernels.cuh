// Internal launch API of the BFV kernels (device pointers, one CUDA stream).
// The C ABI in bfvgpu.cu builds the reference-shaped objects on top of these.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "arith.cuh"
#include "layout.cuh"

namespace bfvgpu {

// Device view of a parameter context.
struct DevParams {
  int logn = 0;
  uint32_t n = 0;
  uint32_t k = 0;   // primes held (data + special)
  uint32_t dk = 0;  // data primes
  uint64_t t = 0;
  int tlog = 0;     // log2 t when t is a power of two, else 0
  uint64_t q_mod_t = 0, upper_half = 0;
  const Modulus* mod = nullptr;       // [k]
  const ulonglong2* fwd = nullptr;    // [k][n]
  const ulonglong2* inv = nullptr;    // [k][n]
  const double2* fwd64 = nullptr;     // [k][n] FP64 twiddles {w_c, fl(w_c / q)} of fwd / inv, used by
  const double2* inv64 = nullptr;     // the primes whose record has f64 set (f64mod.cuh)
  const uint64_t* qjp = nullptr;      // [dk][k]: q_j mod q_p
  const uint64_t* crt_part = nullptr; // [dk][dk] limbs of Q/q_j
  const uint64_t* crt_inv = nullptr;  // [dk][2] Shoup pair of (Q/q_j)^-1 mod q_j
  const uint64_t* crt_q = nullptr;    // [dk] limbs of Q
  uint32_t* err = nullptr;            // kernel-recorded error bits (bfvgpu_ctx_check)
  int product_path = 0;               // 0: tcgen05 where it applies, 1: CUDA cores only (TMA-staged),
                                      // 2: CUDA cores with per-thread asynchronous-copy staging
  int reserved_sms = 0;               // SMs the persistent product kernels leave free
  int split_limbs = 1;                // n = 16384 single-transform kernels: 1 = each limb split
                                      // between the two blocks of a cluster, 0 = one block per limb
};

// Smallest and largest supported log2(n).
constexpr int kMinLogN = 5;
constexpr int kMaxLogN = 14;
bool logn_supported(int logn);

// Opt the kernels into large dynamic shared memory on the current device.
cudaError_t configure_kernels(int logn);

// In-place batched transform of [polys][n]; poly i uses prime offset + i % count.
cudaError_t launch_ntt(const DevParams& P, uint64_t* data, uint64_t polys, uint32_t prime_count,
                       uint32_t prime_offset, bool inverse, cudaStream_t st);

// Centred lift of ring-59 words [blocks][n] into each data prime and forward NTT:
// out [blocks][dk][n].
cudaError_t launch_lift_ntt(const DevParams& P, const uint64_t* ring, uint64_t* out, uint64_t blocks,
                            cudaStream_t st);

// Optional epilogue of the ct-pt product: plaintext mask (c0 -= Delta-scaled mask)
// and Enc(0) re-randomisation from pre-moddown key-level polys x [2][k][n].
struct Protect {
  const uint64_t* mask = nullptr;      // [groups][n] ring-59 words, or null
  const uint64_t* enc0_x = nullptr;    // [groups][2][k][n], or null
};

// out[g][c][p] = INTT( sum_b in[b][c][p] . w[g][b][p] )  (+ protect epilogue)
// in [inputs][2][dk][n] NTT form; w [groups][inputs][dk][n] NTT form.
cudaError_t launch_mac_intt(const DevParams& P, const uint64_t* in, const uint64_t* w, uint64_t* out,
                            uint64_t inputs, uint64_t groups, const Protect& prot, cudaStream_t st);

// selected[g][p][i] = c0[g][p][targets[g*max + i]] for i < counts[g]; if crt != null,
// crt[g][i][dk] = the CRT of the dk residues as dk 64-bit limbs (little endian).
cudaError_t launch_gather_targets(const DevParams& P, const uint64_t* out /*[groups][2][dk][n]*/,
                                  const uint64_t* targets, const uint32_t* counts, uint32_t max_count,
                                  uint64_t groups, uint64_t* selected, uint64_t* crt, cudaStream_t st);

// Galois automorphism g then keyswitch of `count` ciphertexts [count][2][dk][n] with
// key [dk][2][k][n] (NTT form).  acc is scratch [count][2][k][n]; out [count][2][dk][n].
cudaError_t launch_keyswitch(const DevParams& P, const uint64_t* cts, const uint64_t* key, uint32_t elt,
                             uint64_t count, uint64_t* acc, uint64_t* out, cudaStream_t st);

// Hoisted multi-rotation keyswitch (see op_ks_hoist / op_ks_rotate):
//  hoist:   Y [count][dk][k][n] = NTT(c1_j mod q_p); zflag [count] = c1 has a zero word
//  keyprep: prepared [count][(dk*2 + 2)*k][n] = permuted keys and corrections for count
//           keys [count][dk][2][k][n] and Galois elements elts (host array)
//  rotate:  out [count][2][dk][n] = Galois(elt) + keyswitch of every ciphertext, x is
//           scratch [count][2][k][n]
cudaError_t launch_ks_hoist(const DevParams& P, const uint64_t* cts, uint64_t count, uint64_t* Y, uint32_t* zflag,
                            cudaStream_t st);
cudaError_t launch_ks_keyprep(const DevParams& P, const uint64_t* keys, const uint32_t* elts, uint64_t count,
                              uint64_t* prepared, cudaStream_t st);
cudaError_t launch_ks_rotate(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                             const uint32_t* zflag, const uint64_t* prepared, uint32_t elt, uint64_t* x, uint64_t* out,
                             cudaStream_t st);
// Hoisted rotations of many elements in one launch pair (chunks of 256 elements):
// paired != 0 rotates ciphertext i by element i (elements == count; x [count][2][k][n],
// out [count][2][dk][n]); else every element rotates every ciphertext (x
// [elements][count][2][k][n], out [elements][count][2][dk][n]).  prepared [elements][..].
cudaError_t launch_ks_rotate_multi(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                                   const uint32_t* zflag, const uint64_t* prepared, const uint32_t* elts,
                                   uint64_t elements, int paired, uint64_t* x, uint64_t* out, cudaStream_t st);
// The hoisted rotations of `elements` elements (elts host array, prepared [elements][..]),
// software-pipelined: elements + 1 launches, launch r holding the special-prime blocks of
// element r and the data-prime blocks of element r - 1, which finish the keyswitch in shared
// memory and store element r - 1's result into outs[r - 1] (host array of device pointers
// [count][2][dk][n]; entries may repeat).  x: scratch [count][2][k][n]; xs: scratch
// [2][count][2][n].  launch_ks_rotate_pipe_step issues launch r (0 <= r <= elements) alone,
// element r - 1's result going to out_d: a caller that reads each result back as soon as it
// is complete records an event after launch r.
cudaError_t launch_ks_rotate_pipe(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                                  const uint32_t* zflag, const uint64_t* prepared, const uint32_t* elts,
                                  uint64_t elements, uint64_t* x, uint64_t* xs, uint64_t* const* outs, cudaStream_t st);
cudaError_t launch_ks_rotate_pipe_step(const DevParams& P, const uint64_t* cts, uint64_t count, const uint64_t* Y,
                                       const uint32_t* zflag, const uint64_t* prepared, const uint32_t* elts,
                                       uint64_t elements, uint64_t r, uint64_t* x, uint64_t* xs, uint64_t* out_d,
                                       cudaStream_t st);
// acc [2][dk][n] = sum of the groups ciphertexts in [groups][2][dk][n].
cudaError_t launch_sum_cts(const DevParams& P, const uint64_t* in, uint64_t groups, uint64_t* acc, cudaStream_t st);

// Enc(0) pre-moddown polys: x [groups][2][k][n] = INTT(NTT(u) . pk_c) + e_c with
// samples [groups][3][k][n]; scratch u_ntt [groups][k][n].
cudaError_t launch_enc0_x(const DevParams& P, const uint64_t* samples, const uint64_t* pk, uint64_t* u_ntt,
                          uint64_t* x, uint64_t groups, cudaStream_t st);

// Divide-and-round by the special prime: x [groups][2][k][n] -> out [groups][2][dk][n].
cudaError_t launch_moddown(const DevParams& P, const uint64_t* x, uint64_t* out, uint64_t groups,
                           cudaStream_t st);

// c1 . s for each data prime: data [batches][dk][n] in place, sk [dk][n] NTT form.
cudaError_t launch_client_phase(const DevParams& P, uint64_t* data, const uint64_t* sk, uint64_t batches,
                                cudaStream_t st);

// Checks canonical residues of [polys][n] (prime offset + i % count); sets *bad to 1
// if any word is >= its prime.
cudaError_t launch_check_canonical(const DevParams& P, const uint64_t* data, uint64_t polys,
                                   uint32_t prime_count, uint32_t prime_offset, uint32_t* bad,
                                   cudaStream_t st);

// Resident token product (TokenWeights::evaluate_device): inputs [19][slots][2][dk][n]
// NTT form, ring [19][8192] weights, scaled [slots][dk]; weight scratch [19][dk][n];
// out [slots][2][dk][n] after add_shift.
cudaError_t launch_token_evaluate(const DevParams& P, const uint64_t* inputs, uint64_t slots,
                                  const uint64_t* ring, const uint64_t* scaled, uint64_t* wscratch,
                                  uint64_t* acc, uint64_t* out, cudaStream_t st);
// TokenWeights::evaluate_device for `coords` coordinates at once: ring [coords][19][8192] ring
// words, local [coords][slots] local shares (Delta-scaled here into scaled [coords][slots][dk]),
// wscratch [coords][19][dk][n], out [coords][slots][2][dk][n]; n = 16384 only.
cudaError_t launch_token_evaluate_many(const DevParams& P, const uint64_t* inputs, uint64_t slots, const uint64_t* ring,
                                       uint64_t coords, const uint64_t* local, uint64_t* scaled, uint64_t* wscratch,
                                       uint64_t* out, cudaStream_t st);
// One packing-tree level: in [2 pairs][slots] ciphertexts -> sum, diff [pairs][slots]
// (left + X^(n >> (level+1)) right, left - ...).
cudaError_t launch_packing_prepare_many(const DevParams& P, const uint64_t* in, uint64_t pairs, uint64_t slots,
                                        uint64_t* sum, uint64_t* diff, unsigned level, cudaStream_t st);

// Acyclic packing merge prologue (Switch::packing_prepare without its permutation, which
// the keyswitch of the difference applies): sum = L + X^s R, diff = L - X^s R for
// [2][dk][n] ciphertexts, s = n >> (level+1).
cudaError_t launch_packing_prepare(const DevParams& P, const uint64_t* left, const uint64_t* right,
                                   uint64_t* sum, uint64_t* diff, unsigned level, cudaStream_t st);
// c0 [dk][n] += Delta * plain[i] (scaling variant) for i < count, plain < t.
cudaError_t launch_add_plain(const DevParams& P, uint64_t* c0, const uint64_t* plain, uint64_t count,
                             cudaStream_t st);
// Output protection of coefficient-form ciphertexts: out [items][2][dk][n] = cts + Enc(0) -
// [c = 0] Delta masks, Enc(0) from samples [items][3][k][n] (nullable: none) and pk [2][k][n]
// (NTT form) through the scratch u_ntt [items][k][n], x [items][2][k][n]; masks [items][n]
// (nullable).  out may be cts.
cudaError_t launch_protect_ct(const DevParams& P, const uint64_t* cts, uint64_t items, const uint64_t* masks,
                              const uint64_t* samples, const uint64_t* pk, uint64_t* u_ntt, uint64_t* x, uint64_t* out,
                              cudaStream_t st);
// targets [slots][512] = the packed token tile's target coefficient of every coordinate,
// counts [slots] = 512 (the gather_targets operands of a tile return).
cudaError_t launch_packed_targets(uint64_t* targets, uint32_t* counts, uint64_t slots, cudaStream_t st);
// a += b on [polys][n] data-prime polys.
cudaError_t launch_add(const DevParams& P, uint64_t* a, const uint64_t* b, uint64_t polys, cudaStream_t st);
// Public-key encryption of cts plaintexts: samples [cts][3][k][n] (u, e0, e1), pk [2][k][n] NTT
// form, plain [cts][n] -> out [cts][2][dk][n] = moddown(Enc(0)) + Delta plain; scratch u_ntt
// [cts][k][n], x [cts][2][k][n].
cudaError_t launch_encrypt_many(const DevParams& P, const uint64_t* samples, const uint64_t* pk, const uint64_t* plain,
                                uint64_t cts, uint64_t* u_ntt, uint64_t* x, uint64_t* out, cudaStream_t st);

// Layer pipeline over T tiles that share one weight matrix (E = T * groups items, item
// e = t * groups + g):
//  ntt_split:    forward NTT of client limbs [polys][n] (prime i % dk) into out (may be the
//                input), stored in the product's operand form (split30 of each canonical slot).
//  mac_tiles:    acc [T][G][2][dk][n] = sum_b in[t][b][c] . w[g][b]; in [T][I][2][dk][n] from
//                ntt_split, w [G][I][dk][n] NTT form, all primes < 2^60, n >= 32.  Tiles
//                run in launches of 8/4/2/1 (mac_tiles_launches counts them).
//  enc0_prep:    U [E][k][n] = NTT(u) (one launch, a block per (item, prime)), then xs
//                [E][2][n] = special-prime coefficients of INTT(U . pk_c) + e_c (a second
//                launch, a block per (item, c)); samples [E][3][k][n]; pk from pk_prep.
//  intt_protect: out [E][2][dk][n] = INTT(acc + U . pk') + E, i.e. INTT(acc) + Enc(0) (if U)
//                - Delta mask (if masked), the Enc(0) data-prime part folded into the input.
cudaError_t launch_mac_tiles(const DevParams& P, const uint64_t* in, uint64_t tiles, uint64_t inputs,
                             const uint64_t* w, uint64_t groups, uint64_t* acc, cudaStream_t st);
uint64_t mac_tiles_launches(uint64_t tiles);
cudaError_t launch_ntt_split(const DevParams& P, const uint64_t* data, uint64_t* out, uint64_t polys,
                             cudaStream_t st);
//  pk_prep:      prep [2][k][n] = {v, Shoup companion}, v = pk . q_s^-1 (data primes), pk (special)
cudaError_t launch_pk_prep(const DevParams& P, const uint64_t* pk, ulonglong2* prep, cudaStream_t st);
cudaError_t launch_enc0_prep(const DevParams& P, const uint64_t* samples, const ulonglong2* pk, uint64_t items,
                             uint64_t* U, uint64_t* xs, cudaStream_t st);
// enc0_fin: E [items][2][dk][n], the additive output term (Enc(0) divide-and-round part and
// the Delta-scaled mask) after enc0_prep; nothing when samples and mask are both null.
cudaError_t launch_enc0_fin(const DevParams& P, const uint64_t* samples, const uint64_t* xs, const uint64_t* mask,
                            uint64_t items, uint64_t* E, cudaStream_t st);
cudaError_t launch_intt_protect(const DevParams& P, const uint64_t* acc, uint64_t items, const uint64_t* U,
                                const ulonglong2* pk, const uint64_t* E, uint64_t* out, cudaStream_t st);

}  // namespace bfvgpu
