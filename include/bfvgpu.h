/*
 * bfvgpu.h -- C ABI of the B200 (sm_100a) BFV ciphertext-arithmetic library.
 *
 * Drop-in boundary for privacy-rag's GPU backends (IV1 = implementation_v1/ of the
 * reference).  Each object below replaces one reference C++ backend class; the
 * per-function comments name the member it stands in for.  SEAL types do not cross
 * this boundary: ciphertexts, keys and polynomials are flat little-endian uint64
 * arrays in the reference's own layouts ([2][k][n] ciphertexts, [digit][2][k+1][n]
 * keys, [prime][n] polynomials), exactly what the reference adapters copy out of SEAL
 * objects (e.g. IV1/experiments/matrix_gpu/adapter.cpp:27-31).
 *
 * Conventions
 *  - Every function returns an int status: BFVGPU_OK (0) or a stable error code below.
 *    No C++ exception crosses the ABI.  bfvgpu_last_error() gives a thread-local text.
 *    Validation failures correspond to the reference's std::invalid_argument codes,
 *    CUDA failures to its runtime_error("E_...: "+cudaGetErrorString) after release.
 *  - Host pointers are caller-owned and only read/written during the call.
 *  - close() functions are idempotent and never fail; they zero every sensitive device
 *    buffer, synchronise, free it, and report the bytes in bfvgpu_cleanup, like the
 *    reference's Cleanup{first_cuda_error, wiped, freed, closed}
 *    (IV1/experiments/matrix_gpu/matrix.hpp:8).  release() frees the handle itself
 *    (closing first if needed).
 *  - One thread drives an object at a time (the reference's single session thread).
 *  - There is no CPU fallback: without a compute-capability-10.x device every
 *    constructor fails with BFVGPU_E_DEVICE.
 */
#ifndef BFVGPU_H
#define BFVGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum bfvgpu_status {
  BFVGPU_OK = 0,
  BFVGPU_E_ARGUMENT = 1,     /* null pointer / unsupported parameter value          */
  BFVGPU_E_CONTEXT = 2,      /* E_NTT_CONTEXT, MATRIX_GPU_CONTEXT: wrong parameter set */
  BFVGPU_E_SHAPE = 3,        /* MATRIX_GPU_SHAPE, E_SWITCH_SHAPE, E_NTT_SHAPE         */
  BFVGPU_E_CANONICAL = 4,    /* E_NTT_CANONICAL_REQUIRED: residue >= its prime        */
  BFVGPU_E_RING = 5,         /* MATRIX_GPU_RING: ring word >= 2^59                    */
  BFVGPU_E_TARGET_COUNT = 6, /* MATRIX_GPU_TARGET_COUNT: 0 or > 512 targets           */
  BFVGPU_E_TARGET_INDEX = 7, /* MATRIX_GPU_TARGET_INDEX: >= n or not increasing       */
  BFVGPU_E_CLOSED = 8,       /* E_SWITCH_CLOSED, E_NTT_CLOSED, E_RESIDENT_CLOSED      */
  BFVGPU_E_CUDA = 9,         /* a CUDA call failed; the object has been released      */
  BFVGPU_E_DEVICE = 10,      /* no usable sm_100 device (RTX2060_REQUIRED analogue)   */
  BFVGPU_E_STATE = 11,       /* E_PACK_PAIR_STATE, E_CLIENT_KEY_STATE, E_LOCAL_BINDING */
  BFVGPU_E_BOUND = 12,       /* E_RESIDENT_WEIGHT_BOUND: |w| > 2^20                   */
  BFVGPU_E_ELEMENT = 13,     /* Galois element even or >= 2n                          */
  BFVGPU_E_ALLOC = 14        /* device allocation failed                              */
};

typedef struct bfvgpu_cleanup {
  int32_t first_cuda_error; /* first CUDA error seen while releasing, 0 if none */
  int32_t closed;           /* 1 once every device buffer is gone              */
  uint64_t wiped;           /* sensitive bytes zeroed and synchronised          */
  uint64_t freed;           /* sensitive bytes freed                            */
} bfvgpu_cleanup;

typedef struct bfvgpu_ctx bfvgpu_ctx;
typedef struct bfvgpu_ntt bfvgpu_ntt;
typedef struct bfvgpu_matrix bfvgpu_matrix;
typedef struct bfvgpu_switch bfvgpu_switch;
typedef struct bfvgpu_rotations bfvgpu_rotations;
typedef struct bfvgpu_slots bfvgpu_slots;
typedef struct bfvgpu_enc0 bfvgpu_enc0;
typedef struct bfvgpu_token bfvgpu_token;

/* ---- library ---------------------------------------------------------------------- */
int32_t bfvgpu_version(void);
const char *bfvgpu_error_name(int32_t code);
const char *bfvgpu_last_error(void);
/* Number of kernel launches this process has issued through the library. */
uint64_t bfvgpu_launch_count(void);

/* ---- parameters (IV1/native/src/bfv.cpp:91-137) ------------------------------------- */
/* Prime chain for degree n with the given bit sizes, every prime = 1 mod 2n, found by a
 * downward search from 2^bits; equal sizes are handed out smallest first (the rule that
 * yields the locked ART-002 list).  Replaces seal::CoeffModulus::Create at bfv.cpp:95. */
int32_t bfvgpu_find_primes(uint32_t n, const int32_t *bits, uint32_t count, uint64_t *out);

/* Parameter context on one device: n = 2^logn (logn in {5,6,12,13,14}), data primes
 * primes[0..data_primes), then special_primes (0 or 1) special prime, plaintext
 * modulus t (a power of two or < 2^32).  Computes the NTT tables (minimal primitive
 * 2n-th root, reference table layout), BFV scaling and CRT constants, and uploads them;
 * device == -1 builds a host-only context (tables and constants, no device work).
 * Replaces the SEALContext plus the per-backend table extraction
 * (IV1/experiments/matrix_gpu/adapter.cpp:19-31, client_phase/seal_tables.cpp:22-33). */
int32_t bfvgpu_ctx_create(uint32_t n, const uint64_t *primes, uint32_t data_primes,
                          uint32_t special_primes, uint64_t plain_modulus, int32_t device,
                          bfvgpu_ctx **out);
/* The locked ART-002 profile: n = 16384, six 60-bit data primes + one special prime,
 * t = 2^59 (bfv.cpp:91-105; IV1/artifacts/bfv_context.json). */
int32_t bfvgpu_ctx_create_art002(int32_t device, bfvgpu_ctx **out);
int32_t bfvgpu_ctx_destroy(bfvgpu_ctx *ctx);
/* Host copies of prime `prime`'s tables: fwd/inv [n][2] {w, floor(w 2^64/q)} in the
 * reference layout (fwd[brv(i)] = psi^i, inv[brv(i-1)+1] = psi^-i), invn [2]. */
int32_t bfvgpu_ctx_tables(const bfvgpu_ctx *ctx, uint32_t prime, uint64_t *fwd, uint64_t *inv,
                          uint64_t *invn);
/* The 16 words of prime `prime`'s constant record: q, floor((2^128-1)/q) (low, high),
 * n^-1 and its Shoup quotient, q_special^-1 and quotient, floor(q_special/2) mod q,
 * floor(Q/t) mod q and quotient, then zeros.  Diagnostic; used by the CPU pre-checks. */
int32_t bfvgpu_ctx_moduli(const bfvgpu_ctx *ctx, uint32_t prime, uint64_t *out);
/* The context's CUDA stream (cudaStream_t) and device ordinal. */
int32_t bfvgpu_ctx_stream(const bfvgpu_ctx *ctx, void **stream, int32_t *device);

/* ---- device-resident entry points (batched; all pointers are device memory) ------------
 * stream == NULL uses the context stream.  No validation of residue ranges. */
/* In-place negacyclic NTT (inverse != 0: inverse) of [polys][n]; poly i is reduced by
 * prime prime_offset + i % prime_count.  One call replaces the 14 `stage` launches of
 * NttBatch::transform (IV1/native/gpu/client_phase/ntt.cu:152-157). */
int32_t bfvgpu_ntt_device(bfvgpu_ctx *ctx, uint64_t *data, uint64_t polys, uint32_t prime_count,
                          uint32_t prime_offset, int32_t inverse, void *stream);
/* Galois automorphism + keyswitch of count ciphertexts [count][2][dk][n] with one key
 * [dk][2][k][n]; scratch holds bfvgpu_keyswitch_scratch_words(ctx, count) words;
 * out [count][2][dk][n].  Switch::apply for a whole batch (switch.cu:142-154).  Ciphertext
 * and key words must be canonical residues (below their primes), as SEAL produces them: the
 * device entry points assume it (the host objects, Switch and Rotations, check it). */
uint64_t bfvgpu_keyswitch_scratch_words(const bfvgpu_ctx *ctx, uint64_t count);
int32_t bfvgpu_keyswitch_device(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count,
                                const uint64_t *key, uint32_t galois_elt, uint64_t *scratch,
                                uint64_t *out, void *stream);
/* Hoisted multi-rotation keyswitch: the same outputs as bfvgpu_keyswitch_device for
 * every (key, ciphertext) pair, when many Galois elements are applied to one batch.
 *  1. prepare (once per key, any number of keys per call): keys [count][dk][2][k][n]
 *     (device), galois_elts [count] (host); prepared [count][bfvgpu_keyswitch_prepared_words]
 *     = each key with its NTT slots permuted for its element plus the element's negation
 *     correction;
 *  2. hoist (once per ciphertext batch): hoisted [bfvgpu_keyswitch_hoist_words(count)] =
 *     the NTT of every c1 digit reduced into every key-level prime, and a flag per
 *     ciphertext whose c1 holds a zero word (those take an exact per-element path);
 *  3. rotate (per element): out [count][2][dk][n] from hoisted + prepared; scratch holds
 *     count * 2 * k * n words.  galois_elt must be the element the key was prepared for.
 * Per element this runs 2k inverse NTTs per ciphertext instead of dk*k forward + 2k
 * inverse (switch.cu:146-149 runs both per apply).  Keys and ciphertexts canonical, as for
 * bfvgpu_keyswitch_device; prepared keys are laid out for the context's arithmetic mode
 * (bfvgpu_ctx_set_fp64) at the time of preparation. */
uint64_t bfvgpu_keyswitch_prepared_words(const bfvgpu_ctx *ctx);
uint64_t bfvgpu_keyswitch_hoist_words(const bfvgpu_ctx *ctx, uint64_t count);
int32_t bfvgpu_keyswitch_prepare_device(bfvgpu_ctx *ctx, const uint64_t *keys, const uint32_t *galois_elts,
                                        uint64_t count, uint64_t *prepared, void *stream);
int32_t bfvgpu_keyswitch_hoist_device(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count,
                                      uint64_t *hoisted, void *stream);
int32_t bfvgpu_keyswitch_rotate_device(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count,
                                       const uint64_t *hoisted, const uint64_t *prepared,
                                       uint32_t galois_elt, uint64_t *scratch, uint64_t *out,
                                       void *stream);
/* Step 3 for many elements at once, software-pipelined: the same outputs as one
 * bfvgpu_keyswitch_rotate_device call per element (element e's result into outs[e], a host
 * array of `elements` device pointers [count][2][dk][n]; entries may repeat, later elements
 * overwriting earlier ones), in elements + 1 launches instead of 2 * elements: launch r runs
 * the special-prime product and transform of element r beside the data-prime blocks of
 * element r - 1, which complete the keyswitch (divide-and-round by the special prime, c0,
 * Galois permutation) in shared memory.  galois_elts (host) [elements] the elements the keys
 * in prepared [elements][bfvgpu_keyswitch_prepared_words] were prepared for; scratch of
 * bfvgpu_keyswitch_rotate_many_scratch_words(ctx, count) words. */
uint64_t bfvgpu_keyswitch_rotate_many_scratch_words(const bfvgpu_ctx *ctx, uint64_t count);
int32_t bfvgpu_keyswitch_rotate_many_device(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count,
                                            const uint64_t *hoisted, const uint64_t *prepared,
                                            const uint32_t *galois_elts, uint64_t elements, uint64_t *scratch,
                                            uint64_t *const *outs, void *stream);
/* The same keyswitch as bfvgpu_keyswitch_device, for callers that cannot allocate
 * device memory when they need it (a worker whose device footprint is fixed and
 * audited at session start, or code that must not take cudaMalloc's implicit device
 * synchronisation).  No counterpart in the reference.  It allocates nothing: the
 * scratch is a fixed 8 MiB array in the library's device image, which every GPU that
 * loads the library holds until exit.  Limit: count * 2 * k * n * 8 bytes <= 8 MiB
 * (12 ciphertexts at n = 8192 with 4+1 primes, 4 at ART-002); larger counts fail with
 * BFVGPU_E_SHAPE; count == 0 is a no-op.  The first call for a device looks the array's
 * address up with that device current, so make it before any stream capture; the address
 * stays valid only while that device's primary context lives (no calls after a
 * cudaDeviceReset).  All calls share the array: calls that overlap on the GPU race; it
 * keeps the last call's contents (nothing in it needs to start at zero). */
int32_t bfvgpu_keyswitch_device_noalloc(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count,
                                        const uint64_t *key, uint32_t galois_elt, uint64_t *out,
                                        void *stream);
/* Integer-pipe peak microbenchmark (diagnostic; no counterpart in the reference): runs one
 * of the 64-bit modular operations the kernels are built from, from registers only, with
 * independent chains at full occupancy -- kind 0 = NTT butterfly (Harvey lazy, Shoup
 * twiddle of prime 0), 1 = 64x64 -> 128-bit multiply-accumulate, 2 = modular product
 * (128-bit product + Barrett reduction by prime 0), 3 = Shoup product by a fixed operand
 * with its companion, made canonical; on the FP64 pipe (prime 0 below 2^50, else
 * BFVGPU_E_CONTEXT): 4 = NTT butterfly (two per step, one centred reduction per step),
 * 5 = product by a fixed operand.  blocks x 256 threads; *ops receives the operations
 * performed (blocks * 256 * 8 chains * iters, twice that for kind 4); sink [blocks * 256] (device)
 * one checksum word per thread.  Timed by the caller (CUDA events) to give this GPU's
 * operation rates, the denominators of the integer roofline. */
int32_t bfvgpu_int_peak_device(bfvgpu_ctx *ctx, int32_t kind, uint32_t blocks, uint32_t iters, uint64_t *sink,
                               uint64_t *ops, void *stream);
/* Lift + forward NTT of ring-59 weight blocks [blocks][n] -> [blocks][dk][n]. */
int32_t bfvgpu_weights_ntt_device(bfvgpu_ctx *ctx, const uint64_t *ring, uint64_t blocks,
                                  uint64_t *out, void *stream);
/* out[g][c] = INTT(sum_b in[b][c] . w[g][b]) for g < groups, with the optional mask
 * [groups][n] subtracted (Delta-scaled) from c0 and Enc(0) pre-moddown polys
 * enc0_x [groups][2][k][n] added.  in [inputs][2][dk][n] NTT form, w [groups][inputs][dk][n]. */
int32_t bfvgpu_matrix_groups_device(bfvgpu_ctx *ctx, const uint64_t *in, uint64_t inputs,
                                    const uint64_t *w, uint64_t groups, const uint64_t *mask,
                                    const uint64_t *enc0_x, uint64_t *out, void *stream);

/* Synchronises the context's device and returns (then clears) the error bits its kernels
 * recorded: bit 0 = a tensor-core product step whose completion wait expired (the block
 * freed its tensor memory and stopped; the output of that launch is incomplete).  Returns
 * BFVGPU_E_CUDA when any bit was set.  No counterpart in the reference (its kernels have
 * no waits). */
int32_t bfvgpu_ctx_check(bfvgpu_ctx *ctx, uint32_t *flags);
/* Leaves `sms` streaming multiprocessors out of the persistent product kernels' grids (0 by
 * default), so that a collective running beside them (NCCL broadcasts and gathers of a
 * sharded call) finds free SMs.  Results are unchanged. */
int32_t bfvgpu_ctx_set_reserved_sms(bfvgpu_ctx *ctx, int32_t sms);
/* Selects the ct-pt product of bfvgpu_matrix_tiles_device: 0 (default) = tcgen05 kind::i8
 * for launches of 8 tiles with at most 64 input blocks, CUDA cores with TMA-staged operands
 * otherwise; 1 = the TMA-staged CUDA-core product always; 2 = the CUDA-core product with
 * per-thread asynchronous-copy staging (comparison).  Results are identical. */
int32_t bfvgpu_ctx_set_product_path(bfvgpu_ctx *ctx, int32_t path);
/* At n = 16384, the kernels whose only shared-memory work is one transform (batched NTTs,
 * weight lift + NTT, client-limb transform, Enc(0) preparation, protected output transform)
 * split each limb between the two blocks of a thread-block cluster: split = 1 (default), half
 * a limb per block, three blocks per SM, the cross level through distributed shared memory;
 * split = 0, one block holds the whole limb (one block per SM).  Results are identical. */
int32_t bfvgpu_ctx_set_limb_split(bfvgpu_ctx *ctx, int32_t split);
/* Arithmetic of the primes below 2^50 (configs with 36- to 50-bit primes): on = 1 (default),
 * the transforms and products that have an FP64 form (batched NTTs, the per-apply Galois
 * keyswitch, the hoisted rotations and their key preparation) compute on the FP64 pipe with exact integer-valued
 * doubles; on = 0, everything computes on the integer pipe.  Results are identical.
 * Prepared keys are laid out for the mode they were prepared in, so the mode is fixed once
 * the context has prepared keys: changing it then fails with BFVGPU_E_STATE. */
int32_t bfvgpu_ctx_set_fp64(bfvgpu_ctx *ctx, int32_t on);
/* Words of device scratch bfvgpu_matrix_tiles_device needs for tiles * groups outputs:
 * items * (k + 2 + 2 dk) * n with Enc(0) (enc0 != 0), items * 2 dk * n for a mask alone. */
uint64_t bfvgpu_matrix_tiles_scratch_words(const bfvgpu_ctx *ctx, uint64_t tiles, uint64_t groups,
                                           int32_t enc0);
/* Forward NTT of `count` client ciphertexts [count][2][dk][n] (coefficient form) into out
 * (the same size; may be cts itself) in the operand form of bfvgpu_matrix_tiles_device:
 * every canonical NTT slot v is stored as ((v >> 30) << 32) | (v mod 2^30).  Needs data
 * primes < 2^60 and n >= 32. */
int32_t bfvgpu_matrix_tiles_inputs_device(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count, uint64_t *out,
                                          void *stream);
/* The public key pk [2][k][n] (NTT form) prepared for bfvgpu_matrix_tiles_device: pk_prep
 * [2][k][n][2] words = {v, floor(v 2^64 / q)} with v = pk . q_special^-1 mod q for the data
 * primes and v = pk for the special prime.  Once per key. */
int32_t bfvgpu_matrix_tiles_prepare_pk_device(bfvgpu_ctx *ctx, const uint64_t *pk, uint64_t *pk_prep,
                                              void *stream);
/* Server product of `tiles` token tiles that share one weight matrix (the four calls per
 * tile of Transformer::layer_from_shares, model.hpp:173-238, batched over tiles; per tile
 * and group the result is Matrix::evaluate of matrix.cu:90-106 plus the mask and Enc(0) of
 * bfv_matrix.inc:215-227):
 *   out[t][g][c] = INTT(sum_b in[t][b][c] . w[g][b]) + Enc(0)[t][g] - [c=0] Delta masks[t][g]
 * in [tiles][inputs][2][dk][n] from bfvgpu_matrix_tiles_inputs_device, w
 * [groups][inputs][dk][n] NTT form (bfvgpu_weights_ntt_device), masks
 * [tiles][groups][n] ring-59 words or NULL, samples [tiles][groups][3][k][n] or NULL (then
 * pk_prep may be NULL), pk_prep from bfvgpu_matrix_tiles_prepare_pk_device, scratch of
 * bfvgpu_matrix_tiles_scratch_words words (NULL only without masks and samples), out
 * [tiles][groups][2][dk][n].  Each weight word is read once for all tiles. */
int32_t bfvgpu_matrix_tiles_device(bfvgpu_ctx *ctx, const uint64_t *in, uint64_t tiles, uint64_t inputs,
                                   const uint64_t *w, uint64_t groups, const uint64_t *masks,
                                   const uint64_t *samples, const uint64_t *pk_prep, uint64_t *scratch,
                                   uint64_t *out, void *stream);

/* bfvgpu_matrix_tiles_device in two parts, for callers that prepare a call's output
 * protection ahead of its inputs (the Enc(0) randomness and the masks do not depend on
 * them), e.g. on a side stream while the previous call computes:
 *  - protect: the Enc(0) preparation and additive output term of tiles * groups outputs
 *    into scratch (bfvgpu_matrix_tiles_scratch_words words), from masks and/or samples;
 *  - prepared: the product and the protected output transform reading that scratch; enc0
 *    and masked say which of samples / masks the protect call had.  The caller orders the
 *    two (same stream, or an event); out equals bfvgpu_matrix_tiles_device's. */
int32_t bfvgpu_matrix_tiles_protect_device(bfvgpu_ctx *ctx, uint64_t tiles, uint64_t groups,
                                           const uint64_t *masks, const uint64_t *samples,
                                           const uint64_t *pk_prep, uint64_t *scratch, void *stream);
int32_t bfvgpu_matrix_tiles_prepared_device(bfvgpu_ctx *ctx, const uint64_t *in, uint64_t tiles,
                                            uint64_t inputs, const uint64_t *w, uint64_t groups,
                                            int32_t enc0, int32_t masked, const uint64_t *pk_prep,
                                            const uint64_t *scratch, uint64_t *out, void *stream);

/* Enc(0) polynomials before the divide-and-round, for the matrix epilogue: samples
 * [groups][3][k][n] (ternary u, e0, e1), pk [2][k][n] NTT form; u_scratch [groups][k][n];
 * x_out [groups][2][k][n] = INTT(NTT(u) . pk_c) + e_c (enc0.cu:125-134).  Pass x_out as
 * enc0_x of bfvgpu_matrix_groups_device. */
int32_t bfvgpu_enc0_device(bfvgpu_ctx *ctx, const uint64_t *samples, const uint64_t *pk, uint64_t groups,
                           uint64_t *u_scratch, uint64_t *x_out, void *stream);
/* c0 residues at each group's targets (gather_c0, matrix.cu:66-69) and optionally their
 * CRT values: out [groups][2][dk][n]; targets [groups][max_count], counts [groups];
 * selected [groups][dk][max_count]; crt (nullable) [groups][max_count][dk] limbs. */
int32_t bfvgpu_gather_targets_device(bfvgpu_ctx *ctx, const uint64_t *out, uint64_t groups,
                                     const uint64_t *targets, const uint32_t *counts, uint32_t max_count,
                                     uint64_t *selected, uint64_t *crt, void *stream);

/* ---- NttBatch (IV1/native/gpu/client_phase/ntt.hpp:22-40) ------------------------------ */
/* key_level != 0: all k primes, else the dk data primes; batches in [1, 19]. */
int32_t bfvgpu_ntt_open(bfvgpu_ctx *ctx, int32_t key_level, uint64_t batches, bfvgpu_ntt **out);
/* [batches][primes][n] canonical in, out; forward: natural -> bit-reversed order. */
int32_t bfvgpu_ntt_transform(bfvgpu_ntt *h, const uint64_t *in, uint64_t *out, int32_t inverse);
/* Secret key s [dk][n] in NTT form (data level); once per object. */
int32_t bfvgpu_ntt_bind_client_key(bfvgpu_ntt *h, const uint64_t *sk_ntt);
/* c1 [batches][dk][n] -> INTT(NTT(c1) . s) (ntt.cu:181-199). */
int32_t bfvgpu_ntt_client_phase(bfvgpu_ntt *h, const uint64_t *in, uint64_t *out);
int32_t bfvgpu_ntt_close(bfvgpu_ntt *h, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_ntt_release(bfvgpu_ntt *h);

/* ---- Matrix (IV1/experiments/matrix_gpu/matrix.hpp:9-24) -------------------------------- */
/* inputs in [1, 512] coefficient-form ciphertexts [inputs][2][dk][n]; validated
 * canonical, uploaded and forward-transformed once (Matrix::Matrix, matrix.cu:81-87). */
int32_t bfvgpu_matrix_open(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t inputs, bfvgpu_matrix **out);
/* ring [inputs][n] ring-59 words -> out [2][dk][n] (Matrix::evaluate). */
int32_t bfvgpu_matrix_evaluate(bfvgpu_matrix *m, const uint64_t *ring, uint64_t *out);
/* As evaluate, but c0 is zero except at 1..512 strictly increasing targets
 * (Matrix::evaluate_selective, matrix.cu:90-106). */
int32_t bfvgpu_matrix_evaluate_selective(bfvgpu_matrix *m, const uint64_t *ring, const uint64_t *targets,
                                         uint64_t count, uint64_t *out);
/* Public key [2][k][n] (NTT form, key level) for the Enc(0) re-randomisation. */
int32_t bfvgpu_matrix_bind_public_key(bfvgpu_matrix *m, const uint64_t *pk);
/* Several output groups of BfvEngine::matrix's server loop in one call
 * (bfv_matrix.inc:150-233): per group g, W = lift(ring[g]) [inputs][n], product, INTT,
 * c0 -= Delta*mask[g] (mask nullable), + Enc(0) from samples[g] [3][k][n] (nullable;
 * needs the public key), then c1 [g][dk][n] in full and the c0 residues at the group's
 * targets ([g][dk][max_count], targets [g][max_count], counts[g] <= max_count <= 512);
 * c0_crt (nullable) [g][max_count][dk] receives each target's CRT value in [0,Q) as dk
 * little-endian 64-bit limbs (rns_coefficient, bfv.cpp:138-147). */
int32_t bfvgpu_matrix_evaluate_groups(bfvgpu_matrix *m, uint64_t groups, const uint64_t *ring,
                                      const uint64_t *targets, const uint32_t *counts, uint32_t max_count,
                                      const uint64_t *mask, const uint64_t *samples, uint64_t *c1_out,
                                      uint64_t *c0_targets, uint64_t *c0_crt);
int32_t bfvgpu_matrix_device_bytes(const bfvgpu_matrix *m, uint64_t *bytes);
int32_t bfvgpu_matrix_close(bfvgpu_matrix *m, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_matrix_release(bfvgpu_matrix *m);

/* ---- Switch (IV1/experiments/keyswitch_full_gpu/switch.hpp:12-28) ----------------------- */
/* key [dk][2][k][n] NTT form at the key level for Galois element `galois_elt` (odd, < 2n). */
int32_t bfvgpu_switch_open(bfvgpu_ctx *ctx, const uint64_t *key, uint32_t galois_elt, bfvgpu_switch **out);
/* Galois automorphism then keyswitch of one ciphertext [2][dk][n] (Switch::apply). */
int32_t bfvgpu_switch_apply(bfvgpu_switch *s, const uint64_t *ct, uint64_t *out);
/* The same for count ciphertexts [count][2][dk][n] in one transfer and launch. */
int32_t bfvgpu_switch_apply_many(bfvgpu_switch *s, const uint64_t *cts, uint64_t count, uint64_t *out);
/* Acyclic merge (Switch::packing_pair, switch.cu:155-185): s holds element 1, other
 * holds 2^(level+1)+1, level < logn-5 ... out = sw1(L + X^(n>>(level+1)) R) + swg(...). */
int32_t bfvgpu_switch_packing_pair(bfvgpu_switch *s, const uint64_t *left, const uint64_t *right,
                                   bfvgpu_switch *other, uint32_t level, uint64_t *out);
/* Device milliseconds of the last apply: upload, kernels, download (Switch::timing). */
int32_t bfvgpu_switch_timing(const bfvgpu_switch *s, double *upload_ms, double *kernel_ms, double *download_ms);
int32_t bfvgpu_switch_close(bfvgpu_switch *s, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_switch_release(bfvgpu_switch *s);

/* ---- Rotations: many Switch elements over one ciphertext batch (no single counterpart in the
 * reference; each element's result equals Switch::apply with that element's key) ---------- */
/* keys [count][dk][2][k][n] NTT form, galois_elts [count] (odd, < 2n): uploaded and prepared
 * once here, as Switch uploads its key at construction. */
int32_t bfvgpu_rotations_open(bfvgpu_ctx *ctx, const uint64_t *keys, const uint32_t *galois_elts,
                              uint64_t count, bfvgpu_rotations **out);
/* cts [m][2][dk][n] -> out [count][m][2][dk][n]: one upload of the batch, its digit transforms
 * once, then every element with its results copied back while the next element computes.
 * Host buffers should be pinned for full transfer speed. */
int32_t bfvgpu_rotations_apply(bfvgpu_rotations *r, const uint64_t *cts, uint64_t m, uint64_t *out);
int32_t bfvgpu_rotations_close(bfvgpu_rotations *r, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_rotations_release(bfvgpu_rotations *r);

/* ---- Slot-packed matrix-vector product: BFV batching with rotate-and-sum -----------------
 * The slot variant of the ct-pt matvec (the benchmark's config 3: W [O][K] times a vector of
 * K values in Z_t, t = 1 mod 2n).  The reference's matrix protocol packs coefficients, not
 * slots, so this has no counterpart there; it reuses this library's hoisted rotations and
 * its multi-block ct-pt product.  Slots form two rows of n/2; the input ciphertext holds
 * x[i mod K] in row 0 and x[(i + K/2) mod K] in row 1 (K even, K | n/2, O <= n/2).  With
 * baby * giant = K/2 the result's row 0 holds y[i] = sum_j W[i][j] x[j] at slots i < O:
 *   y = sum_g rot(sum_b pt[g][b] . rot(x, b), g*baby), then row 0 + row 1 (swap + add),
 * where pt[g][b] is the diagonal pair (g*baby + b, K/2 + g*baby + b) pre-rotated by
 * -g*baby.  Keys [baby - 1 + giant - 1 + 1][dk][2][k][n] (host, NTT form) for the Galois
 * elements 3^b (b = 1..baby-1), 3^(g*baby) (g = 1..giant-1) and 2n - 1, in that order;
 * plain [giant][baby][n] (device) the encoded plaintext polynomials (coefficients < t),
 * transformed once here.  Per product: one hoist and baby-1 rotations in one launch pair,
 * the input transform, one product launch over all giant*baby plaintexts, one hoist and
 * giant-1 paired rotations, a sum and the row swap. */
int32_t bfvgpu_slots_open(bfvgpu_ctx *ctx, const uint64_t *keys, uint32_t baby, uint32_t giant,
                          const uint64_t *plain, bfvgpu_slots **out);
/* ct [2][dk][n] -> out [2][dk][n], coefficient form; device pointers (stream NULL: the
 * context stream). */
int32_t bfvgpu_slots_apply_device(bfvgpu_slots *s, const uint64_t *ct, uint64_t *out, void *stream);
/* The same from host buffers (upload, product, download, synchronise). */
int32_t bfvgpu_slots_apply(bfvgpu_slots *s, const uint64_t *ct, uint64_t *out);
int32_t bfvgpu_slots_close(bfvgpu_slots *s, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_slots_release(bfvgpu_slots *s);

/* ---- PublicZero (IV1/native/gpu/enc0/enc0.hpp:15-25) ------------------------------------ */
int32_t bfvgpu_enc0_open(bfvgpu_ctx *ctx, const uint64_t *pk, bfvgpu_enc0 **out);
/* samples [3][k][n] (ternary u, e0, e1 as canonical residues) -> Enc(0) [2][dk][n]. */
int32_t bfvgpu_enc0_encrypt_from_samples(bfvgpu_enc0 *e, const uint64_t *samples, uint64_t *out);
/* Public-key encryption of a plaintext (the client's input blocks, bfv_matrix.inc:31-49):
 * Enc(0) from samples, then c0 += Delta-scaled plain[i] for i < count (plain < t). */
int32_t bfvgpu_enc0_encrypt_plain(bfvgpu_enc0 *e, const uint64_t *samples, const uint64_t *plain,
                                  uint64_t count, uint64_t *out);
/* The client's encryption of a call's input blocks in one go (bfv_matrix.inc:31-49 encrypts
 * them one Encryptor::encrypt at a time): device pointers, samples [cts][3][k][n] (ternary u,
 * e0, e1), pk [2][k][n] NTT form, plain [cts][n] plaintext coefficients (< t; no range check
 * on the device path), scratch of bfvgpu_encrypt_many_scratch_words; out [cts][2][dk][n] =
 * moddown(Enc(0)) + Delta-scaled plain, what bfvgpu_enc0_encrypt_plain gives per ciphertext. */
uint64_t bfvgpu_encrypt_many_scratch_words(const bfvgpu_ctx *ctx, uint64_t cts);
int32_t bfvgpu_encrypt_many_device(bfvgpu_ctx *ctx, const uint64_t *samples, const uint64_t *pk,
                                   const uint64_t *plain, uint64_t cts, uint64_t *scratch, uint64_t *out,
                                   void *stream);
/* Output protection of coefficient-form ciphertexts, the server's masking and
 * re-randomisation before a hand-off (sub_plain_inplace + encrypt_zero + add_inplace,
 * bfv_matrix.inc:215-227, bfv_token_batch.inc:271-272), device pointers:
 *   out [count][2][dk][n] = cts - [c = 0] Delta masks + Enc(0),
 * masks [count][n] ring-59 words (nullable: no mask), samples [count][3][k][n] (ternary u,
 * e0, e1; nullable: no Enc(0), then pk and scratch may be NULL), pk [2][k][n] NTT form at
 * the key level, scratch of bfvgpu_protect_scratch_words words.  out may equal cts. */
uint64_t bfvgpu_protect_scratch_words(const bfvgpu_ctx *ctx, uint64_t count);
int32_t bfvgpu_protect_device(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t count, const uint64_t *masks,
                              const uint64_t *samples, const uint64_t *pk, uint64_t *scratch, uint64_t *out,
                              void *stream);
int32_t bfvgpu_enc0_close(bfvgpu_enc0 *e, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_enc0_release(bfvgpu_enc0 *e);

/* ---- TokenWeights (IV1/experiments/resident_token_gpu/resident.hpp:23-48) --------------- */
/* ART-002 only: cts [slots][19][2][dk][n] coefficient form, slots in [1,4]. */
int32_t bfvgpu_token_open(bfvgpu_ctx *ctx, const uint64_t *cts, uint64_t slots, bfvgpu_token **out);
/* ring [19][8192] ring-59 weights with |w| <= 2^20; local [slots] ring-59 local shares;
 * out [slots][2][dk][n] (evaluate_finished + download). */
int32_t bfvgpu_token_evaluate_finished(bfvgpu_token *t, const uint64_t *ring, const uint64_t *local,
                                       uint64_t *out);
/* TokenWeights::evaluate_device (resident.cu:152-173) for `coords` coordinates at once, device
 * pointers: inputs [19][slots][2][dk][n] the NTT-form input ciphertexts (slots <= 4), ring
 * [coords][19][8192] each coordinate's ring-59 weight rows, local [coords][slots] the local
 * shares added (Delta-scaled) at coefficient 8191; scratch of bfvgpu_token_many_scratch_words;
 * out [coords][slots][2][dk][n] the raw products, as bfvgpu_token_evaluate_finished gives them
 * one coordinate at a time.  n = 16384; no range checks on the device path. */
uint64_t bfvgpu_token_many_scratch_words(const bfvgpu_ctx *ctx, uint64_t coords, uint64_t slots);
int32_t bfvgpu_token_evaluate_many_device(bfvgpu_ctx *ctx, const uint64_t *inputs, uint64_t slots,
                                          const uint64_t *ring, uint64_t coords, const uint64_t *local,
                                          uint64_t *scratch, uint64_t *out, void *stream);
/* One level of the token packing tree for many pairs (bfv_token_batch.inc:203-216 merges the
 * same pairs one at a time through a binary-counter stack): pair (m, s) merges left =
 * in[2m][s] and right = in[2m+1][s] as Switch::packing_pair does (switch.cu:155-185),
 *   out[m][s] = ks_1(L + X^(n >> (level+1)) R) + ks_g(L - X^(n >> (level+1)) R),  g = 2^(level+1) + 1,
 * with key_one / key_level [dk][2][k][n] (device, NTT form) the level's keys for 1 and g;
 * in [2 pairs][slots][2][dk][n], out [pairs][slots][2][dk][n], scratch of
 * bfvgpu_packing_level_scratch_words(ctx, pairs * slots). */
uint64_t bfvgpu_packing_level_scratch_words(const bfvgpu_ctx *ctx, uint64_t count);
int32_t bfvgpu_packing_level_device(bfvgpu_ctx *ctx, const uint64_t *in, uint64_t pairs, uint64_t slots,
                                    uint32_t level, const uint64_t *key_one, const uint64_t *key_level,
                                    uint64_t *scratch, uint64_t *out, void *stream);
/* The return of packed token tiles, one per slot (token_packed_many's tile return,
 * bfv_token_batch.inc:266-283, server side), device pointers: packed [slots][2][dk][n] the
 * tiles from the packing tree, masks [slots][n] ring-59 words, samples [slots][3][k][n], pk
 * [2][k][n] (NTT form).  out [slots][2][dk][n] = packed - [c = 0] Delta masks + Enc(0)
 * (out may equal packed; its c1 is what the reference sends, :272) and c0_crt
 * [slots][512][dk] = the CRT of out's c0 at packed_target(coordinate) = 32 * (the 9-bit
 * reversal of the coordinate) for coordinates 0..511 in order, as dk little-endian 64-bit
 * limbs of a value in [0, Q) (rns_coefficient, :273-274).  The mask words at those targets
 * (masks[target], :274) stay with the caller.  ART-002 (n = 16384) only; slots in [1, 4];
 * scratch of bfvgpu_token_finish_scratch_words(ctx, slots) words. */
uint64_t bfvgpu_token_finish_scratch_words(const bfvgpu_ctx *ctx, uint64_t slots);
int32_t bfvgpu_token_finish_device(bfvgpu_ctx *ctx, const uint64_t *packed, uint64_t slots, const uint64_t *masks,
                                   const uint64_t *samples, const uint64_t *pk, uint64_t *scratch, uint64_t *out,
                                   uint64_t *c0_crt, void *stream);
int32_t bfvgpu_token_close(bfvgpu_token *t, bfvgpu_cleanup *cleanup);
int32_t bfvgpu_token_release(bfvgpu_token *t);

#ifdef __cplusplus
}
#endif
#endif /* BFVGPU_H */
