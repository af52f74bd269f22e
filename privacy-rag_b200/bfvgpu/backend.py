"""Python mirror of privacy-rag's GPU backend classes over the bfvgpu C ABI.

Each class keeps the reference class's name, member names, argument meaning and
error behaviour (IV1 = implementation_v1/ of the reference):

* ``NttBatch``      IV1/native/gpu/client_phase/ntt.hpp:22-40
* ``Matrix``        IV1/experiments/matrix_gpu/matrix.hpp:9-24
* ``Switch``        IV1/experiments/keyswitch_full_gpu/switch.hpp:12-28
* ``PublicZero``    IV1/native/gpu/enc0/enc0.hpp:15-25
* ``TokenWeights``  IV1/experiments/resident_token_gpu/resident.hpp:23-48

SEAL objects become flat ``numpy.uint64`` arrays in the layouts the reference
adapters copy out of them.  Validation failures raise ``BfvGpuInvalidArgument``
(a ``ValueError``, the reference's ``std::invalid_argument``); CUDA failures raise
``BfvGpuError`` after the object's device state has been released; ``close()``
never raises and returns the cleanup record.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import Cleanup, U32, U64, VP, check, lib, ptr, u64

ART002_PRIMES = (
    1152921504599080961, 1152921504600260609, 1152921504604979201,
    1152921504605962241, 1152921504606584833, 1152921504606683137,
    1152921504606748673,
)


def find_primes(n: int, bits: list[int]) -> list[int]:
    """Prime chain = 1 mod 2n with the given bit sizes (bfvgpu_find_primes)."""
    out = (U64 * len(bits))()
    arr = (ctypes.c_int32 * len(bits))(*bits)
    check(lib().bfvgpu_find_primes(n, arr, len(bits), out), "find_primes")
    return [int(v) for v in out]


def launch_count() -> int:
    """Kernel launches this process issued through the library."""
    return int(lib().bfvgpu_launch_count())


class Context:
    """Parameter context on one device (device=-1: host-only, tables and constants)."""

    def __init__(self, n: int, primes, data_primes: int, special_primes: int = 1,
                 plain_modulus: int = 1 << 59, device: int = 0):
        self.n = int(n)
        self.primes = [int(p) for p in primes]
        self.data_primes = int(data_primes)
        self.k = self.data_primes + int(special_primes)
        self.t = int(plain_modulus)
        self.device = int(device)
        if len(self.primes) != self.k:
            raise ValueError("E_BFVGPU_PRIME_COUNT")
        arr = u64(self.primes)
        h = VP()
        check(lib().bfvgpu_ctx_create(self.n, ptr(arr), self.data_primes, int(special_primes), self.t,
                                      self.device, ctypes.byref(h)), "Context")
        self._h = h

    @classmethod
    def art002(cls, device: int = 0) -> "Context":
        return cls(16384, ART002_PRIMES, 6, 1, 1 << 59, device)

    @property
    def handle(self):
        return self._h

    @property
    def dk(self) -> int:
        return self.data_primes

    def tables(self, prime: int):
        fwd = np.zeros((self.n, 2), dtype=np.uint64)
        inv = np.zeros((self.n, 2), dtype=np.uint64)
        invn = np.zeros(2, dtype=np.uint64)
        check(lib().bfvgpu_ctx_tables(self._h, prime, ptr(fwd), ptr(inv), ptr(invn)), "tables")
        return fwd, inv, invn

    def moduli(self) -> np.ndarray:
        out = np.zeros((self.k, 16), dtype=np.uint64)
        for p in range(self.k):
            check(lib().bfvgpu_ctx_moduli(self._h, p, ptr(out[p])), "moduli")
        return out

    def stream(self) -> int:
        s = VP()
        check(lib().bfvgpu_ctx_stream(self._h, ctypes.byref(s), None), "stream")
        return s.value or 0

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().bfvgpu_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- device-resident batched entry points (torch CUDA tensors or raw pointers) ----
    @staticmethod
    def _dptr(x) -> int:
        if x is None:
            return 0
        if isinstance(x, int):
            return x
        return int(x.data_ptr())

    def ntt_device(self, data, polys: int, prime_count: int, prime_offset: int = 0, inverse: bool = False,
                   stream: int | None = None) -> None:
        check(lib().bfvgpu_ntt_device(self._h, self._dptr(data), polys, prime_count, prime_offset,
                                      int(bool(inverse)), stream), "ntt_device")

    def keyswitch_scratch_words(self, count: int) -> int:
        return int(lib().bfvgpu_keyswitch_scratch_words(self._h, count))

    def keyswitch_device(self, cts, count: int, key, galois_elt: int, scratch, out, stream: int | None = None):
        check(lib().bfvgpu_keyswitch_device(self._h, self._dptr(cts), count, self._dptr(key), galois_elt,
                                            self._dptr(scratch), self._dptr(out), stream), "keyswitch_device")

    def int_peak_device(self, kind: int, blocks: int, iters: int, sink, stream: int | None = None) -> int:
        """Launch the peak kernel of `kind` (integer pipe: 0 butterfly, 1 multiply-accumulate,
        2 Barrett modular product, 3 Shoup product; FP64 pipe, prime 0 < 2^50: 4 butterfly,
        5 product by a fixed operand); returns the operations it performs.  sink: blocks * 256
        words."""
        ops = U64(0)
        check(lib().bfvgpu_int_peak_device(self._h, kind, blocks, iters, self._dptr(sink), ctypes.byref(ops),
                                           stream), "int_peak_device")
        return int(ops.value)

    def protect_scratch_words(self, count: int) -> int:
        return int(lib().bfvgpu_protect_scratch_words(self._h, count))

    def protect_device(self, cts, count: int, out, masks=None, samples=None, pk=None, scratch=None,
                       stream: int | None = None) -> None:
        """out = cts - Delta masks (c0) + Enc(0) from samples (bfvgpu_protect_device)."""
        check(lib().bfvgpu_protect_device(self._h, self._dptr(cts), count, self._dptr(masks), self._dptr(samples),
                                          self._dptr(pk), self._dptr(scratch), self._dptr(out), stream),
              "protect_device")

    def token_finish_scratch_words(self, slots: int) -> int:
        return int(lib().bfvgpu_token_finish_scratch_words(self._h, slots))

    def token_finish_device(self, packed, slots: int, masks, samples, pk, scratch, out, c0_crt,
                            stream: int | None = None) -> None:
        """Tile return of packed token tiles (bfvgpu_token_finish_device)."""
        check(lib().bfvgpu_token_finish_device(self._h, self._dptr(packed), slots, self._dptr(masks),
                                               self._dptr(samples), self._dptr(pk), self._dptr(scratch),
                                               self._dptr(out), self._dptr(c0_crt), stream), "token_finish_device")

    def keyswitch_rotate_many_scratch_words(self, count: int) -> int:
        return int(lib().bfvgpu_keyswitch_rotate_many_scratch_words(self._h, count))

    def keyswitch_rotate_many_device(self, cts, count: int, hoisted, prepared, galois_elts, scratch, outs,
                                     stream: int | None = None) -> None:
        """The hoisted rotations of every element in galois_elts, software-pipelined; outs: one
        device tensor (or pointer) per element, or a single one that every element overwrites."""
        m = len(galois_elts)
        if not isinstance(outs, (list, tuple)):
            outs = [outs] * m
        el = (U32 * m)(*[int(e) for e in galois_elts])
        op = (VP * m)(*[self._dptr(o) for o in outs])
        check(lib().bfvgpu_keyswitch_rotate_many_device(self._h, self._dptr(cts), count, self._dptr(hoisted),
                                                        self._dptr(prepared), el, m, self._dptr(scratch), op, stream),
              "keyswitch_rotate_many_device")

    def keyswitch_prepared_words(self) -> int:
        return int(lib().bfvgpu_keyswitch_prepared_words(self._h))

    def keyswitch_hoist_words(self, count: int) -> int:
        return int(lib().bfvgpu_keyswitch_hoist_words(self._h, count))

    def keyswitch_prepare_device(self, keys, galois_elts, prepared, stream: int | None = None):
        """keys [count][dk][2][k][n] (device) for the Galois elements galois_elts (ints)
        -> prepared [count][keyswitch_prepared_words()] (device)."""
        elts = [int(e) for e in (galois_elts if hasattr(galois_elts, "__len__") else [galois_elts])]
        arr = (U32 * len(elts))(*elts)
        check(lib().bfvgpu_keyswitch_prepare_device(self._h, self._dptr(keys), arr, len(elts), self._dptr(prepared),
                                                    stream), "keyswitch_prepare_device")

    def keyswitch_hoist_device(self, cts, count: int, hoisted, stream: int | None = None):
        check(lib().bfvgpu_keyswitch_hoist_device(self._h, self._dptr(cts), count, self._dptr(hoisted), stream),
              "keyswitch_hoist_device")

    def keyswitch_rotate_device(self, cts, count: int, hoisted, prepared, galois_elt: int, scratch, out,
                                stream: int | None = None):
        check(lib().bfvgpu_keyswitch_rotate_device(self._h, self._dptr(cts), count, self._dptr(hoisted),
                                                   self._dptr(prepared), galois_elt, self._dptr(scratch),
                                                   self._dptr(out), stream), "keyswitch_rotate_device")

    def weights_ntt_device(self, ring, blocks: int, out, stream: int | None = None):
        check(lib().bfvgpu_weights_ntt_device(self._h, self._dptr(ring), blocks, self._dptr(out), stream),
              "weights_ntt_device")

    def enc0_device(self, samples, pk, groups: int, u_scratch, x_out, stream: int | None = None):
        check(lib().bfvgpu_enc0_device(self._h, self._dptr(samples), self._dptr(pk), groups, self._dptr(u_scratch),
                                       self._dptr(x_out), stream), "enc0_device")

    def gather_targets_device(self, out, groups: int, targets, counts, max_count: int, selected, crt=None,
                              stream: int | None = None):
        check(lib().bfvgpu_gather_targets_device(self._h, self._dptr(out), groups, self._dptr(targets),
                                                 self._dptr(counts), max_count, self._dptr(selected),
                                                 self._dptr(crt) or None, stream), "gather_targets_device")

    def matrix_groups_device(self, inputs_ntt, inputs: int, weights_ntt, groups: int, out, mask=None,
                             enc0_x=None, stream: int | None = None):
        check(lib().bfvgpu_matrix_groups_device(self._h, self._dptr(inputs_ntt), inputs, self._dptr(weights_ntt),
                                                groups, self._dptr(mask) or None, self._dptr(enc0_x) or None,
                                                self._dptr(out), stream), "matrix_groups_device")

    def check(self) -> int:
        """Synchronise and return the kernel-recorded error bits (raises if any is set)."""
        flags = U32(0)
        check(lib().bfvgpu_ctx_check(self._h, ctypes.byref(flags)), "ctx_check")
        return int(flags.value)

    def set_reserved_sms(self, sms: int) -> None:
        """SMs the persistent product kernels leave free (for collectives running beside them)."""
        check(lib().bfvgpu_ctx_set_reserved_sms(self._h, sms), "set_reserved_sms")

    def set_limb_split(self, split: bool) -> None:
        """n = 16384 single-transform kernels: split each limb between the two blocks of a
        cluster (True, the default) or one block per limb (False).  Results are identical."""
        check(lib().bfvgpu_ctx_set_limb_split(self._h, int(bool(split))), "set_limb_split")

    def set_fp64(self, on: bool) -> None:
        """Primes below 2^50: compute the transforms and rotations that have an FP64 form on
        the FP64 pipe (True, the default) or on the integer pipe (False).  Results are
        identical; fixed once the context has prepared keys (BFVGPU_E_STATE)."""
        check(lib().bfvgpu_ctx_set_fp64(self._h, int(bool(on))), "set_fp64")

    def set_product_path(self, path: int) -> None:
        """0: tcgen05 product for 8-tile launches (default); 1: TMA-staged CUDA-core product only;
        2: CUDA-core product with per-thread asynchronous-copy staging."""
        check(lib().bfvgpu_ctx_set_product_path(self._h, path), "set_product_path")

    def matrix_tiles_inputs_device(self, cts, count: int, out=None, stream: int | None = None):
        """Transform client ciphertexts [count][2][dk][n] into out (default: in place) in the
        operand form of matrix_tiles_device (NTT slots with their 30-bit halves split)."""
        check(lib().bfvgpu_matrix_tiles_inputs_device(self._h, self._dptr(cts), count,
                                                      self._dptr(cts if out is None else out), stream),
              "matrix_tiles_inputs_device")

    def matrix_tiles_prepare_pk_device(self, pk, pk_prep, stream: int | None = None):
        """pk [2][k][n] (NTT form) -> pk_prep [2][k][n][2] for matrix_tiles_device."""
        check(lib().bfvgpu_matrix_tiles_prepare_pk_device(self._h, self._dptr(pk), self._dptr(pk_prep), stream),
              "matrix_tiles_prepare_pk_device")

    def matrix_tiles_scratch_words(self, tiles: int, groups: int, enc0: bool = True) -> int:
        return int(lib().bfvgpu_matrix_tiles_scratch_words(self._h, tiles, groups, int(bool(enc0))))

    def matrix_tiles_device(self, inputs_ntt, tiles: int, inputs: int, weights_ntt, groups: int, out, masks=None,
                            samples=None, pk_prep=None, scratch=None, stream: int | None = None):
        """out [tiles][groups][2][dk][n] = product of each tile's inputs [tiles][inputs][2][dk][n]
        (from matrix_tiles_inputs_device) with the shared NTT-form weights
        [groups][inputs][dk][n], plus Enc(0) from samples [tiles][groups][3][k][n] (public key
        from matrix_tiles_prepare_pk_device) and minus the Delta-scaled masks."""
        check(lib().bfvgpu_matrix_tiles_device(self._h, self._dptr(inputs_ntt), tiles, inputs,
                                               self._dptr(weights_ntt), groups, self._dptr(masks) or None,
                                               self._dptr(samples) or None, self._dptr(pk_prep) or None,
                                               self._dptr(scratch) or None, self._dptr(out), stream),
              "matrix_tiles_device")

    def encrypt_many_scratch_words(self, cts: int) -> int:
        return int(lib().bfvgpu_encrypt_many_scratch_words(self._h, cts))

    def encrypt_many_device(self, samples, pk, plain, cts: int, scratch, out, stream: int | None = None):
        """Client encryption of cts plaintexts [cts][n]: out [cts][2][dk][n] (device tensors)."""
        check(lib().bfvgpu_encrypt_many_device(self._h, self._dptr(samples), self._dptr(pk), self._dptr(plain), cts,
                                               self._dptr(scratch), self._dptr(out), stream), "encrypt_many_device")

    def token_many_scratch_words(self, coords: int, slots: int) -> int:
        return int(lib().bfvgpu_token_many_scratch_words(self._h, coords, slots))

    def token_evaluate_many_device(self, inputs_ntt, slots: int, ring, coords: int, local, scratch, out,
                                   stream: int | None = None):
        """Raw token products of `coords` coordinates: out [coords][slots][2][dk][n]."""
        check(lib().bfvgpu_token_evaluate_many_device(self._h, self._dptr(inputs_ntt), slots, self._dptr(ring), coords,
                                                      self._dptr(local), self._dptr(scratch), self._dptr(out), stream),
              "token_evaluate_many_device")

    def packing_level_scratch_words(self, count: int) -> int:
        return int(lib().bfvgpu_packing_level_scratch_words(self._h, count))

    def packing_level_device(self, cts, pairs: int, slots: int, level: int, key_one, key_level, scratch, out,
                             stream: int | None = None):
        """One packing-tree level: cts [2 pairs][slots][2][dk][n] -> out [pairs][slots][2][dk][n]."""
        check(lib().bfvgpu_packing_level_device(self._h, self._dptr(cts), pairs, slots, level, self._dptr(key_one),
                                                self._dptr(key_level), self._dptr(scratch), self._dptr(out), stream),
              "packing_level_device")

    def matrix_tiles_protect_device(self, tiles: int, groups: int, scratch, masks=None, samples=None, pk_prep=None,
                                    stream: int | None = None):
        """The output protection of a matrix_tiles call (Enc(0) preparation and the additive
        output term) into scratch, ahead of the call's inputs."""
        check(lib().bfvgpu_matrix_tiles_protect_device(self._h, tiles, groups, self._dptr(masks) or None,
                                                       self._dptr(samples) or None, self._dptr(pk_prep) or None,
                                                       self._dptr(scratch), stream),
              "matrix_tiles_protect_device")

    def matrix_tiles_prepared_device(self, inputs_ntt, tiles: int, inputs: int, weights_ntt, groups: int, out,
                                     enc0: bool, masked: bool, pk_prep=None, scratch=None,
                                     stream: int | None = None):
        """matrix_tiles_device with its protection already in scratch (matrix_tiles_protect_device)."""
        check(lib().bfvgpu_matrix_tiles_prepared_device(self._h, self._dptr(inputs_ntt), tiles, inputs,
                                                        self._dptr(weights_ntt), groups, int(bool(enc0)),
                                                        int(bool(masked)), self._dptr(pk_prep) or None,
                                                        self._dptr(scratch) or None, self._dptr(out), stream),
              "matrix_tiles_prepared_device")


class _Handle:
    _close_fn = ""
    _release_fn = ""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self._h = None
        self._cleanup = None

    def close(self) -> dict:
        """Wipe and free every sensitive device buffer; idempotent, never raises."""
        c = Cleanup()
        if self._h is not None:
            getattr(lib(), self._close_fn)(self._h, ctypes.byref(c))
            self._cleanup = c.as_dict()
        return self._cleanup or {"first_cuda_error": 0, "closed": True, "wiped": 0, "freed": 0}

    def __del__(self):
        try:
            if self._h is not None:
                getattr(lib(), self._release_fn)(self._h)
                self._h = None
        except Exception:
            pass


class NttBatch(_Handle):
    """Batched canonical NTT/INTT and the client phase c1*s (layout [batch][prime][n])."""

    _close_fn = "bfvgpu_ntt_close"
    _release_fn = "bfvgpu_ntt_release"

    def __init__(self, ctx: Context, key_level: bool, batches: int):
        super().__init__(ctx)
        self.primes = ctx.k if key_level else ctx.dk
        self.batches = int(batches)
        h = VP()
        check(lib().bfvgpu_ntt_open(ctx.handle, int(bool(key_level)), self.batches, ctypes.byref(h)), "NttBatch")
        self._h = h

    def transform(self, data, inverse: bool) -> np.ndarray:
        a = u64(data)
        if a.size != self.batches * self.primes * self.ctx.n:
            raise ValueError("E_NTT_SHAPE")
        out = np.empty_like(a)
        check(lib().bfvgpu_ntt_transform(self._h, ptr(a), ptr(out), int(bool(inverse))), "NttBatch.transform")
        return out

    def bind_client_key(self, ntt_key) -> None:
        k = u64(ntt_key)
        if k.size != self.ctx.dk * self.ctx.n:
            raise ValueError("E_CLIENT_KEY_SHAPE")
        check(lib().bfvgpu_ntt_bind_client_key(self._h, ptr(k)), "NttBatch.bind_client_key")

    def client_phase(self, data) -> np.ndarray:
        a = u64(data)
        if a.size != self.batches * self.primes * self.ctx.n:
            raise ValueError("E_NTT_SHAPE")
        out = np.empty_like(a)
        check(lib().bfvgpu_ntt_client_phase(self._h, ptr(a), ptr(out)), "NttBatch.client_phase")
        return out


class Matrix(_Handle):
    """Coefficient-packed ct-pt product backend of BfvEngine::matrix."""

    _close_fn = "bfvgpu_matrix_close"
    _release_fn = "bfvgpu_matrix_release"

    def __init__(self, ctx: Context, cts):
        super().__init__(ctx)
        a = u64(cts)
        per = 2 * ctx.dk * ctx.n
        if a.size == 0 or a.size % per:
            raise ValueError("MATRIX_GPU_CONTEXT")
        self.blocks = a.size // per
        h = VP()
        check(lib().bfvgpu_matrix_open(ctx.handle, ptr(a), self.blocks, ctypes.byref(h)), "Matrix")
        self._h = h

    def evaluate(self, ring) -> np.ndarray:
        r = u64(ring)
        if r.size != self.blocks * self.ctx.n:
            raise ValueError("MATRIX_GPU_SHAPE")
        out = np.zeros((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_matrix_evaluate(self._h, ptr(r), ptr(out)), "Matrix.evaluate")
        return out

    def evaluate_selective(self, ring, targets) -> np.ndarray:
        r = u64(ring)
        t = u64(targets)
        if r.size != self.blocks * self.ctx.n:
            raise ValueError("MATRIX_GPU_SHAPE")
        out = np.zeros((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_matrix_evaluate_selective(self._h, ptr(r), ptr(t) if t.size else None, t.size,
                                                      ptr(out)), "Matrix.evaluate_selective")
        return out

    def bind_public_key(self, pk) -> None:
        p = u64(pk)
        if p.size != 2 * self.ctx.k * self.ctx.n:
            raise ValueError("E_BFV_KEY")
        check(lib().bfvgpu_matrix_bind_public_key(self._h, ptr(p)), "Matrix.bind_public_key")

    def evaluate_groups(self, ring, targets: list, mask=None, samples=None, crt: bool = False):
        """Several output groups: ring [G][blocks][n]; targets: list of G increasing lists.
        Returns (c1 [G][dk][n], c0 residues [G][dk][max], crt limbs [G][max][dk] or None)."""
        r = u64(ring)
        G = len(targets)
        n, dk = self.ctx.n, self.ctx.dk
        if r.size != G * self.blocks * n:
            raise ValueError("MATRIX_GPU_SHAPE")
        mx = max(1, max(len(t) for t in targets))
        tg = np.zeros((G, mx), dtype=np.uint64)
        counts = (U32 * G)()
        for g, t in enumerate(targets):
            tg[g, :len(t)] = t
            counts[g] = len(t)
        m = u64(mask) if mask is not None else None
        s = u64(samples) if samples is not None else None
        c1 = np.zeros((G, dk, n), dtype=np.uint64)
        c0 = np.zeros((G, dk, mx), dtype=np.uint64)
        cr = np.zeros((G, mx, dk), dtype=np.uint64) if crt else None
        check(lib().bfvgpu_matrix_evaluate_groups(self._h, G, ptr(r), ptr(tg), counts, mx, ptr(m), ptr(s),
                                                  ptr(c1), ptr(c0), ptr(cr)), "Matrix.evaluate_groups")
        return c1, c0, cr

    def device_bytes(self) -> int:
        b = U64()
        check(lib().bfvgpu_matrix_device_bytes(self._h, ctypes.byref(b)), "Matrix.device_bytes")
        return int(b.value)


class Switch(_Handle):
    """Galois automorphism + alpha=1 special-prime keyswitch for one Galois element."""

    _close_fn = "bfvgpu_switch_close"
    _release_fn = "bfvgpu_switch_release"

    def __init__(self, ctx: Context, key, element: int):
        super().__init__(ctx)
        k = u64(key)
        if k.size != ctx.dk * 2 * ctx.k * ctx.n:
            raise ValueError("E_NTT_CONTEXT")
        self.element = int(element)
        h = VP()
        check(lib().bfvgpu_switch_open(ctx.handle, ptr(k), self.element, ctypes.byref(h)), "Switch")
        self._h = h

    def apply(self, ct) -> np.ndarray:
        a = u64(ct)
        if a.size != 2 * self.ctx.dk * self.ctx.n:
            raise ValueError("E_SWITCH_CIPHERTEXT")
        out = np.empty((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_switch_apply(self._h, ptr(a), ptr(out)), "Switch.apply")
        return out

    def apply_many(self, cts) -> np.ndarray:
        a = u64(cts)
        per = 2 * self.ctx.dk * self.ctx.n
        if a.size == 0 or a.size % per:
            raise ValueError("E_SWITCH_CIPHERTEXT")
        out = np.empty((a.size // per, 2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_switch_apply_many(self._h, ptr(a), a.size // per, ptr(out)), "Switch.apply_many")
        return out

    def packing_pair(self, left, right, difference: "Switch", level: int) -> np.ndarray:
        L, R = u64(left), u64(right)
        out = np.empty((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_switch_packing_pair(self._h, ptr(L), ptr(R), difference._h, level, ptr(out)),
              "Switch.packing_pair")
        return out

    def timing(self) -> dict:
        a, b, c = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        check(lib().bfvgpu_switch_timing(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)), "timing")
        return {"upload_ms": a.value, "kernel_ms": b.value, "download_ms": c.value}


class Rotations(_Handle):
    """Many Galois elements over one ciphertext batch: keys prepared once at construction,
    the batch uploaded and its digits transformed once per apply, every element's result
    streamed back while the next element computes."""

    _close_fn = "bfvgpu_rotations_close"
    _release_fn = "bfvgpu_rotations_release"

    def __init__(self, ctx: Context, keys, elements):
        super().__init__(ctx)
        self.elements = [int(e) for e in elements]
        k = u64(keys)
        if k.size != len(self.elements) * ctx.dk * 2 * ctx.k * ctx.n:
            raise ValueError("E_NTT_CONTEXT")
        arr = (U32 * len(self.elements))(*self.elements)
        h = VP()
        check(lib().bfvgpu_rotations_open(ctx.handle, ptr(k), arr, len(self.elements), ctypes.byref(h)), "Rotations")
        self._h = h

    def apply(self, cts, out=None) -> np.ndarray:
        """cts [m][2][dk][n] -> [elements][m][2][dk][n] (into `out` when given, e.g. pinned)."""
        a = u64(cts)
        per = 2 * self.ctx.dk * self.ctx.n
        if a.size == 0 or a.size % per:
            raise ValueError("E_SWITCH_CIPHERTEXT")
        m = a.size // per
        if out is None:
            out = np.empty((len(self.elements), m, 2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        elif out.dtype != np.uint64 or out.size != len(self.elements) * m * per or not out.flags.c_contiguous:
            raise ValueError("E_SWITCH_OUTPUT")
        check(lib().bfvgpu_rotations_apply(self._h, ptr(a), m, ptr(out)), "Rotations.apply")
        return out


class SlotMatvec(_Handle):
    """Slot-packed ct-pt matrix-vector product (BFV batching, rotate-and-sum with baby-step
    giant-step diagonals; bfvgpu.slots builds the plaintexts and the input packing).  Keys
    [baby-1 + giant-1 + 1][dk][2][k][n] (host) for 3^b, 3^(g*baby) and 2n-1; plain
    [giant][baby][n] encoded plaintext polynomials on the device."""

    _close_fn = "bfvgpu_slots_close"
    _release_fn = "bfvgpu_slots_release"

    def __init__(self, ctx: Context, keys, baby: int, giant: int, plain):
        super().__init__(ctx)
        self.baby, self.giant = int(baby), int(giant)
        k = u64(keys)
        if k.size != (self.baby + self.giant - 1) * ctx.dk * 2 * ctx.k * ctx.n:
            raise ValueError("E_SLOTS_KEYS")
        if plain.numel() != self.giant * self.baby * ctx.n:
            raise ValueError("E_SLOTS_PLAIN")
        h = VP()
        check(lib().bfvgpu_slots_open(ctx.handle, ptr(k), self.baby, self.giant, Context._dptr(plain),
                                      ctypes.byref(h)), "SlotMatvec")
        self._h = h

    def apply_device(self, ct, out, stream: int | None = None) -> None:
        """ct, out: device tensors of [2][dk][n] words (coefficient form)."""
        check(lib().bfvgpu_slots_apply_device(self._h, Context._dptr(ct), Context._dptr(out), stream),
              "SlotMatvec.apply_device")

    def apply(self, ct, out=None) -> np.ndarray:
        """Host ciphertext [2][dk][n] -> host result [2][dk][n]."""
        a = u64(ct)
        if a.size != 2 * self.ctx.dk * self.ctx.n:
            raise ValueError("E_SLOTS_CIPHERTEXT")
        if out is None:
            out = np.empty((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_slots_apply(self._h, ptr(a), ptr(out)), "SlotMatvec.apply")
        return out


class PublicZero(_Handle):
    """Enc(0) from explicit samples (u ternary, e0, e1) with a bound public key."""

    _close_fn = "bfvgpu_enc0_close"
    _release_fn = "bfvgpu_enc0_release"

    def __init__(self, ctx: Context, pk):
        super().__init__(ctx)
        p = u64(pk)
        if p.size != 2 * ctx.k * ctx.n:
            raise ValueError("E_NTT_CONTEXT")
        h = VP()
        check(lib().bfvgpu_enc0_open(ctx.handle, ptr(p), ctypes.byref(h)), "PublicZero")
        self._h = h

    def encrypt_from_samples(self, samples) -> np.ndarray:
        s = u64(samples)
        if s.size != 3 * self.ctx.k * self.ctx.n:
            raise ValueError("E_ENC0_SAMPLE_SHAPE")
        out = np.empty((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_enc0_encrypt_from_samples(self._h, ptr(s), ptr(out)), "PublicZero.encrypt_from_samples")
        return out

    def encrypt(self, samples, plain) -> np.ndarray:
        """Enc(0) from samples plus the Delta-scaled plaintext (coefficients < t)."""
        s = u64(samples)
        p = u64(plain).ravel()
        if s.size != 3 * self.ctx.k * self.ctx.n:
            raise ValueError("E_ENC0_SAMPLE_SHAPE")
        out = np.empty((2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_enc0_encrypt_plain(self._h, ptr(s), ptr(p), p.size, ptr(out)), "PublicZero.encrypt")
        return out


class TokenWeights(_Handle):
    """Resident token-lookup product (ART-002): 19 input blocks per slot."""

    _close_fn = "bfvgpu_token_close"
    _release_fn = "bfvgpu_token_release"

    def __init__(self, ctx: Context, cts):
        super().__init__(ctx)
        a = u64(cts)
        per = 19 * 2 * ctx.dk * ctx.n
        if a.size == 0 or a.size % per:
            raise ValueError("E_GPU_TOKEN_CONTEXT_LAYOUT")
        self.slots = a.size // per
        h = VP()
        check(lib().bfvgpu_token_open(ctx.handle, ptr(a), self.slots, ctypes.byref(h)), "TokenWeights")
        self._h = h

    def evaluate_finished(self, weights, local) -> np.ndarray:
        w = u64(weights)
        loc = u64(local)
        if w.size != 19 * 8192:
            raise ValueError("E_RESIDENT_WEIGHT_SHAPE")
        if loc.size != self.slots:
            raise ValueError("E_RESIDENT_LOCAL_SHAPE")
        out = np.empty((self.slots, 2, self.ctx.dk, self.ctx.n), dtype=np.uint64)
        check(lib().bfvgpu_token_evaluate_finished(self._h, ptr(w), ptr(loc), ptr(out)),
              "TokenWeights.evaluate_finished")
        return out
