"""ctypes binding of libbfvgpu.so (include/bfvgpu.h).

The library is built in-tree (``privacy-rag_b200/build.py``) into
``privacy-rag_b200/lib/libbfvgpu.so``.  There is no fallback: if the library is
missing, importing a backend raises ``BfvGpuUnavailable``.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG, "lib", "libbfvgpu.so")

U64 = ctypes.c_uint64
U64P = ctypes.POINTER(ctypes.c_uint64)
U32 = ctypes.c_uint32
U32P = ctypes.POINTER(ctypes.c_uint32)
I32 = ctypes.c_int32
VP = ctypes.c_void_p

ERROR_NAMES = {
    0: "BFVGPU_OK", 1: "BFVGPU_E_ARGUMENT", 2: "BFVGPU_E_CONTEXT", 3: "BFVGPU_E_SHAPE",
    4: "BFVGPU_E_CANONICAL", 5: "BFVGPU_E_RING", 6: "BFVGPU_E_TARGET_COUNT",
    7: "BFVGPU_E_TARGET_INDEX", 8: "BFVGPU_E_CLOSED", 9: "BFVGPU_E_CUDA", 10: "BFVGPU_E_DEVICE",
    11: "BFVGPU_E_STATE", 12: "BFVGPU_E_BOUND", 13: "BFVGPU_E_ELEMENT", 14: "BFVGPU_E_ALLOC",
}


class BfvGpuUnavailable(RuntimeError):
    """The CUDA library is not built or cannot be loaded."""


class BfvGpuError(RuntimeError):
    """A non-zero status from the C ABI; ``code``/``name`` are the stable error code,
    ``detail`` the library's message (the reference's E_* text)."""

    def __init__(self, code: int, detail: str, where: str):
        self.code = code
        self.name = ERROR_NAMES.get(code, f"BFVGPU_E_{code}")
        self.detail = detail
        super().__init__(f"{where}: {self.name}: {detail}")


class Cleanup(ctypes.Structure):
    """bfvgpu_cleanup: the reference's Cleanup{first_cuda_error, wiped, freed, closed}."""

    _fields_ = [("first_cuda_error", I32), ("closed", I32), ("wiped", U64), ("freed", U64)]

    def as_dict(self) -> dict:
        return {"first_cuda_error": int(self.first_cuda_error), "closed": bool(self.closed),
                "wiped": int(self.wiped), "freed": int(self.freed)}


_SIGNATURES = {
    "bfvgpu_version": (I32, []),
    "bfvgpu_error_name": (ctypes.c_char_p, [I32]),
    "bfvgpu_last_error": (ctypes.c_char_p, []),
    "bfvgpu_launch_count": (U64, []),
    "bfvgpu_find_primes": (I32, [U32, ctypes.POINTER(I32), U32, U64P]),
    "bfvgpu_ctx_create": (I32, [U32, U64P, U32, U32, U64, I32, ctypes.POINTER(VP)]),
    "bfvgpu_ctx_create_art002": (I32, [I32, ctypes.POINTER(VP)]),
    "bfvgpu_ctx_destroy": (I32, [VP]),
    "bfvgpu_ctx_tables": (I32, [VP, U32, U64P, U64P, U64P]),
    "bfvgpu_ctx_moduli": (I32, [VP, U32, U64P]),
    "bfvgpu_ctx_stream": (I32, [VP, ctypes.POINTER(VP), ctypes.POINTER(I32)]),
    "bfvgpu_ntt_device": (I32, [VP, VP, U64, U32, U32, I32, VP]),
    "bfvgpu_keyswitch_scratch_words": (U64, [VP, U64]),
    "bfvgpu_keyswitch_device": (I32, [VP, VP, U64, VP, U32, VP, VP, VP]),
    "bfvgpu_keyswitch_device_noalloc": (I32, [VP, VP, U64, VP, U32, VP, VP]),
    "bfvgpu_int_peak_device": (I32, [VP, I32, U32, U32, VP, U64P, VP]),
    "bfvgpu_ctx_set_limb_split": (I32, [VP, I32]),
    "bfvgpu_ctx_set_fp64": (I32, [VP, I32]),
    "bfvgpu_keyswitch_rotate_many_scratch_words": (U64, [VP, U64]),
    "bfvgpu_keyswitch_rotate_many_device": (I32, [VP, VP, U64, VP, VP, U32P, U64, VP, ctypes.POINTER(VP), VP]),
    "bfvgpu_protect_scratch_words": (U64, [VP, U64]),
    "bfvgpu_protect_device": (I32, [VP, VP, U64, VP, VP, VP, VP, VP, VP]),
    "bfvgpu_token_finish_scratch_words": (U64, [VP, U64]),
    "bfvgpu_token_finish_device": (I32, [VP, VP, U64, VP, VP, VP, VP, VP, VP, VP]),
    "bfvgpu_keyswitch_prepared_words": (U64, [VP]),
    "bfvgpu_keyswitch_hoist_words": (U64, [VP, U64]),
    "bfvgpu_keyswitch_prepare_device": (I32, [VP, VP, U32P, U64, VP, VP]),
    "bfvgpu_keyswitch_hoist_device": (I32, [VP, VP, U64, VP, VP]),
    "bfvgpu_keyswitch_rotate_device": (I32, [VP, VP, U64, VP, VP, U32, VP, VP, VP]),
    "bfvgpu_weights_ntt_device": (I32, [VP, VP, U64, VP, VP]),
    "bfvgpu_matrix_groups_device": (I32, [VP, VP, U64, VP, U64, VP, VP, VP, VP]),
    "bfvgpu_ctx_check": (I32, [VP, U32P]),
    "bfvgpu_ctx_set_product_path": (I32, [VP, I32]),
    "bfvgpu_ctx_set_reserved_sms": (I32, [VP, I32]),
    "bfvgpu_matrix_tiles_inputs_device": (I32, [VP, VP, U64, VP, VP]),
    "bfvgpu_matrix_tiles_prepare_pk_device": (I32, [VP, VP, VP, VP]),
    "bfvgpu_matrix_tiles_scratch_words": (U64, [VP, U64, U64, I32]),
    "bfvgpu_matrix_tiles_device": (I32, [VP, VP, U64, U64, VP, U64, VP, VP, VP, VP, VP, VP]),
    "bfvgpu_enc0_device": (I32, [VP, VP, VP, U64, VP, VP, VP]),
    "bfvgpu_gather_targets_device": (I32, [VP, VP, U64, VP, VP, U32, VP, VP, VP]),
    "bfvgpu_ntt_open": (I32, [VP, I32, U64, ctypes.POINTER(VP)]),
    "bfvgpu_ntt_transform": (I32, [VP, U64P, U64P, I32]),
    "bfvgpu_ntt_bind_client_key": (I32, [VP, U64P]),
    "bfvgpu_ntt_client_phase": (I32, [VP, U64P, U64P]),
    "bfvgpu_ntt_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_ntt_release": (I32, [VP]),
    "bfvgpu_matrix_open": (I32, [VP, U64P, U64, ctypes.POINTER(VP)]),
    "bfvgpu_matrix_evaluate": (I32, [VP, U64P, U64P]),
    "bfvgpu_matrix_evaluate_selective": (I32, [VP, U64P, U64P, U64, U64P]),
    "bfvgpu_matrix_bind_public_key": (I32, [VP, U64P]),
    "bfvgpu_matrix_evaluate_groups": (I32, [VP, U64, U64P, U64P, U32P, U32, U64P, U64P, U64P, U64P, U64P]),
    "bfvgpu_matrix_device_bytes": (I32, [VP, U64P]),
    "bfvgpu_matrix_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_matrix_release": (I32, [VP]),
    "bfvgpu_switch_open": (I32, [VP, U64P, U32, ctypes.POINTER(VP)]),
    "bfvgpu_switch_apply": (I32, [VP, U64P, U64P]),
    "bfvgpu_switch_apply_many": (I32, [VP, U64P, U64, U64P]),
    "bfvgpu_rotations_open": (I32, [VP, U64P, U32P, U64, ctypes.POINTER(VP)]),
    "bfvgpu_rotations_apply": (I32, [VP, U64P, U64, U64P]),
    "bfvgpu_rotations_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_rotations_release": (I32, [VP]),
    "bfvgpu_matrix_tiles_protect_device": (I32, [VP, U64, U64, VP, VP, VP, VP, VP]),
    "bfvgpu_matrix_tiles_prepared_device": (I32, [VP, VP, U64, U64, VP, U64, I32, I32, VP, VP, VP, VP]),
    "bfvgpu_token_many_scratch_words": (U64, [VP, U64, U64]),
    "bfvgpu_token_evaluate_many_device": (I32, [VP, VP, U64, VP, U64, VP, VP, VP, VP]),
    "bfvgpu_packing_level_scratch_words": (U64, [VP, U64]),
    "bfvgpu_packing_level_device": (I32, [VP, VP, U64, U64, U32, VP, VP, VP, VP, VP]),
    "bfvgpu_encrypt_many_scratch_words": (U64, [VP, U64]),
    "bfvgpu_encrypt_many_device": (I32, [VP, VP, VP, VP, U64, VP, VP, VP]),
    "bfvgpu_slots_open": (I32, [VP, U64P, U32, U32, VP, ctypes.POINTER(VP)]),
    "bfvgpu_slots_apply_device": (I32, [VP, VP, VP, VP]),
    "bfvgpu_slots_apply": (I32, [VP, U64P, U64P]),
    "bfvgpu_slots_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_slots_release": (I32, [VP]),
    "bfvgpu_switch_packing_pair": (I32, [VP, U64P, U64P, VP, U32, U64P]),
    "bfvgpu_switch_timing": (I32, [VP, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                   ctypes.POINTER(ctypes.c_double)]),
    "bfvgpu_switch_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_switch_release": (I32, [VP]),
    "bfvgpu_enc0_open": (I32, [VP, U64P, ctypes.POINTER(VP)]),
    "bfvgpu_enc0_encrypt_from_samples": (I32, [VP, U64P, U64P]),
    "bfvgpu_enc0_encrypt_plain": (I32, [VP, U64P, U64P, U64, U64P]),
    "bfvgpu_enc0_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_enc0_release": (I32, [VP]),
    "bfvgpu_token_open": (I32, [VP, U64P, U64, ctypes.POINTER(VP)]),
    "bfvgpu_token_evaluate_finished": (I32, [VP, U64P, U64P, U64P]),
    "bfvgpu_token_close": (I32, [VP, ctypes.POINTER(Cleanup)]),
    "bfvgpu_token_release": (I32, [VP]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise BfvGpuUnavailable(
                f"{LIB_PATH} is not built; run `python privacy-rag_b200/build.py` (no CPU fallback exists)")
        try:
            L = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover - environment specific
            raise BfvGpuUnavailable(str(e)) from e
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class BfvGpuInvalidArgument(BfvGpuError, ValueError):
    """Validation failure before any device work (the reference's std::invalid_argument)."""


_VALIDATION = {1, 2, 3, 4, 5, 6, 7, 12, 13}


def check(rc: int, where: str) -> None:
    if rc != 0:
        detail = lib().bfvgpu_last_error().decode(errors="replace")
        cls = BfvGpuInvalidArgument if rc in _VALIDATION else BfvGpuError
        raise cls(rc, detail, where)


def ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(U64P)


def u64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint64))
