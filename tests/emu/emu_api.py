"""ctypes signatures of tests/emu/libemu.so (TEST INFRASTRUCTURE)."""
import ctypes

P = ctypes.POINTER(ctypes.c_uint64)
U64, U32, INT = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int

SIGNATURES = {
    "emu_ntt": [INT, U32, P, P, P, P, U64, U32, U32, INT],
    "emu_ntt_pair": [INT, U32, P, P, P, P, U64, U32, U32, INT],
    "emu_keyswitch": [INT, U32, U32, P, P, P, P, U64, P, U32, P],
    "emu_keyswitch_hoisted": [INT, U32, U32, P, P, P, P, U64, P, U32, P, ctypes.POINTER(ctypes.c_uint32)],
    "emu_keyswitch_pipe": [INT, U32, U32, P, P, P, P, U64, P, ctypes.POINTER(ctypes.c_uint32), U64, P],
    "emu_matrix": [INT, U32, U32, P, P, P, P, U64, P, U64, P, P, P, U64, U64, U64, INT, P],
    "emu_matrix_tiles": [INT, U32, U32, P, P, P, P, U64, U64, P, U64, P, P, P, U64, U64, U64, INT, P, INT],
    "emu_client_phase": [INT, U32, U32, P, P, P, P, P, U64],
    "emu_crt": [U32, U32, P, P, U64, P, P, P, P],
    "emu_token": [U32, U32, P, P, P, P, U64, P, P, P],
    "emu_f64_mulmod": [P, P, U64, U64, P, P, P],
    "emu_f64_convert": [P, U64, P],
    "emu_f64_mulmod_barrett": [P, P, U64, U64, P],
}


def bind(lib):
    for name, args in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = INT
        f.argtypes = args
    return lib


def p(a):
    return None if a is None else a.ctypes.data_as(P)
