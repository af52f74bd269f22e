"""bfvgpu: B200 (sm_100a) BFV ciphertext arithmetic behind privacy-rag's matrix protocol.

Host-side mirror of the reference's GPU backend classes and matrix-protocol engine over
the C ABI in include/bfvgpu.h (libbfvgpu.so, built in-tree by privacy-rag_b200/build.py).
"""
from ._lib import (EXPORTED, LIB_PATH, BfvGpuError, BfvGpuInvalidArgument, BfvGpuUnavailable,  # noqa: F401
                   lib)
from .backend import (ART002_PRIMES, Context, Matrix, NttBatch, PublicZero, Rotations, SlotMatvec, Switch,  # noqa: F401
                      TokenWeights, find_primes, launch_count)
from .layout import (MatrixPacking, matrix_packing, matrix_packing_qk_reverse64,  # noqa: F401
                     pack_inputs, pack_weights, packed_bfv_rows_per_ciphertext, targets)
from . import engine  # noqa: F401,E402
