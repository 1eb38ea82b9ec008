"""ctypes signatures of every function declared in include/metalgym_b200.h.

tests/test_abi.py checks that this table and the header declare the same set
of functions and that the built library exports all of them.
"""
import ctypes as C

P = C.c_void_p
I = C.c_int
U = C.c_uint32
F = C.c_float
U64 = C.c_uint64
S = C.c_char_p
PI = C.POINTER(C.c_int)
PF = C.POINTER(C.c_float)

SIGNATURES = {
    # runtime
    "mg_last_error": (S, []),
    "mg_version": (I, []),
    "mg_device_status": (I, [I, PI]),
    # GEMM
    "mg_gemm_bf16": (I, [P, I, I, P, I, I, I, I, I, I, P, I, P, I, I, P]),
}
