"""ctypes binding of oracle/_ref/libbolt_ref.so -- TEST INFRASTRUCTURE ONLY.

libbolt's own kernels (engine/bolt_kernels.cu compiled for sm_100a from where it lies, and engine/bolt_mma.cu from a
guarded build copy, by build_oracle.py --ref) behind oracle/ref_shim.cu.  The GPU tests run them on the same inputs as the CPU oracle to pin the oracle to the reference
itself, and tests/golden/make_golden.py records their outputs as fixtures.  All arguments are device pointers (ints).
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PATH = os.path.join(HERE, "_ref", "libbolt_ref.so")
_LIB = None


def available():
    return os.path.exists(PATH)


def lib():
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(PATH)
        vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
        sig = {
            "ref_topn": [],
            "ref_quant_rows": [vp, i32, vp, i32, vp, i32, i32, i32],
            "ref_route": [vp, i32, vp, vp, vp, i32, f32, i32],
            "ref_moe_group": [vp, i32, vp, vp, vp, vp, vp],
            "ref_repack_iq2": [vp, vp, vp, sz, i32],
            "ref_moe_up": [vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32],
            "ref_moe_down": [vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32],
            "ref_moe_coop_dense": [vp, vp, vp, vp, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32],
            "ref_combine": [vp, vp, vp, i32],
            "ref_gemv_iq2": [vp, vp, i32, i32, vp, i32, vp, i32, i32, i32],
            "ref_gemv_nv4": [vp, vp, f32, i32, i32, vp, i32, vp, i32, i32],
            "ref_gemv_q8": [vp, vp, i32, i32, vp, i32, vp, i32, i32],
            "ref_tile_nv4": [vp, vp, vp, vp, i32, i32],
            "ref_tile_q8": [vp, vp, vp, i32, i32],
            "ref_tile_iq2": [vp, vp, vp, i32, i32],
            "ref_mma_nv4": [vp, vp, f32, i32, i32, vp, i32, vp, i32, i32],
            "ref_mma_q8": [vp, vp, i32, i32, vp, i32, vp, i32, i32],
            "ref_mma_iq2": [vp, vp, i32, i32, vp, i32, vp, i32, i32, i32],
            "ref_quant_nv4_rows": [vp, i32, vp, vp, i32, i32],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = ctypes.c_int, args
        for name in ("ref_tile_bytes", "ref_tile_scale_bytes"):
            fn = getattr(L, name)
            fn.restype, fn.argtypes = sz, [i32, i32, i32]
        fn = L.ref_time_moe
        fn.restype = ctypes.c_float
        fn.argtypes = [i32, i32, i32, vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32]
        fn = L.ref_time_mma
        fn.restype = ctypes.c_float
        fn.argtypes = [i32, i32, i32, vp, vp, f32, i32, i32, vp, vp, i32]
        _LIB = L
    return _LIB


def call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name}: cudaError {rc}")
