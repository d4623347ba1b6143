"""numpy bindings of the CPU oracle (oracle.c) -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg; never by the product path.  Each function
restates a piece of the reference engine's arithmetic (the C source cites the reference lines).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            import build_oracle  # noqa: F401  (sibling module)
            path = build_oracle.build()
        _LIB = ctypes.CDLL(path)
        L = _LIB
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        sig = {
            "or_h2f": (f32, [ctypes.c_uint16]), "or_f2h": (ctypes.c_uint16, [f32]),
            "or_bf2f": (f32, [ctypes.c_uint16]), "or_f2bf": (ctypes.c_uint16, [f32]),
            "or_e4m3_dec": (f32, [ctypes.c_uint32]), "or_e4m3_enc": (ctypes.c_uint32, [f32]),
            "or_e2m1_enc": (ctypes.c_uint32, [f32]), "or_e2m1_dec": (f32, [ctypes.c_uint32]),
            "or_iq2_tables": (None, [vp, vp, vp, vp]),
            "or_iq2_dequant": (None, [vp, i64, i32, vp]),
            "or_iq2_gemm_exact": (None, [vp, i32, i32, vp, i32, vp, i32]),
            "or_quant_rows": (None, [vp, i64, i32, vp, vp]),
            "or_iq2_chunk_dots": (None, [vp, i32, i32, vp, i32, vp]),
            "or_iq2_gemm_i8": (None, [vp, i32, i32, vp, vp, i32, vp, i32]),
            "or_route_softmax": (None, [vp, i32, i32, i32, vp, vp]),
            "or_route_sigmoid": (None, [vp, i32, vp, i32, i32, i32, f32, vp, vp]),
            "or_group": (None, [vp, i32, i32, vp, vp, vp]),
            "or_combine": (None, [vp, vp, i32, i32, i32, vp]),
            "or_moe_layer": (None, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, f32, i32, vp, vp, vp]),
            "or_nv4_gemm_exact": (None, [vp, vp, f32, i32, i32, vp, i32, vp]),
            "or_quant_nv4_rows": (None, [vp, i32, i32, vp, vp]),
            "or_nv4_gemm_q4": (None, [vp, vp, f32, i32, i32, vp, vp, i32, vp]),
            "or_q8_gemm_exact": (None, [vp, i32, i32, vp, i32, vp]),
            "or_q8_gemm_f16fold": (None, [vp, i32, i32, vp, i32, vp]),
            "or_iq2_gemm_f16fold": (None, [vp, i32, i32, vp, i32, vp, i32]),
            "or_synth_iq2": (None, [ctypes.c_uint64, i64, vp]),
            "or_iq2_gemm_bf16fold": (None, [vp, i32, i32, vp, i32, vp, i32]),
            "or_set_threads": (None, [i32]), "or_max_threads": (i32, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def iq2_tables():
    grid = np.zeros(256, np.uint64)
    signs = np.zeros(128, np.uint8)
    signs64 = np.zeros(128, np.uint64)
    mask = np.zeros(8, np.uint8)
    lib().or_iq2_tables(_p(grid), _p(signs), _p(signs64), _p(mask))
    return grid, signs, signs64, mask


def iq2_dequant(blocks, rows, k):
    out = np.zeros((rows, k), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_iq2_dequant(_p(b), rows, k, _p(out))
    return out


def iq2_gemm_exact(blocks, n, k, x, epi=0):
    x = _c(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_iq2_gemm_exact(_p(b), n, k, _p(x), x.shape[0], _p(y), epi)
    return y


def quant_rows(x, k):
    x = _c(x, np.float32).reshape(-1, k)
    q = np.zeros(x.shape, np.int8)
    s = np.zeros((x.shape[0], k // 32), np.float32)
    lib().or_quant_rows(_p(x), x.shape[0], k, _p(q), _p(s))
    return q, s


def iq2_chunk_dots(blocks, n, k, xq):
    xq = _c(xq, np.int8).reshape(-1, k)
    d = np.zeros((xq.shape[0], n, k // 32), np.int32)
    b = _c(blocks, np.uint8)
    lib().or_iq2_chunk_dots(_p(b), n, k, _p(xq), xq.shape[0], _p(d))
    return d


def iq2_gemm_i8(blocks, n, k, xq, xs, epi=0):
    xq = _c(xq, np.int8).reshape(-1, k)
    xs = _c(xs, np.float32).reshape(-1, k // 32)
    y = np.zeros((xq.shape[0], n), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_iq2_gemm_i8(_p(b), n, k, _p(xq), _p(xs), xq.shape[0], _p(y), epi)
    return y


def route_softmax(logits, topk):
    lg = _c(logits, np.float32)
    T, E = lg.shape
    ridx = np.zeros((T, topk), np.int32)
    rw = np.zeros((T, topk), np.float32)
    lib().or_route_softmax(_p(lg), T, E, topk, _p(ridx), _p(rw))
    return ridx, rw


def route_sigmoid(logits, bias, topk, scale):
    lg = _c(logits, np.float32)
    T, E = lg.shape
    ridx = np.zeros((T, topk), np.int32)
    rw = np.zeros((T, topk), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    lib().or_route_sigmoid(_p(lg), E, _p(b), T, E, topk, float(scale), _p(ridx), _p(rw))
    return ridx, rw


def group(ridx, E):
    r = _c(ridx, np.int32).reshape(-1)
    counts = np.zeros(E, np.int32)
    offsets = np.zeros(E + 1, np.int32)
    order = np.zeros(r.size, np.int32)
    lib().or_group(_p(r), r.size, E, _p(counts), _p(offsets), _p(order))
    return counts, offsets, order


def combine(mo, rw, topk, H):
    mo = _c(mo, np.float32)
    rw = _c(rw, np.float32)
    T = rw.size // topk
    out = np.zeros((T, H), np.float32)
    lib().or_combine(_p(mo), _p(rw), T, topk, H, _p(out))
    return out


def moe_layer(x_bf16, logits_bf16, up, down, sh_up, sh_down, T, H, F, E, topk, route=0, bias=None, scale=1.0, mode=0):
    """x_bf16 / logits_bf16: uint16 bit arrays; up/down: the experts' ggml blocks back to back."""
    x = _c(x_bf16, np.uint16)
    lg = _c(logits_bf16, np.uint16)
    up, down = _c(up, np.uint8), _c(down, np.uint8)
    su = None if sh_up is None else _c(sh_up, np.uint8)
    sd = None if sh_down is None else _c(sh_down, np.uint8)
    b = None if bias is None else _c(bias, np.float32)
    out = np.zeros((T, H), np.float32)
    ridx = np.zeros((T, topk), np.int32)
    rw = np.zeros((T, topk), np.float32)
    lib().or_moe_layer(_p(x), _p(lg), _p(up), _p(down), _p(su), _p(sd), T, H, F, E, topk, route, _p(b), float(scale), mode,
                       _p(out), _p(ridx), _p(rw))
    return out, ridx, rw


def nv4_gemm_exact(q, sc, s2, n, k, x):
    x = _c(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    q, sc = _c(q, np.uint8), _c(sc, np.uint8)
    lib().or_nv4_gemm_exact(_p(q), _p(sc), float(s2), n, k, _p(x), x.shape[0], _p(y))
    return y


def quant_nv4_rows(x, k):
    x = _c(x, np.float32).reshape(-1, k)
    q4 = np.zeros((x.shape[0], k // 2), np.uint8)
    sf = np.zeros((x.shape[0], k // 16), np.uint8)
    lib().or_quant_nv4_rows(_p(x), x.shape[0], k, _p(q4), _p(sf))
    return q4, sf


def nv4_gemm_q4(q, sc, s2, n, k, q4, sf):
    q, sc, q4, sf = _c(q, np.uint8), _c(sc, np.uint8), _c(q4, np.uint8), _c(sf, np.uint8)
    T = q4.size // (k // 2)
    y = np.zeros((T, n), np.float32)
    lib().or_nv4_gemm_q4(_p(q), _p(sc), float(s2), n, k, _p(q4), _p(sf), T, _p(y))
    return y


def q8_gemm_exact(blocks, n, k, x):
    x = _c(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_q8_gemm_exact(_p(b), n, k, _p(x), x.shape[0], _p(y))
    return y


def q8_gemm_f16fold(blocks, n, k, x):
    x = _c(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_q8_gemm_f16fold(_p(b), n, k, _p(x), x.shape[0], _p(y))
    return y


def iq2_gemm_f16fold(blocks, n, k, x, epi=0):
    x = _c(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_iq2_gemm_f16fold(_p(b), n, k, _p(x), x.shape[0], _p(y), epi)
    return y


def iq2_gemm_bf16fold(blocks, n, k, x, epi=0):
    """libbolt's mma_iq2 arithmetic (PIQ2): bf16(bf16(dA) x signed grid) weights; x as given (round it to bf16)"""
    x = _c(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    b = _c(blocks, np.uint8)
    lib().or_iq2_gemm_bf16fold(_p(b), n, k, _p(x), x.shape[0], _p(y), epi)
    return y


def synth_iq2(seed, nblocks):
    """BASELINE's seeded IQ2_XXS blocks [nblocks][66] (the same bytes as the library's generator for the seed)"""
    out = np.empty((nblocks, 66), np.uint8)
    lib().or_synth_iq2(seed, nblocks, _p(out))
    return out


def set_threads(n):
    """the OpenMP threads of the oracle's loops (1: single-thread)"""
    lib().or_set_threads(int(n))


def scalar(name, *args):
    return getattr(lib(), name)(*args)
