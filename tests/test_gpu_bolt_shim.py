"""libbolt's operator launchers (include/b200q_bolt.h: libbolt's own names, signatures and view structs, backed by
libb200q) fed the inputs of the golden fixtures, which hold the outputs of libbolt's own kernels run on a B200: the
shims, called the way libbolt's host code calls its launchers, give libbolt's outputs (bit for bit where the kernel
keeps libbolt's chunk order; the router's weights within 2e-6, its picks exact)."""
import ctypes
import os

import numpy as np
import pytest
import torch

import b200q
from helpers import iq2_blocks

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
DEV = "cuda"
_KEEP = []


def _harness():
    import build_harness
    L = ctypes.CDLL(build_harness.build())
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    sig = {
        "hs_repack_iq2": [vp, vp, vp, vp, sz, i32],
        "hs_k_route": [vp, vp, i32, vp, vp, vp, i32, f32, i32],
        "hs_k_moe_group": [vp, vp, i32, vp, vp, vp, vp, vp],
        "hs_k_quant_rows": [vp, vp, i32, vp, i32, vp, i32, i32, i32],
        "hs_moe_up": [vp, vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32],
        "hs_moe_down": [vp, vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32],
        "hs_moe_coop_dense": [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32],
        "hs_k_combine": [vp, vp, vp, vp, i32],
    }
    for n, a in sig.items():
        getattr(L, n).restype, getattr(L, n).argtypes = None, a
    return L


def golden(name):
    z = np.load(os.path.join(HERE, "golden", f"ref_{name}.npz"))
    return ({k[3:]: z[k] for k in z.files if k.startswith("in_")}, {k[4:]: z[k] for k in z.files if k.startswith("out_")})


def d(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    _KEEP.append(t)
    return t


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def slab(L, blocks, rows, k):
    """the qs / d buffers libbolt's load_slab allocates (rows * k/256 * 64 and * 2 bytes), packed by the shim"""
    qs = torch.empty(rows * (k // 256) * 64, dtype=torch.uint8, device=DEV)
    dd = torch.empty(rows * (k // 256), dtype=torch.float16, device=DEV)
    L.hs_repack_iq2(s(), p(d(blocks.reshape(-1))), p(qs), p(dd), rows, k)
    _KEEP.extend([qs, dd])
    return qs, dd


def test_shim_exports_libbolt_signatures():
    L = _harness()
    assert L.hs_moe_up is not None


def test_shim_router_and_quant_rows_match_libbolt():
    L = _harness()
    i, o = golden("route")
    T, E = i["logits"].shape
    ridx = torch.empty(T * 9, dtype=torch.int32, device=DEV)
    rw = torch.empty(T * 9, dtype=torch.float32, device=DEV)
    L.hs_k_route(s(), p(d(i["logits"])), E, p(d(i["bias"])), p(ridx), p(rw), E, float(i["scale"]), T)
    assert np.array_equal(ridx.cpu().numpy().reshape(T, 9), o["ridx"])
    assert np.allclose(rw.cpu().numpy().reshape(T, 9), o["rw"], rtol=2e-6)
    i, o = golden("quant_rows")
    q = torch.empty(8, 256, dtype=torch.int8, device=DEV)
    sc = torch.empty(8, 8, dtype=torch.float32, device=DEV)
    L.hs_k_quant_rows(s(), p(d(i["x"])), 256, p(q), 256, p(sc), 8, 8, 256)
    assert np.array_equal(q.cpu().numpy(), o["q"]) and np.array_equal(sc.cpu().numpy(), o["s"])


def test_shim_moe_block_matches_libbolt():
    """repack_iq2 into libbolt's buffers, k_moe_group, moe_up, moe_down at libbolt's routed shapes (k 1024 up,
    n 1024 down, 9 experts a token), against libbolt's own act and mo"""
    L = _harness()
    i, o = golden("moe_up_down")
    E, W, H = int(i["E"]), int(i["W"]), int(i["H"])
    pairs = len(i["ridx"])
    uqs, ud = slab(L, iq2_blocks(int(i["up_seed"]), E * W, H), E * W, H)
    dqs, dd = slab(L, iq2_blocks(int(i["down_seed"]), E * H, W), E * H, W)
    cap = 2048 * 9   # libbolt's work arrays: TMAX * TOPN entries
    order, first, count, exp = (torch.zeros(cap, dtype=torch.int32, device=DEV) for _ in range(4))
    nwork = torch.zeros(1, dtype=torch.int32, device=DEV)
    ridx = d(i["ridx"].astype(np.int32))
    L.hs_k_moe_group(s(), p(ridx), pairs, p(order), p(first), p(count), p(exp), p(nwork))
    act = torch.full((pairs, W), -1.0, device=DEV)
    L.hs_moe_up(s(), p(uqs), p(ud), W * (H // 256) * 64, W * (H // 256), p(order), p(first), p(count), p(exp), p(nwork),
                p(d(i["xq"])), p(d(i["xs"])), p(act), W, pairs)
    assert np.array_equal(act.cpu().numpy(), o["act"])
    mo = torch.full((pairs, H), -1.0, device=DEV)
    L.hs_moe_down(s(), p(dqs), p(dd), H * (W // 256) * 64, H * (W // 256), p(order), p(first), p(count), p(exp),
                  p(nwork), p(d(i["aq"])), p(d(i["as"])), p(mo), W, pairs)
    assert np.array_equal(mo.cpu().numpy(), o["mo"])
    assert b200q.device_error() == 0


def test_shim_coop_dense_and_combine_match_libbolt():
    L = _harness()
    i, o = golden("coop_dense")
    n, k = int(i["n"]), int(i["k"])
    qs, dd = slab(L, iq2_blocks(int(i["seed"]), n, k), n, k)
    T = i["xq"].shape[0]
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_moe_coop_dense(s(), p(qs), p(dd), T, p(d(i["xq"])), p(d(i["xs"])), p(y), n, n, k, 1)
    assert np.array_equal(y.cpu().numpy(), o["y"])
    i, o = golden("combine")
    T = o["out"].shape[0]
    out = torch.empty(T, 1024, device=DEV)
    L.hs_k_combine(s(), p(d(i["o"])), p(d(i["rw"])), p(out), T)
    assert np.array_equal(out.cpu().numpy(), o["out"])
