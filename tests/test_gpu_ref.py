"""The CPU oracle against libbolt's own kernels run on the B200 (oracle/_ref/libbolt_ref.so, built from the reference's
engine/bolt_kernels.cu).  Where the reference kernel keeps a per-output chunk order (quant_rows, the int8-per-32
expert kernels, combine) the oracle must agree bit for bit; the fp32 GEMVs sum in a lane-split order, so within 1e-5."""
import numpy as np
import pytest

import oracle as O
import refbind as R
from helpers import iq2_blocks

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason="oracle/_ref/libbolt_ref.so not built")]

import sys, os  # noqa: E402
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
import make_golden as G  # noqa: E402


def test_quant_rows():
    i, o = G.case_quant_rows()
    q, s = O.quant_rows(i["x"], 256)
    assert np.array_equal(q, o["q"]) and np.array_equal(s, o["s"])


def test_route_sigmoid():
    i, o = G.case_route()
    ridx, rw = O.route_sigmoid(i["logits"], i["bias"], int(i["topn"]), float(i["scale"]))
    assert np.array_equal(ridx, o["ridx"])
    assert np.allclose(rw, o["rw"], rtol=2e-6)


def test_coop_dense_int8():
    i, o = G.case_coop_dense()
    n, k = int(i["n"]), int(i["k"])
    y = O.iq2_gemm_i8(iq2_blocks(int(i["seed"]), n, k), n, k, i["xq"], i["xs"], 1)
    assert np.array_equal(y, o["y"])


def test_moe_up_down_int8():
    i, o = G.case_moe_up_down()
    E, W, H = int(i["E"]), int(i["W"]), int(i["H"])
    topn = len(i["ridx"]) // i["xq"].shape[0]
    up = iq2_blocks(int(i["up_seed"]), E * W, H).reshape(E, -1)
    down = iq2_blocks(int(i["down_seed"]), E * H, W).reshape(E, -1)
    for p, e in enumerate(i["ridx"]):
        a = O.iq2_gemm_i8(up[e], W, H, i["xq"][p // topn], i["xs"][p // topn], 1)[0]
        assert np.array_equal(a, o["act"][p])
        m = O.iq2_gemm_i8(down[e], H, W, i["aq"][p], i["as"][p], 0)[0]
        assert np.array_equal(m, o["mo"][p])


def test_combine():
    i, o = G.case_combine()
    assert np.array_equal(O.combine(i["o"], i["rw"], int(i["topn"]), 1024), o["out"])


def test_gemv_iq2_fp32():
    i, o = G.case_gemv_iq2()
    n, k = int(i["n"]), int(i["k"])
    y = O.iq2_gemm_exact(iq2_blocks(int(i["seed"]), n, k), n, k, i["x"])
    assert np.allclose(y, o["y"], rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_gemv_nv4_fp32():
    i, o = G.case_gemv_nv4()
    y = O.nv4_gemm_exact(i["q"], i["sc"], float(i["s2"]), 64, 256, i["x"])
    assert np.allclose(y, o["y"], rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_gemv_q8_fp32():
    i, o = G.case_gemv_q8()
    blocks = np.concatenate([i["d"].view(np.uint8).reshape(64, 8, 2), i["q"].view(np.uint8).reshape(64, 8, 32)], -1)
    y = O.q8_gemm_exact(blocks.reshape(64, -1), 64, 256, i["x"])
    assert np.allclose(y, o["y"], rtol=1e-5, atol=1e-5 * np.abs(y).max())


# ---- bolt_mma.cu, live: the oracle against libbolt's tile GEMMs and row quantiser, and this engine's libbolt-signature
# shims (libb200q through the shim harness) against the same libbolt calls on the same inputs
def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def test_mma_nv4_live():
    i, o = G.case_mma_nv4()
    n, k = o["y"].shape[1], i["x"].shape[1]
    y = O.nv4_gemm_exact(i["q"], i["sc"], float(i["s2"]), n, k, _f16(i["x"]))
    assert np.allclose(o["y"], y, rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_mma_q8_live():
    i, o = G.case_mma_q8()
    n, k = o["y"].shape[1], i["x"].shape[1]
    y = O.q8_gemm_f16fold(i["blocks"], n, k, _f16(i["x"]))
    assert np.allclose(o["y"], y, rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_mma_iq2_live():
    i, o = G.case_mma_iq2()
    n, k = int(i["n"]), int(i["k"])
    blocks = iq2_blocks(int(i["seed"]), n, k)
    for epi in (0, 1):
        y = O.iq2_gemm_bf16fold(blocks, n, k, _bf16(i["x"]), epi)
        assert np.allclose(o[f"y{epi}"], y, rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_quant_nv4_rows_live():
    i, o = G.case_quant_nv4_rows()
    q4, sf = O.quant_nv4_rows(i["x"], i["x"].shape[1])
    assert np.array_equal(q4, o["q4"]) and np.array_equal(sf, o["sf"])


def test_engine_shims_against_libbolt_mma():
    """libbolt's mma_nv4 / mma_q8 / mma_iq2 and this engine's shims of the same names on the same inputs: the NVFP4
    shim rounds the rows to fp16 as libbolt does and both products are exact (within 1e-5); the Q8_0 shim does not
    round the weights to fp16 as libbolt's PQ8 does (exact within 1e-5, libbolt within BASELINE's tolerance); the IQ2
    shim runs the int8-per-32 arithmetic of libbolt's moe_coop_dense where libbolt's mma_iq2 folds into bf16
    (BASELINE's tolerance)"""
    import torch
    import build_harness
    import ctypes
    from helpers import assert_tolerance
    H = ctypes.CDLL(build_harness.build())
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    H.hs_tile_bytes.restype, H.hs_tile_bytes.argtypes = ctypes.c_size_t, [i32, i32, i32, i32]
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def tiles(fmt, n, k):
        return (torch.empty(H.hs_tile_bytes(fmt, 0, n, k), dtype=torch.uint8, device="cuda"),
                torch.empty(H.hs_tile_bytes(fmt, 1, n, k), dtype=torch.uint8, device="cuda"))

    i, o = G.case_mma_nv4()
    n, k, T = o["y"].shape[1], i["x"].shape[1], i["x"].shape[0]
    qt, st = tiles(0, n, k)
    H.hs_tile_nv4(s, p(dev(i["q"])), p(dev(i["sc"])), p(qt), p(st), n, k)
    y = torch.zeros(T, n, device="cuda")
    H.hs_mma_nv4(s, p(qt), p(st), f32(float(i["s2"])), n, k, p(dev(i["x"])), k, p(y), n, T)
    torch.cuda.synchronize()
    assert np.allclose(y.cpu().numpy(), o["y"], rtol=1e-5, atol=1e-5 * np.abs(o["y"]).max())

    # libbolt's PQ8 rounds every weight to fp16(i8 d); the engine keeps i8 x fp16(row) exact and applies d in fp32:
    # within 1e-5 of the exact product, and within BASELINE's tolerance of libbolt's rounded one
    i, o = G.case_mma_q8()
    n, k, T = o["y"].shape[1], i["x"].shape[1], i["x"].shape[0]
    qt, st = tiles(1, n, k)
    H.hs_tile_q8(s, p(dev(i["blocks"])), p(qt), p(st), n, k)
    y = torch.zeros(T, n, device="cuda")
    H.hs_mma_q8(s, p(qt), p(st), n, k, p(dev(i["x"])), k, p(y), n, T)
    torch.cuda.synchronize()
    yq = y.cpu().numpy()
    exact = O.q8_gemm_exact(i["blocks"], n, k, _f16(i["x"]))
    assert np.allclose(yq, exact, rtol=1e-5, atol=1e-5 * np.abs(exact).max())
    assert_tolerance(yq, o["y"])

    i, o = G.case_mma_iq2()
    n, k = int(i["n"]), int(i["k"])
    T = i["x"].shape[0]
    qt, st = tiles(2, n, k)
    H.hs_tile_iq2(s, p(dev(iq2_blocks(int(i["seed"]), n, k).reshape(-1))), p(qt), p(st), n, k)
    for epi in (0, 1):
        y = torch.zeros(T, n, device="cuda")
        H.hs_mma_iq2(s, p(qt), p(st), n, k, p(dev(i["x"])), k, p(y), n, T, epi)
        torch.cuda.synchronize()
        assert_tolerance(y.cpu().numpy(), o[f"y{epi}"])
