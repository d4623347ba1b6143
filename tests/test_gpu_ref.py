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
