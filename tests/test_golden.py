"""The CPU oracle against the committed golden fixtures: outputs of libbolt's own kernels run on a B200
(tests/golden/make_golden.py wrote them).  Same bar as tests/test_gpu_ref.py, on any machine."""
import glob
import os

import numpy as np
import pytest

import oracle as O
from helpers import iq2_blocks

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    path = os.path.join(GOLD, f"ref_{name}.npz")
    if not os.path.exists(path):
        pytest.skip(f"fixture {path} not generated yet")
    z = np.load(path)
    return ({k[3:]: z[k] for k in z.files if k.startswith("in_")}, {k[4:]: z[k] for k in z.files if k.startswith("out_")})


def test_fixtures_present():
    assert len(glob.glob(os.path.join(GOLD, "ref_*.npz"))) >= 8


def test_quant_rows():
    i, o = load("quant_rows")
    q, s = O.quant_rows(i["x"], 256)
    assert np.array_equal(q, o["q"]) and np.array_equal(s, o["s"])


def test_route_sigmoid():
    i, o = load("route")
    ridx, rw = O.route_sigmoid(i["logits"], i["bias"], int(i["topn"]), float(i["scale"]))
    assert np.array_equal(ridx, o["ridx"]) and np.allclose(rw, o["rw"], rtol=2e-6)


def test_coop_dense_int8():
    i, o = load("coop_dense")
    n, k = int(i["n"]), int(i["k"])
    assert np.array_equal(O.iq2_gemm_i8(iq2_blocks(int(i["seed"]), n, k), n, k, i["xq"], i["xs"], 1), o["y"])


def test_moe_up_down_int8():
    i, o = load("moe_up_down")
    E, W, H = int(i["E"]), int(i["W"]), int(i["H"])
    topn = len(i["ridx"]) // i["xq"].shape[0]
    up = iq2_blocks(int(i["up_seed"]), E * W, H).reshape(E, -1)
    down = iq2_blocks(int(i["down_seed"]), E * H, W).reshape(E, -1)
    for p, e in enumerate(i["ridx"]):
        assert np.array_equal(O.iq2_gemm_i8(up[e], W, H, i["xq"][p // topn], i["xs"][p // topn], 1)[0], o["act"][p])
        assert np.array_equal(O.iq2_gemm_i8(down[e], H, W, i["aq"][p], i["as"][p], 0)[0], o["mo"][p])


def test_combine():
    i, o = load("combine")
    assert np.array_equal(O.combine(i["o"], i["rw"], int(i["topn"]), 1024), o["out"])


def test_gemv_fp32():
    i, o = load("gemv_iq2")
    n, k = int(i["n"]), int(i["k"])
    y = O.iq2_gemm_exact(iq2_blocks(int(i["seed"]), n, k), n, k, i["x"])
    assert np.allclose(y, o["y"], rtol=1e-5, atol=1e-5 * np.abs(y).max())
    i, o = load("gemv_nv4")
    y = O.nv4_gemm_exact(i["q"], i["sc"], float(i["s2"]), 64, 256, i["x"])
    assert np.allclose(y, o["y"], rtol=1e-5, atol=1e-5 * np.abs(y).max())
    i, o = load("gemv_q8")
    blocks = np.concatenate([i["d"].view(np.uint8).reshape(64, 8, 2), i["q"].view(np.uint8).reshape(64, 8, 32)], -1)
    y = O.q8_gemm_exact(blocks.reshape(64, -1), 64, 256, i["x"])
    assert np.allclose(y, o["y"], rtol=1e-5, atol=1e-5 * np.abs(y).max())


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def test_mma_nv4_fold():
    """libbolt's mma_nv4 (PNV4): fp16 rows, exact e2m1 x e4m3 operands: the oracle on fp16-rounded rows, 1e-5"""
    i, o = load("mma_nv4")
    n, k = o["y"].shape[1], i["x"].shape[1]
    y = O.nv4_gemm_exact(i["q"], i["sc"], float(i["s2"]), n, k, f16(i["x"]))
    assert np.allclose(o["y"], y, rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_mma_q8_fold():
    """libbolt's mma_q8 (PQ8): fp16 rows, weights fp16(i8 d): the oracle's fp16 fold on fp16-rounded rows, 1e-5"""
    i, o = load("mma_q8")
    n, k = o["y"].shape[1], i["x"].shape[1]
    y = O.q8_gemm_f16fold(i["blocks"], n, k, f16(i["x"]))
    assert np.allclose(o["y"], y, rtol=1e-5, atol=1e-5 * np.abs(y).max())


def test_mma_iq2_bf16_fold():
    """libbolt's mma_iq2 (PIQ2): bf16 rows, weights bf16(bf16(dA) x grid): or_iq2_gemm_bf16fold, 1e-5"""
    i, o = load("mma_iq2")
    n, k = int(i["n"]), int(i["k"])
    blocks = iq2_blocks(int(i["seed"]), n, k)
    for epi in (0, 1):
        y = O.iq2_gemm_bf16fold(blocks, n, k, bf16(i["x"]), epi)
        assert np.allclose(o[f"y{epi}"], y, rtol=1e-5, atol=1e-5 * np.abs(y).max()), epi


def test_quant_nv4_rows_bytes():
    """libbolt's NVFP4 row quantiser (quant_nv4_rows_k): the oracle's codes and scales, byte for byte"""
    i, o = load("quant_nv4_rows")
    q4, sf = O.quant_nv4_rows(i["x"], i["x"].shape[1])
    assert np.array_equal(q4, o["q4"]) and np.array_equal(sf, o["sf"])
