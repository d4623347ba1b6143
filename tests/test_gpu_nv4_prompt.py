"""GPU parity of the NVFP4 prompt path (quant_nv4_rows + the block-scaled fp4 tcgen05 GEMM) against the CPU oracle,
through the C ABI.

The row quantiser is integer/byte work: its tile image must equal, byte for byte, the oracle's codes
(or_quant_nv4_rows, the steps of quant_nv4_rows_k) laid out as stated below.  The GEMM's products (e2m1 x e2m1 x
e4m3 x e4m3) are exact and only the fp32 summation differs from the oracle's fp64 sums (or_nv4_gemm_q4): bar relative
L2 1e-5.  Against the unquantised activations (exact mode) the fp4 rounding of x itself dominates (a few percent, the
reference's own prompt arithmetic); that comparison is reported with a 0.1 bound."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def nv4_weights(seed, n, k):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sc = torch.from_numpy(rng.uniform(0.5, 2.0, (n, k // 16)).astype(np.float32)).to(torch.float8_e4m3fn)
    return q, sc.view(torch.uint8).numpy()


def sw128(r, c):
    """byte offset of 16-byte chunk c of row r in a 128-byte-swizzled K-major tile"""
    return r * 128 + ((c ^ (r & 7)) << 4)


def sf_off(r, j, groups):
    """offset of the scale of (row r, 16-k block j of a 256-k stage) in a record's scale part"""
    kb, s, h, rr = j >> 2, j & 3, r >> 7, r & 127
    return (kb * groups + h) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + s


def np_image(q, sc, rows, k, tile_rows):
    """numpy statement of the fp4 tile image (nv4_gemm.cu): records (tile, 256-k step) of tile_rows x 128 B of
    swizzled e2m1 bytes followed by tile_rows / 128 x 4 scale atoms of 512 B; rows past `rows` are zero."""
    groups = tile_rows // 128
    data = tile_rows * 128
    rec = data + groups * 4 * 512
    nt, ks = -(-rows // tile_rows), k // 256
    out = np.zeros((nt, ks, rec), np.uint8)
    r = np.arange(tile_rows)
    for t in range(nt):
        for s in range(ks):
            for row in range(tile_rows):
                g = t * tile_rows + row
                if g >= rows:
                    break
                for c in range(8):
                    o = sw128(row, c)
                    out[t, s, o:o + 16] = q[g, s * 128 + c * 16: s * 128 + c * 16 + 16]
                for j in range(16):
                    out[t, s, data + sf_off(row, j, groups)] = sc[g, s * 16 + j]
    del r
    return out.reshape(-1)


@pytest.mark.parametrize("n,k", [(256, 256), (300, 512)])
def test_nv4_tc_pack_layout(n, k):
    q, sc = nv4_weights(n * 7 + k, n, k)
    img = b200q.tile_nv4w(dev(q), dev(sc), n, k).cpu().numpy()
    assert img.size == b200q.lib().b200q_nv4_tc_bytes(n, k)
    assert np.array_equal(img, np_image(q, sc, n, k, 256))


def rows_input(seed, T, k):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, k)).astype(np.float32)
    blocks = x.reshape(T, k // 16, 16)
    # per-block magnitudes over a wide range: zeros, e4m3 subnormal scales, ordinary, saturating (amax / 6 >= 448)
    mag = rng.choice(np.array([0.0, 1e-4, 3e-3, 0.05, 1.0, 30.0, 5000.0], np.float32), size=(T, k // 16, 1))
    return (blocks * mag).reshape(T, k)


@pytest.mark.parametrize("T,k,dt", [(1, 256, "f32"), (130, 512, "f32"), (77, 1024, "bf16")])
def test_quant_nv4_rows_bitexact(T, k, dt):
    x = rows_input(T + k, T, k)
    if dt == "bf16":
        xt = dev(x).to(torch.bfloat16)
        x = xt.float().cpu().numpy()
    else:
        xt = dev(x)
    img = b200q.quant_nv4_rows(xt).cpu().numpy()
    q4, sf = O.quant_nv4_rows(x, k)
    assert img.size == b200q.lib().b200q_nv4_rows_bytes(T, k)
    assert np.array_equal(img, np_image(q4, sf, T, k, 128))


@pytest.mark.parametrize("T,n,k", [(1, 256, 256), (130, 384, 512), (300, 520, 1024), (512, 1024, 4096)])
def test_nv4_prompt_gemm(T, n, k):
    q, sc = nv4_weights(n + 3 * T + k, n, k)
    s2 = 0.0123
    rng = np.random.default_rng(T * 5 + n)
    x = rng.standard_normal((T, k)).astype(np.float32)
    w = b200q.tile_nv4w(dev(q), dev(sc), n, k)
    rows = b200q.quant_nv4_rows(dev(x))
    y = b200q.mma_nv4_fp4(w, s2, n, k, rows, T).cpu().numpy()
    assert b200q.device_error() == 0
    q4, sf = O.quant_nv4_rows(x, k)
    ref = O.nv4_gemm_q4(q, sc, s2, n, k, q4, sf)
    assert rel_l2(y, ref) < 1e-5
    assert rel_l2(y, O.nv4_gemm_exact(q, sc, s2, n, k, x)) < 0.1


def test_nv4_prompt_gemm_ldy_and_repeat():
    """an output wider than n (ldy > n) and two calls in a row give the same bytes"""
    T, n, k = 200, 640, 512
    q, sc = nv4_weights(5, n, k)
    x = np.random.default_rng(6).standard_normal((T, k)).astype(np.float32)
    w = b200q.tile_nv4w(dev(q), dev(sc), n, k)
    rows = b200q.quant_nv4_rows(dev(x))
    big = torch.full((T, n + 36), 7.0, device=DEV)
    b200q.mma_nv4_fp4(w, 1.0, n, k, rows, T, y=big)
    first = big.clone()
    b200q.mma_nv4_fp4(w, 1.0, n, k, rows, T, y=big)
    assert torch.equal(first, big)
    assert torch.all(big[:, n:] == 7.0)
    q4, sf = O.quant_nv4_rows(x, k)
    assert rel_l2(big[:, :n].cpu().numpy(), O.nv4_gemm_q4(q, sc, 1.0, n, k, q4, sf)) < 1e-5


def test_nv4_prompt_gemm_split_k():
    """a launch with few tiles cuts K into slices (partials in the workspace, added in slice order): the same sums as
    the oracle's, and as the unsplit launch up to fp32 reassociation"""
    T, n, k = 130, 512, 2048   # 2 x 2 tiles: 4 slices of K
    q, sc = nv4_weights(11, n, k)
    x = np.random.default_rng(12).standard_normal((T, k)).astype(np.float32)
    w = b200q.tile_nv4w(dev(q), dev(sc), n, k)
    rows = b200q.quant_nv4_rows(dev(x))
    assert b200q.lib().b200q_nv4_gemm_workspace_bytes(n, k, T) == 4 * T * n * 4
    y = b200q.mma_nv4_fp4(w, 0.5, n, k, rows, T)
    y1 = torch.empty_like(y)
    st = b200q.lib().b200q_nv4_gemm(b200q._p(w), n, k, 0.5, b200q._p(rows), T, b200q._p(y1), n, None, 0, b200q._s())
    assert st == 0
    y, y1 = y.cpu().numpy(), y1.cpu().numpy()
    assert b200q.device_error() == 0
    q4, sf = O.quant_nv4_rows(x, k)
    ref = O.nv4_gemm_q4(q, sc, 0.5, n, k, q4, sf)
    assert rel_l2(y, ref) < 1e-5 and rel_l2(y1, ref) < 1e-5
    assert rel_l2(y, y1) < 1e-6
