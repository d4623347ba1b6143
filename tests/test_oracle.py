"""CPU tests of the oracle: known-answer checks derived from the reference's sources (the reference ships no golden
vectors for this path), and cross-checks of the C restatement against independent numpy restatements."""
import numpy as np
import pytest
import torch

import oracle as O
from helpers import iq2_blocks, normal_bf16, rel_l2


def popcount(i):
    return bin(i).count("1")


def test_ksigns_is_index_with_parity_bit():
    # bolt_kernels.cu:124 and bolt_mma.cu:320 compute ksigns_iq2xs[i] as i | parity(i) << 7
    _, signs, _, _ = O.iq2_tables()
    for i in range(128):
        assert signs[i] == (i | ((popcount(i) & 1) << 7))


def test_ksigns64_byte_masks():
    _, signs, signs64, _ = O.iq2_tables()
    for i in range(128):
        for j in range(8):
            byte = (int(signs64[i]) >> (8 * j)) & 255
            assert byte == (255 if (signs[i] >> j) & 1 else 0)


def test_kmask():
    _, _, _, mask = O.iq2_tables()
    assert list(mask) == [1 << j for j in range(8)]


def test_grid_magnitudes_and_distinct():
    grid, _, _, _ = O.iq2_tables()
    assert len(set(int(g) for g in grid)) == 256
    for g in grid:
        assert {(int(g) >> (8 * j)) & 255 for j in range(8)} <= {8, 25, 43}


def test_chunk_dot_bound():
    # the int32 chunk dot is at most 32 * 43 * 127 = 174752: a weight row of the largest grid entries against
    # +-127 aligned with the signs
    grid, _, _, _ = O.iq2_tables()
    best = max(sum((int(g) >> (8 * j)) & 255 for j in range(8)) for g in grid)
    assert 4 * best * 127 <= 32 * 43 * 127 < 2 ** 31
    blocks = iq2_blocks(11, 32, 256)
    w = O.iq2_dequant(blocks, 32, 256)
    xq = np.where(w >= 0, 127, -127).astype(np.int8)
    dots = O.iq2_chunk_dots(blocks, 32, 256, xq)
    assert np.abs(dots).max() <= 174752


def test_block_sizes():
    assert O.lib() is not None
    assert iq2_blocks(1, 1, 256).nbytes == 66
    # Q8_0 block: fp16 d + 32 int8 (bolt_host.cu:201)
    assert 2 + 32 == 34


def test_e2m1_code_set():
    vals = [O.scalar("or_e2m1_dec", c) for c in range(16)]
    assert vals[:8] == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert vals[8:] == [-v for v in vals[:8]]
    for c in range(1, 16):
        if c == 8:
            continue
        assert O.scalar("or_e2m1_enc", vals[c]) == c


def test_e4m3_decode_matches_torch_and_roundtrips():
    codes = [c for c in range(256) if (c & 0x7F) != 0x7F]
    ref = torch.tensor(codes, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    got = np.array([O.scalar("or_e4m3_dec", c) for c in codes], np.float32)
    assert np.array_equal(got, ref)
    for c in range(1, 0x7F):
        assert O.scalar("or_e4m3_enc", O.scalar("or_e4m3_dec", c)) == c


def test_e4m3_encode_is_nearest_even():
    v = np.random.default_rng(3).uniform(0, 447.0, 4000).astype(np.float32)
    v = np.concatenate([v, np.random.default_rng(4).uniform(0, 0.02, 1000).astype(np.float32)])
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([O.scalar("or_e4m3_enc", float(x)) for x in v], np.uint8)
    assert np.array_equal(got, ref)


def test_half_conversions_match_numpy():
    v = np.random.default_rng(5).standard_normal(5000).astype(np.float32) * np.float32(3e-3)
    v = np.concatenate([v, np.float32([1e-7, 6.1e-5, 65504.0, -2.0, 0.0])])
    ref = v.astype(np.float16).view(np.uint16)
    got = np.array([O.scalar("or_f2h", float(x)) for x in v], np.uint16)
    assert np.array_equal(got, ref)
    back = np.array([O.scalar("or_h2f", int(h)) for h in ref], np.float32)
    assert np.array_equal(back, ref.view(np.float16).astype(np.float32))


def _np_iq2_dequant(blocks, rows, k):
    """An independent numpy restatement of FmtIQ2::deq (bolt_kernels.cu:110-132)."""
    grid, signs, _, _ = O.iq2_tables()
    b = blocks.reshape(rows, k // 256, 66)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32)[..., 0]
    out = np.zeros((rows, k), np.float32)
    for c in range(8):
        qx = b[:, :, 2 + 8 * c:6 + 8 * c].copy().view(np.uint32)[..., 0]
        qy = b[:, :, 6 + 8 * c:10 + 8 * c].copy().view(np.uint32)[..., 0]
        db = d * (np.float32(0.5) + (qy >> 28).astype(np.float32)) * np.float32(0.25)
        for sub in range(4):
            g = grid[(qx >> (8 * sub)) & 255]
            s = signs[(qy >> (7 * sub)) & 127]
            for j in range(8):
                mag = ((g >> np.uint64(8 * j)) & np.uint64(255)).astype(np.float32)
                neg = ((s >> j) & 1).astype(bool)
                out[:, np.arange(k // 256) * 256 + c * 32 + sub * 8 + j] = np.where(neg, -mag, mag) * db
    return out


def test_iq2_dequant_matches_numpy_restatement():
    blocks = iq2_blocks(21, 8, 512)
    assert np.array_equal(O.iq2_dequant(blocks, 8, 512), _np_iq2_dequant(blocks, 8, 512))


def test_quant_rows_formula():
    x = np.random.default_rng(7).standard_normal((3, 64)).astype(np.float32)
    x[1, :32] = 0.0
    q, s = O.quant_rows(x, 64)
    for r in range(3):
        for b in range(2):
            v = x[r, 32 * b:32 * b + 32]
            am = np.float32(np.abs(v).max())
            inv = np.float32(127.0) / am if am > 0 else np.float32(0.0)
            assert np.array_equal(q[r, 32 * b:32 * b + 32], np.rint(v * inv).astype(np.int8))
            assert s[r, b] == am / np.float32(127.0)
    assert (q[1, :32] == 0).all() and s[1, 0] == 0


def test_int8_gemv_matches_numpy_restatement():
    n, k, T = 16, 512, 3
    blocks = iq2_blocks(31, n, k)
    x = np.random.default_rng(8).standard_normal((T, k)).astype(np.float32)
    xq, xs = O.quant_rows(x, k)
    dots = O.iq2_chunk_dots(blocks, n, k, xq)
    w = _np_iq2_dequant(blocks, n, k)
    # the integer weights are dequant / db; rebuild the chunk dots independently
    b = blocks.reshape(n, k // 256, 66)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32)[..., 0]
    for c in range(k // 32):
        qy = b[:, c // 8, 6 + 8 * (c % 8):10 + 8 * (c % 8)].copy().view(np.uint32)[..., 0]
        db = d[:, c // 8] * (np.float32(0.5) + (qy >> 28).astype(np.float32)) * np.float32(0.25)
        wi = np.rint(w[:, 32 * c:32 * c + 32] / db[:, None]).astype(np.int64)
        ref = xq[:, 32 * c:32 * c + 32].astype(np.int64) @ wi.T
        assert np.array_equal(dots[:, :, c], ref)
    y = O.iq2_gemm_i8(blocks, n, k, xq, xs)
    acc = np.zeros((T, n), np.float32)
    for c in range(k // 32):
        qy = b[:, c // 8, 6 + 8 * (c % 8):10 + 8 * (c % 8)].copy().view(np.uint32)[..., 0]
        dA = d[:, c // 8] * (np.float32(0.5) + (qy >> 28).astype(np.float32)) * np.float32(0.25)
        scale = (dA[None, :] * xs[:, c][:, None]).astype(np.float32)
        prod = scale.astype(np.float64) * dots[:, :, c].astype(np.float64) + acc.astype(np.float64)
        acc = prod.astype(np.float32)   # one rounding: fmaf
    assert np.array_equal(y, acc)


def test_int8_mode_is_within_tolerance_of_exact():
    n, k, T = 64, 4096, 4
    blocks = iq2_blocks(41, n, k)
    _, x = normal_bf16(9, (T, k))
    xq, xs = O.quant_rows(x, k)
    e = rel_l2(O.iq2_gemm_i8(blocks, n, k, xq, xs), O.iq2_gemm_exact(blocks, n, k, x))
    assert 1e-4 < e < 1e-2


def test_route_softmax_semantics():
    lg = np.array([[0.0, 2.0, 2.0, 1.0, -1.0, 2.0]], np.float32)
    ridx, rw = O.route_softmax(lg, 3)
    assert list(ridx[0]) == [1, 2, 5]   # ties to the lower index
    assert np.allclose(rw[0], [1 / 3] * 3)
    lg = np.random.default_rng(1).standard_normal((5, 128)).astype(np.float32)
    ridx, rw = O.route_softmax(lg, 6)
    for t in range(5):
        top = np.argsort(-lg[t], kind="stable")[:6]
        assert list(ridx[t]) == list(top)
        e = np.exp(lg[t, top].astype(np.float64) - lg[t].max())
        assert np.allclose(rw[t], e / e.sum(), rtol=1e-6)


def test_route_sigmoid_semantics():
    lg = np.random.default_rng(2).standard_normal((4, 64)).astype(np.float32)
    bias = np.random.default_rng(3).standard_normal(64).astype(np.float32) * np.float32(0.1)
    ridx, rw = O.route_sigmoid(lg, bias, 9, 5.0)
    for t in range(4):
        sig = (1 / (1 + np.exp(-lg[t].astype(np.float64)))).astype(np.float32)
        top = np.argsort(-(sig + bias), kind="stable")[:9]
        assert list(ridx[t]) == list(top)
        assert np.allclose(rw[t], sig[top] / sig[top].sum() * 5.0, rtol=1e-6)


def test_group_semantics():
    ridx = np.array([3, 1, 3, 0, 1, 3], np.int32)
    counts, offsets, order = O.group(ridx, 5)
    assert list(counts) == [1, 2, 0, 3, 0]
    assert list(offsets) == [0, 1, 3, 3, 6, 6]
    assert list(order) == [3, 1, 4, 0, 2, 5]


def test_combine():
    rng = np.random.default_rng(4)
    mo = rng.standard_normal((12, 16)).astype(np.float32)
    rw = rng.random((4, 3)).astype(np.float32)
    out = O.combine(mo, rw, 3, 16)
    ref = np.einsum("tk,tkh->th", rw.astype(np.float64), mo.reshape(4, 3, 16).astype(np.float64))
    assert np.allclose(out, ref, rtol=1e-6, atol=1e-6)


def test_moe_layer_int8_vs_exact_small():
    T, H, F, E, topk = 5, 512, 256, 8, 3
    xb, _ = normal_bf16(1, (T, H))
    lb, _ = normal_bf16(2, (T, E))
    up = iq2_blocks(3, E * F, H)
    down = iq2_blocks(4, E * H, F)
    su, sd = iq2_blocks(5, F, H), iq2_blocks(6, H, F)
    o8, r8, w8 = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=0)
    oe, re, we = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=1)
    assert np.array_equal(r8, re) and np.array_equal(w8, we)
    assert rel_l2(o8, oe) < 3e-2


def _np_nv4(q, sc, s2, n, k):
    lo, hi = q & 15, q >> 4
    nib = np.stack([lo, hi], -1).reshape(n, k)
    mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
    v = np.where(nib & 8, -1.0, 1.0).astype(np.float32) * mag[nib & 7]
    scale = torch.from_numpy(sc.copy()).view(torch.float8_e4m3fn).float().numpy()
    return v * np.repeat(scale, 16, axis=1), s2


def test_nv4_gemm_exact_and_quant():
    n, k, T = 32, 256, 3
    rng = np.random.default_rng(6)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sc = np.array([O.scalar("or_e4m3_enc", float(v)) for v in rng.uniform(0.5, 2, n * k // 16)], np.uint8).reshape(n, k // 16)
    x = rng.standard_normal((T, k)).astype(np.float32)
    w, s2 = _np_nv4(q, sc, 0.37, n, k)
    ref = (x.astype(np.float64) @ w.astype(np.float64).T) * 0.37
    assert np.allclose(O.nv4_gemm_exact(q, sc, 0.37, n, k, x), ref, rtol=1e-6, atol=1e-5)
    q4, sf = O.quant_nv4_rows(x, k)
    xd, _ = _np_nv4(q4, sf, 1.0, T, k)
    scale = np.repeat(torch.from_numpy(sf.copy()).view(torch.float8_e4m3fn).float().numpy(), 16, axis=1)
    assert (np.abs(xd - x) <= scale * 1.0 + 1e-6).all()   # within half the largest e2m1 step (2 -> 3 -> 4 -> 6)
    y4 = O.nv4_gemm_q4(q, sc, 0.37, n, k, q4, sf)
    assert np.allclose(y4, (xd.astype(np.float64) @ w.astype(np.float64).T) * 0.37, rtol=1e-6, atol=1e-5)


def test_q8_gemm_exact():
    n, k, T = 16, 256, 2
    rng = np.random.default_rng(12)
    qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
    d = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    blocks = np.concatenate([d.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1).reshape(n, -1)
    x = rng.standard_normal((T, k)).astype(np.float32)
    w = (qv.astype(np.float32) * d.astype(np.float32)[..., None]).reshape(n, k)
    assert np.allclose(O.q8_gemm_exact(blocks, n, k, x), x.astype(np.float64) @ w.T, rtol=1e-6, atol=1e-6)
    wf = (qv.astype(np.float32) * d.astype(np.float32)[..., None]).astype(np.float16).astype(np.float32).reshape(n, k)
    assert np.allclose(O.q8_gemm_f16fold(blocks, n, k, x), x.astype(np.float64) @ wf.T, rtol=1e-6, atol=1e-6)


def test_oracle_generator_matches_the_library():
    """the bench's CPU arm makes its weights with the oracle's statement of the seeded generator: the same bytes as
    the library's host generator for the same seed"""
    import b200q
    a = O.synth_iq2(1001, 3000)
    b = np.asarray(b200q.synth_iq2_host(1001, 3000)).reshape(a.shape)
    assert np.array_equal(a, b)
