"""GPU parity of the IQ2_XXS path against the CPU oracle, through the C ABI.

Bar: the int32 chunk dots are bit-exact; every int8-mode output is bit-exact against the oracle's int8 mode (the
kernels keep the reference's per-row chunk order); outputs against the oracle's exact mode are within BASELINE's
tolerance (relative L2 <= 1e-2, per-row max-abs-relative <= 2e-2)."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import assert_tolerance, bf16_bits, iq2_blocks, normal_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def packed(blocks, n, k):
    return b200q.repack_iq2(dev(blocks.reshape(-1)), n, k)


def np_pack_rt32(blocks, n, k):
    """numpy statement of the rt32 layout: per (32-row tile, 256-k super-block) unit, [4 chunk pairs][32 rows][16 B]
    of the rows' ggml chunk bytes, then the 32 rows' fp16 d."""
    nb = k // 256
    b = blocks.reshape(n, nb, 66).copy()
    # each chunk's sign word -> four bytes: 7-bit sign index g | bit g of the sub-scale << 7
    qy = b[:, :, 2:].reshape(n, nb, 8, 8)[..., 4:8].copy().view(np.uint32)[..., 0]
    enc = np.zeros_like(qy)
    for g in range(4):
        enc |= (((qy >> (7 * g)) & 127) | (((qy >> (28 + g)) & 1) << 7)) << (8 * g)
    chunks = b[:, :, 2:].reshape(n, nb, 8, 8)
    chunks[..., 4:8] = enc[..., None].view(np.uint8).reshape(n, nb, 8, 4)
    b[:, :, 2:] = chunks.reshape(n, nb, 64)
    qs = b[:, :, 2:].reshape(n // 32, 32, nb, 4, 16).transpose(0, 2, 3, 1, 4).reshape(n // 32, nb, 2048)
    d = b[:, :, :2].reshape(n // 32, 32, nb, 2).transpose(0, 2, 1, 3).reshape(n // 32, nb, 64)
    return np.concatenate([qs, d], axis=2).reshape(-1)


@pytest.mark.parametrize("n,k", [(32, 256), (64, 1024), (2048, 4096)])
def test_pack_layout(n, k):
    blocks = iq2_blocks(100 + n, n, k)
    got = packed(blocks, n, k).cpu().numpy()
    assert np.array_equal(got, np_pack_rt32(blocks, n, k))


def test_device_generator_matches_host():
    host = b200q.synth_iq2_host(1234, 5000)
    devb = b200q.synth_iq2(1234, 5000).cpu().numpy()
    assert np.array_equal(host, devb)


@pytest.mark.parametrize("n,k,T", [(64, 512, 3), (256, 4096, 1), (96, 2048, 17)])
def test_chunk_dots_bit_exact(n, k, T):
    blocks = iq2_blocks(7 + T, n, k)
    x = np.random.default_rng(T).standard_normal((T, k)).astype(np.float32)
    xq, _ = O.quant_rows(x, k)
    got = b200q.iq2_chunk_dots(packed(blocks, n, k), n, k, dev(xq)).cpu().numpy()
    assert np.array_equal(got, O.iq2_chunk_dots(blocks, n, k, xq))


def test_chunk_dots_extreme_inputs():
    n, k = 32, 256
    blocks = iq2_blocks(5, n, k)
    for xv in (127, -127, -128):
        xq = np.full((2, k), xv, np.int8)
        got = b200q.iq2_chunk_dots(packed(blocks, n, k), n, k, dev(xq)).cpu().numpy()
        assert np.array_equal(got, O.iq2_chunk_dots(blocks, n, k, xq))


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.bfloat16])
def test_quant_rows_bit_exact(x_dtype):
    x = torch.randn(37, 4096, generator=torch.Generator().manual_seed(3)).to(x_dtype)
    x[5, :64] = 0
    q, s = b200q.k_quant_rows(x.to(DEV))
    oq, os_ = O.quant_rows(x.float().numpy(), 4096)
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(s.cpu().numpy(), os_)


@pytest.mark.parametrize("n,k,T,epi", [(2048, 4096, 1, 0), (4096, 2048, 16, 0), (2048, 4096, 5, 1), (64, 256, 40, 1)])
def test_gemv_int8_bit_exact_and_tolerance(n, k, T, epi):
    blocks = iq2_blocks(50 + T, n, k)
    _, x = normal_bf16(60 + T, (T, k))
    xq, xs = O.quant_rows(x, k)
    y = b200q.mma_iq2(packed(blocks, n, k), n, k, dev(xq), dev(xs), epi).cpu().numpy()
    assert np.array_equal(y, O.iq2_gemm_i8(blocks, n, k, xq, xs, epi))
    assert_tolerance(y, O.iq2_gemm_exact(blocks, n, k, x, epi))


@pytest.mark.parametrize("mode", [b200q.ROUTE_SOFTMAX, b200q.ROUTE_SIGMOID])
@pytest.mark.parametrize("T,E,topk", [(16, 128, 6), (3, 512, 9), (1, 8, 8)])
def test_route(mode, T, E, topk):
    bits, lg = normal_bf16(T * E + topk, (T, E))
    bias = np.random.default_rng(E).standard_normal(E).astype(np.float32) * np.float32(0.05)
    b_dev = dev(bias) if mode == b200q.ROUTE_SIGMOID else None
    ridx, rw = b200q.k_route(dev(bits).view(torch.bfloat16), topk, mode, b_dev, 2.5)
    if mode == b200q.ROUTE_SOFTMAX:
        oi, ow = O.route_softmax(lg, topk)
    else:
        oi, ow = O.route_sigmoid(lg, bias, topk, 2.5)
    assert np.array_equal(ridx.cpu().numpy(), oi)
    assert np.allclose(rw.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("mode", [b200q.ROUTE_SOFTMAX, b200q.ROUTE_SIGMOID])
def test_route_ties_go_to_the_lower_index(mode):
    """logits from {0, 1, 2, 3}: most picks are ties, which route_k's warp argmax breaks towards the lower expert
    index (bolt_kernels.cu:1676-1692); the oracle does the same"""
    T, E, topk = 16, 128, 6
    lg = np.random.default_rng(77).integers(0, 4, (T, E)).astype(np.float32)
    bits = bf16_bits(lg)
    ridx, rw = b200q.k_route(dev(bits).view(torch.bfloat16), topk, mode, None, 1.0)
    if mode == b200q.ROUTE_SOFTMAX:
        oi, ow = O.route_softmax(lg, topk)
    else:
        oi, ow = O.route_sigmoid(lg, None, topk, 1.0)
    assert np.array_equal(ridx.cpu().numpy(), oi)
    # every token's picks: its highest value's experts in index order
    for t in range(T):
        order = sorted(range(E), key=lambda i: (-lg[t, i], i))[:topk]
        assert oi[t].tolist() == order
    assert np.allclose(rw.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("pairs,E", [(96, 128), (1, 4), (4096, 512), (0, 16)])
def test_group(pairs, E):
    ridx = np.random.default_rng(pairs).integers(0, E, pairs).astype(np.int32)
    counts, offsets, order = b200q.k_moe_group(dev(ridx), E)
    oc, oo, oord = O.group(ridx, E)
    assert np.array_equal(counts.cpu().numpy(), oc)
    assert np.array_equal(offsets.cpu().numpy(), oo)
    assert np.array_equal(order.cpu().numpy(), oord)


def test_combine():
    rng = np.random.default_rng(9)
    T, topk, H = 16, 6, 4096
    mo = rng.standard_normal((T * topk, H)).astype(np.float32)
    rw = rng.random((T, topk)).astype(np.float32)
    sh = rng.standard_normal((T, H)).astype(np.float32)
    out = b200q.k_combine(dev(mo), dev(rw), topk).cpu().numpy()
    assert np.array_equal(out, O.combine(mo, rw, topk, H))
    out2 = b200q.k_combine(dev(mo), dev(rw), topk, shared=dev(sh)).cpu().numpy()
    assert np.array_equal(out2, O.combine(mo, rw, topk, H) + sh)


def test_moe_up_down_grouped():
    T, H, F, E, topk = 7, 1024, 512, 16, 4
    up = iq2_blocks(1, E * F, H)
    down = iq2_blocks(2, E * H, F)
    _, x = normal_bf16(3, (T, H))
    _, lg = normal_bf16(4, (T, E))
    ridx, _ = O.route_softmax(lg, topk)
    counts, offsets, order = b200q.k_moe_group(dev(ridx.reshape(-1)), E)
    xq, xs = O.quant_rows(x, H)
    pu, pd = packed(up, E * F, H), packed(down, E * H, F)
    act = b200q.moe_up(pu, E, F, H, counts, offsets, order, topk, dev(xq), dev(xs), epi=1).cpu().numpy()
    ub = up.reshape(E, -1)
    db = down.reshape(E, -1)
    ref_act = np.stack([O.iq2_gemm_i8(ub[ridx.reshape(-1)[p]], F, H, xq[p // topk], xs[p // topk], 1)[0] for p in range(T * topk)])
    assert np.array_equal(act, ref_act)
    aq, as_ = b200q.moe_up_q8(pu, E, F, H, counts, offsets, order, topk, dev(xq), dev(xs))
    oaq, oas = O.quant_rows(ref_act, F)
    assert np.array_equal(aq.cpu().numpy(), oaq) and np.array_equal(as_.cpu().numpy(), oas)
    mo = b200q.moe_down(pd, E, H, F, counts, offsets, order, aq, as_).cpu().numpy()
    ref_mo = np.stack([O.iq2_gemm_i8(db[ridx.reshape(-1)[p]], H, F, oaq[p], oas[p], 0)[0] for p in range(T * topk)])
    assert np.array_equal(mo, ref_mo)


def _layer(T, H, F, E, topk, shared, route=b200q.ROUTE_SOFTMAX, seed=0):
    up = iq2_blocks(seed + 1, E * F, H)
    down = iq2_blocks(seed + 2, E * H, F)
    su = iq2_blocks(seed + 3, F, H) if shared else None
    sd = iq2_blocks(seed + 4, H, F) if shared else None
    xb, _ = normal_bf16(seed + 5, (T, H))
    lb, _ = normal_bf16(seed + 6, (T, E))
    layer = b200q.MoeDecodeLayer(packed(up, E * F, H), packed(down, E * H, F),
                                 packed(su, F, H) if shared else None, packed(sd, H, F) if shared else None,
                                 H, F, E, topk, route=route, max_tokens=max(T, 16))
    ridx = torch.empty(T, topk, dtype=torch.int32, device=DEV)
    rw = torch.empty(T, topk, dtype=torch.float32, device=DEV)
    out = layer(dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16), ridx=ridx, rw=rw).cpu().numpy()
    return out, ridx.cpu().numpy(), rw.cpu().numpy(), (xb, lb, up, down, su, sd)


@pytest.mark.parametrize("T,H,F,E,topk,shared", [(5, 512, 256, 8, 3, True), (16, 1024, 512, 32, 6, False), (1, 256, 256, 4, 4, True)])
def test_decode_layer_small(T, H, F, E, topk, shared):
    out, ridx, rw, (xb, lb, up, down, su, sd) = _layer(T, H, F, E, topk, shared)
    o8, r8, w8 = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=0)
    assert np.array_equal(ridx, r8)
    assert np.allclose(rw, w8, rtol=2e-6)
    assert np.allclose(out, o8, rtol=1e-4, atol=1e-6 * np.abs(o8).max())
    oe, _, _ = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=1)
    assert_tolerance(out, oe, rel=3e-2, row=6e-2)   # two int8 quantisations (x and the up output) in series


def test_decode_layer_baseline_config2():
    """BASELINE config 2 at full size: 16 tokens, hidden 4096, 128 experts, top-6 + 1 shared, F 2048."""
    T, H, F, E, topk = 16, 4096, 2048, 128, 6
    out, ridx, rw, (xb, lb, up, down, su, sd) = _layer(T, H, F, E, topk, True, seed=1000)
    o8, r8, w8 = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=0)
    assert np.array_equal(ridx, r8)
    assert np.allclose(out, o8, rtol=1e-4, atol=1e-6 * np.abs(o8).max())
