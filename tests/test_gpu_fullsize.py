"""GPU parity of the prompt paths at BASELINE's full shapes, through the C ABI, and the decode layer's measured
deviation from the exact arithmetic at config 2.

At these sizes the scalar oracle is too slow for every output, so the checker is the oracle's own dequantisation
(or_iq2_dequant, the e2m1 / e4m3 decodes, the oracle's row quantiser) followed by an fp64 numpy product: the same
operands as the oracle's GEMMs (fp16-rounded weights for the PIQ2 / PQ8 folds, exact e2m1 x e4m3 products for NVFP4),
summed in fp64 in another order, which moves nothing at the bars used here.  Each test first pins that checker to the
scalar oracle on a few rows.  Rows compared:

- config 4 prompt MoE (8192 tokens x top-6 = 49152 pairs, Zipf(1.1) over 128 experts through a seeded permutation,
  H 4096, F 2048, ReLU^2): every pair of the hottest expert, every pair of the least loaded one, and 1024 seeded pairs
  of 14 other experts;
- config 3 NVFP4 prompt: in_proj 4096 -> 18560 (the last 256-row tile of the weights is ragged) and out_proj
  8192 -> 4096, at M 512 (every row) and 4096 (the first and last 128-row tiles of the rows and 256 seeded rows);
- config 4 Q8_0 GQA at 8192 tokens: q/k/v fused (6144 x 4096) and o (4096 x 4096), 512 rows of each.

Bars: the kernels' own arithmetic within 1e-4 relative L2 (fp16-fold products, fp32 sums) or 1e-5 (NVFP4), and
BASELINE's tolerance (relative L2 1e-2, per-row max-abs-relative 2e-2) against the exact arithmetic."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import assert_tolerance, max_abs_rel_per_row, normal_bf16, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def zipf_routing(seed, tokens, E, topk, s=1.1):
    """BASELINE config 4's routing: Zipf(s) over the experts through a seeded rank -> expert permutation, top-k
    distinct experts a token"""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    ridx = np.empty((tokens, topk), np.int32)
    for t in range(tokens):
        ridx[t] = perm[rng.choice(E, size=topk, replace=False, p=p)]
    return ridx


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float64)


def test_config4_moe_prompt_full():
    T, H, F, E, topk = 8192, 4096, 2048, 128, 6
    up = O.synth_iq2(4000, E * F * (H // 256)).reshape(E, F, -1)
    down = O.synth_iq2(4001, E * H * (F // 256)).reshape(E, H, -1)
    xb, x = normal_bf16(4002, (T, H))
    ridx = zipf_routing(4003, T, E, topk)
    counts, offsets, order = b200q.k_moe_group_large(dev(ridx.reshape(-1)), E)
    pu = b200q.repack_iq2(dev(up.reshape(-1)), E * F, H)
    pd = b200q.repack_iq2(dev(down.reshape(-1)), E * H, F)
    pairs = T * topk
    act = torch.full((pairs, F), float("nan"), dtype=torch.float16, device=DEV)
    y = b200q.moe_prompt(pu, pd, E, H, F, counts, offsets, order, topk, dev(xb).view(torch.bfloat16), act=act)
    torch.cuda.synchronize()
    assert b200q.device_error() == 0
    cnt = counts.cpu().numpy()
    assert cnt.sum() == pairs and cnt.max() > 5000   # the hottest Zipf expert holds about 13.5 % of the pairs
    r = ridx.reshape(-1)
    hot, cold = int(cnt.argmax()), int(cnt.argmin())
    rng = np.random.default_rng(4004)
    others = rng.choice(np.setdiff1d(np.arange(E), [hot, cold]), size=14, replace=False)
    pool = np.nonzero(np.isin(r, others))[0]
    sample = np.sort(rng.choice(pool, size=1024, replace=False))
    checked = 0
    for e in [hot, cold, *others.tolist()]:
        rows = np.nonzero(r == e)[0] if e in (hot, cold) else sample[r[sample] == e]
        if rows.size == 0:
            continue
        wu = O.iq2_dequant(up[e], F, H).astype(np.float64)
        wd = O.iq2_dequant(down[e], H, F).astype(np.float64)
        ri = torch.from_numpy(rows).to(DEV)
        a_gpu = act.index_select(0, ri).float().cpu().numpy().astype(np.float64)
        y_gpu = y.index_select(0, ri).cpu().numpy().astype(np.float64)
        xe = x[rows // topk].astype(np.float64)
        if e == hot:   # pin the numpy checker to the scalar oracle on a few rows
            a_or = O.iq2_gemm_f16fold(up[e], F, H, x[rows[:3] // topk], 1)
            h = xe[:3] @ f16(wu).T
            assert rel_l2(np.where(h > 0, h * h, 0), a_or) < 1e-6
            assert rel_l2(a_gpu[:3] @ f16(wd).T, O.iq2_gemm_f16fold(down[e], H, F, a_gpu[:3], 0)) < 1e-6
        h = xe @ f16(wu).T
        a_ref = np.where(h > 0, h * h, 0)
        assert rel_l2(a_gpu, f16(a_ref)) < 2e-3, e          # the up output is stored as fp16
        assert rel_l2(y_gpu, a_gpu @ f16(wd).T) < 1e-4, e    # the down GEMM on the stored fp16 rows
        he = xe @ wu.T
        assert_tolerance(y_gpu, np.where(he > 0, he * he, 0) @ wd.T)
        checked += rows.size
    assert checked >= int(cnt[hot]) + int(cnt[cold]) + 1024
    print(f"config 4 prompt MoE: {checked} pairs checked; hottest expert {cnt[hot]} rows, least loaded {cnt[cold]}")


def nv4_weights(seed, n, k):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sc = torch.from_numpy(rng.uniform(0.5, 2.0, (n, k // 16)).astype(np.float32)).to(torch.float8_e4m3fn)
    return q, sc.view(torch.uint8).numpy()


E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def nv4_values(q, sc, k):
    """e2m1 codes (low nibble first) x e4m3 scales per 16 -> fp64 values [rows][k] (every product exact)"""
    v = np.stack([E2M1[q & 15], E2M1[q >> 4]], -1).reshape(q.shape[0], k)
    s = torch.from_numpy(np.ascontiguousarray(sc)).view(torch.float8_e4m3fn).float().numpy().astype(np.float64)
    return v * np.repeat(s, 16, axis=1)


@pytest.mark.parametrize("name,n,k", [("in_proj", 18560, 4096), ("out_proj", 4096, 8192)])
def test_config3_nvfp4_prompt_full(name, n, k):
    q, sc = nv4_weights(n + k, n, k)
    s2 = 0.01
    w = b200q.tile_nv4w(dev(q), dev(sc), n, k)
    wv = nv4_values(q, sc, k) * s2
    for M in (512, 4096):
        rng = np.random.default_rng(M + n)
        x = rng.standard_normal((M, k)).astype(np.float32)
        xt = dev(x).to(torch.bfloat16)
        xf = xt.float().cpu().numpy()
        y = b200q.mma_nv4_fp4(w, s2, n, k, b200q.quant_nv4_rows(xt), M)
        torch.cuda.synchronize()
        assert b200q.device_error() == 0
        rows = np.arange(M) if M <= 512 else np.unique(np.concatenate(
            [np.arange(128), np.arange(M - 128, M), rng.choice(M, 256, replace=False)]))
        y_gpu = y.index_select(0, torch.from_numpy(rows).to(DEV)).cpu().numpy()
        q4, sf = O.quant_nv4_rows(xf[rows], k)
        ref = nv4_values(q4, sf, k) @ wv.T
        if M == 512:   # pin the numpy checker to the scalar oracle on two rows
            assert rel_l2(ref[:2], O.nv4_gemm_q4(q, sc, s2, n, k, q4[:2], sf[:2])) < 1e-6
        assert rel_l2(y_gpu, ref) < 1e-5, (name, M)
        assert rel_l2(y_gpu, xf[rows].astype(np.float64) @ wv.T) < 0.1   # the fp4 rounding of x itself


def q8_blocks(seed, n, k):
    rng = np.random.default_rng(seed)
    qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
    d = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    return np.concatenate([d.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1).reshape(n, -1), qv, d


@pytest.mark.parametrize("name,n", [("qkv", 6144), ("o", 4096)])
def test_config4_q8_gqa_full(name, n):
    T, k = 8192, 4096
    blocks, qv, d = q8_blocks(n + 77, n, k)
    xb, x = normal_bf16(n + 78, (T, k))
    y = b200q.mma_q8_prompt(b200q.tile_q8_tc(dev(blocks), n, k), n, k, dev(xb).view(torch.bfloat16))
    torch.cuda.synchronize()
    assert b200q.device_error() == 0
    rng = np.random.default_rng(n)
    rows = np.unique(np.concatenate([np.arange(128), np.arange(T - 128, T), rng.choice(T, 256, replace=False)]))
    y_gpu = y.index_select(0, torch.from_numpy(rows).to(DEV)).cpu().numpy()
    w_exact = (qv.astype(np.float64) * d.astype(np.float64)[..., None]).reshape(n, k)
    w_fold = f16(qv.astype(np.float32) * d.astype(np.float32)[..., None]).reshape(n, k)
    xr = x[rows].astype(np.float64)
    assert rel_l2(xr[:2] @ w_fold.T, O.q8_gemm_f16fold(blocks, n, k, x[rows[:2]])) < 1e-6
    assert rel_l2(y_gpu, xr @ w_fold.T) < 1e-4
    assert_tolerance(y_gpu, xr @ w_exact.T)


def test_config2_decode_layer_vs_exact():
    """The config-2 decode layer against the oracle's exact mode (fp32 weights, unquantised activations): the int8
    arithmetic of the reference (two int8-per-32 quantisations in series, x and the up output) against exact
    arithmetic.  The measured deviations are printed; the bar is BASELINE's tolerance."""
    T, H, F, E, topk = 16, 4096, 2048, 128, 6
    up, down = O.synth_iq2(5000, E * F * (H // 256)), O.synth_iq2(5001, E * H * (F // 256))
    su, sd = O.synth_iq2(5002, F * (H // 256)), O.synth_iq2(5003, H * (F // 256))
    xb, _ = normal_bf16(5004, (T, H))
    lb, _ = normal_bf16(5005, (T, E))
    pk = lambda b, n, kk: b200q.repack_iq2(dev(b.reshape(-1)), n, kk)
    layer = b200q.MoeDecodeLayer(pk(up, E * F, H), pk(down, E * H, F), pk(su, F, H), pk(sd, H, F), H, F, E, topk,
                                 max_tokens=T)
    out = layer(dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16)).cpu().numpy()
    o8, _, _ = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=0)
    oe, _, _ = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=1)
    e_int8 = rel_l2(out, o8)
    e1, e2 = rel_l2(out, oe), max_abs_rel_per_row(out, oe)
    print(f"config 2 decode layer: vs the int8 oracle rel L2 {e_int8:.2e}; vs exact rel L2 {e1:.4e}, "
          f"row max-abs-rel {e2:.4e}")
    assert e_int8 < 1e-4
    assert_tolerance(out, oe)
