"""GPU parity of the prompt-length tcgen05 GEMMs against the CPU oracle, through the C ABI.

The tensor cores multiply fp16 operands exactly and accumulate in fp32; the oracle uses the same fp16 operands (the
scale folded into the weights, rounded once: libbolt's PQ8 / PIQ2 arithmetic) and sums in fp64.  Bar: relative L2
1e-4 against that oracle, and BASELINE's tolerance (1e-2 / 2e-2) against the exact-mode oracle."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import assert_tolerance, iq2_blocks, normal_bf16, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def q8_blocks(seed, n, k):
    rng = np.random.default_rng(seed)
    qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
    d = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    return np.concatenate([d.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1).reshape(n, -1)


def np_q8_tc(blocks, n, k):
    """numpy statement of the q8 tc layout: units (32-row tile, 32-k block) of [32][32] int8 then [32] fp16 d"""
    b = blocks.reshape(n // 32, 32, k // 32, 34).transpose(0, 2, 1, 3)   # [t][kb][lane][34]
    q = b[..., 2:].reshape(n // 32, k // 32, 1024)
    d = b[..., :2].reshape(n // 32, k // 32, 64)
    return np.concatenate([q, d], -1).reshape(-1)


def test_q8_tc_pack_layout():
    n, k = 64, 512
    blocks = q8_blocks(3, n, k)
    got = b200q.tile_q8_tc(dev(blocks), n, k).cpu().numpy()
    assert np.array_equal(got, np_q8_tc(blocks, n, k))


@pytest.mark.parametrize("n,k,T,dt", [(256, 256, 1, "bf16"), (288, 512, 5, "f32"), (512, 1024, 300, "bf16"),
                                      (6144, 4096, 256, "bf16"), (1024, 512, 515, "f32")])
def test_q8_prompt_gemm(n, k, T, dt):
    blocks = q8_blocks(n + T, n, k)
    xb, x = normal_bf16(n * 3 + T, (T, k))
    xt = dev(xb).view(torch.bfloat16) if dt == "bf16" else dev(x)
    w = b200q.tile_q8_tc(dev(blocks), n, k)
    y = b200q.mma_q8_prompt(w, n, k, xt).cpu().numpy()
    assert b200q.device_error() == 0
    assert rel_l2(y, O.q8_gemm_f16fold(blocks, n, k, x)) < 1e-4
    assert_tolerance(y, O.q8_gemm_exact(blocks, n, k, x))


def test_group_large():
    pairs, E = 49152, 128
    rng = np.random.default_rng(1)
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    ridx = rng.permutation(E)[rng.choice(E, size=pairs, p=p / p.sum())].astype(np.int32)
    counts, offsets, order = b200q.k_moe_group_large(dev(ridx), E)
    oc, oo, oord = O.group(ridx, E)
    assert np.array_equal(counts.cpu().numpy(), oc)
    assert np.array_equal(offsets.cpu().numpy(), oo)
    got = order.cpu().numpy()
    for e in range(E):   # the order inside an expert's run is free; its set is not
        assert np.array_equal(np.sort(got[oo[e]:oo[e + 1]]), oord[oo[e]:oo[e + 1]])


@pytest.mark.parametrize("T,H,F,E,topk", [(40, 512, 256, 8, 3), (300, 1024, 512, 16, 6), (700, 512, 768, 4, 2)])
def test_moe_prompt(T, H, F, E, topk):
    up = iq2_blocks(7 + T, E * F, H)
    down = iq2_blocks(8 + T, E * H, F)
    xb, x = normal_bf16(9 + T, (T, H))
    _, lg = normal_bf16(10 + T, (T, E))
    ridx, _ = O.route_softmax(lg, topk)
    counts, offsets, order = b200q.k_moe_group_large(dev(ridx.reshape(-1)), E)
    pu = b200q.repack_iq2(dev(up.reshape(-1)), E * F, H)
    pd = b200q.repack_iq2(dev(down.reshape(-1)), E * H, F)
    pairs = T * topk
    act = torch.full((pairs, F), float("nan"), dtype=torch.float16, device=DEV)
    y = b200q.moe_prompt(pu, pd, E, H, F, counts, offsets, order, topk, dev(xb).view(torch.bfloat16), act=act)
    y = y.cpu().numpy()
    act_np = act.float().cpu().numpy()
    assert b200q.device_error() == 0
    ub, db = up.reshape(E, -1), down.reshape(E, -1)
    r = ridx.reshape(-1)
    ref_act = np.stack([O.iq2_gemm_f16fold(ub[r[p]], F, H, x[p // topk], 1)[0] for p in range(pairs)])
    assert rel_l2(act_np, ref_act.astype(np.float16).astype(np.float32)) < 2e-3   # act is rounded to fp16
    ref_y = np.stack([O.iq2_gemm_f16fold(db[r[p]], H, F, act_np[p], 0)[0] for p in range(pairs)])
    assert rel_l2(y, ref_y) < 1e-4
    ex_act = np.stack([O.iq2_gemm_exact(ub[r[p]], F, H, x[p // topk], 1)[0] for p in range(pairs)])
    assert_tolerance(act_np, ex_act)
