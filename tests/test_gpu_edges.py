"""GPU edge cases of the IQ2_XXS MoE paths against the CPU oracle, through the C ABI: every token routed to the same
experts (the largest per-expert counts a decode step can have, units of three tokens back to back), the decode
layer at its maximum shape (64 tokens x top-16 = 1024 pairs over 512 experts), and a prompt block whose rows all go
to two experts while the others get none (empty groups inside the grouped GEMMs).

Bars as in test_gpu_iq2.py / test_gpu_prefill.py: router picks exact; decode outputs within 1e-4 of the oracle's
int8 mode; prompt outputs within 1e-4 of the fp16-fold oracle."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import assert_tolerance, bf16_bits, bf16_to_f32, iq2_blocks, normal_bf16, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def packed(blocks, n, k):
    return b200q.repack_iq2(dev(blocks.reshape(-1)), n, k)


def skewed_logits(seed, T, E, hot, boost=8.0):
    """bf16 logits ~ N(0, 1) with `boost` added to the columns in `hot`: every token's top picks are those experts"""
    x = np.random.default_rng(seed).standard_normal((T, E)).astype(np.float32)
    x[:, hot] += boost
    return bf16_bits(x)


def decode_layer(T, H, F, E, topk, lb, seed):
    up = iq2_blocks(seed + 1, E * F, H)
    down = iq2_blocks(seed + 2, E * H, F)
    su, sd = iq2_blocks(seed + 3, F, H), iq2_blocks(seed + 4, H, F)
    xb, _ = normal_bf16(seed + 5, (T, H))
    layer = b200q.MoeDecodeLayer(packed(up, E * F, H), packed(down, E * H, F), packed(su, F, H), packed(sd, H, F),
                                 H, F, E, topk, max_tokens=T)
    ridx = torch.empty(T, topk, dtype=torch.int32, device=DEV)
    rw = torch.empty(T, topk, dtype=torch.float32, device=DEV)
    out = layer(dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16), ridx=ridx, rw=rw).cpu().numpy()
    o8, r8, w8 = O.moe_layer(xb, lb, up, down, su, sd, T, H, F, E, topk, mode=0)
    assert np.array_equal(ridx.cpu().numpy(), r8)
    assert np.allclose(rw.cpu().numpy(), w8, rtol=2e-6)
    assert np.allclose(out, o8, rtol=1e-4, atol=1e-6 * np.abs(o8).max())
    assert b200q.device_error() == 0
    return r8


def test_decode_every_token_on_the_same_experts():
    """16 tokens x top-6 on the same six of 128 experts: six slots of 16 tokens (units of 3, 3, 3, 3, 3, 1) plus the
    shared expert's 16, every other slot empty"""
    T, H, F, E, topk = 16, 1024, 512, 128, 6
    hot = [3, 17, 40, 77, 100, 127]
    r8 = decode_layer(T, H, F, E, topk, skewed_logits(60, T, E, hot), seed=600)
    assert sorted(set(r8.reshape(-1).tolist())) == hot


def test_decode_layer_maximum_shape():
    """the decode layer's limits: 64 tokens, top-16, 512 experts (1024 pairs, the router's and grouping's capacity)"""
    T, H, F, E, topk = 64, 256, 256, 512, 16
    lb, _ = normal_bf16(61, (T, E))
    decode_layer(T, H, F, E, topk, lb, seed=700)


def test_prompt_rows_on_two_experts_others_empty():
    """300 tokens x top-2 all on experts 2 and 5 of 8: two groups of 300 rows, six empty ones"""
    T, H, F, E, topk = 300, 512, 256, 8, 2
    up = iq2_blocks(71, E * F, H)
    down = iq2_blocks(72, E * H, F)
    xb, x = normal_bf16(73, (T, H))
    lg = bf16_to_f32(skewed_logits(74, T, E, [2, 5]))
    ridx, _ = O.route_softmax(lg, topk)
    assert sorted(set(ridx.reshape(-1).tolist())) == [2, 5]
    counts, offsets, order = b200q.k_moe_group_large(dev(ridx.reshape(-1)), E)
    assert counts.cpu().numpy().tolist() == [0, 0, T, 0, 0, T, 0, 0]
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
