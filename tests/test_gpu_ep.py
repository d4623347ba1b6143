"""The expert-parallel layer's GPU pieces on one rank (no process group): the received-row expert GEMMs
(LocalExperts.decode / .prompt), the shared expert, the exchange layouts and the combine, against the fused
single-GPU decode layer (b200q_moe_decode) and the CPU oracle.  The exchange sends bf16 rows both ways, so the bar
is BASELINE's tolerance (relative L2 1e-2, max-abs-relative 2e-2 per row)."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from ep import ExpertParallelMoE, LocalExperts, Placement, SharedExpert, slice_slab
from helpers import assert_tolerance, iq2_blocks, normal_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("layout,form,dt", [("capacity", "decode", "bfloat16"), ("exact", "decode", "bfloat16"),
                                          ("capacity", "decode", "float32"), ("exact", "prompt", "bfloat16")])
def test_ep_one_rank_matches_fused_layer(layout, form, dt):
    T, H, F, E, topk = 16, 512, 256, 16, 4
    up = iq2_blocks(1, E * F, H)
    down = iq2_blocks(2, E * H, F)
    su, sd = iq2_blocks(3, F, H), iq2_blocks(4, H, F)
    xb, x = normal_bf16(5, (T, H))
    lb, lg = normal_bf16(6, (T, E))
    pu = b200q.repack_iq2(dev(up.reshape(-1)), E * F, H)
    pd = b200q.repack_iq2(dev(down.reshape(-1)), E * H, F)
    psu, psd = b200q.repack_iq2(dev(su.reshape(-1)), F, H), b200q.repack_iq2(dev(sd.reshape(-1)), H, F)
    xt, lt = dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16)
    fused = b200q.MoeDecodeLayer(pu, pd, psu, psd, H, F, E, topk, route=b200q.ROUTE_SOFTMAX, max_tokens=T)
    want = fused(xt, lt).cpu().numpy()

    pl = Placement(E, 1, seed=3)
    loc = pl.local[0]
    ub, db = b200q.iq2_bytes(F, H), b200q.iq2_bytes(H, F)
    ex = LocalExperts(slice_slab(pu, loc, ub), slice_slab(pd, loc, db), len(loc), H, F)
    fn = ex.decode if form == "decode" else ex.prompt
    moe = ExpertParallelMoE(pl, 0, 1, H, topk, fn, shared_fn=SharedExpert(psu, psd, H, F, T, DEV), layout=layout,
                            send_dtype=getattr(torch, dt), device=torch.device(DEV))
    ridx, rw = b200q.k_route(lt, topk)
    got = moe(xt, ridx, rw).cpu().numpy()
    assert b200q.device_error() == 0
    if form == "decode" and dt == "float32":
        assert np.array_equal(got, want)   # the same kernels in the same order: identical bytes
    assert_tolerance(got, want)
    # and against the oracle's int8 arithmetic (the decode kernels' own; the prompt form's fp16 fold is within it too)
    ref, _, _ = O.moe_layer(xb, lb, up.reshape(-1), down.reshape(-1), su.reshape(-1), sd.reshape(-1), T, H, F, E, topk,
                            mode=0)
    assert_tolerance(got, ref)
