"""The expert-parallel layer's GPU pieces on one rank (no process group): the received-row expert GEMMs
(LocalExperts.decode / .prompt), the shared expert, the exchange layouts and the combine, against the fused
single-GPU decode layer (b200q_moe_decode) and the CPU oracle.  The exchange sends bf16 rows both ways, so the bar
is BASELINE's tolerance (relative L2 1e-2, max-abs-relative 2e-2 per row)."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from ep import ExpertParallelMoE, LocalExperts, PeerDecodeMoE, Placement, SharedExpert, slice_slab
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


@pytest.mark.parametrize("R,H,F,n_local,dt", [(40, 512, 256, 5, "bfloat16"), (96, 1024, 2048, 16, "float32"),
                                              (7, 256, 512, 3, "bfloat16")])
def test_experts_decode_matches_grouped_gemvs(R, H, F, n_local, dt):
    """b200q_moe_experts_decode (one prologue: grouping, slot schedule, int8 rows; then the two GEMVs) against the
    grouped operators it fuses (k_quant_rows, k_moe_group, moe_up_q8, moe_down): the same arithmetic, so the same
    bytes; padding rows (local index n_local or above) are left alone, one expert gets no rows, and the rows sit at a
    padded stride as the exchange leaves them"""
    rng = np.random.default_rng(R + H)
    up = iq2_blocks(21, n_local * F, H)
    down = iq2_blocks(22, n_local * H, F)
    pu = b200q.repack_iq2(dev(up.reshape(-1)), n_local * F, H)
    pd = b200q.repack_iq2(dev(down.reshape(-1)), n_local * H, F)
    lidx = rng.integers(0, n_local - 1, R).astype(np.int32)   # expert n_local - 1 gets none
    lidx[::5] = n_local                                        # padding rows
    lidx[1::11] = n_local + 7
    buf = torch.randn(R, H + 64, device=DEV).to(getattr(torch, dt))
    rows = buf[:, :H]
    li = dev(lidx)
    sentinel = torch.full((R, H), 12345.0, device=DEV)
    got = b200q.ExpertsDecode(pu, pd, n_local, H, F)(rows, li, y=sentinel.clone()).cpu().numpy()
    # the grouped operators on the same rows (padding grouped into slot n_local and not computed)
    xq, xs = b200q.k_quant_rows(rows.contiguous())
    gl = torch.where(li >= n_local, torch.full_like(li, n_local), li)
    counts, offsets, order = b200q.k_moe_group(gl, n_local + 1)
    aq, as_ = b200q.moe_up_q8(pu, n_local, F, H, counts, offsets, order, 1, xq, xs)
    want = b200q.moe_down(pd, n_local, H, F, counts, offsets, order, aq, as_).cpu().numpy()
    real = lidx < n_local
    assert np.array_equal(got[real], want[real])
    assert (got[~real] == 12345.0).all()
    # and the oracle's int8 arithmetic, row by row
    xq_n, xs_n = xq.cpu().numpy(), xs.cpu().numpy()
    ub, db = up.reshape(n_local, -1), down.reshape(n_local, -1)
    for r in np.nonzero(real)[0][:6]:
        a = O.iq2_gemm_i8(ub[lidx[r]], F, H, xq_n[r], xs_n[r], 1)
        aq_r, as_r = O.quant_rows(a, F)
        assert np.array_equal(got[r], O.iq2_gemm_i8(db[lidx[r]], H, F, aq_r, as_r, 0)[0])
    assert b200q.device_error() == 0


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
def test_fused_capacity_exchange_matches_tensor_form(dt):
    """the capacity exchange as b200q_ep_pack + the local experts + b200q_ep_combine against its tensor-operation
    form on the same inputs: the same values reach the same places, so the same bytes come out; and the send buffer
    itself: every pair's row in its destination block at its place in pair order, indices after the values"""
    T, H, F, E, topk = 16, 512, 256, 16, 4
    up = iq2_blocks(31, E * F, H)
    down = iq2_blocks(32, E * H, F)
    su, sd = iq2_blocks(33, F, H), iq2_blocks(34, H, F)
    xb, _ = normal_bf16(35, (T, H))
    lb, _ = normal_bf16(36, (T, E))
    pu = b200q.repack_iq2(dev(up.reshape(-1)), E * F, H)
    pd = b200q.repack_iq2(dev(down.reshape(-1)), E * H, F)
    psu, psd = b200q.repack_iq2(dev(su.reshape(-1)), F, H), b200q.repack_iq2(dev(sd.reshape(-1)), H, F)
    xt, lt = dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16)
    pl = Placement(E, 1, seed=5)
    loc = pl.local[0]
    ex = LocalExperts(slice_slab(pu, loc, b200q.iq2_bytes(F, H)), slice_slab(pd, loc, b200q.iq2_bytes(H, F)), len(loc),
                      H, F)
    moe = ExpertParallelMoE(pl, 0, 1, H, topk, ex.decode, shared_fn=SharedExpert(psu, psd, H, F, T, DEV),
                            layout="capacity", send_dtype=getattr(torch, dt), device=torch.device(DEV))
    ridx, rw = b200q.k_route(lt, topk)
    fused = moe(xt, ridx, rw).cpu().numpy()
    moe.fused = False
    plain = moe(xt, ridx, rw).cpu().numpy()
    assert np.array_equal(fused, plain)
    # the send buffer
    cap = T * topk
    send, slot = b200q.ep_pack(xt, ridx, moe.dest_32, moe.lidx_32, moe.nrep_32, 1, cap, len(loc), getattr(torch, dt))
    r = ridx.reshape(-1).cpu().numpy()
    s = slot.cpu().numpy()
    assert np.array_equal(np.sort(s), np.arange(cap))            # one rank: every pair in order of the pairs
    assert np.array_equal(s, np.arange(cap))
    idx = b200q.ep_index_view(send, H).cpu().numpy()
    assert np.array_equal(idx, np.array([pl.lidx[(int(e), 0)] for e in r]))
    assert np.array_equal(send[:, :H].float().cpu().numpy(), xt.float().repeat_interleave(topk, 0).cpu().numpy())


def test_ep_pack_and_combine_layout_four_ranks():
    """b200q_ep_pack for a 4-rank placement (with a replicated expert) against a numpy statement of the send layout:
    destination blocks of cap rows, each holding its pairs in pair order with their values and local indices, the rest
    carrying the discard index; b200q_ep_combine against the weighted sum it restates"""
    T, H, E, topk, world = 16, 256, 16, 6, 4
    rng = np.random.default_rng(41)
    loads = rng.uniform(1, 10, E)
    loads[3] = 200.0
    pl = Placement(E, world, loads=loads, replicate=1)
    assert max(len(o) for o in pl.owners) > 1
    dest_t, lidx_t, nrep_t = (t.to(torch.int32) for t in pl.tables(torch.device(DEV)))
    x = torch.randn(T, H, device=DEV)
    ridx = torch.from_numpy(rng.integers(0, E, (T, topk)).astype(np.int32)).to(DEV)
    cap = T * topk
    discard = max(len(l) for l in pl.local)
    send, slot = b200q.ep_pack(x, ridx, dest_t, lidx_t, nrep_t, world, cap, discard, torch.float32)
    s_np, idx = send[:, :H].cpu().numpy(), b200q.ep_index_view(send, H).cpu().numpy()
    slot_np, x_np, r = slot.cpu().numpy(), x.cpu().numpy(), ridx.cpu().numpy().reshape(-1)
    fill = np.zeros(world, int)
    seen = np.zeros(world * cap, bool)
    for p in range(cap):
        e, t = int(r[p]), p // topk
        owner = pl.owners[e][t % len(pl.owners[e])]
        row = owner * cap + fill[owner]
        fill[owner] += 1
        assert slot_np[p] == row
        assert idx[row] == pl.lidx[(e, owner)]
        assert np.array_equal(s_np[row], x_np[t])
        seen[row] = True
    assert (idx[~seen] == discard).all()
    # the combine over a return buffer holding anything in the unused rows
    back = torch.randn(world * cap, H, device=DEV).to(torch.bfloat16)
    rw = torch.rand(T, topk, device=DEV)
    shared = torch.randn(T, H, device=DEV)
    got = b200q.ep_combine(back, slot, rw, topk, shared).cpu().numpy()
    b, w = back.float().cpu().numpy(), rw.cpu().numpy()
    want = np.zeros((T, H), np.float32)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for k in range(topk):
            acc = (np.float64(w[t, k]) * b[slot_np[t * topk + k]] + acc).astype(np.float32)   # fma: one rounding
        want[t] = acc + shared[t].cpu().numpy()
    assert np.array_equal(got, want)


def _peer_layer(T, H, F, E, topk, dt, seed=50):
    up = iq2_blocks(seed + 1, E * F, H)
    down = iq2_blocks(seed + 2, E * H, F)
    su, sd = iq2_blocks(seed + 3, F, H), iq2_blocks(seed + 4, H, F)
    pu = b200q.repack_iq2(dev(up.reshape(-1)), E * F, H)
    pd = b200q.repack_iq2(dev(down.reshape(-1)), E * H, F)
    psu, psd = b200q.repack_iq2(dev(su.reshape(-1)), F, H), b200q.repack_iq2(dev(sd.reshape(-1)), H, F)
    pl = Placement(E, 1, seed=9)
    loc = pl.local[0]
    moe = PeerDecodeMoE(pl, 0, 1, H, F, T, topk, slice_slab(pu, loc, b200q.iq2_bytes(F, H)),
                        slice_slab(pd, loc, b200q.iq2_bytes(H, F)), psu, psd, ret_dtype=getattr(torch, dt),
                        device=torch.device(DEV))
    fused = b200q.MoeDecodeLayer(pu, pd, psu, psd, H, F, E, topk, route=b200q.ROUTE_SOFTMAX, max_tokens=T)
    return moe, fused, (up, down, su, sd)


@pytest.mark.parametrize("T,H,F,E,topk,dt", [(16, 512, 256, 16, 4, "float32"), (16, 512, 256, 16, 4, "bfloat16"),
                                             (16, 4096, 2048, 128, 6, "float32"), (3, 256, 512, 8, 2, "bfloat16")])
def test_peer_decode_one_rank_matches_fused_layer(T, H, F, E, topk, dt):
    """b200q_ep_peer_decode on one rank (its exchange stores into its own region): the rows go out as the int8 rows
    the fused layer computes too, so with fp32 outputs returned the combine adds the fused layer's values in its
    order: the same bytes; with bf16 outputs returned they round, within BASELINE's tolerance of the fused layer and
    of the oracle.  Several steps in a row: the epochs advance and the region's rows are reused."""
    moe, fused, (up, down, su, sd) = _peer_layer(T, H, F, E, topk, dt)
    try:
        for step in range(3):
            xb, _ = normal_bf16(60 + step, (T, H))
            lb, _ = normal_bf16(70 + step, (T, E))
            xt, lt = dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16)
            ridx = torch.empty(T, topk, dtype=torch.int32, device=DEV)
            got = moe(xt, lt, ridx=ridx).cpu().numpy()
            want_ridx = torch.empty(T, topk, dtype=torch.int32, device=DEV)
            want = fused(xt, lt, ridx=want_ridx).cpu().numpy()
            assert moe.error() == 0 and b200q.device_error() == 0
            assert torch.equal(ridx, want_ridx)
            if dt == "float32":
                assert np.array_equal(got, want)
            assert_tolerance(got, want)
            if H <= 512:
                ref, _, _ = O.moe_layer(xb, lb, up.reshape(-1), down.reshape(-1), su.reshape(-1), sd.reshape(-1), T,
                                        H, F, E, topk, mode=0)
                assert_tolerance(got, ref)
        assert int(moe.state[0].item()) == 3   # one epoch a step
    finally:
        moe.close()


def test_peer_decode_wait_runs_out_with_an_error_not_a_hang():
    """A bounded wait that nothing satisfies: the step's epoch set ahead of every flag, so the local experts' prologue
    (the senders' flags) and then the combine (the owners' flags) each give up after their time limit, record their
    bit and return; the stream stays usable, and once the epoch is back where the flags are a full step is right."""
    T, H, F, E, topk = 2, 256, 256, 4, 2
    moe, fused, _ = _peer_layer(T, H, F, E, topk, "bfloat16", seed=80)
    try:
        xb, _ = normal_bf16(81, (T, H))
        lb, _ = normal_bf16(82, (T, E))
        xt, lt = dev(xb).view(torch.bfloat16), dev(lb).view(torch.bfloat16)
        moe(xt, lt)
        assert moe.error() == 0
        moe.state[0] = 100                 # no sender has published step 100
        moe(xt, lt, phases=2)
        torch.cuda.synchronize()
        assert moe.error() == 1
        moe.state[0] = 200                 # no owner has published step 200 (the GEMVs above published 100)
        moe(xt, lt, phases=4)
        torch.cuda.synchronize()
        assert moe.error() == 2
        moe.state[0] = 100                 # where every flag now is: the next step publishes and waits for 101
        got = moe(xt, lt).cpu().numpy()
        assert moe.error() == 0
        assert_tolerance(got, fused(xt, lt).cpu().numpy())
    finally:
        moe.close()
