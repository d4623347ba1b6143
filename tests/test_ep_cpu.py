"""Expert-parallel MoE host logic on CPU: placement, and the dispatch / expert / return / combine exchange as
world_size-2, 4 and 8 gloo ranks against a single-process computation of the same layer.

The experts here are small dense fp32 matrices applied one row at a time (the same operations in both computations),
so with fp32 transfers the expert-parallel result must equal the single-process one exactly; with bf16 transfers
(the default on B200) it stays within the BASELINE tolerance."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ep import ExpertParallelMoE, Placement

E, H, F, TOPK, T = 8, 64, 32, 2, 5


def _weights():
    g = torch.Generator().manual_seed(3)
    up = torch.randn(E, F, H, generator=g) / 8
    down = torch.randn(E, H, F, generator=g) / 6
    shared = torch.randn(H, H, generator=g) / 8
    return up, down, shared


def _expert(up, down, e, row):
    a = torch.relu(up[e] @ row) ** 2
    return down[e] @ a


def _tokens(rank):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    top = torch.topk(torch.softmax(logits, -1), TOPK, dim=-1)
    rw = top.values / top.values.sum(-1, keepdim=True)
    return x, top.indices.to(torch.int32), rw.float()


def _combine(mo, rw, shared):
    out = (mo.view(-1, TOPK, H) * rw.view(-1, TOPK, 1)).sum(1)
    return out + shared if shared is not None else out


def _reference(rank):
    up, down, shared = _weights()
    x, ridx, rw = _tokens(rank)
    xf = x.float()
    mo = torch.stack([_expert(up, down, int(ridx.reshape(-1)[p]), xf[p // TOPK]) for p in range(T * TOPK)])
    return _combine(mo, rw, xf @ shared.T)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, layout, dtype_name, replicate, q, chunks=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        up, down, shared = _weights()
        loads = np.array([8.0, 5, 3, 2, 1, 1, 1, 1]) if replicate else None
        pl = Placement(E, world, loads=loads, replicate=replicate, seed=1)
        local = pl.local[rank]

        def expert_fn(rows, lidx, n_local):
            out = torch.zeros(rows.shape[0], H)
            for i in range(rows.shape[0]):
                j = int(lidx[i])
                if j < n_local:
                    out[i] = _expert(up, down, local[j], rows[i].float())
            return out

        moe = ExpertParallelMoE(pl, rank, world, H, TOPK, expert_fn, shared_fn=lambda x: x.float() @ shared.T,
                                combine_fn=_combine, layout=layout, send_dtype=getattr(torch, dtype_name), chunks=chunks)
        x, ridx, rw = _tokens(rank)
        out = moe(x, ridx, rw)
        q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


def _run(layout, dtype_name, replicate=0, world=2, chunks=1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, layout, dtype_name, replicate, q, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("layout", ["capacity", "exact"])
def test_ep_matches_single_process_fp32(layout):
    got = _run(layout, "float32")
    for r, out in got.items():
        assert np.array_equal(out, _reference(r).numpy())


@pytest.mark.parametrize("layout,world", [("capacity", 4), ("exact", 4), ("capacity", 8)])
def test_ep_matches_single_process_more_ranks(layout, world):
    """the scaling run's rank counts: 8 experts over 4 ranks (2 each) and 8 ranks (1 each), fp32 transfers"""
    got = _run(layout, "float32", world=world)
    assert sorted(got) == list(range(world))
    for r, out in got.items():
        assert np.array_equal(out, _reference(r).numpy())


@pytest.mark.parametrize("world,chunks,replicate", [(2, 3, 0), (4, 2, 0), (2, 7, 0), (2, 2, 2)])
def test_ep_exact_pipelined_chunks(world, chunks, replicate):
    """the exact layout as a pipeline over pieces of the tokens (5 tokens: pieces of 1 and 2 tokens, and more pieces
    than tokens, some empty): the same values reach the same places, so the same bytes as the single-process layer;
    with replicated experts the copies are chosen by the global token index, as without pieces"""
    got = _run("exact", "float32", replicate=replicate, world=world, chunks=chunks)
    assert sorted(got) == list(range(world))
    for r, out in got.items():
        assert np.array_equal(out, _reference(r).numpy())


def test_ep_bf16_transfers_within_tolerance():
    got = _run("capacity", "bfloat16")
    for r, out in got.items():
        ref = _reference(r).numpy()
        assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-2


def test_ep_with_replicated_experts():
    got = _run("exact", "float32", replicate=2)
    for r, out in got.items():
        assert np.array_equal(out, _reference(r).numpy())


def test_placement_properties():
    pl = Placement(128, 8, seed=0)
    assert sorted(e for l in pl.local for e in l) == list(range(128))
    assert all(len(l) == 16 for l in pl.local)
    # Zipf(1.1) loads of 8192 tokens x 6 distinct experts (BASELINE config 4's routing)
    rng = np.random.default_rng(0)
    p = 1.0 / np.arange(1, 129) ** 1.1
    p = rng.permutation(p / p.sum())
    loads = np.zeros(128)
    for _ in range(2048):
        loads[rng.choice(128, 6, replace=False, p=p)] += 4
    lpt = Placement(128, 8, loads=loads)
    # LPT cannot beat the hottest expert's own share; it comes within 5 % of that bound
    assert lpt.imbalance() <= 1.05 * max(1.0, loads.max() / (loads.sum() / 8))
    rep = Placement(128, 8, loads=loads, replicate=4)
    assert rep.imbalance() < 1.25 and rep.imbalance() < lpt.imbalance()
    for e in range(128):
        assert len(set(rep.owners[e])) == len(rep.owners[e])   # copies on distinct ranks
        for r in rep.owners[e]:
            assert rep.local[r][rep.lidx[(e, r)]] == e


def _dying_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise SystemExit(3)   # leaves between steps, before its collective
    pl = Placement(E, world, seed=1)
    moe = ExpertParallelMoE(pl, rank, world, H, TOPK, lambda r, l, n: torch.zeros(r.shape[0], H), combine_fn=_combine,
                            layout="exact", send_dtype=torch.float32)
    x, ridx, rw = _tokens(rank)
    try:
        moe(x, ridx, rw)
        q.put("completed")
    except Exception as e:   # the peer is gone: the collective ends with an error instead of waiting for good
        q.put("error: " + type(e).__name__)


def test_ep_peer_failure_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error")
