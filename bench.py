"""Benchmark of the B200 quantized-GEMM engine on BASELINE's headline workload.

Workload: one decode MoE layer of 16 tokens, hidden 4096, 128 routed IQ2_XXS experts, top-6
(softmax, renormalised) plus one shared expert, expert FFN 2048 with ReLU^2.  A step is one pass of the layer
(router -> up -> down -> combine) over one batch of 16 tokens.  Metric: IQ2_XXS MoE decode GB/s = the algorithmic
bytes of the step (every touched expert's up and down weights read once, plus x, the logits and the output) / the
step time.  L2 is defeated by rotating 4 layer copies (2.2 GB of experts) and 8 token batches.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's arithmetic on the host cores: the CPU oracle (a scalar C restatement of
libbolt's kernels; libbolt has no CPU implementation of this path) with every host thread, on a bounded sample.
Under torchrun (N > 1) the layer runs expert-parallel: 128/N experts a rank, 16 tokens a rank,
NCCL all-to-all dispatch and combine; the line's value is the decode GB/s over all ranks (weak scaling), its
"prefill" the prompt layer at 8192 tokens a rank.  At N = 1 the "ep" object reports the same expert-parallel code on
one rank, the basis of the scaling.
"""
import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "nemotron-3.5-bolt-tensorfold-dgx-spark_b200")
sys.path[:0] = [PKG]

METRIC = "IQ2_XXS MoE decode GB/s"
T, H, F, E, TOPK = 16, 4096, 2048, 128, 6
LAYERS, BATCHES = 4, 8
EXPERT_BYTES = 2 * (F * (H // 256) * 66)      # up [F][H] + down [H][F]: 4,325,376 B
# DRAM bytes (read + write) of one captured decode_layer_k launch at config 2, per the ncu summary in profiles/:
# 281,733,632 read + 4,721,152 written for a launch whose batch routes to 63 distinct experts (277,221,376
# algorithmic bytes).  Traffic grows with the experts read, so a launch's traffic is that ratio times its bytes.
LAYER_TRAFFIC_CAPTURED = (281_733_632 + 4_721_152, 277_221_376)
LAYER_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one decode_layer_k launch at config 2 "
                        "(63 distinct experts), scaled by the algorithmic bytes to the timed launches' mean")


def config2():
    """the config object of the headline line, the same in both arms"""
    return {"workload": "BASELINE config 2: decode MoE layer, 16 tokens, hidden 4096, 128 IQ2_XXS experts top-6 "
                        "(softmax, renormalised) + 1 shared, FFN 2048, ReLU^2",
            "tokens": T, "hidden": H, "experts": E, "topk": TOPK, "ffn": F, "shared_experts": 1,
            "l2": f"inputs larger than L2: {LAYERS} rotating layer copies "
                  f"({LAYERS * (E + 1) * EXPERT_BYTES / 1e9:.2f} GB) and {BATCHES} token batches (the 126 MB L2)",
            "parallelism": "single"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampled every 50 ms in the background during the timed region (one query after it if the region was
    shorter than that)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index          # an int, or a comma-separated list of indices (one sampler for all the ranks)
        self.proc = None
        self.path = os.path.join("/tmp", f"b200q_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()
            if os.path.exists(self.path) and os.path.getsize(self.path) == 0:
                # a timed region shorter than the polling interval: one query right after it
                with open(self.path, "w") as f:
                    subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                    "--format=csv,noheader,nounits"], stdout=f, stderr=subprocess.DEVNULL, timeout=30)

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_layers(b200q, device):
    """4 layer copies of 128 experts (packed rt32) + a shared expert each, generated on the device."""
    up_b, down_b = b200q.iq2_bytes(F, H), b200q.iq2_bytes(H, F)
    layers = []
    for L in range(LAYERS):
        up = torch.empty(E * up_b, dtype=torch.uint8, device=device)
        down = torch.empty(E * down_b, dtype=torch.uint8, device=device)
        raw = b200q.synth_iq2(1000 + 10 * L, E * F * (H // 256), device)
        b200q.repack_iq2(raw, E * F, H, out=up)
        raw = b200q.synth_iq2(1001 + 10 * L, E * H * (F // 256), device)
        b200q.repack_iq2(raw, E * H, F, out=down)
        del raw
        su = b200q.repack_iq2(b200q.synth_iq2(1002 + 10 * L, F * (H // 256), device), F, H)
        sd = b200q.repack_iq2(b200q.synth_iq2(1003 + 10 * L, H * (F // 256), device), H, F)
        layers.append(b200q.MoeDecodeLayer(up, down, su, sd, H, F, E, TOPK, route=b200q.ROUTE_SOFTMAX, max_tokens=T))
    torch.cuda.synchronize()
    return layers


def zipf_routing(seed, tokens, topk, s=1.1, perm_seed=None):
    """BASELINE config 4's routing: Zipf(s) over the experts through a seeded rank -> expert permutation (from
    perm_seed when given, so that several draws share the experts' popularity), top-k distinct experts a token."""
    rng = np.random.default_rng(seed)
    perm = np.random.default_rng(perm_seed).permutation(E) if perm_seed is not None else rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    ridx = np.empty((tokens, topk), np.int32)
    for t in range(tokens):
        ridx[t] = perm[rng.choice(E, size=topk, replace=False, p=p)]
    return ridx


def graph_ms(call, n, reps=5):
    """ms per call of call(i), i = 0 .. n-1, captured once as a CUDA graph and replayed `reps` times: the decode GEMVs
    take some 10-60 us of GPU time, less than a Python-side launch, so timing them launch by launch would time the
    host.  The caller has run call(i) eagerly first (warm-up, workspaces sized)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            for i in range(n):
                call(i)
    torch.cuda.current_stream().wait_stream(side)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * n)
    del g
    return ms


def pipelined_e2e(run, xh, lh, steps, first, device, out_shape, bufs=None):
    """`steps` calls run(i, x, logits, out) of the public layer over pinned host buffers, each step's inputs copied
    host -> device and its output device -> host inside the timed region, as a serving loop does it: the copies on a
    stream of their own, overlapped with the neighbouring steps' kernels (step i + 1's inputs go up while step i
    runs, step i's output comes back while step i + 1 runs), device buffers doubled: step i reads bufs[i & 1] (two
    (x, logits) pairs; fresh ones by default) and writes out[i & 1], or returns the tensor it wrote (a graph's output).
    -> ms from before the first copy to after the last one (CUDA events on the compute stream)."""
    comp = torch.cuda.current_stream()
    copy = torch.cuda.Stream(device=device)
    if bufs is None:
        bufs = [(torch.empty(xh[0].shape, dtype=xh[0].dtype, device=device),
                 torch.empty(lh[0].shape, dtype=lh[0].dtype, device=device)) for _ in range(2)]
    xd, ld = [b[0] for b in bufs], [b[1] for b in bufs]
    od = [torch.empty(out_shape, dtype=torch.float32, device=device) for _ in range(2)]
    oh = [torch.empty(out_shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("inp", "done", "outp")}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nb = len(xh)
    torch.cuda.synchronize()
    e0.record(comp)
    copy.wait_stream(comp)

    def upload(i, b):
        with torch.cuda.stream(copy):
            xd[b].copy_(xh[(first + i) % nb], non_blocking=True)
            ld[b].copy_(lh[(first + i) % nb], non_blocking=True)
            ev["inp"][b].record(copy)

    upload(0, 0)
    for i in range(steps):
        b = i & 1
        if i + 1 < steps:
            if i >= 1:
                copy.wait_event(ev["done"][1 - b])   # step i - 1 is done with the other buffers
            upload(i + 1, 1 - b)
        comp.wait_event(ev["inp"][b])
        if i >= 2:
            comp.wait_event(ev["outp"][b])           # step i - 2's output has left od[b]
        y = run(i, xd[b], ld[b], od[b])
        if y is None:
            y = od[b]
        elif y is not od[b]:
            y.record_stream(copy)   # a tensor the layer allocated: not reused before its copy ends
        ev["done"][b].record(comp)
        copy.wait_event(ev["done"][b])
        with torch.cuda.stream(copy):
            oh[b].copy_(y, non_blocking=True)
            ev["outp"][b].record(copy)
    comp.wait_stream(copy)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def _event_ms(fn, n):
    """mean ms of n calls fn(i) on the current stream, CUDA events around them"""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(n):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def prefill_bench(b200q, layer, device, iters=5):
    """BASELINE config 4 on the tcgen05 prompt GEMMs: the routed experts' grouped up (ReLU^2) and down GEMMs over
    8192 tokens x top-6 (Zipf 1.1), and the Q8_0 GQA projections (q/k/v fused, then o) on the same 8192 tokens."""
    Tp = 8192
    g = torch.Generator().manual_seed(11)
    x = torch.randn(Tp, H, generator=g).to(torch.bfloat16).to(device)
    ridx = torch.from_numpy(zipf_routing(12, Tp, TOPK).reshape(-1)).to(device)
    pairs = Tp * TOPK
    counts, offsets, order = b200q.k_moe_group_large(ridx, E)
    y = torch.empty(pairs, H, dtype=torch.float32, device=device)
    # Q8_0 GQA weights (32 q heads / 8 kv heads x 128): int8 U{-127..127}, fp16 d per 32
    def q8(seed, n, k):
        r = np.random.default_rng(seed)
        qv = r.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
        d = r.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
        raw = np.concatenate([d.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1).reshape(-1)
        return b200q.tile_q8_tc(torch.from_numpy(raw).to(device), n, k)
    wqkv, wo = q8(21, 6144, H), q8(22, H, H)
    qkv = torch.empty(Tp, 6144, dtype=torch.float32, device=device)
    attn = torch.randn(Tp, H, generator=g).to(torch.bfloat16).to(device)
    o = torch.empty(Tp, H, dtype=torch.float32, device=device)

    def moe():
        b200q.moe_prompt(layer.up, layer.down, E, H, F, counts, offsets, order, TOPK, x, mo=y)

    def gqa():
        b200q.mma_q8_prompt(wqkv, 6144, H, x, y=qkv)
        b200q.mma_q8_prompt(wo, H, H, attn, y=o)

    res = {}
    s = torch.cuda.current_stream()
    for name, fn, flops in (("moe", moe, 2.0 * pairs * H * F * 2), ("gqa", gqa, 2.0 * Tp * H * (6144 + H))):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(iters):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        res[name] = (ms, flops / (ms * 1e-3) / 1e12)
    # the same GQA projections at decode sizes (M = 1 / 16 rows) on the t16 Q8_0 GEMV, GB/s over weights + x + y,
    # rotating 10 weight copies of q/k/v (267 MB, twice the L2), timed as a CUDA graph of 60 calls
    dec = {}
    copies = 10
    wd = []
    for c in range(copies):
        r = np.random.default_rng(40 + c)
        raw = np.concatenate([r.uniform(1e-3, 1e-2, (6144, H // 32)).astype(np.float16).view(np.uint8).reshape(6144, H // 32, 2),
                              r.integers(-127, 128, (6144, H // 32, 32), dtype=np.int8).view(np.uint8)], -1).reshape(-1)
        wd.append(b200q.tile_q8(torch.from_numpy(raw).to(device), 6144, H))
    for M in (1, 16):
        xd = torch.randn(M, H, generator=g).to(torch.bfloat16).to(device)
        yd = torch.empty(M, 6144, dtype=torch.float32, device=device)
        for i in range(3):
            b200q.mma_q8(wd[i % copies], 6144, H, xd, y=yd)
        torch.cuda.synchronize()
        ms = graph_ms(lambda i: b200q.mma_q8(wd[i % copies], 6144, H, xd, y=yd), 60)
        nbytes = 6144 * H * 34 // 32 + M * H * 2 + M * 6144 * 4
        dec[f"gqa_qkv_decode_M{M}_gbs"] = round(nbytes / (ms * 1e-3) / 1e9, 1)
    # the model's lm_head (Q8_0 131072 x 4096, 570 MB: larger than L2, no copies needed) at decode rows (M = 1 / 16, the
    # t16 GEMV) and verify windows (M = 128, the tcgen05 prompt GEMM): GB/s over weights + x + y, and TFLOPS
    r = np.random.default_rng(50)
    nl = 131072
    raw = np.concatenate([r.uniform(1e-3, 1e-2, (nl, H // 32)).astype(np.float16).view(np.uint8).reshape(nl, H // 32, 2),
                          r.integers(-127, 128, (nl, H // 32, 32), dtype=np.int8).view(np.uint8)], -1).reshape(-1)
    raw_d = torch.from_numpy(raw).to(device)
    del raw
    w16, wtc = b200q.tile_q8(raw_d, nl, H), b200q.tile_q8_tc(raw_d, nl, H)
    del raw_d
    for M in (1, 16, 128):
        xd = torch.randn(M, H, generator=g).to(torch.bfloat16).to(device)
        yd = torch.empty(M, nl, dtype=torch.float32, device=device)
        if M <= 16:
            fn = lambda i, xd=xd, yd=yd: b200q.mma_q8(w16, nl, H, xd, y=yd)
        else:
            fn = lambda i, xd=xd, yd=yd: b200q.mma_q8_prompt(wtc, nl, H, xd, y=yd)
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        ms = graph_ms(fn, 20) if M <= 16 else _event_ms(fn, 20)
        nbytes = nl * H * 34 // 32 + M * H * 2 + M * nl * 4
        dec[f"lm_head_M{M}_gbs"] = round(nbytes / (ms * 1e-3) / 1e9, 1)
        if M > 16:
            dec[f"lm_head_M{M}_tflops"] = round(2.0 * M * nl * H / (ms * 1e-3) / 1e12, 1)
    del w16, wtc
    err = b200q.device_error()
    cnt = counts.cpu().numpy()
    return {"workload": "BASELINE config 4: 8192 tokens x top-6 = 49152 rows over 128 IQ2_XXS experts (Zipf 1.1, "
                        "seeded permutation), 4096 -> 2048 -> 4096 ReLU^2; Q8_0 GQA q/k/v (fused 6144) + o on the "
                        "same 8192 tokens; the lm_head (Q8_0 131072 x 4096) at 1 / 16 decode rows and 128 verify rows",
            "arithmetic": "fp16 operands (scales folded, rounded once), fp32 accumulation: tcgen05.mma kind::f16",
            "moe_ms": round(res["moe"][0], 4), "moe_tflops": round(res["moe"][1], 1),
            "gqa_ms": round(res["gqa"][0], 4), "gqa_tflops": round(res["gqa"][1], 1), **dec,
            "hottest_expert_rows": int(cnt.max()), "device_error": err}


def full_layer(b200q, device, L):
    """layer copy L of make_layers: the packed up / down slabs of all experts and the shared expert (same seeds)"""
    up = b200q.repack_iq2(b200q.synth_iq2(1000 + 10 * L, E * F * (H // 256), device), E * F, H)
    down = b200q.repack_iq2(b200q.synth_iq2(1001 + 10 * L, E * H * (F // 256), device), E * H, F)
    su = b200q.repack_iq2(b200q.synth_iq2(1002 + 10 * L, F * (H // 256), device), F, H)
    sd = b200q.repack_iq2(b200q.synth_iq2(1003 + 10 * L, H * (F // 256), device), H, F)
    return up, down, su, sd


def ep_bench(b200q, rank, world, device, steps, warmup, prefill=True, clk=None):
    """the MoE layer expert-parallel over the ranks (128 / N experts a rank), each rank with its
    own tokens.  decode: 16 tokens a rank, uniform placement, fixed-capacity exchange, shared expert on every rank;
    GB/s = the touched experts' bytes over all ranks (+ activations) / the slowest rank's step time.  prefill: 8192
    tokens a rank, Zipf(1.1) routing, LPT placement with the hottest experts split; TFLOPS over all ranks."""
    from ep import ExpertParallelMoE, GraphedStep, LocalExperts, PeerDecodeMoE, Placement, SharedExpert, slice_slab
    dist = world > 1
    # decode exchange: "peer" (NVLink peer stores and loads, b200q_ep_peer_decode) or "nccl" (all-to-alls)
    exchange = os.environ.get("B200Q_EP_EXCHANGE", "peer")
    up_b, down_b = b200q.iq2_bytes(F, H), b200q.iq2_bytes(H, F)

    def barrier():
        if dist:
            torch.distributed.barrier()

    def max_ms(ms):
        if dist:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    res = {}
    # ---- decode ----------------------------------------------------------------------------------------------
    pl = Placement(E, world, seed=7)
    loc = pl.local[rank]
    layers, ex_ms = [], []
    for L in range(LAYERS):
        up, down, su, sd = full_layer(b200q, device, L)
        if exchange == "peer":
            moe = PeerDecodeMoE(pl, rank, world, H, F, T, TOPK, slice_slab(up, loc, up_b),
                                slice_slab(down, loc, down_b), su, sd, device=device)
        else:
            ex = LocalExperts(slice_slab(up, loc, up_b), slice_slab(down, loc, down_b), len(loc), H, F)
            moe = ExpertParallelMoE(pl, rank, world, H, TOPK, ex.decode,
                                    shared_fn=SharedExpert(su, sd, H, F, T, device), layout="capacity", device=device)
            moe.ex = ex
        del up, down
        layers.append(moe)
    torch.cuda.synchronize()
    xs_h, ls_h = make_batches(rank, device)
    xs = [x.to(device) for x in xs_h]
    ls = [l.to(device) for l in ls_h]

    # the step's tokens and logits (graph inputs), two pairs so that the end-to-end loop uploads the next step's
    # while the current one runs
    xin = [torch.empty(T, H, dtype=torch.bfloat16, device=device) for _ in range(2)]
    lin = [torch.empty(T, E, dtype=torch.bfloat16, device=device) for _ in range(2)]

    def eager_on(L, x, lg):
        if exchange == "peer":
            return layers[L](x, lg)
        ridx, rw = b200q.k_route(lg, TOPK)
        return layers[L](x, ridx, rw)

    def eager_step(L, b):
        return eager_on(L, xs[b], ls[b])

    # the step as a CUDA graph: no host read in the exchange, so the whole step (router, packing, the exchange, expert
    # kernels, combine) replays as one launch.  The device-resident loop replays a graph per (layer copy, batch) pair
    # it visits, over the batch's own buffers (no input copy in the timed region); the end-to-end loop a graph per
    # layer copy and input pair, over the buffers its host copies fill.  Every rank captures them in the same order.
    graphs, graphs_res = [], {}
    if os.environ.get("B200Q_EP_GRAPH", "1") != "0":
        span = LAYERS * BATCHES // math.gcd(LAYERS, BATCHES)
        for key in sorted({(i % LAYERS, i % BATCHES) for i in range(span)}):
            graphs_res[key] = GraphedStep(lambda L=key[0], b=key[1]: eager_on(L, xs[b], ls[b]), world)
        for p in range(2):
            xin[p].copy_(xs[0])
            lin[p].copy_(ls[0])
        graphs = [[GraphedStep(lambda L=L, p=p: eager_on(L, xin[p], lin[p]), world) for p in range(2)]
                  for L in range(LAYERS)]
    graphed = bool(graphs) and all(g.ok for gl in graphs for g in gl) and all(g.ok for g in graphs_res.values())

    def step(i):
        L, b = i % LAYERS, i % BATCHES
        if graphed:
            return graphs_res[(L, b)]()
        return eager_step(L, b)

    # bytes of a step of batch b over all ranks: every rank's touched local experts + its shared expert + activations
    step_bytes_b, rank_hits = [], []
    for b in range(BATCHES):
        ridx, _ = b200q.k_route(ls[b], TOPK)
        if dist:
            allr = [torch.empty_like(ridx) for _ in range(world)]
            torch.distributed.all_gather(allr, ridx)
        else:
            allr = [ridx]
        hit = np.unique(torch.cat(allr).cpu().numpy())
        n_hit = sum(len(pl.owners[e]) for e in hit)
        step_bytes_b.append((n_hit + world) * EXPERT_BYTES + world * (T * H * 2 + T * E * 2 + T * H * 4))
        rank_hits.append(sum(1 for e in hit if rank in pl.owners[e]))
    for i in range(warmup):
        step(i)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    if clk:
        clk.__enter__()
    ev0.record()
    for i in range(steps):
        step(warmup + i)
    ev1.record()
    torch.cuda.synchronize()
    if clk:
        clk.__exit__()
    barrier()
    ms = max_ms(ev0.elapsed_time(ev1))
    nbytes = sum(step_bytes_b[(warmup + i) % BATCHES] for i in range(steps))
    # a second pass with events around the exchanges and the local expert GEMVs
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in evs:
        e.record()
    acc = np.zeros(3)
    nprof = min(steps, 50)

    def alone(fn):
        """one piece of a step timed alone: every rank ready first, the GPU kept busy while the host enqueues (no
        launch gap inside the events)"""
        barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(400000)
        evs[4].record()
        fn()
        evs[5].record()
        torch.cuda.synchronize()
        return evs[4].elapsed_time(evs[5])

    for i in range(nprof if exchange == "peer" else 0):
        # after a full step every flag holds its epoch, so the local experts (with their flags) and the combine run
        # again without waiting; the dispatch alone publishes the next epoch on every rank, and the next full step
        # goes on from there
        L, b = (warmup + i) % LAYERS, (warmup + i) % BATCHES
        layers[L](xs[b], ls[b])
        t_exp = alone(lambda: layers[L](xs[b], ls[b], phases=2))
        t_comb = alone(lambda: layers[L](xs[b], ls[b], phases=4))
        t_disp = alone(lambda: layers[L](xs[b], ls[b], phases=1))
        acc += [t_disp, t_comb, t_exp]
    barrier()
    for i in range(nprof if exchange != "peer" else 0):   # eager, with events between the pieces
        moe = layers[(warmup + i) % LAYERS]
        moe.timing = evs[:4]
        inner = moe.expert_fn

        def timed(rows, lidx, n, inner=inner, **kw):
            evs[4].record()
            y = inner(rows, lidx, n, **kw)
            evs[5].record()
            return y
        moe.expert_fn = timed
        eager_step((warmup + i) % LAYERS, (warmup + i) % BATCHES)
        moe.expert_fn, moe.timing = inner, None
        torch.cuda.synchronize()
        acc += [evs[0].elapsed_time(evs[1]), evs[2].elapsed_time(evs[3]), evs[4].elapsed_time(evs[5])]
    acc /= nprof
    # end to end: every step copies its tokens and logits from pinned host memory and reads the output back, the
    # copies overlapped with the neighbouring steps (pipelined_e2e); step i replays the graph over input pair i & 1
    xh = [x.pin_memory() for x in xs_h]
    lh = [l.pin_memory() for l in ls_h]

    def e2e_run(i, x, lg, o):
        L = (warmup + i) % LAYERS
        return graphs[L][i & 1]() if graphed else eager_on(L, x, lg)

    barrier()
    e2e_ms = pipelined_e2e(e2e_run, xh, lh, steps, warmup, device, (T, H), bufs=list(zip(xin, lin)))
    barrier()
    e2e_ms = max_ms(e2e_ms)
    if exchange == "peer" and dist:   # each piece's slowest rank
        t = torch.tensor(acc, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        acc = t.cpu().numpy()
    errors = [m.error() for m in layers] if exchange == "peer" else []
    if exchange == "peer":
        pieces = {"exchange": "peer memory (NVLink stores and loads, no collective)",
                  "dispatch_ms": round(float(acc[0]), 5),
                  "combine_ms": round(float(acc[1]), 5),
                  "comm_ms": round(float(acc[0] + acc[1]), 5),
                  "comm_note": "each piece timed alone on every rank (no waiting on other ranks), the slowest rank's: "
                               "dispatch = routing + the int8 row stores to the owners + the flags; local experts = "
                               "prologue + fused up/down GEMVs + the flags; combine = the owners' output rows loaded "
                               "and summed.  The step (CUDA graph) minus their sum is the ranks' waiting on one "
                               "another and the launch overlap",
                  "peer_errors": int(np.bitwise_or.reduce(errors)) if errors else 0}
    else:
        pieces = {"exchange": "NCCL all_to_all_single, fixed capacity", "layout": "capacity",
                  "dispatch_plus_shared_ms": round(float(acc[0]), 5), "return_ms": round(float(acc[1]), 5),
                  "comm_ms": round(float(acc[0] + acc[1]), 5)}
    res["decode"] = {"gbs": round(nbytes / (ms * 1e-3) / 1e9, 2), "ms_per_step": round(ms / steps, 5),
                     "steps": steps, "experts_per_rank": len(loc), **pieces,
                     "local_experts_ms": round(float(acc[2]), 5), "step_bytes_mean": float(np.mean(step_bytes_b)),
                     "rank_local_expert_bytes": float(np.mean(rank_hits)) * EXPERT_BYTES,
                     "e2e_gbs": round(nbytes / (e2e_ms * 1e-3) / 1e9, 2),
                     "h2d_bytes_per_step": T * H * 2 + T * E * 2, "d2h_bytes_per_step": T * H * 4,
                     "cuda_graph": graphed}
    del graphs, graphs_res
    if exchange == "peer":   # collective: every rank unmaps, then frees
        for m in layers:
            m.close()
    del layers
    import gc
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    # ---- prefill -------------------------------------------------------------------------------------------
    if prefill:
        Tp = 8192
        calib = zipf_routing(999, 2048, TOPK, perm_seed=12)
        loads = np.bincount(calib.reshape(-1), minlength=E).astype(np.float64)
        plp = Placement(E, world, loads=loads, replicate=8 if world > 1 else 0)
        locp = plp.local[rank]
        up, down, _, _ = full_layer(b200q, device, 0)
        ex = LocalExperts(slice_slab(up, locp, up_b), slice_slab(down, locp, down_b), len(locp), H, F)
        del up, down
        # the exchange in one piece: a pipeline over pieces (B200Q_EP_CHUNKS) measured slower at 2 GPUs (815 / 774 / 630
        # TFLOPS for 1 / 2 / 4 pieces): the persistent GEMMs hold every SM, so NCCL's kernels wait for them
        chunks = int(os.environ.get("B200Q_EP_CHUNKS", "1"))
        moe = ExpertParallelMoE(plp, rank, world, H, TOPK, ex.prompt, layout="exact", device=device, chunks=chunks,
                                sm_reserve=int(os.environ.get("B200Q_EP_SM_RESERVE", "16")))
        g = torch.Generator().manual_seed(300 + rank)
        x = torch.randn(Tp, H, generator=g).to(torch.bfloat16).to(device)
        ridx = torch.from_numpy(zipf_routing(12 + 1000 * rank, Tp, TOPK, perm_seed=12)).to(device)
        rw = torch.full((Tp, TOPK), 1.0 / TOPK, device=device)
        for _ in range(2):
            moe(x, ridx, rw)
        iters = 5
        barrier()
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(iters):
            moe(x, ridx, rw)
        ev1.record()
        torch.cuda.synchronize()
        barrier()
        pms = max_ms(ev0.elapsed_time(ev1)) / iters
        # where a step's time goes (one more step, events between its pieces): routing + counts exchange + host read
        # + dispatch of the first piece, the local experts' GEMMs, the returns, and the combine
        parts = None
        if dist:   # (on one rank nothing is exchanged)
            pev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            moe.timing = pev[1:5]
            barrier()
            torch.cuda.synchronize()
            pev[0].record()
            moe(x, ridx, rw)
            pev[5].record()
            torch.cuda.synchronize()
            moe.timing = None
            t = torch.tensor([pev[i].elapsed_time(pev[i + 1]) for i in range(5)], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            parts = t.cpu().tolist()
        flops = world * 2.0 * Tp * TOPK * H * F * 2
        res["prefill"] = {"tflops": round(flops / (pms * 1e-3) / 1e12, 1), "ms": round(pms, 4),
                          "tokens_per_rank": Tp, "experts_per_rank": len(locp),
                          "expected_rank_imbalance": round(plp.imbalance(), 4),
                          "copies": int(sum(len(o) for o in plp.owners)), "layout": "exact", "pieces": chunks,
                          "step_parts_ms": None if parts is None else {
                              "route_counts_hostread": round(parts[0], 4), "dispatch_first_piece": round(parts[1], 4),
                              "experts_all_pieces": round(parts[2], 4), "returns": round(parts[3], 4),
                              "combine": round(parts[4], 4),
                              "note": "one step with events between its pieces, each the slowest rank's"},
                          "step": "dispatch + group + tcgen05 up/down + return + combine"}
        del moe, ex
        torch.cuda.empty_cache()
    res["device_error"] = b200q.device_error()
    return res


def nvfp4_bench(b200q, device, iters=20):
    """the NVFP4 Mamba-2 projections, in_proj 4096 -> 18560 and out_proj 8192 -> 4096 (e2m1 codes
    U{0..15}, e4m3 scales U[0.5, 2] per 16, an fp32 tensor scale), activations bf16 N(0, 1).  M <= 16: the t16 decode
    GEMV, GB/s over weights + x + y, rotating weight copies of twice the L2 (6 of in_proj, 14 of out_proj), timed as a
    CUDA graph of 60 calls.  M >= 512: quant_nv4_rows + the block-scaled fp4 tcgen05 GEMM, TFLOPS of the GEMM alone
    and of quantiser + GEMM, each timed as a CUDA graph of `iters` calls."""
    shapes = {"in_proj": (18560, 4096), "out_proj": (4096, 8192)}
    ncopies = {"in_proj": 6, "out_proj": 14}
    g = torch.Generator(device="cpu").manual_seed(31)
    W = {}
    for name, (n, k) in shapes.items():
        W[name] = []
        for c in range(ncopies[name]):
            q = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g).to(device)
            sc = (torch.rand(n, k // 16, generator=g) * 1.5 + 0.5).to(torch.float8_e4m3fn).view(torch.uint8).to(device)
            W[name].append((b200q.tile_nv4(q, sc, n, k), b200q.tile_nv4w(q, sc, n, k) if c == 0 else None))
    s2 = 0.01
    out = {}
    # the decode GEMVs of both matrices first, then the prompt GEMMs: a GEMV timed right after seconds of
    # back-to-back fp4 GEMMs runs on a GPU held at its power cap (out_proj M = 1 measured 7 % lower there)
    for name, (n, k) in shapes.items():
        copies = ncopies[name]
        for M in (1, 16):
            x = torch.randn(M, k, generator=g).to(torch.bfloat16).to(device)
            y = torch.empty(M, n, device=device)
            for i in range(3):
                b200q.mma_nv4(W[name][i % copies][0], s2, n, k, x, y=y)
            torch.cuda.synchronize()
            ms = graph_ms(lambda i: b200q.mma_nv4(W[name][i % copies][0], s2, n, k, x, y=y), 60)
            nbytes = n * k // 2 + n * k // 16 + M * k * 2 + M * n * 4
            out[f"{name}_M{M}_gbs"] = round(nbytes / (ms * 1e-3) / 1e9, 1)
    for name, (n, k) in shapes.items():
        for M in (512, 4096):
            x = torch.randn(M, k, generator=g).to(torch.bfloat16).to(device)
            rows = b200q.quant_nv4_rows(x)
            y = torch.empty(M, n, device=device)
            wt = W[name][0][1]
            for _ in range(3):
                b200q.quant_nv4_rows(x, out=rows)
                b200q.mma_nv4_fp4(wt, s2, n, k, rows, M, y=y)
            torch.cuda.synchronize()
            # as CUDA graphs of `iters` calls: at M = 512 a call is some 10-40 us of GPU time, about what the Python
            # side of a launch takes, so launch-by-launch timing would measure the host
            gemm_ms = graph_ms(lambda i: b200q.mma_nv4_fp4(wt, s2, n, k, rows, M, y=y), iters)

            def both(i):
                b200q.quant_nv4_rows(x, out=rows)
                b200q.mma_nv4_fp4(wt, s2, n, k, rows, M, y=y)
            both_ms = graph_ms(both, iters)
            fl = 2.0 * M * n * k
            out[f"{name}_M{M}_tflops"] = round(fl / (gemm_ms * 1e-3) / 1e12, 1)
            out[f"{name}_M{M}_with_quant_tflops"] = round(fl / (both_ms * 1e-3) / 1e12, 1)
    out["device_error"] = b200q.device_error()
    out["fp4_peak_tflops"] = 9000.0
    out["fp4_peak_kind"] = "nominal dense FP4 (no measured FP4 figure on this pool)"
    out["workload"] = ("BASELINE config 3: NVFP4 in_proj 4096->18560 and out_proj 8192->4096; M 1/16 on the decode "
                       "GEMV (fp16 mma.sync, exact e2m1*e4m3 operands), M 512/4096 on tcgen05.mma kind::mxf4nvf4")
    return out


def make_batches(rank, device):
    g = torch.Generator().manual_seed(77 + rank)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(BATCHES)]
    ls = [torch.randn(T, E, generator=g).to(torch.bfloat16) for _ in range(BATCHES)]
    return xs, ls


def step_bytes(ridx_np):
    """algorithmic bytes of one step: distinct routed experts + the shared one, read once; x, logits, output."""
    distinct = len(np.unique(ridx_np))
    return (distinct + 1) * EXPERT_BYTES + T * H * 2 + T * E * 2 + T * H * 4, distinct


def run_ep(args, rank, world, local_rank):
    """N > 1: BASELINE config 5, the MoE layer expert-parallel over the ranks (see ep_bench); rank 0 prints."""
    import b200q
    import datetime
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    # one nvidia-smi sampler (on local rank 0) for all the node's ranks: a poller per rank stalls the launches
    clk = Clocks(",".join(str(i) for i in range(int(os.environ.get("LOCAL_WORLD_SIZE", world))))) if local_rank == 0 else None
    r = ep_bench(b200q, rank, world, device, args.steps, args.warmup, prefill=args.prefill, clk=clk)
    line = None
    if rank == 0:
        d = r["decode"]
        peak, peak_kind = peaks()
        ach = d["rank_local_expert_bytes"] / (d["local_experts_ms"] * 1e-3) / 1e9 if d["local_experts_ms"] else None
        line = {
            "metric": METRIC, "value": d["gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": d["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "BASELINE config 5 (decode): the config-2 MoE layer expert-parallel over N GPUs, "
                                   "128/N experts a GPU, 16 tokens a GPU, token rows dispatched (int8, the rows the "
                                   "GEMVs read) and outputs combined (bf16) over NVLink peer memory (NCCL all-to-alls "
                                   "of bf16 rows with B200Q_EP_EXCHANGE=nccl)",
                       "tokens_per_gpu": T, "hidden": H, "experts": E, "topk": TOPK, "ffn": F, "shared_experts": 1,
                       "l2": f"{LAYERS} rotating layer copies and {BATCHES} token batches",
                       "parallelism": f"ep{world}"},
            "hbm_fraction": round(d["gbs"] / world / peak, 4),
            "roofline": {"bound": "hbm", "kernel": "local expert GEMVs (int8 up + down) on rank 0",
                         "achieved": round(ach, 1) if ach else None, "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4) if ach else None, "traffic": None, "peak_kind": peak_kind},
            "cpu_baseline": None,
            "cpu_baseline_note": "the CPU oracle is timed at N=1 only",
            "e2e": {"value": d["e2e_gbs"], "unit": "GB/s", "h2d_bytes_per_step": d["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": d["d2h_bytes_per_step"]},
            # peer exchange: dispatch, expert prologue, fused up/down GEMV, combine a step
            "gpu_launches": (4 if d.get("exchange", "").startswith("peer") else 9) * args.steps,
            "clocks": clk.summary() if clk else None,
            "ep": r,
        }
        if "prefill" in r:
            line["prefill"] = r["prefill"]
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()
    return line


def run_ours(args, rank, world, local_rank):
    import b200q
    if world > 1:
        return run_ep(args, rank, world, local_rank)
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = world > 1
    if dist:
        import torch.distributed as td
        import datetime
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    layers = make_layers(b200q, device)
    xs_h, ls_h = make_batches(rank, device)
    xs = [x.to(device) for x in xs_h]
    ls = [l.to(device) for l in ls_h]
    out = torch.empty(T, H, dtype=torch.float32, device=device)
    ridx = [torch.empty(T, TOPK, dtype=torch.int32, device=device) for _ in range(BATCHES)]
    rw = torch.empty(T, TOPK, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream()

    def step(i, **kw):
        layers[i % LAYERS](xs[i % BATCHES], ls[i % BATCHES], out=out, ridx=ridx[i % BATCHES], rw=rw, **kw)

    def barrier():
        if dist:
            torch.distributed.barrier()

    for i in range(BATCHES):      # one untimed pass over every batch records its routing for the byte count
        step(i)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    byts = [step_bytes(r.cpu().numpy()) for r in ridx]

    # ---- the timed region: K steps, device-timed with events, barrier + synchronize on both sides
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the K-step region is repeated R times (R chosen so the repeats span about half a second, at least 5) and the
    # median is the value; the clock sampler runs across all of them
    ev0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    ev1.record(stream)
    torch.cuda.synchronize()
    est = max(ev0.elapsed_time(ev1), 1e-3)
    reps = int(min(500, max(5, 500.0 / est)))
    runs = []
    with Clocks(local_rank) as clk:
        for _ in range(reps):
            barrier()
            torch.cuda.synchronize()
            ev0.record(stream)
            for i in range(args.steps):
                step(args.warmup + i)
            ev1.record(stream)
            torch.cuda.synchronize()
            barrier()
            runs.append(ev0.elapsed_time(ev1))
    ms = float(np.median(runs))
    if dist:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    timed = {"repeats": reps, "steps_each": args.steps, "ms_median": round(ms, 5), "ms_min": round(min(runs), 5),
             "ms_max": round(max(runs), 5), "value_is": "the median repeat"}
    total_bytes = sum(byts[(args.warmup + i) % BATCHES][0] for i in range(args.steps))
    gbs_rank = total_bytes / (ms * 1e-3) / 1e9
    value = gbs_rank * world      # every rank does the same amount of work; the time is the max over ranks

    # ---- the layer kernel's own duration: the layer is one launch (decode_layer_k: router, grouping, the int8 rows
    # of x, up with relu^2, down, combine); a second pass with events around each launch (events between launches stop
    # the programmatic overlap with the next step, so this is the kernel alone, ramp included)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for e in evs:
        e.record(stream)      # torch creates the CUDA event on its first record
    kern_ms, kern_bytes = [], []
    nprof = max(args.steps, 4)
    for i in range(nprof):
        step(args.warmup + i, stage_events=evs)
        torch.cuda.synchronize()
        kern_ms.append(evs[0].elapsed_time(evs[4]))
        kern_bytes.append(byts[(args.warmup + i) % BATCHES][0])
    mean_distinct = np.mean([byts[(args.warmup + i) % BATCHES][1] for i in range(nprof)])
    dom_ms = float(np.mean(kern_ms))
    dom_bytes = float(np.mean(kern_bytes))
    peak, peak_kind = peaks()
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9

    # ---- e2e: the public API with host buffers (pinned), H2D of x and logits, D2H of the output, every step; the
    # copies overlapped with the neighbouring steps' kernels (pipelined_e2e), as a serving loop runs them
    xh = [x.pin_memory() for x in xs_h]
    lh = [l.pin_memory() for l in ls_h]
    barrier()
    e2e_ms = pipelined_e2e(lambda i, xd, ld, od: layers[(args.warmup + i) % LAYERS](xd, ld, out=od), xh, lh,
                           args.steps, args.warmup, device, (T, H))
    barrier()
    if dist:
        t = torch.tensor([e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_gbs = total_bytes / (e2e_ms * 1e-3) / 1e9 * world

    line = None
    if rank == 0:
        pre = prefill_bench(b200q, layers[0], device) if args.prefill else None
        if pre:
            bf16_peak = 1590.0
            pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
            if os.path.exists(pk):
                with open(pk) as f:
                    bf16_peak = float(json.load(f).get("bf16_tflops", bf16_peak))
            pre["peak_tflops"] = bf16_peak
            pre["peak_kind"] = "measured cuBLAS bf16 burst (fp16 runs at the same dense rate)"
            pre["moe_frac"] = round(pre["moe_tflops"] / bf16_peak, 4)
            pre["gqa_frac"] = round(pre["gqa_tflops"] / bf16_peak, 4)
        cpu = cpu_baseline(threads=os.cpu_count() or 1, min_seconds=args.cpu_seconds,
                           single_seconds=max(1.0, args.cpu_seconds / 2))
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config2(),
            "routing": {"mean_distinct_experts": round(float(mean_distinct), 2)},
            "timed_region": timed,
            "hbm_fraction": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "kernel": "decode_layer_k (the whole layer, one launch)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": round(dom_bytes * LAYER_TRAFFIC_CAPTURED[0] / LAYER_TRAFFIC_CAPTURED[1]),
                         "traffic_source": LAYER_TRAFFIC_SOURCE,
                         "algorithmic_bytes": round(dom_bytes), "peak_kind": peak_kind,
                         "kernel_ms": round(dom_ms, 5)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": T * H * 2 + T * E * 2,
                    "d2h_bytes_per_step": T * H * 4,
                    "copies": "every step's inputs host -> device and output device -> host inside the timed region, "
                              "on a copy stream overlapped with the neighbouring steps' kernels (double-buffered)"},
            "gpu_launches": args.steps,   # one decode_layer_k launch a step
            "clocks": clk.summary(),
        }
        if pre:
            line["prefill"] = pre
        line["ep"] = ep_bench(b200q, 0, 1, device, min(args.steps, 500), args.warmup, prefill=args.prefill)
        line["libbolt_shapes"] = libbolt_shapes("ours", device)
        try:
            line["ckpt"] = ckpt_bench(b200q, device)["ckpt"]
        except OSError as e:   # a measurement beside the line (it needs 0.6 GB of scratch disk)
            line["ckpt"] = {"unavailable": str(e)}
        if args.prefill:
            line["nvfp4"] = nvfp4_bench(b200q, device)
    if dist:
        torch.distributed.destroy_process_group()
    return line


_CPU_LAYER = {}


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


def _cpu_layer():
    """The config-2 layer for the CPU oracle: all 128 experts + the shared one of layer copy 0, made by the oracle's
    statement of the seeded generator from the GPU arm's seeds (the same bytes), without the product library."""
    if not _CPU_LAYER:
        O = _oracle()
        _CPU_LAYER["up"] = O.synth_iq2(1000, E * F * (H // 256))
        _CPU_LAYER["down"] = O.synth_iq2(1001, E * H * (F // 256))
        _CPU_LAYER["su"] = O.synth_iq2(1002, F * (H // 256))
        _CPU_LAYER["sd"] = O.synth_iq2(1003, H * (F // 256))
    return _CPU_LAYER


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def _cpu_passes(threads, min_seconds, max_passes, seed=5):
    O = _oracle()
    O.set_threads(threads)
    L = _cpu_layer()
    g = torch.Generator().manual_seed(seed)
    nbytes, passes, t0 = 0, 0, time.perf_counter()
    while passes < max_passes and (passes == 0 or time.perf_counter() - t0 < min_seconds):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        lg = torch.randn(T, E, generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        _, ridx, _ = O.moe_layer(x, lg, L["up"], L["down"], L["su"], L["sd"], T, H, F, E, TOPK, mode=0)
        nbytes += (len(np.unique(ridx)) + 1) * EXPERT_BYTES + T * H * 2 + T * E * 2 + T * H * 4
        passes += 1
    return nbytes, passes, time.perf_counter() - t0


def cpu_baseline(threads, min_seconds=10.0, max_passes=1000, single_seconds=None):
    """The CPU oracle (the int8-per-32 arithmetic of libbolt's expert kernels) on the config-2 layer: whole 16-token
    passes repeated until `min_seconds` have gone by, OpenMP over rows with `threads` threads; GB/s over each pass's
    touched experts, as the GPU line counts them.  With single_seconds, also one thread alone for that long."""
    nbytes, passes, dt = _cpu_passes(threads, min_seconds, max_passes)
    out = {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": f"{passes} passes of the 16-token config-2 layer in {dt:.1f} s (CPU oracle, int8-per-32 "
                     f"arithmetic, OpenMP over rows, {threads} threads)",
           "nproc": os.cpu_count(), "cpu_model": cpu_model()}
    if single_seconds:
        nb1, p1, dt1 = _cpu_passes(1, single_seconds, max_passes, seed=6)
        out["single_thread"] = {"value": round(nb1 / dt1 / 1e9, 3), "unit": "GB/s", "cores": 1,
                                "sample": f"{p1} passes in {dt1:.1f} s on one thread"}
    return out


def run_reference(args, rank, world):
    """The reference arm: libbolt has no CPU implementation of this path, so its arithmetic is timed through the CPU
    oracle (kind "port") on the host cores, a step being one 16-token pass of the same layer; the run is bounded
    (warm-up passes, then `steps` passes or about a minute, whichever ends first)."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    cpu_baseline(threads, min_seconds=0.0, max_passes=min(args.warmup, 3))
    c = cpu_baseline(threads, min_seconds=60.0, max_passes=args.steps)
    v = c["value"]
    lb = None
    if torch.cuda.is_available() and os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libbolt_ref.so")):
        try:
            lb = libbolt_shapes("reference", torch.device("cuda", 0))
        except Exception as e:   # a measurement beside the line: its failure does not take the line down
            lb = {"unavailable": f"{type(e).__name__}: {e}"}
    return {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "libbolt_gpu": lb,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "impl": "reference",
            "config": config2(),
            "cpu_baseline": c,
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def decode_only(b200q, device, steps, warmup):
    """The config-2 decode layer alone, `warmup` then `steps` steps over the --layers copies, timed with events (the
    small case the profiling commands capture)."""
    layers = make_layers(b200q, device)
    xs_h, ls_h = make_batches(0, device)
    xs = [x.to(device) for x in xs_h]
    ls = [l.to(device) for l in ls_h]
    out = torch.empty(T, H, dtype=torch.float32, device=device)
    ridx = [torch.empty(T, TOPK, dtype=torch.int32, device=device) for _ in range(BATCHES)]
    for i in range(warmup):
        layers[i % LAYERS](xs[i % BATCHES], ls[i % BATCHES], out=out, ridx=ridx[i % BATCHES])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        layers[i % LAYERS](xs[i % BATCHES], ls[i % BATCHES], out=out, ridx=ridx[i % BATCHES])
    e1.record()
    torch.cuda.synchronize()
    nb = sum(step_bytes(ridx[i % BATCHES].cpu().numpy())[0] for i in range(steps))
    ms = e0.elapsed_time(e1)
    return {"decode": {"gbs": round(nb / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms / steps, 5),
                       "layers": LAYERS, "device_error": b200q.device_error()}}


# libbolt's routed experts are compiled for its model: a latent of 1024 and TOPN = 9 (bolt_common.h:25,
# bolt_kernels.cu:682-695); the comparison runs them there, with this layer's 128 experts and FFN width 2048
LB_T, LB_E, LB_W, LB_LATENT, LB_TOPN = 16, 128, 2048, 1024, 9


def libbolt_shapes(kind, device, iters=50):
    """libbolt's operator launchers at libbolt's own shapes, on the B200: kind "reference" times libbolt's kernels
    (engine/bolt_kernels.cu and bolt_mma.cu built for sm_100a into oracle/_ref, the reference arm only); "ours" times
    this engine's shims of the same names and signatures (include/b200q_bolt.h, through the shim harness).  Both get the
    same seeded inputs (weights from the seeded generator, routing from each side's k_route, which agree index for
    index) and the same timed loop (`iters` launches on a stream, CUDA events, weight copies rotated past the L2).
    Returns GB/s of weights streamed a launch for: moe_up / moe_down (16 tokens, 128 experts, top-9, width 2048,
    latent 1024), mma_nv4 (in_proj 18560 x 4096, 1 and 16 rows), mma_q8 (q/k/v 6144 x 4096, 1 and 16 rows), mma_iq2
    (the shared expert's up, 2048 x 4096, 16 rows)."""
    import ctypes
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    if kind == "reference":
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        import refbind as R
        L = R.lib()

        def run(name, *a):
            R.call("ref_" + name, *a)
        synth = lambda seed, nb: torch.from_numpy(O.synth_iq2(seed, nb).reshape(-1)).to(device)
        tile_bytes = lambda f, n, k: (L.ref_tile_bytes(f, n, k), L.ref_tile_scale_bytes(f, n, k))
        time_moe, time_mma = L.ref_time_moe, L.ref_time_mma
    else:
        import b200q
        path = os.path.join(ROOT, "tests", "_build", "libbolt_shim_harness.so")
        if not os.path.exists(path):
            return {"unavailable": "the shim harness is not built (tests/build_harness.py)"}
        L = ctypes.CDLL(path)
        L.hs_tile_bytes.restype, L.hs_tile_bytes.argtypes = sz, [i32, i32, i32, i32]
        L.hs_time_moe.restype = L.hs_time_mma.restype = f32
        L.hs_time_moe.argtypes = [i32, i32, i32, vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32]
        L.hs_time_mma.argtypes = [i32, i32, i32, vp, vp, f32, i32, i32, vp, vp, i32]
        names = {"repack_iq2": ("hs_repack_iq2", [vp, vp, vp, vp, sz, i32]),
                 "route": ("hs_k_route", [vp, vp, i32, vp, vp, vp, i32, f32, i32]),
                 "moe_group": ("hs_k_moe_group", [vp, vp, i32, vp, vp, vp, vp, vp]),
                 "quant_rows": ("hs_k_quant_rows", [vp, vp, i32, vp, i32, vp, i32, i32, i32]),
                 "tile_nv4": ("hs_tile_nv4", [vp, vp, vp, vp, vp, i32, i32]),
                 "tile_q8": ("hs_tile_q8", [vp, vp, vp, vp, i32, i32]),
                 "tile_iq2": ("hs_tile_iq2", [vp, vp, vp, vp, i32, i32])}
        for fn, args in names.values():
            getattr(L, fn).restype, getattr(L, fn).argtypes = None, args

        def run(name, *a):
            getattr(L, names[name][0])(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), *a)
            torch.cuda.synchronize()
        synth = lambda seed, nb: b200q.synth_iq2(seed, nb, device)
        tile_bytes = lambda f, n, k: (L.hs_tile_bytes(f, 0, n, k), L.hs_tile_bytes(f, 1, n, k))
        time_moe, time_mma = L.hs_time_moe, L.hs_time_mma
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    ptrs = lambda ts: ctypes.cast((ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts]), ctypes.c_void_p)
    u8 = lambda n: torch.empty(n, dtype=torch.uint8, device=device)
    out = {}
    g = torch.Generator().manual_seed(61)
    # ---- routed experts: libbolt's planar slabs (its repack_iq2 / the shim's, into the same buffers), two copies
    T, E, W, K, topn = LB_T, LB_E, LB_W, LB_LATENT, LB_TOPN
    pairs = T * topn
    ups, downs = [], []
    for c in range(2):
        for proj, rows, k, dst in (("up", E * W, K, ups), ("down", E * K, W, downs)):
            raw = synth(6100 + 2 * c + (proj == "down"), rows * (k // 256))
            qs, d = u8(rows * (k // 256) * 64), u8(rows * (k // 256) * 2)
            run("repack_iq2", P(raw), P(qs), P(d), rows, k)
            dst.append((qs, d))
            del raw
    logits = torch.randn(T, E, generator=g).to(device)
    bias = torch.zeros(E, device=device)
    ridx = torch.empty(pairs, dtype=torch.int32, device=device)
    rw = torch.empty(pairs, device=device)
    run("route", P(logits), E, P(bias), P(ridx), P(rw), E, 1.0, T)
    # the work lists at libbolt's own sizes (bolt_host.cu:1076: TMAX * TOPN entries; the shim writes one item a slot)
    work = [torch.zeros(4096, dtype=torch.int32, device=device) for _ in range(4)] + \
        [torch.zeros(1, dtype=torch.int32, device=device)]
    run("moe_group", P(ridx), pairs, *[P(w) for w in work])
    x = torch.randn(T, K, generator=g).to(device)
    xq, xs = torch.empty(T, K, dtype=torch.int8, device=device), torch.empty(T, K // 32, device=device)
    run("quant_rows", P(x), K, P(xq), K, P(xs), K // 32, T, K)
    act = torch.empty(pairs, W, device=device)
    distinct = len(torch.unique(ridx))
    wbytes = distinct * W * (K // 256) * 66
    ms = time_moe(0, iters, 2, ptrs([q for q, _ in ups]), ptrs([d for _, d in ups]), W * (K // 256) * 64,
                  W * (K // 256), *[P(w) for w in work], P(xq), P(xs), P(act), W, pairs)
    out["moe_up_gbs"] = round(wbytes / (ms * 1e-3) / 1e9, 1) if ms > 0 else None
    aq, as_ = torch.empty(pairs, W, dtype=torch.int8, device=device), torch.empty(pairs, W // 32, device=device)
    run("quant_rows", P(act), W, P(aq), W, P(as_), W // 32, pairs, W)
    mo = torch.empty(pairs, K, device=device)
    ms = time_moe(1, iters, 2, ptrs([q for q, _ in downs]), ptrs([d for _, d in downs]), K * (W // 256) * 64,
                  K * (W // 256), *[P(w) for w in work], P(aq), P(as_), P(mo), W, pairs)
    out["moe_down_gbs"] = round(wbytes / (ms * 1e-3) / 1e9, 1) if ms > 0 else None
    out["moe_distinct_experts"] = distinct
    del ups, downs
    # ---- the tile GEMMs over weight copies past the L2
    rng = np.random.default_rng(62)
    for fmt, name, n, k, copies, rows_list in ((0, "mma_nv4", 18560, 4096, 4, (1, 16)), (1, "mma_q8", 6144, 4096, 6, (1, 16)),
                                              (2, "mma_iq2", 2048, 4096, 32, (16,))):
        cb, sb = tile_bytes(fmt, n, k)
        qts, sts = [], []
        for c in range(copies):
            qt, st = u8(cb), u8(sb)
            if fmt == 0:
                q = torch.from_numpy(rng.integers(0, 256, (n, k // 2), dtype=np.uint8)).to(device)
                sc = (torch.rand(n, k // 16, generator=g) * 1.5 + 0.5).to(torch.float8_e4m3fn).view(torch.uint8).to(device)
                run("tile_nv4", P(q), P(sc), P(qt), P(st), n, k)
                wb = n * k // 2 + n * k // 16
            elif fmt == 1:
                qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
                dv = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
                raw = torch.from_numpy(np.concatenate([dv.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)],
                                                      -1).reshape(-1)).to(device)
                run("tile_q8", P(raw), P(qt), P(st), n, k)
                wb = n * k // 32 * 34
            else:
                raw = synth(6200 + c, n * (k // 256))
                run("tile_iq2", P(raw), P(qt), P(st), n, k)
                wb = n * k // 256 * 66
            qts.append(qt)
            sts.append(st)
        for M in rows_list:
            xm = torch.randn(M, k, generator=g).to(device)
            ym = torch.empty(M, n, device=device)
            ms = time_mma(fmt, iters, copies, ptrs(qts), ptrs(sts), 0.01, n, k, P(xm), P(ym), M)
            out[f"{name}_M{M}_gbs"] = round(wb / (ms * 1e-3) / 1e9, 1) if ms > 0 else None
        del qts, sts
    out["shapes"] = ("moe_up/moe_down: 16 tokens, 128 experts, top-9, width 2048, latent 1024; mma_nv4 18560 x 4096; "
                     "mma_q8 6144 x 4096; mma_iq2 2048 x 4096; GB/s of weights a launch")
    torch.cuda.synchronize()
    return out


def ckpt_bench(b200q, device, reps=3):
    """Checkpoint ingestion (b200q_ckpt_*, b200q.Checkpoint.pack_moe_layer): one MoE layer of the model's schedule
    (layer 1: 240 IQ2_XXS experts, width 2048, latent 1024, and its shared expert, 5376 x 4096) under the model's own
    tensor names (language_model.backbone.layers.1.mixer...), written to two safetensors shards, then packed from the
    mapped shards into the device slabs.  GB/s = raw checkpoint bytes / wall time of the layer's packs, best of `reps`
    with the shards in the page cache (the first pass maps the shards and faults their pages in)."""
    import shutil
    layer, experts, width, latent, hidden, sw = 1, 240, 2048, 1024, 4096, 5376
    d = os.path.join(ROOT, "_build", "ckpt_bench")
    shutil.rmtree(d, ignore_errors=True)
    os.makedirs(d)
    try:
        names = b200q.moe_layer_tensor_names(layer, experts)
        weight_map, nbytes = {}, 0
        shards = {"experts": [], "shared": []}
        for e in range(experts):
            shards["experts"].append((names["up"][e], width, latent, 7000 + e))
            shards["experts"].append((names["down"][e], latent, width, 7000 + experts + e))
        shards["shared"] = [(names["shared_up"], sw, hidden, 7900), (names["shared_down"], hidden, sw, 7901)]
        for shard, tensors in shards.items():
            header, blobs, off = {}, [], 0
            for name, rows, k, seed in tensors:
                blob = b200q.synth_iq2_host(seed, rows * (k // 256)).tobytes()
                header[name] = {"dtype": "U8", "shape": [rows, k // 256, 66], "data_offsets": [off, off + len(blob)]}
                off += len(blob)
                blobs.append(blob)
                weight_map[name] = f"model-{shard}.safetensors"
            nbytes += off
            h = json.dumps(header).encode()
            h += b" " * ((8 - len(h) % 8) % 8)
            with open(os.path.join(d, f"model-{shard}.safetensors"), "wb") as f:
                f.write(len(h).to_bytes(8, "little"))
                f.write(h)
                for blob in blobs:
                    f.write(blob)
        with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": weight_map}, f)
        ck = b200q.Checkpoint(d)
        best = None
        for _ in range(reps + 1):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            packed = ck.pack_moe_layer(layer, experts, width, latent, device=device)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            best = dt if best is None or dt < best else best
            del packed
        ck.close()
        return {"ckpt": {"workload": "one MoE layer of the model's schedule (layer 1: 240 IQ2_XXS experts, width 2048, "
                                     "latent 1024, + the 5376-wide shared expert) under the model's tensor names, two "
                                     "safetensors shards, page-cache resident",
                         "bytes": nbytes, "ms": round(best * 1e3, 2), "gbs": round(nbytes / best / 1e9, 2),
                         "device_error": b200q.device_error()}}
    finally:
        shutil.rmtree(d, ignore_errors=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=4, help="layer copies rotated to defeat L2 (1 for small profiles)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="length of the CPU-baseline sample")
    ap.add_argument("--no-prefill", dest="prefill", action="store_false", help="skip the config-4 prefill GEMMs")
    ap.add_argument("--only", choices=["decode", "prefill", "nvfp4", "ep", "ckpt", "libbolt"], default=None,
                    help="run one sub-measurement on one GPU and print its object (for profiling)")
    args = ap.parse_args()
    global LAYERS
    LAYERS = max(1, args.layers)
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.only:
        import b200q
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        if args.only == "libbolt":
            line = {"libbolt_shapes": libbolt_shapes("ours", device)}
        elif args.only == "decode":
            line = decode_only(b200q, device, args.steps, args.warmup)
        elif args.only == "prefill":
            up, down, _, _ = full_layer(b200q, device, 0)
            line = prefill_bench(b200q, type("L", (), {"up": up, "down": down}), device)
        elif args.only == "nvfp4":
            line = nvfp4_bench(b200q, device)
        elif args.only == "ckpt":
            line = ckpt_bench(b200q, device)
        else:
            line = ep_bench(b200q, 0, 1, device, min(args.steps, 500), args.warmup)
    elif args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        line = run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
