"""Expert-parallel MoE across the GPUs of one box: the routed experts are sharded over the ranks, the tokens move by
all-to-all (NCCL over NVLink/NVSwitch on B200; the exchange itself runs on any torch.distributed backend).

libbolt runs every expert of a layer on its one GB10 (the MoE block of enqueue_block, bolt_host.cu:665-720: route,
group, up, down, combine).  Across ranks the same layer becomes, per step:

  1. route locally (b200q_route over this rank's tokens);
  2. give every (token, expert) pair a destination: the rank holding the expert (a replicated expert's pairs are
     split between its copies by token index);
  3. dispatch the pairs' token rows (bf16, hidden 8 KB) with all_to_all_single, and with them the expert's local
     index on the destination;
  4. run the grouped expert GEMMs on the received rows (decode: the int8 IQ2 GEMVs; prompt: the tcgen05 GEMMs);
  5. return the pair outputs (bf16 by default) with the reverse all_to_all_single;
  6. combine them with the router weights at the source (b200q_combine), adding the shared expert, which every
     rank runs for its own tokens while the dispatch is in flight.

Two exchange layouts:
  * "capacity" (decode): every rank sends a fixed `cap` rows to every peer (cap = the most pairs a rank can route,
    T * topk, so nothing is ever dropped); rows past a peer's real count carry the discard index and are never
    computed.  No device-to-host read, so a decode step can be captured in a CUDA graph.
  * "exact" (prompt): the per-peer counts are exchanged first and read on the host to size the transfers.

Placement: with uniform loads, a round-robin over a seeded permutation of the experts.  With expected loads, the
`replicate` hottest experts are cut into copies of at most half a rank's mean load, and the pieces are placed by LPT
(largest first, each to the least-loaded rank that does not hold that expert yet).
"""
import numpy as np
import torch
import torch.distributed as dist


class Placement:
    """Where the experts live.  owners[e]: the ranks holding expert e (pair with token t -> owners[e][t % n]);
    local[r]: the experts of rank r in local order; lidx[(e, r)]: e's index on rank r."""

    def __init__(self, E, world, loads=None, replicate=0, seed=0):
        self.E, self.world = E, world
        if loads is None:
            rng = np.random.default_rng(seed)
            perm = rng.permutation(E)
            owners = [[] for _ in range(E)]
            for i, e in enumerate(perm):
                owners[e].append(i % world)
            rank_load = np.zeros(world)
        else:
            # the `replicate` hottest experts are cut into copies of at most half a rank's mean load each; then LPT
            # over the pieces, largest first, each to the least-loaded rank that does not hold that expert yet
            loads = np.asarray(loads, np.float64)
            hot = set(np.argsort(-loads, kind="stable")[:replicate].tolist()) if world > 1 else set()
            piece_cap = loads.sum() / world / 2
            pieces = []
            for e in range(E):
                n = min(world, max(1, int(np.ceil(loads[e] / piece_cap)))) if e in hot and piece_cap > 0 else 1
                pieces += [(loads[e] / n, e)] * n
            owners = [[] for _ in range(E)]
            rank_load = np.zeros(world)
            for share, e in sorted(pieces, key=lambda t: (-t[0], t[1])):
                r = min((r for r in range(world) if r not in owners[e]), key=lambda r: (rank_load[r], r))
                owners[e].append(r)
                rank_load[r] += share
        self.owners = owners
        self.rank_load = rank_load
        self.local = [[] for _ in range(world)]
        self.lidx = {}
        for e in range(E):
            for r in owners[e]:
                self.lidx[(e, r)] = len(self.local[r])
                self.local[r].append(e)
        self.max_rep = max(len(o) for o in owners)

    def tables(self, device):
        """dest [E][max_rep], lidx [E][max_rep] (int64), nrep [E] as tensors for the device-side lookup."""
        dest = torch.zeros(self.E, self.max_rep, dtype=torch.int64)
        lid = torch.zeros(self.E, self.max_rep, dtype=torch.int64)
        nrep = torch.zeros(self.E, dtype=torch.int64)
        for e in range(self.E):
            nrep[e] = len(self.owners[e])
            for j in range(self.max_rep):
                r = self.owners[e][j % len(self.owners[e])]
                dest[e, j] = r
                lid[e, j] = self.lidx[(e, r)]
        return dest.to(device), lid.to(device), nrep.to(device)

    def imbalance(self):
        """max over mean of the expected per-rank loads"""
        m = self.rank_load.mean()
        return float(self.rank_load.max() / m) if m > 0 else 1.0


class ExpertParallelMoE:
    """One expert-parallel MoE layer on this rank.

    expert_fn(rows [R][H] (send dtype), lidx [R], n_local[, out_dtype]) -> [R][H]: the local experts applied to the
    received rows; rows whose lidx >= n_local are padding and may hold anything.  The tensor-operation form passes
    lidx as int64 and takes fp32 back; the fused CUDA form (capacity layout) passes an int32 index view of the received
    rows and asks for out_dtype = the send dtype.
    combine_fn(mo [pairs][H] fp32, rw [T][topk] fp32, shared [T][H] fp32 or None) -> [T][H] fp32; b200q_combine by
    default.  shared_fn(x) -> [T][H] fp32 or None: the shared expert on this rank's tokens."""

    def __init__(self, placement, rank, world, H, topk, expert_fn, shared_fn=None, combine_fn=None, group=None,
                 layout="capacity", send_dtype=torch.bfloat16, device=None, chunks=1, sm_reserve=16):
        self.p, self.rank, self.world, self.H, self.topk = placement, rank, world, H, topk
        # the exact layout's tokens in `chunks` consecutive pieces, exchanged and computed as a pipeline: the rows of
        # piece c + 1 travel while the experts run on piece c, and piece c's outputs return while piece c + 1 runs.
        # The same on every rank (the collectives must match); 1: one exchange each way
        self.chunks = max(1, int(chunks))
        # with more than one piece on CUDA, the SMs the persistent prompt GEMMs leave free while the pipeline runs, so
        # that the collectives' kernels can run beside them (b200q_set_sm_reserve)
        self.sm_reserve = int(sm_reserve)
        self.n_local = len(placement.local[rank])
        self.expert_fn, self.shared_fn = expert_fn, shared_fn
        self.combine_fn = combine_fn or _gpu_combine(topk)
        self._own_combine = combine_fn is None
        self.group, self.layout, self.send_dtype = group, layout, send_dtype
        self.device = device or torch.device("cpu")
        self.dest_t, self.lidx_t, self.nrep_t = placement.tables(self.device)
        # int32 copies for the fused capacity exchange on CUDA (b200q_ep_pack)
        self.dest_32, self.lidx_32, self.nrep_32 = (t.to(torch.int32) for t in (self.dest_t, self.lidx_t, self.nrep_t))
        self.timing = None   # optional: a list of 4 CUDA events (dispatch start/end, return start/end)
        # on CUDA the exchanges run in their fused forms (expert_fn then takes an out_dtype keyword, an int32 index view
        # in the capacity layout, and a topk keyword on one rank in the exact layout); False keeps the
        # tensor-operation form, which the CPU tests use
        self.fused = True

    # -- the pieces ----------------------------------------------------------------------------------------
    def _route(self, ridx, t0=0):
        """per pair: destination rank, local expert index there, the order that sorts pairs by destination, and
        the pair's position inside its destination's block; the tokens are t0, t0 + 1, ... (a replicated expert's pairs
        go to its copies by token index)"""
        e = ridx.reshape(-1).to(torch.int64)
        pairs = e.numel()
        tok = torch.arange(pairs, device=e.device) // self.topk
        rep = (tok + t0) % self.nrep_t[e]
        dest = self.dest_t[e, rep]
        lidx = self.lidx_t[e, rep]
        order = torch.sort(dest, stable=True).indices
        counts = torch.zeros(self.world, dtype=torch.int64, device=e.device).scatter_add_(0, dest, torch.ones_like(dest))
        starts = torch.cumsum(counts, 0) - counts
        pos = torch.arange(pairs, device=e.device) - starts[dest[order]]
        return dest, lidx, order, counts, pos, tok

    def _a2a(self, out, inp, out_splits=None, in_splits=None, async_op=False):
        if self.world == 1:   # one rank: the exchange is a copy (no process group needed)
            out.copy_(inp)
            return _Done()
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=async_op)

    def _capacity_fused(self, x, ridx, rw):
        """the capacity exchange on CUDA in four kernels around the two all-to-alls: b200q_ep_pack (route lookup,
        places, rows and local indices into the send buffer), the local experts on the received rows (their indices
        read from the rows; outputs written in the send dtype), b200q_ep_combine (the pairs' outputs gathered from the
        return buffer, weighted, plus the shared expert).  Same values as the tensor-operation form below."""
        import b200q
        T, H, topk = x.shape[0], self.H, self.topk
        cap = T * topk
        send, slot = b200q.ep_pack(x, ridx.to(torch.int32), self.dest_32, self.lidx_32, self.nrep_32, self.world, cap,
                                   self.n_local_max_peer(), self.send_dtype)
        recv = torch.empty_like(send)
        ev = self.timing
        if ev:
            ev[0].record()
        w1 = self._a2a(recv, send, async_op=True)
        shared = self.shared_fn(x) if self.shared_fn else None   # overlaps the dispatch
        w1.wait()
        if ev:
            ev[1].record()
        y = self.expert_fn(recv[:, :H], b200q.ep_index_view(recv, H), self.n_local, out_dtype=self.send_dtype)
        back = torch.empty_like(y)
        if ev:
            ev[2].record()
        self._a2a(back, y)
        if ev:
            ev[3].record()
        return b200q.ep_combine(back, slot, rw, topk, shared)

    def _exact_fused(self, x, ridx, rw):
        """the exact exchange on CUDA: the expert outputs come back in the send dtype and b200q_ep_combine gathers,
        weights and sums them from the return buffer.  On one rank nothing is exchanged: the local experts run on the
        tokens' pairs in place (expert_fn with topk) and b200q_combine sums their fp32 outputs."""
        import b200q
        if self.world == 1:
            lidx = self._route(ridx)[1]
            shared = self.shared_fn(x) if self.shared_fn else None
            mo = self.expert_fn(x, lidx, self.n_local, topk=self.topk)
            return b200q.k_combine(mo, rw.reshape(-1).contiguous(), self.topk, shared=shared)
        return self._exact(x, ridx, rw, fused=True)

    def _exact(self, x, ridx, rw, fused):
        """the exact exchange, as a pipeline over self.chunks pieces of consecutive tokens: every piece's per-peer
        counts in one exchange (one host read for all pieces), then per piece the rows (send dtype) and their local
        indices out, the local experts on the received rows, the outputs back; the next piece's rows are sent before
        this piece's experts run, so the transfers overlap the GEMMs.  Then one combine over all pairs (fused: the
        outputs gathered from the return buffer by b200q_ep_combine; otherwise the tensor-operation form)."""
        T, H, topk, C = x.shape[0], self.H, self.topk, self.chunks
        pairs = T * topk
        tb = [T * c // C for c in range(C + 1)]
        routes = [self._route(ridx[tb[c]:tb[c + 1]], tb[c]) for c in range(C)]
        counts = torch.stack([r[3] for r in routes], 1).contiguous()        # [world][C]
        rc = torch.empty_like(counts)
        self._a2a(rc.view(-1), counts.view(-1))
        send_splits = counts.t().tolist()                                   # [C][world]
        recv_splits = rc.t().tolist()
        got = torch.empty(pairs, H, dtype=self.send_dtype, device=x.device)
        ev = self.timing

        def dispatch(c):
            dest, lidx, order, _, _, tok = routes[c]
            send = x[tb[c]:tb[c + 1]].to(self.send_dtype).index_select(0, tok[order])
            send_l = lidx[order]
            nr = sum(recv_splits[c])
            recv = torch.empty(nr, H, dtype=self.send_dtype, device=x.device)
            recv_l = torch.empty(nr, dtype=torch.int64, device=x.device)
            w1 = self._a2a(recv, send, recv_splits[c], send_splits[c], async_op=True)
            w2 = self._a2a(recv_l, send_l, recv_splits[c], send_splits[c], async_op=True)
            return recv, recv_l, w1, w2

        if ev:
            ev[0].record()
        reserve = fused and C > 1 and x.is_cuda
        if reserve:
            import b200q
            b200q.lib().b200q_set_sm_reserve(self.sm_reserve)
        try:
            return self._exact_pieces(x, rw, fused, tb, routes, send_splits, recv_splits, got, dispatch)
        finally:
            if reserve:
                b200q.lib().b200q_set_sm_reserve(0)

    def _exact_pieces(self, x, rw, fused, tb, routes, send_splits, recv_splits, got, dispatch):
        """the pipeline of _exact over its pieces, and the combine"""
        T, H, topk, C = x.shape[0], self.H, self.topk, self.chunks
        pairs = T * topk
        ev = self.timing
        pend = dispatch(0)
        shared = self.shared_fn(x) if self.shared_fn else None   # overlaps the first piece's dispatch
        back = []
        for c in range(C):
            nxt = dispatch(c + 1) if c + 1 < C else None
            recv, recv_l, w1, w2 = pend
            w1.wait()
            w2.wait()
            if ev and c == 0:
                ev[1].record()
            if fused:
                y = self.expert_fn(recv, recv_l, self.n_local, out_dtype=self.send_dtype)
            else:
                y = self.expert_fn(recv, recv_l, self.n_local).to(self.send_dtype)
            if ev and c == C - 1:
                ev[2].record()
            back.append(self._a2a(got[tb[c] * topk:tb[c + 1] * topk], y, send_splits[c], recv_splits[c],
                                  async_op=True))
            pend = nxt
        for w in back:
            w.wait()
        if ev:
            ev[3].record()
        if fused:
            import b200q
            slot = torch.empty(pairs, dtype=torch.int32, device=x.device)   # pair p's row in got
            for c in range(C):
                p0, p1 = tb[c] * topk, tb[c + 1] * topk
                slot[p0:p1].scatter_(0, routes[c][2], torch.arange(p0, p1, dtype=torch.int32, device=x.device))
            return b200q.ep_combine(got, slot, rw, topk, shared)
        mo = torch.empty(pairs, H, dtype=torch.float32, device=x.device)
        for c in range(C):
            p0, p1 = tb[c] * topk, tb[c + 1] * topk
            mo[p0:p1].index_copy_(0, routes[c][2], got[p0:p1].to(torch.float32))
        return self.combine_fn(mo, rw, shared)

    def __call__(self, x, ridx, rw):
        """x [T][H] (this rank's tokens), ridx [T][topk] global expert ids, rw [T][topk] -> out [T][H] fp32"""
        T, H, topk = x.shape[0], self.H, self.topk
        pairs = T * topk
        if x.is_cuda and self.fused and self._own_combine:
            if self.layout == "capacity":
                return self._capacity_fused(x, ridx, rw)
            return self._exact_fused(x, ridx, rw)
        if self.layout != "capacity":
            return self._exact(x, ridx, rw, fused=False)
        dest, lidx, order, counts, pos, tok = self._route(ridx)
        xs = x.to(self.send_dtype)
        ev = self.timing
        if self.layout == "capacity":
            cap = pairs
            slot = dest[order] * cap + pos                       # where each sorted pair sits in the send buffer
            # one exchange: each row is the token's H values, then 16 bytes whose first 8 hold the local expert index
            pad = 16 // xs.element_size()
            send = torch.empty(self.world * cap, H + pad, dtype=self.send_dtype, device=x.device)
            send_l = _index_view(send, H)
            send_l.fill_(self.n_local_max_peer())
            send[:, :H].index_copy_(0, slot, xs.index_select(0, tok[order]))
            send_l.index_copy_(0, slot, lidx[order])
            recv = torch.empty_like(send)
            if ev:
                ev[0].record()
            w1 = self._a2a(recv, send, async_op=True)
            shared = self.shared_fn(x) if self.shared_fn else None   # overlaps the dispatch
            w1.wait()
            if ev:
                ev[1].record()
            recv_l = _index_view(recv, H)
            recv_l = torch.where(recv_l >= self.n_local, torch.full_like(recv_l, self.n_local), recv_l)
            y = self.expert_fn(recv[:, :H], recv_l, self.n_local).to(self.send_dtype)
            back = torch.empty_like(y)
            if ev:
                ev[2].record()
            self._a2a(back, y)
            if ev:
                ev[3].record()
            got = back.index_select(0, slot)                     # sorted pair order
        mo = torch.empty(pairs, H, dtype=torch.float32, device=x.device)
        mo.index_copy_(0, order, got.to(torch.float32))
        return self.combine_fn(mo, rw, shared)

    def n_local_max_peer(self):
        """the discard index every receiver maps to its own n_local (any index >= its expert count)"""
        return max(len(l) for l in self.p.local)


def _index_view(buf, H):
    """the int64 stored in bytes 0..7 after the H values of every row of buf [R][H + pad], as an [R] view"""
    n = 8 // buf.element_size()
    return buf[:, H:H + n].view(torch.int64).view(-1)


class _Done:
    def wait(self):
        pass


def _gpu_combine(topk):
    def f(mo, rw, shared):
        import b200q
        return b200q.k_combine(mo, rw.reshape(-1).contiguous(), topk, shared=shared)
    return f


class LocalExperts:
    """The routed experts one rank holds (packed rt32 slabs of its local experts, in local order) and their grouped
    GEMMs on received rows; lidx == n_local marks padding rows, which are grouped but never computed."""

    def __init__(self, up, down, n_local, H, F):
        self.up, self.down, self.n, self.H, self.F = up, down, n_local, H, F
        self._dec = None

    def decode(self, rows, lidx, n_local, out_dtype=torch.float32, topk=1):
        """b200q_moe_experts_decode: grouping, slot schedule and int8 rows in one launch, then the two GEMVs; with
        topk > 1, pair p (one lidx each) reads row p // topk"""
        import b200q
        if topk > 1:
            rows = rows.index_select(0, torch.arange(lidx.numel(), device=rows.device) // topk)
        if rows.shape[0] == 0 or self.n == 0:
            return torch.zeros(rows.shape[0], self.H, dtype=out_dtype, device=rows.device)
        if self._dec is None:
            self._dec = b200q.ExpertsDecode(self.up, self.down, self.n, self.H, self.F)
        return self._dec(rows, lidx, out_dtype=out_dtype)

    def prompt(self, rows, lidx, n_local, out_dtype=torch.float32, topk=1):
        """the tcgen05 prompt GEMMs over pairs: pair p (one lidx each, all local: the exact layout has no padding)
        reads row p // topk of rows; -> [pairs][H] in out_dtype"""
        import b200q
        pairs = lidx.numel()
        if pairs == 0 or self.n == 0:
            return torch.zeros(pairs, self.H, dtype=out_dtype, device=rows.device)
        out = torch.empty(pairs, self.H, dtype=out_dtype, device=rows.device)
        counts, offsets, order = b200q.k_moe_group_large(lidx.to(torch.int32), n_local + 1)
        return b200q.moe_prompt(self.up, self.down, n_local, self.H, self.F, counts, offsets, order, topk, rows, mo=out)


def slice_slab(slab, experts, expert_bytes):
    """the packed rt32 matrices of `experts` (in that order) out of a full slab, as one local slab"""
    if len(experts) == 0:
        return slab[:0].clone()
    return torch.cat([slab[e * expert_bytes:(e + 1) * expert_bytes] for e in experts])


class SharedExpert:
    """The shared expert on a rank's own decode tokens: the int8 GEMV pair over all T rows as one expert
    (b200q_moe_experts_decode with every row's local index 0)."""

    def __init__(self, up, down, H, F, T, device):
        self.up, self.down, self.H, self.F, self.T = up, down, H, F, T
        self.lidx = torch.zeros(T, dtype=torch.int32, device=device)
        self._dec = None

    def __call__(self, x):
        import b200q
        T = x.shape[0]
        if T != self.T:
            raise ValueError(f"SharedExpert was built for {self.T} tokens, got {T}")
        if self._dec is None:
            self._dec = b200q.ExpertsDecode(self.up, self.down, 1, self.H, self.F)
        return self._dec(x, self.lidx)


class PeerDecodeMoE:
    """The expert-parallel decode layer with its exchange over NVLink peer memory (b200q_ep_peer_decode): per step four
    launches on this rank's stream and no collective.  The dispatch stores each pair's token row straight into its
    owner's region, as the int8 row the GEMVs read; the owner's expert prologue waits for every sender's flag; the
    combine reads each pair's output row (ret_dtype: bf16, or fp32 for the fused layer's exact bytes) from its owner's
    region.  Nothing is read back to the host, so a step captures as a CUDA graph.

    The shared expert is the last local expert of every rank (run on that rank's own tokens inside the same GEMV
    launches as the routed ones).  Construction is collective (the ranks exchange their regions' IPC handles and check
    that they sit on distinct GPUs: ranks that wait on one another must never share a GPU); close() is collective too
    and must run before the process group is destroyed.  T (tokens a rank a step) is fixed: the region's layout
    depends on it, the same on every rank."""

    def __init__(self, placement, rank, world, H, F, T, topk, up_local, down_local, shared_up, shared_down,
                 group=None, ret_dtype=torch.bfloat16, device=None, route=0, bias=None, scale=1.0):
        import b200q
        self.p, self.rank, self.world, self.H, self.F, self.T, self.topk = placement, rank, world, H, F, T, topk
        self.group, self.ret_dtype, self.route, self.bias, self.scale = group, ret_dtype, route, bias, scale
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.n_local = len(placement.local[rank])
        self.discard = max(len(l) for l in placement.local) + 1   # above every rank's local experts + its shared one
        self.up = torch.cat([up_local, shared_up]).contiguous()
        self.down = torch.cat([down_local, shared_down]).contiguous()
        dest, lidx, nrep = placement.tables(self.device)
        self.dest, self.lidx, self.nrep = (t.to(torch.int32).contiguous() for t in (dest, lidx, nrep))
        L = b200q.lib()
        code = b200q.BF16 if ret_dtype == torch.bfloat16 else b200q.F32
        if world > 1:
            uuids = [None] * world
            dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid), group=group)
            if len(set(uuids)) != world:
                raise RuntimeError("the peer-memory exchange needs every rank on its own GPU")
        self.region = b200q.PeerRegion(L.b200q_ep_peer_region_bytes(world, T, H, topk, code), self.device)
        handles = [self.region.handle()] * world
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, self.region.handle(), group=group)
        ptrs = [self.region.ptr if r == rank else self.region.open(handles[r]) for r in range(world)]
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.state = torch.zeros(L.b200q_ep_peer_state_bytes(T, topk) // 4, dtype=torch.int32, device=self.device)
        nws = L.b200q_ep_peer_workspace_bytes(world, T, H, F, topk, self.n_local)
        self._ws = torch.empty(nws + 256, dtype=torch.uint8, device=self.device)
        self.ws = (self._ws.data_ptr() + (-self._ws.data_ptr()) % 256, nws)
        if world > 1:   # every mapping in place before any rank's first step
            dist.barrier(group=group)

    def __call__(self, x, logits, out=None, ridx=None, rw=None, phases=7):
        """x [T][H], logits [T][E] (this rank's tokens) -> out [T][H] fp32.  phases: the subset of the step's
        launches (bit 0 dispatch, bit 1 local experts + their flags, bit 2 combine), for timing the pieces."""
        import b200q
        if x.shape[0] != self.T or logits.shape[0] != self.T:
            raise ValueError(f"the layer was built for {self.T} tokens a step, got {x.shape[0]}")
        return b200q.ep_peer_decode(x, logits, self.topk, self.dest, self.lidx, self.nrep, self.region.ptr,
                                    self.peers, self.world, self.rank, self.n_local, self.discard, self.up, self.down,
                                    self.state, self.ws, self.H, self.F, ret_dtype=self.ret_dtype, out=out,
                                    route=self.route, bias=self.bias, scale=self.scale, ridx=ridx, rw=rw,
                                    phases=phases)

    def error(self, clear=True):
        """the bits the step's bounded waits recorded (0: none; bit 0 senders, bit 1 owners did not arrive)"""
        import b200q
        return b200q.ep_peer_error(self.state, clear)

    def close(self):
        """collective: unmap the other ranks' regions once every rank is done with its steps, then free this one once
        every rank has unmapped it"""
        if self.region is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        self.region.unmap()
        if self.world > 1:
            dist.barrier(group=self.group)
        self.region.free()
        self.region = None


class GraphedStep:
    """A decode step captured once as a CUDA graph and replayed.  With the capacity exchange the expert-parallel layer
    reads nothing back to the host, so router, packing, the NCCL all-to-alls, the expert kernels and the combine
    capture as one graph, which removes the per-launch host latency that dominates a 16-token step.  Every rank must
    build the same GraphedSteps in the same order (the warm-up runs the collectives eagerly); `ok` is agreed across
    the ranks before any replay, so either all ranks replay or all run eagerly.  Drop the object (and with it the
    graph's NCCL work) before destroying the process group."""

    def __init__(self, fn, world, group=None, warm=2):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        ok = 1
        self.g, self.out = None, None
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = fn()
            self.g, self.out = g, out
        except Exception:   # a capture the runtime refuses: this rank falls back, and so do the others below
            ok = 0
        torch.cuda.synchronize()
        if world > 1:
            t = torch.tensor([ok], dtype=torch.int32, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
            ok = int(t.item())
        self.ok = bool(ok)
        self.fn = fn
        if self.ok:   # the first replay carries one-time setup (the captured collectives'); keep it out of any timing
            self.g.replay()
            torch.cuda.synchronize()

    def __call__(self):
        if self.ok:
            self.g.replay()
            return self.out
        return self.fn()
