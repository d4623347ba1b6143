"""Host-side mirror of libbolt's operator interface over libb200q's C ABI (include/b200q.h).

The reference engine's operators are C++ launchers (engine/bolt_common.h:77-157): k_route, k_moe_group,
k_quant_rows, moe_up, moe_down, k_combine, mma_iq2, mma_nv4, mma_q8, quant_nv4_rows, repack_iq2, tile_*.  This module
gives the same operators by the same names, taking torch tensors for device memory and the current torch stream,
and calling the sm_100a kernels through ctypes.  Errors raise B200QError with libb200q's status (the reference
returns void and logs; its C ABI returns -1/-3).  There is no CPU fallback: without libb200q.so, or without a GPU,
every operator raises.
"""
import ctypes
import json
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
# the library: B200Q_LIB if set (like libbolt's TENSORFOLD_BOLT_LIB lookup, bolt_api.zig:128-140), else the in-place build
LIB_PATH = os.environ.get("B200Q_LIB") or os.path.join(HERE, "libb200q.so")

OK, EINVAL, ENOSPACE, ECUDA = 0, -1, -2, -3
F32, BF16 = 0, 1
ROUTE_SOFTMAX, ROUTE_SIGMOID = 0, 1

_LIB = None


class B200QError(RuntimeError):
    def __init__(self, status, what):
        self.status = status
        msg = lib().b200q_strerror(status).decode()
        if status == ECUDA:
            msg += f" (cudaError {lib().b200q_last_cuda_error()})"
        super().__init__(f"{what}: {msg}")


def lib():
    """The loaded libb200q.so (built in place by build.py; a missing library is an error, never a fallback)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libb200q.so is missing at {LIB_PATH}: run build.py (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, i64, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
        sig = {
            "b200q_abi": (i32, []), "b200q_last_cuda_error": (i32, []), "b200q_strerror": (ctypes.c_char_p, [i32]),
            "b200q_iq2_bytes": (sz, [i64, i32]), "b200q_iq2_pack": (i32, [vp, vp, i64, i32, vp]),
            "b200q_quant_rows": (i32, [vp, i32, i32, vp, i32, vp, i32, i32, i32, vp]),
            "b200q_route": (i32, [vp, i32, i32, vp, i32, i32, i32, i32, f32, vp, vp, vp]),
            "b200q_moe_group": (i32, [vp, i32, i32, vp, vp, vp, vp]),
            "b200q_combine": (i32, [vp, vp, vp, i32, i32, i32, vp, i32, vp]),
            "b200q_iq2_gemv": (i32, [vp, i32, i32, vp, vp, i32, vp, i32, i32, vp]),
            "b200q_iq2_chunk_dots": (i32, [vp, i32, i32, vp, i32, vp, vp]),
            "b200q_moe_up": (i32, [vp, i32, i32, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, vp]),
            "b200q_moe_up_q8": (i32, [vp, i32, i32, i32, vp, vp, vp, i32, vp, vp, vp, vp, vp]),
            "b200q_moe_down": (i32, [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp, i32, vp]),
            "b200q_moe_decode_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
            "b200q_moe_experts_workspace_bytes": (sz, [i32, i32, i32, i32]),
            "b200q_moe_experts_decode": (i32, [vp, i32, i32, i32, i32, i32, vp, i32, i32, vp, vp, vp, i32, i32, vp, sz,
                                               vp]),
            "b200q_ep_pack": (i32, [vp, i32, i32, i32, vp, i32, vp, vp, vp, i32, i32, i32, i32, vp, i32, i32, vp, vp]),
            "b200q_ep_combine": (i32, [vp, i32, i32, vp, vp, vp, i32, i32, i32, vp, i32, vp]),
            "b200q_ep_peer_region_bytes": (sz, [i32, i32, i32, i32, i32]),
            "b200q_ep_peer_state_bytes": (sz, [i32, i32]),
            "b200q_ep_peer_workspace_bytes": (sz, [i32, i32, i32, i32, i32, i32]),
            "b200q_peer_alloc": (i32, [sz, ctypes.POINTER(vp)]), "b200q_peer_free": (i32, [vp]),
            "b200q_peer_handle_bytes": (sz, []), "b200q_peer_export": (i32, [vp, ctypes.c_char_p]),
            "b200q_peer_open": (i32, [ctypes.c_char_p, ctypes.POINTER(vp)]), "b200q_peer_close": (i32, [vp]),
            "b200q_ep_peer_error": (i32, [vp, i32]),
            "b200q_set_sm_reserve": (i32, [i32]),
            "b200q_ep_peer_decode": (i32, [vp, i32, vp, i32, i32, i32, i32, i32, i32, i32, vp, f32, vp, vp, vp, i32,
                                           vp, vp, i32, i32, i32, i32, vp, vp, i32, vp, vp, sz, vp, i32, vp, vp, i32,
                                           vp]),
            "b200q_moe_decode": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, f32, vp, i32, vp, sz,
                                       vp, vp, vp, vp]),
            "b200q_synth_iq2_host": (None, [ctypes.c_uint64, i64, vp]),
            "b200q_synth_iq2": (i32, [ctypes.c_uint64, i64, vp, vp]),
            "b200q_nv4_bytes": (sz, [i64, i32]), "b200q_nv4_pack": (i32, [vp, vp, vp, i64, i32, vp]),
            "b200q_q8_bytes": (sz, [i64, i32]), "b200q_q8_pack": (i32, [vp, vp, i64, i32, vp]),
            "b200q_nv4_gemv_workspace_bytes": (sz, [i32, i32, i32]),
            "b200q_nv4_gemv": (i32, [vp, f32, i32, i32, vp, i32, i32, i32, vp, i32, vp, sz, vp]),
            "b200q_q8_gemv_workspace_bytes": (sz, [i32, i32, i32]),
            "b200q_q8_gemv": (i32, [vp, i32, i32, vp, i32, i32, i32, vp, i32, vp, sz, vp]),
            "b200q_moe_group_large": (i32, [vp, i32, i32, vp, vp, vp, vp, vp]),
            "b200q_moe_prompt_workspace_bytes": (sz, [i32, i32, i32, i32]),
            "b200q_moe_prompt": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, i32, i32, vp, i32, vp, i32, vp, vp, sz, vp]),
            "b200q_q8_tc_bytes": (sz, [i64, i32]),
            "b200q_q8_tc_pack": (i32, [vp, vp, i64, i32, vp]),
            "b200q_q8_gemm_workspace_bytes": (sz, [i32, i32]),
            "b200q_q8_gemm": (i32, [vp, i32, i32, vp, i32, i32, i32, vp, i32, vp, sz, vp]),
            "b200q_device_error": (i32, [i32]),
            "b200q_nv4_tc_bytes": (sz, [i64, i32]),
            "b200q_nv4_tc_pack": (i32, [vp, vp, vp, i64, i32, vp]),
            "b200q_nv4_rows_bytes": (sz, [i32, i32]),
            "b200q_quant_nv4_rows": (i32, [vp, i32, i32, i32, i32, vp, vp]),
            "b200q_nv4_gemm_workspace_bytes": (sz, [i32, i32, i32]),
            "b200q_nv4_gemm": (i32, [vp, i32, i32, f32, vp, i32, vp, i32, vp, sz, vp]),
            "b200q_ckpt_open": (vp, [ctypes.c_char_p]),
            "b200q_ckpt_close": (None, [vp]),
            "b200q_ckpt_count": (i64, [vp]),
            "b200q_ckpt_tensor": (i32, [vp, ctypes.c_char_p, ctypes.POINTER(vp), ctypes.POINTER(sz),
                                        ctypes.POINTER(i64), ctypes.POINTER(i32), ctypes.c_char_p]),
            "b200q_ckpt_staging_bytes": (sz, [i32, i32, i32]),
            "b200q_ckpt_pack_iq2_slab": (i32, [vp, ctypes.POINTER(ctypes.c_char_p), i32, i32, i32, vp, vp, sz, vp]),
            "b200q_ckpt_pack_nv4": (i32, [vp, ctypes.c_char_p, i32, i32, vp, ctypes.POINTER(f32), vp, sz, vp]),
            "b200q_ckpt_pack_q8": (i32, [vp, ctypes.c_char_p, i32, i32, vp, vp, sz, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _LIB = L
    return _LIB


def _p(t):
    """the device address of a CUDA tensor for the C ABI (None -> NULL).  Anything else is refused before any launch:
    a host tensor's address would reach a kernel."""
    if t is None:
        return None
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise B200QError(EINVAL, "operands of the C ABI must be CUDA tensors")
    return ctypes.c_void_p(t.data_ptr())


def _s(stream=None):
    return ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)


def _check(status, what):
    if status != OK:
        raise B200QError(status, what)


def _dev(t, name, rows=False):
    """a CUDA tensor, contiguous (rows=True: each row contiguous, rows at any 16-byte-multiple stride)"""
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise B200QError(EINVAL, f"{name} must be a CUDA tensor")
    if rows:
        if t.dim() != 2 or t.stride(1) != 1 or (t.stride(0) * t.element_size()) % 16:
            raise B200QError(EINVAL, f"{name} must be rows with contiguous elements and a 16-byte row stride")
    elif not t.is_contiguous():
        raise B200QError(EINVAL, f"{name} must be contiguous")
    return t


def _rows_any(t, name):
    """a CUDA tensor of rows, each row's elements contiguous, the rows at any pitch (x of the decode GEMVs)"""
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise B200QError(EINVAL, f"{name} must be a CUDA tensor")
    if t.dim() != 2 or t.stride(1) != 1:
        raise B200QError(EINVAL, f"{name} must be rows with contiguous elements")
    return t


def _dtype_code(t):
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise B200QError(EINVAL, f"unsupported activation dtype {t.dtype}")


# -------------------------------------------------------------------------------------------------------------
# load-time packing (repack_iq2 / load_slab, bolt_kernels.cu:1054-1068, bolt_host.cu:306-328)
# -------------------------------------------------------------------------------------------------------------
def iq2_bytes(n, k):
    return lib().b200q_iq2_bytes(n, k)


def repack_iq2(raw, n, k, out=None):
    """ggml IQ2_XXS blocks (uint8 CUDA tensor, [n][k/256][66] bytes) -> the rt32 device layout (same byte count)."""
    _dev(raw, "raw")
    if out is None:
        out = torch.empty(iq2_bytes(n, k), dtype=torch.uint8, device=raw.device)
    _check(lib().b200q_iq2_pack(_p(raw), _p(out), n, k, _s()), "repack_iq2")
    return out


def synth_iq2(seed, nblocks, device="cuda"):
    """BASELINE's synthetic IQ2_XXS blocks, generated on the device (the same bytes as synth_iq2_host)."""
    out = torch.empty(nblocks * 66, dtype=torch.uint8, device=device)
    _check(lib().b200q_synth_iq2(seed, nblocks, _p(out), _s()), "synth_iq2")
    return out


def synth_iq2_host(seed, nblocks):
    import numpy as np
    out = np.zeros(nblocks * 66, np.uint8)
    lib().b200q_synth_iq2_host(seed, nblocks, out.ctypes.data_as(ctypes.c_void_p))
    return out


# -------------------------------------------------------------------------------------------------------------
# router, grouping, activation quantisation, combine
# -------------------------------------------------------------------------------------------------------------
def k_quant_rows(x, q=None, s=None):
    """int8 per 32 (quant_rows_k): x [rows][k] fp32/bf16 (rows may be strided) -> q [rows][k] int8, s [rows][k/32]."""
    _dev(x, "x", rows=True)
    rows, k = x.shape
    q = torch.empty(rows, k, dtype=torch.int8, device=x.device) if q is None else q
    s = torch.empty(rows, k // 32, dtype=torch.float32, device=x.device) if s is None else s
    _check(lib().b200q_quant_rows(_p(x), _dtype_code(x), x.stride(0), _p(q), k, _p(s), k // 32, rows, k, _s()),
           "k_quant_rows")
    return q, s


def k_route(logits, topk, mode=ROUTE_SOFTMAX, bias=None, scale=1.0):
    """Router (route_k): logits [T][E] -> ridx [T][topk] int32, rw [T][topk] fp32."""
    _dev(logits, "logits")
    T, E = logits.shape
    ridx = torch.empty(T, topk, dtype=torch.int32, device=logits.device)
    rw = torch.empty(T, topk, dtype=torch.float32, device=logits.device)
    _check(lib().b200q_route(_p(logits), _dtype_code(logits), E, _p(bias), T, E, topk, mode, float(scale), _p(ridx),
                             _p(rw), _s()), "k_route")
    return ridx, rw


def k_moe_group(ridx, E):
    """Counting sort of the pairs by expert (moe_group_k): counts [E], offsets [E+1], order [pairs]."""
    _dev(ridx, "ridx")
    pairs = ridx.numel()
    counts = torch.empty(E, dtype=torch.int32, device=ridx.device)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=ridx.device)
    order = torch.empty(max(pairs, 1), dtype=torch.int32, device=ridx.device)
    _check(lib().b200q_moe_group(_p(ridx), pairs, E, _p(counts), _p(offsets), _p(order), _s()), "k_moe_group")
    return counts, offsets, order[:pairs]


def k_combine(mo, rw, topk, shared=None, out_dtype=torch.float32):
    """out[t] = sum_k rw[t][k] mo[t*topk+k] (+ shared[t]) (combine_k)."""
    _dev(mo, "mo")
    T = rw.numel() // topk
    H = mo.shape[-1]
    out = torch.empty(T, H, dtype=out_dtype, device=mo.device)
    _check(lib().b200q_combine(_p(mo), _p(rw), _p(shared), T, topk, H, _p(out), _dtype_code(out), _s()), "k_combine")
    return out


# -------------------------------------------------------------------------------------------------------------
# IQ2_XXS GEMVs over int8 rows
# -------------------------------------------------------------------------------------------------------------
def mma_iq2(w, n, k, xq, xs, epi=0):
    """Dense IQ2_XXS GEMV (mma_iq2 / moe_coop_dense): y [T][n] fp32 = W . x for the int8 rows xq/xs."""
    T = xq.shape[0]
    y = torch.empty(T, n, dtype=torch.float32, device=xq.device)
    _check(lib().b200q_iq2_gemv(_p(w), n, k, _p(_dev(xq, "xq")), _p(_dev(xs, "xs")), T, _p(y), n, epi, _s()), "mma_iq2")
    return y


def iq2_chunk_dots(w, n, k, xq):
    T = xq.shape[0]
    d = torch.empty(T, n, k // 32, dtype=torch.int32, device=xq.device)
    _check(lib().b200q_iq2_chunk_dots(_p(w), n, k, _p(_dev(xq, "xq")), T, _p(d), _s()), "iq2_chunk_dots")
    return d


def moe_up(slab, E, n, k, counts, offsets, order, topk, xq, xs, epi=1):
    pairs = order.numel()
    y = torch.empty(max(pairs, 1), n, dtype=torch.float32, device=xq.device)
    _check(lib().b200q_moe_up(_p(slab), E, n, k, _p(counts), _p(offsets), _p(order), topk, _p(xq), _p(xs), _p(y), n, epi,
                              _s()), "moe_up")
    return y[:pairs]


def moe_up_q8(slab, E, n, k, counts, offsets, order, topk, xq, xs):
    pairs = order.numel()
    aq = torch.empty(max(pairs, 1), n, dtype=torch.int8, device=xq.device)
    as_ = torch.empty(max(pairs, 1), n // 32, dtype=torch.float32, device=xq.device)
    _check(lib().b200q_moe_up_q8(_p(slab), E, n, k, _p(counts), _p(offsets), _p(order), topk, _p(xq), _p(xs), _p(aq),
                                 _p(as_), _s()), "moe_up_q8")
    return aq[:pairs], as_[:pairs]


def moe_down(slab, E, n, k, counts, offsets, order, aq, as_):
    pairs = order.numel()
    y = torch.empty(max(pairs, 1), n, dtype=torch.float32, device=aq.device)
    _check(lib().b200q_moe_down(_p(slab), E, n, k, _p(counts), _p(offsets), _p(order), _p(aq), _p(as_), _p(y), n, _s()),
           "moe_down")
    return y[:pairs]


class ExpertsDecode:
    """The routed experts of one rank of the expert-parallel decode layer (b200q_moe_experts_decode): the received
    rows through their local experts, up, relu^2, down.  The workspace grows to the largest row count seen."""

    def __init__(self, up, down, n_local, H, F):
        self.up, self.down, self.n, self.H, self.F = up, down, n_local, H, F
        self.buf, self.ptr, self.nbytes = None, None, 0

    def __call__(self, rows, lidx, y=None, out_dtype=torch.float32):
        """rows [R][H] fp32 or bf16 (each row contiguous, any row stride), lidx [R] int32 at any stride (n_local or
        more: padding) -> y [R][H] fp32 or bf16 (out_dtype; padding rows unwritten)"""
        _dev(rows, "rows", rows=True)
        R = rows.shape[0]
        y = torch.empty(R, self.H, dtype=out_dtype, device=rows.device) if y is None else y
        if R == 0:
            return y
        need = lib().b200q_moe_experts_workspace_bytes(R, self.H, self.F, self.n)
        if self.buf is None or self.nbytes < need or self.buf.device != rows.device:
            self.buf = torch.empty(need + 256, dtype=torch.uint8, device=rows.device)
            self.ptr = self.buf.data_ptr() + (-self.buf.data_ptr()) % 256
            self.nbytes = need
        li = lidx if lidx.dtype == torch.int32 else lidx.to(torch.int32)
        if li.dim() != 1 or li.numel() != R:
            raise B200QError(EINVAL, "lidx must hold one index a row")
        _check(lib().b200q_moe_experts_decode(_p(rows), _dtype_code(rows), rows.stride(0), R, self.H, self.F,
                                              _p(li), max(li.stride(0), 1), self.n, _p(self.up), _p(self.down), _p(y),
                                              _dtype_code(y), y.stride(0), ctypes.c_void_p(self.ptr), self.nbytes,
                                              _s()), "moe_experts_decode")
        return y


def ep_pack(x, ridx, dest, lidx, nrep, world, cap, discard, send_dtype=torch.bfloat16):
    """The expert-parallel send buffer (b200q_ep_pack): x [T][H], ridx [T][topk] int32, placement tables dest / lidx
    [E][max_rep] and nrep [E] (int32) -> send [world * cap][H + 16 bytes] of send_dtype, each row's local index as an
    int32 after its H values, and slot [T * topk] int32 (each pair's send row)."""
    _dev(x, "x")
    T, H = x.shape
    topk = ridx.shape[-1]
    pad = 16 // torch.empty(0, dtype=send_dtype).element_size()
    send = torch.empty(world * cap, H + pad, dtype=send_dtype, device=x.device)
    slot = torch.empty(T * topk, dtype=torch.int32, device=x.device)
    _check(lib().b200q_ep_pack(_p(x), _dtype_code(x), T, H, _p(_dev(ridx, "ridx")), topk, _p(_dev(dest, "dest")),
                               _p(_dev(lidx, "lidx")), _p(_dev(nrep, "nrep")), dest.shape[1], world, cap, int(discard),
                               _p(send), _dtype_code(send), send.stride(0), _p(slot), _s()), "ep_pack")
    return send, slot


def ep_index_view(buf, H):
    """the int32 local index b200q_ep_pack stores after the H values of each row of buf, as an [R] strided view"""
    return buf.view(torch.int32)[:, H * buf.element_size() // 4]


def ep_combine(back, slot, rw, topk, shared=None, out_dtype=torch.float32):
    """out[t] = sum_k rw[t][k] back[slot[t * topk + k]] (+ shared[t]) (b200q_ep_combine): the return buffer's rows
    weighted in combine_k's order"""
    _dev(back, "back", rows=True)
    T = rw.numel() // topk
    H = back.shape[1]
    out = torch.empty(T, H, dtype=out_dtype, device=back.device)
    rwc = rw.contiguous()
    _check(lib().b200q_ep_combine(_p(back), _dtype_code(back), back.stride(0), _p(slot), _p(rwc), _p(shared), T,
                                  topk, H, _p(out), _dtype_code(out), _s()), "ep_combine")
    return out


class PeerRegion:
    """One rank's region of the expert-parallel exchange over peer memory (b200q_ep_peer_decode): a zeroed device
    allocation of its own (not the caching allocator's: a CUDA IPC handle names a whole allocation), exported to the
    other ranks of the box, and the other ranks' regions mapped into this process.  unmap() then free(): the caller
    makes sure that no rank still uses a mapping when it is unmapped and that every rank has unmapped this region before
    it is freed (ep.PeerDecodeMoE.close puts barriers between the steps)."""

    def __init__(self, nbytes, device):
        p = ctypes.c_void_p()
        with torch.cuda.device(device):
            _check(lib().b200q_peer_alloc(nbytes, ctypes.byref(p)), "peer_alloc")
        self.ptr, self.nbytes, self.device = p.value, nbytes, device
        self.opened = []

    def handle(self):
        """the CUDA IPC handle of this region (bytes)"""
        buf = ctypes.create_string_buffer(lib().b200q_peer_handle_bytes())
        _check(lib().b200q_peer_export(self.ptr, buf), "peer_export")
        return buf.raw

    def open(self, handle):
        """map another rank's region (its handle()) into this process; -> its device address here"""
        p = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _check(lib().b200q_peer_open(handle, ctypes.byref(p)), "peer_open")
        self.opened.append(p.value)
        return p.value

    def unmap(self):
        """unmap the other ranks' regions"""
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for q in self.opened:
                lib().b200q_peer_close(q)
        self.opened = []

    def free(self):
        """free this rank's region (after every other rank has unmapped it)"""
        with torch.cuda.device(self.device):
            if self.ptr:
                lib().b200q_peer_free(self.ptr)
        self.ptr = None


def ep_peer_decode(x, logits, topk, dest, lidx, nrep, region, peers, world, rank, n_local, discard, up, down, state,
                   workspace, H, F, ret_dtype=torch.bfloat16, out=None, out_dtype=torch.float32,
                   route=ROUTE_SOFTMAX, bias=None, scale=1.0, ridx=None, rw=None, phases=7):
    """b200q_ep_peer_decode: one rank's expert-parallel decode step with the exchange over peer memory (token rows go
    out as int8 rows, outputs come back in ret_dtype).
    x [T][H], logits [T][E] (bf16 or fp32); dest / lidx [E][max_rep], nrep [E] int32; region: this rank's PeerRegion
    address; peers: int64 device tensor of every rank's region address in this process; up / down: the local slabs with
    the shared expert last; state: int32 device tensor (b200q_ep_peer_state_bytes, zeroed once); workspace: (address,
    bytes), 256-byte aligned.  -> out [T][H]"""
    _dev(x, "x")
    _dev(logits, "logits")
    T, E = logits.shape
    if out is None:
        out = torch.empty(T, H, dtype=out_dtype, device=x.device)
    _check(lib().b200q_ep_peer_decode(_p(x), _dtype_code(x), _p(logits), _dtype_code(logits), T, H, F, E, topk, route,
                                      _p(bias), float(scale), _p(dest), _p(lidx), _p(nrep), dest.shape[1], region,
                                      _p(peers), world, rank, n_local, discard, _p(up), _p(down),
                                      BF16 if ret_dtype == torch.bfloat16 else F32, _p(state), workspace[0],
                                      workspace[1], _p(out), _dtype_code(out), _p(ridx), _p(rw), phases, _s()),
           "ep_peer_decode")
    return out


def ep_peer_error(state, clear=True):
    """the error bits b200q_ep_peer_decode's bounded waits recorded in state (0: none); synchronous"""
    return lib().b200q_ep_peer_error(_p(state), 1 if clear else 0)


# -------------------------------------------------------------------------------------------------------------
# NVFP4 and Q8_0 (tile_nv4 / tile_q8 packing; mma_nv4 / mma_q8 at decode row counts)
# -------------------------------------------------------------------------------------------------------------
def tile_nv4(q, sc, n, k):
    """NVFP4 q [n][k/2] and e4m3 sc [n][k/16] (uint8 CUDA tensors) -> the t16 layout."""
    out = torch.empty(lib().b200q_nv4_bytes(n, k), dtype=torch.uint8, device=q.device)
    _check(lib().b200q_nv4_pack(_p(_dev(q, "q")), _p(_dev(sc, "sc")), _p(out), n, k, _s()), "tile_nv4")
    return out


def tile_q8(raw, n, k):
    """Q8_0 ggml blocks [n][k/32][34] (uint8 CUDA tensor) -> the t16 layout."""
    out = torch.empty(lib().b200q_q8_bytes(n, k), dtype=torch.uint8, device=raw.device)
    _check(lib().b200q_q8_pack(_p(_dev(raw, "raw")), _p(out), n, k, _s()), "tile_q8")
    return out


class _Workspace:
    def __init__(self):
        self.buf = None

    def get(self, nbytes, device):
        if nbytes == 0:
            return None, 0
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return ctypes.c_void_p(self.buf.data_ptr()), self.buf.numel()


_WS = _Workspace()


def mma_nv4(w, s2, n, k, x, y=None):
    """y [T][n] fp32 = s2 * W . x for T <= 16 rows of x (fp32 or bf16; rows at any pitch)."""
    _rows_any(x, "x")
    T = x.shape[0]
    y = torch.empty(T, n, dtype=torch.float32, device=x.device) if y is None else y
    ws, wb = _WS.get(lib().b200q_nv4_gemv_workspace_bytes(n, k, T), x.device)
    _check(lib().b200q_nv4_gemv(_p(w), float(s2), n, k, _p(x), _dtype_code(x), x.stride(0), T, _p(y), y.stride(0), ws, wb,
                                _s()), "mma_nv4")
    return y


def mma_q8(w, n, k, x, y=None):
    """y [T][n] fp32 = W . x for T <= 16 rows of x (fp32 or bf16; rows at any pitch)."""
    _rows_any(x, "x")
    T = x.shape[0]
    y = torch.empty(T, n, dtype=torch.float32, device=x.device) if y is None else y
    ws, wb = _WS.get(lib().b200q_q8_gemv_workspace_bytes(n, k, T), x.device)
    _check(lib().b200q_q8_gemv(_p(w), n, k, _p(x), _dtype_code(x), x.stride(0), T, _p(y), y.stride(0), ws, wb, _s()),
           "mma_q8")
    return y


# -------------------------------------------------------------------------------------------------------------
# prompt-length GEMMs (tcgen05)
# -------------------------------------------------------------------------------------------------------------
def device_error(clear=True):
    """Errors the kernels recorded on this device (0: none), see b200q_device_error."""
    return lib().b200q_device_error(1 if clear else 0)


def tile_q8_tc(raw, n, k):
    """Q8_0 ggml blocks [n][k/32][34] -> the prompt GEMM's q8 tc layout (units of 32 rows x 32 k)."""
    out = torch.empty(lib().b200q_q8_tc_bytes(n, k), dtype=torch.uint8, device=raw.device)
    _check(lib().b200q_q8_tc_pack(_p(_dev(raw, "raw")), _p(out), n, k, _s()), "tile_q8_tc")
    return out


def mma_q8_prompt(w_tc, n, k, x, y=None):
    """y [T][n] fp32 = fp16(q d) . fp16(x) for any T (the tcgen05 prompt GEMM; its rows image in a cached workspace)."""
    _dev(x, "x")
    T = x.shape[0]
    y = torch.empty(T, n, dtype=torch.float32, device=x.device) if y is None else y
    ws, wb = _WS.get(lib().b200q_q8_gemm_workspace_bytes(T, k), x.device)
    _check(lib().b200q_q8_gemm(_p(w_tc), n, k, _p(x), _dtype_code(x), x.stride(0), T, _p(y), y.stride(0), ws, wb,
                               _s()), "mma_q8_prompt")
    return y


def tile_nv4w(q, sc, n, k):
    """NVFP4 q [n][k/2] + sc [n][k/16] e4m3 -> the block-scaled fp4 prompt GEMM's tile image (tile_nv4w)."""
    out = torch.empty(lib().b200q_nv4_tc_bytes(n, k), dtype=torch.uint8, device=q.device)
    _check(lib().b200q_nv4_tc_pack(_p(_dev(q, "q")), _p(_dev(sc, "sc")), _p(out), n, k, _s()), "tile_nv4w")
    return out


def quant_nv4_rows(x, k=None, out=None):
    """Rows x [T][k] (fp32 or bf16) -> NVFP4 rows tile image (quant_nv4_rows: e4m3 scale amax/6 per 16, e2m1 values)."""
    _dev(x, "x")
    T, k = x.shape[0], x.shape[1] if k is None else k
    nb = lib().b200q_nv4_rows_bytes(T, k)
    out = torch.empty(nb, dtype=torch.uint8, device=x.device) if out is None else out
    _check(lib().b200q_quant_nv4_rows(_p(x), _dtype_code(x), x.stride(0), T, k, _p(out), _s()), "quant_nv4_rows")
    return out


def mma_nv4_fp4(w_tc, s2, n, k, rows, T, y=None):
    """y [T][n] fp32 = s2 * (NVFP4 rows) . (NVFP4 weights) on the block-scaled fp4 tensor cores (mma_nv4_fp4)."""
    y = torch.empty(T, n, dtype=torch.float32, device=rows.device) if y is None else y
    ws, wb = _WS.get(lib().b200q_nv4_gemm_workspace_bytes(n, k, T), rows.device)
    _check(lib().b200q_nv4_gemm(_p(w_tc), n, k, float(s2), _p(rows), T, _p(y), y.stride(0), ws, wb, _s()),
           "mma_nv4_fp4")
    return y


def k_moe_group_large(ridx, E):
    """Grouping for any number of pairs: counts [E], offsets [E+1], order [pairs]."""
    _dev(ridx, "ridx")
    pairs = ridx.numel()
    counts = torch.empty(E, dtype=torch.int32, device=ridx.device)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=ridx.device)
    order = torch.empty(max(pairs, 1), dtype=torch.int32, device=ridx.device)
    fill = torch.empty(E, dtype=torch.int32, device=ridx.device)
    _check(lib().b200q_moe_group_large(_p(ridx), pairs, E, _p(counts), _p(offsets), _p(order), _p(fill), _s()),
           "k_moe_group_large")
    return counts, offsets, order[:pairs]


def moe_prompt(up, down, E, H, F, counts, offsets, order, topk, x, mo=None, act=None, workspace=None,
               out_dtype=torch.float32):
    """Prompt path of the routed experts (moe_up_tile + moe_down_tile): mo [pairs][H] (fp32, or bf16 with out_dtype /
    a bf16 mo) = W_down[e] . act[p], act[p] = fp16(relu(W_up[e] . x[p / topk])^2); act (optional, [pairs][F] fp16)
    receives the intermediate."""
    _dev(x, "x")
    pairs = order.numel()
    mo = torch.empty(pairs, H, dtype=out_dtype, device=x.device) if mo is None else mo
    nb = lib().b200q_moe_prompt_workspace_bytes(pairs, E, H, F)
    if workspace is None:
        ws, wb = _WS.get(nb, x.device)
    else:
        ws, wb = _p(workspace), workspace.numel()
    _check(lib().b200q_moe_prompt(_p(up), _p(down), E, H, F, _p(counts), _p(offsets), _p(order), topk, pairs, _p(x),
                                  _dtype_code(x), _p(mo), _dtype_code(mo), _p(act) if act is not None else None, ws, wb,
                                  _s()), "moe_prompt")
    return mo


# -------------------------------------------------------------------------------------------------------------
# checkpoint ingestion (open_store / lookup / load_slab / load_nv4 / load_q8, bolt_host.cu:61-345)
# -------------------------------------------------------------------------------------------------------------
# The model's checkpoint layout (libbolt's loader, bolt_host.cu:126, 959-1011): tensors named under
# language_model.backbone.layers.<layer>, routed experts in the MoE latent space of 1024
MODEL_PREFIX = "language_model.backbone.layers"
MODEL_LATENT = 1024


def moe_layer_tensor_names(layer, experts, prefix=MODEL_PREFIX):
    """the tensor names libbolt's loader reads for MoE layer `layer` (bolt_host.cu:316, 994-995)"""
    p = f"{prefix}.{layer}.mixer"
    return {"up": [f"{p}.experts.{e}.up_proj.weight" for e in range(experts)],
            "down": [f"{p}.experts.{e}.down_proj.weight" for e in range(experts)],
            "shared_up": f"{p}.shared_experts.up_proj.weight",
            "shared_down": f"{p}.shared_experts.down_proj.weight"}


def read_moe_schedule(path):
    """The model's MoE schedule from its contract file (a JSON object with "moe_schedule": [{"layer", "experts",
    "width", "top_k"}...], "moe_latent_size", "shared_expert_width"): a list of (layer, experts, width, top_k) and a
    dict of the shared sizes.  Every entry is checked (positive sizes, widths a multiple of 256)."""
    with open(path) as f:
        c = json.load(f)
    sched = []
    for m in c["moe_schedule"]:
        L, e, w, k = int(m["layer"]), int(m["experts"]), int(m["width"]), int(m["top_k"])
        if L < 0 or e <= 0 or k <= 0 or k > e or w <= 0 or w % 256:
            raise B200QError(EINVAL, f"bad MoE schedule entry {m}")
        sched.append((L, e, w, k))
    info = {"latent": int(c.get("moe_latent_size", MODEL_LATENT)), "shared_width": int(c.get("shared_expert_width", 0)),
            "hidden": int(c.get("hidden", 4096))}
    return sched, info


class _Mapping:
    """The library's handle of an opened checkpoint.  The shards stay mapped while this object lives: the Checkpoint
    and every tensor view it handed out hold a reference, so a view never outlives the memory it reads."""

    def __init__(self, h):
        self.h = h

    def __del__(self):
        try:
            if self.h:
                lib().b200q_ckpt_close(self.h)
                self.h = None
        except Exception:
            pass


class Checkpoint:
    """A model directory of safetensors shards (model.safetensors.index.json, or one model.safetensors), mapped by the
    library; tensors are read in place and packed into this library's device layouts through a device staging
    buffer.

    The packs of one Checkpoint share one staging buffer; a pack on a different stream from the previous one first
    makes its stream wait for the previous stream's work, so the staging bytes are never overwritten while a pack
    kernel still reads them."""

    def __init__(self, path):
        h = lib().b200q_ckpt_open(os.fsencode(path))
        if not h:
            raise B200QError(EINVAL, f"no readable safetensors checkpoint at {path}")
        self._map = _Mapping(h)
        self._staging = None
        self._staging_stream = None

    @property
    def _h(self):
        if self._map is None:
            raise B200QError(EINVAL, "checkpoint is closed")
        return self._map.h

    def close(self):
        """Drop this object's hold on the mapping; views handed out by tensor() keep it mapped until they go."""
        self._map = None
        self._staging = None

    def __len__(self):
        return int(lib().b200q_ckpt_count(self._h))

    def tensor(self, name):
        """(a read-only uint8 numpy view of the tensor's bytes in the mapping, shape, safetensors dtype).  The view
        keeps the mapping alive: it stays valid after close() or after this Checkpoint is gone."""
        import numpy as np
        data, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        shape, ndim, dtype = (ctypes.c_int64 * 8)(), ctypes.c_int(), ctypes.create_string_buffer(16)
        _check(lib().b200q_ckpt_tensor(self._h, name.encode(), ctypes.byref(data), ctypes.byref(nbytes), shape,
                                       ctypes.byref(ndim), dtype), f"tensor {name}")
        if nbytes.value:
            buf = (ctypes.c_uint8 * nbytes.value).from_address(data.value)
            buf._mapping = self._map   # the numpy array below holds buf, buf holds the mapping
            view = np.frombuffer(buf, dtype=np.uint8)
        else:
            view = np.zeros(0, np.uint8)
        view.flags.writeable = False
        return view, tuple(shape[i] for i in range(ndim.value)), dtype.value.decode()

    def _stage(self, fmt, n, k, device):
        need = lib().b200q_ckpt_staging_bytes(fmt, n, k)
        cur = torch.cuda.current_stream(torch.device(device))
        if self._staging is None or self._staging.numel() < need or self._staging.device != torch.device(device):
            if self._staging is not None and self._staging_stream is not None:
                # the old buffer's memory is reused only after the work its last pack enqueued
                self._staging.record_stream(self._staging_stream)
            self._staging = torch.empty(need, dtype=torch.uint8, device=device)
        elif self._staging_stream is not None and self._staging_stream != cur:
            cur.wait_stream(self._staging_stream)   # the previous pack's kernel has read the staging bytes
        self._staging_stream = cur
        return self._staging

    def pack_iq2_slab(self, names, rows, k, device="cuda"):
        """the experts' IQ2_XXS tensors (names[e]: [rows][k/256][66] blocks) -> one packed slab (load_slab)"""
        st = self._stage(0, rows, k, device)
        out = torch.empty(len(names) * iq2_bytes(rows, k), dtype=torch.uint8, device=device)
        arr = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        _check(lib().b200q_ckpt_pack_iq2_slab(self._h, arr, len(names), rows, k, _p(out), _p(st), st.numel(), _s()),
               "pack_iq2_slab")
        return out

    def tensor_shape(self, name):
        """a tensor's shape (the safetensors header's), without reading its bytes"""
        return self.tensor(name)[1]

    def pack_moe_layer(self, layer, experts, width, latent=MODEL_LATENT, prefix=MODEL_PREFIX, device="cuda"):
        """One MoE layer of the model's checkpoint, as libbolt's loader takes it (bolt_host.cu:994-1003, load_slab
        :306-328): the routed experts' up projections (prefix.<layer>.mixer.experts.<e>.up_proj.weight, [width][latent]
        each) and down projections ([latent][width]) into one slab each, and the shared expert's up and down
        (prefix.<layer>.mixer.shared_experts.{up,down}_proj.weight, their shapes read from the checkpoint).  Returns
        {"up", "down", "shared_up", "shared_down": packed rt32 tensors, "shared_width", "hidden"}."""
        names = moe_layer_tensor_names(layer, experts, prefix)
        up = self.pack_iq2_slab(names["up"], width, latent, device)
        down = self.pack_iq2_slab(names["down"], latent, width, device)
        out = {"up": up, "down": down}
        su, sd = self.tensor_shape(names["shared_up"]), self.tensor_shape(names["shared_down"])
        if len(su) != 3 or len(sd) != 3 or su[2] != 66 or sd[2] != 66:
            raise B200QError(EINVAL, f"layer {layer}: the shared expert is not IQ2_XXS ([rows][k/256][66])")
        sw, hidden = int(su[0]), int(su[1]) * 256
        if int(sd[0]) != hidden or int(sd[1]) * 256 != sw:
            raise B200QError(EINVAL, f"layer {layer}: shared expert shapes {su} / {sd} do not chain")
        out["shared_up"] = self.pack_iq2_slab([names["shared_up"]], sw, hidden, device)
        out["shared_down"] = self.pack_iq2_slab([names["shared_down"]], hidden, sw, device)
        out["shared_width"], out["hidden"] = sw, hidden
        return out

    def pack_nv4(self, prefix, n, k, device="cuda"):
        """prefix.weight / .weight_scale / .weight_scale_2 -> (the t16 layout, the tensor scale s2) (load_nv4)"""
        st = self._stage(1, n, k, device)
        out = torch.empty(lib().b200q_nv4_bytes(n, k), dtype=torch.uint8, device=device)
        s2 = ctypes.c_float()
        _check(lib().b200q_ckpt_pack_nv4(self._h, prefix.encode(), n, k, _p(out), ctypes.byref(s2), _p(st), st.numel(),
                                         _s()), "pack_nv4")
        return out, s2.value

    def pack_q8(self, name, n, k, device="cuda"):
        """a Q8_0 tensor ([n][k/32][34] blocks) -> the t16 layout (load_q8)"""
        st = self._stage(2, n, k, device)
        out = torch.empty(lib().b200q_q8_bytes(n, k), dtype=torch.uint8, device=device)
        _check(lib().b200q_ckpt_pack_q8(self._h, name.encode(), n, k, _p(out), _p(st), st.numel(), _s()), "pack_q8")
        return out


# -------------------------------------------------------------------------------------------------------------
# the decode MoE layer
# -------------------------------------------------------------------------------------------------------------
class MoeDecodeLayer:
    """One decode MoE layer (router, up with relu^2, down, combine, shared expert) over packed IQ2_XXS slabs.

    up: packed [E] x [F][H], down: packed [E] x [H][F] (CUDA uint8 tensors in the rt32 layout); shared_up/down
    optional.  The workspace is allocated once here, for up to max_tokens tokens; __call__ only launches kernels.
    """

    def __init__(self, up, down, shared_up, shared_down, H, F, E, topk, route=ROUTE_SOFTMAX, bias=None, scale=1.0,
                 max_tokens=16):
        self.up, self.down, self.shared_up, self.shared_down = up, down, shared_up, shared_down
        self.H, self.F, self.E, self.topk, self.route, self.bias, self.scale = H, F, E, topk, route, bias, scale
        self.max_tokens = max_tokens
        nbytes = lib().b200q_moe_decode_workspace_bytes(max_tokens, H, F, E, topk)
        self.workspace = torch.empty(nbytes + 256, dtype=torch.uint8, device=up.device)
        off = (-self.workspace.data_ptr()) % 256
        self._ws_ptr = self.workspace.data_ptr() + off
        self._ws_bytes = nbytes

    def __call__(self, x, logits, out=None, ridx=None, rw=None, stream=None, stage_events=None):
        """x [T][H] bf16, logits [T][E] bf16 (CUDA) -> out [T][H]; stage_events: 5 torch.cuda.Event for profiling."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise B200QError(EINVAL, f"{T} tokens > max_tokens {self.max_tokens}")
        out = torch.empty(T, self.H, dtype=torch.float32, device=x.device) if out is None else out
        need = lib().b200q_moe_decode_workspace_bytes(T, self.H, self.F, self.E, self.topk)
        ev = None
        if stage_events is not None:
            ev = (ctypes.c_void_p * 5)(*[e.cuda_event for e in stage_events])
        _check(lib().b200q_moe_decode(_p(x), _p(logits), _p(self.up), _p(self.down), _p(self.shared_up),
                                      _p(self.shared_down), T, self.H, self.F, self.E, self.topk, self.route, _p(self.bias),
                                      float(self.scale), _p(out), _dtype_code(out), ctypes.c_void_p(self._ws_ptr), need,
                                      _p(ridx), _p(rw), ev, _s(stream)), "moe_decode")
        return out
