"""libbolt's operator launchers (include/b200q_bolt.h: libbolt's own names, signatures and view structs, backed by
libb200q) fed the inputs of the golden fixtures, which hold the outputs of libbolt's own kernels run on a B200: the
shims, called the way libbolt's host code calls its launchers, give libbolt's outputs (bit for bit where the kernel
keeps libbolt's chunk order; the router's weights within 2e-6, its picks exact)."""
import ctypes
import os

import numpy as np
import pytest
import torch

import b200q
from helpers import iq2_blocks

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
DEV = "cuda"
_KEEP = []


def _harness():
    import build_harness
    L = ctypes.CDLL(build_harness.build())
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    sig = {
        "hs_repack_iq2": [vp, vp, vp, vp, sz, i32],
        "hs_k_route": [vp, vp, i32, vp, vp, vp, i32, f32, i32],
        "hs_k_moe_group": [vp, vp, i32, vp, vp, vp, vp, vp],
        "hs_k_quant_rows": [vp, vp, i32, vp, i32, vp, i32, i32, i32],
        "hs_moe_up": [vp, vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32],
        "hs_moe_down": [vp, vp, vp, sz, sz, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32],
        "hs_moe_coop_dense": [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32],
        "hs_k_combine": [vp, vp, vp, vp, i32],
        "hs_moe_tile_dense": [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32],
        "hs_tile_nv4": [vp, vp, vp, vp, vp, i32, i32],
        "hs_tile_q8": [vp, vp, vp, vp, i32, i32],
        "hs_mma_nv4": [vp, vp, vp, f32, i32, i32, vp, i32, vp, i32, i32],
        "hs_mma_q8": [vp, vp, vp, i32, i32, vp, i32, vp, i32, i32],
        "hs_mma_q8_multi": [vp, vp, vp, vp, i32, vp, i32, vp, vp, i32],
        "hs_tile_iq2": [vp, vp, vp, vp, i32, i32],
        "hs_mma_iq2": [vp, vp, vp, i32, i32, vp, i32, vp, i32, i32, i32],
        "hs_tile_nv4w": [vp, vp, vp, vp, vp, i32, i32],
        "hs_quant_nv4_rows": [vp, vp, i32, vp, vp, i32, i32],
        "hs_mma_nv4_fp4": [vp, vp, vp, f32, i32, i32, vp, vp, vp, i32, i32],
    }
    for n, a in sig.items():
        getattr(L, n).restype, getattr(L, n).argtypes = None, a
    L.hs_tile_bytes.restype, L.hs_tile_bytes.argtypes = sz, [i32, i32, i32, i32]
    return L


def golden(name):
    z = np.load(os.path.join(HERE, "golden", f"ref_{name}.npz"))
    return ({k[3:]: z[k] for k in z.files if k.startswith("in_")}, {k[4:]: z[k] for k in z.files if k.startswith("out_")})


def d(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    _KEEP.append(t)
    return t


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def slab(L, blocks, rows, k):
    """the qs / d buffers libbolt's load_slab allocates (rows * k/256 * 64 and * 2 bytes), packed by the shim"""
    qs = torch.empty(rows * (k // 256) * 64, dtype=torch.uint8, device=DEV)
    dd = torch.empty(rows * (k // 256), dtype=torch.float16, device=DEV)
    L.hs_repack_iq2(s(), p(d(blocks.reshape(-1))), p(qs), p(dd), rows, k)
    _KEEP.extend([qs, dd])
    return qs, dd


def test_shim_exports_libbolt_signatures():
    L = _harness()
    assert L.hs_moe_up is not None


def test_shim_router_and_quant_rows_match_libbolt():
    L = _harness()
    i, o = golden("route")
    T, E = i["logits"].shape
    ridx = torch.empty(T * 9, dtype=torch.int32, device=DEV)
    rw = torch.empty(T * 9, dtype=torch.float32, device=DEV)
    L.hs_k_route(s(), p(d(i["logits"])), E, p(d(i["bias"])), p(ridx), p(rw), E, float(i["scale"]), T)
    assert np.array_equal(ridx.cpu().numpy().reshape(T, 9), o["ridx"])
    assert np.allclose(rw.cpu().numpy().reshape(T, 9), o["rw"], rtol=2e-6)
    i, o = golden("quant_rows")
    q = torch.empty(8, 256, dtype=torch.int8, device=DEV)
    sc = torch.empty(8, 8, dtype=torch.float32, device=DEV)
    L.hs_k_quant_rows(s(), p(d(i["x"])), 256, p(q), 256, p(sc), 8, 8, 256)
    assert np.array_equal(q.cpu().numpy(), o["q"]) and np.array_equal(sc.cpu().numpy(), o["s"])


def test_shim_moe_block_matches_libbolt():
    """repack_iq2 into libbolt's buffers, k_moe_group, moe_up, moe_down at libbolt's routed shapes (k 1024 up,
    n 1024 down, 9 experts a token), against libbolt's own act and mo"""
    L = _harness()
    i, o = golden("moe_up_down")
    E, W, H = int(i["E"]), int(i["W"]), int(i["H"])
    pairs = len(i["ridx"])
    uqs, ud = slab(L, iq2_blocks(int(i["up_seed"]), E * W, H), E * W, H)
    dqs, dd = slab(L, iq2_blocks(int(i["down_seed"]), E * H, W), E * H, W)
    cap = 2048 * 9   # libbolt's work arrays: TMAX * TOPN entries
    order, first, count, exp = (torch.zeros(cap, dtype=torch.int32, device=DEV) for _ in range(4))
    nwork = torch.zeros(1, dtype=torch.int32, device=DEV)
    ridx = d(i["ridx"].astype(np.int32))
    L.hs_k_moe_group(s(), p(ridx), pairs, p(order), p(first), p(count), p(exp), p(nwork))
    act = torch.full((pairs, W), -1.0, device=DEV)
    L.hs_moe_up(s(), p(uqs), p(ud), W * (H // 256) * 64, W * (H // 256), p(order), p(first), p(count), p(exp), p(nwork),
                p(d(i["xq"])), p(d(i["xs"])), p(act), W, pairs)
    assert np.array_equal(act.cpu().numpy(), o["act"])
    mo = torch.full((pairs, H), -1.0, device=DEV)
    L.hs_moe_down(s(), p(dqs), p(dd), H * (W // 256) * 64, H * (W // 256), p(order), p(first), p(count), p(exp),
                  p(nwork), p(d(i["aq"])), p(d(i["as"])), p(mo), W, pairs)
    assert np.array_equal(mo.cpu().numpy(), o["mo"])
    assert b200q.device_error() == 0


def test_shim_coop_dense_and_combine_match_libbolt():
    L = _harness()
    i, o = golden("coop_dense")
    n, k = int(i["n"]), int(i["k"])
    qs, dd = slab(L, iq2_blocks(int(i["seed"]), n, k), n, k)
    T = i["xq"].shape[0]
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_moe_coop_dense(s(), p(qs), p(dd), T, p(d(i["xq"])), p(d(i["xs"])), p(y), n, n, k, 1)
    assert np.array_equal(y.cpu().numpy(), o["y"])
    y2 = torch.full((T, n), -1.0, device=DEV)   # moe_tile_dense, enqueue_block's choice at prompt row counts
    L.hs_moe_tile_dense(s(), p(qs), p(dd), T, p(d(i["xq"])), p(d(i["xs"])), p(y2), n, n, k, 1)
    assert np.array_equal(y2.cpu().numpy(), o["y"])
    i, o = golden("combine")
    T = o["out"].shape[0]
    out = torch.empty(T, 1024, device=DEV)
    L.hs_k_combine(s(), p(d(i["o"])), p(d(i["rw"])), p(out), T)
    assert np.array_equal(out.cpu().numpy(), o["out"])


def nv4_tiles(L, q, sc, n, k):
    """the qt / sct buffers load_nv4 allocates (tile_bytes_nv4, tile_scale_bytes_nv4), filled by tile_nv4"""
    qt = torch.empty(L.hs_tile_bytes(0, 0, n, k), dtype=torch.uint8, device=DEV)
    sct = torch.empty(L.hs_tile_bytes(0, 1, n, k), dtype=torch.uint8, device=DEV)
    L.hs_tile_nv4(s(), p(d(q)), p(d(sc)), p(qt), p(sct), n, k)
    _KEEP.extend([qt, sct])
    return qt, sct


def q8_tiles(L, blocks, n, k):
    qt = torch.empty(L.hs_tile_bytes(1, 0, n, k), dtype=torch.uint8, device=DEV)
    dt = torch.empty(L.hs_tile_bytes(1, 1, n, k), dtype=torch.uint8, device=DEV)
    L.hs_tile_q8(s(), p(d(blocks)), p(qt), p(dt), n, k)
    _KEEP.extend([qt, dt])
    return qt, dt


def golden_q8_blocks(i):
    n, k = i["q"].shape
    blocks = np.concatenate([i["d"].view(np.uint8).reshape(n, k // 32, 2), i["q"].view(np.uint8).reshape(n, k // 32, 32)],
                            -1)
    return blocks.reshape(n, -1)


def test_shim_nv4_q8_decode_match_libbolt():
    """tile_nv4 + mma_nv4 and tile_q8 + mma_q8 on the golden cases' inputs.  libbolt's mma_nv4 / mma_q8 round the fp32
    rows to fp16 before the tensor cores (PNV4 / PQ8 kBF = false, bolt_mma.cu:103, 182), as the shims do: against
    the oracle on those rounded rows 1e-5 (fp32 sums in another order); against the fixtures, which hold libbolt's
    fp32-row gemv_nv4 / gemv_q8, within the rows' fp16 rounding (relative L2 1e-3)."""
    import oracle as O
    from helpers import rel_l2
    L = _harness()
    i, o = golden("gemv_nv4")
    n, k = i["q"].shape[0], i["q"].shape[1] * 2
    T = i["x"].shape[0]
    x16 = i["x"].astype(np.float16).astype(np.float32)
    qt, sct = nv4_tiles(L, i["q"], i["sc"], n, k)
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_mma_nv4(s(), p(qt), p(sct), float(i["s2"]), n, k, p(d(i["x"])), k, p(y), n, T)
    y = y.cpu().numpy()
    ref = O.nv4_gemm_exact(i["q"], i["sc"], float(i["s2"]), n, k, x16)
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    assert rel_l2(y, o["y"]) < 1e-3
    i, o = golden("gemv_q8")
    n, k = i["q"].shape
    x16 = i["x"].astype(np.float16).astype(np.float32)
    blocks = golden_q8_blocks(i)
    qt, dt = q8_tiles(L, blocks, n, k)
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_mma_q8(s(), p(qt), p(dt), n, k, p(d(i["x"])), k, p(y), n, T)
    y = y.cpu().numpy()
    ref = O.q8_gemm_exact(blocks, n, k, x16)
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    assert rel_l2(y, o["y"]) < 1e-3
    assert b200q.device_error() == 0


@pytest.mark.parametrize("n,k", [(64, 256), (4096, 2048)])
def test_shim_tiles_are_the_split_t16_units(n, k):
    """libbolt's two tile buffers hold this engine's t16 units split in two: the 512 code bytes of each unit in qt,
    its 64 (NVFP4) or 32 (Q8_0) scale bytes in sct / dt, in unit order"""
    from test_gpu_nv4_q8 import nv4_weights, q8_blocks
    L = _harness()
    q, sc = nv4_weights(n + 1, n, k)
    qt, sct = nv4_tiles(L, q, sc, n, k)
    units = b200q.tile_nv4(d(q), d(sc), n, k).view(-1, 576)
    assert torch.equal(qt.view(-1, 512), units[:, :512]) and torch.equal(sct.view(-1, 64), units[:, 512:])
    blocks = q8_blocks(n + 2, n, k)
    qt, dt = q8_tiles(L, blocks, n, k)
    units = b200q.tile_q8(d(blocks), n, k).view(-1, 544)
    assert torch.equal(qt.view(-1, 512), units[:, :512]) and torch.equal(dt.view(-1, 32), units[:, 512:])


def test_shim_mma_rows_and_multi_match_engine_gemv():
    """mma_nv4 / mma_q8 over T = 37 fp32 rows run 16-row decode GEMVs on the split planes: bit for bit the engine's
    GEMV on the joined units, piece by piece; mma_q8_multi (q, k, v and a zeroed slot) is each mma_q8 alone"""
    from test_gpu_nv4_q8 import nv4_weights, q8_blocks
    L = _harness()
    n, k, T = 4096, 4096, 37
    x = torch.randn(T, k, device=DEV)
    q, sc = nv4_weights(5, n, k)
    qt, sct = nv4_tiles(L, q, sc, n, k)
    w = b200q.tile_nv4(d(q), d(sc), n, k)
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_mma_nv4(s(), p(qt), p(sct), 0.37, n, k, p(x), k, p(y), n, T)
    ref = torch.cat([b200q.mma_nv4(w, 0.37, n, k, x[t0:t0 + 16]) for t0 in range(0, T, 16)])
    assert torch.equal(y, ref)
    ns = [4096, 1024, 1024]
    tiles = [q8_tiles(L, q8_blocks(20 + j, nj, k), nj, k) for j, nj in enumerate(ns)]
    refs = []
    for j, nj in enumerate(ns):
        yj = torch.full((T, nj), -1.0, device=DEV)
        L.hs_mma_q8(s(), p(tiles[j][0]), p(tiles[j][1]), nj, k, p(x), k, p(yj), nj, T)
        wj = b200q.tile_q8(d(q8_blocks(20 + j, nj, k)), nj, k)
        assert torch.equal(yj, torch.cat([b200q.mma_q8(wj, nj, k, x[t0:t0 + 16]) for t0 in range(0, T, 16)]))
        refs.append(yj)
    for used in ([0, 1, 2], [0, 2]):
        ys = [torch.full((T, nj), -1.0, device=DEV) for nj in ns]
        arr = lambda vals, ty: (ty * 3)(*vals)
        qv = arr([tiles[j][0].data_ptr() if j in used else 0 for j in range(3)], ctypes.c_void_p)
        dv = arr([tiles[j][1].data_ptr() if j in used else 0 for j in range(3)], ctypes.c_void_p)
        nv = arr([ns[j] if j in used else 0 for j in range(3)], ctypes.c_int)
        yv = arr([ys[j].data_ptr() for j in range(3)], ctypes.c_void_p)
        lv = arr(ns, ctypes.c_int)
        L.hs_mma_q8_multi(s(), qv, dv, nv, k, p(x), k, yv, lv, T)
        for j in range(3):
            if j in used:
                assert torch.equal(ys[j], refs[j])
            else:
                assert bool((ys[j] == -1.0).all())
    assert b200q.device_error() == 0


def iq2_tiles(L, blocks, n, k):
    """the qt / dt buffers load_iq2 allocates (tile_bytes_iq2, tile_scale_bytes_iq2), filled by tile_iq2"""
    qt = torch.empty(L.hs_tile_bytes(2, 0, n, k), dtype=torch.uint8, device=DEV)
    dt = torch.empty(L.hs_tile_bytes(2, 1, n, k), dtype=torch.uint8, device=DEV)
    L.hs_tile_iq2(s(), p(d(blocks.reshape(-1))), p(qt), p(dt), n, k)
    _KEEP.extend([qt, dt])
    return qt, dt


def test_shim_iq2_tiles_are_repack_iq2_planes():
    """tile_iq2 fills libbolt's tile buffers (the same byte counts as load_slab's qs / d) exactly as repack_iq2"""
    L = _harness()
    n, k = 256, 1024
    blocks = iq2_blocks(41, n, k)
    assert L.hs_tile_bytes(2, 0, n, k) == n * (k // 256) * 64 and L.hs_tile_bytes(2, 1, n, k) == n * (k // 256) * 2
    qt, dt = iq2_tiles(L, blocks, n, k)
    qs, dd = slab(L, blocks, n, k)
    assert torch.equal(qt, qs) and torch.equal(dt, dd.view(torch.uint8))


def test_shim_mma_iq2_shared_expert():
    """mma_iq2 (the shared expert's up with relu^2, then down): bit for bit the oracle's int8-row arithmetic
    (quant_rows_k, int32 chunk dots, fp32 chunk-order sums); against libbolt's fp32-row gemv_iq2 fixture and the
    exact dequantised product within the tolerance BASELINE states for fp32 outputs (relative L2 1e-2)"""
    import oracle as O
    from helpers import rel_l2
    L = _harness()
    i, o = golden("gemv_iq2")
    n, k = int(i["n"]), int(i["k"])
    T = i["x"].shape[0]
    blocks = iq2_blocks(int(i["seed"]), n, k)
    qt, dt = iq2_tiles(L, blocks, n, k)
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_mma_iq2(s(), p(qt), p(dt), n, k, p(d(i["x"])), k, p(y), n, T, 0)
    y = y.cpu().numpy()
    xq, xs = O.quant_rows(i["x"], k)
    assert np.array_equal(y, O.iq2_gemm_i8(blocks, n, k, xq, xs, 0))
    assert rel_l2(y, o["y"]) < 1e-2
    # the model's shared expert shapes: latent 1024 -> 5376 (relu^2) -> 1024, T = 21 rows
    H, F, T = 1024, 5376, 21
    up, down = iq2_blocks(42, F, H), iq2_blocks(43, H, F)
    uqt, udt = iq2_tiles(L, up, F, H)
    dqt, ddt = iq2_tiles(L, down, H, F)
    x = np.random.default_rng(44).standard_normal((T, H)).astype(np.float32)
    act = torch.full((T, F), -1.0, device=DEV)
    L.hs_mma_iq2(s(), p(uqt), p(udt), F, H, p(d(x)), H, p(act), F, T, 1)
    out = torch.full((T, H), -1.0, device=DEV)
    L.hs_mma_iq2(s(), p(dqt), p(ddt), H, F, p(act), F, p(out), H, T, 0)
    act_ref = O.iq2_gemm_i8(up, F, H, *O.quant_rows(x, H), 1)
    assert np.array_equal(act.cpu().numpy(), act_ref)
    out_ref = O.iq2_gemm_i8(down, H, F, *O.quant_rows(act_ref, F), 0)
    assert np.array_equal(out.cpu().numpy(), out_ref)
    # each projection against the exact product of its own input rows
    assert rel_l2(act_ref, O.iq2_gemm_exact(up, F, H, x, 1)) < 1e-2
    assert rel_l2(out_ref, O.iq2_gemm_exact(down, H, F, act_ref, 0)) < 1e-2
    assert b200q.device_error() == 0


def _guarded(nbytes, fill=0xA5, guard=4096):
    """a device buffer of exactly nbytes followed by a guard of a known byte (to catch writes past libbolt's sizes)"""
    t = torch.full((nbytes + guard,), fill, dtype=torch.uint8, device=DEV)
    _KEEP.append(t)
    return t


def test_shim_quant_nv4_rows_matches_libbolt():
    """quant_nv4_rows writes libbolt's plain rows (q4 [T][k/2], sf [T][k/16]): libbolt's own B200 output, byte for byte,
    and nothing past T rows"""
    L = _harness()
    i, o = golden("quant_nv4_rows")
    T, k = i["x"].shape
    q4, sf = _guarded(T * k // 2), _guarded(T * k // 16)
    L.hs_quant_nv4_rows(s(), p(d(i["x"])), k, p(q4), p(sf), T, k)
    q4, sf = q4.cpu().numpy(), sf.cpu().numpy()
    assert np.array_equal(q4[:T * k // 2].reshape(T, k // 2), o["q4"])
    assert np.array_equal(sf[:T * k // 16].reshape(T, k // 16), o["sf"])
    assert (q4[T * k // 2:] == 0xA5).all() and (sf[T * k // 16:] == 0xA5).all()
    assert b200q.device_error() == 0


@pytest.mark.parametrize("n,k,T", [(18560, 4096, 300), (4096, 8192, 256), (640, 512, 37)])
def test_shim_nv4_fp4_prompt_path(n, k, T):
    """libbolt's BOLT_NV4_FP4 sequence (load_nv4w's tile_nv4w into buffers of libbolt's tile_bytes_nv4 /
    tile_scale_bytes_nv4 sizes, then quant_nv4_rows + mma_nv4_fp4 per chunk) at config 3's in_proj (18560 rows: the
    weight planes end in a 128-row tile) and out_proj, and a small ragged case: nothing written past libbolt's buffer
    sizes; the result is this engine's own NVFP4 prompt GEMM's (b200q_quant_nv4_rows + b200q_nv4_gemm: the same
    products and fp32 sums, relative L2 1e-6) and the oracle's NVFP4 x NVFP4 sum on sampled rows (1e-5)."""
    import oracle as O
    from helpers import rel_l2
    from test_gpu_nv4_prompt import nv4_weights
    L = _harness()
    q, sc = nv4_weights(n + k, n, k)
    s2 = 0.75
    x = np.random.default_rng(T).standard_normal((T, k)).astype(np.float32)
    qb, sb = L.hs_tile_bytes(0, 0, n, k), L.hs_tile_bytes(0, 1, n, k)
    assert (qb, sb) == (n * k // 2, n * k // 16)
    qw, sfw = _guarded(qb), _guarded(sb)
    L.hs_tile_nv4w(s(), p(d(q)), p(d(sc)), p(qw), p(sfw), n, k)
    q4, sf = _guarded(T * k // 2), _guarded(T * k // 16)
    xt = d(x)
    L.hs_quant_nv4_rows(s(), p(xt), k, p(q4), p(sf), T, k)
    y = torch.full((T, n), -1.0, device=DEV)
    L.hs_mma_nv4_fp4(s(), p(qw), p(sfw), s2, n, k, p(q4), p(sf), p(y), n, T)
    torch.cuda.synchronize()
    for buf, nb in ((qw, qb), (sfw, sb), (q4, T * k // 2), (sf, T * k // 16)):
        assert (buf[nb:] == 0xA5).all()
    assert b200q.device_error() == 0
    got = y.cpu().numpy()
    w = b200q.tile_nv4w(d(q), d(sc), n, k)
    want = b200q.mma_nv4_fp4(w, s2, n, k, b200q.quant_nv4_rows(xt), T).cpu().numpy()
    assert rel_l2(got, want) < 1e-6
    rows = np.unique(np.r_[0, T - 1, np.random.default_rng(1).integers(0, T, 4)])
    q4h, sfh = q4[:T * k // 2].cpu().numpy().reshape(T, k // 2), sf[:T * k // 16].cpu().numpy().reshape(T, k // 16)
    ref = O.nv4_gemm_q4(q, sc, s2, n, k, q4h[rows], sfh[rows])
    assert rel_l2(got[rows], ref) < 1e-5
