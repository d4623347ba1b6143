"""Golden fixtures from libbolt's own kernels run on a B200 -- TEST INFRASTRUCTURE.

The reference ships no golden vectors for its quantized GEMMs.  This script runs the reference's kernels
(engine/bolt_kernels.cu and engine/bolt_mma.cu compiled for sm_100a, oracle/_ref/libbolt_ref.so) on seeded inputs and
writes their outputs to tests/golden/ref_<case>.npz; tests/test_golden.py then checks the CPU oracle against them on
any machine.  Large weights are not stored: they are regenerated from their seed by the library's host generator
(b200q.synth_iq2_host, deterministic per seed).

Run on a GPU box:  python tests/golden/make_golden.py [out_dir]   (default: tests/golden)
Each case function returns (inputs, outputs) as dicts of numpy arrays; tests/test_gpu_ref.py calls the same functions.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "nemotron-3.5-bolt-tensorfold-dgx-spark_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import refbind as R  # noqa: E402
from helpers import iq2_blocks, normal_bf16  # noqa: E402

DEV = "cuda"
_KEEP = []   # device copies stay alive until the next case: a pointer taken from a temporary would be recycled


def _d(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    _KEEP.append(t)
    return t


def _p(t):
    return t.data_ptr()


def planar_iq2(blocks, rows, k):
    """libbolt's planar IQ2W layout via its own repack_iq2: qs [rows][k/256][64], d [rows][k/256] fp16."""
    raw = _d(blocks.reshape(-1))
    qs = torch.empty(rows * (k // 256) * 64, dtype=torch.uint8, device=DEV)
    d = torch.empty(rows * (k // 256), dtype=torch.float16, device=DEV)
    R.call("ref_repack_iq2", _p(raw), _p(qs), _p(d), rows, k)
    return qs, d


def case_quant_rows():
    x = np.random.default_rng(1).standard_normal((8, 256)).astype(np.float32)
    x[2, :32] = 0.0
    xd = _d(x)
    q = torch.empty(8, 256, dtype=torch.int8, device=DEV)
    s = torch.empty(8, 8, dtype=torch.float32, device=DEV)
    R.call("ref_quant_rows", _p(xd), 256, _p(q), 256, _p(s), 8, 8, 256)
    return {"x": x}, {"q": q.cpu().numpy(), "s": s.cpu().numpy()}


def case_route():
    T, E = 6, 128
    topn = R.lib().ref_topn()
    lg = np.random.default_rng(2).standard_normal((T, E)).astype(np.float32)
    bias = (np.random.default_rng(3).standard_normal(E) * 0.05).astype(np.float32)
    ridx = torch.empty(T * topn, dtype=torch.int32, device=DEV)
    rw = torch.empty(T * topn, dtype=torch.float32, device=DEV)
    R.call("ref_route", _p(_d(lg)), E, _p(_d(bias)), _p(ridx), _p(rw), E, 2.5, T)
    return {"logits": lg, "bias": bias, "scale": np.float32(2.5), "topn": np.int32(topn)}, \
        {"ridx": ridx.cpu().numpy().reshape(T, topn), "rw": rw.cpu().numpy().reshape(T, topn)}


def _work(pairs):
    return [torch.zeros(max(pairs, 1), dtype=torch.int32, device=DEV) for _ in range(4)] + \
        [torch.zeros(1, dtype=torch.int32, device=DEV)]


def case_coop_dense():
    """moe_coop_dense: one IQ2 matrix (n 64, k 512) over 5 int8 rows, relu^2, the int8-per-32 arithmetic."""
    n, k, T, seed = 64, 512, 5, 71
    blocks = iq2_blocks(seed, n, k)
    x = np.random.default_rng(4).standard_normal((T, k)).astype(np.float32)
    import oracle as O
    xq, xs = O.quant_rows(x, k)
    qs, d = planar_iq2(blocks, n, k)
    order, first, count, exp, nwork = _work(T)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    R.call("ref_moe_coop_dense", _p(qs), _p(d), _p(order), _p(first), _p(count), _p(exp), _p(nwork), T, _p(_d(xq)),
           _p(_d(xs)), _p(y), n, n, k, 1)
    return {"seed": np.int64(seed), "n": np.int32(n), "k": np.int32(k), "xq": xq, "xs": xs}, {"y": y.cpu().numpy()}


def case_moe_up_down():
    """moe_up / moe_down at libbolt's own routed shapes (k 1024 up, n 1024 down, TOPN pairs a token)."""
    import oracle as O
    topn = R.lib().ref_topn()
    T, E, W, H = 3, 16, 256, 1024
    pairs = T * topn
    up = iq2_blocks(81, E * W, H)
    down = iq2_blocks(82, E * H, W)
    lg = np.random.default_rng(5).standard_normal((T, E)).astype(np.float32)
    x = np.random.default_rng(6).standard_normal((T, H)).astype(np.float32)
    ridx = torch.empty(pairs, dtype=torch.int32, device=DEV)
    rw = torch.empty(pairs, dtype=torch.float32, device=DEV)
    zero_bias = torch.zeros(E, dtype=torch.float32, device=DEV)   # route_k reads bias[i] unconditionally
    R.call("ref_route", _p(_d(lg)), E, _p(zero_bias), _p(ridx), _p(rw), E, 1.0, T)
    order, first, count, exp, nwork = _work(pairs)
    R.call("ref_moe_group", _p(ridx), pairs, _p(order), _p(first), _p(count), _p(exp), _p(nwork))
    xq, xs = O.quant_rows(x, H)
    uqs, ud = planar_iq2(up, E * W, H)
    dqs, dd = planar_iq2(down, E * H, W)
    act = torch.zeros(pairs, W, dtype=torch.float32, device=DEV)
    R.call("ref_moe_up", _p(uqs), _p(ud), W * (H // 256) * 64, W * (H // 256), _p(order), _p(first), _p(count), _p(exp),
           _p(nwork), _p(_d(xq)), _p(_d(xs)), _p(act), W, pairs)
    aq, as_ = O.quant_rows(act.cpu().numpy(), W)
    mo = torch.zeros(pairs, H, dtype=torch.float32, device=DEV)
    R.call("ref_moe_down", _p(dqs), _p(dd), H * (W // 256) * 64, H * (W // 256), _p(order), _p(first), _p(count), _p(exp),
           _p(nwork), _p(_d(aq)), _p(_d(as_)), _p(mo), W, pairs)
    return ({"up_seed": np.int64(81), "down_seed": np.int64(82), "E": np.int32(E), "W": np.int32(W), "H": np.int32(H),
             "ridx": ridx.cpu().numpy(), "xq": xq, "xs": xs, "aq": aq, "as": as_},
            {"act": act.cpu().numpy(), "mo": mo.cpu().numpy()})


def case_combine():
    topn = R.lib().ref_topn()
    T = 2
    o = np.random.default_rng(7).standard_normal((T * topn, 1024)).astype(np.float32)
    rw = np.random.default_rng(8).random(T * topn).astype(np.float32)
    out = torch.zeros(T, 1024, dtype=torch.float32, device=DEV)
    R.call("ref_combine", _p(_d(o)), _p(_d(rw)), _p(out), T)
    return {"o": o, "rw": rw, "topn": np.int32(topn)}, {"out": out.cpu().numpy()}


def case_gemv_iq2():
    # T is one of gemv_k's template row counts (1, 2, 4, 8, 16): gemv_body reads that many x rows
    n, k, T, seed = 64, 512, 4, 91
    blocks = iq2_blocks(seed, n, k)
    _, x = normal_bf16(9, (T, k))
    qs, d = planar_iq2(blocks, n, k)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    R.call("ref_gemv_iq2", _p(qs), _p(d), n, k, _p(_d(x)), k, _p(y), n, T, 0)
    return {"seed": np.int64(seed), "n": np.int32(n), "k": np.int32(k), "x": x}, {"y": y.cpu().numpy()}


def case_gemv_nv4():
    import oracle as O
    n, k, T = 64, 256, 2
    rng = np.random.default_rng(10)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sc = np.array([O.scalar("or_e4m3_enc", float(v)) for v in rng.uniform(0.5, 2, n * k // 16)], np.uint8).reshape(n, k // 16)
    x = rng.standard_normal((T, k)).astype(np.float32)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    R.call("ref_gemv_nv4", _p(_d(q)), _p(_d(sc)), 0.625, n, k, _p(_d(x)), k, _p(y), n, T)
    return {"q": q, "sc": sc, "s2": np.float32(0.625), "x": x}, {"y": y.cpu().numpy()}


def case_gemv_q8():
    n, k, T = 64, 256, 2
    rng = np.random.default_rng(11)
    qv = rng.integers(-127, 128, (n, k), dtype=np.int8)
    dv = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    x = rng.standard_normal((T, k)).astype(np.float32)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    R.call("ref_gemv_q8", _p(_d(qv)), _p(_d(dv)), n, k, _p(_d(x)), k, _p(y), n, T)
    return {"q": qv, "d": dv, "x": x}, {"y": y.cpu().numpy()}


def _tiles(fmt, n, k):
    code = torch.empty(R.lib().ref_tile_bytes(fmt, n, k), dtype=torch.uint8, device=DEV)
    scale = torch.empty(R.lib().ref_tile_scale_bytes(fmt, n, k), dtype=torch.uint8, device=DEV)
    return code, scale


def case_mma_nv4():
    """bolt_mma.cu's NVFP4 tile GEMM (tile_nv4 + mma_nv4: fp16 rows, the e4m3 scales folded exactly into fp16
    operands), n 80 (five 16-row tiles), k 512, 5 rows."""
    import oracle as O
    n, k, T = 80, 512, 5
    rng = np.random.default_rng(12)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sc = np.array([O.scalar("or_e4m3_enc", float(v)) for v in rng.uniform(0.5, 2, n * k // 16)], np.uint8).reshape(n, k // 16)
    x = rng.standard_normal((T, k)).astype(np.float32)
    qt, st = _tiles(0, n, k)
    R.call("ref_tile_nv4", _p(_d(q)), _p(_d(sc)), _p(qt), _p(st), n, k)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    R.call("ref_mma_nv4", _p(qt), _p(st), 0.375, n, k, _p(_d(x)), k, _p(y), n, T)
    return {"q": q, "sc": sc, "s2": np.float32(0.375), "x": x}, {"y": y.cpu().numpy()}


def case_mma_q8():
    """bolt_mma.cu's Q8_0 tile GEMM (tile_q8 + mma_q8: fp16 rows, weights fp16(i8 d)), n 80, k 512, 5 rows."""
    n, k, T = 80, 512, 5
    rng = np.random.default_rng(13)
    qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
    dv = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    blocks = np.concatenate([dv.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1).reshape(n, -1)
    x = rng.standard_normal((T, k)).astype(np.float32)
    qt, st = _tiles(1, n, k)
    R.call("ref_tile_q8", _p(_d(blocks)), _p(qt), _p(st), n, k)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    R.call("ref_mma_q8", _p(qt), _p(st), n, k, _p(_d(x)), k, _p(y), n, T)
    return {"blocks": blocks, "x": x}, {"y": y.cpu().numpy()}


def case_mma_iq2():
    """bolt_mma.cu's IQ2_XXS tile GEMM, the shared expert's (tile_iq2 + mma_iq2: PIQ2's bf16 fold, bf16 rows), n 64,
    k 512, 5 rows, without and with relu^2."""
    n, k, T, seed = 64, 512, 5, 93
    blocks = iq2_blocks(seed, n, k)
    x = np.random.default_rng(14).standard_normal((T, k)).astype(np.float32)
    qt, st = _tiles(2, n, k)
    R.call("ref_tile_iq2", _p(_d(blocks)), _p(qt), _p(st), n, k)
    out = {}
    for epi in (0, 1):
        y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
        R.call("ref_mma_iq2", _p(qt), _p(st), n, k, _p(_d(x)), k, _p(y), n, T, epi)
        out[f"y{epi}"] = y.cpu().numpy()
    return {"seed": np.int64(seed), "n": np.int32(n), "k": np.int32(k), "x": x}, out


def case_quant_nv4_rows():
    """bolt_mma.cu's row quantiser of the NVFP4 prompt path (quant_nv4_rows_k: e4m3 scale amax/6 a block of 16,
    nearest e2m1), 37 rows of k 512 with per-block magnitudes from zero through e4m3 subnormal scales to saturation;
    the scales are returned in [rows][k/16] order (the kernel stores them step-major, [k/64][(T+3)&~3][4])."""
    T, k = 37, 512
    rng = np.random.default_rng(15)
    x = rng.standard_normal((T, k)).astype(np.float32)
    mag = rng.choice(np.array([0.0, 1e-4, 3e-3, 0.05, 1.0, 30.0, 5000.0], np.float32), size=(T, k // 16, 1))
    x = (x.reshape(T, k // 16, 16) * mag).reshape(T, k)
    Tp = (T + 3) & ~3
    q4 = torch.zeros(T, k // 2, dtype=torch.uint8, device=DEV)
    sf = torch.zeros(k // 64, Tp, 4, dtype=torch.uint8, device=DEV)
    R.call("ref_quant_nv4_rows", _p(_d(x)), k, _p(q4), _p(sf), T, k)
    sf_rows = sf.cpu().numpy()[:, :T, :].transpose(1, 0, 2).reshape(T, k // 16)
    return {"x": x}, {"q4": q4.cpu().numpy(), "sf": sf_rows}


CASES = {name[5:]: fn for name, fn in dict(globals()).items() if name.startswith("case_")}


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    for name, fn in CASES.items():
        inputs, outputs = fn()
        _KEEP.clear()
        np.savez_compressed(os.path.join(out_dir, f"ref_{name}.npz"),
                            **{f"in_{k}": v for k, v in inputs.items()}, **{f"out_{k}": v for k, v in outputs.items()})
        print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
