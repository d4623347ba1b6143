"""GPU parity of the NVFP4 and Q8_0 decode GEMVs (T <= 16) against the CPU oracle's exact mode, through the C ABI.

The kernels' operands are exact (e2m1 * e4m3 and int8 in fp16, bf16 activations in fp16) and only the fp32 summation
order differs from the oracle's fp64 sums, so the bar is far inside BASELINE's (relative L2 <= 1e-2): here 1e-5."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import assert_tolerance, normal_bf16, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def nv4_weights(seed, n, k):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sc = torch.from_numpy(rng.uniform(0.5, 2.0, (n, k // 16)).astype(np.float32)).to(torch.float8_e4m3fn)
    return q, sc.view(torch.uint8).numpy()


def q8_blocks(seed, n, k):
    rng = np.random.default_rng(seed)
    qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
    d = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    return np.concatenate([d.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1).reshape(n, -1)


def np_nv4_t16(q, sc, n, k):
    """numpy statement of the NVFP4 t16 layout (gemv_tc.cu)."""
    nib = np.stack([q & 15, q >> 4], -1).reshape(n, k).astype(np.uint32)
    out = np.zeros((n // 16, k // 64, 576), np.uint8)
    for lane in range(32):
        g, t = lane // 4, lane % 4
        for j in range(4):
            k0 = 16 * j + 2 * t
            rows = [g, g + 8, g, g + 8]
            ks = [k0, k0, k0 + 8, k0 + 8]
            w = np.zeros((n // 16, k // 64), np.uint32)
            for r in range(4):
                lo = nib.reshape(n // 16, 16, k // 64, 64)[:, rows[r], :, ks[r]]
                hi = nib.reshape(n // 16, 16, k // 64, 64)[:, rows[r], :, ks[r] + 1]
                w |= (lo | hi << 4) << (8 * r)
            out[:, :, 16 * lane + 4 * j:16 * lane + 4 * j + 4] = w[..., None].view(np.uint8).reshape(n // 16, k // 64, 4)
    s = sc.reshape(n // 16, 16, k // 64, 4)
    for g in range(8):
        out[:, :, 512 + 8 * g:512 + 8 * g + 4] = s[:, g]
        out[:, :, 512 + 8 * g + 4:512 + 8 * g + 8] = s[:, g + 8]
    return out.reshape(-1)


@pytest.mark.parametrize("n,k", [(16, 256), (64, 512)])
def test_nv4_pack_layout(n, k):
    q, sc = nv4_weights(n + k, n, k)
    got = b200q.tile_nv4(dev(q), dev(sc), n, k).cpu().numpy()
    assert np.array_equal(got, np_nv4_t16(q, sc, n, k))


@pytest.mark.parametrize("n,k,T", [(16, 256, 1), (48, 512, 3), (64, 1024, 9), (18560, 4096, 1), (18560, 4096, 16),
                                   (4096, 8192, 1), (4096, 8192, 16)])
def test_nv4_gemv(n, k, T):
    q, sc = nv4_weights(7 * n + k, n, k)
    xb, x = normal_bf16(T + n, (T, k))
    w = b200q.tile_nv4(dev(q), dev(sc), n, k)
    y = b200q.mma_nv4(w, 0.37, n, k, dev(xb).view(torch.bfloat16)).cpu().numpy()
    ref = O.nv4_gemm_exact(q, sc, 0.37, n, k, x)
    assert rel_l2(y, ref) < 1e-5
    assert_tolerance(y, ref)


def test_nv4_gemv_fp32_input():
    n, k, T = 128, 2048, 5
    q, sc = nv4_weights(3, n, k)
    x = np.random.default_rng(4).standard_normal((T, k)).astype(np.float32)
    w = b200q.tile_nv4(dev(q), dev(sc), n, k)
    y = b200q.mma_nv4(w, 1.0, n, k, dev(x)).cpu().numpy()
    # fp32 activations are rounded to fp16 once (2^-11): compare with the oracle on those rounded rows
    ref = O.nv4_gemm_exact(q, sc, 1.0, n, k, x.astype(np.float16).astype(np.float32))
    assert rel_l2(y, ref) < 1e-5


@pytest.mark.parametrize("n,k,T", [(16, 256, 2), (4096, 4096, 1), (4096, 4096, 16), (1024, 4096, 16), (64, 512, 11)])
def test_q8_gemv(n, k, T):
    blocks = q8_blocks(n + T, n, k)
    xb, x = normal_bf16(3 * T + n, (T, k))
    w = b200q.tile_q8(dev(blocks), n, k)
    y = b200q.mma_q8(w, n, k, dev(xb).view(torch.bfloat16)).cpu().numpy()
    ref = O.q8_gemm_exact(blocks, n, k, x)
    assert rel_l2(y, ref) < 1e-5
    assert_tolerance(y, ref)


def test_gemv_without_workspace_matches_split():
    n, k, T = 256, 4096, 4
    q, sc = nv4_weights(9, n, k)
    xb, _ = normal_bf16(10, (T, k))
    w = b200q.tile_nv4(dev(q), dev(sc), n, k)
    x = dev(xb).view(torch.bfloat16)
    y1 = b200q.mma_nv4(w, 1.0, n, k, x)
    y2 = torch.empty_like(y1)
    L = b200q.lib()
    import ctypes
    st = L.b200q_nv4_gemv(ctypes.c_void_p(w.data_ptr()), 1.0, n, k, ctypes.c_void_p(x.data_ptr()), 1, k, T,
                          ctypes.c_void_p(y2.data_ptr()), n, None, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    assert rel_l2(y2.cpu().numpy(), y1.cpu().numpy()) < 1e-5   # the same products, summed in another order


@pytest.mark.parametrize("fmt", ["nv4", "q8"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T", [1, 3, 16])
@pytest.mark.parametrize("shift", [1, 2])
def test_gemv_unaligned_rows_match_aligned(fmt, dtype, T, shift):
    """x's rows staged four values a load (rows on 4 elements), by pairs (a view 2 elements in, even row pitch) and one
    value at a time (1 element in, odd pitch): the same fp16 operands, so the same outputs bit for bit; the columns
    split over several K slices."""
    n, k = 256, 4096
    if fmt == "nv4":
        q, sc = nv4_weights(91, n, k)
        w = b200q.tile_nv4(dev(q), dev(sc), n, k)
        run = lambda x: b200q.mma_nv4(w, 0.5, n, k, x)
    else:
        w = b200q.tile_q8(dev(q8_blocks(92, n, k)), n, k)
        run = lambda x: b200q.mma_q8(w, n, k, x)
    g = torch.Generator().manual_seed(93 + T)
    x = torch.randn(T, k, generator=g).to(dtype).to(DEV)
    pitch = k + (3 if shift == 1 else 2)
    wide = torch.zeros(T, pitch, dtype=dtype, device=DEV)
    wide[:, shift:k + shift] = x
    xv = wide[:, shift:k + shift]
    assert xv.stride(0) == pitch and xv.data_ptr() % (4 * x.element_size()) != 0
    y0 = run(x).cpu()
    y1 = run(xv).cpu()
    assert b200q.device_error() == 0
    assert torch.equal(y0, y1)
    assert torch.isfinite(y0).all()


def test_gemv_refuses_x_off_its_element_size():
    """an x pointer that is not on its element size is refused on the host, before any launch"""
    import ctypes
    n, k, T = 64, 512, 1
    w = b200q.tile_q8(dev(q8_blocks(94, n, k)), n, k)
    x = torch.zeros(T, k + 8, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(T, n, dtype=torch.float32, device=DEV)
    st = b200q.lib().b200q_q8_gemv(ctypes.c_void_p(w.data_ptr()), n, k, ctypes.c_void_p(x.data_ptr() + 1),
                                   b200q.BF16, k + 8, T, ctypes.c_void_p(y.data_ptr()), n, None, 0, None)
    assert st == b200q.EINVAL
