"""CPU tests of the C ABI: the library loads, exports every entry point include/b200q.h declares, validates its
arguments before touching the GPU, and its host-side generator is deterministic."""
import ctypes
import os
import re

import numpy as np

import b200q
from conftest import ROOT


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "b200q.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200q_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(b200q.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_abi_and_strerror():
    L = b200q.lib()
    assert L.b200q_abi() == 1
    assert L.b200q_strerror(b200q.EINVAL).startswith(b"invalid")


def test_bad_arguments_fail_before_any_launch():
    L = b200q.lib()
    null = None
    assert L.b200q_iq2_pack(null, null, 32, 256, null) == b200q.EINVAL
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert L.b200q_iq2_pack(p, p, 31, 256, null) == b200q.EINVAL       # rows not a multiple of 32
    assert L.b200q_iq2_pack(p, p, 32, 300, null) == b200q.EINVAL       # k not a multiple of 256
    assert L.b200q_route(p, 1, 128, null, 4, 600, 6, 0, 1.0, p, p, null) == b200q.EINVAL   # E > 512
    assert L.b200q_route(p, 1, 128, null, 4, 128, 20, 0, 1.0, p, p, null) == b200q.EINVAL  # topk > 16
    assert L.b200q_moe_group(p, 5000, 128, p, p, p, null) == b200q.EINVAL
    assert L.b200q_quant_rows(p, 0, 64, p, 64, p, 2, 4, 48, null) == b200q.EINVAL         # k % 32
    # decode GEMVs: x off its element size is refused before anything touches it (the addresses are never read)
    w, y = ctypes.c_void_p(0x100000), ctypes.c_void_p(0x300000)
    for x, dt in ((0x200001, b200q.BF16), (0x200002, b200q.F32)):
        assert L.b200q_q8_gemv(w, 64, 512, ctypes.c_void_p(x), dt, 512, 1, y, 64, null, 0, null) == b200q.EINVAL
        assert L.b200q_nv4_gemv(w, 1.0, 64, 512, ctypes.c_void_p(x), dt, 512, 1, y, 64, null, 0, null) == b200q.EINVAL
    # workspace too small / misaligned
    ws = L.b200q_moe_decode_workspace_bytes(16, 4096, 2048, 128, 6)
    assert ws > 16 * 6 * 4096 * 4
    assert L.b200q_moe_decode(p, p, p, p, null, null, 16, 4096, 2048, 128, 6, 0, null, 1.0, p, 0,
                              ctypes.c_void_p(256), ws - 1, null, null, null, null) == b200q.ENOSPACE
    assert L.b200q_moe_decode(p, p, p, p, null, null, 16, 4096, 2048, 128, 6, 0, null, 1.0, p, 0,
                              ctypes.c_void_p(257), ws, null, null, null, null) == b200q.EINVAL
    assert L.b200q_moe_decode(p, p, p, p, p, null, 16, 4096, 2048, 128, 6, 0, null, 1.0, p, 0,
                              ctypes.c_void_p(256), ws, null, null, null, null) == b200q.EINVAL   # half a shared expert


def test_host_generator_is_deterministic_and_in_range():
    a = b200q.synth_iq2_host(7, 100)
    b = b200q.synth_iq2_host(7, 100)
    c = b200q.synth_iq2_host(8, 100)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    blocks = a.reshape(100, 66)
    d = blocks[:, :2].copy().view(np.float16).astype(np.float32)[:, 0]
    assert (d >= 9.99e-4).all() and (d <= 1.001e-2).all()
    qy = np.stack([blocks[:, 6 + 8 * c:10 + 8 * c].copy().view(np.uint32)[:, 0] for c in range(8)], 1)
    s4 = qy >> 28
    assert s4.min() == 0 and s4.max() == 15
    # block i depends only on (seed, i)
    assert np.array_equal(b200q.synth_iq2_host(7, 10), a[:660])


def test_library_exports_the_libbolt_signature_shims():
    """include/b200q_bolt.h's launchers (libbolt's C++ names and signatures) are defined in the library"""
    import shutil
    import subprocess
    import pytest
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    text = open(os.path.join(ROOT, "include", "b200q_bolt.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"^void (\w+)\(", text, flags=re.M)))
    assert {"moe_up", "moe_down", "k_moe_group", "repack_iq2"} <= set(names)
    out = subprocess.run([nm, "-DC", "--defined-only", b200q.LIB_PATH], capture_output=True, text=True).stdout
    missing = [n for n in names if not re.search(r"\b" + n + r"\(CUstream_st\*", out)]
    assert not missing, missing
    sizes = sorted(set(re.findall(r"^size_t (\w+)\(int n, int k\)", text, flags=re.M)))
    assert {"tile_bytes_nv4", "tile_scale_bytes_q8"} <= set(sizes)
    missing = [n for n in sizes if not re.search(r"\b" + n + r"\(int, int\)", out)]
    assert not missing, missing


def test_libbolt_shims_reject_bad_shapes_before_any_launch(capfd):
    """the libbolt-signature shims return nothing, as libbolt's launchers do: a bad shape is reported on stderr
    (prefix "b200q shim") before any CUDA call, so these run without a GPU"""
    import build_harness
    L = ctypes.CDLL(build_harness.build())
    vp = ctypes.c_void_p
    buf = ctypes.create_string_buffer(256)
    p = ctypes.cast(buf, vp)
    L.hs_tile_nv4.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int]
    L.hs_tile_nv4(None, p, p, p, p, 20, 256)                  # n % 16
    L.hs_tile_q8.argtypes = [vp, vp, vp, vp, ctypes.c_int, ctypes.c_int]
    L.hs_tile_q8(None, p, p, p, 32, 300)                      # k % 256
    L.hs_tile_iq2.argtypes = [vp, vp, vp, vp, ctypes.c_int, ctypes.c_int]
    L.hs_tile_iq2(None, p, p, p, 48, 256)                     # n % 32
    L.hs_repack_iq2.argtypes = [vp, vp, vp, vp, ctypes.c_size_t, ctypes.c_int]
    L.hs_repack_iq2(None, p, p, p, 31, 256)                   # rows % 32
    L.hs_mma_iq2.argtypes = [vp, vp, vp] + [ctypes.c_int] * 2 + [vp, ctypes.c_int, vp] + [ctypes.c_int] * 3
    L.hs_mma_iq2(None, p, p, 48, 256, p, 256, p, 48, 4, 1)   # n % 32
    L.hs_mma_nv4.argtypes = [vp, vp, vp, ctypes.c_float] + [ctypes.c_int] * 2 + [vp, ctypes.c_int, vp] + [ctypes.c_int] * 2
    L.hs_mma_nv4(None, p, p, 1.0, 20, 256, p, 256, p, 20, 2)  # n % 16
    err = capfd.readouterr().err
    for name in ("tile_nv4", "tile_q8", "tile_iq2", "repack_iq2", "mma_iq2", "mma_nv4"):
        assert f"b200q shim: {name} failed: invalid" in err, (name, err)
    # libbolt's opt-in bf16 routed path is not provided: moe_bf16() says so, and its launchers only report
    L.hs_moe_bf16.restype = ctypes.c_int
    assert L.hs_moe_bf16() == 0
    L.hs_moe_up_bf.argtypes = [vp]
    L.hs_moe_up_bf(None)
    err = capfd.readouterr().err
    assert "b200q shim: moe_up_bf failed" in err and "b200q shim: moe_down_bf failed" in err
