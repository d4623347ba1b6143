"""libbolt as a drop-in: the reference's own host code and kernels (engine/bolt_host.cu, bolt_kernels.cu, bolt_draft.cu,
bolt_mma.cu from a guarded build copy) compiled for sm_100a and linked against libb200q.so with their hot-path launchers
made local (oracle/build_oracle.py build_bolt_link), so that bolt_host.cu's MoE block and projections call this
engine's shims.  The link must export every symbol of libbolt's C ABI (engine/bolt.def, the 45 names TensorFold's
lane backend binds) and leave each launcher libb200q.so defines undefined, bound to libb200q.so at load time."""
import ctypes
import os
import subprocess

import pytest

import build_oracle

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_LIB = os.path.join(os.path.dirname(HERE), "nemotron-3.5-bolt-tensorfold-dgx-spark_b200", "libb200q.so")
BOLT_DEF = os.path.join(build_oracle.ENGINE, "bolt.def")


def _dyn(path, flag):
    r = subprocess.run(["nm", "-D", flag, path], capture_output=True, text=True, check=True)
    return {f[-1] for f in (l.split() for l in r.stdout.splitlines()) if f}


@pytest.fixture(scope="module")
def linked():
    # built here from the reference's sources; where they are absent (a GPU box), the prebuilt library that travels
    # with the repository
    path = build_oracle.build_bolt_link()
    if not path or not os.path.exists(path):
        pytest.skip("neither the reference checkout nor a prebuilt linked library is present")
    return path


def test_exports_libbolt_c_abi(linked):
    if not os.path.exists(BOLT_DEF):
        pytest.skip("the reference checkout (engine/bolt.def) is not present")
    names = [l.strip() for l in open(BOLT_DEF) if l.strip().startswith("bolt_")]
    assert len(names) == 45
    exported = _dyn(linked, "--defined-only")
    assert set(names) <= exported, sorted(set(names) - exported)


def test_hot_path_binds_to_libb200q(linked):
    # libb200q's libbolt-signature launchers: its exports other than the C ABI and C++ standard-library template
    # instances (which every C++ library exports alike)
    std = ("_ZNSt", "_ZSt", "_ZNKSt", "_ZN9__gnu_cxx", "_ZNK9__gnu_cxx")
    shims = {s for s in _dyn(PKG_LIB, "--defined-only") if not s.startswith("b200q_") and not s.startswith(std)}
    undefined = _dyn(linked, "--undefined-only")
    bound = shims & undefined
    # the routed-expert block, the shared expert, the decode projections and the NVFP4 prompt path (BOLT_NV4_FP4):
    # 28 launchers with libbolt's names
    demangled = subprocess.run(["c++filt"], input="\n".join(sorted(bound)), capture_output=True, text=True).stdout
    for name in ("moe_up(", "moe_down(", "k_route(", "k_moe_group(", "k_quant_rows(", "k_combine(", "repack_iq2(",
                 "moe_coop_dense(", "mma_nv4(", "mma_q8(", "mma_q8_multi(", "mma_iq2(", "tile_nv4(", "tile_q8(",
                 "tile_iq2(", "tile_nv4w(", "quant_nv4_rows(", "mma_nv4_fp4("):
        assert name in demangled, name
    assert len(bound) == 28
    # and none of them is still defined inside the linked library
    assert not (shims & _dyn(linked, "--defined-only"))
    needed = subprocess.run(["readelf", "-d", linked], capture_output=True, text=True, check=True).stdout
    assert "[libb200q.so]" in needed


@pytest.mark.gpu
def test_linked_library_loads_and_answers(linked):
    """on a GPU box (the driver's libcuda present): the linked libbolt loads, its dependency resolves to this engine,
    and its ABI version is libbolt's (bolt_abi, bolt_native.zig checks 3)"""
    L = ctypes.CDLL(linked)
    L.bolt_abi.restype = ctypes.c_int
    assert L.bolt_abi() == 3
