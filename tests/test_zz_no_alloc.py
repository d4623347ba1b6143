"""The allocation-free decode MoE entry point (b200q_moe_decode_noalloc), for callers that cannot allocate device
memory: a host whose allocator owns the GPU's memory, a plugin that receives only tensors, a loop that must not take
cudaMalloc's implicit synchronisation.  It runs the same launches as b200q_moe_decode on a scratch array that lives
in the library, so its output must match the workspace entry point's.

Collected last (the file name sorts after the others), and written to pass both alone in a fresh process and after
the other tests: the first call on the device sets up the array's address."""
import ctypes

import numpy as np
import pytest
import torch

import b200q

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    L = b200q.lib()
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.b200q_moe_decode_noalloc.restype = i32
    L.b200q_moe_decode_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, f32, vp, i32, vp, vp, vp]
    L.b200q_moe_decode_noalloc_max_bytes.restype = ctypes.c_size_t
    L.b200q_moe_decode_noalloc_max_bytes.argtypes = []
    return L


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _weights(T, H, F, E, seed):
    up = b200q.repack_iq2(b200q.synth_iq2(seed, E * F * (H // 256)), E * F, H)
    down = b200q.repack_iq2(b200q.synth_iq2(seed + 1, E * H * (F // 256)), E * H, F)
    su = b200q.repack_iq2(b200q.synth_iq2(seed + 2, F * (H // 256)), F, H)
    sd = b200q.repack_iq2(b200q.synth_iq2(seed + 3, H * (F // 256)), H, F)
    return up, down, su, sd


def _inputs(T, H, E, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV), torch.randn(T, E, generator=g).to(torch.bfloat16).to(DEV))


@pytest.mark.parametrize("T,H,F,E,topk", [(16, 4096, 2048, 128, 6), (5, 1024, 512, 16, 3)])
def test_noalloc_matches_workspace_entry_point_twice(T, H, F, E, topk):
    L = _lib()
    up, down, su, sd = _weights(T, H, F, E, 900 + E)
    layer = b200q.MoeDecodeLayer(up, down, su, sd, H, F, E, topk, max_tokens=T)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):   # two calls in a row: the second must not see the first one's scratch
        x, lg = _inputs(T, H, E, 10 * call + T)
        want_ridx = torch.full((T, topk), -1, dtype=torch.int32, device=DEV)
        want_rw = torch.zeros(T, topk, dtype=torch.float32, device=DEV)
        want = layer(x, lg, ridx=want_ridx, rw=want_rw).cpu().numpy()
        out = torch.full((T, H), float("nan"), dtype=torch.float32, device=DEV)
        ridx = torch.full((T, topk), -1, dtype=torch.int32, device=DEV)
        rw = torch.zeros(T, topk, dtype=torch.float32, device=DEV)
        st = L.b200q_moe_decode_noalloc(_p(x), _p(lg), _p(up), _p(down), _p(su), _p(sd), T, H, F, E, topk,
                                        b200q.ROUTE_SOFTMAX, None, 1.0, _p(out), b200q.F32, _p(ridx), _p(rw), stream)
        assert st == b200q.OK, L.b200q_strerror(st)
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        # the same deterministic launches on the same inputs: identical bits, routing included
        assert np.array_equal(got, want)
        assert np.array_equal(ridx.cpu().numpy(), want_ridx.cpu().numpy())
        assert np.array_equal(rw.cpu().numpy(), want_rw.cpu().numpy())


def test_noalloc_refuses_shapes_beyond_its_scratch():
    L = _lib()
    assert L.b200q_moe_decode_noalloc_max_bytes() == 3 << 20
    buf = torch.zeros(256, dtype=torch.uint8, device=DEV)
    p = _p(buf)
    # 64 tokens of hidden 8192 need far more than 3 MiB of scratch
    st = L.b200q_moe_decode_noalloc(p, p, p, p, None, None, 64, 8192, 4096, 128, 8, 0, None, 1.0, p, 0, None, None, None)
    assert st == b200q.ENOSPACE
