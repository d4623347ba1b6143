"""GPU parity of checkpoint ingestion: the packers of b200q_ckpt_* (the mapped shard bytes, staged on the device and
packed there) give byte for byte what the layout packers give for the same raw bytes uploaded directly."""
import numpy as np
import pytest
import torch

import b200q
from test_ckpt_cpu import synthetic_model

pytestmark = pytest.mark.gpu
DEV = "cuda"


def dev(b):
    return torch.from_numpy(np.frombuffer(b, dtype=np.uint8).copy()).to(DEV)


def test_checkpoint_packs_match_the_layout_packers(tmp_path):
    rows, k, experts, n = 64, 512, 3, 64
    t = synthetic_model(str(tmp_path), seed=5, rows=rows, k=k, experts=experts, n=n)
    ck = b200q.Checkpoint(str(tmp_path))
    names = [x for x in t if ".experts." in x]
    slab = ck.pack_iq2_slab(names, rows, k)
    raw = b"".join(t[x][2] for x in names)
    assert torch.equal(slab, b200q.repack_iq2(dev(raw), experts * rows, k))
    p = "layers.0.mixer.in_proj"
    w, s2 = ck.pack_nv4(p, n, k)
    assert s2 == 0.375
    assert torch.equal(w, b200q.tile_nv4(dev(t[p + ".weight"][2]), dev(t[p + ".weight_scale"][2]), n, k))
    q = "layers.2.self_attn.q_proj.weight"
    assert torch.equal(ck.pack_q8(q, n, k), b200q.tile_q8(dev(t[q][2]), n, k))
    assert b200q.device_error() == 0
    ck.close()
