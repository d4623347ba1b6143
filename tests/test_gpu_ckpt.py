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


def test_checkpoint_packs_a_model_moe_layer(tmp_path):
    """pack_moe_layer over the model's naming: the routed slabs and the shared expert byte for byte as the layout
    packer makes them from the same raw bytes"""
    from test_ckpt_cpu import model_moe_checkpoint
    t = model_moe_checkpoint(str(tmp_path))
    ck = b200q.Checkpoint(str(tmp_path))
    for layer, experts, width in ((1, 3, 512), (3, 2, 256)):
        got = ck.pack_moe_layer(layer, experts, width, latent=256)
        names = b200q.moe_layer_tensor_names(layer, experts)
        assert torch.equal(got["up"], b200q.repack_iq2(dev(b"".join(t[x][2] for x in names["up"])), experts * width, 256))
        assert torch.equal(got["down"], b200q.repack_iq2(dev(b"".join(t[x][2] for x in names["down"])), experts * 256, width))
        assert got["shared_width"] == 768 and got["hidden"] == 512
        assert torch.equal(got["shared_up"], b200q.repack_iq2(dev(t[names["shared_up"]][2]), 768, 512))
        assert torch.equal(got["shared_down"], b200q.repack_iq2(dev(t[names["shared_down"]][2]), 512, 768))
    assert b200q.device_error() == 0
    ck.close()
