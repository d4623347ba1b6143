"""CPU tests of checkpoint ingestion (b200q_ckpt_*, csrc/ckpt.cu): safetensors shards written here, opened through the
index or as one file, looked up by name (bytes, shape and dtype exactly as written), and every malformed or missing
piece refused with EINVAL (a NULL handle for the directory itself) before anything reaches the GPU.  The packers'
checks (staging size, names, byte counts) run before their first copy, so they are tested here too."""
import ctypes
import json
import os
import struct

import numpy as np
import pytest

import b200q


def write_safetensors(path, tensors, header_extra=None, raw_header=None):
    """tensors: {name: (dtype, shape, bytes)} -> a safetensors file (8-byte little-endian header length, the JSON
    header padded with spaces to 8 bytes, then the data in order)"""
    header, off, blobs = {}, 0, []
    for name, (dt, shape, data) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        off += len(data)
        blobs.append(data)
    if header_extra:
        header.update(header_extra)
    h = raw_header if raw_header is not None else json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_index(d, weight_map):
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": weight_map}, f)


def synthetic_model(d, seed=0, rows=64, k=512, experts=3, n=64):
    """a two-shard model: IQ2_XXS experts, an NVFP4 projection and a Q8_0 projection of the given sizes; returns
    {name: (dtype, shape, bytes)}"""
    rng = np.random.default_rng(seed)
    t = {}
    for e in range(experts):
        blocks = b200q.synth_iq2_host(seed * 100 + e, rows * (k // 256))
        t[f"layers.1.mixer.experts.{e}.up_proj.weight"] = ("U8", (rows, k // 256, 66), blocks.tobytes())
    t["layers.0.mixer.in_proj.weight"] = ("U8", (n, k // 2), rng.integers(0, 256, n * k // 2, dtype=np.uint8).tobytes())
    sc = rng.integers(0x30, 0x40, n * k // 16, dtype=np.uint8)   # e4m3 codes between 0.5 and 1.9
    t["layers.0.mixer.in_proj.weight_scale"] = ("F8_E4M3", (n, k // 16), sc.tobytes())
    t["layers.0.mixer.in_proj.weight_scale_2"] = ("F32", (), np.float32(0.375).tobytes())
    qv = rng.integers(-127, 128, (n, k // 32, 32), dtype=np.int8)
    dq = rng.uniform(1e-3, 1e-2, (n, k // 32)).astype(np.float16)
    q8 = np.concatenate([dq.view(np.uint8).reshape(n, k // 32, 2), qv.view(np.uint8)], -1)
    t["layers.2.self_attn.q_proj.weight"] = ("U8", (n, k // 32, 34), q8.tobytes())
    t["layers.3.norm.weight"] = ("F32", (4,), np.arange(4, dtype=np.float32).tobytes())
    names = list(t)
    a, b = names[: experts], names[experts:]
    write_safetensors(os.path.join(d, "model-00001-of-00002.safetensors"), {x: t[x] for x in a},
                      header_extra={"__metadata__": {"format": "pt"}})
    write_safetensors(os.path.join(d, "model-00002-of-00002.safetensors"), {x: t[x] for x in b})
    write_index(d, {**{x: "model-00001-of-00002.safetensors" for x in a},
                    **{x: "model-00002-of-00002.safetensors" for x in b}})
    return t


def test_open_index_and_read_tensors(tmp_path):
    t = synthetic_model(str(tmp_path))
    ck = b200q.Checkpoint(str(tmp_path))
    assert len(ck) == len(t)
    for name, (dt, shape, data) in t.items():
        view, shp, dtype = ck.tensor(name)
        assert view.tobytes() == data and shp == tuple(shape) and dtype == dt
    with pytest.raises(b200q.B200QError):
        ck.tensor("layers.9.missing.weight")
    ck.close()


def test_single_file_without_index(tmp_path):
    data = np.arange(24, dtype=np.int32).tobytes()
    write_safetensors(str(tmp_path / "model.safetensors"),
                      {"a": ("I32", (2, 3, 4), data), "café \"q\"": ("U8", (3,), b"xyz")})
    ck = b200q.Checkpoint(str(tmp_path))
    assert len(ck) == 2
    view, shp, dt = ck.tensor("a")
    assert view.tobytes() == data and shp == (2, 3, 4) and dt == "I32"
    assert ck.tensor("café \"q\"")[0].tobytes() == b"xyz"   # escapes and UTF-8 in the JSON header


def test_empty_directory_and_bad_index_are_refused(tmp_path):
    with pytest.raises(b200q.B200QError):
        b200q.Checkpoint(str(tmp_path))
    (tmp_path / "model.safetensors.index.json").write_text('{"weight_map": {"a": "s.safetensors",}}')
    with pytest.raises(b200q.B200QError):
        b200q.Checkpoint(str(tmp_path))
    write_index(str(tmp_path), {"a": "../outside.safetensors"})   # a shard outside the directory
    with pytest.raises(b200q.B200QError):
        b200q.Checkpoint(str(tmp_path))


@pytest.mark.parametrize("case", ["offset past the file", "bytes not dtype x shape", "header longer than the file",
                                  "header not JSON", "offsets reversed"])
def test_malformed_shards_are_refused(tmp_path, case):
    d = str(tmp_path)
    path = os.path.join(d, "s.safetensors")
    good = {"a": ("F32", (2,), np.zeros(2, np.float32).tobytes())}
    if case == "offset past the file":
        write_safetensors(path, good, raw_header=json.dumps(
            {"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode())
    elif case == "bytes not dtype x shape":
        write_safetensors(path, {"a": ("F32", (3,), np.zeros(2, np.float32).tobytes())})
    elif case == "header longer than the file":
        write_safetensors(path, good)
        with open(path, "r+b") as f:
            f.write(struct.pack("<Q", 1 << 20))
    elif case == "header not JSON":
        write_safetensors(path, good, raw_header=b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]')
    else:
        write_safetensors(path, good, raw_header=json.dumps(
            {"a": {"dtype": "F32", "shape": [2], "data_offsets": [8, 0]}}).encode())
    write_index(d, {"a": "s.safetensors"})
    ck = b200q.Checkpoint(d)   # the index opens; the shard is read at the first lookup
    with pytest.raises(b200q.B200QError):
        ck.tensor("a")


def test_packers_check_everything_before_the_first_copy(tmp_path):
    """staging too small, a missing expert among present ones, a tensor of the wrong size, an NVFP4 prefix without
    its scale: refused before any copy (fake device pointers, never touched)"""
    t = synthetic_model(str(tmp_path), rows=64, k=512, experts=3, n=64)
    L = b200q.lib()
    h = L.b200q_ckpt_open(os.fsencode(str(tmp_path)))
    assert h
    fake, null = ctypes.c_void_p(1 << 20), ctypes.c_void_p()
    rows, k = 64, 512
    need = L.b200q_ckpt_staging_bytes(0, rows, k)
    assert need == rows * (k // 256) * 66
    names = [n for n in t if ".experts." in n]
    arr = lambda xs: (ctypes.c_char_p * len(xs))(*[x.encode() for x in xs])
    assert L.b200q_ckpt_pack_iq2_slab(h, arr(names), 3, rows, k, fake, fake, need - 16, null) == b200q.ENOSPACE
    assert L.b200q_ckpt_pack_iq2_slab(h, arr(names[:2] + ["no.such.weight"]), 3, rows, k, fake, fake, need,
                                      null) == b200q.EINVAL
    assert L.b200q_ckpt_pack_iq2_slab(h, arr(names), 3, rows, 256, fake, fake, need, null) == b200q.EINVAL   # sizes
    assert L.b200q_ckpt_pack_iq2_slab(h, arr(names), 3, 48, k, fake, fake, need, null) == b200q.EINVAL      # rows % 32
    s2 = ctypes.c_float()
    nv = L.b200q_ckpt_staging_bytes(1, 64, 512)
    assert L.b200q_ckpt_pack_nv4(h, b"layers.0.mixer.in_proj", 64, 512, fake, ctypes.byref(s2), fake, nv - 1,
                                 null) == b200q.ENOSPACE
    assert L.b200q_ckpt_pack_nv4(h, b"layers.0.mixer.out_proj", 64, 512, fake, ctypes.byref(s2), fake, nv,
                                 null) == b200q.EINVAL
    q8 = L.b200q_ckpt_staging_bytes(2, 64, 512)
    assert q8 == 64 * 16 * 34
    assert L.b200q_ckpt_pack_q8(h, b"layers.2.self_attn.q_proj.weight", 64, 256, fake, fake, q8, null) == b200q.EINVAL
    assert L.b200q_ckpt_pack_q8(h, b"layers.3.norm.weight", 64, 512, fake, fake, q8, null) == b200q.EINVAL
    L.b200q_ckpt_close(h)


def test_packers_refuse_a_swapped_shape(tmp_path):
    """rows and k swapped give the same byte count in another layout: the packers read the shape, as the reference's
    loaders do (load_iq2 / load_q8 / load_nv4 take n and k from it), and refuse before any copy"""
    rng = np.random.default_rng(4)
    iq2 = b200q.synth_iq2_host(3, 64 * 4).tobytes()                       # 64 rows, k 1024
    q8 = rng.integers(0, 256, 64 * 16 * 34, dtype=np.uint8).tobytes()      # n 64, k 512
    nq = rng.integers(0, 256, 64 * 256, dtype=np.uint8).tobytes()          # n 64, k 512
    ns = rng.integers(0x30, 0x40, 64 * 32, dtype=np.uint8).tobytes()
    write_safetensors(os.path.join(str(tmp_path), "model.safetensors"), {
        "e.weight": ("U8", (64, 4, 66), iq2), "q.weight": ("U8", (64, 16, 34), q8),
        "p.weight": ("U8", (64, 256), nq), "p.weight_scale": ("F8_E4M3", (64, 32), ns),
        "p.weight_scale_2": ("F32", (), np.float32(1).tobytes()),
    })
    L = b200q.lib()
    h = L.b200q_ckpt_open(os.fsencode(str(tmp_path)))
    assert h
    fake, null = ctypes.c_void_p(1 << 20), ctypes.c_void_p()
    arr = lambda xs: (ctypes.c_char_p * len(xs))(*[x.encode() for x in xs])
    # each request below has the tensor's byte count but not its shape
    need = L.b200q_ckpt_staging_bytes(0, 256, 256)
    assert need == len(iq2)
    assert L.b200q_ckpt_pack_iq2_slab(h, arr(["e.weight"]), 1, 256, 256, fake, fake, need, null) == b200q.EINVAL
    q8b = L.b200q_ckpt_staging_bytes(2, 16, 2048)
    assert q8b == len(q8)
    assert L.b200q_ckpt_pack_q8(h, b"q.weight", 16, 2048, fake, fake, q8b, null) == b200q.EINVAL
    s2 = ctypes.c_float()
    nv = L.b200q_ckpt_staging_bytes(1, 128, 256)
    assert L.b200q_ckpt_pack_nv4(h, b"p", 128, 256, fake, ctypes.byref(s2), fake, nv, null) == b200q.EINVAL
    L.b200q_ckpt_close(h)


def test_tensor_view_outlives_the_checkpoint(tmp_path):
    """a view from tensor() keeps the shard mapped: reading it after close() or after the Checkpoint is collected
    returns the bytes (it used to read unmapped memory)"""
    import gc
    t = synthetic_model(str(tmp_path))
    name = "layers.2.self_attn.q_proj.weight"
    ck = b200q.Checkpoint(str(tmp_path))
    v1 = ck.tensor(name)[0]
    ck.close()
    with pytest.raises(b200q.B200QError):
        ck.tensor(name)
    v2 = b200q.Checkpoint(str(tmp_path)).tensor(name)[0]   # the Checkpoint object is dropped at once
    gc.collect()
    assert v1.tobytes() == t[name][2] and v2.tobytes() == t[name][2]
    del v1, v2
    gc.collect()


def test_mutated_headers_never_escape_the_file(tmp_path):
    """300 seeded mutations (byte flips, cuts, duplications) of a valid header: every lookup either fails with EINVAL
    or returns a tensor that lies inside the file with a byte count matching its dtype and shape; nothing crashes"""
    rng = np.random.default_rng(11)
    tensors = {"w": ("F32", (3, 5), np.arange(15, dtype=np.float32).tobytes()),
               "b": ("BF16", (7,), bytes(14)), "s": ("U8", (2, 2, 2), bytes(range(8)))}
    base = json.dumps({n: {"dtype": dt, "shape": list(sh), "data_offsets": [o, o + len(b)]}
                       for (n, (dt, sh, b)), o in zip(tensors.items(), [0, 60, 74])}).encode()
    data = b"".join(b for _, _, b in tensors.values())
    elt = {"F32": 4, "BF16": 2, "U8": 1}
    for i in range(300):
        h = bytearray(base)
        for _ in range(int(rng.integers(1, 4))):
            op, at = int(rng.integers(0, 3)), int(rng.integers(0, len(h)))
            if op == 0:
                h[at] = int(rng.integers(0, 256))
            elif op == 1:
                del h[at:at + int(rng.integers(1, 8))]
            else:
                h[at:at] = h[max(0, at - 8):at]
        d = tmp_path / f"m{i}"
        d.mkdir()
        hb = bytes(h) + b" " * ((8 - len(h) % 8) % 8)
        with open(d / "model.safetensors", "wb") as f:
            f.write(struct.pack("<Q", len(hb)) + hb + data)
        try:
            ck = b200q.Checkpoint(str(d))
        except b200q.B200QError:
            continue
        size = os.path.getsize(d / "model.safetensors")
        for name in ["w", "b", "s", "x"]:
            try:
                view, shape, dt = ck.tensor(name)
            except b200q.B200QError:
                continue
            n = int(np.prod(shape)) if shape else 1
            assert dt not in elt or view.nbytes == n * elt[dt]
            assert view.nbytes <= size - 8 - len(hb)
        ck.close()


def model_moe_checkpoint(d, layers=((1, 3, 512), (3, 2, 256)), latent=256, hidden=512, shared_width=768, seed=7):
    """a checkpoint with the model's own tensor names (libbolt's loader, bolt_host.cu:316, 994-995) at small sizes:
    MoE layers (layer, experts, width), each with its routed experts in the latent space and one shared expert on the
    hidden size; returns {name: (dtype, shape, bytes)}"""
    t = {}
    for li, (layer, experts, width) in enumerate(layers):
        names = b200q.moe_layer_tensor_names(layer, experts)
        for e in range(experts):
            for name, rows, k in ((names["up"][e], width, latent), (names["down"][e], latent, width)):
                blob = b200q.synth_iq2_host(seed * 1000 + li * 100 + e * 2 + (rows == latent), rows * (k // 256)).tobytes()
                t[name] = ("U8", (rows, k // 256, 66), blob)
        for name, rows, k in ((names["shared_up"], shared_width, hidden), (names["shared_down"], hidden, shared_width)):
            t[name] = ("U8", (rows, k // 256, 66), b200q.synth_iq2_host(seed + rows + k, rows * (k // 256)).tobytes())
    t["language_model.backbone.norm_f.weight"] = ("F32", (4,), np.ones(4, np.float32).tobytes())
    names = sorted(t)
    half = len(names) // 2
    for i, part in enumerate((names[:half], names[half:])):
        write_safetensors(os.path.join(d, f"model-{i + 1:05d}-of-00002.safetensors"), {x: t[x] for x in part})
    write_index(d, {x: f"model-{(0 if j < half else 1) + 1:05d}-of-00002.safetensors" for j, x in enumerate(names)})
    return t


def test_model_names_resolve(tmp_path):
    """every tensor libbolt's loader asks for, by the model's naming, is found with its shape"""
    t = model_moe_checkpoint(str(tmp_path))
    ck = b200q.Checkpoint(str(tmp_path))
    for layer, experts, width in ((1, 3, 512), (3, 2, 256)):
        names = b200q.moe_layer_tensor_names(layer, experts)
        for e in range(experts):
            assert ck.tensor_shape(names["up"][e]) == (width, 1, 66)
            assert ck.tensor_shape(names["down"][e]) == (256, width // 256, 66)
        assert ck.tensor_shape(names["shared_up"]) == (768, 2, 66)
        assert ck.tensor_shape(names["shared_down"]) == (512, 3, 66)
    assert names["up"][0] == "language_model.backbone.layers.3.mixer.experts.0.up_proj.weight"
    with pytest.raises(b200q.B200QError):
        ck.tensor_shape(b200q.moe_layer_tensor_names(1, 4)["up"][3])   # layer 1 has three experts
    ck.close()


def test_moe_schedule_reader(tmp_path):
    """the contract's MoE schedule: parsed and checked entry by entry"""
    c = {"hidden": 4096, "moe_latent_size": 1024, "shared_expert_width": 5376,
         "moe_schedule": [{"layer": 1, "experts": 240, "width": 2048, "top_k": 9},
                          {"layer": 3, "experts": 240, "width": 1536, "top_k": 9}]}
    p = tmp_path / "bolt.json"
    p.write_text(json.dumps(c))
    sched, info = b200q.read_moe_schedule(str(p))
    assert sched == [(1, 240, 2048, 9), (3, 240, 1536, 9)]
    assert info == {"latent": 1024, "shared_width": 5376, "hidden": 4096}
    c["moe_schedule"].append({"layer": 5, "experts": 240, "width": 1000, "top_k": 9})   # not a multiple of 256
    p.write_text(json.dumps(c))
    with pytest.raises(b200q.B200QError):
        b200q.read_moe_schedule(str(p))


def test_real_contract_schedule():
    """the reference's own contract, where its checkout is at hand: 40 MoE layers of 240 to 496 experts, widths 1536
    to 2560, top-9, latent 1024, shared expert 5376 wide"""
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.environ.get("B200Q_CONTRACT",
                          os.path.join(os.path.dirname(os.path.dirname(here)), "reference", "contract", "bolt.json"))
    if not os.path.exists(path):
        pytest.skip("the model's contract file is not present")
    sched, info = b200q.read_moe_schedule(path)
    assert len(sched) == 40 and info["latent"] == 1024 and info["shared_width"] == 5376
    assert {e for _, e, _, _ in sched} <= {240, 304, 368, 432, 496}
    assert {w for _, _, w, _ in sched} <= {1536, 2048, 2304, 2560} and {k for *_, k in sched} == {9}
