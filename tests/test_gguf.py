"""GGUF reader (b2q_gguf_*) on the CPU: files written by gguf-py parse back to
the same tensor names, ggml types, shapes and bytes; corrupt files are
rejected with an error status, never a crash."""
import ctypes as C

import numpy as np
import pytest

import b2q
from b2q import synth

gguf = pytest.importorskip("gguf")


def write(path, tensors, alignment=None):
    w = gguf.GGUFWriter(str(path), "siglip2")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_string("general.name", "reader test")
    w.add_array("test.ints", [1, 2, 3])
    w.add_array("test.strings", ["x", "yz"])
    w.add_float32("test.f", 1.5)
    for name, (arr, raw) in tensors.items():
        if raw is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.mark.parametrize("alignment", [None, 64])
def test_reader_roundtrip(tmp_path, alignment):
    rng = np.random.default_rng(0)
    a32 = rng.standard_normal((3, 40)).astype(np.float32)
    a16 = rng.standard_normal(96).astype(np.float16)
    wq = synth.quantize_q8_0(rng.standard_normal((4, 64)).astype(np.float32))
    scal = np.array([2.302585], np.float32)
    p = tmp_path / "t.gguf"
    write(p, {"v.a": (a32, None), "v.b.bias": (a16, None),
              "v.c.weight": (wq.reshape(4, 2 * 34), gguf.GGMLQuantizationType.Q8_0),
              "mm.logit_scale": (scal, None)}, alignment)
    g = b2q.Gguf(p)
    ts = {n: (t, ne, addr) for n, t, ne, addr in g.tensors()}
    assert list(ts) == ["v.a", "v.b.bias", "v.c.weight", "mm.logit_scale"]
    assert ts["v.a"][:2] == (b2q.GGML_F32, (40, 3))
    assert ts["v.b.bias"][:2] == (1, (96,))
    assert ts["v.c.weight"][:2] == (b2q.GGML_Q8_0, (64, 4))
    assert C.string_at(ts["v.a"][2], a32.nbytes) == a32.tobytes()
    assert C.string_at(ts["v.b.bias"][2], a16.nbytes) == a16.tobytes()
    assert C.string_at(ts["v.c.weight"][2], wq.nbytes) == wq.tobytes()
    assert g.scalar("mm.logit_scale") == np.float32(2.302585)
    with pytest.raises(b2q.B2QError):
        g.scalar("no.such.tensor")
    g.close()


def test_reader_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(b2q.B2QError) as e:
        b2q.Gguf(p)
    assert e.value.status == b2q.ERR_INVALID
    good = tmp_path / "good.gguf"
    write(good, {"v.a": (np.ones((2, 8), np.float32), None)})
    data = good.read_bytes()
    for cut in (20, len(data) // 2, len(data) - 8):
        t = tmp_path / f"cut{cut}.gguf"
        t.write_bytes(data[:cut])
        with pytest.raises(b2q.B2QError):
            b2q.Gguf(t)
    with pytest.raises(b2q.B2QError):
        b2q.Gguf(tmp_path / "missing.gguf")


def test_synthetic_checkpoint_lists_every_tensor(tmp_path):
    from gguf_util import write_checkpoint
    cfg = synth.TowerConfig(n_layer=1, vocab=64)
    ck = synth.text_checkpoint(cfg, seed=1)
    p = tmp_path / "text.gguf"
    write_checkpoint(p, ck)
    g = b2q.Gguf(p)
    names = {n: (t, ne) for n, t, ne, _ in g.tensors()}
    assert set(names) == set(ck.tensors)
    assert names["t.token_embd.weight"] == (b2q.GGML_Q8_0, (1152, 64))
    assert names["t.blk.0.ffn_down.weight"] == (b2q.GGML_Q8_0, (4320, 1152))
    assert names["t.final_ln.weight"] == (b2q.GGML_F32, (1152,))


def _patched(data: bytes, name: str, ne0=None, offset=None) -> bytes:
    """The file with one tensor-info entry's ne[0] and/or data offset
    overwritten (entry layout: u64 name length, name, u32 n_dims,
    u64 ne[n_dims], u32 type, u64 offset)."""
    import struct
    key = struct.pack("<Q", len(name)) + name.encode()
    i = data.index(key) + len(key)
    n_dims = struct.unpack_from("<I", data, i)[0]
    b = bytearray(data)
    if ne0 is not None:
        struct.pack_into("<Q", b, i + 4, ne0)
    if offset is not None:
        struct.pack_into("<Q", b, i + 4 + 8 * n_dims + 4, offset)
    return bytes(b)


@pytest.mark.parametrize("field,value", [
    ("ne0", 1 << 61),            # 2 x 2^61 F32 elements: 2^64 bytes, a size that wraps to 0
    ("ne0", (1 << 61) - 1),      # 2^64 - 8 bytes: offset + size wraps past the file end
    ("offset", (1 << 64) - 64),  # an offset that wraps when added to the data start
    ("offset", 1 << 40),         # simply past the end of the file
])
def test_reader_rejects_overflowing_sizes(tmp_path, field, value):
    # shapes or offsets whose byte arithmetic would wrap a 64-bit size are
    # reported as errors, never accepted with a wrapped size
    good = tmp_path / "good.gguf"
    write(good, {"v.a": (np.ones((2, 8), np.float32), None)})
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(_patched(good.read_bytes(), "v.a", **{field: value}))
    with pytest.raises(b2q.B2QError):
        b2q.Gguf(bad)
