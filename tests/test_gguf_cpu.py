"""The C++ GGUF reader (q8lin_gguf_*) on files written by tests/gguf_writer.py.

No GPU: parsing, metadata, tensor infos and bytes, and the rejection of malformed
files (the reader maps the file and must never read outside it).
"""
import struct

import numpy as np
import pytest

from talechime_b200 import _lib, synth
from talechime_b200._lib import Q8LinError
from talechime_b200.gguf import GGUFFile
from tests import gguf_writer as gw


def _sample(version=3, alignment=32):
    rng = np.random.default_rng(5)
    w = gw.Writer(version=version, alignment=alignment)
    w.add("general.architecture", gw.STRING, "minicpm4")
    w.add("minicpm4.block_count", gw.U32, 28)
    w.add("minicpm4.embedding_length", gw.U32, 2048)
    w.add("u8", gw.U8, 200).add("i8", gw.I8, -5).add("u16", gw.U16, 65000).add("i16", gw.I16, -30000)
    w.add("i32", gw.I32, -7).add("f32", gw.F32, 1.5).add("flag", gw.BOOL, 1).add("u64", gw.U64, 2 ** 40)
    w.add("i64", gw.I64, -(2 ** 40)).add("f64", gw.F64, 2.25).add("empty", gw.STRING, "")
    w.add("ints", gw.ARRAY, (gw.I32, [1, -2, 3]))
    w.add("tokens", gw.ARRAY, (gw.STRING, ["<s>", "héllo", ""]))
    w.add("nested", gw.ARRAY, (gw.ARRAY, [(gw.U8, [1, 2]), (gw.U8, [])]))
    norm = rng.standard_normal(96).astype(np.float32)
    half = rng.standard_normal((3, 8)).astype(np.float16)
    blocks = synth.q8_0_blocks(rng, 5, 64)
    w.f32("blk.0.attn_norm.weight", norm)
    w.tensor("half", (8, 3), gw.GGML_F16, half.tobytes())
    w.q8_0("blk.0.attn_q.weight", blocks, 64)
    return w, norm, half, blocks


def test_reads_metadata_tensor_infos_and_bytes(tmp_path):
    w, norm, half, blocks = _sample()
    with GGUFFile(w.write(tmp_path / "a.gguf")) as g:
        assert g.version == 3
        assert g.value("general.architecture") == "minicpm4"
        g.expect_string("general.architecture", "minicpm4")
        g.expect_u32("minicpm4.block_count", 28)
        assert g.value("u8") == 200 and g.value("i8") == -5 and g.value("u16") == 65000
        assert g.value("i16") == -30000 and g.value("i32") == -7 and g.value("f32") == 1.5
        assert g.value("flag") is True and g.value("u64") == 2 ** 40 and g.value("i64") == -(2 ** 40)
        assert g.value("f64") == 2.25 and g.value("empty") == ""
        assert g.value("ints").tolist() == [1, -2, 3]
        assert g.value("tokens") == ["<s>", "héllo", ""]
        assert g.tensor_names() == ["blk.0.attn_norm.weight", "half", "blk.0.attn_q.weight"]
        info = g.tensor_info("blk.0.attn_q.weight")
        assert info.ggml_type == gw.GGML_Q8_0 and info.ne == (64, 5) and info.shape == (5, 64)
        assert info.nbytes == 5 * 2 * 34
        assert np.array_equal(g.q8_0_blocks("blk.0.attn_q.weight"), blocks.reshape(5, 68))
        assert np.array_equal(g.tensor("blk.0.attn_norm.weight"), norm)
        assert np.array_equal(g.tensor("half"), half.astype(np.float32))
        assert "half" in g and "missing" not in g


@pytest.mark.parametrize("version,alignment", [(2, 32), (3, 64), (3, 8)])
def test_versions_and_alignment(tmp_path, version, alignment):
    w, norm, _, blocks = _sample(version, alignment)
    with GGUFFile(w.write(tmp_path / "a.gguf")) as g:
        assert g.version == version
        assert np.array_equal(g.tensor("blk.0.attn_norm.weight"), norm)
        assert np.array_equal(g.q8_0_blocks("blk.0.attn_q.weight"), blocks.reshape(5, 68))


def test_reference_error_messages(tmp_path):
    w, *_ = _sample()
    with GGUFFile(w.write(tmp_path / "a.gguf")) as g:
        with pytest.raises(Q8LinError, match="unsupported GGUF minicpm4.block_count=28; expected 24"):
            g.expect_u32("minicpm4.block_count", 24)
        with pytest.raises(Q8LinError, match="missing GGUF metadata minicpm4.vocab_size"):
            g.expect_u32("minicpm4.vocab_size", 73448)
        with pytest.raises(Q8LinError) as e:
            g.to_u32("i32")  # a u32 getter takes U32 values only
        assert e.value.status == _lib.ERR_FORMAT
        with pytest.raises(Q8LinError) as e:
            g.tensor_info("blk.9.attn_q.weight")
        assert e.value.status == _lib.ERR_NOT_FOUND
        with pytest.raises(Q8LinError) as e:
            g.tensor("blk.0.attn_q.weight")  # Q8_0 stays quantized
        assert e.value.status == _lib.ERR_FORMAT


def _status(path):
    import ctypes

    h = ctypes.c_void_p()
    st = _lib.lib().q8lin_gguf_open(str(path).encode(), ctypes.byref(h))
    if st == _lib.OK:
        _lib.lib().q8lin_gguf_close(h)
    return st


def test_rejects_malformed_files(tmp_path):
    assert _status(tmp_path / "nope.gguf") == _lib.ERR_IO
    good = _sample()[0].build()
    cases = {
        "magic": b"GGUG" + good[4:],
        "version1": good[:4] + struct.pack("<I", 1) + good[8:],
        "huge_counts": good[:8] + struct.pack("<QQ", 2 ** 62, 2 ** 62) + good[24:],
        "empty": b"",
    }
    w = gw.Writer().tensor("t", (32, 2), gw.GGML_Q8_0, bytes(68), offset=4)  # offset not aligned
    cases["misaligned"] = w.build()
    w = gw.Writer().tensor("t", (32, 2), gw.GGML_Q8_0, bytes(68)).tensor("t", (32, 2), gw.GGML_Q8_0, bytes(68))
    cases["dup_tensor"] = w.build()
    cases["dup_key"] = gw.Writer().add("a", gw.U32, 1).add("a", gw.U32, 2).build()
    cases["five_dims"] = gw.Writer().tensor("t", (1, 1, 1, 1, 1), gw.GGML_F32, bytes(4)).build()
    cases["zero_dim"] = gw.Writer().tensor("t", (0, 4), gw.GGML_F32, b"").build()
    cases["ragged_q8"] = gw.Writer().tensor("t", (48, 2), gw.GGML_Q8_0, bytes(102)).build()
    cases["past_end"] = gw.Writer().tensor("t", (32, 2), gw.GGML_Q8_0, bytes(68), offset=4096).build()
    cases["bad_bool"] = gw.Writer().add("b", gw.BOOL, 7).build()
    cases["bad_type"] = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + _bad_type_kv()
    cases["bad_alignment"] = gw.Writer().add("general.alignment", gw.U32, 24).build()
    for name, data in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(data)
        st = _status(p)
        assert st == _lib.ERR_FORMAT, (name, st, _lib.lib().q8lin_last_error())


def _bad_type_kv():
    return struct.pack("<Q", 1) + b"k" + struct.pack("<I", 13) + b"\0" * 8


def test_every_truncation_is_rejected(tmp_path):
    data = _sample()[0].build()
    p = tmp_path / "t.gguf"
    last_data = len(data) - 1  # cutting anywhere drops bytes some tensor or header needs
    for cut in list(range(0, 400)) + list(range(400, last_data, 97)) + [last_data]:
        p.write_bytes(data[:cut])
        assert _status(p) in (_lib.ERR_FORMAT,), cut


def test_random_corruption_never_reads_outside_the_file(tmp_path):
    """Flip header bytes at random: every open must return a status (OK or FORMAT)."""
    data = bytearray(_sample()[0].build())
    rng = np.random.default_rng(9)
    p = tmp_path / "c.gguf"
    hdr = len(data) - 5 * 68 - 96 * 4 - 48 - 64
    for _ in range(400):
        d = bytearray(data)
        for i in rng.integers(0, hdr, size=rng.integers(1, 4)):
            d[i] = rng.integers(0, 256)
        p.write_bytes(bytes(d))
        assert _status(p) in (_lib.OK, _lib.ERR_FORMAT)
