"""The GGUF reader (drift_b200/gguf.py) against files gguf-py's GGUFWriter
writes -- the writer the reference's own GGUF fixture comes from
(runner/fixtures/generate.py:143-176: every metadata value type, F32 and F16
tensors, quantized rows of the golden fixture blocks) -- and the reference
reader's refusals (formats/Gguf.scala:185-287; GgufTests)."""

import os
import struct

import numpy as np
import pytest

import oracle
from drift_b200 import gguf
from tests.conftest import read_safetensors

gguf_py = pytest.importorskip("gguf")


def write(path, tensors=True, alignment=None):
    from gguf import GGMLQuantizationType as T
    from gguf import GGUFWriter

    writer = GGUFWriter(str(path), "llama")
    if alignment:
        writer.add_custom_alignment(alignment)
    writer.add_uint8("test.u8", 200)
    writer.add_int8("test.i8", -100)
    writer.add_uint16("test.u16", 60000)
    writer.add_int16("test.i16", -30000)
    writer.add_uint32("test.u32", 4000000000)
    writer.add_int32("test.i32", -2000000000)
    writer.add_float32("test.f32", 1.5)
    writer.add_uint64("test.u64", 2**63 + 5)
    writer.add_int64("test.i64", -(2**62))
    writer.add_float64("test.f64", 2.25)
    writer.add_bool("test.bool", True)
    writer.add_string("test.string", "héllo")
    writer.add_array("test.ints", [1, 2, 3])
    writer.add_array("test.strings", ["a", "bc"])
    expected = {}
    if tensors:
        f32 = np.arange(15, dtype=np.float32).reshape(3, 5)
        writer.add_tensor("f32", f32)
        expected["f32"] = (oracle.F32, f32)
        writer.add_tensor("f16", f32.astype(np.float16))
        expected["f16"] = (oracle.F16, f32)
        golden = os.path.join(os.path.dirname(__file__), "golden", "quants")
        for quant, name, dtype in [(T.Q8_0, "q8_0", oracle.Q8_0), (T.Q4_K, "q4_k", oracle.Q4_K),
                                   (T.Q6_K, "q6_k", oracle.Q6_K), (T.Q4_1, "q4_1", oracle.Q4_1)]:
            fixture = read_safetensors(os.path.join(golden, f"{name}.safetensors"))
            blocks, values = fixture["blocks"][2:4], fixture["expected"][2:4]
            writer.add_tensor(name, blocks.reshape(1, -1), raw_dtype=quant)
            expected[name] = (dtype, values.reshape(1, -1))
        # a type this library has no kernels for
        q5k = np.zeros((1, 176), dtype=np.uint8)
        writer.add_tensor("q5_k", q5k, raw_dtype=T.Q5_K)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    return expected


def test_metadata_of_every_type(tmp_path):
    path = tmp_path / "tiny.gguf"
    write(path)
    f = gguf.open_file(str(path))
    assert f.version == 3 and f.alignment == 32
    assert f.architecture == "llama"
    assert f.long("test.u8") == 200 and f.long("test.i8") == -100
    assert f.long("test.u16") == 60000 and f.long("test.i16") == -30000
    assert f.long("test.u32") == 4000000000 and f.long("test.i32") == -2000000000
    assert f.double("test.f32") == 1.5 and f.double("test.f64") == 2.25
    assert f.metadata["test.u64"] == 2**63 + 5  # above a Long: kept, and not a long
    with pytest.raises(gguf.FormatError, match="test.u64"):
        f.long("test.u64")
    assert f.long("test.i64") == -(2**62)
    assert f.boolean("test.bool") is True
    assert f.string("test.string") == "héllo"
    assert f.metadata["test.ints"] == [1, 2, 3]
    assert f.strings("test.strings") == ["a", "bc"]
    with pytest.raises(gguf.FormatError, match="has no test.missing"):
        f.string("test.missing")
    with pytest.raises(gguf.FormatError, match="test.u8 is"):
        f.string("test.u8")


def test_tensors_decode_to_their_values(tmp_path):
    path = tmp_path / "tiny.gguf"
    expected = write(path)
    f = gguf.open_file(str(path))
    assert set(f.tensors) == set(expected)
    assert "q5_k" in f.unsupported
    for name, (dtype, values) in expected.items():
        t = f.tensors[name]
        assert t.dtype == dtype
        assert t.shape == values.shape  # outermost first
        decoded = oracle.decode(dtype, np.asarray(t.data), values.size).reshape(values.shape)
        assert np.array_equal(decoded.view(np.uint32), values.astype(np.float32).view(np.uint32))
        assert t.offset % f.alignment == 0


def test_alignment_from_metadata(tmp_path):
    path = tmp_path / "aligned.gguf"
    write(path, alignment=64)
    f = gguf.open_file(str(path))
    assert f.alignment == 64
    assert all(t.offset % 64 == 0 for t in f.tensors.values())


def refused(data, match):
    with pytest.raises(gguf.FormatError, match=match):
        gguf.read(bytes(data), "bad.gguf")


def test_refusals(tmp_path):
    path = tmp_path / "tiny.gguf"
    write(path)
    good = bytearray(open(path, "rb").read())
    bad = bytearray(good)
    bad[0:4] = b"GGUG"
    refused(bad, "not a GGUF file")
    bad = bytearray(good)
    bad[4:8] = struct.pack("<I", 4)
    refused(bad, "GGUF version 4 is not supported")
    bad = bytearray(good)
    bad[4:8] = struct.pack(">I", 3)
    refused(bad, "big-endian GGUF is not supported")
    refused(good[:6], "truncated at byte")
    refused(good[:200], "truncated")
    bad = bytearray(good)
    bad[8:16] = struct.pack("<q", -1)
    refused(bad, "tensor count of -1 is not plausible")
    # the data section cut short inside a tensor
    last = gguf.read(bytes(good)).tensors["q4_1"]
    refused(good[:last.offset + last.nbytes - 8], "runs past the end of the file")


def test_a_type_id_read_as_another_type_is_caught_by_its_span(tmp_path):
    """Each tensor's bytes must fill the room up to the next tensor (less
    than the alignment left over): an f32 tensor relabelled as f16 fails."""
    from gguf import GGUFWriter

    path = tmp_path / "span.gguf"
    writer = GGUFWriter(str(path), "llama")
    writer.add_tensor("a", np.zeros((4, 64), dtype=np.float32))
    writer.add_tensor("b", np.zeros((4, 64), dtype=np.float32))
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    data = bytearray(open(path, "rb").read())
    assert gguf.read(bytes(data)).tensors["a"].dtype == oracle.F32
    # tensor "a"'s info: name (8 + 1 bytes), rank, 2 dims, then its type id
    at = data.index(b"\x01\x00\x00\x00\x00\x00\x00\x00a") + 9
    at += 4 + 2 * 8
    assert struct.unpack_from("<I", data, at)[0] == 0
    data[at:at + 4] = struct.pack("<I", 1)  # F16
    refused(data, "a is F16 \\[4, 64\\], 512 bytes, but the file gives it 1024")
