"""Checkpoint ingestion on the CPU: the library's safetensors and PWEXPRT1
readers (csrc/pw_checkpoint.cpp) through the C ABI.  No GPU is needed to open,
validate or read a file.  Cases follow the reference's own tests
(src/lib.rs:7734 mapped_safetensors_returns_exact_immutable_tensor_bytes,
:7764 mapped_safetensors_rejects_ambiguous_or_invalid_layouts, :8178
expert_container_round_trips_and_detects_tampering).
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from mimo_prismwing_b200 import checkpoint as C

PW_ERR_FORMAT, PW_ERR_IO = -10, -11


def write_safetensors(path, header: str, payload: bytes, pad=True):
    """The reference test helper's layout: u64 header length, the header padded
    with spaces to a multiple of 8, the payload."""
    h = header.encode()
    while pad and len(h) % 8:
        h += b" "
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + payload)


def test_mapped_safetensors_returns_exact_tensor_bytes(tmp_path):
    p = str(tmp_path / "valid.safetensors")
    write_safetensors(p, '{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},'
                         '"y":{"dtype":"U8","shape":[2],"data_offsets":[8,10]}}', bytes(range(1, 11)))
    with C.MappedSafetensors.open(p) as f:
        assert f.tensor_count() == 2
        x = f.tensor("x")
        assert x.dtype == "F32" and x.shape == (2,)
        assert x.numpy().tobytes() == bytes([1, 2, 3, 4, 5, 6, 7, 8])
        assert f.tensor("y").numpy().tolist() == [9, 10]
        with pytest.raises(C.CheckpointError):
            f.tensor("missing")
        assert f.names() == ["x", "y"]


@pytest.mark.parametrize("name,header,payload", [
    ("duplicate", '{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},'
                  '"x":{"dtype":"U8","shape":[1],"data_offsets":[1,2]}}', bytes(2)),
    ("nested-duplicate", '{"x":{"dtype":"U8","dtype":"U8","shape":[1],"data_offsets":[0,1]}}', bytes(1)),
    ("unknown-dtype", '{"x":{"dtype":"MYSTERY","shape":[1],"data_offsets":[0,1]}}', bytes(1)),
    ("shape-bytes", '{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', bytes(4)),
    ("overlap", '{"x":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},'
                '"y":{"dtype":"U8","shape":[2],"data_offsets":[1,3]}}', bytes(3)),
    ("truncated", '{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}', bytes(7)),
    ("zero-shape", '{"x":{"dtype":"U8","shape":[0],"data_offsets":[0,0]}}', b""),
    ("empty-shape", '{"x":{"dtype":"U8","shape":[],"data_offsets":[0,1]}}', bytes(1)),
    ("reversed", '{"x":{"dtype":"U8","shape":[1],"data_offsets":[1,0]}}', bytes(1)),
    ("negative", '{"x":{"dtype":"U8","shape":[-1],"data_offsets":[0,1]}}', bytes(1)),
    ("fraction", '{"x":{"dtype":"U8","shape":[1.0],"data_offsets":[0,1]}}', bytes(1)),
    ("no-tensors", '{"__metadata__":{"format":"pt"}}', b""),
    ("metadata-not-object", '{"__metadata__":[1],"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}',
     bytes(1)),
    ("not-object", '[1,2]', b""),
    ("bad-json", '{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}', bytes(1)),
    ("trailing-json", '{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}} x', bytes(1)),
    ("three-offsets", '{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1,2]}}', bytes(2)),
])
def test_mapped_safetensors_rejects_ambiguous_or_invalid_layouts(tmp_path, name, header, payload):
    p = str(tmp_path / f"{name}.safetensors")
    write_safetensors(p, header, payload)
    with pytest.raises(C.CheckpointError) as e:
        C.MappedSafetensors.open(p)
    assert e.value.status == PW_ERR_FORMAT, (name, str(e.value))


def test_safetensors_header_length_rules(tmp_path):
    # src/lib.rs:795-808: non-zero, a multiple of 8, inside the file; >= 16 bytes
    good = '{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}'
    p = str(tmp_path / "unpadded.safetensors")
    h = good.encode()
    assert len(h) % 8 != 0
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"\0")
    with pytest.raises(C.CheckpointError):
        C.MappedSafetensors.open(p)
    for label, blob in [("short", b"\0" * 10), ("zero", struct.pack("<Q", 0) + b" " * 16),
                        ("beyond", struct.pack("<Q", 4096) + b" " * 16)]:
        q = str(tmp_path / f"{label}.safetensors")
        with open(q, "wb") as f:
            f.write(blob)
        with pytest.raises(C.CheckpointError) as e:
            C.MappedSafetensors.open(q)
        assert e.value.status == PW_ERR_FORMAT
    with pytest.raises(C.CheckpointError) as e:
        C.MappedSafetensors.open(str(tmp_path / "absent.safetensors"))
    assert e.value.status == PW_ERR_IO


def test_json_strings_escapes_and_utf8(tmp_path):
    # a tensor name with escapes and multi-byte UTF-8 round-trips; invalid UTF-8 is rejected
    p = str(tmp_path / "names.safetensors")
    write_safetensors(p, '{"a\\u00e9\\ud83d\\ude00\\n\\"b":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},'
                         '"ü":{"dtype":"U8","shape":[1],"data_offsets":[1,2]}}', b"\x07\x08")
    with C.MappedSafetensors.open(p) as f:
        assert f.tensor("aé\U0001F600\n\"b").numpy().tolist() == [7]
        assert f.tensor("ü").numpy().tolist() == [8]
    q = str(tmp_path / "badutf8.safetensors")
    h = b'{"\xff":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}'
    while len(h) % 8:
        h += b" "
    with open(q, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"\0")
    with pytest.raises(C.CheckpointError):
        C.MappedSafetensors.open(q)


def test_reads_files_written_by_the_safetensors_library(tmp_path):
    # the checkpoint's own writer (safetensors.torch) with an F8_E4M3 weight,
    # its F32 _scale_inv grid and a BF16 vector
    torch = pytest.importorskip("torch")
    st = pytest.importorskip("safetensors.torch")
    w = (torch.randn(256, 128) * 0.02).to(torch.float8_e4m3fn)
    s = torch.rand(2, 1)
    n = torch.randn(128).to(torch.bfloat16)
    p = str(tmp_path / "model-00001-of-00002.safetensors")
    st.save_file({"model.layers.3.mlp.experts.0.gate_proj.weight": w,
                  "model.layers.3.mlp.experts.0.gate_proj.weight_scale_inv": s,
                  "model.layers.3.post_attention_layernorm.weight": n}, p)
    with C.MappedSafetensors.open(p) as f:
        tw = f.tensor("model.layers.3.mlp.experts.0.gate_proj.weight")
        assert tw.dtype == "F8_E4M3" and tw.shape == (256, 128)
        assert np.array_equal(tw.numpy(), w.view(torch.uint8).numpy())
        ts = f.tensor("model.layers.3.mlp.experts.0.gate_proj.weight_scale_inv")
        assert ts.dtype == "F32" and np.array_equal(ts.numpy(), s.numpy())
        tn = f.tensor("model.layers.3.post_attention_layernorm.weight")
        assert tn.dtype == "BF16" and np.array_equal(tn.numpy(), n.view(torch.int16).numpy().view(np.uint16))


def test_expert_container_round_trips_and_detects_tampering(tmp_path):
    source = str(tmp_path / "source.safetensors")
    output = str(tmp_path / "expert.pwexpert")
    header = json.dumps({"tensor.b": {"dtype": "U8", "shape": [3], "data_offsets": [4, 7]},
                         "tensor.a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}})
    write_safetensors(source, header, bytes([1, 2, 3, 4, 9, 8, 7]))
    packed = C.repack_expert_container(source, output, ["tensor.b", "tensor.a"])
    assert packed.names() == ["tensor.a", "tensor.b"]
    assert packed.tensor("tensor.a").numpy().tolist() == [1, 2, 3, 4]
    assert packed.tensor("tensor.b").numpy().tolist() == [9, 8, 7]
    packed.close()
    # the header records the source identity and every payload's SHA-256
    raw = open(output, "rb").read()
    assert raw[:8] == b"PWEXPRT1"
    hlen = struct.unpack("<Q", raw[8:16])[0]
    hdr = json.loads(raw[16:16 + hlen])
    assert hdr["schema_version"] == 1 and hdr["payload_alignment"] == 64
    assert hdr["source_file"] == "source.safetensors"
    assert hdr["source_sha256"] == hashlib.sha256(open(source, "rb").read()).hexdigest()
    assert hdr["tensors"][0]["sha256"] == hashlib.sha256(bytes([1, 2, 3, 4])).hexdigest()
    assert [t["payload_offset"] % 64 for t in hdr["tensors"]] == [0, 0]
    assert hdr["tensors"][1]["source_data_offsets"] == [4, 7]
    assert C.verify_expert_container(output).tensor_count() == 2
    # refuses to overwrite; no temporary file is left behind
    with pytest.raises(C.CheckpointError) as e:
        C.repack_expert_container(source, output, ["tensor.a"])
    assert "refusing to overwrite" in str(e.value)
    assert sorted(os.listdir(tmp_path)) == ["expert.pwexpert", "source.safetensors"]
    # tamper one payload byte
    payload_start = (16 + hlen + 63) // 64 * 64
    bad = bytearray(raw)
    bad[payload_start] ^= 0xFF
    tp = str(tmp_path / "tampered.pwexpert")
    open(tp, "wb").write(bytes(bad))
    with pytest.raises(C.CheckpointError) as e:
        C.verify_expert_container(tp)
    assert "hash mismatch" in str(e.value)
    # trailing bytes, unknown magic, truncation
    for label, blob in [("trailing", raw + b"\0"), ("magic", b"PWEXPRT2" + raw[8:]), ("truncated", raw[:-1])]:
        q = str(tmp_path / f"{label}.pwexpert")
        open(q, "wb").write(blob)
        with pytest.raises(C.CheckpointError) as e:
            C.verify_expert_container(q)
        assert e.value.status == PW_ERR_FORMAT, label


def test_repack_rejects_bad_requests(tmp_path):
    source = str(tmp_path / "s.safetensors")
    write_safetensors(source, '{"a":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', b"\x01")
    with pytest.raises(C.CheckpointError):
        C.repack_expert_container(source, str(tmp_path / "o1.pwexpert"), [])
    with pytest.raises(C.CheckpointError):
        C.repack_expert_container(source, str(tmp_path / "o2.pwexpert"), ["a", "a"])
    with pytest.raises(C.CheckpointError):
        C.repack_expert_container(source, str(tmp_path / "o3.pwexpert"), ["missing"])
    assert sorted(os.listdir(tmp_path)) == ["s.safetensors"]


def test_sha256_of_large_payload_matches_hashlib(tmp_path):
    # multi-block SHA-256 (payload not a multiple of 64 bytes)
    rng = np.random.default_rng(1)
    data = rng.integers(0, 256, 100003, dtype=np.uint8).tobytes()
    source = str(tmp_path / "big.safetensors")
    write_safetensors(source, json.dumps({"w": {"dtype": "U8", "shape": [len(data)],
                                                "data_offsets": [0, len(data)]}}), data)
    out = str(tmp_path / "big.pwexpert")
    C.repack_expert_container(source, out, ["w"]).close()
    raw = open(out, "rb").read()
    hlen = struct.unpack("<Q", raw[8:16])[0]
    assert json.loads(raw[16:16 + hlen])["tensors"][0]["sha256"] == hashlib.sha256(data).hexdigest()
