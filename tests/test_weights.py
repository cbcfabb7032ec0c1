"""Weight ingest on CPU: sharded safetensors and the .rembedpack format
(internal/packfile/packfile_test.go's round trip and corrupt-header cases)."""

import json
import struct

import numpy as np
import pytest

from rembed_b200 import synth, weights as W


def test_pack_round_trip(tmp_path):
    src = {"a": np.arange(1, 7, dtype=np.float32).reshape(2, 3), "scale": np.array([0.5], np.float32),
           "big": (np.arange(1000, dtype=np.float32) * 0.25).reshape(10, 100), "empty": np.zeros((0,), np.float32)}
    path = W.write_pack(tmp_path / "w.rembedpack", src, source="src-fingerprint-v1")
    pk = W.read_pack(path)
    for name, a in src.items():
        got = pk.f32(name, *a.shape)
        assert got.shape == a.shape and np.array_equal(got, a)
    assert pk.source == "src-fingerprint-v1"
    with pytest.raises(W.WeightsError, match="missing tensor"):
        pk.f32("missing", 1)
    with pytest.raises(W.WeightsError, match="shape"):
        pk.f32("a", 3, 2)
    # the data section starts on a 64-byte boundary
    (hlen,) = struct.unpack("<Q", path.read_bytes()[:8])
    assert pk._data_off % 64 == 0 and pk._data_off >= 8 + hlen


def _write_raw(path, header: dict, data: bytes = b""):
    hb = json.dumps(header).encode()
    pad = ((8 + len(hb) + 63) & ~63) - 8 - len(hb)
    path.write_bytes(struct.pack("<Q", len(hb)) + hb + b"\0" * pad + data)


@pytest.mark.parametrize("header,match", [
    ({"rembedpack": 2, "tensors": []}, "version"),
    ({"rembedpack": 1, "tensors": [{"name": "x", "shape": [2], "off": 2, "nbytes": 8}]}, "aligned"),
    ({"rembedpack": 1, "tensors": [{"name": "x", "shape": [3], "off": 0, "nbytes": 8}]}, "length"),
    ({"rembedpack": 1, "tensors": [{"name": "x", "shape": [4], "off": 0, "nbytes": 16}]}, "out of data section"),
])
def test_pack_rejects_corrupt_header(tmp_path, header, match):
    p = tmp_path / "bad.rembedpack"
    _write_raw(p, header, b"\0" * 8)
    with pytest.raises(W.WeightsError, match=match):
        W.read_pack(p)
    (tmp_path / "short").write_bytes(b"\1\2")
    with pytest.raises(W.WeightsError, match="too short"):
        W.read_pack(tmp_path / "short")


def test_sharded_checkpoint_and_disk_pack(tmp_path):
    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=3)
    names = sorted(w)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    for f, ns in shards.items():
        synth.write_safetensors(tmp_path / f, {n: w[n] for n in ns})
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {n: f for f, ns in shards.items() for n in ns}}))
    got = W.read_checkpoint(tmp_path)
    assert set(got) == set(w) and all(np.array_equal(got[n], w[n]) for n in w)
    # WithDiskWeights: packed on first use, reused while the fingerprint holds
    mapped = W.disk_weights(tmp_path)
    pack = tmp_path / W.PACK_NAME
    assert pack.exists() and all(np.array_equal(mapped[n], w[n]) for n in w)
    before = pack.stat().st_mtime_ns
    W.disk_weights(tmp_path)
    assert pack.stat().st_mtime_ns == before
    assert W.read_pack(pack).source == W.source_fingerprint(tmp_path)


def test_unsafe_shard_name_rejected(tmp_path):
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"a": "../evil.safetensors"}}))
    with pytest.raises(W.WeightsError, match="unsafe shard name"):
        W.read_checkpoint(tmp_path)
    assert not W.valid_shard_name("..") and not W.valid_shard_name("a\\b") and W.valid_shard_name("x.safetensors")
