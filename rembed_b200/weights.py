"""Weight ingest: the checkpoint formats the reference host parses, read into
numpy arrays that `Embedder` hands to `rg_upload_weight`.

* ``read_checkpoint(dir)``: ``model.safetensors``, or the sharded set named
  by ``model.safetensors.index.json`` when the single file is absent
  (internal/safetensors/reader.go:31-70); F32 / F16 / BF16 widened to fp32
  (safetensors.go:188-209).
* ``write_pack`` / ``read_pack``: the ``.rembedpack`` file of
  internal/packfile/packfile.go — an 8-byte little-endian header length, a
  JSON header ``{"rembedpack": 1, "source": ..., "tensors": [{name, shape,
  off, nbytes}]}``, then fp32 data starting at the next 64-byte boundary.
  ``read_pack`` maps the file (``np.memmap``: zero copy, pages in on access)
  and validates every entry before handing out arrays, as ``packfile.Open``
  does.
* ``source_fingerprint(dir)``: the staleness fingerprint the reference
  records in a pack (qwen3.go:200-240).
"""

from __future__ import annotations

import json
import os
import struct
from pathlib import Path

import numpy as np

from .synth import read_safetensors

PACK_VERSION = 1
PACK_NAME = "weights.rembedpack"


class WeightsError(ValueError):
    """A checkpoint or pack file that cannot be read."""


def valid_shard_name(name: str) -> bool:
    """A shard named by the index must be a plain file name
    (safetensors.go:47-52)."""
    return name not in ("", ".", "..") and "/" not in name and "\\" not in name


def _shard_files(model_dir: Path) -> list[Path]:
    idx = model_dir / "model.safetensors.index.json"
    try:
        index = json.loads(idx.read_text())
    except FileNotFoundError:
        raise WeightsError(f"safetensors: {model_dir / 'model.safetensors'} not found (and no index beside it)")
    except ValueError as e:
        raise WeightsError(f"safetensors {idx}: bad index JSON: {e}")
    names = set()
    for f in index.get("weight_map", {}).values():
        if not valid_shard_name(f):
            raise WeightsError(f"safetensors {idx}: unsafe shard name {f!r} in index")
        names.add(f)
    return [model_dir / f for f in sorted(names)]


def read_checkpoint(model_dir: str | os.PathLike) -> dict[str, np.ndarray]:
    """All tensors of a model directory's single-file or sharded checkpoint."""
    d = Path(model_dir)
    single = d / "model.safetensors"
    if single.exists():
        return read_safetensors(single)
    out: dict[str, np.ndarray] = {}
    for f in _shard_files(d):
        for name, arr in read_safetensors(f).items():
            if name in out:
                raise WeightsError(f"safetensors {f}: tensor {name} appears in two shards")
            out[name] = arr
    return out


def source_fingerprint(model_dir: str | os.PathLike) -> str:
    """``name:size:mtime_ns`` of each checkpoint file, sorted by path: what a
    pack records so a re-downloaded checkpoint is not served from a stale pack."""
    d = Path(model_dir)
    single = d / "model.safetensors"
    files = [single] if single.exists() else [d / "model.safetensors.index.json", *_shard_files(d)]
    lines = []
    for f in sorted(files):
        st = f.stat()
        lines.append(f"{f.name}:{st.st_size}:{st.st_mtime_ns}\n")
    return "".join(lines)


def _data_start(header_len: int) -> int:
    return (8 + header_len + 63) & ~63


def write_pack(path: str | os.PathLike, tensors: dict[str, np.ndarray], source: str = "") -> Path:
    """Write tensors (widened to fp32) as a pack file, atomically (temp + rename)."""
    p = Path(path)
    entries, off = [], 0
    for name, a in tensors.items():
        nb = int(np.prod(a.shape, dtype=np.int64)) * 4
        entries.append({"name": name, "shape": [int(x) for x in a.shape], "off": off, "nbytes": nb})
        off += nb
    head = {"rembedpack": PACK_VERSION, "tensors": entries}
    if source:
        head["source"] = source
    hb = json.dumps(head, separators=(",", ":")).encode()
    tmp = p.with_name(f".{p.name}.{os.getpid()}.tmp")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        f.write(b"\0" * (_data_start(len(hb)) - 8 - len(hb)))
        for name, a in tensors.items():
            f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())
    os.replace(tmp, p)
    return p


class Pack:
    """A mapped pack file: ``source``, ``shape(name)``, ``f32(name, *shape)``."""

    def __init__(self, path: str | os.PathLike):
        p = Path(path)
        size = p.stat().st_size
        if size < 8:
            raise WeightsError(f"packfile {p}: too short")
        with open(p, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            if hlen > size - 8:
                raise WeightsError(f"packfile {p}: header length {hlen} exceeds file")
            try:
                head = json.loads(f.read(hlen))
            except ValueError as e:
                raise WeightsError(f"packfile {p}: bad header: {e}")
        if head.get("rembedpack") != PACK_VERSION:
            raise WeightsError(f"packfile {p}: version {head.get('rembedpack')}, want {PACK_VERSION}")
        self.path, self.source = p, head.get("source", "")
        self._data_off = _data_start(hlen)
        data_len = size - self._data_off
        self._entries = {}
        for e in head.get("tensors", []):
            name, shape, off, nb = e["name"], list(e["shape"]), int(e["off"]), int(e["nbytes"])
            if off % 4 or nb % 4:
                raise WeightsError(f"packfile {p}: tensor {name!r} offset/length not 4-byte aligned")
            if nb != int(np.prod(shape, dtype=np.int64)) * 4:
                raise WeightsError(f"packfile {p}: tensor {name!r} length {nb} != shape {shape}")
            if off < 0 or nb < 0 or off + nb > data_len:
                raise WeightsError(f"packfile {p}: tensor {name!r} range [{off},{off + nb}) out of data section "
                                   f"{data_len}")
            self._entries[name] = (shape, off, nb)
        self._map = np.memmap(p, dtype=np.uint8, mode="r") if size > 0 else None

    def names(self) -> list[str]:
        return list(self._entries)

    def shape(self, name: str):
        e = self._entries.get(name)
        return None if e is None else list(e[0])

    def f32(self, name: str, *want_shape: int) -> np.ndarray:
        e = self._entries.get(name)
        if e is None:
            raise WeightsError(f"packfile: missing tensor {name!r}")
        shape, off, nb = e
        if want_shape and list(want_shape) != shape:
            raise WeightsError(f"packfile: tensor {name!r} shape {shape}, want {list(want_shape)}")
        start = self._data_off + off
        return self._map[start:start + nb].view("<f4").reshape(shape)

    def tensors(self) -> dict[str, np.ndarray]:
        return {n: self.f32(n) for n in self._entries}


def read_pack(path: str | os.PathLike) -> Pack:
    return Pack(path)


def disk_weights(model_dir: str | os.PathLike) -> dict[str, np.ndarray]:
    """WithDiskWeights (rembed.go:82-92, qwen3.go:247-280): the model's
    weights mapped from ``<dir>/weights.rembedpack``, which is (re)built from
    the checkpoint when it is missing or its recorded source fingerprint no
    longer matches."""
    d = Path(model_dir)
    pack_path = d / PACK_NAME
    fp = source_fingerprint(d)
    if pack_path.exists():
        try:
            pk = Pack(pack_path)
            if pk.source == fp:
                return pk.tensors()
        except WeightsError:
            pass  # unreadable or old: rebuild below
    write_pack(pack_path, read_checkpoint(d), source=fp)
    return Pack(pack_path).tensors()
