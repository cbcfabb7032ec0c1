"""Seeded synthetic models and token batches for the benchmark configs.

There are no real checkpoints or datasets on the benchmark hosts, so every
parity test and benchmark runs on random-init weights of the named
architecture and on seeded token-id batches with the configured length
distribution.  One generator serves the CUDA path and the CPU oracle alike,
so both always see identical inputs.

Initialisation: every matrix, embedding table and bias is N(0, 0.02);
LayerNorm/RMSNorm gains are 1 + N(0, 0.02) and LayerNorm biases
N(0, 0.02).  Tensor names are the Hugging Face names the reference loader
reads (internal/model/bert.go:381-470).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from .config import Config

__all__ = ["PRESETS", "preset", "make_weights", "make_batch", "write_model_dir", "read_safetensors"]


def _bert(name, H, L, heads, I, pooling, vocab=30522, max_pos=512):
    return Config(name=name, model_type="bert", hidden_size=H, num_hidden_layers=L,
                  num_attention_heads=heads, intermediate_size=I, vocab_size=vocab,
                  max_position_embeddings=max_pos, layer_norm_eps=1e-12, pooling=pooling,
                  normalize=True, cls_token="[CLS]", sep_token="[SEP]", unk_token="[UNK]")


# Architectures of the benchmark configurations (BERT family first).
PRESETS = {
    # MiniLM-L6-v2: 6 layers, hidden 384, 12 heads x 32, FFN 1536, mean pool.
    "minilm-l6": lambda: _bert("synthetic/all-MiniLM-L6-v2", 384, 6, 12, 1536, "mean"),
    # bge-base-en-v1.5 (BERT-base): 12 layers, hidden 768, 12 x 64, FFN 3072, CLS pool.
    "bge-base": lambda: _bert("synthetic/bge-base-en-v1.5", 768, 12, 12, 3072, "cls"),
    # A tiny BERT for fast unit tests (same code path, small dims).
    "tiny-bert": lambda: _bert("synthetic/tiny-bert", 128, 2, 2, 512, "mean", vocab=4096, max_pos=256),
}


def preset(name: str) -> Config:
    return PRESETS[name]().validate(name)


def _bert_shapes(cfg: Config) -> dict[str, tuple]:
    H, I = cfg.hidden_size, cfg.intermediate_size
    s: dict[str, tuple] = {
        "embeddings.word_embeddings.weight": (cfg.vocab_size, H),
        "embeddings.position_embeddings.weight": (cfg.max_position_embeddings, H),
        "embeddings.token_type_embeddings.weight": (cfg.type_vocab_size, H),
        "embeddings.LayerNorm.weight": (H,),
        "embeddings.LayerNorm.bias": (H,),
    }
    for i in range(cfg.num_hidden_layers):
        p = f"encoder.layer.{i}."
        for nm in ("query", "key", "value"):
            s[p + f"attention.self.{nm}.weight"] = (H, H)
            s[p + f"attention.self.{nm}.bias"] = (H,)
        s[p + "attention.output.dense.weight"] = (H, H)
        s[p + "attention.output.dense.bias"] = (H,)
        s[p + "attention.output.LayerNorm.weight"] = (H,)
        s[p + "attention.output.LayerNorm.bias"] = (H,)
        s[p + "intermediate.dense.weight"] = (I, H)
        s[p + "intermediate.dense.bias"] = (I,)
        s[p + "output.dense.weight"] = (H, I)
        s[p + "output.dense.bias"] = (H,)
        s[p + "output.LayerNorm.weight"] = (H,)
        s[p + "output.LayerNorm.bias"] = (H,)
    return s


def tensor_shapes(cfg: Config) -> dict[str, tuple]:
    if cfg.model_type in ("", "bert"):
        return _bert_shapes(cfg)
    raise NotImplementedError(f"synthetic weights for model_type {cfg.model_type!r}")


def make_weights(cfg: Config, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded float32 weights for cfg, keyed by Hugging Face tensor name."""
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for name, shape in tensor_shapes(cfg).items():
        w = rng.standard_normal(shape, dtype=np.float32)
        w *= np.float32(std)
        if name.endswith("LayerNorm.weight") or name.endswith("norm.weight") or name.endswith("_norm.weight"):
            w += np.float32(1.0)
        out[name] = np.ascontiguousarray(w)
    return out


def make_batch(cfg: Config, nseq: int, lo: int, hi: int, seed: int = 1,
               framed: bool = True, id_lo: int = 1000, id_hi: int | None = None,
               cls_id: int = 101, sep_id: int = 102) -> tuple[np.ndarray, np.ndarray]:
    """Packed token-id batch: (ids int64 [T], cu_seqlens int32 [nseq+1]).

    Lengths are uniform integers in [lo, hi]; with ``framed`` each sequence
    is CLS + ids uniform in [id_lo, id_hi] + SEP, the layout a WordPiece
    tokenizer produces for BERT-family models.
    """
    rng = np.random.default_rng(seed)
    hi = min(hi, cfg.max_seq_len())
    lens = rng.integers(lo, hi + 1, size=nseq) if hi > lo else np.full(nseq, lo)
    id_hi = cfg.vocab_size - 1 if id_hi is None else id_hi
    cu = np.zeros(nseq + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    ids = rng.integers(id_lo, id_hi + 1, size=int(cu[-1]), dtype=np.int64)
    if framed:
        for i in range(nseq):
            ids[cu[i]] = cls_id
            if lens[i] > 1:
                ids[cu[i + 1] - 1] = sep_id
    return ids, cu


# -- minimal safetensors I/O (for manifest directories) --------------------
_DT = {"F32": np.float32, "F16": np.float16, "BF16": None}


def write_safetensors(path: str | Path, tensors: dict[str, np.ndarray]) -> None:
    header, offset, blobs = {}, 0, []
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, dtype=np.float32)
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [offset, offset + a.nbytes]}
        blobs.append(a.tobytes())
        offset += a.nbytes
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str | Path) -> dict[str, np.ndarray]:
    """Read F32/F16/BF16 tensors, widening to float32 (safetensors.go:188-209)."""
    raw = Path(path).read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    base = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        lo, hi = meta["data_offsets"]
        buf = raw[base + lo: base + hi]
        dt = meta["dtype"]
        if dt == "F32":
            a = np.frombuffer(buf, dtype=np.float32)
        elif dt == "F16":
            a = np.frombuffer(buf, dtype=np.float16).astype(np.float32)
        elif dt == "BF16":
            a = (np.frombuffer(buf, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {dt}")
        out[name] = a.reshape(meta["shape"]).copy()
    return out


def write_model_dir(path: str | Path, cfg: Config, weights: dict[str, np.ndarray]) -> Path:
    """A converted model directory: manifest.json + model.safetensors."""
    p = Path(path)
    p.mkdir(parents=True, exist_ok=True)
    (p / "manifest.json").write_text(cfg.to_json())
    write_safetensors(p / "model.safetensors", weights)
    return p
