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

__all__ = ["PRESETS", "preset", "make_weights", "make_batch", "batch_of_lengths", "write_model_dir", "read_safetensors"]


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
    # The other BERT-path encoders (bert.go:338-518), small dims.
    "tiny-distilbert": lambda: _variant("distilbert", "synthetic/tiny-distilbert"),
    "tiny-roberta": lambda: _variant("roberta", "synthetic/tiny-roberta", pad_token_id=1, max_pos=258),
    "tiny-mpnet": lambda: _variant("mpnet", "synthetic/tiny-mpnet", pad_token_id=1, max_pos=258,
                                   relative_attention_num_buckets=32),
    # all-mpnet-base-v2 architecture (12 layers, hidden 768, 12 x 64, FFN 3072, mean pool).
    "mpnet-base": lambda: _variant("mpnet", "synthetic/all-mpnet-base-v2", H=768, L=12, heads=12, I=3072,
                                   vocab=30527, pad_token_id=1, max_pos=514, relative_attention_num_buckets=32,
                                   eps=1e-5),
}


def _qwen3(name, H, L, nq, nkv, dh, I, vocab, max_pos):
    return Config(name=name, model_type="qwen3", hidden_size=H, num_hidden_layers=L, num_attention_heads=nq,
                  num_key_value_heads=nkv, head_dim=dh, intermediate_size=I, vocab_size=vocab,
                  max_position_embeddings=max_pos, layer_norm_eps=1e-6, rope_theta=1e6, pooling="lasttoken",
                  normalize=True)


def _modernbert(name, H, L, heads, I, vocab, max_pos, local_attention):
    return Config(name=name, model_type="modernbert", hidden_size=H, num_hidden_layers=L,
                  num_attention_heads=heads, intermediate_size=I, vocab_size=vocab,
                  max_position_embeddings=max_pos, layer_norm_eps=1e-5, global_attn_every_n_layers=3,
                  local_attention=local_attention, global_rope_theta=160000.0, local_rope_theta=10000.0,
                  pooling="mean", normalize=True)


def _gemma3(name, H, L, nq, nkv, dh, I, vocab, max_pos, window, pattern, dense):
    return Config(name=name, model_type="gemma3", hidden_size=H, num_hidden_layers=L, num_attention_heads=nq,
                  num_key_value_heads=nkv, head_dim=dh, intermediate_size=I, vocab_size=vocab,
                  max_position_embeddings=max_pos, layer_norm_eps=1e-6, sliding_window=window,
                  sliding_window_pattern=pattern, query_pre_attn_scalar=dh, global_rope_theta=1e6,
                  local_rope_theta=1e4, dense_hidden=dense, pooling="mean", normalize=True, tokenizer="gemma")


def _nomic(name, H, L, heads, I, vocab, max_pos):
    return Config(name=name, model_type="nomic_bert", hidden_size=H, num_hidden_layers=L,
                  num_attention_heads=heads, head_dim=H // heads, intermediate_size=I, vocab_size=vocab,
                  max_position_embeddings=max_pos, layer_norm_eps=1e-12, rope_theta=1000.0, pooling="mean",
                  normalize=True)


PRESETS.update({
    # Qwen3-Embedding-0.6B: causal decoder, 28 layers, hidden 1024, 16 q / 8 kv heads x 128,
    # SwiGLU 3072, RMSNorm 1e-6, RoPE 1e6, last-token pooling.
    "qwen3-0.6b": lambda: _qwen3("synthetic/Qwen3-Embedding-0.6B", 1024, 28, 16, 8, 128, 3072, 151669, 32768),
    "tiny-qwen3": lambda: _qwen3("synthetic/tiny-qwen3", 256, 2, 4, 2, 64, 512, 2048, 1024),
    # ModernBERT-base: 22 layers, hidden 768, 12 x 64, GeGLU 1152, global every 3rd layer
    # (RoPE 160000), local window 128 (RoPE 10000).
    "modernbert-base": lambda: _modernbert("synthetic/ModernBERT-base", 768, 22, 12, 1152, 50368, 8192, 128),
    "tiny-modernbert": lambda: _modernbert("synthetic/tiny-modernbert", 128, 4, 2, 256, 2048, 1024, 16),
    # EmbeddingGemma-300m: 24 layers, hidden 768, 3 q / 1 kv head x 256, GeGLU-tanh 1152,
    # alternating local (effective window 257) / global, Dense head 768->3072->768.
    "embeddinggemma-300m": lambda: _gemma3("synthetic/embeddinggemma-300m", 768, 24, 3, 1, 256, 1152, 262144,
                                           2048, 257, 2, 3072),
    "tiny-gemma3": lambda: _gemma3("synthetic/tiny-gemma3", 128, 4, 2, 1, 64, 256, 2048, 512, 9, 2, 256),
    # nomic-embed-text-v1.5: post-norm, RoPE 1000, SwiGLU fc11 * silu(fc12).
    "nomic-embed-v1.5": lambda: _nomic("synthetic/nomic-embed-text-v1.5", 768, 12, 12, 3072, 30528, 2048),
    "tiny-nomic": lambda: _nomic("synthetic/tiny-nomic", 128, 2, 2, 256, 2048, 512),
    # Full-width, reduced-depth variants of three benchmark architectures for
    # parity at the configurations' longest sequences, where a full-depth CPU
    # forward would take hours: every layer kind stays present (ModernBERT:
    # layer 0 global, 1-2 local; Gemma: layer 0 local, 1 global; Qwen3: two
    # causal layers).
    "modernbert-base-3l": lambda: _modernbert("synthetic/ModernBERT-base-3l", 768, 3, 12, 1152, 50368, 8192, 128),
    "qwen3-0.6b-2l": lambda: _qwen3("synthetic/Qwen3-Embedding-0.6B-2l", 1024, 2, 16, 8, 128, 3072, 151669, 32768),
    "embeddinggemma-300m-2l": lambda: _gemma3("synthetic/embeddinggemma-300m-2l", 768, 2, 3, 1, 256, 1152, 262144,
                                              2048, 257, 2, 3072),
})

# Families whose token ids are not framed by CLS/SEP in the synthetic batches.
UNFRAMED = {"qwen3", "modernbert", "gemma3"}


def _variant(model_type, name, H=128, L=2, heads=2, I=512, vocab=4096, max_pos=256, eps=1e-12, **kw):
    c = _bert(name, H, L, heads, I, "mean", vocab=vocab, max_pos=max_pos)
    c.model_type = model_type
    c.layer_norm_eps = eps
    if model_type == "roberta":
        c.type_vocab_size = 1
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def preset(name: str) -> Config:
    return PRESETS[name]().validate(name)


def _bert_shapes(cfg: Config) -> dict[str, tuple]:
    """HF tensor names of the BERT-path encoders (bert.go:381-470, 495-515)."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    mt = cfg.model_type
    pre = {"roberta": "roberta.", "mpnet": "mpnet.", "distilbert": "distilbert."}.get(mt, "")
    s: dict[str, tuple] = {
        pre + "embeddings.word_embeddings.weight": (cfg.vocab_size, H),
        pre + "embeddings.position_embeddings.weight": (cfg.max_position_embeddings, H),
        pre + "embeddings.LayerNorm.weight": (H,),
        pre + "embeddings.LayerNorm.bias": (H,),
    }
    if mt not in ("distilbert", "mpnet"):
        s[pre + "embeddings.token_type_embeddings.weight"] = (cfg.type_vocab_size, H)
    if mt == "mpnet":
        s[pre + "encoder.relative_attention_bias.weight"] = (cfg.relative_attention_num_buckets,
                                                             cfg.num_attention_heads)
    for i in range(cfg.num_hidden_layers):
        if mt == "distilbert":
            p = f"{pre}transformer.layer.{i}."
            attn = {"q_lin": "attention.q_lin", "k_lin": "attention.k_lin", "v_lin": "attention.v_lin",
                    "out": "attention.out_lin"}
            names = [(attn["q_lin"], (H, H)), (attn["k_lin"], (H, H)), (attn["v_lin"], (H, H)),
                     (attn["out"], (H, H)), ("ffn.lin1", (I, H)), ("ffn.lin2", (H, I))]
            norms = ["sa_layer_norm", "output_layer_norm"]
        else:
            p = f"{pre}encoder.layer.{i}."
            if mt == "mpnet":
                qkvo = ["attention.attn.q", "attention.attn.k", "attention.attn.v", "attention.attn.o"]
                norms = ["attention.LayerNorm", "output.LayerNorm"]
            else:
                qkvo = ["attention.self.query", "attention.self.key", "attention.self.value",
                        "attention.output.dense"]
                norms = ["attention.output.LayerNorm", "output.LayerNorm"]
            names = [(qkvo[0], (H, H)), (qkvo[1], (H, H)), (qkvo[2], (H, H)), (qkvo[3], (H, H)),
                     ("intermediate.dense", (I, H)), ("output.dense", (H, I))]
        for nm, shp in names:
            s[p + nm + ".weight"] = shp
            s[p + nm + ".bias"] = (shp[0],)
        for nm in norms:
            s[p + nm + ".weight"] = (H,)
            s[p + nm + ".bias"] = (H,)
    return s


def _decoder_shapes(cfg: Config) -> dict[str, tuple]:
    """HF tensor names of the Qwen3 / Gemma3 / ModernBERT / nomic loaders
    (qwen3.go:87-110, gemma3.go:103-170, modernbert.go:55-103, nomic.go:36-110)."""
    H, I, mt = cfg.hidden_size, cfg.intermediate_size, cfg.model_type
    dh = cfg.attn_head_dim
    nq, nkv = cfg.num_attention_heads, (cfg.num_key_value_heads or cfg.num_attention_heads)
    s: dict[str, tuple] = {}
    if mt in ("qwen3", "gemma3"):
        s["embed_tokens.weight"] = (cfg.vocab_size, H)
        s["norm.weight"] = (H,)
        for i in range(cfg.num_hidden_layers):
            p = f"layers.{i}."
            s[p + "input_layernorm.weight"] = (H,)
            s[p + "post_attention_layernorm.weight"] = (H,)
            if mt == "gemma3":
                s[p + "pre_feedforward_layernorm.weight"] = (H,)
                s[p + "post_feedforward_layernorm.weight"] = (H,)
            s[p + "self_attn.q_proj.weight"] = (nq * dh, H)
            s[p + "self_attn.k_proj.weight"] = (nkv * dh, H)
            s[p + "self_attn.v_proj.weight"] = (nkv * dh, H)
            s[p + "self_attn.o_proj.weight"] = (H, nq * dh)
            s[p + "self_attn.q_norm.weight"] = (dh,)
            s[p + "self_attn.k_norm.weight"] = (dh,)
            s[p + "mlp.gate_proj.weight"] = (I, H)
            s[p + "mlp.up_proj.weight"] = (I, H)
            s[p + "mlp.down_proj.weight"] = (H, I)
        if mt == "gemma3":
            s["2_Dense.linear.weight"] = (cfg.dense_hidden, H)
            s["3_Dense.linear.weight"] = (H, cfg.dense_hidden)
    elif mt == "modernbert":
        s["embeddings.tok_embeddings.weight"] = (cfg.vocab_size, H)
        s["embeddings.norm.weight"] = (H,)
        s["final_norm.weight"] = (H,)
        for i in range(cfg.num_hidden_layers):
            p = f"layers.{i}."
            if i != 0:
                s[p + "attn_norm.weight"] = (H,)
            s[p + "attn.Wqkv.weight"] = (3 * H, H)
            s[p + "attn.Wo.weight"] = (H, H)
            s[p + "mlp_norm.weight"] = (H,)
            s[p + "mlp.Wi.weight"] = (2 * I, H)
            s[p + "mlp.Wo.weight"] = (H, I)
    else:  # nomic_bert
        s["embeddings.word_embeddings.weight"] = (cfg.vocab_size, H)
        s["embeddings.token_type_embeddings.weight"] = (2, H)
        s["emb_ln.weight"] = (H,)
        s["emb_ln.bias"] = (H,)
        for i in range(cfg.num_hidden_layers):
            p = f"encoder.layers.{i}."
            s[p + "attn.Wqkv.weight"] = (3 * H, H)
            s[p + "attn.out_proj.weight"] = (H, H)
            s[p + "mlp.fc11.weight"] = (I, H)
            s[p + "mlp.fc12.weight"] = (I, H)
            s[p + "mlp.fc2.weight"] = (H, I)
            for n in ("norm1", "norm2"):
                s[p + n + ".weight"] = (H,)
                s[p + n + ".bias"] = (H,)
    return s


def tensor_shapes(cfg: Config) -> dict[str, tuple]:
    if cfg.model_type in ("", "bert", "distilbert", "roberta", "mpnet"):
        return _bert_shapes(cfg)
    if cfg.model_type in ("qwen3", "gemma3", "modernbert", "nomic_bert"):
        return _decoder_shapes(cfg)
    raise NotImplementedError(f"synthetic weights for model_type {cfg.model_type!r}")


def _is_gain(name: str) -> bool:
    return name.endswith(("LayerNorm.weight", "norm.weight", "_norm.weight", "layer_norm.weight", "layernorm.weight",
                          "emb_ln.weight", "norm1.weight", "norm2.weight"))


def make_weights(cfg: Config, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded float32 weights for cfg, keyed by Hugging Face tensor name."""
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for name, shape in tensor_shapes(cfg).items():
        w = rng.standard_normal(shape, dtype=np.float32)
        w *= np.float32(std)
        # Norm gains are 1 + N(0, std), except Gemma's, whose stored weights
        # are the offset from 1 (the loader adds it: gemma3.go:44-50).
        if _is_gain(name) and cfg.model_type != "gemma3":
            w += np.float32(1.0)
        if cfg.model_type == "qwen3":
            # bf16 checkpoint widened to float32 (safetensors.go:188-209)
            w = (w.view(np.uint32) + np.uint32(0x7FFF) + ((w.view(np.uint32) >> 16) & 1)) & np.uint32(0xFFFF0000)
            w = w.view(np.float32)
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
    if cfg.model_type in UNFRAMED:
        framed = False
        id_lo = 0 if id_lo == 1000 else id_lo
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


def batch_of_lengths(cfg: Config, lens, seed: int = 1, id_lo: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Packed batch with the given sequence lengths; ids uniform in
    [id_lo, vocab) (framed by CLS/SEP for the BERT family, as make_batch)."""
    framed = cfg.model_type not in UNFRAMED
    if framed and id_lo == 0:
        id_lo = 1000
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int64)
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    ids = rng.integers(id_lo, cfg.vocab_size, size=int(cu[-1]), dtype=np.int64)
    if framed:
        for i in range(len(lens)):
            ids[cu[i]] = 101
            if lens[i] > 1:
                ids[cu[i + 1] - 1] = 102
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
