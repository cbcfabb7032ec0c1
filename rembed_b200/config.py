"""Model manifest: the host-side mirror of rembed's ``model.Config``.

Field names and JSON keys follow ``internal/model/config.go:15-78`` so a
``manifest.json`` written for the reference loads unchanged.  ``validate``
restates ``config.go:112-232`` rule for rule with the same error wording,
and ``position_offset`` / ``max_seq_len`` restate ``config.go:84-95``.
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from pathlib import Path

__all__ = ["Config", "ConfigError", "ARCH_IDS", "POOL_IDS"]

# Numeric ids used across the C ABI (include/rembed_gpu.h: RG_ARCH_*).
ARCH_IDS = {
    "": 0, "bert": 0, "distilbert": 1, "roberta": 2, "mpnet": 3,
    "modernbert": 4, "qwen3": 5, "gemma3": 6, "nomic_bert": 7,
}
# RG_POOL_*: mean, cls, lasttoken (bert.go:670-679).
POOL_IDS = {"mean": 0, "cls": 1, "lasttoken": 2}


class ConfigError(ValueError):
    """A manifest that the reference's validate() would refuse."""


@dataclass
class Config:
    name: str = ""
    model_type: str = ""
    hidden_size: int = 0
    num_hidden_layers: int = 0
    num_attention_heads: int = 0
    intermediate_size: int = 0
    vocab_size: int = 0
    max_position_embeddings: int = 0
    layer_norm_eps: float = 0.0
    do_lower_case: bool = False
    cls_token: str = ""
    sep_token: str = ""
    unk_token: str = ""
    pooling: str = "mean"
    normalize: bool = True
    tokenizer: str = ""
    # MPNet
    relative_attention_num_buckets: int = 0
    pad_token_id: int = 0
    # ModernBERT
    global_attn_every_n_layers: int = 0
    local_attention: int = 0
    global_rope_theta: float = 0.0
    local_rope_theta: float = 0.0
    # Qwen3 / Gemma3 / nomic
    head_dim: int = 0
    num_key_value_heads: int = 0
    rope_theta: float = 0.0
    # Gemma3
    sliding_window: int = 0
    sliding_window_pattern: int = 0
    query_pre_attn_scalar: int = 0
    dense_hidden: int = 0
    # Token-type table rows (not in the reference manifest: the reference
    # reads the table's first dimension from the checkpoint, bert.go:507-515).
    type_vocab_size: int = field(default=2, metadata={"manifest": False})

    # -- config.go:84-95 ------------------------------------------------
    def position_offset(self) -> int:
        """Row offset of position 0 in the position table (config.go:84-89)."""
        if self.model_type in ("mpnet", "roberta"):
            return self.pad_token_id + 1
        return 0

    def max_seq_len(self) -> int:
        """Longest encodable sequence (config.go:93-95)."""
        return self.max_position_embeddings - self.position_offset()

    # -- config.go:112-232 ----------------------------------------------
    def validate(self, source: str = "config") -> "Config":
        c = self
        if (c.hidden_size <= 0 or c.num_hidden_layers <= 0 or c.num_attention_heads <= 0
                or c.intermediate_size <= 0 or c.vocab_size <= 0 or c.max_position_embeddings <= 0):
            raise ConfigError(f"{source}: missing or non-positive architecture fields: {c}")
        if c.hidden_size % c.num_attention_heads != 0:
            raise ConfigError(f"{source}: hidden_size {c.hidden_size} not divisible by "
                              f"num_attention_heads {c.num_attention_heads}")
        if c.pooling not in ("mean", "cls", "lasttoken"):
            raise ConfigError(f"{source}: pooling {c.pooling!r} unsupported (mean, cls, or lasttoken)")
        if c.tokenizer not in ("", "sentencepiece", "gemma"):
            raise ConfigError(f'{source}: tokenizer {c.tokenizer!r} unsupported ("", sentencepiece, or gemma)')
        mt = c.model_type
        if mt in ("", "bert", "distilbert"):
            pass
        elif mt == "modernbert":
            if c.global_attn_every_n_layers < 1:
                raise ConfigError(f"{source}: modernbert requires global_attn_every_n_layers >= 1 "
                                  f"(found {c.global_attn_every_n_layers})")
            if c.local_attention < 2 or c.local_attention % 2 != 0:
                raise ConfigError(f"{source}: modernbert requires an even local_attention >= 2 "
                                  f"(found {c.local_attention})")
            if c.global_rope_theta <= 0 or c.local_rope_theta <= 0:
                raise ConfigError(f"{source}: modernbert requires positive global_rope_theta and "
                                  f"local_rope_theta (found {c.global_rope_theta:g} and {c.local_rope_theta:g})")
            dh = c.hidden_size // c.num_attention_heads
            if dh % 2 != 0:
                raise ConfigError(f"{source}: modernbert head_dim {dh} must be even for RoPE")
        elif mt == "qwen3":
            if c.head_dim <= 0 or c.head_dim % 2 != 0:
                raise ConfigError(f"{source}: qwen3 requires an even head_dim > 0 (found {c.head_dim})")
            if c.num_key_value_heads <= 0 or c.num_attention_heads % c.num_key_value_heads != 0:
                raise ConfigError(f"{source}: qwen3 requires num_attention_heads ({c.num_attention_heads}) "
                                  f"divisible by num_key_value_heads ({c.num_key_value_heads})")
            if c.rope_theta <= 0:
                raise ConfigError(f"{source}: qwen3 requires a positive rope_theta (found {c.rope_theta:g})")
        elif mt == "nomic_bert":
            if c.head_dim <= 0 or c.head_dim % 2 != 0:
                raise ConfigError(f"{source}: nomic_bert requires an even head_dim > 0 (found {c.head_dim})")
            if c.head_dim * c.num_attention_heads != c.hidden_size:
                raise ConfigError(f"{source}: nomic_bert head_dim*heads ({c.head_dim}*{c.num_attention_heads}) "
                                  f"must equal hidden_size {c.hidden_size}")
            if c.rope_theta <= 0:
                raise ConfigError(f"{source}: nomic_bert requires a positive rope_theta (found {c.rope_theta:g})")
        elif mt == "gemma3":
            if c.head_dim <= 0 or c.head_dim % 2 != 0:
                raise ConfigError(f"{source}: gemma3 requires an even head_dim > 0 (found {c.head_dim})")
            if c.num_key_value_heads <= 0 or c.num_attention_heads % c.num_key_value_heads != 0:
                raise ConfigError(f"{source}: gemma3 requires num_attention_heads ({c.num_attention_heads}) "
                                  f"divisible by num_key_value_heads ({c.num_key_value_heads})")
            if c.sliding_window < 1 or c.sliding_window_pattern < 1:
                raise ConfigError(f"{source}: gemma3 requires positive sliding_window and sliding_window_pattern "
                                  f"(found {c.sliding_window} and {c.sliding_window_pattern})")
            if c.query_pre_attn_scalar < 1:
                raise ConfigError(f"{source}: gemma3 requires a positive query_pre_attn_scalar "
                                  f"(found {c.query_pre_attn_scalar})")
            if c.global_rope_theta <= 0 or c.local_rope_theta <= 0:
                raise ConfigError(f"{source}: gemma3 requires positive global_rope_theta and local_rope_theta "
                                  f"(found {c.global_rope_theta:g} and {c.local_rope_theta:g})")
            if c.dense_hidden < 1:
                raise ConfigError(f"{source}: gemma3 requires a positive dense_hidden (found {c.dense_hidden})")
        elif mt == "roberta":
            if c.pad_token_id < 1:
                raise ConfigError(f"{source}: roberta requires pad_token_id >= 1 (found {c.pad_token_id} — "
                                  f"a manifest without the field reads as 0)")
            if c.max_seq_len() <= 0:
                raise ConfigError(f"{source}: pad_token_id {c.pad_token_id} leaves no usable positions "
                                  f"(max_position_embeddings {c.max_position_embeddings})")
        elif mt == "mpnet":
            if c.relative_attention_num_buckets != 32:
                raise ConfigError(f"{source}: relative_attention_num_buckets={c.relative_attention_num_buckets} — "
                                  f"HF's MPNet hardcodes 32 regardless of config, so rembed only accepts 32")
            if c.pad_token_id != 1:
                raise ConfigError(f"{source}: pad_token_id={c.pad_token_id} — HF's MPNet embeddings hardcode "
                                  f"padding_idx=1 regardless of config, so rembed only accepts 1")
        else:
            raise ConfigError(f"{source}: model_type {mt!r} unsupported (bert, distilbert, modernbert, qwen3, "
                              f"gemma3, nomic_bert, roberta, or mpnet)")
        if c.layer_norm_eps == 0:
            c.layer_norm_eps = 1e-12
        return c

    # -- helpers ----------------------------------------------------------
    @property
    def arch_id(self) -> int:
        return ARCH_IDS[self.model_type]

    @property
    def pool_id(self) -> int:
        return POOL_IDS[self.pooling]

    @property
    def attn_head_dim(self) -> int:
        return self.head_dim if self.head_dim else self.hidden_size // self.num_attention_heads

    @classmethod
    def from_json(cls, raw: str | bytes, source: str = "manifest") -> "Config":
        data = json.loads(raw)
        known = {f.name for f in dataclasses.fields(cls)}
        c = cls(**{k: v for k, v in data.items() if k in known})
        return c.validate(source)

    @classmethod
    def load(cls, path: str | Path) -> "Config":
        """LoadConfig (config.go:98-108): read and validate a manifest.json."""
        p = Path(path)
        return cls.from_json(p.read_bytes(), str(p))

    def to_json(self) -> str:
        d = {f.name: getattr(self, f.name) for f in dataclasses.fields(self)
             if f.metadata.get("manifest", True)}
        return json.dumps(d, indent=1)
