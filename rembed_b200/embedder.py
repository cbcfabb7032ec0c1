"""Host-side mirror of rembed's public API over librembed_gpu.so.

Names and meaning follow the reference (rembed.go and its Python binding
python/rembed/__init__.py):

* ``load(ref, int8=..., int8_activations=..., dim=..., disk_weights=...)``
  = ``rembed.Load`` with ``WithInt8`` / ``WithInt8Activations`` /
  ``WithDim`` / ``WithDiskWeights`` (rembed.go:60-121, 139-270), over a
  converted model directory (manifest.json + model.safetensors or a sharded
  set, or the weights.rembedpack file; see weights.py); ``fp16=False``
  selects bf16 tensor-core operands and ``strict_fp32=True`` the strict
  fp32 path;
* ``Embedder.embed`` = ``Embed`` (rembed.go:287-332): one L2-normalised
  vector per sequence, truncated to ``dim`` and re-normalised;
* ``Embedder.embed_tokens`` = ``EmbedTokens`` (rembed.go:370-411);
* ``quantized()`` / ``quantized_activations()`` = the reference's mode
  probes (rembed.go:424-432); ``dim`` / ``model`` / ``close``.

Inputs are token ids (tokenisation stays on the CPU, in the caller).  The
whole batch goes to the GPU in one ``rg_forward`` call.  There is no CPU
fallback: if the CUDA library is missing or refuses the model, this module
raises.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable, Sequence

import numpy as np

from .config import Config

__all__ = ["Embedder", "Pending", "RembedError", "TokenEmbeddings", "load", "library"]

RG_MODE_BF16, RG_MODE_F16, RG_MODE_INT8_W, RG_MODE_INT8_FULL, RG_MODE_FP32 = 0, 1, 2, 3, 4
RG_DTYPE_F32, RG_DTYPE_F16, RG_DTYPE_BF16 = 0, 1, 2
RG_OUT_POOLED, RG_OUT_TOKENS = 0, 1

_PKG = Path(__file__).resolve().parent


class RembedError(RuntimeError):
    """An error reported by the rembed GPU engine."""


class _Desc(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_int),
        ("hidden_size", ctypes.c_int), ("num_hidden_layers", ctypes.c_int),
        ("num_attention_heads", ctypes.c_int), ("intermediate_size", ctypes.c_int),
        ("vocab_size", ctypes.c_int), ("max_position_embeddings", ctypes.c_int),
        ("layer_norm_eps", ctypes.c_float),
        ("pooling", ctypes.c_int), ("normalize", ctypes.c_int),
        ("pad_token_id", ctypes.c_int), ("relative_attention_num_buckets", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("num_key_value_heads", ctypes.c_int),
        ("rope_theta", ctypes.c_double), ("global_rope_theta", ctypes.c_double),
        ("local_rope_theta", ctypes.c_double),
        ("global_attn_every_n_layers", ctypes.c_int), ("local_attention", ctypes.c_int),
        ("sliding_window", ctypes.c_int), ("sliding_window_pattern", ctypes.c_int),
        ("query_pre_attn_scalar", ctypes.c_int), ("dense_hidden", ctypes.c_int),
    ]


def desc_from_config(cfg: Config) -> _Desc:
    d = _Desc()
    d.arch = cfg.arch_id
    d.hidden_size, d.num_hidden_layers = cfg.hidden_size, cfg.num_hidden_layers
    d.num_attention_heads, d.intermediate_size = cfg.num_attention_heads, cfg.intermediate_size
    d.vocab_size, d.max_position_embeddings = cfg.vocab_size, cfg.max_position_embeddings
    d.layer_norm_eps = cfg.layer_norm_eps
    d.pooling, d.normalize = cfg.pool_id, int(bool(cfg.normalize))
    d.pad_token_id, d.relative_attention_num_buckets = cfg.pad_token_id, cfg.relative_attention_num_buckets
    d.head_dim, d.num_key_value_heads = cfg.head_dim, cfg.num_key_value_heads
    d.rope_theta, d.global_rope_theta, d.local_rope_theta = cfg.rope_theta, cfg.global_rope_theta, cfg.local_rope_theta
    d.global_attn_every_n_layers, d.local_attention = cfg.global_attn_every_n_layers, cfg.local_attention
    d.sliding_window, d.sliding_window_pattern = cfg.sliding_window, cfg.sliding_window_pattern
    d.query_pre_attn_scalar, d.dense_hidden = cfg.query_pre_attn_scalar, cfg.dense_hidden
    return d


# The exported C ABI (include/rembed_gpu.h), name -> (restype, argtypes).
_VP, _CP = ctypes.c_void_p, ctypes.c_char_p
_ERR = ctypes.POINTER(ctypes.c_char_p)
SIGNATURES = {
    "rg_init": (ctypes.c_int, [ctypes.POINTER(_Desc), ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int,
                               ctypes.POINTER(_VP), _ERR]),
    "rg_upload_weight": (ctypes.c_int, [_VP, _CP, ctypes.c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_int,
                                        _VP, _ERR]),
    "rg_finalize": (ctypes.c_int, [_VP, _ERR]),
    "rg_forward": (ctypes.c_int, [_VP, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float), _ERR]),
    "rg_submit": (ctypes.c_int, [_VP, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
                                 ctypes.POINTER(ctypes.c_int64), _ERR]),
    "rg_collect": (ctypes.c_int, [_VP, ctypes.c_int64, _ERR]),
    "rg_forward_device": (ctypes.c_int, [_VP, ctypes.c_int, _VP, _VP, ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, _VP, _VP, _ERR]),
    "rg_sync": (ctypes.c_int, [_VP, ctypes.c_int, _ERR]),
    "rg_hidden": (ctypes.c_int, [_VP]),
    "rg_mode_active": (ctypes.c_int, [_VP]),
    "rg_last_launches": (ctypes.c_int, [_VP, ctypes.c_int]),
    "rg_profile": (ctypes.c_int, [_VP, ctypes.c_int, ctypes.c_int]),
    "rg_profile_stats": (ctypes.c_int, [_VP, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_double)]),
    "rg_free": (None, [_VP]),
    "rg_free_string": (None, [ctypes.c_void_p]),
    "rg_dense_bf16": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, _VP, _ERR]),
    "rg_dense_residual_layernorm_bf16": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_float, _VP, _VP,
                                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP, _ERR]),
    "rg_dense_residual_layernorm_bf16_noalloc": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_float, _VP,
                                                                _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP,
                                                                _ERR]),
    "rg_kernel_status": (ctypes.c_int, [_VP, _ERR]),
    "rg_test_inject": (ctypes.c_int, [_VP, ctypes.c_int, ctypes.c_longlong, _ERR]),
    "rg_attention": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP,
                                    ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP,
                                    ctypes.c_int, _VP, _ERR]),
    "rg_quantize_rows_s8": (ctypes.c_int, [_VP, ctypes.c_int, ctypes.c_int, _VP, _VP, _VP, _ERR]),
    "rg_dense_s8": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP,
                                   _ERR]),
}

_lib = None


def library_path() -> Path:
    env = os.environ.get("REMBED_GPU_LIB")
    if env:
        p = Path(env)
        if not p.is_file():
            raise RembedError(f"REMBED_GPU_LIB={env} does not exist")
        return p
    p = _PKG / "librembed_gpu.so"
    if not p.is_file():
        raise RembedError("librembed_gpu.so not found: build it with `python -m rembed_b200.build`")
    return p


def library() -> ctypes.CDLL:
    """Load librembed_gpu.so and bind every exported entry point."""
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(library_path()))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def take_error(err: ctypes.c_char_p) -> str:
    msg = err.value.decode("utf-8", "replace") if err.value else "unknown error"
    library().rg_free_string(ctypes.cast(err, ctypes.c_void_p))
    return msg


def _call(fn, *args):
    err = ctypes.c_char_p()
    rc = fn(*args, ctypes.byref(err))
    if rc != 0:
        raise RembedError(take_error(err))


@dataclass
class TokenEmbeddings:
    """One text's per-token final hidden states (rembed.go:351-362)."""

    ids: np.ndarray
    vectors: np.ndarray  # [len(ids) x hidden]


class Pending:
    """A submitted batch (Embedder.submit); ``result()`` waits for it once."""

    def __init__(self, emb: "Embedder", ticket: int, out: np.ndarray):
        self._emb, self._ticket, self._out = emb, ticket, out
        self._done = False

    def result(self) -> np.ndarray:
        if not self._done:
            self._done = True
            _call(self._emb._lib.rg_collect, self._emb._ctx, self._ticket)
        return self._out


def pack(seqs: Iterable[Sequence[int]]) -> tuple[np.ndarray, np.ndarray]:
    """Pack token-id sequences into (ids int64 [T], cu_seqlens int32 [n+1])."""
    seqs = [np.asarray(s, dtype=np.int64).reshape(-1) for s in seqs]
    cu = np.zeros(len(seqs) + 1, dtype=np.int32)
    if seqs:
        cu[1:] = np.cumsum([len(s) for s in seqs])
    ids = np.concatenate(seqs) if seqs else np.zeros(0, dtype=np.int64)
    return np.ascontiguousarray(ids, dtype=np.int64), cu


class Embedder:
    """A model resident on one or more GPUs (one weight replica each).

    Thread-safe: the C library serialises calls per device.
    """

    def __init__(self, config: Config, weights: dict, *, int8: bool = False, int8_activations: bool = False,
                 dim: int = 0, devices: Sequence[int] = (0,), fp16: bool = True, strict_fp32: bool = False,
                 workers: int = 0):
        # workers = WithWorkers (rembed.go:109-121): a cap on the CPU fan-out
        # of one Embed call.  The GPU forward has no CPU fan-out (one stream
        # per device, the whole batch in one pass), so the cap is accepted for
        # drop-in use and has no effect.
        del workers
        self._lib = library()
        self._ctx = None
        self.config = config.validate(config.name or "config")
        # WithInt8Activations implies WithInt8 (rembed.go:79-81).  The
        # unquantised path runs fp16 tensor-core operands by default (closest
        # to the reference's fp32; an fp16 overflow is reported, never
        # silently turned into inf); fp16=False selects bf16 operands.
        # strict_fp32 keeps fp32 activations end to end (3xTF32 projections).
        mode = (RG_MODE_INT8_FULL if int8_activations else RG_MODE_INT8_W if int8
                else RG_MODE_FP32 if strict_fp32 else RG_MODE_F16 if fp16 else RG_MODE_BF16)
        H = config.hidden_size
        if dim and not (1 <= dim <= H):
            raise RembedError(f"rembed: WithDim({dim}) out of range [1, {H}]")
        self._dim = dim or H
        devs = (ctypes.c_int * len(devices))(*devices)
        ctx = ctypes.c_void_p()
        desc = desc_from_config(config)
        _call(self._lib.rg_init, ctypes.byref(desc), devs, len(devices), mode, ctypes.byref(ctx))
        self._ctx = ctx
        try:
            for name, arr in weights.items():
                self.upload(name, arr)
            _call(self._lib.rg_finalize, self._ctx)
        except Exception:
            self.close()
            raise

    def upload(self, name: str, arr) -> None:
        a = np.ascontiguousarray(arr)
        if a.dtype == np.float32:
            dt = RG_DTYPE_F32
        elif a.dtype == np.float16:
            dt = RG_DTYPE_F16
        elif a.dtype == np.uint16:  # raw bf16 bits
            dt = RG_DTYPE_BF16
        else:
            a = a.astype(np.float32)
            dt = RG_DTYPE_F32
        shape = (ctypes.c_int64 * a.ndim)(*a.shape)
        _call(self._lib.rg_upload_weight, self._ctx, name.encode(), dt, shape, a.ndim,
              a.ctypes.data_as(ctypes.c_void_p))

    # -- reference API ---------------------------------------------------
    @property
    def dim(self) -> int:
        """Output dimensionality: the WithDim truncation, else hidden_size."""
        return self._dim

    @property
    def model(self) -> str:
        return self.config.name

    def quantized(self) -> bool:
        return self._lib.rg_mode_active(self._ctx) in (RG_MODE_INT8_W, RG_MODE_INT8_FULL)

    def quantized_activations(self) -> bool:
        return self._lib.rg_mode_active(self._ctx) == RG_MODE_INT8_FULL

    def embed(self, seqs: Iterable[Sequence[int]]) -> np.ndarray:
        """One embedding per token-id sequence: (n, dim) float32."""
        ids, cu = pack(seqs)
        return self.embed_packed(ids, cu)

    def embed_packed(self, ids: np.ndarray, cu_seqlens: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        self._check_open()
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        n = len(cu) - 1
        if out is None:
            out = np.empty((n, self._dim), dtype=np.float32)
        if n > 0:
            _call(self._lib.rg_forward, self._ctx, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                  cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, RG_OUT_POOLED, self._dim,
                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return out

    def submit(self, ids: np.ndarray, cu_seqlens: np.ndarray, out: np.ndarray | None = None) -> "Pending":
        """Start embedding a packed batch and return at once (rg_submit): the
        next batch can be prepared while this one runs.  ``result()`` on the
        returned handle waits for it.  Two batches may be in flight."""
        self._check_open()
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        n = len(cu) - 1
        if out is None:
            out = np.empty((n, self._dim), dtype=np.float32)
        ticket = ctypes.c_int64(-1)
        _call(self._lib.rg_submit, self._ctx, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
              cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, RG_OUT_POOLED, self._dim,
              out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), ctypes.byref(ticket))
        return Pending(self, ticket.value, out)

    def embed_stream(self, batches: Iterable[tuple[np.ndarray, np.ndarray]]):
        """Embed packed (ids, cu_seqlens) batches in order, yielding each
        result while the next batch is already on the GPU (one submission
        ahead of the consumer)."""
        pending = None
        for ids, cu in batches:
            nxt = self.submit(ids, cu)
            if pending is not None:
                yield pending.result()
            pending = nxt
        if pending is not None:
            yield pending.result()

    def embed_tokens(self, seqs: Iterable[Sequence[int]]) -> list[TokenEmbeddings]:
        """Per-token final hidden states, unpooled and unnormalised."""
        self._check_open()
        seqs = [np.asarray(s, dtype=np.int64).reshape(-1) for s in seqs]
        ids, cu = pack(seqs)
        H = self.config.hidden_size
        flat = np.empty((int(cu[-1]), H), dtype=np.float32)
        if seqs:
            _call(self._lib.rg_forward, self._ctx, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                  cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(seqs), RG_OUT_TOKENS, H,
                  flat.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return [TokenEmbeddings(ids=s, vectors=flat[cu[i]:cu[i + 1]]) for i, s in enumerate(seqs)]

    def forward_device(self, d_ids: int, d_cu: int, cu_host: np.ndarray, d_out: int, stream: int = 0,
                       dev_index: int = 0, tokens: bool = False) -> None:
        """rg_forward_device over device pointers (ints), no synchronisation."""
        cu = np.ascontiguousarray(cu_host, dtype=np.int32)
        n = len(cu) - 1
        kind = RG_OUT_TOKENS if tokens else RG_OUT_POOLED
        dim = self.config.hidden_size if tokens else self._dim
        _call(self._lib.rg_forward_device, self._ctx, dev_index, ctypes.c_void_p(d_ids), ctypes.c_void_p(d_cu),
              cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, kind, dim, ctypes.c_void_p(d_out),
              ctypes.c_void_p(stream))

    def sync(self, dev_index: int = 0) -> None:
        _call(self._lib.rg_sync, self._ctx, dev_index)

    def last_launches(self, dev_index: int = 0) -> int:
        return self._lib.rg_last_launches(self._ctx, dev_index)

    KERNEL_CLASSES = ("gemm", "attention", "norm", "pool", "quant")

    def profile(self, enable: bool, dev_index: int = 0) -> None:
        """Bracket every launch with CUDA events (rg_profile); clears counters."""
        if self._lib.rg_profile(self._ctx, dev_index, 1 if enable else 0) != 0:
            raise RembedError("rg_profile failed")

    def profile_stats(self, dev_index: int = 0) -> dict:
        """{class: {ms, launches, flops, bytes}} since the last profile(True)."""
        out = {}
        for k, name in enumerate(self.KERNEL_CLASSES):
            ms, n, fl, by = ctypes.c_double(), ctypes.c_int(), ctypes.c_double(), ctypes.c_double()
            if self._lib.rg_profile_stats(self._ctx, dev_index, k, ctypes.byref(ms), ctypes.byref(n),
                                          ctypes.byref(fl), ctypes.byref(by)) != 0:
                raise RembedError("rg_profile_stats failed")
            out[name] = {"ms": ms.value, "launches": n.value, "flops": fl.value, "bytes": by.value}
        return out

    def _check_open(self):
        if not self._ctx:
            raise RembedError("embedder is closed")

    def close(self) -> None:
        if self._ctx:
            self._lib.rg_free(self._ctx)
            self._ctx = None

    def __enter__(self) -> "Embedder":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load(ref: str | os.PathLike, *, int8: bool = False, int8_activations: bool = False, dim: int = 0,
         devices: Sequence[int] = (0,), fp16: bool = True, strict_fp32: bool = False,
         disk_weights: bool = False, workers: int = 0) -> Embedder:
    """rembed.Load over a converted model directory: manifest.json plus
    model.safetensors or a sharded set (model.safetensors.index.json).
    disk_weights = WithDiskWeights: the weights are mapped from
    <dir>/weights.rembedpack, built from the checkpoint on first use;
    workers = WithWorkers, accepted with no effect (no CPU fan-out here).  Hub
    download and HF-config derivation stay with the reference host."""
    from . import weights as W

    p = Path(ref)
    cfg = Config.load(p / "manifest.json")
    tensors = W.disk_weights(p) if disk_weights else W.read_checkpoint(p)
    return Embedder(cfg, tensors, int8=int8, int8_activations=int8_activations, dim=dim, devices=devices,
                    fp16=fp16, strict_fp32=strict_fp32, workers=workers)
