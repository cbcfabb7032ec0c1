"""ctypes front end for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY.  The oracle restates rembed's CPU forward pass in
C (oracle_prims.c, oracle_model.c) and serves two roles: the parity checker
for the CUDA path (tests/, __graft_entry__.smoke) and the timed CPU baseline
in bench.py.  The product package never imports this module.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

ARCH = {"": 0, "bert": 0, "distilbert": 1, "roberta": 2, "mpnet": 3, "modernbert": 4,
        "qwen3": 5, "gemma3": 6, "nomic_bert": 7}
POOL = {"mean": 0, "cls": 1, "lasttoken": 2}
QUANT_NONE, QUANT_WEIGHTS, QUANT_FULL = 0, 1, 2


class OracleError(RuntimeError):
    pass


class _Cfg(ctypes.Structure):
    _fields_ = [
        ("arch", ctypes.c_int),
        ("hidden", ctypes.c_int), ("layers", ctypes.c_int), ("heads", ctypes.c_int),
        ("inter", ctypes.c_int), ("vocab", ctypes.c_int), ("max_pos", ctypes.c_int),
        ("type_vocab", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("pooling", ctypes.c_int), ("normalize", ctypes.c_int),
        ("pad_token_id", ctypes.c_int), ("rel_buckets", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("kv_heads", ctypes.c_int),
        ("rope_theta", ctypes.c_double), ("global_theta", ctypes.c_double), ("local_theta", ctypes.c_double),
        ("global_every", ctypes.c_int), ("local_attention", ctypes.c_int),
        ("sliding_window", ctypes.c_int), ("sliding_pattern", ctypes.c_int),
        ("query_pre_attn_scalar", ctypes.c_int), ("dense_hidden", ctypes.c_int),
    ]


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the committed Makefile."""
    if force or not _LIB_PATH.exists():
        subprocess.run(["make", "-C", str(_HERE), "-s"] + (["-B"] if force else []), check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        f32p = ctypes.POINTER(ctypes.c_float)
        L.or_expf32.restype = ctypes.c_float
        L.or_expf32.argtypes = [ctypes.c_float]
        L.or_expnonpos.restype = ctypes.c_float
        L.or_expnonpos.argtypes = [ctypes.c_float]
        L.or_erff32.restype = ctypes.c_float
        L.or_erff32.argtypes = [ctypes.c_float]
        L.or_relpos_bucket.restype = ctypes.c_int
        L.or_relpos_bucket.argtypes = [ctypes.c_int, ctypes.c_int]
        L.or_quantize_row_u8.restype = ctypes.c_float
        L.or_model_new.restype = ctypes.c_void_p
        L.or_model_new.argtypes = [ctypes.POINTER(_Cfg), ctypes.c_int]
        L.or_model_set.restype = ctypes.c_int
        L.or_model_set.argtypes = [ctypes.c_void_p, ctypes.c_char_p, f32p, ctypes.c_int64]
        L.or_model_finalize.restype = ctypes.c_int
        L.or_model_finalize.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        L.or_model_free.restype = None
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_flash_attn_causal_head.restype = ctypes.c_int
        L.or_flash_attn_causal_head.argtypes = [f32p, f32p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.or_embed_batch.restype = ctypes.c_int
        L.or_embed_batch.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                                     ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, f32p, ctypes.c_char_p]
        _lib = L
    return _lib


def _p(a: np.ndarray, ct=ctypes.c_float):
    return a.ctypes.data_as(ctypes.POINTER(ct))


# ---- primitives (each mutates a float32 copy and returns it) -------------
def _inplace(fn, x, *args):
    x = np.array(x, dtype=np.float32, copy=True)
    getattr(lib(), fn)(_p(x), *args)
    return x


def softmax(x, m, n):
    return _inplace("or_softmax", x, ctypes.c_int(m), ctypes.c_int(n))


def layernorm(x, g, b, m, n, eps):
    g = np.ascontiguousarray(g, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return _inplace("or_layernorm", x, _p(g), _p(b), ctypes.c_int(m), ctypes.c_int(n), ctypes.c_float(eps))


def rmsnorm(x, g, m, n, eps):
    g = np.ascontiguousarray(g, dtype=np.float32)
    return _inplace("or_rmsnorm", x, _p(g), ctypes.c_int(m), ctypes.c_int(n), ctypes.c_float(eps))


def gelu(x):
    x = np.asarray(x, dtype=np.float32)
    return _inplace("or_gelu", x, ctypes.c_int(x.size))


def gelu_tanh(x):
    x = np.asarray(x, dtype=np.float32)
    return _inplace("or_gelu_tanh", x, ctypes.c_int(x.size))


def silu(x):
    x = np.asarray(x, dtype=np.float32)
    return _inplace("or_silu", x, ctypes.c_int(x.size))


def l2normalize(x):
    x = np.asarray(x, dtype=np.float32)
    return _inplace("or_l2normalize", x, ctypes.c_int(x.size))


def add_bias(x, bias, m, n):
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    return _inplace("or_add_bias", x, _p(bias), ctypes.c_int(m), ctypes.c_int(n))


def add(dst, src):
    src = np.ascontiguousarray(src, dtype=np.float32)
    dst = np.asarray(dst, dtype=np.float32)
    return _inplace("or_add", dst, _p(src), ctypes.c_int(dst.size))


def expf32(x):
    return lib().or_expf32(float(x))


def expnonpos(x):
    return lib().or_expnonpos(float(x))


def erff32(x):
    return lib().or_erff32(float(x))


def relpos_bucket(rel, nb=32):
    return lib().or_relpos_bucket(int(rel), int(nb))


def _mm(fn, a, bT, m, k, n):
    a = np.ascontiguousarray(a, dtype=np.float32)
    bT = np.ascontiguousarray(bT, dtype=np.float32)
    dst = np.zeros((m, n), dtype=np.float32)
    getattr(lib(), fn)(_p(dst), _p(a), _p(bT), ctypes.c_int(m), ctypes.c_int(k), ctypes.c_int(n))
    return dst


def matmul_packed(a, bT, m, k, n):
    return _mm("or_matmul_packed", a, bT, m, k, n)


def matmul_serial(a, bT, m, k, n):
    return _mm("or_matmul_serial", a, bT, m, k, n)


def packb8(bT, k, n):
    bT = np.ascontiguousarray(bT, dtype=np.float32)
    q = np.zeros((n, k), dtype=np.int8)
    s = np.zeros(n, dtype=np.float32)
    rc = lib().or_packb8(_p(bT), ctypes.c_int(k), ctypes.c_int(n), _p(q, ctypes.c_int8), _p(s))
    if rc != 0:
        raise OracleError("PackB8 rejected the weight")
    return q, s


def packb8vnni(bT, k, n):
    bT = np.ascontiguousarray(bT, dtype=np.float32)
    q = np.zeros((n, k), dtype=np.int8)
    cs = np.zeros(n, dtype=np.int32)
    s = np.zeros(n, dtype=np.float32)
    rc = lib().or_packb8vnni(_p(bT), ctypes.c_int(k), ctypes.c_int(n), _p(q, ctypes.c_int8),
                             _p(cs, ctypes.c_int32), _p(s))
    if rc != 0:
        raise OracleError("PackB8VNNI rejected the weight")
    return q, cs, s


def quantize_row_u8(a, kpad=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    kpad = a.size if kpad is None else kpad
    dst = np.full(kpad, 0xAB, dtype=np.uint8)
    s = lib().or_quantize_row_u8(_p(dst, ctypes.c_uint8), _p(a), ctypes.c_int(a.size), ctypes.c_int(kpad))
    return dst, s


def matmul_packed8(a, q, scales, m, k, n):
    a = np.ascontiguousarray(a, dtype=np.float32)
    dst = np.zeros((m, n), dtype=np.float32)
    lib().or_matmul_packed8(_p(dst), _p(a), _p(np.ascontiguousarray(q), ctypes.c_int8),
                            _p(np.ascontiguousarray(scales, dtype=np.float32)),
                            ctypes.c_int(m), ctypes.c_int(k), ctypes.c_int(n))
    return dst


def matmul_vnni(a, q, colsum, scales, m, k, n):
    a = np.ascontiguousarray(a, dtype=np.float32)
    dst = np.zeros((m, n), dtype=np.float32)
    lib().or_matmul_vnni(_p(dst), _p(a), _p(np.ascontiguousarray(q), ctypes.c_int8),
                         _p(np.ascontiguousarray(colsum, dtype=np.int32), ctypes.c_int32),
                         _p(np.ascontiguousarray(scales, dtype=np.float32)),
                         ctypes.c_int(m), ctypes.c_int(k), ctypes.c_int(n))
    return dst


def flash_attn_causal_head(q, k, v, scale):
    """flashAttnCausalHead (qwen3.go:307-390) on one head: q, k, v [seq x dh]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    seq, dh = q.shape
    out = np.zeros((seq, dh), dtype=np.float32)
    if lib().or_flash_attn_causal_head(_p(q), _p(k), _p(v), _p(out), seq, dh, float(scale)) != 0:
        raise OracleError("flash attention scratch allocation failed")
    return out


# ---- model ----------------------------------------------------------------
class OracleModel:
    """The reference forward for one model, over borrowed float32 weights."""

    def __init__(self, cfg, weights: dict, quant: int = QUANT_NONE):
        self.cfg = cfg
        c = _Cfg()
        c.arch = ARCH[cfg.model_type]
        c.hidden, c.layers, c.heads = cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads
        c.inter, c.vocab, c.max_pos = cfg.intermediate_size, cfg.vocab_size, cfg.max_position_embeddings
        c.type_vocab = getattr(cfg, "type_vocab_size", 2)
        c.eps = cfg.layer_norm_eps
        c.pooling, c.normalize = POOL[cfg.pooling], int(bool(cfg.normalize))
        c.pad_token_id, c.rel_buckets = cfg.pad_token_id, cfg.relative_attention_num_buckets
        c.head_dim, c.kv_heads = cfg.head_dim, cfg.num_key_value_heads
        c.rope_theta, c.global_theta, c.local_theta = cfg.rope_theta, cfg.global_rope_theta, cfg.local_rope_theta
        c.global_every, c.local_attention = cfg.global_attn_every_n_layers, cfg.local_attention
        c.sliding_window, c.sliding_pattern = cfg.sliding_window, cfg.sliding_window_pattern
        c.query_pre_attn_scalar, c.dense_hidden = cfg.query_pre_attn_scalar, cfg.dense_hidden
        L = lib()
        self._h = L.or_model_new(ctypes.byref(c), int(quant))
        self._keep = []
        for name, arr in weights.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            self._keep.append(a)
            if L.or_model_set(self._h, name.encode(), _p(a), a.size) != 0:
                raise OracleError(f"cannot set tensor {name}")
        err = ctypes.create_string_buffer(512)
        if L.or_model_finalize(self._h, err) != 0:
            raise OracleError(err.value.decode())

    def embed(self, ids, cu_seqlens, nthreads: int | None = None, dim: int = 0, tokens: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        nseq = len(cu) - 1
        H = self.cfg.hidden_size
        dim = H if dim <= 0 else dim
        nthreads = nthreads or os.cpu_count() or 1
        out = np.zeros((int(cu[-1]), H) if tokens else (nseq, dim), dtype=np.float32)
        err = ctypes.create_string_buffer(512)
        rc = lib().or_embed_batch(self._h, _p(ids, ctypes.c_int64), _p(cu, ctypes.c_int32), nseq, int(nthreads),
                                  1 if tokens else 0, int(dim), _p(out), err)
        if rc != 0:
            raise OracleError(err.value.decode())
        return out

    def close(self):
        if getattr(self, "_h", None):
            lib().or_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
