"""Parity at the benchmark configurations' longest sequences.

The oracle's embeddings of full-width, reduced-depth variants of ModernBERT
(513, 2049 and 8192 tokens: the global layer sees the whole sequence with
RoPE theta 160000, the local layers the 128-wide window), Qwen3-0.6B (511 and
1024 tokens, causal, GQA 16:8, RoPE 1e6) and EmbeddingGemma-300m (2048 and
300 tokens, a local layer with the 257 window and a global one) are frozen in
tests/golden/oracle_long.npz (made by tests/golden/make_long_golden.py, whose
seeds this test reuses).  Every numeric mode runs the same batch through the
C ABI:
  bf16 / fp16: cosine >= 0.9999 and max-abs <= 2e-3 per embedding;
  strict fp32: max-abs <= 1e-4;
  weight-only int8 (against the oracle's own int8 path): cosine >= 0.999.
"""

import importlib.util
from pathlib import Path

import numpy as np
import pytest

from rembed_b200.embedder import Embedder

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _maker():
    spec = importlib.util.spec_from_file_location("make_long_golden", GOLDEN / "make_long_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


MODES = {"bf16": dict(fp16=False), "f16": dict(fp16=True), "fp32": dict(strict_fp32=True),
         "int8w": dict(int8=True)}


@pytest.fixture(scope="module")
def fixture():
    return np.load(GOLDEN / "oracle_long.npz")


@pytest.mark.parametrize("name", ["modernbert-base-3l", "qwen3-0.6b-2l", "embeddinggemma-300m-2l"])
def test_long_sequences_every_mode(cuda, fixture, name):
    mk = _maker()
    cfg, w, ids, cu = mk.inputs(name)
    assert np.array_equal(ids, fixture[f"{name}/ids"]) and np.array_equal(cu, fixture[f"{name}/cu"])
    assert np.array_equal(mk.weights_checksum(w), fixture[f"{name}/wsum"]), "weight generator drifted"
    for mode, kw in MODES.items():
        with Embedder(cfg, w, **kw) as e:
            got = e.embed_packed(ids, cu)
        want = fixture[f"{name}/{'int8w' if mode == 'int8w' else 'fp32'}"]
        cos = cosines(got, want)
        err = float(np.abs(got - want).max())
        print(f"\n[long parity] {name} {mode} lens {np.diff(cu).tolist()}: min cos {cos.min():.7f}, max abs {err:.2e}")
        if mode == "fp32":
            assert err <= 1e-4, (mode, err)
        elif mode == "int8w":
            assert cos.min() >= 0.999, (mode, cos)
        else:
            assert cos.min() >= 0.9999 and err <= 2e-3, (mode, cos.min(), err)
