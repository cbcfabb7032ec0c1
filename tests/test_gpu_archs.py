"""Parity of the CUDA forward pass for the RoPE / gated-FFN architectures
(Qwen3, ModernBERT, EmbeddingGemma, nomic-bert) against the CPU oracle.

The sequence lengths reach past each model's local attention window so that
the windowed layers (ModernBERT's local_attention, Gemma's sliding_window)
are exercised, and past one 64-key block so that the causal flash blocks of
Qwen3 are too.  Same thresholds as the BERT family: cosine >= 0.9999 and
max-abs <= 2e-3 per pooled embedding.
"""

import numpy as np
import pytest

import oracle
from rembed_b200 import synth
from rembed_b200.embedder import Embedder

pytestmark = pytest.mark.gpu

COS_BF16, MAXABS_BF16 = 0.9999, 2e-3


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def run(name, nseq, lo, hi, seed=31, dim=0, out_tokens=False):
    cfg = synth.preset(name)
    w = synth.make_weights(cfg, seed=seed)
    gpu = Embedder(cfg, w, dim=dim)
    ref = oracle.OracleModel(cfg, w, oracle.QUANT_NONE)
    ids, cu = synth.make_batch(cfg, nseq, lo, hi, seed=seed + 1)
    try:
        if out_tokens:
            seqs = [ids[cu[i]:cu[i + 1]] for i in range(len(cu) - 1)]
            got = np.concatenate([t.vectors for t in gpu.embed_tokens(seqs)])
            return got, ref.embed(ids, cu, tokens=True), cfg
        return gpu.embed_packed(ids, cu), ref.embed(ids, cu, dim=dim), cfg
    finally:
        gpu.close()


@pytest.mark.parametrize("name,nseq,lo,hi", [
    ("tiny-qwen3", 7, 1, 200),        # causal, GQA 2:1, last-token pooling
    ("tiny-modernbert", 7, 1, 120),   # local window 16 every layer but the 1st of 3
    ("tiny-gemma3", 7, 1, 100),       # sliding window 9, GQA 2:1, Dense head
    ("tiny-nomic", 7, 1, 200),        # post-norm + RoPE + SwiGLU
])
def test_arch_parity_tiny(cuda, name, nseq, lo, hi):
    got, want, _ = run(name, nseq, lo, hi)
    cos = cosines(got, want)
    print(f"\n[parity] {name}: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert np.isfinite(got).all()
    assert cos.min() >= COS_BF16
    assert np.abs(got - want).max() <= MAXABS_BF16


@pytest.mark.parametrize("name,nseq,lo,hi", [
    ("modernbert-base", 4, 100, 300),
    ("nomic-embed-v1.5", 4, 16, 256),
    ("embeddinggemma-300m", 3, 200, 400),   # lengths past the 257-token window
    ("qwen3-0.6b", 3, 16, 160),             # head_dim 128
])
def test_arch_parity_full_size(cuda, name, nseq, lo, hi):
    got, want, _ = run(name, nseq, lo, hi)
    cos = cosines(got, want)
    print(f"\n[parity] {name}: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= COS_BF16
    assert np.abs(got - want).max() <= MAXABS_BF16


def test_gemma_matryoshka_dim(cuda):
    """Dense head, then L2, then truncate + re-normalise (gemma3.go:177-198,
    rembed.go:441-448)."""
    got, want, _ = run("tiny-gemma3", 5, 1, 60, dim=64)
    assert got.shape == (5, 64)
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    assert cosines(got, want).min() >= COS_BF16


@pytest.mark.parametrize("name", ["tiny-qwen3", "tiny-modernbert"])
def test_arch_tokens(cuda, name):
    """Per-token hidden states after the final norm."""
    got, want, cfg = run(name, 4, 1, 90, out_tokens=True)
    assert got.shape == want.shape
    cos = cosines(got, want)
    print(f"\n[parity] {name} tokens: min cos {cos.min():.7f}")
    assert cos.min() >= 0.999
