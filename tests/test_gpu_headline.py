"""Parity of the exact batch the headline benchmark times.

bench.py's default line embeds, on every rank, 256 sequences of 128 tokens of
the bge-base architecture (weights seed 0, the rank's batch seed 1000 + rank)
in the bf16 mode with the post-norm LayerNorms folded into the GEMMs.  Here
rank 0's batch runs through the same C ABI and is compared, all 256
embeddings, with the CPU oracle (cosine >= 0.9999, max-abs <= 2e-3), and the
int8 modes' results on the first 32 sequences with the oracle's own int8
paths (weight-only int8 cosine >= 0.999, full int8 cosine >= 0.998).  Also
here: the full-size EmbeddingGemma with WithDim(256), the Matryoshka variant
of its benchmark configuration (Dense head, L2, truncate to 256, re-normalise:
gemma3.go:177-198, rembed.go:441-448).
"""

import os

import numpy as np
import pytest

import oracle
from rembed_b200 import ranks, synth
from rembed_b200.embedder import Embedder

pytestmark = pytest.mark.gpu


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


@pytest.fixture(scope="module")
def headline():
    cfg = synth.preset("bge-base")
    w = synth.make_weights(cfg, seed=0)
    ids, cu = synth.make_batch(cfg, 256, 128, 128, seed=ranks.batch_seed(0))
    return cfg, w, ids, cu


def test_headline_batch_bf16_all_256(cuda, headline):
    cfg, w, ids, cu = headline
    with Embedder(cfg, w, fp16=False) as e:
        got = e.embed_packed(ids, cu)
    want = oracle.OracleModel(cfg, w, oracle.QUANT_NONE).embed(ids, cu, nthreads=os.cpu_count())
    cos = cosines(got, want)
    err = float(np.abs(got - want).max())
    print(f"\n[headline parity] bf16 256x128: min cos {cos.min():.7f}, max abs {err:.2e}")
    assert cos.min() >= 0.9999 and err <= 2e-3
    # The bar discriminates sequences: random-init weights give embeddings
    # with a large common component (mean pairwise cosine about 0.997 here),
    # yet every GPU embedding is closer to its own sequence's oracle
    # embedding than to any other's, and the mean pairwise distance is at
    # least ten times the parity bar's.
    off = (want @ want.T)[~np.eye(len(want), dtype=bool)]
    assert 1.0 - float(off.mean()) >= 10 * (1.0 - 0.9999)
    assert np.array_equal(np.argmax(got @ want.T, axis=1), np.arange(len(got)))


@pytest.mark.parametrize("kw,quant,bar", [(dict(int8=True), oracle.QUANT_WEIGHTS, 0.999),
                                          (dict(int8_activations=True), oracle.QUANT_FULL, 0.998)])
def test_headline_batch_int8_modes(cuda, headline, kw, quant, bar):
    cfg, w, ids, cu = headline
    n = 32
    ids_n, cu_n = ids[: cu[n]], cu[: n + 1]
    with Embedder(cfg, w, **kw) as e:
        got = e.embed_packed(ids, cu)[:n]
    want = oracle.OracleModel(cfg, w, quant).embed(ids_n, cu_n, nthreads=os.cpu_count())
    cos = cosines(got, want)
    print(f"\n[headline parity] {kw}: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= bar


def test_gemma_full_size_matryoshka_256(cuda):
    cfg = synth.preset("embeddinggemma-300m")
    w = synth.make_weights(cfg, seed=77)
    ids, cu = synth.make_batch(cfg, 4, 16, 300, seed=78)
    with Embedder(cfg, w, dim=256) as e:
        got = e.embed_packed(ids, cu)
    want = oracle.OracleModel(cfg, w, oracle.QUANT_NONE).embed(ids, cu, dim=256, nthreads=os.cpu_count())
    assert got.shape == (4, 256)
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    cos = cosines(got, want)
    err = float(np.abs(got - want).max())
    print(f"\n[parity] embeddinggemma-300m dim 256: min cos {cos.min():.7f}, max abs {err:.2e}")
    assert cos.min() >= 0.9999 and err <= 2e-3
