"""The committed golden fixture (tests/golden/oracle_tiny.npz, made by
tests/golden/make_golden.py): the oracle's embeddings of seeded tiny models of
every architecture.

CPU: the oracle reproduces the fixture bit for bit (its arithmetic is
deterministic, one serial forward per sequence).  GPU: the CUDA path, through
the C ABI, against the frozen fixture with the same bars as the live-oracle
tests: fp16 cosine >= 0.9999 and max-abs <= 2e-3, strict fp32 max-abs <= 1e-4,
weight-only int8 cosine >= 0.999, full int8 cosine >= 0.998.
"""

import importlib.util
from pathlib import Path

import numpy as np
import pytest

from rembed_b200 import synth

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURE = GOLDEN / "oracle_tiny.npz"


def _maker():
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CASES = ["tiny-bert", "tiny-distilbert", "tiny-roberta", "tiny-mpnet", "tiny-qwen3", "tiny-modernbert",
         "tiny-gemma3", "tiny-nomic"]
WEIGHT_SEED, BATCH_SEED = 101, 102
SHAPES = {"tiny-bert": (5, 1, 90), "tiny-distilbert": (4, 2, 70), "tiny-roberta": (4, 2, 70),
          "tiny-mpnet": (4, 2, 70), "tiny-qwen3": (4, 1, 90), "tiny-modernbert": (4, 1, 90),
          "tiny-gemma3": (4, 1, 70), "tiny-nomic": (4, 1, 90)}


def _inputs(name):
    cfg = synth.preset(name)
    nseq, lo, hi = SHAPES[name]
    return cfg, synth.make_weights(cfg, seed=WEIGHT_SEED), *synth.make_batch(cfg, nseq, lo, hi, seed=BATCH_SEED)


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def test_fixture_cases_match_the_generator():
    mk = _maker()
    assert list(mk.CASES) == CASES and mk.CASES == SHAPES
    assert (mk.WEIGHT_SEED, mk.BATCH_SEED) == (WEIGHT_SEED, BATCH_SEED)


def test_oracle_reproduces_the_fixture():
    want = np.load(FIXTURE)
    got = _maker().compute()
    assert sorted(got) == sorted(want.files)
    for k in want.files:
        assert np.array_equal(got[k], want[k]), k


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_gpu_matches_the_fixture(cuda, name):
    from rembed_b200.embedder import Embedder

    g = np.load(FIXTURE)
    cfg, w, ids, cu = _inputs(name)
    assert np.array_equal(ids, g[f"{name}/ids"]) and np.array_equal(cu, g[f"{name}/cu"])
    want = g[f"{name}/fp32"]
    with Embedder(cfg, w) as e:  # fp16 operands
        got = e.embed_packed(ids, cu)
    cos = cosines(got, want)
    print(f"\n[golden] {name} fp16: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= 0.9999 and np.abs(got - want).max() <= 2e-3
    with Embedder(cfg, w, strict_fp32=True) as e:
        got = e.embed_packed(ids, cu)
    print(f"[golden] {name} strict fp32: max abs {np.abs(got - want).max():.2e}")
    assert np.abs(got - want).max() <= 1e-4


@pytest.mark.gpu
def test_gpu_int8_matches_the_fixture(cuda):
    from rembed_b200.embedder import Embedder

    g = np.load(FIXTURE)
    cfg, w, ids, cu = _inputs("tiny-bert")
    with Embedder(cfg, w, int8=True) as e:
        assert cosines(e.embed_packed(ids, cu), g["tiny-bert/int8w"]).min() >= 0.999
    with Embedder(cfg, w, int8_activations=True) as e:
        assert cosines(e.embed_packed(ids, cu), g["tiny-bert/int8full"]).min() >= 0.998
