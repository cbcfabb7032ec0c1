"""Golden fixture for parity at the benchmark configurations' longest
sequences: the oracle's pooled embeddings of full-width, reduced-depth
variants of ModernBERT-base (8192 tokens: its global layers see the whole
sequence, RoPE theta 160000), Qwen3-0.6B (1024 tokens, causal, RoPE 1e6)
and EmbeddingGemma-300m (2048 tokens, a global and a local layer), in the
oracle's fp32 and weight-only int8 paths.

    python tests/golden/make_long_golden.py   # writes tests/golden/oracle_long.npz

A full-depth CPU forward of these lengths takes hours, and even these
reduced stacks take minutes per sequence (the 8192-token ModernBERT one about
three), so the oracle's outputs are frozen here and the GPU test
(tests/test_gpu_long.py) regenerates only the seeded weights and ids.  The
fixture also stores the ids and a checksum of the weights so a drifting
generator fails loudly instead of comparing different models.
"""

from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from rembed_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "oracle_long.npz"
WEIGHT_SEED, BATCH_SEED = 211, 212
# preset -> sequence lengths (each config's maximum, plus a shorter one)
CASES = {
    "modernbert-base-3l": [513, 2049, 8192],
    "qwen3-0.6b-2l": [511, 1024],
    "embeddinggemma-300m-2l": [2048, 300],
}
QUANTS = {"fp32": oracle.QUANT_NONE, "int8w": oracle.QUANT_WEIGHTS}


def weights_checksum(w: dict) -> np.ndarray:
    """float64 sums of every tensor, in name order."""
    return np.array([float(np.sum(w[k], dtype=np.float64)) for k in sorted(w)])


def inputs(name: str):
    cfg = synth.preset(name)
    w = synth.make_weights(cfg, seed=WEIGHT_SEED)
    ids, cu = synth.batch_of_lengths(cfg, CASES[name], seed=BATCH_SEED)
    return cfg, w, ids, cu


def compute() -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    for name in CASES:
        cfg, w, ids, cu = inputs(name)
        out[f"{name}/ids"] = ids
        out[f"{name}/cu"] = cu
        out[f"{name}/wsum"] = weights_checksum(w)
        for tag, q in QUANTS.items():
            t = time.time()
            out[f"{name}/{tag}"] = oracle.OracleModel(cfg, w, q).embed(ids, cu, nthreads=len(CASES[name]))
            print(f"{name} {tag}: {time.time() - t:.0f} s", flush=True)
    return out


if __name__ == "__main__":
    np.savez_compressed(OUT, **compute())
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")
