"""Golden fixtures of the oracle (the CPU restatement of the reference's
forward): seeded synthetic weights and token batches for every architecture
the path supports, and the oracle's pooled embeddings for them.

    python tests/golden/make_golden.py        # writes tests/golden/oracle_tiny.npz

The fixture pins the oracle (tests/test_golden.py recomputes it bit for bit
on the CPU) and gives the GPU tests a frozen reference that does not depend
on the oracle being rebuilt on the GPU host.  Inputs are fully determined by
the seeds below; the arrays store them anyway so a reader can see what was
embedded.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from rembed_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "oracle_tiny.npz"

# name -> (nseq, min length, max length): lengths reach past one 64-key block
# and past the local windows of ModernBERT (16) and Gemma (9).
CASES = {
    "tiny-bert": (5, 1, 90),
    "tiny-distilbert": (4, 2, 70),
    "tiny-roberta": (4, 2, 70),
    "tiny-mpnet": (4, 2, 70),
    "tiny-qwen3": (4, 1, 90),
    "tiny-modernbert": (4, 1, 90),
    "tiny-gemma3": (4, 1, 70),
    "tiny-nomic": (4, 1, 90),
}
WEIGHT_SEED, BATCH_SEED = 101, 102
QUANT_CASES = {"tiny-bert": (oracle.QUANT_WEIGHTS, oracle.QUANT_FULL)}


def inputs(name: str):
    cfg = synth.preset(name)
    nseq, lo, hi = CASES[name]
    w = synth.make_weights(cfg, seed=WEIGHT_SEED)
    ids, cu = synth.make_batch(cfg, nseq, lo, hi, seed=BATCH_SEED)
    return cfg, w, ids, cu


def compute() -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    for name in CASES:
        cfg, w, ids, cu = inputs(name)
        out[f"{name}/ids"] = ids
        out[f"{name}/cu"] = cu
        out[f"{name}/fp32"] = oracle.OracleModel(cfg, w, oracle.QUANT_NONE).embed(ids, cu, nthreads=1)
        for q in QUANT_CASES.get(name, ()):
            tag = "int8w" if q == oracle.QUANT_WEIGHTS else "int8full"
            out[f"{name}/{tag}"] = oracle.OracleModel(cfg, w, q).embed(ids, cu, nthreads=1)
    return out


if __name__ == "__main__":
    np.savez_compressed(OUT, **compute())
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")
