"""The numeric modes against the CPU oracle.

fp16 (RG_MODE_F16, the default unquantised path): fp16 tensor-core operands,
fp32 accumulation and fp32 residual stream; cosine >= 0.9999 and max-abs
<= 2e-3 per embedding.
bf16 (RG_MODE_BF16): the same bar, except tiny-gemma3, whose bf16 floor is
measured at max-abs 3.1e-3: its fp32 weights rounded to bf16 (3.1e-3 -> 1.1e-3
when the weights are bf16-exact), unit-gain post-sublayer norms that carry
each sublayer's rounding into the residual, and 128-wide embeddings whose
elements are 2.4x those of the 768-wide production model (which meets 2e-3).
Weight-only int8 (RG_MODE_INT8_W, WithInt8): the PackB8 quantiser
(pack8.go:25-76), int8 weights widened to fp16 inside the GEMM mainloop;
compared with the oracle's own weight-int8 path, cosine >= 0.999
(the north-star bar for w-int8).
"""

import numpy as np
import pytest

import oracle
from rembed_b200 import synth
from rembed_b200.embedder import Embedder

pytestmark = pytest.mark.gpu

COS_BF16, MAXABS_BF16 = 0.9999, 2e-3
COS_INT8_W = 0.999


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


CASES = [("tiny-bert", 9, 1, 200), ("minilm-l6", 12, 8, 128), ("bge-base", 6, 16, 384),
         ("tiny-mpnet", 7, 1, 256), ("tiny-qwen3", 7, 1, 200), ("tiny-modernbert", 7, 1, 120),
         ("tiny-gemma3", 7, 1, 100), ("tiny-nomic", 7, 1, 200), ("qwen3-0.6b", 3, 16, 160),
         ("embeddinggemma-300m", 3, 200, 400)]


@pytest.mark.parametrize("name,nseq,lo,hi", CASES)
def test_fp16_parity(cuda, name, nseq, lo, hi):
    cfg = synth.preset(name)
    w = synth.make_weights(cfg, seed=41)
    ids, cu = synth.make_batch(cfg, nseq, lo, hi, seed=42)
    gpu = Embedder(cfg, w, fp16=True)
    got = gpu.embed_packed(ids, cu)
    gpu.close()
    want = oracle.OracleModel(cfg, w, oracle.QUANT_NONE).embed(ids, cu)
    cos = cosines(got, want)
    print(f"\n[parity] {name} fp16: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= COS_BF16
    assert np.abs(got - want).max() <= MAXABS_BF16


# bf16 max-abs floor of a 128-wide gemma3 stack with fp32 weights (see above)
MAXABS_BF16_TINY_GEMMA = 4e-3


@pytest.mark.parametrize("name,nseq,lo,hi", CASES)
def test_bf16_parity(cuda, name, nseq, lo, hi):
    cfg = synth.preset(name)
    w = synth.make_weights(cfg, seed=31)
    ids, cu = synth.make_batch(cfg, nseq, lo, hi, seed=32)
    gpu = Embedder(cfg, w, fp16=False)
    got = gpu.embed_packed(ids, cu)
    gpu.close()
    want = oracle.OracleModel(cfg, w, oracle.QUANT_NONE).embed(ids, cu)
    cos = cosines(got, want)
    print(f"\n[parity] {name} bf16: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= COS_BF16
    assert np.abs(got - want).max() <= (MAXABS_BF16_TINY_GEMMA if name == "tiny-gemma3" else MAXABS_BF16)


@pytest.mark.parametrize("name,nseq,lo,hi", CASES)
def test_int8_weights_parity(cuda, name, nseq, lo, hi):
    cfg = synth.preset(name)
    w = synth.make_weights(cfg, seed=43)
    ids, cu = synth.make_batch(cfg, nseq, lo, hi, seed=44)
    gpu = Embedder(cfg, w, int8=True)
    assert gpu.quantized() and not gpu.quantized_activations()
    got = gpu.embed_packed(ids, cu)
    gpu.close()
    want = oracle.OracleModel(cfg, w, oracle.QUANT_WEIGHTS).embed(ids, cu)
    cos = cosines(got, want)
    print(f"\n[parity] {name} w-int8: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= COS_INT8_W


def test_fp16_rejects_out_of_range_weight(cuda):
    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=45)
    name = next(k for k in w if k.endswith("attention.self.query.weight"))
    w[name] = w[name].copy()
    w[name][3, 5] = 1e6
    with pytest.raises(Exception, match="fp16 range"):
        Embedder(cfg, w, fp16=True)


def test_fp16_activation_overflow_is_reported(cuda):
    """Weights inside the fp16 range whose FFN activations are not: the
    forward fails with the overflow named; bf16 runs the same model."""
    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=46)
    for k in list(w):
        if k.endswith("intermediate.dense.weight"):
            w[k] = (w[k] * 200000.0).astype(np.float32)  # max |w| ~ 2e4, outputs ~ 5e4 rms
    ids, cu = synth.make_batch(cfg, 3, 4, 30, seed=47)
    gpu = Embedder(cfg, w, fp16=True)
    with pytest.raises(Exception, match="fp16 range"):
        gpu.embed_packed(ids, cu)
    gpu.close()
    gpu = Embedder(cfg, w, fp16=False)
    assert np.isfinite(gpu.embed_packed(ids, cu)).all()
    gpu.close()


def test_fp16_residual_copy_overflow_is_reported(cuda):
    """With the post-norm LayerNorms folded, the residual GEMM also writes
    the unnormalised rows as fp16 for the next GEMM: a residual outside the
    fp16 range fails loudly there instead of turning into inf; in bf16 the
    same model stays finite (its accuracy is not the point: a row mean this
    far above the row's spread is not what a LayerNorm input looks like)."""
    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=50)
    k = next(n for n in w if n.endswith("layer.0.output.dense.bias"))
    w[k] = w[k] + np.float32(1e5)  # the residual after layer 0's FFN, finite in fp32
    ids, cu = synth.make_batch(cfg, 3, 4, 30, seed=51)
    gpu = Embedder(cfg, w, fp16=True)
    with pytest.raises(Exception, match="fp16 range"):
        gpu.embed_packed(ids, cu)
    gpu.close()
    gpu = Embedder(cfg, w, fp16=False)
    assert np.isfinite(gpu.embed_packed(ids, cu)).all()
    gpu.close()


def test_int8_weights_large_batch_widened_path(cuda):
    """At >= 4096 tokens the weight-only int8 GEMMs widen each int8 weight to
    fp16 just before the GEMM instead of converting inside the mainloop; the
    arithmetic is the same (exact integer weights, fp16 activations, fp32
    accumulation, per-channel scale in the epilogue), so a sequence embeds
    bit-identically on either path, and the batch matches the oracle."""
    cfg = synth.preset("bge-base")
    w = synth.make_weights(cfg, seed=48)
    ids, cu = synth.make_batch(cfg, 40, 128, 128, seed=49)  # 5120 tokens
    gpu = Embedder(cfg, w, int8=True)
    big = gpu.embed_packed(ids, cu)
    small = gpu.embed_packed(ids[:cu[6]], cu[:7])  # 768 tokens: in-mainloop int8 path
    gpu.close()
    assert np.array_equal(big[:6], small)
    want = oracle.OracleModel(cfg, w, oracle.QUANT_WEIGHTS).embed(ids[:cu[8]], cu[:9])
    cos = cosines(big[:8], want)
    print(f"\n[parity] bge-base w-int8 widened path: min cos {cos.min():.7f}")
    assert cos.min() >= COS_INT8_W


# strict fp32 (RG_MODE_FP32): the north-star bar, max-abs <= 1e-4 per embedding
MAXABS_STRICT = 1e-4


@pytest.mark.parametrize("name,nseq,lo,hi", CASES + [("modernbert-base", 3, 100, 300), ("nomic-embed-v1.5", 3, 16, 256),
                                                     ("mpnet-base", 3, 16, 300), ("tiny-roberta", 5, 1, 200)])
def test_strict_fp32_parity(cuda, name, nseq, lo, hi):
    cfg = synth.preset(name)
    w = synth.make_weights(cfg, seed=51)
    ids, cu = synth.make_batch(cfg, nseq, lo, hi, seed=52)
    gpu = Embedder(cfg, w, strict_fp32=True)
    assert not gpu.quantized()
    got = gpu.embed_packed(ids, cu)
    gpu.close()
    want = oracle.OracleModel(cfg, w, oracle.QUANT_NONE).embed(ids, cu)
    err = np.abs(got - want).max()
    print(f"\n[parity] {name} strict fp32: min cos {cosines(got, want).min():.9f}, max abs {err:.2e}")
    assert err <= MAXABS_STRICT
