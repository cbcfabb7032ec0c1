"""End-to-end parity of the CUDA forward pass against the CPU oracle.

Same seeded weights and token ids on both sides; the CUDA path is reached
only through the C ABI (rembed_b200.Embedder -> librembed_gpu.so).
Thresholds (per embedding): bf16 path cosine >= 0.9999 and max-abs <= 2e-3;
full int8 cosine >= 0.998 against the oracle's own full-int8 path.
"""

import numpy as np
import pytest

import oracle
from rembed_b200 import synth
from rembed_b200.embedder import Embedder, RembedError

pytestmark = pytest.mark.gpu

COS_BF16, MAXABS_BF16 = 0.9999, 2e-3
COS_INT8_FULL = 0.998


def cosines(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def mean_pairwise_cos(e):
    e = e.astype(np.float64)
    e = e / np.linalg.norm(e, axis=1, keepdims=True)
    c = e @ e.T
    n = len(e)
    return (c.sum() - np.trace(c)) / (n * (n - 1))


class Model:
    def __init__(self, name, seed=0, quant=oracle.QUANT_NONE, **kw):
        self.cfg = synth.preset(name)
        self.w = synth.make_weights(self.cfg, seed=seed)
        self.gpu = Embedder(self.cfg, self.w, int8_activations=quant == oracle.QUANT_FULL,
                            int8=quant == oracle.QUANT_WEIGHTS, **kw)
        self.ref = oracle.OracleModel(self.cfg, self.w, quant)


@pytest.fixture(scope="module")
def tiny(cuda):
    return Model("tiny-bert")


@pytest.fixture(scope="module")
def minilm(cuda):
    return Model("minilm-l6")


@pytest.fixture(scope="module")
def bge(cuda):
    return Model("bge-base")


@pytest.mark.parametrize("which,nseq,lo,hi", [("tiny", 9, 1, 200), ("minilm", 16, 8, 128), ("bge", 8, 16, 512),
                                              ("bge", 12, 1, 128)])
def test_pooled_parity(request, which, nseq, lo, hi):
    m = request.getfixturevalue(which)
    ids, cu = synth.make_batch(m.cfg, nseq, lo, hi, seed=11, id_hi=min(m.cfg.vocab_size - 1, 30521))
    got = m.gpu.embed_packed(ids, cu)
    want = m.ref.embed(ids, cu)
    cos = cosines(got, want)
    maxabs = np.abs(got - want).max(1)
    print(f"\n[parity] {which}: min cos {cos.min():.7f}, max abs {maxabs.max():.2e}, "
          f"mean pairwise cos between texts {mean_pairwise_cos(want):.5f}")
    assert cos.min() >= COS_BF16, cos
    assert maxabs.max() <= MAXABS_BF16, maxabs
    # The check is meaningful only if different texts are much further apart
    # than the parity threshold allows (random-init CLS pooling is close).
    assert mean_pairwise_cos(want) < 1 - 10 * (1 - COS_BF16)


def test_bge_fixed_128(bge):
    ids, cu = synth.make_batch(bge.cfg, 6, 128, 128, seed=5)
    got = bge.gpu.embed_packed(ids, cu)
    want = bge.ref.embed(ids, cu)
    assert cosines(got, want).min() >= COS_BF16
    assert np.abs(got - want).max() <= MAXABS_BF16


def test_tokens_parity(minilm):
    ids, cu = synth.make_batch(minilm.cfg, 5, 3, 70, seed=12)
    seqs = [ids[cu[i]:cu[i + 1]] for i in range(len(cu) - 1)]
    got = minilm.gpu.embed_tokens(seqs)
    want = minilm.ref.embed(ids, cu, tokens=True)
    for i, te in enumerate(got):
        w = want[cu[i]:cu[i + 1]]
        assert te.vectors.shape == w.shape
        assert np.array_equal(te.ids, seqs[i])
        assert cosines(te.vectors, w).min() >= COS_BF16
    # EmbedTokens pools to Embed (rembed_test.go:1321-1357): mean pool + L2
    pooled = np.stack([t.vectors.mean(0) for t in got])
    pooled /= np.linalg.norm(pooled, axis=1, keepdims=True)
    assert cosines(pooled, minilm.gpu.embed(seqs)).min() >= 0.99999


@pytest.mark.parametrize("name,first", [("bge-base", True), ("tiny-qwen3", False)])
def test_pooled_row_equals_token_output(cuda, name, first):
    """CLS / last-token pooling normalises only the pooled rows at the end
    of the stack: without the L2 step the pooled vector is bit-identical to
    that row of the per-token output, which normalises every row."""
    cfg = synth.preset(name)
    cfg.normalize = False
    w = synth.make_weights(cfg, seed=61)
    ids, cu = synth.make_batch(cfg, 6, 5, 90, seed=62)
    seqs = [ids[cu[i]:cu[i + 1]] for i in range(len(cu) - 1)]
    e = Embedder(cfg, w)
    pooled = e.embed_packed(ids, cu)
    toks = e.embed_tokens(seqs)
    e.close()
    for i, t in enumerate(toks):
        assert np.array_equal(pooled[i], t.vectors[0 if first else -1]), i


def test_batch_equals_single_bit_identical(minilm):
    """Packed varlen batching changes nothing (rembed_test.go:1265-1315)."""
    ids, cu = synth.make_batch(minilm.cfg, 7, 1, 128, seed=13)
    batch = minilm.gpu.embed_packed(ids, cu)
    for i in range(len(cu) - 1):
        one = minilm.gpu.embed([ids[cu[i]:cu[i + 1]]])
        assert np.array_equal(one[0], batch[i]), i
    again = minilm.gpu.embed_packed(ids, cu)
    assert np.array_equal(again, batch)


def test_matryoshka_dim(minilm):
    ids, cu = synth.make_batch(minilm.cfg, 4, 5, 60, seed=14)
    full = minilm.gpu.embed_packed(ids, cu)
    e = Embedder(minilm.cfg, minilm.w, dim=100)
    assert e.dim == 100
    short = e.embed_packed(ids, cu)
    want = full[:, :100] / np.linalg.norm(full[:, :100].astype(np.float64), axis=1, keepdims=True)
    assert np.abs(short - want).max() <= 1e-6
    ref = minilm.ref.embed(ids, cu, dim=100)
    assert cosines(short, ref).min() >= COS_BF16
    e.close()


def test_errors_match_reference_wording(tiny):
    g = tiny.gpu
    with pytest.raises(RembedError, match="empty token sequence"):
        g.embed([[101, 102], []])
    with pytest.raises(RembedError, match="exceeds the model's maximum"):
        g.embed([[5] * (tiny.cfg.max_seq_len() + 1)])
    with pytest.raises(RembedError, match="out of vocab range"):
        g.embed([[101, tiny.cfg.vocab_size, 102]])
    with pytest.raises(RembedError, match="out of vocab range"):
        g.embed([[101, -1, 102]])
    # the context is still usable after a rejected call
    assert g.embed([[101, 7, 102]]).shape == (1, tiny.cfg.hidden_size)


def test_bad_id_on_device_path_is_reported(tiny, cuda):
    torch = cuda
    ids = torch.tensor([101, 5, tiny.cfg.vocab_size + 3, 102], device="cuda", dtype=torch.int64)
    cu_h = np.array([0, 4], dtype=np.int32)
    cu = torch.from_numpy(cu_h).cuda()
    out = torch.empty((1, tiny.cfg.hidden_size), device="cuda")
    torch.cuda.synchronize()
    tiny.gpu.forward_device(ids.data_ptr(), cu.data_ptr(), cu_h, out.data_ptr())
    with pytest.raises(RembedError, match="token id out of vocab range"):
        tiny.gpu.sync()
    tiny.gpu.sync()  # status cleared once reported


def test_full_int8_parity(minilm_int8):
    m = minilm_int8
    assert m.gpu.quantized() and m.gpu.quantized_activations()
    ids, cu = synth.make_batch(m.cfg, 12, 8, 128, seed=15)
    got = m.gpu.embed_packed(ids, cu)
    want = m.ref.embed(ids, cu)
    print(f"\n[parity] minilm full int8: min cos {cosines(got, want).min():.6f}, "
          f"max abs {np.abs(got - want).max():.2e}")
    assert cosines(got, want).min() >= COS_INT8_FULL
    # "quant must be active": the int8 result differs from the fp32 oracle
    fp = oracle.OracleModel(m.cfg, m.w, oracle.QUANT_NONE).embed(ids, cu)
    assert np.abs(want - fp).max() > 1e-4


@pytest.fixture(scope="module")
def minilm_int8(cuda):
    return Model("minilm-l6", quant=oracle.QUANT_FULL)


@pytest.mark.parametrize("name,nseq,lo,hi", [("tiny-distilbert", 7, 1, 200), ("tiny-roberta", 7, 1, 256),
                                             ("tiny-mpnet", 9, 1, 256), ("mpnet-base", 6, 16, 384)])
def test_bert_path_variants(cuda, name, nseq, lo, hi):
    """DistilBERT names, RoBERTa's position offset and MPNet's relative
    attention bias (bert.go:338-518, 820-830, 876-889) on the same kernels."""
    m = Model(name)
    ids, cu = synth.make_batch(m.cfg, nseq, lo, hi, seed=21, id_lo=5, id_hi=m.cfg.vocab_size - 1, cls_id=0, sep_id=2)
    got = m.gpu.embed_packed(ids, cu)
    want = m.ref.embed(ids, cu)
    cos = cosines(got, want)
    print(f"\n[parity] {name}: min cos {cos.min():.7f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= COS_BF16
    assert np.abs(got - want).max() <= MAXABS_BF16
    m.gpu.close()


def test_full_int8_parity_bge(cuda):
    m = Model("bge-base", quant=oracle.QUANT_FULL)
    ids, cu = synth.make_batch(m.cfg, 6, 16, 256, seed=16)
    got = m.gpu.embed_packed(ids, cu)
    want = m.ref.embed(ids, cu)
    cos = cosines(got, want)
    print(f"\n[parity] bge full int8: min cos {cos.min():.6f}, max abs {np.abs(got - want).max():.2e}")
    assert cos.min() >= COS_INT8_FULL
    m.gpu.close()


def test_multi_device_context_matches_single_device(cuda):
    """rg_forward over a context holding two devices assigns the sequences
    to the devices by estimated cost (longest first, each to the least
    loaded device), each result landing in its own row of the output; the
    result equals one device's bit for bit."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    cfg = synth.preset("minilm-l6")
    w = synth.make_weights(cfg, seed=61)
    ids, cu = synth.make_batch(cfg, 21, 4, 128, seed=62)
    one = Embedder(cfg, w, devices=(0,))
    two = Embedder(cfg, w, devices=(0, 1))
    a = one.embed_packed(ids, cu)
    b = two.embed_packed(ids, cu)
    one.close()
    two.close()
    assert np.array_equal(a, b)


def test_load_sharded_and_disk_weights(cuda, tmp_path):
    """load() over a sharded checkpoint and over the weights.rembedpack it
    builds (WithDiskWeights) gives the same embeddings as the in-memory
    weights."""
    import json

    from rembed_b200.embedder import load

    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=71)
    names = sorted(w)
    shards = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    for f, ns in shards.items():
        synth.write_safetensors(tmp_path / f, {n: w[n] for n in ns})
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {n: f for f, ns in shards.items() for n in ns}}))
    (tmp_path / "manifest.json").write_text(cfg.to_json())
    ids, cu = synth.make_batch(cfg, 5, 3, 60, seed=72)
    ref = Embedder(cfg, w)
    want = ref.embed_packed(ids, cu)
    ref.close()
    for disk in (False, True):
        e = load(tmp_path, disk_weights=disk)
        assert np.array_equal(e.embed_packed(ids, cu), want)
        e.close()
    assert (tmp_path / "weights.rembedpack").exists()


def test_submit_collect_pipeline(minilm):
    """rg_submit / rg_collect: two batches in flight, results identical to
    the synchronous call; a third submission is refused until one is
    collected; a collected ticket cannot be collected again."""
    b1 = synth.make_batch(minilm.cfg, 9, 4, 128, seed=81)
    b2 = synth.make_batch(minilm.cfg, 5, 4, 128, seed=82)
    b3 = synth.make_batch(minilm.cfg, 7, 4, 128, seed=83)
    want = [minilm.gpu.embed_packed(*b) for b in (b1, b2, b3)]
    p1 = minilm.gpu.submit(*b1)
    p2 = minilm.gpu.submit(*b2)
    with pytest.raises(RembedError, match="outstanding"):
        minilm.gpu.submit(*b3)
    assert np.array_equal(p1.result(), want[0])
    p3 = minilm.gpu.submit(*b3)
    assert np.array_equal(p2.result(), want[1])
    assert np.array_equal(p3.result(), want[2])
    got = list(minilm.gpu.embed_stream([b1, b2, b3, b1]))
    assert all(np.array_equal(g, w) for g, w in zip(got, want + [want[0]]))
    import ctypes

    err = ctypes.c_char_p()
    assert minilm.gpu._lib.rg_collect(minilm.gpu._ctx, 0, ctypes.byref(err)) != 0
    minilm.gpu._lib.rg_free_string(ctypes.cast(err, ctypes.c_void_p))


def test_concurrent_forward_calls(minilm):
    """The Embedder is safe for concurrent use (rembed.go:37-41): four
    threads calling the synchronous forward on one context all succeed and
    get the single-threaded results."""
    import threading

    batches = [synth.make_batch(minilm.cfg, 6, 4, 100, seed=90 + k) for k in range(4)]
    want = [minilm.gpu.embed_packed(*b) for b in batches]
    got, errs = [None] * 4, []

    def run(k):
        try:
            for _ in range(3):
                got[k] = minilm.gpu.embed_packed(*batches[k])
        except Exception as e:  # pragma: no cover - reported below
            errs.append(e)

    th = [threading.Thread(target=run, args=(k,)) for k in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errs
    assert all(np.array_equal(g, w) for g, w in zip(got, want))
