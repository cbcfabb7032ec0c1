"""CPU tokenisation overlapping the GPU forward (rembed.go's Embed
tokenises on the CPU, tokenizer/tokenizer.go:198-218, then embeds; the GPU
path keeps tokenisation on the host and runs the forward one batch ahead).

A BERT WordPiece tokeniser over a seeded synthetic vocabulary (the
`tokenizers` library, no files needed) turns seeded random text into token
ids; `Embedder.embed_stream` takes a lazy generator of tokenised batches,
so batch k + 1 is tokenised on the CPU while batch k runs on the GPU.  The
test checks that the streamed embeddings equal the ones of tokenising and
embedding each batch in turn, and prints the times of both schedules (the
timing bound is loose on purpose: the GPUs are shared).
"""

import time

import numpy as np
import pytest

from rembed_b200 import synth
from rembed_b200.embedder import Embedder, pack

pytestmark = pytest.mark.gpu

tokenizers = pytest.importorskip("tokenizers")

LETTERS = "abcdefghijklmnopqrstuvwxyz"


def wordpiece(vocab_size: int, seed: int):
    """A BertTokenizer-style pipeline over `vocab_size` synthetic entries:
    the special tokens at their BERT ids, single letters and their '##'
    continuations, then seeded 2-6 letter pieces (whole words and '##'
    continuations)."""
    rng = np.random.default_rng(seed)
    vocab = {"[PAD]": 0, "[UNK]": 100, "[CLS]": 101, "[SEP]": 102, "[MASK]": 103}
    nxt = 104
    for ch in LETTERS:
        for piece in (ch, "##" + ch):
            vocab[piece] = nxt
            nxt += 1
    while nxt < vocab_size:
        n = int(rng.integers(2, 7))
        word = "".join(rng.choice(list(LETTERS), n))
        piece = word if rng.random() < 0.6 else "##" + word
        if piece not in vocab:
            vocab[piece] = nxt
            nxt += 1
    tok = tokenizers.Tokenizer(tokenizers.models.WordPiece(vocab, unk_token="[UNK]", max_input_chars_per_word=100))
    tok.normalizer = tokenizers.normalizers.BertNormalizer(lowercase=True)
    tok.pre_tokenizer = tokenizers.pre_tokenizers.BertPreTokenizer()
    tok.post_processor = tokenizers.processors.TemplateProcessing(
        single="[CLS] $A [SEP]", special_tokens=[("[CLS]", 101), ("[SEP]", 102)])
    tok.enable_truncation(max_length=128)
    return tok


def texts(n: int, seed: int) -> list[str]:
    """n seeded texts of 40-110 words of 2-9 letters."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        words = ["".join(rng.choice(list(LETTERS), int(rng.integers(2, 10)))) for _ in range(int(rng.integers(40, 110)))]
        out.append(" ".join(words))
    return out


def test_tokenisation_overlaps_the_forward(cuda):
    cfg = synth.preset("bge-base")
    w = synth.make_weights(cfg, seed=21)
    tok = wordpiece(cfg.vocab_size, seed=22)
    chunks = [texts(256, seed=100 + k) for k in range(8)]

    def tokenised(chunk):
        return pack([e.ids for e in tok.encode_batch(chunk)])

    with Embedder(cfg, w) as emb:
        emb.embed_packed(*tokenised(chunks[0]))  # warm-up
        # tokenise, then embed, one batch at a time
        t0 = time.perf_counter()
        serial = [emb.embed_packed(*tokenised(c)) for c in chunks]
        t_serial = time.perf_counter() - t0
        # the tokenisation alone
        t0 = time.perf_counter()
        packed = [tokenised(c) for c in chunks]
        t_tok = time.perf_counter() - t0
        # the forward alone, one batch ahead
        t0 = time.perf_counter()
        list(emb.embed_stream(packed))
        t_gpu = time.perf_counter() - t0
        # batch k + 1 tokenised while batch k runs
        t0 = time.perf_counter()
        streamed = list(emb.embed_stream(tokenised(c) for c in chunks))
        t_stream = time.perf_counter() - t0

    for a, b in zip(serial, streamed):
        assert np.array_equal(a, b)
    hidden = (t_serial - t_stream) / max(min(t_tok, t_gpu), 1e-9)
    print(f"\n[pipeline] 8 x 256 texts: tokenise {1e3 * t_tok:.1f} ms, forward {1e3 * t_gpu:.1f} ms, "
          f"one after the other {1e3 * t_serial:.1f} ms, overlapped {1e3 * t_stream:.1f} ms "
          f"({100 * hidden:.0f}% of the shorter side hidden)")
    assert t_stream <= 1.05 * t_serial
