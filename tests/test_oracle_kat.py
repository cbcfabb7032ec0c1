"""Pin the CPU oracle against the reference's own known-answer tests.

Each test restates one test of rostamlabs/rembed (file:line cited) with the
same inputs, expected values and tolerances, applied to the C oracle.
"""

import math

import numpy as np
import pytest

import oracle


def almost(got, want, tol):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= tol), (got, want)


def test_softmax():  # tensor_test.go:154-168
    x = oracle.softmax([1, 2, 3, 0, 0, 0], 2, 3)
    e1, e2, e3 = math.exp(1), math.exp(2), math.exp(3)
    s = e1 + e2 + e3
    almost(x, [e1 / s, e2 / s, e3 / s, 1 / 3, 1 / 3, 1 / 3], 1e-6)
    almost(oracle.softmax([1000, 1000], 1, 2), [0.5, 0.5], 1e-6)


def test_layernorm():  # tensor_test.go:170-185
    inv = 1 / math.sqrt(2.0 / 3.0)
    almost(oracle.layernorm([1, 2, 3], [1, 1, 1], [0, 0, 0], 1, 3, 0.0), [-inv, 0, inv], 1e-6)
    almost(oracle.layernorm([1, 2, 3], [2, 2, 2], [1, 1, 1], 1, 3, 0.0), [1 - 2 * inv, 1, 1 + 2 * inv], 1e-6)


def test_gelu():  # tensor_test.go:187-200
    x = np.arange(-6, 6.0001, 0.25, dtype=np.float32)
    want = [0.5 * float(v) * (1 + math.erf(float(v) / math.sqrt(2))) for v in x]
    almost(oracle.gelu(x), np.float32(want), 1e-6)


def test_gelu_tanh():  # tensor_test.go:206-220
    c = 0.7978845608028654
    x = np.arange(-6, 6.0001, 0.25, dtype=np.float32)
    want = [0.5 * float(d) * (1 + math.tanh(c * (float(d) + 0.044715 * float(d) ** 3))) for d in x]
    almost(oracle.gelu_tanh(x), np.float32(want), 1e-6)


def test_l2normalize():  # tensor_test.go:253-259
    almost(oracle.l2normalize([3, 4]), [0.6, 0.8], 1e-7)
    z = oracle.l2normalize([0, 0])
    assert not np.any(np.isnan(z)) and np.all(z == 0)


def test_add_bias_and_add():  # tensor_test.go:261-267
    x = oracle.add_bias([1, 2, 3, 4], [10, 20], 2, 2)
    almost(x, [11, 22, 13, 24], 0)
    almost(oracle.add(x, [1, 1, 1, 1]), [12, 23, 14, 25], 0)


def test_expf32_against_float64():  # fastmath_test.go:14-45
    xs = np.arange(-87, 88, 0.01, dtype=np.float32)
    for x in xs[::7]:
        got = oracle.expf32(x)
        want = math.exp(float(x))
        bound = 5e-7 if -20 < x < 20 else 5e-6
        assert abs(got - want) / want <= bound, x
    for x in (88.1, 88.5, 88.7):
        assert math.isfinite(oracle.expf32(np.float32(x)))
    assert oracle.expf32(-100) == 0
    assert math.isinf(oracle.expf32(200))
    assert oracle.expf32(0) == 1


def test_erff32_against_float64():  # fastmath_test.go:48-58
    for x in np.arange(-10, 10, 0.003, dtype=np.float32):
        assert abs(oracle.erff32(x) - math.erf(float(x))) <= 5e-7, x
    assert oracle.erff32(0) == 0


def test_relpos_bucket():  # mpnet_test.go:18-38
    cases = [(-513, 15), (-512, 15), (-129, 15), (-128, 15), (-127, 15), (-64, 14), (-17, 10), (-16, 10),
             (-9, 8), (-8, 8), (-7, 7), (-1, 1), (0, 0), (1, 17), (7, 23), (8, 24), (9, 24), (16, 26),
             (17, 26), (64, 30), (127, 31), (128, 31), (129, 31), (512, 31), (513, 31)]
    for rel, want in cases:
        assert oracle.relpos_bucket(rel, 32) == want, rel
    for d in range(-513, 514):
        assert 0 <= oracle.relpos_bucket(d, 32) < 32


def test_quantize_row_u8_rails():  # vnni_test.go:118-134
    dst, s = oracle.quantize_row_u8([127, -127, 0, 63.5], kpad=8)
    assert s != 0
    assert dst[0] == 255 and dst[1] == 1 and dst[2] == 128
    assert dst[4] == 0 and dst[7] == 0
    _, s0 = oracle.quantize_row_u8([0, 0, 0, 0])
    assert s0 == 1


def vnni_reference(a, bT, m, k, n):
    """vnni_test.go:16-58 restated in numpy (float64 weight scale, float32
    activation scale and reciprocal, +128 offset, int32 accumulate)."""
    out = np.zeros((m, n), dtype=np.float32)
    for c in range(n):
        w = bT[c].astype(np.float64)
        scale = np.abs(w).max() / 127
        scale = 1.0 if scale == 0 else scale
        qw = np.rint(w / scale).astype(np.int32)
        colsum = int(qw.sum())
        for r in range(m):
            row = a[r]
            rs = np.float32(np.abs(row).max()) / np.float32(127)
            rs = np.float32(1) if rs == 0 else rs
            inv = np.float32(1) / rs
            q = np.clip(np.rint((row * inv).astype(np.float32).astype(np.float64)).astype(np.int64) + 128, 0, 255)
            acc = int((q * qw).sum())
            out[r, c] = np.float32(np.float32(acc - 128 * colsum) * rs) * np.float32(scale)
    return out


@pytest.mark.parametrize("m,k,n", [(1, 1, 16), (1, 3, 16), (2, 4, 16), (3, 5, 32), (4, 8, 16), (5, 7, 48),
                                   (7, 384, 384), (13, 129, 64)])
def test_matmul_vnni_exact(m, k, n):  # vnni_test.go:63-116
    rng = np.random.default_rng(99)
    a = (rng.random((m, k), dtype=np.float32) * 4 - 2).astype(np.float32)
    bT = (rng.random((n, k), dtype=np.float32) * 2 - 1).astype(np.float32)
    if k > 2:
        a[0, 0], a[0, 1], a[0, 2] = 127.4, -127.4, 0.0001
    q, cs, s = oracle.packb8vnni(bT, k, n)
    got = oracle.matmul_vnni(a, q, cs, s, m, k, n)
    want = vnni_reference(a, bT, m, k, n)
    assert np.array_equal(got, want), np.abs(got - want).max()


@pytest.mark.parametrize("m,k,n", [(1, 1, 16), (3, 7, 16), (4, 33, 32), (5, 384, 48), (12, 384, 384),
                                   (13, 1536, 384), (64, 100, 64)])
def test_matmul_packed8_against_dequantized(m, k, n):  # pack8_test.go:17-97
    rng = np.random.default_rng(23)
    a = (rng.random((m, k), dtype=np.float32) * 2 - 1).astype(np.float32)
    bT = (rng.random((n, k), dtype=np.float32) * 2 - 1).astype(np.float32)
    bT[n // 2, :] = 0
    q, s = oracle.packb8(bT, k, n)
    deq = q.astype(np.float64) * s.astype(np.float64)[:, None]
    want = a.astype(np.float64) @ deq.T
    got = oracle.matmul_packed8(a, q, s, m, k, n)
    tol = max(1e-5, 1e-6 * math.sqrt(k)) * (1 + np.abs(want))
    assert np.all(np.abs(got - want) <= tol)


def test_packb8_rejects_non_finite():  # pack8_test.go:104-117
    bT = np.zeros((16, 4), dtype=np.float32)
    bT.flat[7] = np.nan
    with pytest.raises(oracle.OracleError):
        oracle.packb8(bT, 4, 16)
    bT.flat[7] = np.inf
    with pytest.raises(oracle.OracleError):
        oracle.packb8(bT, 4, 16)


def test_packb8_quantization_error():  # pack8_test.go:119-145
    rng = np.random.default_rng(29)
    k, n = 100, 32
    bT = ((rng.random((n, k), dtype=np.float32) * 2 - 1) *
          np.exp(rng.integers(0, 6, size=(n, k))).astype(np.float32)).astype(np.float32)
    q, s = oracle.packb8(bT, k, n)
    for j in range(n):
        bound = np.abs(bT[j].astype(np.float64)).max() / 254 + 1e-9
        deq = q[j].astype(np.float64) * float(s[j])
        assert np.all(np.abs(deq - bT[j]) <= bound)


def test_matmul_packed_against_float64():  # pack_test.go:17 (tolerance form of tensor_test.go:66)
    rng = np.random.default_rng(5)
    for m, k, n in [(1, 1, 16), (3, 7, 16), (13, 129, 48), (37, 384, 384)]:
        a = (rng.random((m, k), dtype=np.float32) * 2 - 1).astype(np.float32)
        bT = (rng.random((n, k), dtype=np.float32) * 2 - 1).astype(np.float32)
        want = a.astype(np.float64) @ bT.astype(np.float64).T
        got = oracle.matmul_packed(a, bT, m, k, n)
        assert np.all(np.abs(got - want) <= 1e-5 * (1 + np.abs(want)) * math.sqrt(k))
        # k-ordered fused multiply-add from zero, per element (gemm_amd64.s:14-75)
        ref = np.zeros((m, n), dtype=np.float32)
        if m * n * k <= 4096:
            for i in range(m):
                for j in range(n):
                    acc = np.float32(0)
                    for p in range(k):
                        acc = np.float32(np.float64(a[i, p]) * np.float64(bT[j, p]) + np.float64(acc))
                    ref[i, j] = acc
            assert np.array_equal(got, ref)


def test_flash_semantics_of_oracle_attention_matmul():
    """dot4 order (dot_amd64.s:13-80): serial matmul equals float64 within fp32 rounding."""
    rng = np.random.default_rng(7)
    for m, k, n in [(5, 64, 5), (63, 64, 63), (65, 64, 65), (7, 13, 6)]:
        a = (rng.random((m, k), dtype=np.float32) * 2 - 1).astype(np.float32)
        bT = (rng.random((n, k), dtype=np.float32) * 2 - 1).astype(np.float32)
        want = a.astype(np.float64) @ bT.astype(np.float64).T
        got = oracle.matmul_serial(a, bT, m, k, n)
        assert np.all(np.abs(got - want) <= 1e-5 * math.sqrt(k))


def naive_causal_attention(q, k, v, scale):
    """The naive float64 causal softmax of qwen3_test.go:15-43 (per query i,
    softmax over keys [0, i] of (q_i . k_j) * scale, then the weighted sum of
    v_j), vectorised."""
    q, k, v = (np.asarray(a, dtype=np.float64) for a in (q, k, v))
    seq = q.shape[0]
    s = (q @ k.T) * float(scale)
    s[np.triu_indices(seq, 1)] = -np.inf
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return p @ v


FLASH_SEQS = [1, 2, 5, 63, 64, 65, 120, 127, 128, 129, 200]


@pytest.mark.parametrize("seq", FLASH_SEQS)
def test_flash_attn_causal_head(seq):  # qwen3_test.go:45-80
    """The oracle's flashAttnCausalHead against the naive softmax at sizes
    below, at and across the 64-row block boundary, max-abs <= 1e-4 (the
    reference test's bar).  Inputs uniform in [-1, 1) from a fixed seed (the
    reference draws them from Go's math/rand with seed 7; any uniform draw
    exercises the same block logic)."""
    rng = np.random.default_rng(7 + seq)
    dh = 64
    q, k, v = (rng.uniform(-1, 1, size=(seq, dh)).astype(np.float32) for _ in range(3))
    scale = np.float32(1 / math.sqrt(dh))
    got = oracle.flash_attn_causal_head(q, k, v, scale)
    want = naive_causal_attention(q, k, v, scale)
    assert float(np.abs(got - want).max()) <= 1e-4
