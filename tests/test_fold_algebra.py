"""The algebra behind the folded post-norm LayerNorms (CPU, float64).

In the 16-bit modes the BERT family's inner LayerNorms run no kernel: the
residual GEMM writes the unnormalised rows y and the (mean, M2) of each
32-column chunk of every row, a merge forms the row's (mean, rstd), and the
next GEMM uses the weight W' = W * gamma (gamma along K) with the epilogue
    rstd * (y . W'^T) + (b + beta . W^T - rstd * mean * c1),  c1 = sum_k W'.
These tests check that identity against LN(y) . W^T + b, the chunk merge
against a direct two-pass mean / variance, the LayerNorm-on-load rebuild of
the residual (the reference's LayerNorm, bert.go:905-918), and the RMSNorm
form the pre-norm stacks fold (no mean; both halves of a gated FFN).
"""

import numpy as np
import pytest


def layer_norm(y, g, b, eps):
    mean = y.mean(axis=1, keepdims=True)
    var = ((y - mean) ** 2).mean(axis=1, keepdims=True)
    return (y - mean) / np.sqrt(var + eps) * g + b


def chunk_stats(y):
    """(mean, M2) of each 32-column chunk, chunk-major [H/32, T, 2]."""
    T, H = y.shape
    c = y.reshape(T, H // 32, 32)
    m = c.mean(axis=2)
    m2 = ((c - m[:, :, None]) ** 2).sum(axis=2)
    return np.stack([m.T, m2.T], axis=2)


def merge(parts, eps):
    """The merge in the runtime's fixed order: mean of the chunk means, then
    M2 = sum(M2_i + 32 (mean_i - mean)^2); rstd = 1 / sqrt(M2 / H + eps)."""
    n = parts.shape[0]
    mean = parts[:, :, 0].sum(axis=0) / n
    m2 = (parts[:, :, 1] + 32.0 * (parts[:, :, 0] - mean) ** 2).sum(axis=0)
    return mean, 1.0 / np.sqrt(m2 / (32 * n) + eps)


@pytest.mark.parametrize("T,H", [(7, 128), (33, 768), (5, 384), (3, 1024)])
def test_chunk_merge_equals_direct_statistics(T, H):
    rng = np.random.default_rng(T * H)
    y = rng.normal(0.3, 2.0, size=(T, H)) + rng.normal(0, 5, size=(1, H))  # outlier columns
    mean, rstd = merge(chunk_stats(y), 1e-12)
    var = ((y - y.mean(axis=1, keepdims=True)) ** 2).mean(axis=1)
    assert np.allclose(mean, y.mean(axis=1), rtol=1e-12, atol=1e-12)
    assert np.allclose(rstd, 1.0 / np.sqrt(var + 1e-12), rtol=1e-10)


@pytest.mark.parametrize("T,H,N", [(7, 128, 96), (33, 768, 256), (5, 384, 1536)])
def test_folded_gemm_equals_layernorm_then_gemm(T, H, N):
    rng = np.random.default_rng(N)
    eps = 1e-12
    y = rng.normal(0.1, 1.5, size=(T, H))
    g = rng.normal(1.0, 0.1, size=H)
    beta = rng.normal(0.0, 0.05, size=H)
    W = rng.normal(0.0, 0.02, size=(N, H))
    bias = rng.normal(0.0, 0.02, size=N)
    want = layer_norm(y, g, beta, eps) @ W.T + bias
    mean, rstd = merge(chunk_stats(y), eps)
    Wf = W * g[None, :]                 # gain folded along K
    c1 = Wf.sum(axis=1)                 # column sums of the folded weight
    bf = bias + W @ beta                # folded bias
    got = rstd[:, None] * (y @ Wf.T) + (bf[None, :] - (rstd * mean)[:, None] * c1[None, :])
    assert np.allclose(got, want, rtol=1e-10, atol=1e-12)


def test_layernorm_on_load_rebuild():
    """The next residual GEMM adds (r - mean) * rstd * g + b, the LayerNorm
    output never written in fp32, from the same merged statistics."""
    rng = np.random.default_rng(3)
    T, H = 9, 768
    r = rng.normal(0.2, 3.0, size=(T, H))
    g = rng.normal(1.0, 0.1, size=H)
    b = rng.normal(0.0, 0.1, size=H)
    mean, rstd = merge(chunk_stats(r), 1e-12)
    got = (r - mean[:, None]) * rstd[:, None] * g + b
    assert np.allclose(got, layer_norm(r, g, b, 1e-12), rtol=1e-10, atol=1e-12)


def merge_rms(parts, eps):
    """The RMSNorm merge: sum(y^2) = sum(M2_i + 32 mean_i^2) in chunk order."""
    n = parts.shape[0]
    ss = (parts[:, :, 1] + 32.0 * parts[:, :, 0] ** 2).sum(axis=0)
    return 1.0 / np.sqrt(ss / (32 * n) + eps)


@pytest.mark.parametrize("T,H,I", [(6, 256, 512), (17, 1024, 3072)])
def test_folded_rmsnorm_gated_ffn(T, H, I):
    """Pre-norm (Qwen3): RMSNorm(y) . W^T = rstd * (y . (W * g)^T), applied
    to both halves of the gated FFN before the activation."""
    rng = np.random.default_rng(I)
    eps = 1e-6
    y = rng.normal(0.0, 3.0, size=(T, H))
    y[:, 7] *= 50.0  # a massive-activation column
    g = rng.normal(1.0, 0.2, size=H)
    Wg = rng.normal(0.0, 0.02, size=(I, H))
    Wu = rng.normal(0.0, 0.02, size=(I, H))
    xn = y / np.sqrt((y ** 2).mean(axis=1, keepdims=True) + eps) * g
    silu = lambda a: a / (1.0 + np.exp(-a))
    want = silu(xn @ Wg.T) * (xn @ Wu.T)
    rstd = merge_rms(chunk_stats(y), eps)
    a = rstd[:, None] * (y @ (Wg * g).T)
    b = rstd[:, None] * (y @ (Wu * g).T)
    assert np.allclose(silu(a) * b, want, rtol=1e-10, atol=1e-12)
