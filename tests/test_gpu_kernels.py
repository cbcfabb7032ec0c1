"""Kernel-level parity through the C ABI: the fused attention kernel and the
full-int8 quantiser + integer GEMM.

Attention (rg_attention) is pinned the way the reference pins its own flash
kernel: qwen3_test.go:45-80 (TestFlashAttnCausalHead) compares the tiled
online-softmax attention with a naive softmax at sequence lengths below, at
and across its 64-row block boundary, max-abs <= 1e-4.  Here the same length
list runs as one packed varlen batch through the tcgen05 kernel (bf16, fp16)
and the strict fp32 kernel, against a float64 naive softmax of the same
(16-bit rounded) inputs.  Bars:
  fp32: 1e-4, the reference test's own;
  fp16: 1e-3 and bf16: 8e-3, i.e. 2u (u = 2^-11 / 2^-8, the unit roundoff):
    the probabilities P enter the P.V product rounded to 16 bits (relative
    error u, |v| <= 1) and the output is rounded to 16 bits (u |o| <= u).
Windowed, bidirectional and grouped-query variants and the long lengths of
the benchmark configurations (ModernBERT's global layers at 8192 tokens,
Qwen3's causal layers at 1024) use the same bars.

Full int8 (rg_quantize_rows_s8 + rg_dense_s8) must equal the oracle's
restatement of QuantizeRowU8 and MatMulPackedVNNI (pack_vnni.go:85-176) bit
for bit: s8 x s8 kind::i8 accumulates sum(q * w) exactly, which is the
reference's acc - 128 * colSum, and the dequantisation (acc * rowScale) *
colScale, then + bias, rounds in the reference's order.
"""

import ctypes
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

RG_DTYPE_F32, RG_DTYPE_F16, RG_DTYPE_BF16 = 0, 1, 2
BIG = 1 << 30
FLASH_SEQS = [1, 2, 5, 63, 64, 65, 120, 127, 128, 129, 200]
BARS = {RG_DTYPE_F32: 1e-4, RG_DTYPE_F16: 1e-3, RG_DTYPE_BF16: 8e-3}


def _call(name, *args):
    from rembed_b200.embedder import RembedError, library, take_error

    err = ctypes.c_char_p()
    rc = getattr(library(), name)(*args, ctypes.byref(err))
    if rc != 0:
        raise RembedError(take_error(err))


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def kernel_status(torch):
    _call("rg_kernel_status", ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def naive_attention(q, k, v, cu, heads, kv_heads, dh, scale, lo, hi):
    """float64 softmax(Q K^T * scale, keys lo <= j - i <= hi) V per sequence and head."""
    out = np.zeros((q.shape[0], heads * dh))
    group = heads // kv_heads
    for s in range(len(cu) - 1):
        a, b = int(cu[s]), int(cu[s + 1])
        L = b - a
        rel = np.arange(L)[None, :] - np.arange(L)[:, None]
        allowed = (rel >= lo) & (rel <= hi)
        for h in range(heads):
            hk = h // group
            Q = q[a:b, h * dh:(h + 1) * dh]
            K = k[a:b, hk * dh:(hk + 1) * dh]
            V = v[a:b, hk * dh:(hk + 1) * dh]
            for r0 in range(0, L, 2048):  # row blocks bound the score matrix
                S = (Q[r0:r0 + 2048] @ K.T) * float(scale)
                S[~allowed[r0:r0 + 2048]] = -np.inf
                S -= S.max(axis=1, keepdims=True)
                P = np.exp(S)
                P /= P.sum(axis=1, keepdims=True)
                out[a + r0:a + r0 + S.shape[0], h * dh:(h + 1) * dh] = P @ V
    return out


def run_attention(torch, lens, heads, kv_heads, dh, lo, hi, dtype, seed):
    """Uniform [-1, 1) q/k/v for a packed batch of `lens`; returns (got, want)."""
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    T = int(cu[-1])
    rng = np.random.default_rng(seed)
    tdt = {RG_DTYPE_F32: torch.float32, RG_DTYPE_F16: torch.float16, RG_DTYPE_BF16: torch.bfloat16}[dtype]
    q = torch.from_numpy(rng.uniform(-1, 1, (T, heads * dh)).astype(np.float32)).to("cuda", tdt)
    k = torch.from_numpy(rng.uniform(-1, 1, (T, kv_heads * dh)).astype(np.float32)).to("cuda", tdt)
    v = torch.from_numpy(rng.uniform(-1, 1, (T, kv_heads * dh)).astype(np.float32)).to("cuda", tdt)
    out = torch.full((T, heads * dh), float("nan"), device="cuda", dtype=tdt)
    d_cu = torch.from_numpy(cu).to("cuda")
    scale = 1.0 / math.sqrt(dh)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _call("rg_attention", _vp(q), _vp(k), _vp(v), heads * dh, kv_heads * dh, kv_heads * dh, _vp(d_cu),
          cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(lens), heads, kv_heads, dh, ctypes.c_float(scale),
          lo, hi, dtype, _vp(out), heads * dh, st)
    kernel_status(torch)
    got = out.float().cpu().numpy().astype(np.float64)
    want = naive_attention(q.float().cpu().numpy().astype(np.float64), k.float().cpu().numpy().astype(np.float64),
                           v.float().cpu().numpy().astype(np.float64), cu, heads, kv_heads, dh,
                           np.float32(scale), lo, hi)
    return got, want


@pytest.mark.parametrize("dtype", [RG_DTYPE_F32, RG_DTYPE_F16, RG_DTYPE_BF16])
@pytest.mark.parametrize("dh", [64, 128])
def test_attention_causal_kat(cuda, dtype, dh):
    """TestFlashAttnCausalHead (qwen3_test.go:45-80) on the GPU kernels, the
    whole length list as one packed batch, two query heads sharing one
    key/value head (Qwen3's grouping)."""
    got, want = run_attention(cuda, FLASH_SEQS, 2, 1, dh, -BIG, 0, dtype, seed=7 + dh)
    err = float(np.abs(got - want).max())
    assert err <= BARS[dtype], err


@pytest.mark.parametrize("dtype", [RG_DTYPE_F32, RG_DTYPE_BF16])
@pytest.mark.parametrize("case", [
    # (lens, heads, kv_heads, dh, lo, hi): ModernBERT local (|i-j| <= 64), Gemma local (|i-j| < 257),
    # bidirectional BERT / MiniLM heads
    ([7, 129, 300, 64, 513], 3, 3, 64, -64, 64),
    ([16, 700, 257, 258], 3, 1, 256, -256, 256),
    ([1, 31, 32, 33, 128, 400], 4, 4, 32, -BIG, BIG),
    ([200, 384, 65], 2, 2, 128, -BIG, BIG),
    # long batches (several query tiles per CTA on the 16-bit paths), with
    # sequences shorter than one tile among them: bidirectional with GQA,
    # causal, and a window
    ([1, 700, 130, 1500, 257], 4, 2, 64, -BIG, BIG),
    ([3, 1100, 640], 2, 1, 128, -BIG, 0),
    ([900, 5, 1200], 2, 2, 64, -64, 64),
    ([1500, 700, 33], 2, 2, 64, -600, 600),
    ([2000, 130], 2, 1, 128, -700, 0),
    # head dim 128 with windows of at least 1024 keys (the two-tile kernel:
    # each tile's key range differs, the tiles walk their union)
    ([2500, 900, 64], 2, 1, 128, -600, 600),
    ([1800, 5, 1300], 4, 2, 128, -1100, 0),
])
def test_attention_windows_and_heads(cuda, dtype, case):
    lens, heads, kv_heads, dh, lo, hi = case
    got, want = run_attention(cuda, lens, heads, kv_heads, dh, lo, hi, dtype, seed=sum(lens))
    err = float(np.abs(got - want).max())
    assert err <= BARS[dtype], err


@pytest.mark.parametrize("dtype", [RG_DTYPE_F16, RG_DTYPE_BF16])
@pytest.mark.parametrize("case", [
    # ModernBERT global layer at the config's longest sequence, and a local one
    ([8192], 1, 1, 64, -BIG, BIG),
    ([8192, 2049], 1, 1, 64, -64, 64),
    # Qwen3's causal layers at the config's longest sequence (GQA 2:1)
    ([1024, 511], 2, 1, 128, -BIG, 0),
    # Gemma's global and local layers at 2048
    ([2048], 1, 1, 256, -BIG, BIG),
    ([2048], 1, 1, 256, -256, 256),
])
def test_attention_at_benchmark_lengths(cuda, dtype, case):
    lens, heads, kv_heads, dh, lo, hi = case
    got, want = run_attention(cuda, lens, heads, kv_heads, dh, lo, hi, dtype, seed=3 + sum(lens))
    err = float(np.abs(got - want).max())
    assert err <= BARS[dtype], err


def _bf16_exact(rng, shape, scale):
    """float32 values that are exactly representable in bf16."""
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    u = x.view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> 16) & 1)) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (257, 768, 768), (1000, 2304, 768), (300, 768, 3072)])
def test_full_int8_bit_exact(cuda, M, N, K):
    torch = cuda
    rng = np.random.default_rng(M + N + K)
    x = _bf16_exact(rng, (M, K), 1.0)
    x[0, :] = 0.0  # an all-zero row takes scale 1 (pack_vnni.go:93-96)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    wq, colsum, wscale = oracle.packb8vnni(w, K, N)
    # oracle: QuantizeRowU8 per row, then MatMulPackedVNNI and AddBias
    want_q = np.zeros((M, K), dtype=np.int16)
    want_s = np.zeros(M, dtype=np.float32)
    for r in range(M):
        qa, s = oracle.quantize_row_u8(x[r])
        want_q[r] = qa.astype(np.int16) - 128
        want_s[r] = s
    want_y = oracle.matmul_vnni(x, wq, colsum, wscale, M, K, N)
    want_yb = oracle.add_bias(want_y, bias, M, N).reshape(M, N)

    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dx = torch.from_numpy(x).to("cuda", torch.bfloat16)
    assert np.array_equal(dx.float().cpu().numpy(), x)
    dq = torch.empty((M, K), device="cuda", dtype=torch.int8)
    ds = torch.empty((M,), device="cuda", dtype=torch.float32)
    _call("rg_quantize_rows_s8", _vp(dx), M, K, _vp(dq), _vp(ds), st)
    dw = torch.from_numpy(wq).to("cuda")
    dws = torch.from_numpy(wscale).to("cuda")
    db = torch.from_numpy(bias).to("cuda")
    y = torch.empty((M, N), device="cuda", dtype=torch.float32)
    yb = torch.empty((M, N), device="cuda", dtype=torch.float32)
    _call("rg_dense_s8", _vp(dq), _vp(ds), _vp(dw), _vp(dws), ctypes.c_void_p(0), _vp(y), M, N, K, st)
    _call("rg_dense_s8", _vp(dq), _vp(ds), _vp(dw), _vp(dws), _vp(db), _vp(yb), M, N, K, st)
    kernel_status(torch)
    assert np.array_equal(dq.cpu().numpy().astype(np.int16), want_q)
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), want_s.view(np.uint32))
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want_y.view(np.uint32))
    assert np.array_equal(yb.cpu().numpy().view(np.uint32), want_yb.view(np.uint32))


def test_kernel_level_shape_errors(cuda):
    from rembed_b200.embedder import RembedError

    torch = cuda
    z = torch.zeros(256, device="cuda")
    cu = np.array([0, 4], dtype=np.int32)
    with pytest.raises(RembedError, match="head dim 48 unsupported"):
        _call("rg_attention", _vp(z), _vp(z), _vp(z), 48, 48, 48, _vp(z), cu.ctypes.data_as(
            ctypes.POINTER(ctypes.c_int32)), 1, 1, 1, 48, ctypes.c_float(1.0), -4, 4, RG_DTYPE_BF16, _vp(z), 48,
            ctypes.c_void_p(0))
    with pytest.raises(RembedError, match="K % 128 == 0"):
        _call("rg_dense_s8", _vp(z), _vp(z), _vp(z), _vp(z), ctypes.c_void_p(0), _vp(z), 4, 128, 64,
              ctypes.c_void_p(0))
    kernel_status(torch)
