"""tcgen05 GEMM parity: rg_dense_bf16 (through the C ABI) against a plain
torch fp32 reference of the same op on the same bf16-rounded operands.

Tolerances: fp32 outputs within 1e-4 * (1 + |ref|) * sqrt(K/64) (only the
accumulation order differs); bf16 outputs within one bf16 rounding
(2^-8 relative) of the fp32 reference plus that."""

import ctypes
import math

import pytest

pytestmark = pytest.mark.gpu

SHAPES = [
    (1, 128, 64), (100, 256, 64), (128, 384, 128), (300, 768, 768), (1000, 1152, 384),
    (257, 2304, 768), (4096, 768, 3072), (33, 1536, 384),
]


def run_dense(torch, x, w, bias, res, epi):
    from rembed_b200.embedder import library, take_error

    M, K = x.shape
    N = w.shape[0]
    y = torch.empty((M, N), device="cuda", dtype=torch.float32 if epi in (2, 3) else torch.bfloat16)
    err = ctypes.c_char_p()
    rc = library().rg_dense_bf16(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()),
        ctypes.c_void_p(bias.data_ptr() if bias is not None else 0),
        ctypes.c_void_p(res.data_ptr() if res is not None else 0), ctypes.c_void_p(y.data_ptr()),
        M, N, K, epi, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(err))
    if rc != 0:
        raise RuntimeError(take_error(err))
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_dense_matches_fp32(cuda, M, N, K, epi):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K + epi)
    x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((N, K), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn((N,), device="cuda", generator=g)
    res = torch.randn((M, N), device="cuda", generator=g) if epi == 2 else None
    y = run_dense(torch, x, w, bias, res, epi).float()
    ref = x.float() @ w.float().t() + bias
    if epi == 1:
        ref = torch.nn.functional.gelu(ref)  # exact erf GELU
    if epi == 2:
        ref = res + ref
    tol = 1e-4 * (1 + ref.abs()) * math.sqrt(K / 64)
    if epi in (0, 1):
        tol = tol + ref.abs() * 2.0 ** -8
    bad = (y - ref).abs() > tol
    assert not bool(bad.any()), f"max err {(y - ref).abs().max().item()} at {bad.nonzero()[:4].tolist()}"


def test_dense_rejects_bad_shapes(cuda):
    torch = cuda
    x = torch.zeros((4, 96), device="cuda", dtype=torch.bfloat16)
    w = torch.zeros((128, 96), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="K % 64"):
        run_dense(torch, x, w, None, None, 0)


def run_sublayer(torch, x, w, bias, res, gamma, beta, eps, fn="rg_dense_residual_layernorm_bf16"):
    from rembed_b200.embedder import RembedError, library, take_error

    M, K = x.shape
    N = w.shape[0]
    out32 = torch.empty((M, N), device="cuda", dtype=torch.float32)
    outb = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    err = ctypes.c_char_p()
    rc = getattr(library(), fn)(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(bias.data_ptr()),
        ctypes.c_void_p(res.data_ptr()), ctypes.c_void_p(gamma.data_ptr()), ctypes.c_void_p(beta.data_ptr()),
        ctypes.c_float(eps), ctypes.c_void_p(out32.data_ptr()), ctypes.c_void_p(outb.data_ptr()), M, N, K,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(err))
    if rc != 0:
        raise RembedError(take_error(err))
    torch.cuda.synchronize()
    return out32, outb


def sublayer_inputs(torch, M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((N, K), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn((N,), device="cuda", generator=g) * 0.1
    res = torch.randn((M, N), device="cuda", generator=g)
    gamma = 1 + 0.02 * torch.randn((N,), device="cuda", generator=g)
    beta = 0.02 * torch.randn((N,), device="cuda", generator=g)
    return x, w, bias, res, gamma, beta


def sublayer_reference(x, w, bias, res, gamma, beta, eps):
    """Add then two-pass LayerNorm in fp32 (tensor.go:383-387, 433-452)."""
    s = res + (x.float() @ w.float().t() + bias)
    mean = s.mean(1, keepdim=True)
    var = ((s - mean) ** 2).mean(1, keepdim=True)
    return (s - mean) / (var + eps).sqrt() * gamma + beta


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (300, 384, 384), (1000, 768, 768), (257, 768, 3072),
                                   (64, 1024, 1024)])
def test_dense_residual_layernorm(cuda, M, N, K):
    torch = cuda
    eps = 1e-12
    args = sublayer_inputs(torch, M, N, K, seed=M + N + K)
    out32, outb = run_sublayer(torch, *args, eps)
    ref = sublayer_reference(*args, eps)
    tol = 2e-4 * (1 + ref.abs()) * math.sqrt(K / 64)
    assert float(((out32 - ref).abs() - tol).max()) <= 0, float((out32 - ref).abs().max())
    assert torch.equal(outb, out32.to(torch.bfloat16))


def test_dense_residual_layernorm_rejects_bad_width(cuda):
    torch = cuda
    from rembed_b200.embedder import RembedError

    args = sublayer_inputs(torch, 4, 640, 64, seed=1)
    with pytest.raises(RembedError, match="unsupported shape"):
        run_sublayer(torch, *args, 1e-12)
