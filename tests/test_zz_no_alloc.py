"""The allocation-free sublayer entry point against the allocating one.

rg_dense_residual_layernorm_bf16_noalloc exists for callers that cannot let a
library call cudaMalloc: a host whose memory manager owns every byte of
device memory (an arena carved out of HBM up front, or an allocator that
accounts for each buffer), or a latency-bound caller that cannot afford the
device synchronisation an allocation may bring.  It keeps its scratch in a
fixed 16 MiB static device array instead of the per-device buffer that
rg_dense_residual_layernorm_bf16 allocates.

Both are called through the C ABI on the same inputs.  The outputs must agree
within the tolerance the kernel tests use (test_gpu_gemm.py), on two calls in
a row with different shapes, so the second call also proves that what the
first call left in the shared array does not leak into the result; each is
also checked against the plain fp32 torch reference of the sublayer, and
rg_kernel_status (which reads the array's status word) must report no
failure.  The file is named to be collected last and must pass alone in a
fresh process too.
"""

import ctypes
import math

import pytest

pytestmark = pytest.mark.gpu


def call(torch, fn, x, w, bias, res, gamma, beta, eps):
    from rembed_b200.embedder import RembedError, library, take_error

    M, K = x.shape
    N = w.shape[0]
    out32 = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    outb = torch.zeros((M, N), device="cuda", dtype=torch.bfloat16)
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


def inputs(torch, M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((N, K), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn((N,), device="cuda", generator=g) * 0.1
    res = torch.randn((M, N), device="cuda", generator=g)
    gamma = 1 + 0.02 * torch.randn((N,), device="cuda", generator=g)
    beta = 0.02 * torch.randn((N,), device="cuda", generator=g)
    return x, w, bias, res, gamma, beta


def test_noalloc_matches_allocating_entry_point_on_two_calls(cuda):
    torch = cuda
    eps = 1e-12
    # Two calls in a row: the larger one first, then a smaller one with other
    # data, so stale scratch from the first call would show in the second.
    for M, N, K, seed in [(1000, 768, 768, 5), (300, 384, 384, 6)]:
        args = inputs(torch, M, N, K, seed)
        want32, wantb = call(torch, "rg_dense_residual_layernorm_bf16", *args, eps)
        got32, gotb = call(torch, "rg_dense_residual_layernorm_bf16_noalloc", *args, eps)
        tol = 2e-4 * (1 + want32.abs()) * math.sqrt(K / 64)
        assert not bool(torch.isnan(got32).any())
        assert float(((got32 - want32).abs() - tol).max()) <= 0, float((got32 - want32).abs().max())
        assert float((gotb.float() - wantb.float()).abs().max()) <= float((want32.abs() * 2.0 ** -7 + 1e-3).max())
        ref = fp32_reference(*args, eps)
        tol = 2e-4 * (1 + ref.abs()) * math.sqrt(K / 64)
        assert float(((got32 - ref).abs() - tol).max()) <= 0, float((got32 - ref).abs().max())
        kernel_status(torch)


def fp32_reference(x, w, bias, res, gamma, beta, eps):
    """Add then two-pass LayerNorm in fp32 (tensor.go:383-387, 433-452)."""
    s = res + (x.float() @ w.float().t() + bias)
    mean = s.mean(1, keepdim=True)
    var = ((s - mean) ** 2).mean(1, keepdim=True)
    return (s - mean) / (var + eps).sqrt() * gamma + beta


def kernel_status(torch):
    from rembed_b200.embedder import RembedError, library, take_error

    err = ctypes.c_char_p()
    if library().rg_kernel_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(err)) != 0:
        raise RembedError(take_error(err))


def test_noalloc_rejects_more_than_its_scratch(cuda):
    torch = cuda
    from rembed_b200.embedder import RembedError

    max_floats = 4 * 1024 * 1024  # RG_NOALLOC_SCRATCH_FLOATS
    N, K = 1024, 64
    M = max_floats // N + 1
    args = inputs(torch, M, N, K, seed=7)
    with pytest.raises(RembedError, match="exceeds the fixed scratch"):
        call(torch, "rg_dense_residual_layernorm_bf16_noalloc", *args, 1e-12)
