"""Failure detection and recovery, with every failure made on purpose in a
way that faults, traps or hangs no GPU.

* A non-finite weight under an int8 mode is refused at finalize, as the
  reference's quantisers refuse it (pack8.go:43-48, pack_vnni.go:54-55).
* A device pipeline wait that runs out: a test hook makes one GEMM withhold a
  barrier arrival and bounds its waits at ~10 ms; the kernel stops, drains
  its copies and MMAs, frees its tensor memory and records the timeout in the
  device status word; rg_kernel_status reports it and the next call on the
  same context is correct.
* A host allocation failure (injected) fails the call with the allocator's
  message; the context stays usable.
* A failing device worker in a context of two replicas: the call returns the
  worker's error after the other replica's work is collected, never hangs,
  and the next call is bit-identical to a one-replica context (the two
  replicas share one GPU here, so the test needs one device).
"""

import ctypes
import math

import numpy as np
import pytest

from rembed_b200 import synth
from rembed_b200.embedder import Embedder, RembedError, library, take_error

pytestmark = pytest.mark.gpu

RG_INJECT_GEMM_WAIT, RG_INJECT_HOST_ALLOC, RG_INJECT_REPLICA = 1, 2, 3


def inject(ctx, what, arg=0):
    err = ctypes.c_char_p()
    if library().rg_test_inject(ctx, what, arg, ctypes.byref(err)) != 0:
        raise RembedError(take_error(err))


def kernel_status(torch):
    err = ctypes.c_char_p()
    if library().rg_kernel_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(err)) != 0:
        raise RembedError(take_error(err))


@pytest.mark.parametrize("kw", [dict(int8=True), dict(int8_activations=True)])
@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_non_finite_weight_refused_under_int8(cuda, kw, bad):
    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=5)
    w["encoder.layer.1.intermediate.dense.weight"][3, 7] = bad
    with pytest.raises(RembedError, match="finite"):
        Embedder(cfg, w, **kw)


def _dense(torch, x, w, bias):
    M, K = x.shape
    N = w.shape[0]
    y = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    err = ctypes.c_char_p()
    rc = library().rg_dense_bf16(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                 ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(0), ctypes.c_void_p(y.data_ptr()),
                                 M, N, K, 3, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                 ctypes.byref(err))
    if rc != 0:
        raise RembedError(take_error(err))
    return y


def test_gemm_wait_timeout_is_reported_and_recovered(cuda):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(11)
    M, N, K = 1000, 768, 768
    x = torch.randn((M, K), device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((N, K), device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn((N,), device="cuda", generator=g)
    kernel_status(torch)  # nothing pending
    inject(None, RG_INJECT_GEMM_WAIT, 20_000_000)  # ~10 ms at the B200's clock
    _dense(torch, x, w, bias)
    with pytest.raises(RembedError, match="wait timed out"):
        kernel_status(torch)
    kernel_status(torch)  # the report cleared the word
    # the same device and library serve the next call correctly
    y = _dense(torch, x, w, bias)
    kernel_status(torch)
    ref = x.float() @ w.float().t() + bias
    assert float(((y - ref).abs() - 1e-4 * (1 + ref.abs()) * math.sqrt(K / 64)).max()) <= 0


def test_host_allocation_failure_is_reported(cuda):
    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=6)
    ids, cu = synth.make_batch(cfg, 5, 1, 90, seed=7, id_hi=4000)
    with Embedder(cfg, w) as e:
        want = e.embed_packed(ids, cu)
        inject(e._ctx, RG_INJECT_HOST_ALLOC)
        with pytest.raises(RembedError, match="out of memory"):
            e.embed_packed(ids, cu)
        assert np.array_equal(e.embed_packed(ids, cu), want)


def test_worker_failure_in_two_replica_context(cuda):
    cfg = synth.preset("tiny-modernbert")
    w = synth.make_weights(cfg, seed=8)
    # lengths spread 16x, as ModernBERT's configuration: the split by cost
    # gives the two replicas different sequence counts
    ids, cu = synth.batch_of_lengths(cfg, [60, 900, 33, 512, 1000, 17, 250, 640, 64, 128], seed=9)
    with Embedder(cfg, w, devices=(0,)) as one:
        want = one.embed_packed(ids, cu)
    with Embedder(cfg, w, devices=(0, 0)) as two:
        assert np.array_equal(two.embed_packed(ids, cu), want)
        inject(two._ctx, RG_INJECT_REPLICA, 1)
        with pytest.raises(RembedError, match="worker of device 0 failed"):
            two.embed_packed(ids, cu)
        assert np.array_equal(two.embed_packed(ids, cu), want)
        # and through the pipelined submit / collect path
        p = two.submit(ids, cu)
        assert np.array_equal(p.result(), want)


def test_injection_arguments_are_checked(cuda):
    with pytest.raises(RembedError, match="unknown injection"):
        inject(None, 99)
    with pytest.raises(RembedError, match="positive"):
        inject(None, RG_INJECT_GEMM_WAIT, 0)
